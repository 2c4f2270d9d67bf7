// Tensor-core self-test: one 128 x 64 x 128 bf16 GEMM through the same shared-memory
// layouts, descriptors and TMEM path the chunk kernels use.  It lets a test pin the
// descriptor encoding (K-major and MN-major operands) against a plain matmul
// independently of the SSD arithmetic.
#include "common.cuh"
#include "launch.h"

namespace m3b {

// D[m][n] = sum_k A[m][k] * B[n][k];  A (128 x 128), B (64 x 128), row-major bf16 in global memory.
// mode 0: A staged K-major (tile row = m).  mode 1: A staged as A^T (tile row = k) and read MN-major.
// mode 2: A K-major, B staged as B^T (tile row = k, 64 columns n) and read MN-major.
__global__ void __launch_bounds__(128, 1) umma_selftest_kernel(const __nv_bfloat16* __restrict__ A,
                                                               const __nv_bfloat16* __restrict__ B,
                                                               float* __restrict__ D, int mode, int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* tA = sm;              // 32 KB
  uint8_t* tB = sm + 32768;      // 16 KB (64 rows x 128, or 128 rows x 64 in mode 2)
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + 49152);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + 49152 + 16);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp == 0) {
    tmem_alloc(tslot, 64);
    tmem_relinquish();
  }
  if (threadIdx.x == 32) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  for (int u = threadIdx.x; u < 128 * 16; u += blockDim.x) {
    const int row = u / 16, c = u % 16;
    uint4 v;
    if (mode != 1) {
      v = *reinterpret_cast<const uint4*>(A + row * 128 + c * 8);
    } else {  // tile row = k, columns = m
      uint32_t w[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const __nv_bfloat16 lo = A[(c * 8 + 2 * e) * 128 + row];
        const __nv_bfloat16 hi = A[(c * 8 + 2 * e + 1) * 128 + row];
        w[e] = (uint32_t)__bfloat16_as_ushort(lo) | ((uint32_t)__bfloat16_as_ushort(hi) << 16);
      }
      v = make_uint4(w[0], w[1], w[2], w[3]);
    }
    sw128_store_chunk(tA, row, c, 128, v);
  }
  if (mode != 2) {
    for (int u = threadIdx.x; u < 64 * 16; u += blockDim.x) {
      const int row = u / 16, c = u % 16;
      sw128_store_chunk(tB, row, c, 64, *reinterpret_cast<const uint4*>(B + row * 128 + c * 8));
    }
  } else {  // tile row = k (128 rows), 8 chunks of 8 n
    for (int u = threadIdx.x; u < 128 * 8; u += blockDim.x) {
      const int row = u / 8, c = u % 8;
      uint32_t w[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const __nv_bfloat16 lo = B[(c * 8 + 2 * e) * 128 + row];
        const __nv_bfloat16 hi = B[(c * 8 + 2 * e + 1) * 128 + row];
        w[e] = (uint32_t)__bfloat16_as_ushort(lo) | ((uint32_t)__bfloat16_as_ushort(hi) << 16);
      }
      sw128_store_chunk(tB, row, c, 128, make_uint4(w[0], w[1], w[2], w[3]));
    }
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  if (threadIdx.x == 0) {
    const uint32_t idesc = idesc_bf16(128, 64, mode == 1, mode == 2);
    for (int kk = 0; kk < 8; ++kk) {
      const uint64_t ad = mode == 1 ? mnmajor_desc(tA, 128, kk * 16) : kmajor_desc(tA, 128, kk * 16);
      const uint64_t bd = mode == 2 ? mnmajor_desc(tB, 128, kk * 16) : kmajor_desc(tB, 64, kk * 16);
      umma_bf16(tbase, ad, bd, idesc, kk > 0 ? 1u : 0u);
    }
    umma_commit(bar);
  }
  bool ok = mbar_wait(bar, 0);
  __syncwarp();
  ok = __syncthreads_and(ok);
  tc_fence_after();
  if (ok) {
    const int m = 32 * warp + lane;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      float v[32];
      tmem_ld32(tbase + ((uint32_t)(32 * warp) << 16) + 32 * half, v);
#pragma unroll
      for (int j = 0; j < 32; ++j) D[m * 64 + 32 * half + j] = v[j];
    }
  } else if (threadIdx.x == 0) {
    record_error(err, M3B_ERR_TIMEOUT);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, 64);
  }
}

// The same GEMM with fp32 operands on kind::tf32 (mode 3: A and B K-major, the layout the fp32
// chunk kernels use): A (128 x 128 fp32), B (64 x 128 fp32) row-major; tiles of fp32 words in
// 128-byte column blocks of 32 elements.
__global__ void __launch_bounds__(128, 1) umma_selftest_tf32_kernel(const float* __restrict__ A,
                                                                    const float* __restrict__ B,
                                                                    float* __restrict__ D, int mode, int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* tA = sm;          // 64 KB
  uint8_t* tB = sm + 65536;  // 32 KB
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + 98304);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + 98304 + 16);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp == 0) {
    tmem_alloc(tslot, 64);
    tmem_relinquish();
  }
  if (threadIdx.x == 32) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  // tile A: 128 rows x 128 columns (32 chunks of 4 words per row)
  for (int u = threadIdx.x; u < 128 * 32; u += blockDim.x) {
    const int row = u / 32, c = u % 32;
    float w[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) w[e] = A[row * 128 + c * 4 + e];
    sw128_store_chunk(tA, row, c, 128,
                      make_uint4(__float_as_uint(w[0]), __float_as_uint(w[1]), __float_as_uint(w[2]),
                                 __float_as_uint(w[3])));
  }
  for (int u = threadIdx.x; u < 64 * 32; u += blockDim.x) {  // tile B: 64 rows (n) x 128 columns (k)
    const int row = u / 32, c = u % 32;
    const float4 v = *reinterpret_cast<const float4*>(B + row * 128 + c * 4);
    sw128_store_chunk(tB, row, c, 64,
                      make_uint4(__float_as_uint(v.x), __float_as_uint(v.y), __float_as_uint(v.z),
                                 __float_as_uint(v.w)));
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  if (threadIdx.x == 0) {
    const uint32_t idesc = idesc_tf32(128, 64, false, false);
    for (int kk = 0; kk < 16; ++kk)
      umma_tf32(tbase, kmajor_desc_b(tA, 128, kk * 32), kmajor_desc_b(tB, 64, kk * 32), idesc, kk > 0 ? 1u : 0u);
    umma_commit(bar);
  }
  bool ok = mbar_wait(bar, 0);
  __syncwarp();
  ok = __syncthreads_and(ok);
  tc_fence_after();
  if (ok) {
    const int m = 32 * warp + lane;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      float v[32];
      tmem_ld32(tbase + ((uint32_t)(32 * warp) << 16) + 32 * half, v);
#pragma unroll
      for (int j = 0; j < 32; ++j) D[m * 64 + 32 * half + j] = v[j];
    }
  } else if (threadIdx.x == 0) {
    record_error(err, M3B_ERR_TIMEOUT);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, 64);
  }
}

// The bf16 GEMM with A held in TMEM (mode 6): each thread stores its row m of A (128 bf16, packed
// two per column) into TMEM columns [0, 64); the MMA reads A from TMEM and B K-major from shared
// memory into D at columns [64, 128).  Pins the TMEM operand layout the fused kernel's P tile uses.
__global__ void __launch_bounds__(128, 1) umma_selftest_ts_kernel(const __nv_bfloat16* __restrict__ A,
                                                                  const __nv_bfloat16* __restrict__ B,
                                                                  float* __restrict__ D, int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* tB = sm;  // 16 KB: 64 rows (n) x 128 (k)
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + 16384);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + 16384 + 16);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp == 0) {
    tmem_alloc(tslot, 128);
    tmem_relinquish();
  }
  if (threadIdx.x == 32) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  for (int u = threadIdx.x; u < 64 * 16; u += blockDim.x) {
    const int row = u / 16, c = u % 16;
    sw128_store_chunk(tB, row, c, 64, *reinterpret_cast<const uint4*>(B + row * 128 + c * 8));
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  const int m = 32 * warp + lane;
  const uint32_t trow = tbase + ((uint32_t)(32 * warp) << 16);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint32_t w[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) w[e] = reinterpret_cast<const uint32_t*>(A + m * 128 + 32 * q)[e];
    tmem_st16_nowait(trow + 16 * q, w);
  }
  tmem_wait_st();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (threadIdx.x == 0) {
    const uint32_t idesc = idesc_bf16(128, 64, false, false);
    for (int kk = 0; kk < 8; ++kk) umma_bf16_ts(tbase + 64, tbase + kk * 8, kmajor_desc(tB, 64, kk * 16), idesc, kk > 0 ? 1u : 0u);
    umma_commit(bar);
  }
  bool ok = mbar_wait(bar, 0);
  __syncwarp();
  ok = __syncthreads_and(ok);
  tc_fence_after();
  if (ok) {
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      float v[32];
      tmem_ld32(trow + 64 + 32 * half, v);
#pragma unroll
      for (int j = 0; j < 32; ++j) D[m * 64 + 32 * half + j] = v[j];
    }
  } else if (threadIdx.x == 0) {
    record_error(err, M3B_ERR_TIMEOUT);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, 128);
  }
}

// One thread waits (bounded by limit_ns) on the flag (mode 0) or on an mbarrier phase nothing
// completes (mode 1); a wait that runs out records M3B_ERR_TIMEOUT.
__global__ void __launch_bounds__(32, 1) wait_selftest_kernel(const int* flag, int target, int mode,
                                                             uint64_t limit_ns, int* err) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncwarp();
  if (threadIdx.x == 0) {
    const bool ok = mode == 0 ? flag_wait_geq(flag, target, limit_ns) : mbar_wait(&bar, 0, limit_ns);
    if (!ok) record_error(err, M3B_ERR_TIMEOUT);
  }
}

}  // namespace m3b

extern "C" int m3b_selftest_wait(const int* flag, int target, int mode, int64_t limit_ns, int* err, void* stream) {
  m3b::clear_error();
  if (mode < 0 || mode > 1 || (mode == 0 && !flag) || !err)
    return m3b::fail(M3B_ERR_INVALID_ARG, "selftest_wait: mode 0 (flag) or 1 (mbarrier) and an err word");
  if (limit_ns <= 0 || limit_ns > 1000000000ll)
    return m3b::fail(M3B_ERR_INVALID_ARG, "selftest_wait: limit_ns must be in (0, 1e9]");
  m3b::wait_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(flag, target, mode,
                                                                            (uint64_t)limit_ns, err);
  return m3b::check_launch("selftest_wait");
}

extern "C" int m3b_selftest_umma(const void* A, const void* B, float* D, int mode, int* err, void* stream) {
  if (!A || !B || !D || mode < 0 || mode > 6 || mode == 4 || mode == 5)
    return m3b::fail(M3B_ERR_INVALID_ARG, "selftest_umma: bad args");
  if (!m3b::aligned16(A) || !m3b::aligned16(B)) return m3b::fail(M3B_ERR_ALIGNMENT, "selftest_umma: alignment");
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (mode == 6) {
    const int bytes = 16384 + 64 + 1024;
    m3b::umma_selftest_ts_kernel<<<1, 128, bytes, st>>>(static_cast<const __nv_bfloat16*>(A),
                                                        static_cast<const __nv_bfloat16*>(B), D, err);
    return m3b::check_launch("selftest_umma");
  }
  if (mode == 3) {
    const int bytes = 98304 + 64 + 1024;
    cudaError_t e =
        cudaFuncSetAttribute(m3b::umma_selftest_tf32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) return m3b::fail(M3B_ERR_CUDA, "selftest_umma: %s", cudaGetErrorString(e));
    m3b::umma_selftest_tf32_kernel<<<1, 128, bytes, st>>>(static_cast<const float*>(A),
                                                          static_cast<const float*>(B), D, mode, err);
    return m3b::check_launch("selftest_umma");
  }
  const int bytes = 49152 + 64 + 1024;
  cudaError_t e = cudaFuncSetAttribute(m3b::umma_selftest_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return m3b::fail(M3B_ERR_CUDA, "selftest_umma: %s", cudaGetErrorString(e));
  m3b::umma_selftest_kernel<<<1, 128, bytes, st>>>(
      static_cast<const __nv_bfloat16*>(A), static_cast<const __nv_bfloat16*>(B), D, mode, err);
  return m3b::check_launch("selftest_umma");
}
