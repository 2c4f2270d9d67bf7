// Input projection with the layer's per-token prologue in its epilogue (sm_100a).
//
//   proj = x W^T (+ bias)        mamba3/mamba3.py:197 (nn.Linear), bf16 in / out, fp32 accumulate
//   rms[t, g] = 1/rms(B_g), 1/rms(C_g) of the rounded proj row   B_norm / C_norm, mamba3.py:200-204
//
// One persistent CTA per SM, three roles:
//   warp 0      TMA producer: x tile (128 rows x 64 K) and W tile (up to 256 output columns x 64 K)
//               per stage, 128-byte swizzled, into a 4-stage shared-memory ring;
//   warp 1      MMA issuer: tcgen05.mma 128 x width x 16 into one of two TMEM accumulators
//               (256 columns each), so the epilogue of one tile overlaps the next tile's MMAs;
//   warps 2-5   epilogue: TMEM -> registers (one output row per thread), + bias, bf16 rounding;
//               each warp stages 32 rows x 64 columns in a swizzled shared-memory box (two per
//               warp, alternating) that one TMA store writes out, so a store request carries whole
//               128-byte rows; for the columns of a group's B or C the thread also sums the squares
//               of its rounded values and, after the last piece, writes rsqrt(sum / (N R) + eps).
// The output columns are cut into segments of at most 256: the z | x columns, every group's B and
// C columns (one unit of ceil(N R / 256) pieces each, so one thread sees a whole B or C row), and
// the dt | lam | theta tail.  A job is (128-row tile, unit); job j runs on CTA j mod grid.
#include <mutex>
#include <set>
#include <utility>

#include "common.cuh"
#include "launch.h"
#include "tmap.h"

namespace m3b {

namespace {

constexpr int kIpBM = 128;      // rows per tile = TMEM lanes
constexpr int kIpBN = 256;      // columns per segment at most = one TMEM accumulator
constexpr int kIpBK = 64;       // K per stage: one 128-byte swizzle atom row of bf16
constexpr int kIpStages = 4;
constexpr int kIpThreads = 192;
constexpr int kIpMaxSeg = 128;   // the segment tables travel in the kernel's parameters (4 KB)
constexpr int kIpMaxUnit = 128;
constexpr uint32_t kIpStageA = kIpBM * kIpBK * 2;  // 16 KB
constexpr uint32_t kIpStageB = kIpBN * kIpBK * 2;  // 32 KB
constexpr uint32_t kIpBox = 32 * 128;                          // staging box: 32 rows x 64 bf16
constexpr uint32_t kIpStgOff = kIpStages * (kIpStageA + kIpStageB);
constexpr uint32_t kIpBarOff = kIpStgOff + 4 * 2 * kIpBox;      // two boxes per epilogue warp
constexpr uint32_t kIpSmem = kIpBarOff + 256 + 1024;  // + barriers, TMEM slot, abort flag; + alignment
static_assert(kIpSmem <= 227 * 1024, "shared memory plan");

struct IpParams {
  int64_t M;        // rows
  int K;            // d_model
  int ncols;        // d_proj
  int mtiles, nunit, nseg;
  const __nv_bfloat16* bias;
  __nv_bfloat16* out;
  int64_t ldo;
  float* rms;       // (M, G, 2) or null
  int G;
  float nr, eps;     // N R, the length of a group's B / C row; the norms' eps
  int* err;
  uint64_t wait_ns;
  int4 seg[kIpMaxSeg];    // col0, width (multiple of 16), kind (0 plain, 1 B, 2 C) | group << 2, last piece
  int2 unit[kIpMaxUnit];  // [first segment, end segment)
};

__device__ __forceinline__ void ip_fail(const IpParams& a, volatile int* abort_flag) {
  *abort_flag = 1;
  record_error(a.err, M3B_ERR_TIMEOUT);
}

__global__ void __launch_bounds__(kIpThreads, 1)
    in_proj_kernel(const __grid_constant__ IpParams a, const __grid_constant__ CUtensorMap tm_x,
                   const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_o) {
  extern __shared__ uint8_t smraw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smraw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + kIpBarOff);
  uint64_t* full = bars;                  // [kIpStages]: the stage's two copies landed
  uint64_t* empty = bars + kIpStages;     // [kIpStages]: the MMAs reading the stage completed
  uint64_t* accf = bars + 2 * kIpStages;  // [2]: accumulator holds a finished segment
  uint64_t* acce = accf + 2;              // [2]: the epilogue has read the accumulator
  uint32_t* tslot = reinterpret_cast<uint32_t*>(acce + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kIpStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&accf[i], 1);
      mbar_init(&acce[i], 4);  // one arrival per epilogue warp
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tslot, 512);
    tmem_relinquish();
  }
  if (warp == 1 && lane == 0) {
    prefetch_tensormap(&tm_x);
    prefetch_tensormap(&tm_w);
    prefetch_tensormap(&tm_o);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  const int64_t njobs = (int64_t)a.mtiles * a.nunit;
  const int nk = (a.K + kIpBK - 1) / kIpBK;

  if (warp == 0) {
    if (lane == 0) {
      uint32_t it = 0;
      for (int64_t j = blockIdx.x; j < njobs && !*abort_flag; j += gridDim.x) {
        const int mt = (int)(j / a.nunit), u = (int)(j % a.nunit);
        for (int sg = a.unit[u].x; sg < a.unit[u].y; ++sg) {
          const int col0 = a.seg[sg].x;
          for (int kb = 0; kb < nk; ++kb, ++it) {
            const int s = (int)(it % kIpStages);
            if (!mbar_wait(&empty[s], ((it / kIpStages) & 1) ^ 1, a.wait_ns)) {
              ip_fail(a, abort_flag);
              break;
            }
            mbar_arrive_expect_tx(&full[s], kIpStageA + kIpStageB);
            tma_load_2d(sm + s * kIpStageA, &tm_x, kb * kIpBK, mt * kIpBM, &full[s]);
            tma_load_2d(sm + kIpStages * kIpStageA + s * kIpStageB, &tm_w, kb * kIpBK, col0, &full[s]);
          }
          if (*abort_flag) break;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      uint32_t it = 0, sc = 0;
      for (int64_t j = blockIdx.x; j < njobs && !*abort_flag; j += gridDim.x) {
        const int u = (int)(j % a.nunit);
        for (int sg = a.unit[u].x; sg < a.unit[u].y; ++sg, ++sc) {
          const int acc = (int)(sc & 1);
          if (!mbar_wait(&acce[acc], ((sc >> 1) & 1) ^ 1, a.wait_ns)) {
            ip_fail(a, abort_flag);
            break;
          }
          tc_fence_after();
          const uint32_t idesc = idesc_bf16(kIpBM, a.seg[sg].y, false, false);
          const uint32_t dt = tbase + (uint32_t)(acc * kIpBN);
          for (int kb = 0; kb < nk; ++kb, ++it) {
            const int s = (int)(it % kIpStages);
            if (!mbar_wait(&full[s], (it / kIpStages) & 1, a.wait_ns)) {
              ip_fail(a, abort_flag);
              break;
            }
            tc_fence_after();
            const uint8_t* tA = sm + s * kIpStageA;
            const uint8_t* tB = sm + kIpStages * kIpStageA + s * kIpStageB;
#pragma unroll
            for (int kk = 0; kk < kIpBK / 16; ++kk)
              umma_bf16(dt, kmajor_desc(tA, kIpBM, kk * 16), kmajor_desc(tB, kIpBN, kk * 16), idesc,
                        (kb | kk) != 0 ? 1u : 0u);
            umma_commit(&empty[s]);  // the stage is free once these MMAs have read it
          }
          if (*abort_flag) break;
          umma_commit(&accf[acc]);
        }
      }
    }
  } else {
    // epilogue: warp w reads TMEM lanes 32 (w mod 4) .. + 31, one output row per thread
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const uint32_t tl = tbase + ((uint32_t)(q * 32) << 16);
    uint8_t* stg = sm + kIpStgOff + (uint32_t)q * 2 * kIpBox;
    int sb = 0;
    uint32_t sc = 0;
    float ss = 0.f;
    // + bias, round to bf16 pairs, and the B / C sum of squares, for 16 columns at c
    auto finish16 = [&](const uint32_t* r, int col, int kind, uint32_t* w) {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float v0 = __uint_as_float(r[2 * e]), v1 = __uint_as_float(r[2 * e + 1]);
        if (a.bias && col + 2 * e < a.ncols) {
          v0 += __bfloat162float(a.bias[col + 2 * e]);
          v1 += __bfloat162float(a.bias[col + 2 * e + 1]);
        }
        w[e] = pack_bf16x2(v0, v1);
      }
      if (kind != 0) {
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float2 f = bf2_to_f2(w[e]);
          ss = fmaf(f.x, f.x, fmaf(f.y, f.y, ss));
        }
      }
    };
    for (int64_t j = blockIdx.x; j < njobs && !*abort_flag; j += gridDim.x) {
      const int mt = (int)(j / a.nunit), u = (int)(j % a.nunit);
      const int64_t grow = (int64_t)mt * kIpBM + row;
      const bool rok = grow < a.M;
      for (int sg = a.unit[u].x; sg < a.unit[u].y; ++sg, ++sc) {
        const int acc = (int)(sc & 1);
        if (!mbar_wait(&accf[acc], (sc >> 1) & 1, a.wait_ns)) {
          ip_fail(a, abort_flag);
          break;
        }
        tc_fence_after();
        const int4 sd = a.seg[sg];
        const int col0 = sd.x, width = sd.y, kind = sd.z & 3;
        const uint32_t tc = tl + (uint32_t)(acc * kIpBN);
        int c = 0;
        for (; c + 64 <= width; c += 64) {
          uint32_t ra[32], rb[32];
          tmem_ld32_async(tc + c, ra);
          tmem_ld32_async(tc + c + 32, rb);
          tmem_wait_ld(ra, rb);
          uint32_t w[32];
          finish16(ra, col0 + c, kind, w);
          finish16(ra + 16, col0 + c + 16, kind, w + 8);
          finish16(rb, col0 + c + 32, kind, w + 16);
          finish16(rb + 16, col0 + c + 48, kind, w + 24);
          // this warp's rows x 64 columns through a 128-byte-swizzled box: chunk k of row l at
          // (k ^ (l mod 8)) -- the layout the tensor map's 128-byte swizzle reads back
          if (lane == 0) bulk_wait_group_read<1>();  // the box written two rounds ago has been read
          __syncwarp();
          uint8_t* box = stg + sb * kIpBox;
#pragma unroll
          for (int k = 0; k < 8; ++k)
            *reinterpret_cast<uint4*>(box + lane * 128 + ((k ^ (lane & 7)) << 4)) =
                make_uint4(w[4 * k], w[4 * k + 1], w[4 * k + 2], w[4 * k + 3]);
          fence_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tm_o, box, col0 + c, mt * kIpBM + q * 32);  // rows / columns past the end are not written
            bulk_commit_group();
          }
          sb ^= 1;
        }
        // a remainder of 16, 32 or 48 columns (the segment width is a multiple of 16): direct stores
        __nv_bfloat16* orow = a.out + grow * a.ldo + col0;
        for (; c < width; c += 16) {
          uint32_t r16[16];
          tmem_ld16_async(tc + c, r16);
          tmem_wait_ld(r16);
          uint32_t w[8];
          finish16(r16, col0 + c, kind, w);
          if (rok) {
#pragma unroll
            for (int h8 = 0; h8 < 2; ++h8)
              if (col0 + c + 8 * h8 + 8 <= a.ncols)
                *reinterpret_cast<uint4*>(orow + c + 8 * h8) =
                    make_uint4(w[4 * h8], w[4 * h8 + 1], w[4 * h8 + 2], w[4 * h8 + 3]);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acce[acc]);
        if (kind != 0 && sd.w) {  // last piece of a group's B or C row
          if (rok && a.rms) a.rms[(grow * a.G + (sd.z >> 2)) * 2 + (kind - 1)] = rsqrtf(ss / a.nr + a.eps);
          ss = 0.f;
        }
      }
    }
    if (lane == 0) bulk_wait_group_all();  // the boxes stay in use until their stores are done
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

// 2-D bf16 map (inner, outer) with a (64, box_rows) box, 128-byte swizzle; out-of-range reads zero
// (and out-of-range parts of a stored box are not written).
bool make_map(CUtensorMap* m, const void* base, int64_t inner, int64_t outer, int64_t stride_elems, int box_rows) {
  const EncodeTiledFn enc = encode_tiled();
  if (!enc) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
  const cuuint64_t strides[1] = {(cuuint64_t)stride_elems * 2};
  const cuuint32_t box[2] = {(cuuint32_t)kIpBK, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int opt_in_smem() {
  static std::mutex mu;
  static std::set<int> done;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(mu);
  if (done.count(dev)) return M3B_OK;
  const cudaError_t e =
      cudaFuncSetAttribute((const void*)in_proj_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kIpSmem);
  if (e != cudaSuccess) return fail(M3B_ERR_CUDA, "in_proj: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  done.insert(dev);
  return M3B_OK;
}

// Cut [c0, c1) into segments of at most 256 columns (widths rounded up to 16); `unit` groups
// them into one job when they must meet in one thread (a group's B or C row).
bool add_range(IpParams& p, int c0, int c1, int kind, int group, bool unit) {
  if (c1 <= c0) return true;
  const int first = p.nseg;
  for (int c = c0; c < c1; c += kIpBN) {
    if (p.nseg >= kIpMaxSeg) return false;
    const int w = (c1 - c < kIpBN ? c1 - c : kIpBN);
    p.seg[p.nseg++] = make_int4(c, (w + 15) / 16 * 16, kind | (group << 2), c + kIpBN >= c1 ? 1 : 0);
    if (!unit) {
      if (p.nunit >= kIpMaxUnit) return false;
      p.unit[p.nunit++] = make_int2(p.nseg - 1, p.nseg);
    }
  }
  if (unit) {
    if (p.nunit >= kIpMaxUnit) return false;
    p.unit[p.nunit++] = make_int2(first, p.nseg);
  }
  return true;
}

}  // namespace

int launch_in_proj(const m3b_in_proj_args* a, cudaStream_t st) {
  if (!a->x || !a->weight || !a->proj) return fail(M3B_ERR_INVALID_ARG, "in_proj: null pointer");
  if (a->rows < 0 || a->d_model <= 0 || a->d_proj <= 0) return fail(M3B_ERR_INVALID_ARG, "in_proj: bad sizes");
  if (a->d_model % 8 || a->d_proj % 8 || a->x_stride % 8 || a->proj_stride % 8 || a->x_stride < a->d_model ||
      a->proj_stride < a->d_proj)
    return fail(M3B_ERR_INVALID_ARG, "in_proj: d_model, d_proj and the row strides must be multiples of 8");
  if (!aligned16(a->x) || !aligned16(a->weight) || !aligned16(a->proj))
    return fail(M3B_ERR_INVALID_ARG, "in_proj: x, weight and proj must be 16-byte aligned");
  if (a->rows == 0) return M3B_OK;
  if (a->rows > (int64_t(1) << 31) - kIpBM) return fail(M3B_ERR_INVALID_ARG, "in_proj: too many rows");
  IpParams p{};
  p.M = a->rows;
  p.K = a->d_model;
  p.ncols = a->d_proj;
  p.bias = static_cast<const __nv_bfloat16*>(a->bias);
  p.out = static_cast<__nv_bfloat16*>(a->proj);
  p.ldo = a->proj_stride;
  p.rms = a->rms;
  p.err = a->err;
  p.wait_ns = a->wait_limit_ns > 0 ? (uint64_t)a->wait_limit_ns : kWaitLimitNs;
  bool ok = true;
  if (a->rms) {
    const m3b_layer_params& q = a->prm;
    if (q.H <= 0 || q.P <= 0 || q.N <= 0 || q.R <= 0 || q.G <= 0 || q.H % q.G)
      return fail(M3B_ERR_INVALID_ARG, "in_proj: bad layer dimensions");
    const int64_t offB = 2 * (int64_t)q.H * q.P, NR = (int64_t)q.N * q.R, bc_end = offB + 2 * q.G * NR;
    if (offB % 16 || NR % 16 || bc_end > a->d_proj)
      return fail(M3B_ERR_INVALID_ARG, "in_proj: the B / C columns must start and end on multiples of 16");
    p.G = q.G;
    p.nr = (float)NR;
    p.eps = q.norm_eps;
    ok = add_range(p, 0, (int)offB, 0, 0, false);
    for (int g = 0; ok && g < q.G; ++g) ok = add_range(p, (int)(offB + g * NR), (int)(offB + (g + 1) * NR), 1, g, true);
    for (int g = 0; ok && g < q.G; ++g)
      ok = add_range(p, (int)(offB + (q.G + g) * NR), (int)(offB + (q.G + g + 1) * NR), 2, g, true);
    ok = ok && add_range(p, (int)bc_end, a->d_proj, 0, 0, false);
  } else {
    ok = add_range(p, 0, a->d_proj, 0, 0, false);
  }
  if (!ok) return fail(M3B_ERR_UNSUPPORTED, "in_proj: more than %d column segments", kIpMaxSeg);
  p.mtiles = (int)((a->rows + kIpBM - 1) / kIpBM);
  CUtensorMap tm_x{}, tm_w{}, tm_o{};
  if (!make_map(&tm_x, a->x, a->d_model, a->rows, a->x_stride, kIpBM) ||
      !make_map(&tm_w, a->weight, a->d_model, a->d_proj, a->d_model, kIpBN) ||
      !make_map(&tm_o, a->proj, a->d_proj, a->rows, a->proj_stride, 32))
    return fail(M3B_ERR_CUDA, "in_proj: cuTensorMapEncodeTiled refused the operands");
  int rc = opt_in_smem();
  if (rc != M3B_OK) return rc;
  const int64_t njobs = (int64_t)p.mtiles * p.nunit;
  const int grid = (int)(njobs < num_sms() ? njobs : num_sms());
  in_proj_kernel<<<grid, kIpThreads, kIpSmem, st>>>(p, tm_x, tm_w, tm_o);
  return check_launch("in_proj_kernel");
}

}  // namespace m3b

extern "C" int m3b_in_proj(const m3b_in_proj_args* a, void* stream) {
  m3b::clear_error();
  if (!a) return m3b::fail(M3B_ERR_INVALID_ARG, "in_proj: null args");
  return m3b::launch_in_proj(a, static_cast<cudaStream_t>(stream));
}
