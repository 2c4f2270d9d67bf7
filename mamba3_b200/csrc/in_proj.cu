// Input projection with the layer's per-token prologue in its epilogue (sm_100a).
//
//   proj = x W^T (+ bias)        mamba3/mamba3.py:197 (nn.Linear), bf16 in / out, fp32 accumulate
//   rms[t, g] = 1/rms(B_g), 1/rms(C_g) of the rounded proj row   B_norm / C_norm, mamba3.py:200-204
//
// Persistent CTA pairs: a cluster of two CTAs on two SMs computes 256-row tiles with
// tcgen05.mma.cta_group::2 (each CTA holds 128 rows of x and half of the tile's W rows, and gets
// its 128 rows of the result in its own TMEM), so every SM stages half the W bytes per MMA that a
// lone 128-row CTA would.  Three roles per CTA:
//   warp 0      TMA producer: this CTA's x rows (128 x 64 K) and W rows (width / 2 x 64 K) per
//               stage, 128-byte swizzled, into a 6-stage ring; the copies of both CTAs complete
//               on the first CTA's stage barrier;
//   warp 1      MMA issuer (first CTA only): 256 x width x 16 MMAs into one of two TMEM
//               accumulators (256 columns each, in both SMs), so the epilogue of one tile
//               overlaps the next tile's MMAs; its commits free the stage and hand the
//               accumulator over in both CTAs;
//   warps 2-5   epilogue: TMEM -> registers (one output row per thread), + bias, bf16 rounding;
//               each warp stages 32 rows x 64 columns in a swizzled shared-memory box (two per
//               warp, alternating) that one TMA store writes out, so a store request carries whole
//               128-byte rows; for the columns of a group's B or C the thread also sums the squares
//               of its rounded values and, after the last piece, writes rsqrt(sum / (N R) + eps).
// The output columns are cut into segments of at most 256: the z | x columns, every group's B and
// C columns (one unit of ceil(N R / 256) pieces each, so one thread sees a whole B or C row), and
// the dt | lam | theta tail.  A job is (256-row tile, unit); job j runs on pair j mod pairs.
// Where no CTA pair can be resident, the same kernel runs single CTAs over 128-row tiles
// (cta_group::1, the whole W tile per CTA, 4 stages).
#include <map>
#include <mutex>

#include "common.cuh"
#include "launch.h"
#include "tmap.h"

namespace m3b {

namespace {

constexpr int kIpBM = 128;      // rows per CTA = TMEM lanes
constexpr int kIpBN = 256;      // columns per segment at most = one TMEM accumulator
constexpr int kIpBK = 64;       // K per stage: one 128-byte swizzle atom row of bf16
constexpr int kIpThreads = 192;
constexpr int kIpMaxSeg = 128;   // the segment tables travel in the kernel's parameters (4 KB)
constexpr int kIpMaxUnit = 128;
constexpr uint32_t kIpStageA = kIpBM * kIpBK * 2;  // 16 KB
constexpr uint32_t kIpRing = 192 * 1024;            // stages: 6 x (16 + 16) KB paired, 4 x (16 + 32) KB single
constexpr uint32_t kIpBox = 32 * 128;                          // staging box: 32 rows x 64 bf16
constexpr uint32_t kIpStgOff = kIpRing;
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

// ---- CTA-pair forms (PAIR) next to the single-CTA ones ----
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// The shared::cluster address of the same offset in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
template <bool PAIR>
__device__ __forceinline__ void ip_tmem_alloc(uint32_t* dst, uint32_t ncols) {
  if constexpr (PAIR) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  } else {
    tmem_alloc(dst, ncols);
    tmem_relinquish();
  }
}
template <bool PAIR>
__device__ __forceinline__ void ip_tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  if constexpr (PAIR)
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
  else
    tmem_dealloc(taddr, ncols);
}
// D (+)= A B^T over the pair: A rows [0, 128) from the first CTA's shared memory, [128, 256) from
// the second's (same offset), B rows likewise split in halves; D rows in each CTA's TMEM.
__device__ __forceinline__ void umma_bf16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on the mbarrier at shared::cluster address `bar` (this CTA's or its peer's) when the
// pair MMAs issued so far by this thread have completed.
__device__ __forceinline__ void umma_commit_pair(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
// TMA load into this CTA's shared memory whose completion counts on the mbarrier at shared::cluster
// address `bar`, which may be the peer CTA's (no multicast: every CTA fetches its own box).
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const void* tmap, int c0, int c1, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(smem_u32(dst)),
      "l"(tmap), "r"(c0), "r"(c1), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar) : "memory");
}
// mbar_wait with cluster-scope acquire (the phase completes by arrivals from the peer CTA too).
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
  auto try_wait = [&]() {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity), "r"(100000u)
        : "memory");
    return done != 0;
  };
  if (try_wait()) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (try_wait()) return true;
    if (globaltimer_ns() - t0 > limit_ns) return false;
  }
}

template <bool PAIR>
__global__ void __launch_bounds__(kIpThreads, 1)
    in_proj_kernel(const __grid_constant__ IpParams a, const __grid_constant__ CUtensorMap tm_x,
                   const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_o) {
  constexpr int kIpStages = PAIR ? 6 : 4;
  constexpr uint32_t kIpStageB = (PAIR ? kIpBN / 2 : kIpBN) * kIpBK * 2;  // 16 KB paired, 32 KB single
  constexpr int kTileM = PAIR ? 2 * kIpBM : kIpBM;
  static_assert(kIpStages * (kIpStageA + kIpStageB) == kIpRing, "stage ring");
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
      mbar_init(&acce[i], PAIR ? 8 : 4);  // one arrival per epilogue warp (of both CTAs)
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) ip_tmem_alloc<PAIR>(tslot, 512);
  if (warp == 1 && lane == 0) {
    prefetch_tensormap(&tm_x);
    prefetch_tensormap(&tm_w);
    prefetch_tensormap(&tm_o);
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync();  // both CTAs' barriers are initialised before any remote use
  tc_fence_after();
  const uint32_t tbase = *tslot;
  const uint32_t rank = PAIR ? cluster_rank() : 0u;
  const int64_t worker = PAIR ? blockIdx.x / 2 : blockIdx.x, nworkers = PAIR ? gridDim.x / 2 : gridDim.x;
  const int64_t njobs = (int64_t)a.mtiles * a.nunit;
  const int nk = (a.K + kIpBK - 1) / kIpBK;

  if (warp == 0) {
    if (lane == 0) {
      uint32_t it = 0;
      for (int64_t j = worker; j < njobs && !*abort_flag; j += nworkers) {
        const int mt = (int)(j / a.nunit), u = (int)(j % a.nunit);
        for (int sg = a.unit[u].x; sg < a.unit[u].y; ++sg) {
          // this CTA's x rows and W rows (paired: the second CTA holds the upper half of the tile)
          const int arow = mt * kTileM + (int)rank * kIpBM;
          const int brow = a.seg[sg].x + (int)rank * (a.seg[sg].y / 2);
          for (int kb = 0; kb < nk; ++kb, ++it) {
            const int s = (int)(it % kIpStages);
            if (!mbar_wait(&empty[s], ((it / kIpStages) & 1) ^ 1, a.wait_ns)) {
              ip_fail(a, abort_flag);
              break;
            }
            uint8_t* dA = sm + s * kIpStageA;
            uint8_t* dB = sm + kIpStages * kIpStageA + s * kIpStageB;
            if constexpr (PAIR) {
              // both CTAs' copies complete on the first CTA's barrier, which expects all of them
              if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * (kIpStageA + kIpStageB));
              const uint32_t fb = mapa_shared(smem_u32(&full[s]), 0);
              tma_load_2d_pair(dA, &tm_x, kb * kIpBK, arow, fb);
              tma_load_2d_pair(dB, &tm_w, kb * kIpBK, brow, fb);
            } else {
              mbar_arrive_expect_tx(&full[s], kIpStageA + kIpStageB);
              tma_load_2d(dA, &tm_x, kb * kIpBK, arow, &full[s]);
              tma_load_2d(dB, &tm_w, kb * kIpBK, brow, &full[s]);
            }
          }
          if (*abort_flag) break;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      // the commits that hand a stage back / the accumulator over reach both CTAs when paired
      auto commit_both = [&](uint64_t* bar) {
        if constexpr (PAIR) {
          umma_commit_pair(smem_u32(bar));
          umma_commit_pair(mapa_shared(smem_u32(bar), 1));
        } else {
          umma_commit(bar);
        }
      };
      uint32_t it = 0, sc = 0;
      for (int64_t j = worker; j < njobs && !*abort_flag; j += nworkers) {
        const int u = (int)(j % a.nunit);
        for (int sg = a.unit[u].x; sg < a.unit[u].y; ++sg, ++sc) {
          const int acc = (int)(sc & 1);
          const bool drained = PAIR ? mbar_wait_cluster(&acce[acc], ((sc >> 1) & 1) ^ 1, a.wait_ns)
                                    : mbar_wait(&acce[acc], ((sc >> 1) & 1) ^ 1, a.wait_ns);
          if (!drained) {
            ip_fail(a, abort_flag);
            break;
          }
          tc_fence_after();
          const uint32_t idesc = idesc_bf16(kTileM, a.seg[sg].y, false, false);
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
            for (int kk = 0; kk < kIpBK / 16; ++kk) {
              const uint64_t da = kmajor_desc(tA, kIpBM, kk * 16), db = kmajor_desc(tB, kIpBN, kk * 16);
              if constexpr (PAIR)
                umma_bf16_pair(dt, da, db, idesc, (kb | kk) != 0 ? 1u : 0u);
              else
                umma_bf16(dt, da, db, idesc, (kb | kk) != 0 ? 1u : 0u);
            }
            commit_both(&empty[s]);  // the stage is free once these MMAs have read it
          }
          if (*abort_flag) break;
          commit_both(&accf[acc]);
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
    for (int64_t j = worker; j < njobs && !*abort_flag; j += nworkers) {
      const int mt = (int)(j / a.nunit), u = (int)(j % a.nunit);
      const int64_t grow = (int64_t)mt * kTileM + (int64_t)rank * kIpBM + row;
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
          const int64_t brow0 = (int64_t)mt * kTileM + (int64_t)rank * kIpBM + q * 32;
          if (lane == 0 && brow0 < a.M) {  // a box that starts past the last row is not issued
            // rows / columns past the end are not written
            tma_store_2d(&tm_o, box, col0 + c, (int)brow0);
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
        if (lane == 0) {
          if constexpr (PAIR)
            mbar_arrive_cluster(mapa_shared(smem_u32(&acce[acc]), 0));  // the MMA issuer's barrier
          else
            mbar_arrive(&acce[acc]);
        }
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
  if constexpr (PAIR) cluster_sync();  // no remote arrivals or MMAs into this CTA remain
  if (warp == 0) {
    tc_fence_after();
    ip_tmem_dealloc<PAIR>(tbase, 512);
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

// Per device: opt both kernels into their shared memory and find how many CTA pairs can be
// resident at once (0: run single CTAs).
int device_setup(int* pairs) {
  static std::mutex mu;
  static std::map<int, int> done;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(mu);
  auto f = done.find(dev);
  if (f != done.end()) {
    *pairs = f->second;
    return M3B_OK;
  }
  for (const void* k : {(const void*)in_proj_kernel<true>, (const void*)in_proj_kernel<false>}) {
    const cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kIpSmem);
    if (e != cudaSuccess) return fail(M3B_ERR_CUDA, "in_proj: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  }
  cudaLaunchConfig_t cfg{};
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(2 * (unsigned)(num_sms() / 2));
  cfg.blockDim = dim3(kIpThreads);
  cfg.dynamicSmemBytes = kIpSmem;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, (const void*)in_proj_kernel<true>, &cfg) != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  done[dev] = n;
  *pairs = n;
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
  int pairs = 0;
  int rc = device_setup(&pairs);
  if (rc != M3B_OK) return rc;
  const bool paired = pairs > 0;
  const int tile_m = paired ? 2 * kIpBM : kIpBM;
  p.mtiles = (int)((a->rows + tile_m - 1) / tile_m);
  CUtensorMap tm_x{}, tm_w{}, tm_o{};
  if (!make_map(&tm_x, a->x, a->d_model, a->rows, a->x_stride, kIpBM) ||
      !make_map(&tm_w, a->weight, a->d_model, a->d_proj, a->d_model, paired ? kIpBN / 2 : kIpBN) ||
      !make_map(&tm_o, a->proj, a->d_proj, a->rows, a->proj_stride, 32))
    return fail(M3B_ERR_CUDA, "in_proj: cuTensorMapEncodeTiled refused the operands");
  const int64_t njobs = (int64_t)p.mtiles * p.nunit;
  if (!paired) {
    const int grid = (int)(njobs < num_sms() ? njobs : num_sms());
    in_proj_kernel<false><<<grid, kIpThreads, kIpSmem, st>>>(p, tm_x, tm_w, tm_o);
    return check_launch("in_proj_kernel");
  }
  cudaLaunchConfig_t cfg{};
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(2 * (unsigned)(njobs < pairs ? njobs : pairs));
  cfg.blockDim = dim3(kIpThreads);
  cfg.dynamicSmemBytes = kIpSmem;
  cfg.stream = st;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, in_proj_kernel<true>, p, tm_x, tm_w, tm_o);
  if (e != cudaSuccess) return fail(M3B_ERR_CUDA, "in_proj_kernel: %s", cudaGetErrorString(e));
  return check_launch("in_proj_kernel");
}

}  // namespace m3b

extern "C" int m3b_in_proj(const m3b_in_proj_args* a, void* stream) {
  m3b::clear_error();
  if (!a) return m3b::fail(M3B_ERR_INVALID_ARG, "in_proj: null args");
  return m3b::launch_in_proj(a, static_cast<cudaStream_t>(stream));
}
