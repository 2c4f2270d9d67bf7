// chunked_ssd on pre-processed tensors (the reference's mamba3/ssd.py:118-244 API).
//
// Inputs are per-head and already rotated: x_g, x_b, x_raw (B,T,H,P,R), B_g, B_b, C
// (B,T,H,N,R), dt (B,T,H), A, D (H).  The token input is the rank-RI product
// u_s = sum_q Xt[s,:,q] Bt[s,:,q]^T with Xt = [x_g | x_b], Bt = [B_g | B_b]
// (RI = 2R, or R without the beta half), weighted by dt_s (mamba3/ssd.py:185-198):
//   y_t     = sum_{s<=t} exp(cum_t - cum_s) dt_s C_t . u_s + exp(cum_t) C_t . H_k + D x_raw_t
//   S_k     = sum_s exp(cum_last - cum_s) dt_s u_s,   H_{k+1} = exp(cum_last) H_k + S_k
// Same tile machinery as the fused layer kernels (chunk.cu): rows (t,r) = 128, the
// (s,q) columns are L * RI rounded up to 128 or 256, so one UMMA covers the score tile.
#include <mutex>
#include <set>
#include <utility>

#include "chunk.cuh"

namespace m3b {

struct SsdParams {
  int64_t B, T;
  int H, P, N, R, K, L;
  const void *x_g, *x_b, *B_g, *B_b, *C, *x_raw, *dt, *A, *D;
  int dt_dtype, ad_dtype;
  void* sstate;
  void* hstate;
  float* decay;
  void* y;
  int* err;
};

// ST: the state kernel's plan, which needs no C and no H tile (about 99 KB instead of 147 KB
// at NC = 256, so two state CTAs share an SM)
template <int RP, int RIP, bool ST = false>
struct GPlan {
  static constexpr int L = 128 / RP;
  static constexpr int NC = L * RIP;                 // (s,q) columns: 128 or 256
  static constexpr int tileC = 0;                    // 128 x 128 (not in the state plan)
  static constexpr int tileB = ST ? 0 : 32768;       // NC x 128
  static constexpr int tileX = tileB + NC * 256;     // 64 x NC
  static constexpr int tileH = tileX + NC * 128;     // 64 x 128
  static constexpr int cum2 = tileH + (ST ? 0 : 16384);  // the H tile is not in the state plan
  static constexpr int dtv = cum2 + (L + 1) * 4;
  static constexpr int wgt = dtv + (L + 1) * 4;
  static constexpr int bars = (wgt + L * 4 + 15) & ~15;
  static constexpr int taddr = bars + 32;
  static constexpr int bytes = taddr + 16 + 1024;
  static constexpr int tcols = NC == 256 ? 512 : 256;
  static constexpr int colY = NC, colYi = NC + 64;
  static_assert(NC == 128 || NC == 256, "column tile must be 128 or 256");
  static_assert(bytes <= 227 * 1024, "shared memory");
};

template <typename TA, int R, bool BETA, bool ST = false>
__device__ void gen_scalars(const SsdParams& a, uint8_t* sm, int b, int k, int h) {
  constexpr int RP = rp_of(R), RIP = rp_of(BETA ? 2 * R : R);
  using PL = GPlan<RP, RIP, ST>;
  constexpr int L = PL::L;
  float* cum2 = reinterpret_cast<float*>(sm + PL::cum2);
  float* dtv = reinterpret_cast<float*>(sm + PL::dtv);
  const float A = ldf(a.A, h, a.ad_dtype);
  for (int s = threadIdx.x; s < L; s += kCT) {
    const int64_t t = (int64_t)k * L + s;
    dtv[s] = t < a.T ? ldf(a.dt, ((int64_t)b * a.T + t) * a.H + h, a.dt_dtype) : 0.f;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    constexpr int PER = L / 32;
    const int lane = threadIdx.x;
    float v[PER];
    float run = 0.f;
#pragma unroll
    for (int e = 0; e < PER; ++e) {
      run += A * dtv[lane * PER + e];
      v[e] = run;
    }
    float incl = run;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float n = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += n;
    }
    const float excl = incl - run;
#pragma unroll
    for (int e = 0; e < PER; ++e) cum2[lane * PER + e] = (v[e] + excl) * kLog2e;
  }
  __syncthreads();
}

// K-major tile rows (s*RIP + q), columns n: q < R from src0, R <= q < 2R from src1.
template <typename TA, int R, int RIP>
__device__ void gen_rows(const SsdParams& a, uint8_t* tile, const void* src0, const void* src1, int b, int k,
                         int h, int L) {
  constexpr int NCH = kNS / 8;
  const int rows_per_tok = RIP;
  for (int u = threadIdx.x; u < L * NCH; u += kCT) {
    const int s = u / NCH, c = u % NCH;
    const int64_t t = (int64_t)k * L + s;
    const bool valid = (t < a.T) && (c * 8 < a.N);
    float v0[8 * R], v1[8 * R];
    if (valid) {
      const int64_t off = (((int64_t)b * a.T + t) * a.H + h) * (int64_t)a.N * R + c * 8 * R;
#pragma unroll
      for (int j = 0; j < R; ++j) {
        float tmp[8];
        load8<TA>(reinterpret_cast<const TA*>(src0) + off + j * 8, tmp);
#pragma unroll
        for (int e = 0; e < 8; ++e) v0[j * 8 + e] = tmp[e];
        if (src1) {
          load8<TA>(reinterpret_cast<const TA*>(src1) + off + j * 8, tmp);
#pragma unroll
          for (int e = 0; e < 8; ++e) v1[j * 8 + e] = tmp[e];
        }
      }
    }
#pragma unroll
    for (int q = 0; q < rows_per_tok; ++q) {
      uint4 o = make_uint4(0, 0, 0, 0);
      const float* v = q < R ? v0 : v1;
      const int r = q < R ? q : q - R;
      if (valid && (q < R || (src1 && q < 2 * R))) {
        o.x = pack_bf16x2(v[0 * R + r], v[1 * R + r]);
        o.y = pack_bf16x2(v[2 * R + r], v[3 * R + r]);
        o.z = pack_bf16x2(v[4 * R + r], v[5 * R + r]);
        o.w = pack_bf16x2(v[6 * R + r], v[7 * R + r]);
      }
      sw128_store_chunk(tile, s * rows_per_tok + q, c, rows_per_tok * L, o);
    }
  }
}

// X^T tile: row p, column (s*RIP + q) = Xt[s,p,q] (* wgt[s] when WEIGHTED).
template <typename TA, int R, int RIP, bool WEIGHTED>
__device__ void gen_x(const SsdParams& a, uint8_t* tile, const float* wgt, int b, int k, int h, int L) {
  const int NC = L * RIP;
  const int ncc = NC / 8;
  for (int u = threadIdx.x; u < kPP * ncc; u += kCT) {
    const int pp = u % kPP, cc = u / kPP;
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int col = cc * 8 + e;
      const int s = col / RIP, q = col % RIP;
      const int64_t t = (int64_t)k * L + s;
      float val = 0.f;
      if (pp < a.P && t < a.T && q < 2 * R) {
        const void* src = q < R ? a.x_g : a.x_b;
        if (src) {
          const int r = q < R ? q : q - R;
          val = io<TA>::ld(reinterpret_cast<const TA*>(src) +
                           ((((int64_t)b * a.T + t) * a.H + h) * a.P + pp) * R + r);
          if (WEIGHTED) val *= wgt[s];
        }
      }
      v[e] = val;
    }
    uint4 o;
    o.x = pack_bf16x2(v[0], v[1]);
    o.y = pack_bf16x2(v[2], v[3]);
    o.z = pack_bf16x2(v[4], v[5]);
    o.w = pack_bf16x2(v[6], v[7]);
    sw128_store_chunk(tile, pp, cc, kPP, o);
  }
}

template <typename TA, typename TS, int R, bool BETA>
__global__ void __launch_bounds__(kCT, 1) gen_state_kernel(SsdParams a) {
  constexpr int RP = rp_of(R), RIP = rp_of(BETA ? 2 * R : R);
  using PL = GPlan<RP, RIP, true>;
  constexpr int L = PL::L, NC = PL::NC;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  const int h = blockIdx.x, k = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + PL::bars);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + PL::taddr);
  if (warp == 0) {
    tmem_alloc(tslot, 64);
    tmem_relinquish();
  }
  if (threadIdx.x == 32) {
    mbar_init(&bar[0], 1);
    fence_mbar_init();
  }
  gen_scalars<TA, R, BETA, true>(a, sm, b, k, h);
  const float* cum2 = reinterpret_cast<const float*>(sm + PL::cum2);
  const float* dtv = reinterpret_cast<const float*>(sm + PL::dtv);
  float* wgt = reinterpret_cast<float*>(sm + PL::wgt);
  for (int s = threadIdx.x; s < L; s += kCT) wgt[s] = exp2f(cum2[L - 1] - cum2[s]) * dtv[s];
  if (threadIdx.x == 0) a.decay[((int64_t)b * a.K + k) * a.H + h] = exp2f(cum2[L - 1]);
  __syncthreads();
  gen_rows<TA, R, RIP>(a, sm + PL::tileB, a.B_g, BETA ? a.B_b : nullptr, b, k, h, L);
  gen_x<TA, R, RIP, true>(a, sm + PL::tileX, wgt, b, k, h, L);
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  if (threadIdx.x == 0) {
    constexpr uint32_t idesc = idesc_bf16(128, kPP, true, false);
#pragma unroll
    for (int kk = 0; kk < NC / 16; ++kk)
      umma_bf16(tbase, mnmajor_desc(sm + PL::tileB, NC, kk * 16), kmajor_desc(sm + PL::tileX, kPP, kk * 16), idesc,
                kk > 0 ? 1u : 0u);
    umma_commit(&bar[0]);
  }
  bool ok = mbar_wait(&bar[0], 0);
  __syncwarp();
  ok = __syncthreads_and(ok);
  tc_fence_after();
  if (ok) {
    const int lq = warp & 3, half = warp >> 2;
    const int n = 32 * lq + lane;
    float v[32];
    tmem_ld32(tbase + ((uint32_t)(32 * lq) << 16) + 32 * half, v);
    if (n < a.N) {
      TS* out = reinterpret_cast<TS*>(a.sstate) + (((int64_t)b * a.K + k) * a.H + h) * (int64_t)a.P * a.N + n;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int pp = 32 * half + j;
        if (pp < a.P) io<TS>::st(out + (int64_t)pp * a.N, v[j]);
      }
    }
  } else if (threadIdx.x == 0) {
    record_error(a.err, M3B_ERR_TIMEOUT);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, 64);
  }
}

template <typename TA, typename TS, int R, bool BETA>
__global__ void __launch_bounds__(kCT, 1) gen_out_kernel(SsdParams a) {
  constexpr int RP = rp_of(R), RIP = rp_of(BETA ? 2 * R : R);
  using PL = GPlan<RP, RIP>;
  constexpr int L = PL::L, NC = PL::NC;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  const int h = blockIdx.x, k = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + PL::bars);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + PL::taddr);
  if (warp == 0) {
    tmem_alloc(tslot, PL::tcols);
    tmem_relinquish();
  }
  if (threadIdx.x == 32) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    fence_mbar_init();
  }
  gen_scalars<TA, R, BETA>(a, sm, b, k, h);
  const float* cum2 = reinterpret_cast<const float*>(sm + PL::cum2);
  const float* dtv = reinterpret_cast<const float*>(sm + PL::dtv);
  // C rows (t*RP + r): reuse the row producer with RIP = RP and no second source
  gen_rows<TA, R, RP>(a, sm + PL::tileC, a.C, nullptr, b, k, h, L);
  gen_rows<TA, R, RIP>(a, sm + PL::tileB, a.B_g, BETA ? a.B_b : nullptr, b, k, h, L);
  gen_x<TA, R, RIP, false>(a, sm + PL::tileX, nullptr, b, k, h, L);
  {
    uint8_t* tH = sm + PL::tileH;
    const TS* hs = reinterpret_cast<const TS*>(a.hstate) + (((int64_t)b * a.K + k) * a.H + h) * (int64_t)a.P * a.N;
    for (int u = threadIdx.x; u < kPP * (kNS / 8); u += kCT) {
      const int pp = u / (kNS / 8), c = u % (kNS / 8);
      float v[8];
      if (pp < a.P && c * 8 < a.N) {
        load8<TS>(hs + (int64_t)pp * a.N + c * 8, v);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = 0.f;
      }
      uint4 o;
      o.x = pack_bf16x2(v[0], v[1]);
      o.y = pack_bf16x2(v[2], v[3]);
      o.z = pack_bf16x2(v[4], v[5]);
      o.w = pack_bf16x2(v[6], v[7]);
      sw128_store_chunk(tH, pp, c, kPP, o);
    }
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  if (threadIdx.x == 0) {
    constexpr uint32_t id_s = idesc_bf16(128, NC, false, false);
    constexpr uint32_t id_o = idesc_bf16(128, kPP, false, false);
#pragma unroll
    for (int kk = 0; kk < 8; ++kk)
      umma_bf16(tbase, kmajor_desc(sm + PL::tileC, 128, kk * 16), kmajor_desc(sm + PL::tileB, NC, kk * 16), id_s,
                kk > 0 ? 1u : 0u);
#pragma unroll
    for (int kk = 0; kk < 8; ++kk)
      umma_bf16(tbase + PL::colYi, kmajor_desc(sm + PL::tileC, 128, kk * 16),
                kmajor_desc(sm + PL::tileH, kPP, kk * 16), id_o, kk > 0 ? 1u : 0u);
    umma_commit(&bar[0]);
  }
  bool ok = mbar_wait(&bar[0], 0);
  __syncwarp();
  ok = __syncthreads_and(ok);
  tc_fence_after();
  const int lq = warp & 3, half = warp >> 2;
  const int m = 32 * lq + lane;
  const int t = m / RP, r = m % RP;
  const uint32_t trow = tbase + ((uint32_t)(32 * lq) << 16);
  if (ok) {
    uint8_t* tP = sm + PL::tileB;  // P = mask(S) overwrites the B tile (128 x NC, K-major)
    const float ct = cum2[t];
#pragma unroll
    for (int g2 = 0; g2 < NC / 64; ++g2) {
      const int c0 = (NC / 2) * half + 32 * g2;
      float v[32];
      tmem_ld32(trow + c0, v);
#pragma unroll
      for (int j = 0; j < 32; j += RIP) {
        const int s = (c0 + j) / RIP;
        const float w = s <= t ? exp2f(ct - cum2[s]) * dtv[s] : 0.f;
#pragma unroll
        for (int q = 0; q < RIP; ++q) v[j + q] *= w;
      }
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        uint4 o;
        o.x = pack_bf16x2(v[8 * cc + 0], v[8 * cc + 1]);
        o.y = pack_bf16x2(v[8 * cc + 2], v[8 * cc + 3]);
        o.z = pack_bf16x2(v[8 * cc + 4], v[8 * cc + 5]);
        o.w = pack_bf16x2(v[8 * cc + 6], v[8 * cc + 7]);
        sw128_store_chunk(tP, m, c0 / 8 + cc, 128, o);
      }
    }
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (ok && threadIdx.x == 0) {
    constexpr uint32_t id_o = idesc_bf16(128, kPP, false, false);
#pragma unroll
    for (int kk = 0; kk < NC / 16; ++kk)
      umma_bf16(tbase + PL::colY, kmajor_desc(sm + PL::tileB, 128, kk * 16), kmajor_desc(sm + PL::tileX, kPP, kk * 16),
                id_o, kk > 0 ? 1u : 0u);
    umma_commit(&bar[1]);
  }
  if (ok) ok = mbar_wait(&bar[1], 0);
  __syncwarp();
  ok = __syncthreads_and(ok);
  tc_fence_after();
  if (ok) {
    float Y[32], Yi[32];
    tmem_ld32(trow + PL::colY + 32 * half, Y);
    tmem_ld32(trow + PL::colYi + 32 * half, Yi);
    const int64_t tok = (int64_t)k * L + t;
    if (tok < a.T && r < R) {
      const float ec = exp2f(cum2[t]);
      const float Dh = ldf(a.D, h, a.ad_dtype);
      const int64_t base = (((int64_t)b * a.T + tok) * a.H + h) * (int64_t)a.P * R + r;
      const TA* xr = reinterpret_cast<const TA*>(a.x_raw) + base;
      TA* yo = reinterpret_cast<TA*>(a.y) + base;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int pp = 32 * half + j;
        if (pp < a.P) io<TA>::st(yo + (int64_t)pp * R, Y[j] + ec * Yi[j] + Dh * io<TA>::ld(xr + (int64_t)pp * R));
      }
    }
  } else if (threadIdx.x == 0) {
    record_error(a.err, M3B_ERR_TIMEOUT);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, PL::tcols);
  }
}

namespace {

int ensure_smem_g(const void* kernel, int bytes) {
  static std::mutex mu;
  static std::set<std::pair<const void*, int>> done;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(mu);
  if (done.count({kernel, dev})) return M3B_OK;
  const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return fail(M3B_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  done.insert({kernel, dev});
  return M3B_OK;
}

size_t up256(size_t x) { return (x + 255) & ~size_t(255); }

struct GLayout {
  size_t sstate, hstate, decay, total;
};

GLayout glayout(const m3b_ssd_args* a, int L) {
  const int64_t K = (a->seqlen + L - 1) / L;
  const size_t ssz = a->dtype == M3B_BF16 ? 2 : 4;
  GLayout w;
  size_t o = 0;
  w.sstate = o; o += up256((size_t)a->batch * K * a->H * a->P * a->N * ssz);
  w.hstate = o; o += up256((size_t)a->batch * K * a->H * a->P * a->N * ssz);
  w.decay = o; o += up256((size_t)a->batch * K * a->H * 4);
  w.total = o;
  return w;
}

template <typename TA, typename TS, int R, bool BETA>
int run_general(SsdParams& sp, const m3b_ssd_args* a, cudaStream_t st) {
  constexpr int RP = rp_of(R), RIP = rp_of(BETA ? 2 * R : R);
  using PL = GPlan<RP, RIP>;
  int rc;
  dim3 grid((unsigned)sp.H, (unsigned)sp.K, (unsigned)sp.B);
  using PS = GPlan<RP, RIP, true>;
  if ((rc = ensure_smem_g((const void*)gen_state_kernel<TA, TS, R, BETA>, PS::bytes)) != M3B_OK) return rc;
  gen_state_kernel<TA, TS, R, BETA><<<grid, kCT, PS::bytes, st>>>(sp);
  if ((rc = check_launch("ssd_state")) != M3B_OK) return rc;
  ScanLaunch s{sp.decay, sp.sstate, a->h_init, nullptr, nullptr, sp.hstate, a->h_final,
               sp.B, sp.K, sp.H, (int64_t)sp.P * sp.N, io<TS>::code};
  if ((rc = launch_scan(s, st)) != M3B_OK) return rc;
  if ((rc = ensure_smem_g((const void*)gen_out_kernel<TA, TS, R, BETA>, PL::bytes)) != M3B_OK) return rc;
  gen_out_kernel<TA, TS, R, BETA><<<grid, kCT, PL::bytes, st>>>(sp);
  return check_launch("ssd_out");
}

template <typename TA, typename TS>
int dispatch_general(SsdParams& sp, const m3b_ssd_args* a, cudaStream_t st) {
  const bool beta = a->x_b != nullptr;
  switch (a->R * 2 + (beta ? 1 : 0)) {
    case 2: return run_general<TA, TS, 1, false>(sp, a, st);
    case 3: return run_general<TA, TS, 1, true>(sp, a, st);
    case 4: return run_general<TA, TS, 2, false>(sp, a, st);
    case 5: return run_general<TA, TS, 2, true>(sp, a, st);
    case 8: return run_general<TA, TS, 4, false>(sp, a, st);
    case 9: return run_general<TA, TS, 4, true>(sp, a, st);
    default: return fail(M3B_ERR_UNSUPPORTED, "chunked_ssd: rank %d not built (1, 2, 4)", a->R);
  }
}

int gvalidate(const m3b_ssd_args* a) {
  if (!a->x_g || !a->B_g || !a->C || !a->x_raw || !a->dt || !a->A || !a->D || !a->y)
    return fail(M3B_ERR_INVALID_ARG, "chunked_ssd: null pointer");
  if ((a->x_b == nullptr) != (a->B_b == nullptr))
    return fail(M3B_ERR_INVALID_ARG, "chunked_ssd: x_b and B_b must both be given or both be NULL");
  if (a->H <= 0 || a->P <= 0 || a->N <= 0 || a->R <= 0)
    return fail(M3B_ERR_INVALID_ARG, "chunked_ssd: bad dims");
  if (a->P > kPP || a->N > kNS || a->N % 8 != 0)
    return fail(M3B_ERR_UNSUPPORTED, "chunked_ssd: needs P <= 64, N <= 128, N %% 8 == 0");
  if (a->dtype != M3B_BF16 && a->dtype != M3B_F32) return fail(M3B_ERR_UNSUPPORTED, "chunked_ssd: dtype");
  const void* vecs[] = {a->B_g, a->B_b, a->C};
  for (const void* p : vecs)
    if (p && !aligned16(p)) return fail(M3B_ERR_ALIGNMENT, "chunked_ssd: B/C need 16-byte alignment");
  if (a->batch > 65535) return fail(M3B_ERR_UNSUPPORTED, "chunked_ssd: batch > 65535");
  return M3B_OK;
}

}  // namespace

}  // namespace m3b

extern "C" size_t m3b_chunked_ssd_workspace(const m3b_ssd_args* a) {
  if (!a || m3b::gvalidate(a) != M3B_OK) return 0;
  return m3b::glayout(a, 128 / m3b::rp_of(a->R)).total;
}

extern "C" int m3b_chunked_ssd(const m3b_ssd_args* a, void* ws, size_t ws_bytes, void* stream) {
  using namespace m3b;
  if (!a) return fail(M3B_ERR_INVALID_ARG, "chunked_ssd: null args");
  int rc = gvalidate(a);
  if (rc != M3B_OK) return rc;
  if (a->batch <= 0 || a->seqlen <= 0) return M3B_OK;
  const int L = 128 / rp_of(a->R);
  const GLayout w = glayout(a, L);
  if (!ws || ws_bytes < w.total) return fail(M3B_ERR_WORKSPACE, "chunked_ssd: need %zu workspace bytes", w.total);
  if ((a->seqlen + L - 1) / L > 65535) return fail(M3B_ERR_UNSUPPORTED, "chunked_ssd: too many chunks");
  uint8_t* base = static_cast<uint8_t*>(ws);
  SsdParams sp{};
  sp.B = a->batch;
  sp.T = a->seqlen;
  sp.H = a->H;
  sp.P = a->P;
  sp.N = a->N;
  sp.R = a->R;
  sp.L = L;
  sp.K = (int)((a->seqlen + L - 1) / L);
  sp.x_g = a->x_g;
  sp.x_b = a->x_b;
  sp.B_g = a->B_g;
  sp.B_b = a->B_b;
  sp.C = a->C;
  sp.x_raw = a->x_raw;
  sp.dt = a->dt;
  sp.A = a->A;
  sp.D = a->D;
  sp.dt_dtype = a->dt_dtype;
  sp.ad_dtype = a->ad_dtype;
  sp.sstate = base + w.sstate;
  sp.hstate = base + w.hstate;
  sp.decay = reinterpret_cast<float*>(base + w.decay);
  sp.y = a->y;
  sp.err = a->err;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (a->dtype == M3B_BF16) return dispatch_general<__nv_bfloat16, __nv_bfloat16>(sp, a, st);
  return dispatch_general<float, float>(sp, a, st);
}
