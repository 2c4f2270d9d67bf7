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
  int xvec;  // x tensors take the vector loader (P % 8 == 0, 16-byte aligned): X tiles as (s, q) rows
  int yvec;  // y and x_raw are 16-byte aligned too: the output goes through a shared-memory stage
};

// The (s, q) columns of a chunk are taken one rank half at a time -- the gamma half (x_g, B_g)
// and, with the trapezoid, the beta half (x_b, B_b) -- so every column tile is L RP = 128 wide
// and the halves accumulate into the same TMEM result: 98 KB of shared memory for the output
// kernel (two CTAs per SM) and 49 KB for the state kernel (three).
// ST: the state kernel's plan, which needs no C and no H tile.
// SP (state plan only): the weighted X^T operand is also kept as its bf16 remainder (a second
// tile), so the chunk states are accurate to about 2^-17 (the backward's states).
template <int RP, int RIP, bool ST = false, bool SP = false>
struct GPlan {
  static constexpr int L = 128 / RP;
  static constexpr int NC = L * RP;                  // (s, q) columns of one rank half: 128
  static constexpr int tileC = 0;                    // 128 x 128 (not in the state plan)
  static constexpr int tileB = ST ? 0 : 32768;       // NC x 128
  static constexpr int tileX = tileB + NC * 256;     // 64 x NC
  static constexpr int tileH = tileX + NC * 128;     // 64 x 128
  static constexpr int tileXlo = tileH;             // SP: the remainder of the weighted X^T tile
  static constexpr int cum2 = tileH + (ST ? (SP ? NC * 128 : 0) : 16384);  // no H tile in the state plan
  static constexpr int dtv = cum2 + (L + 1) * 4;
  static constexpr int wgt = dtv + (L + 1) * 4;
  static constexpr int bars = (wgt + L * 4 + 15) & ~15;
  static constexpr int taddr = bars + 32;
  static constexpr int bytes = taddr + 16 + 1024;
  static constexpr int tcols = 256;
  static constexpr int colY = NC, colYi = NC + 64;
  static_assert(NC == 128, "one rank half is 128 columns");
  static_assert(ST || L * (kPP * RP + 4) * 4 <= tileH - tileB, "gen_out's fp32 output stage fits the B / X tiles");
  static_assert(bytes <= 113 * 1024, "two CTAs per SM");
};

template <typename TA, int R, bool BETA, bool ST = false, bool SP = false>
__device__ void gen_scalars(const SsdParams& a, uint8_t* sm, int b, int k, int h) {
  constexpr int RP = rp_of(R), RIP = rp_of(BETA ? 2 * R : R);
  using PL = GPlan<RP, RIP, ST, SP>;
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

// X^T tile of one rank half: row p, column (s*RP + q) = src[s,p,q] (* wgt[s] when WEIGHTED),
// q < R (zero for the padding ranks); with `lo`, also the bf16 remainder of each entry
// (entry - bf16(entry)) in a second tile.
template <typename TA, int R, bool WEIGHTED>
__device__ void gen_x(const SsdParams& a, uint8_t* tile, const float* wgt, const void* src, int b, int k, int h,
                      int L, uint8_t* lo = nullptr) {
  constexpr int RP = rp_of(R);
  const int NC = L * RP;
  const int ncc = NC / 8;
  for (int u = threadIdx.x; u < kPP * ncc; u += kCT) {
    const int pp = u % kPP, cc = u / kPP;
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int col = cc * 8 + e;
      const int s = col / RP, q = col % RP;
      const int64_t t = (int64_t)k * L + s;
      float val = 0.f;
      if (pp < a.P && t < a.T && q < R && src) {
        val = io<TA>::ld(reinterpret_cast<const TA*>(src) + ((((int64_t)b * a.T + t) * a.H + h) * a.P + pp) * R + q);
        if (WEIGHTED) val *= wgt[s];
      }
      v[e] = val;
    }
    uint32_t wh[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) wh[e] = pack_bf16x2(v[2 * e], v[2 * e + 1]);
    sw128_store_chunk(tile, pp, cc, kPP, make_uint4(wh[0], wh[1], wh[2], wh[3]));
    if (lo) {
      uint32_t wl[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 hv = bf2_to_f2(wh[e]);
        wl[e] = pack_bf16x2(v[2 * e] - hv.x, v[2 * e + 1] - hv.y);
      }
      sw128_store_chunk(lo, pp, cc, kPP, make_uint4(wl[0], wl[1], wl[2], wl[3]));
    }
  }
}

// The same X operand as rows (s RP + q) x columns p of one rank half (* wgt[s] when WEIGHTED),
// loaded with 16-byte vectors along p (P % 8 == 0, 16-byte aligned tensors) and read by the MMA
// as an MN-major operand (N = p); with `lo`, the bf16 remainder too.
template <typename TA, int R, bool WEIGHTED>
__device__ void gen_xrows(const SsdParams& a, uint8_t* tile, const float* wgt, const void* src, int b, int k, int h,
                          int L, uint8_t* lo = nullptr) {
  constexpr int RP = rp_of(R);
  constexpr int NCH = kPP / 8;
  for (int u = threadIdx.x; u < L * NCH; u += kCT) {
    const int s = u / NCH, c = u % NCH;
    const int64_t t = (int64_t)k * L + s;
    const bool valid = src && t < a.T && c * 8 < a.P;
    float v[8 * R];
    if (valid) {
      const int64_t off = (((int64_t)b * a.T + t) * a.H + h) * (int64_t)a.P * R + c * 8 * R;
#pragma unroll
      for (int j = 0; j < R; ++j) {
        float tmp[8];
        load8<TA>(reinterpret_cast<const TA*>(src) + off + j * 8, tmp);
#pragma unroll
        for (int e = 0; e < 8; ++e) v[j * 8 + e] = tmp[e];
      }
      if (WEIGHTED) {
        const float w = wgt[s];
#pragma unroll
        for (int e = 0; e < 8 * R; ++e) v[e] *= w;
      }
    }
#pragma unroll
    for (int q = 0; q < RP; ++q) {
      uint32_t wh[4] = {0u, 0u, 0u, 0u}, wl[4] = {0u, 0u, 0u, 0u};
      if (valid && q < R) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float x0 = v[(2 * e) * R + q], x1 = v[(2 * e + 1) * R + q];
          wh[e] = pack_bf16x2(x0, x1);
          const float2 hv = bf2_to_f2(wh[e]);
          wl[e] = pack_bf16x2(x0 - hv.x, x1 - hv.y);
        }
      }
      sw128_store_chunk(tile, s * RP + q, c, 128, make_uint4(wh[0], wh[1], wh[2], wh[3]));
      if (lo) sw128_store_chunk(lo, s * RP + q, c, 128, make_uint4(wl[0], wl[1], wl[2], wl[3]));
    }
  }
}

// Requests the chunk's token rows of up to four (B, T, H, W, R) tensors into L2 (one bulk
// prefetch per token and tensor; null tensors are skipped), so that the tile loaders that follow
// wait on L2 rather than on HBM.  W R elements of TA per row, 16-byte aligned rows.
template <typename TA, int R>
__device__ void prefetch_rows(const SsdParams& a, int b, int k, int h, int L, const void* t0, int w0, const void* t1,
                              int w1, const void* t2, int w2, const void* t3, int w3) {
  const void* src[4] = {t0, t1, t2, t3};
  const int wid[4] = {w0, w1, w2, w3};
  for (int u = threadIdx.x; u < 4 * L; u += kCT) {
    const int which = u / L, s = u % L;
    const int64_t t = (int64_t)k * L + s;
    const uint32_t bytes = (uint32_t)(wid[which] * R * sizeof(TA));
    // the bulk prefetch wants a 16-byte aligned address and size: other shapes go without it
    if (src[which] && t < a.T && bytes % 16 == 0 && (reinterpret_cast<uintptr_t>(src[which]) & 15) == 0)
      prefetch_l2(reinterpret_cast<const TA*>(src[which]) + (((int64_t)b * a.T + t) * a.H + h) * wid[which] * R, bytes);
  }
}

// REV (the backward's reverse chunk scan): the chunk's contribution to dL/dh at its start,
// sum_t exp(cum_t) x_t^T B_t with x = dy, B = C (weights exp(cum_t), no dt), and the chunk's
// decay, stored at chunk index K-1-k so that the forward scan kernel runs the reverse scan.
// SP: the weighted X^T operand as a hi / lo pair (two MMA groups), for states accurate to fp32.
template <typename TA, typename TS, int R, bool BETA, bool REV = false, bool SP = false>
__global__ void __launch_bounds__(kCT, 3) gen_state_kernel(SsdParams a) {
  constexpr int RP = rp_of(R), RIP = rp_of(BETA ? 2 * R : R);
  using PL = GPlan<RP, RIP, true, SP>;
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
  prefetch_rows<TA, R>(a, b, k, h, 128 / RP, a.B_g, a.N, BETA ? a.B_b : nullptr, a.N, a.x_g, a.P,
                       BETA ? a.x_b : nullptr, a.P);
  gen_scalars<TA, R, BETA, true, SP>(a, sm, b, k, h);
  const float* cum2 = reinterpret_cast<const float*>(sm + PL::cum2);
  const float* dtv = reinterpret_cast<const float*>(sm + PL::dtv);
  float* wgt = reinterpret_cast<float*>(sm + PL::wgt);
  for (int s = threadIdx.x; s < L; s += kCT) wgt[s] = REV ? exp2f(cum2[s]) : exp2f(cum2[L - 1] - cum2[s]) * dtv[s];
  const int ko = REV ? a.K - 1 - k : k;  // chunk index of the outputs
  if (threadIdx.x == 0) a.decay[((int64_t)b * a.K + ko) * a.H + h] = exp2f(cum2[L - 1]);
  __syncthreads();
  const uint32_t tbase = *tslot;
  bool ok = true;
  constexpr int NH = BETA ? 2 : 1;
  for (int hb = 0; hb < NH && ok; ++hb) {  // rank halves, accumulated into one state
    gen_rows<TA, R, RP>(a, sm + PL::tileB, hb ? a.B_b : a.B_g, nullptr, b, k, h, L);
    if (a.xvec)
      gen_xrows<TA, R, true>(a, sm + PL::tileX, wgt, hb ? a.x_b : a.x_g, b, k, h, L, SP ? sm + PL::tileXlo : nullptr);
    else
      gen_x<TA, R, true>(a, sm + PL::tileX, wgt, hb ? a.x_b : a.x_g, b, k, h, L, SP ? sm + PL::tileXlo : nullptr);
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (threadIdx.x == 0) {
      // X read K-major (rows p) from gen_x, or MN-major (rows (s, q)) from gen_xrows
      const uint32_t idesc = a.xvec ? idesc_bf16(128, kPP, true, true) : idesc_bf16(128, kPP, true, false);
      auto xdesc = [&](const uint8_t* t, int kk) {
        return a.xvec ? mnmajor_desc(t, NC, kk * 16) : kmajor_desc(t, kPP, kk * 16);
      };
#pragma unroll
      for (int kk = 0; kk < NC / 16; ++kk)
        umma_bf16(tbase, mnmajor_desc(sm + PL::tileB, NC, kk * 16), xdesc(sm + PL::tileX, kk), idesc,
                  (hb > 0 || kk > 0) ? 1u : 0u);
      if constexpr (SP) {
#pragma unroll
        for (int kk = 0; kk < NC / 16; ++kk)
          umma_bf16(tbase, mnmajor_desc(sm + PL::tileB, NC, kk * 16), xdesc(sm + PL::tileXlo, kk), idesc, 1u);
      }
      umma_commit(&bar[0]);
    }
    // the half's tiles are read until its MMAs complete
    ok = mbar_wait(&bar[0], hb & 1);
    __syncwarp();
    ok = __syncthreads_and(ok);
    tc_fence_after();
  }
  if (ok) {
    const int lq = warp & 3, half = warp >> 2;
    const int n = 32 * lq + lane;
    float v[32];
    tmem_ld32(tbase + ((uint32_t)(32 * lq) << 16) + 32 * half, v);
    if (n < a.N) {
      TS* out = reinterpret_cast<TS*>(a.sstate) + (((int64_t)b * a.K + ko) * a.H + h) * (int64_t)a.P * a.N + n;
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
__global__ void __launch_bounds__(kCT, 2) gen_out_kernel(SsdParams a) {
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
  prefetch_rows<TA, R>(a, b, k, h, 128 / RP, a.C, a.N, a.B_g, a.N, BETA ? a.B_b : nullptr, a.N, a.x_g, a.P);
  prefetch_rows<TA, R>(a, b, k, h, 128 / RP, BETA ? a.x_b : nullptr, a.P, a.x_raw, a.P, nullptr, 0, nullptr, 0);
  gen_scalars<TA, R, BETA>(a, sm, b, k, h);
  const float* cum2 = reinterpret_cast<const float*>(sm + PL::cum2);
  const float* dtv = reinterpret_cast<const float*>(sm + PL::dtv);
  // C rows (t*RP + r) and the H tile, shared by both rank halves
  gen_rows<TA, R, RP>(a, sm + PL::tileC, a.C, nullptr, b, k, h, L);
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
  const uint32_t tbase = *tslot;
  const int lq = warp & 3, half = warp >> 2;
  const int m = 32 * lq + lane;
  const int t = m / RP, r = m % RP;
  const uint32_t trow = tbase + ((uint32_t)(32 * lq) << 16);
  bool ok = true;
  constexpr int NH = BETA ? 2 : 1;
  for (int hb = 0; hb < NH && ok; ++hb) {  // rank halves: S and P per half, Y accumulated
    gen_rows<TA, R, RP>(a, sm + PL::tileB, hb ? a.B_b : a.B_g, nullptr, b, k, h, L);
    if (a.xvec)
      gen_xrows<TA, R, false>(a, sm + PL::tileX, nullptr, hb ? a.x_b : a.x_g, b, k, h, L);
    else
      gen_x<TA, R, false>(a, sm + PL::tileX, nullptr, hb ? a.x_b : a.x_g, b, k, h, L);
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (threadIdx.x == 0) {
      constexpr uint32_t id_s = idesc_bf16(128, NC, false, false);
      constexpr uint32_t id_o = idesc_bf16(128, kPP, false, false);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk)
        umma_bf16(tbase, kmajor_desc(sm + PL::tileC, 128, kk * 16), kmajor_desc(sm + PL::tileB, NC, kk * 16), id_s,
                  kk > 0 ? 1u : 0u);
      if (hb == 0) {
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_bf16(tbase + PL::colYi, kmajor_desc(sm + PL::tileC, 128, kk * 16),
                    kmajor_desc(sm + PL::tileH, kPP, kk * 16), id_o, kk > 0 ? 1u : 0u);
      }
      umma_commit(&bar[0]);
    }
    ok = mbar_wait(&bar[0], hb & 1);
    __syncwarp();
    ok = __syncthreads_and(ok);
    tc_fence_after();
    if (ok) {
      uint8_t* tP = sm + PL::tileB;  // P = mask(S) overwrites the B tile (128 x NC, K-major)
      const float ct = cum2[t];
#pragma unroll
      for (int g2 = 0; g2 < NC / 64; ++g2) {
        const int c0 = (NC / 2) * half + 32 * g2;
        float v[32];
        tmem_ld32(trow + c0, v);
#pragma unroll
        for (int j = 0; j < 32; j += RP) {
          const int s = (c0 + j) / RP;
          const float w = s <= t ? exp2f(ct - cum2[s]) * dtv[s] : 0.f;
#pragma unroll
          for (int q = 0; q < RP; ++q) v[j + q] *= w;
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
      const uint32_t id_o = a.xvec ? idesc_bf16(128, kPP, false, true) : idesc_bf16(128, kPP, false, false);
#pragma unroll
      for (int kk = 0; kk < NC / 16; ++kk)
        umma_bf16(tbase + PL::colY, kmajor_desc(sm + PL::tileB, 128, kk * 16),
                  a.xvec ? mnmajor_desc(sm + PL::tileX, NC, kk * 16) : kmajor_desc(sm + PL::tileX, kPP, kk * 16), id_o,
                  (hb > 0 || kk > 0) ? 1u : 0u);
      umma_commit(&bar[1]);
    }
    // the half's B / P and X tiles are read until its MMAs complete
    if (ok) ok = mbar_wait(&bar[1], hb & 1);
    __syncwarp();
    ok = __syncthreads_and(ok);
    tc_fence_after();
  }
  if (ok) {
    float Y[32], Yi[32];
    tmem_ld32(trow + PL::colY + 32 * half, Y);
    tmem_ld32(trow + PL::colYi + 32 * half, Yi);
    const int64_t tok = (int64_t)k * L + t;
    if (a.yvec) {
      // Y + e^cum Yi as fp32 rows (t, p R + r) in the free B / X tile space; D x_raw is added and y
      // stored below with 16-byte vectors per token row
      float* stage = reinterpret_cast<float*>(sm + PL::tileB);
      const int pitch = a.P * R + 4;
      const float ec = exp2f(cum2[t]);
      if (r < R) {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int pp = 32 * half + j;
          if (pp < a.P) stage[t * pitch + pp * R + r] = fmaf(ec, Yi[j], Y[j]);
        }
      }
    } else if (tok < a.T && r < R) {
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
  if (ok && a.yvec) {
    const float* stage = reinterpret_cast<const float*>(sm + PL::tileB);
    const int PR = a.P * R, pitch = PR + 4, nv = PR / 8;
    const float Dh = ldf(a.D, h, a.ad_dtype);
    for (int u = threadIdx.x; u < L * nv; u += kCT) {
      const int s = u / nv, c = u % nv;
      const int64_t tok = (int64_t)k * L + s;
      if (tok >= a.T) continue;
      const int64_t off = (((int64_t)b * a.T + tok) * a.H + h) * (int64_t)PR + 8 * c;
      float xv[8], o[8];
      load8<TA>(reinterpret_cast<const TA*>(a.x_raw) + off, xv);
      const float4 v0 = *reinterpret_cast<const float4*>(stage + s * pitch + 8 * c);
      const float4 v1 = *reinterpret_cast<const float4*>(stage + s * pitch + 8 * c + 4);
      const float vv[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = fmaf(Dh, xv[e], vv[e]);
      store8<TA>(reinterpret_cast<TA*>(a.y) + off, o);
    }
  }
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, PL::tcols);
  }
}

// ---------------------------------------------------------------------------
// Backward on tensor cores: the gradients of the forward above (the reference gets them from
// torch autograd through mamba3/ssd.py:27-115 and mamba3/scan.py:65-140), chunk by chunk.
// Per (batch, head), with Gamma(t, s) = exp(cum_t - cum_s) (s <= t, one chunk), h_k the state
// entering chunk k (forward chunk scan) and Gx_k = dL/dh at chunk k's end (reverse chunk scan:
// Gx_{k-1} = exp(cum_last_k) Gx_k + sum_t exp(cum_t) dy_t^T C_t, Gx_{K-1} = dh_final), the
// score tiles M = C Bt^T and W = dy Xt^T over (t, q) x (s, j) give
//   dXt_s = dt_s (sum_t (M o Gamma)^T dy + Gamma(end, s) Gx Bt_s)
//   dBt_s = sum_t (W o Gamma dt_s)^T C + Gamma(end, s) dt_s Gx^T Xt_s
//   dC_t  = sum_s (W o Gamma dt_s) Bt + exp(cum_t) dy_t h_k
// and the per-token scalars fr_t = <Xt_t, dXt_t> / dt_t, e_t = <C_t, dC_t> of the suffix pass
// that gives ddt and dA (in the token-sweep backward's finishing kernel).  One CTA per
// (head, chunk, batch row); the (s, j) columns are taken in halves (the gamma and the beta
// rank halves, R columns per token each) so a half's tiles and both masked score tiles fit in
// shared memory at once: 6 + 2 GEMM groups per half on tcgen05, fp32 accumulators in TMEM.
// ---------------------------------------------------------------------------
struct BwdTcParams {
  SsdParams s;
  const void* dy;
  const void* hstate;  // (B, K, H, P, N): state entering chunk k
  const void* gstate;  // (B, K, H, P, N): dL/dh at the end of chunk K-1-k
  void *dx_g, *dx_b, *dB_g, *dB_b, *dC, *dx_raw;
  float* fw;   // (B H, T, 8) partial sums of fr_t
  float* ew;   // (B H, T, 8) partial sums of e_t
  float* dDk;  // (B, K, H) per-chunk sums of dy . x_raw
};

// Gradient rows staged in shared memory: token s's W x R entries (the layout of the global
// tensor) at row pitch W R + 8 elements (16-byte aligned rows, staggered banks).
__host__ __device__ constexpr int bwd_pitch(int W, int R) { return W * R + 8; }

template <int RP>
struct BPlan {
  static constexpr int L = 128 / RP;
  static constexpr int tC = 0, tDY = 32768, tG = 49152, tGlo = 65536, tB = 81920, tX = 114688;
  static constexpr int tMg = 131072, tWg = 163840;
  static constexpr int tH = tMg, tHlo = tMg + 16384;  // loaded after both halves (tMg is free then)
  static constexpr int LP = ((L + 1) * 4 + 15) & ~15;
  static constexpr int cum2 = 196608, dtv = cum2 + LP;
  static constexpr int colred = dtv + LP;        // [lane quadrant][column] fp32 column sums
  static constexpr int fw = colred + 4 * 128 * 4;  // [slot][token]: partials of fr_t (6 slots)
  static constexpr int ew = fw + 6 * L * 4;        // [slot][token]: partials of e_t (6 slots)
  static constexpr int red = ew + 6 * L * 4;       // 8 floats
  static constexpr int bars = red + 32;            // 3 mbarriers
  static constexpr int taddr = bars + 32;
  static constexpr int bytes = taddr + 16 + 1024;
  static_assert(bytes <= 227 * 1024, "shared memory");
  // staged gradient rows (bf16): dBt then dXt rows in the score-tile space, dC rows in tB / tX
  static_assert(L * (bwd_pitch(kNS, RP) + bwd_pitch(kPP, RP)) * 2 <= 65536, "dBt / dXt staging");
  static_assert(L * bwd_pitch(kNS, RP) * 2 <= tMg - tB, "dC staging");
};

// Tile rows (s RP + q) x columns w < Wpad of src (B, T, H, W, R) for the L tokens of chunk k
// (K-major, 128-byte swizzle, 128 rows); zero past T, W and q >= R.
template <typename TA, int R>
__device__ void bwd_rows(uint8_t* tile, const void* src, const SsdParams& a, int W, int Wpad, int b, int k, int h) {
  constexpr int RP = rp_of(R), L = 128 / RP;
  const int NCH = Wpad / 8;
  for (int u = threadIdx.x; u < L * NCH; u += kCT) {
    const int s = u / NCH, c = u % NCH;
    const int64_t t = (int64_t)k * L + s;
    const bool valid = t < a.T && c * 8 < W;
    float v[8 * R];
    if (valid) {
      const int64_t off = (((int64_t)b * a.T + t) * a.H + h) * (int64_t)W * R + c * 8 * R;
#pragma unroll
      for (int j = 0; j < R; ++j) {
        float tmp[8];
        load8<TA>(reinterpret_cast<const TA*>(src) + off + j * 8, tmp);
#pragma unroll
        for (int e = 0; e < 8; ++e) v[j * 8 + e] = tmp[e];
      }
    }
#pragma unroll
    for (int q = 0; q < RP; ++q) {
      uint4 o = make_uint4(0, 0, 0, 0);
      if (valid && q < R) {
        o.x = pack_bf16x2(v[0 * R + q], v[1 * R + q]);
        o.y = pack_bf16x2(v[2 * R + q], v[3 * R + q]);
        o.z = pack_bf16x2(v[4 * R + q], v[5 * R + q]);
        o.w = pack_bf16x2(v[6 * R + q], v[7 * R + q]);
      }
      sw128_store_chunk(tile, s * RP + q, c, 128, o);
    }
  }
}

// Tile rows p < 64 x columns n < 128 of one fp32 (P, N) state as a split pair, hi = bf16(v) and
// lo = bf16(v - hi), so that two bf16 products carry the state to about 2^-17 (zero padded).
__device__ void bwd_state_tiles(uint8_t* hi, uint8_t* lo, const float* st, int P, int N) {
  for (int u = threadIdx.x; u < kPP * (kNS / 8); u += kCT) {
    const int pp = u / (kNS / 8), c = u % (kNS / 8);
    float v[8];
    if (pp < P && c * 8 < N) {
      load8<float>(st + (int64_t)pp * N + c * 8, v);
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = 0.f;
    }
    uint32_t wh[4], wl[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      wh[e] = pack_bf16x2(v[2 * e], v[2 * e + 1]);
      const float2 hv = bf2_to_f2(wh[e]);
      wl[e] = pack_bf16x2(v[2 * e] - hv.x, v[2 * e + 1] - hv.y);
    }
    sw128_store_chunk(hi, pp, c, kPP, make_uint4(wh[0], wh[1], wh[2], wh[3]));
    sw128_store_chunk(lo, pp, c, kPP, make_uint4(wl[0], wl[1], wl[2], wl[3]));
  }
}


// Copies the staged rows of the chunk's live tokens to dst (B, T, H, W, R) with 16-byte vectors.
template <typename TA>
__device__ void bwd_copy_out(void* dst, const uint8_t* stage, const SsdParams& a, int W, int R, int L, int b, int k,
                             int h) {
  const int WR = W * R, nv = WR / 8, pitch = bwd_pitch(W, R);
  for (int u = threadIdx.x; u < L * nv; u += kCT) {
    const int s = u / nv, c = u % nv;
    const int64_t tok = (int64_t)k * L + s;
    if (tok >= a.T) continue;
    const uint4 v = *reinterpret_cast<const uint4*>(stage + ((int64_t)s * pitch + 8 * c) * sizeof(TA));
    *reinterpret_cast<uint4*>(reinterpret_cast<TA*>(dst) + (((int64_t)b * a.T + tok) * a.H + h) * (int64_t)WR +
                              8 * c) = v;
  }
}

// waits on `bar` (thread 0), then every thread; false (for all) once the wait has timed out
__device__ __forceinline__ bool bwd_sync_wait(uint64_t* bar, uint32_t parity, bool ok, int* err) {
  if (threadIdx.x == 0 && ok && !mbar_wait(bar, parity)) {
    ok = false;
    record_error(err, M3B_ERR_TIMEOUT);
  }
  ok = __syncthreads_and(ok);
  tc_fence_after();
  return ok;
}

// Per-token scalars of the suffix pass, to fp32 accuracy: the bf16 score tiles only feed the
// stored gradients.  With the fp32 tiles M, W in TMEM (exact products of the bf16 inputs),
//   e_t  = sum_(s,j) (W o Gamma dt_s)(M) over row (t, q)     + exp(cum_t) <C_t, dy_t h_k>
//   fr_s = sum_(t,q) (M o Gamma)(W) over column (s, j)       + Gamma(end, s) <Xt_s, Gx Bt_s>
// where the state products use the split (hi + lo) state tiles.
template <typename TA, typename TS, int R, bool BETA>
__global__ void __launch_bounds__(kCT, 1) bwd_out_kernel(BwdTcParams p) {
  constexpr int RP = rp_of(R);
  using PL = BPlan<RP>;
  constexpr int L = PL::L;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  const SsdParams& a = p.s;
  const int h = blockIdx.x, k = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int lq = warp & 3, ch = warp >> 2;
  const int m = 32 * lq + lane;  // tile row = TMEM lane
  const int tr = m / RP, qr = m % RP;
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + PL::bars);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + PL::taddr);
  float* colred = reinterpret_cast<float*>(sm + PL::colred);
  float* fws = reinterpret_cast<float*>(sm + PL::fw);
  float* ews = reinterpret_cast<float*>(sm + PL::ew);
  float* red = reinterpret_cast<float*>(sm + PL::red);
  if (warp == 0) {
    tmem_alloc(tslot, 512);
    tmem_relinquish();
  }
  if (threadIdx.x == 32) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    mbar_init(&bar[2], 1);
    fence_mbar_init();
  }
  // cum2 (log2 units) and dt of the chunk's tokens
  float* cum2 = reinterpret_cast<float*>(sm + PL::cum2);
  float* dtv = reinterpret_cast<float*>(sm + PL::dtv);
  {
    const float A = ldf(a.A, h, a.ad_dtype);
    for (int s = threadIdx.x; s < L; s += kCT) {
      const int64_t t = (int64_t)k * L + s;
      dtv[s] = t < a.T ? ldf(a.dt, ((int64_t)b * a.T + t) * a.H + h, a.dt_dtype) : 0.f;
    }
    __syncthreads();
    if (threadIdx.x < 32) {
      constexpr int PER = L / 32;
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
  }
  for (int e = threadIdx.x; e < 6 * L; e += kCT) {
    fws[e] = 0.f;
    ews[e] = 0.f;
  }
  // every token row this CTA reads (C, dy, both halves of Bt and Xt, x_raw) and the two states,
  // requested into L2 up front: the tile loaders below then wait on L2, not on HBM
  {
    const int64_t PN = (int64_t)a.P * a.N;
    const void* rows[7] = {a.C, p.dy, a.B_g, a.x_g, BETA ? a.B_b : nullptr, BETA ? a.x_b : nullptr, a.x_raw};
    const int width[7] = {a.N, a.P, a.N, a.P, a.N, a.P, a.P};
    for (int u = threadIdx.x; u < 7 * L; u += kCT) {
      const int which = u / L, s = u % L;
      const int64_t t = (int64_t)k * L + s;
      if (rows[which] && t < a.T) {
        const uint32_t bytes = (uint32_t)(width[which] * R * sizeof(TA));
        prefetch_l2(reinterpret_cast<const TA*>(rows[which]) + (((int64_t)b * a.T + t) * a.H + h) * width[which] * R,
                    bytes);
      }
    }
    if (threadIdx.x < 2) {
      const float* st = threadIdx.x == 0 ? reinterpret_cast<const float*>(p.gstate) +
                                               (((int64_t)b * a.K + (a.K - 1 - k)) * a.H + h) * PN
                                         : reinterpret_cast<const float*>(p.hstate) + (((int64_t)b * a.K + k) * a.H + h) * PN;
      for (int64_t off = 0; off < PN; off += 4096) prefetch_l2(st + off, (uint32_t)((PN - off < 4096 ? PN - off : 4096) * 4));
    }
  }
  // operands shared by both halves: C, dy, Gx_k (split)
  bwd_rows<TA, R>(sm + PL::tC, a.C, a, a.N, kNS, b, k, h);
  bwd_rows<TA, R>(sm + PL::tDY, p.dy, a, a.P, kPP, b, k, h);
  const int64_t PN = (int64_t)a.P * a.N;
  bwd_state_tiles(sm + PL::tG, sm + PL::tGlo,
                  reinterpret_cast<const float*>(p.gstate) + (((int64_t)b * a.K + (a.K - 1 - k)) * a.H + h) * PN, a.P,
                  a.N);
  __syncthreads();
  const uint32_t tbase = *tslot;
  const uint32_t trow = tbase + ((uint32_t)(32 * lq) << 16);
  const float clast = cum2[L - 1];
  bool ok = true;
  constexpr int NH = BETA ? 2 : 1;
  for (int half = 0; half < NH; ++half) {
    const void* Bsrc = half ? a.B_b : a.B_g;
    const void* Xsrc = half ? a.x_b : a.x_g;
    bwd_rows<TA, R>(sm + PL::tB, Bsrc, a, a.N, kNS, b, k, h);
    bwd_rows<TA, R>(sm + PL::tX, Xsrc, a, a.P, kPP, b, k, h);
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (threadIdx.x == 0 && ok) {
      constexpr uint32_t id = idesc_bf16(128, 128, false, false);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk)  // M = C Bt^T (K = n)
        umma_bf16(tbase, kmajor_desc(sm + PL::tC, 128, kk * 16), kmajor_desc(sm + PL::tB, 128, kk * 16), id,
                  kk > 0 ? 1u : 0u);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)  // W = dy Xt^T (K = p)
        umma_bf16(tbase + 128, kmajor_desc(sm + PL::tDY, 128, kk * 16), kmajor_desc(sm + PL::tX, 128, kk * 16), id,
                  kk > 0 ? 1u : 0u);
      umma_commit(&bar[0]);
    }
    ok = bwd_sync_wait(&bar[0], half & 1, ok, a.err);
    // ---- masked score tiles Mg = M o Gamma, Wg = W o Gamma dt_s (bf16, rows (t, q), columns
    // (s, j)) and, from the fp32 tiles, the intra-chunk parts of e_t (row sums of Wg M) and of
    // fr_s (column sums of Mg W)
    if (ok) {
      const float ct = cum2[tr];
      float erow = 0.f;
#pragma unroll
      for (int c32 = 0; c32 < 2; ++c32) {
        const int c0 = 64 * ch + 32 * c32;
        float vm[32], vw[32];
        tmem_ld32(trow + c0, vm);
        tmem_ld32(trow + 128 + c0, vw);
#pragma unroll
        for (int jj = 0; jj < 32; jj += RP) {
          const int sj = (c0 + jj) / RP;
          const float g = sj <= tr ? exp2f(ct - cum2[sj]) : 0.f;
          const float gd = g * dtv[sj];
#pragma unroll
          for (int q = 0; q < RP; ++q) {
            const float mg = vm[jj + q] * g, wg = vw[jj + q] * gd;
            erow = fmaf(wg, vm[jj + q], erow);
            vw[jj + q] = wg;
            vm[jj + q] = mg;
          }
        }
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          uint4 o;
          o.x = pack_bf16x2(vm[8 * cc + 0], vm[8 * cc + 1]);
          o.y = pack_bf16x2(vm[8 * cc + 2], vm[8 * cc + 3]);
          o.z = pack_bf16x2(vm[8 * cc + 4], vm[8 * cc + 5]);
          o.w = pack_bf16x2(vm[8 * cc + 6], vm[8 * cc + 7]);
          sw128_store_chunk(sm + PL::tMg, m, c0 / 8 + cc, 128, o);
          o.x = pack_bf16x2(vw[8 * cc + 0], vw[8 * cc + 1]);
          o.y = pack_bf16x2(vw[8 * cc + 2], vw[8 * cc + 3]);
          o.z = pack_bf16x2(vw[8 * cc + 4], vw[8 * cc + 5]);
          o.w = pack_bf16x2(vw[8 * cc + 6], vw[8 * cc + 7]);
          sw128_store_chunk(sm + PL::tWg, m, c0 / 8 + cc, 128, o);
        }
        // Mg W column sums over this warp's 32 rows: a reduce-scatter leaves column c0 + lane in
        // lane `lane` (each halving step keeps the half picked by one lane bit)
        float cv[32];
        tmem_ld32(trow + 128 + c0, cv);
#pragma unroll
        for (int i = 0; i < 32; ++i) cv[i] *= vm[i];
#pragma unroll
        for (int o = 16, w = 16; o >= 1; o >>= 1, w >>= 1) {
          const bool up = (lane & o) != 0;
#pragma unroll
          for (int e = 0; e < w; ++e) {
            const float send = up ? cv[e] : cv[e + w];
            const float keep = up ? cv[e + w] : cv[e];
            cv[e] = keep + __shfl_xor_sync(0xffffffffu, send, o);
          }
        }
        colred[lq * 128 + c0 + lane] = cv[0];
      }
#pragma unroll
      for (int o = 1; o < RP; o <<= 1) erow += __shfl_xor_sync(0xffffffffu, erow, o);
      if (qr == 0) ews[(half * 2 + ch) * L + tr] = erow;
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (threadIdx.x == 0 && ok) {
      constexpr uint32_t id64mm = idesc_bf16(128, 64, true, true), id64kk = idesc_bf16(128, 64, false, false);
      constexpr uint32_t id128mm = idesc_bf16(128, 128, true, true), id128km = idesc_bf16(128, 128, false, true);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk)  // dXt (no dt): Mg^T dy, K = (t, q)
        umma_bf16(tbase + 256, mnmajor_desc(sm + PL::tMg, 128, kk * 16), mnmajor_desc(sm + PL::tDY, 128, kk * 16),
                  id64mm, kk > 0 ? 1u : 0u);
#pragma unroll
      for (int kk = 0; kk < 16; ++kk)  // Bt (Gx_hi + Gx_lo)^T, K = n
        umma_bf16(tbase + 320, kmajor_desc(sm + PL::tB, 128, (kk & 7) * 16),
                  kmajor_desc(sm + (kk < 8 ? PL::tG : PL::tGlo), 64, (kk & 7) * 16), id64kk, kk > 0 ? 1u : 0u);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk)  // dBt: Wg^T C, K = (t, q)
        umma_bf16(tbase, mnmajor_desc(sm + PL::tWg, 128, kk * 16), mnmajor_desc(sm + PL::tC, 128, kk * 16), id128mm,
                  kk > 0 ? 1u : 0u);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk)  // Xt (Gx_hi + Gx_lo), K = p
        umma_bf16(tbase + 128, kmajor_desc(sm + PL::tX, 128, (kk & 3) * 16),
                  mnmajor_desc(sm + (kk < 4 ? PL::tG : PL::tGlo), 64, (kk & 3) * 16), id128km, kk > 0 ? 1u : 0u);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk)  // dC += Wg Bt, K = (s, j), both halves into one accumulator
        umma_bf16(tbase + 384, kmajor_desc(sm + PL::tWg, 128, kk * 16), mnmajor_desc(sm + PL::tB, 128, kk * 16),
                  id128km, (half > 0 || kk > 0) ? 1u : 0u);
      umma_commit(&bar[1]);
    }
    // the column sums of this half, per token, in a fixed order (lane quadrants, then ranks)
    if (threadIdx.x < L) {
      float f = 0.f;
#pragma unroll
      for (int j = 0; j < RP; ++j)
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) f += colred[q4 * 128 + threadIdx.x * RP + j];
      fws[half * L + threadIdx.x] = f;
    }
    ok = bwd_sync_wait(&bar[1], half & 1, ok, a.err);
    // ---- dXt, dBt of this half: rows (s, j), s = tr, j = qr
    if (ok) {
      const int64_t tok = (int64_t)k * L + tr;
      const bool live = tok < a.T && qr < R;
      const float ge = exp2f(clast - cum2[tr]);  // Gamma(end, s)
      const float dts = dtv[tr];
      float frs = 0.f;  // <Xt_s, Gx Bt_s> (inter-chunk part of fr_s)
      {
        float v1[32], v2[32];
        tmem_ld32(trow + 256 + 32 * ch, v1);
        tmem_ld32(trow + 320 + 32 * ch, v2);
        // staged (s, p, j) rows: after the dBt rows in the free score-tile space
        TA* dst = reinterpret_cast<TA*>(sm + PL::tMg + L * bwd_pitch(kNS, R) * (int)sizeof(TA)) +
                  tr * bwd_pitch(a.P, R) + qr;
#pragma unroll
        for (int c8 = 0; c8 < 4; ++c8) {
          const int p0 = 32 * ch + 8 * c8;
          const uint4 xq = *reinterpret_cast<const uint4*>(sm + PL::tX + sw128_offset(m, p0, 128));
          const uint32_t xw[4] = {xq.x, xq.y, xq.z, xq.w};
#pragma unroll
          for (int e2 = 0; e2 < 4; ++e2) {
            const float2 xv = bf2_to_f2(xw[e2]);
            const int i = 8 * c8 + 2 * e2;
            frs = fmaf(xv.x, v2[i], fmaf(xv.y, v2[i + 1], frs));
            if (live) {
              if (p0 + 2 * e2 < a.P) io<TA>::st(dst + (p0 + 2 * e2) * R, dts * fmaf(ge, v2[i], v1[i]));
              if (p0 + 2 * e2 + 1 < a.P) io<TA>::st(dst + (p0 + 2 * e2 + 1) * R, dts * fmaf(ge, v2[i + 1], v1[i + 1]));
            }
          }
        }
      }
#pragma unroll
      for (int o = 1; o < RP; o <<= 1) frs += __shfl_xor_sync(0xffffffffu, frs, o);
      if (qr == 0) fws[(2 + half * 2 + ch) * L + tr] = ge * frs;
      const float tail = ge * dts;
      TA* dstB = reinterpret_cast<TA*>(sm + PL::tMg) + tr * bwd_pitch(a.N, R) + qr;  // staged (s, n, j) rows
#pragma unroll
      for (int c32 = 0; c32 < 2; ++c32) {
        const int n0 = 64 * ch + 32 * c32;
        float v3[32], v4[32];
        tmem_ld32(trow + n0, v3);
        tmem_ld32(trow + 128 + n0, v4);
        if (live) {
#pragma unroll
          for (int e = 0; e < 32; ++e)
            if (n0 + e < a.N) io<TA>::st(dstB + (n0 + e) * R, fmaf(tail, v4[e], v3[e]));
        }
      }
    }
    tc_fence_before();
    __syncthreads();  // TMEM columns 0-383 and the half's tiles are free again; the rows are staged
    tc_fence_after();
    if (ok) {
      bwd_copy_out<TA>(half ? p.dB_b : p.dB_g, sm + PL::tMg, a, a.N, R, L, b, k, h);
      bwd_copy_out<TA>(half ? p.dx_b : p.dx_g, sm + PL::tMg + L * bwd_pitch(kNS, R) * (int)sizeof(TA), a, a.P, R, L,
                       b, k, h);
    }
    __syncthreads();  // the staging space is the next half's score tiles
  }
  // ---- dC = Wg Bt (both halves) + exp(cum_t) dy h_k, h_k split into the free score-tile space
  bwd_state_tiles(sm + PL::tH, sm + PL::tHlo,
                  reinterpret_cast<const float*>(p.hstate) + (((int64_t)b * a.K + k) * a.H + h) * PN, a.P, a.N);
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (threadIdx.x == 0 && ok) {
    constexpr uint32_t id128km = idesc_bf16(128, 128, false, true);
#pragma unroll
    for (int kk = 0; kk < 8; ++kk)
      umma_bf16(tbase, kmajor_desc(sm + PL::tDY, 128, (kk & 3) * 16),
                mnmajor_desc(sm + (kk < 4 ? PL::tH : PL::tHlo), 64, (kk & 3) * 16), id128km, kk > 0 ? 1u : 0u);
    umma_commit(&bar[2]);
  }
  ok = bwd_sync_wait(&bar[2], 0, ok, a.err);
  if (ok) {
    const int64_t tok = (int64_t)k * L + tr;
    const bool live = tok < a.T && qr < R;
    const float ec = exp2f(cum2[tr]);
    float es = 0.f;  // <C_t, dy_t h_k> (inter-chunk part of e_t, before exp(cum_t))
    TA* dst = reinterpret_cast<TA*>(sm + PL::tB) + tr * bwd_pitch(a.N, R) + qr;  // staged (t, n, q) rows
#pragma unroll
    for (int c32 = 0; c32 < 2; ++c32) {
      const int n0 = 64 * ch + 32 * c32;
      float v5[32], v6[32];
      tmem_ld32(trow + 384 + n0, v5);
      tmem_ld32(trow + n0, v6);
#pragma unroll
      for (int c8 = 0; c8 < 4; ++c8) {
        const uint4 cq = *reinterpret_cast<const uint4*>(sm + PL::tC + sw128_offset(m, n0 + 8 * c8, 128));
        const uint32_t cw[4] = {cq.x, cq.y, cq.z, cq.w};
#pragma unroll
        for (int e2 = 0; e2 < 4; ++e2) {
          const float2 cv = bf2_to_f2(cw[e2]);
          const int i = 8 * c8 + 2 * e2;
          es = fmaf(cv.x, v6[i], fmaf(cv.y, v6[i + 1], es));
          if (live) {
            if (n0 + i < a.N) io<TA>::st(dst + (n0 + i) * R, fmaf(ec, v6[i], v5[i]));
            if (n0 + i + 1 < a.N) io<TA>::st(dst + (n0 + i + 1) * R, fmaf(ec, v6[i + 1], v5[i + 1]));
          }
        }
      }
    }
#pragma unroll
    for (int o = 1; o < RP; o <<= 1) es += __shfl_xor_sync(0xffffffffu, es, o);
    if (qr == 0) ews[(4 + ch) * L + tr] = ec * es;
  }
  __syncthreads();
  if (ok) bwd_copy_out<TA>(p.dC, sm + PL::tB, a, a.N, R, L, b, k, h);
  // ---- dx_raw = D dy and this chunk's share of dD = sum dy . x_raw
  float dd = 0.f;
  {
    const float Dh = ldf(a.D, h, a.ad_dtype);
    const int PR = a.P * R, n8 = PR / 8;
    for (int u = threadIdx.x; u < L * n8; u += kCT) {
      const int s = u / n8, c = u % n8;
      const int64_t tok = (int64_t)k * L + s;
      if (tok >= a.T) continue;
      const int64_t off = (((int64_t)b * a.T + tok) * a.H + h) * (int64_t)PR + 8 * c;
      float dv[8], xv[8], o[8];
      load8<TA>(reinterpret_cast<const TA*>(p.dy) + off, dv);
      load8<TA>(reinterpret_cast<const TA*>(a.x_raw) + off, xv);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        o[e] = Dh * dv[e];
        dd = fmaf(dv[e], xv[e], dd);
      }
      store8<TA>(reinterpret_cast<TA*>(p.dx_raw) + off, o);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) dd += __shfl_xor_sync(0xffffffffu, dd, o);
    if (lane == 0) red[warp] = dd;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float sd = 0.f;
    for (int w = 0; w < kCT / 32; ++w) sd += red[w];
    p.dDk[((int64_t)b * a.K + k) * a.H + h] = sd;
  }
  // ---- per-token partials of fr_t and e_t for the suffix pass (8 slots per token)
  for (int u = threadIdx.x; u < L * 8; u += kCT) {
    const int s = u / 8, w = u % 8;
    const int64_t tok = (int64_t)k * L + s;
    if (tok >= a.T) continue;
    const int64_t o = (((int64_t)b * a.H + h) * a.T + tok) * 8 + w;
    p.fw[o] = w < 6 && ok ? fws[w * L + s] : 0.f;
    p.ew[o] = w < 6 && ok ? ews[w * L + s] : 0.f;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

// m_T = <dh_final, h_final> and sum_k dDk per (batch, head), in a fixed order
__global__ void __launch_bounds__(256) bwd_tc_sums_kernel(const float* dhf, const float* hfin, const float* dDk,
                                                          float* mT, float* dDf, int K, int H, int64_t PN) {
  __shared__ float red[8];
  const int64_t bh = blockIdx.x;
  const int64_t b = bh / H;
  const int h = (int)(bh - b * H);
  float s = 0.f;
  if (dhf)
    for (int64_t i = threadIdx.x; i < PN; i += 256) s = fmaf(dhf[bh * PN + i], hfin[bh * PN + i], s);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < 8; ++w) t += red[w];
    mT[bh] = t;
    float d = 0.f;
    for (int k = 0; k < K; ++k) d += dDk[(b * K + k) * H + h];
    dDf[bh] = d;
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
  sp.xvec = a->P % 8 == 0 && aligned16(a->x_g) && (!a->x_b || aligned16(a->x_b));
  sp.yvec = sp.xvec && aligned16(a->x_raw) && aligned16(a->y);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (a->dtype == M3B_BF16) return dispatch_general<__nv_bfloat16, __nv_bfloat16>(sp, a, st);
  return dispatch_general<float, float>(sp, a, st);
}

// ---------------------------------------------------------------------------
// Backward on tensor cores: host side (called by m3b_chunked_ssd_bwd, which then runs the
// suffix pass and the head sums of the token-sweep backward on the partials written here).
// ---------------------------------------------------------------------------
namespace m3b {

namespace {

struct BwdTcLayout {
  size_t sstate, hstate, gsstate, gstate, decay_f, decay_r, hfin, dDk, total;
};

BwdTcLayout bwd_tc_layout(const m3b_ssd_bwd_args* a) {
  const int L = 128 / rp_of(a->R);
  const size_t K = (size_t)((a->seqlen + L - 1) / L);
  const size_t st = (size_t)a->batch * K * a->H * a->P * a->N * 4;  // fp32 states
  const size_t dec = (size_t)a->batch * K * a->H * 4;
  BwdTcLayout w{};
  size_t o = 0;
  w.sstate = o; o += up256(st);
  w.hstate = o; o += up256(st);
  w.gsstate = o; o += up256(st);
  w.gstate = o; o += up256(st);
  w.decay_f = o; o += up256(dec);
  w.decay_r = o; o += up256(dec);
  w.hfin = o; o += up256((size_t)a->batch * a->H * a->P * a->N * 4);
  w.dDk = o; o += up256(dec);
  w.total = o;
  return w;
}

template <int R, bool BETA>
int bwd_tc_t(const m3b_ssd_bwd_args* a, uint8_t* base, float* fw, float* ew, float* mT, float* dDf, cudaStream_t st) {
  using TA = __nv_bfloat16;
  constexpr int RP = rp_of(R), RIP = rp_of(BETA ? 2 * R : R), L = 128 / RP;
  const BwdTcLayout w = bwd_tc_layout(a);
  const int K = (int)((a->seqlen + L - 1) / L);
  const int64_t PN = (int64_t)a->P * a->N;
  SsdParams f{};
  f.B = a->batch;
  f.T = a->seqlen;
  f.H = a->H;
  f.P = a->P;
  f.N = a->N;
  f.R = a->R;
  f.L = L;
  f.K = K;
  f.x_g = a->x_g;
  f.x_b = a->x_b;
  f.B_g = a->B_g;
  f.B_b = a->B_b;
  f.C = a->C;
  f.x_raw = a->x_raw;
  f.dt = a->dt;
  f.A = a->A;
  f.D = a->D;
  f.dt_dtype = a->dt_dtype;
  f.ad_dtype = a->ad_dtype;
  f.xvec = 1;  // bwd_tc_ok: P % 8 == 0 and 16-byte aligned tensors (dy included)
  f.sstate = base + w.sstate;
  f.hstate = base + w.hstate;
  f.decay = reinterpret_cast<float*>(base + w.decay_f);
  dim3 grid((unsigned)a->H, (unsigned)K, (unsigned)a->batch);
  int rc;
  // states entering each chunk: chunk increments, then the forward scan (h_final kept for m_T)
  using PS = GPlan<RP, RIP, true, true>;
  if ((rc = ensure_smem_g((const void*)gen_state_kernel<TA, float, R, BETA, false, true>, PS::bytes)) != M3B_OK)
    return rc;
  gen_state_kernel<TA, float, R, BETA, false, true><<<grid, kCT, PS::bytes, st>>>(f);
  if ((rc = check_launch("chunked_ssd_bwd (states)")) != M3B_OK) return rc;
  float* hfin = reinterpret_cast<float*>(base + w.hfin);
  ScanLaunch sf{f.decay, f.sstate, a->h_init, nullptr, nullptr, f.hstate, hfin, f.B, K, f.H, PN, M3B_F32};
  if ((rc = launch_scan(sf, st)) != M3B_OK) return rc;
  // dL/dh at each chunk's end: chunk contributions sum_t exp(cum_t) dy_t^T C_t in reversed chunk
  // order, then the same scan from dh_final (its final state is dh_init)
  SsdParams r = f;
  r.x_g = a->dy;
  r.x_b = nullptr;
  r.B_g = a->C;
  r.B_b = nullptr;
  r.sstate = base + w.gsstate;
  r.decay = reinterpret_cast<float*>(base + w.decay_r);
  using PR = GPlan<RP, RP, true, true>;
  if ((rc = ensure_smem_g((const void*)gen_state_kernel<TA, float, R, false, true, true>, PR::bytes)) != M3B_OK)
    return rc;
  gen_state_kernel<TA, float, R, false, true, true><<<grid, kCT, PR::bytes, st>>>(r);
  if ((rc = check_launch("chunked_ssd_bwd (reverse states)")) != M3B_OK) return rc;
  ScanLaunch sr{r.decay, r.sstate, a->dh_final, nullptr, nullptr, base + w.gstate, a->dh_init, f.B, K, f.H, PN,
                M3B_F32};
  if ((rc = launch_scan(sr, st)) != M3B_OK) return rc;
  // per-chunk gradients and per-token partials
  BwdTcParams bp{};
  bp.s = f;
  bp.dy = a->dy;
  bp.hstate = f.hstate;
  bp.gstate = base + w.gstate;
  bp.dx_g = a->dx_g;
  bp.dx_b = a->dx_b;
  bp.dB_g = a->dB_g;
  bp.dB_b = a->dB_b;
  bp.dC = a->dC;
  bp.dx_raw = a->dx_raw;
  bp.fw = fw;
  bp.ew = ew;
  bp.dDk = reinterpret_cast<float*>(base + w.dDk);
  using PB = BPlan<RP>;
  if ((rc = ensure_smem_g((const void*)bwd_out_kernel<TA, float, R, BETA>, PB::bytes)) != M3B_OK) return rc;
  bwd_out_kernel<TA, float, R, BETA><<<grid, kCT, PB::bytes, st>>>(bp);
  if ((rc = check_launch("chunked_ssd_bwd (chunk gradients)")) != M3B_OK) return rc;
  bwd_tc_sums_kernel<<<(unsigned)(a->batch * a->H), 256, 0, st>>>(a->dh_final, hfin, bp.dDk, mT, dDf, K, a->H, PN);
  return check_launch("chunked_ssd_bwd (sums)");
}

}  // namespace

bool bwd_tc_ok(const m3b_ssd_bwd_args* a) {
  const void* vec[] = {a->x_g, a->x_b, a->B_g, a->B_b, a->C, a->x_raw, a->dy, a->dx_g, a->dx_b, a->dB_g, a->dB_b,
                       a->dC, a->dx_raw};
  for (const void* p : vec)
    if (p && !aligned16(p)) return false;
  const int L = 128 / rp_of(a->R);
  return a->dtype == M3B_BF16 && a->N <= kNS && a->N % 8 == 0 && a->P <= kPP && a->P % 8 == 0 &&
         (a->R == 1 || a->R == 2 || a->R == 4) && a->seqlen > 0 && a->batch > 0 && a->batch <= 65535 &&
         (a->seqlen + L - 1) / L <= 65535;
}

size_t bwd_tc_workspace(const m3b_ssd_bwd_args* a) { return bwd_tc_layout(a).total; }

int bwd_tc_run(const m3b_ssd_bwd_args* a, void* ws, float* fw, float* ew, float* mT, float* dDf, cudaStream_t st) {
  uint8_t* base = static_cast<uint8_t*>(ws);
  const bool beta = a->x_b != nullptr;
  switch (a->R * 2 + (beta ? 1 : 0)) {
    case 2: return bwd_tc_t<1, false>(a, base, fw, ew, mT, dDf, st);
    case 3: return bwd_tc_t<1, true>(a, base, fw, ew, mT, dDf, st);
    case 4: return bwd_tc_t<2, false>(a, base, fw, ew, mT, dDf, st);
    case 5: return bwd_tc_t<2, true>(a, base, fw, ew, mT, dDf, st);
    case 8: return bwd_tc_t<4, false>(a, base, fw, ew, mT, dDf, st);
    case 9: return bwd_tc_t<4, true>(a, base, fw, ew, mT, dDf, st);
    default: return fail(M3B_ERR_UNSUPPORTED, "chunked_ssd_bwd: rank %d", a->R);
  }
}

}  // namespace m3b
