// Layer forward (parallel chunked form) of the Mamba-3 SSD:
//   K0  prep_kernel          per token: 1/rms of B and C; per chunk: sum of dt*theta
//   K0b angle_prefix_kernel  angle before every chunk (cross-chunk prefix in fp64)
//   K2  chunk_state_kernel   S'_k = (w B^)^T X  on tcgen05 (M = N = 128 state rows, N = 64 head dims)
//   K3  scan (scan.cu)       H'_{k+1} = d_k H'_k + S'_k, h_final
//   K14 chunk_out_kernel     S = C^ B^T -> decay mask -> P X, plus C^ H'_k, D x, gate, MIMO down
//   last_bx_kernel           prefill's prev_BX (mamba3/mamba3.py:248-250)
// The reference computation these replace is mamba3/mamba3.py:198-256 with
// mamba3/ssd.py:118-244; the algebra is written out in chunk.cuh.
#include <map>
#include <mutex>
#include <set>
#include <tuple>
#include <utility>
#include <vector>

#include "chunk.cuh"

namespace m3b {

// ---------------------------------------------------------------------------
// K0: per-token 1/rms of the B and C rows of every group, per-chunk angle sums
// ---------------------------------------------------------------------------
template <typename TA>
__global__ void __launch_bounds__(kCT) prep_kernel(FwdParams a) {
  __shared__ float s_th[128][64];
  __shared__ float s_dt[128][32];
  const m3b_layer_params& p = a.prm;
  const int k = blockIdx.x, b = blockIdx.y;
  const int L = a.L;
  const int64_t t0 = (int64_t)k * L;
  const int nt = (int)((a.T - t0) < L ? (a.T - t0) : L);
  const int G = p.G, NR = p.N * p.R, H = p.H;
  const int offB = 2 * H * p.P, offC = offB + G * NR;
  const TA* base = reinterpret_cast<const TA*>(a.proj) + ((int64_t)b * a.T + t0) * a.proj_stride;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int pr = warp; pr < nt * G; pr += kCT / 32) {
    const int t = pr / G, g = pr % G;
    const TA* row = base + (int64_t)t * a.proj_stride;
    float sb = 0.f, sc = 0.f;
    for (int e = lane; e < NR; e += 32) {
      const float vb = io<TA>::ld(row + offB + g * NR + e);
      const float vc = io<TA>::ld(row + offC + g * NR + e);
      sb = fmaf(vb, vb, sb);
      sc = fmaf(vc, vc, sc);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      sb += __shfl_xor_sync(0xffffffffu, sb, o);
      sc += __shfl_xor_sync(0xffffffffu, sc, o);
    }
    if (lane == 0) {
      float* o = a.rms + (((int64_t)b * a.T + t0 + t) * G + g) * 2;
      o[0] = rsqrtf(sb / (float)NR + p.norm_eps);
      o[1] = rsqrtf(sc / (float)NR + p.norm_eps);
    }
  }
  if (!p.complex_ssm || !a.asum) return;
  const int nh2 = p.N / 2;
  const int offTh = offC + G * NR + H + (p.trapezoidal ? H : 0);
  for (int e = threadIdx.x; e < nt * nh2; e += kCT) {
    const int t = e / nh2, i = e % nh2;
    s_th[t][i] = io<TA>::ld(base + (int64_t)t * a.proj_stride + offTh + i);
  }
  for (int hb = 0; hb < H; hb += 32) {
    __syncthreads();
    for (int e = threadIdx.x; e < nt * 32; e += kCT) {
      const int t = e >> 5, hh = e & 31;
      if (hb + hh < H)
        s_dt[t][hh] = token_dt<TA>(a, base + (int64_t)t * a.proj_stride, (int64_t)b * a.T + t0 + t, hb + hh);
    }
    __syncthreads();
    for (int e = threadIdx.x; e < 32 * nh2; e += kCT) {
      const int hh = e / nh2, i = e % nh2;
      if (hb + hh >= H) continue;
      float acc = 0.f;
      for (int t = 0; t < nt; ++t) acc = fmaf(s_dt[t][hh], s_th[t][i], acc);
      a.asum[(((int64_t)b * a.K + k) * H + hb + hh) * nh2 + i] = acc;
    }
  }
}

// ---------------------------------------------------------------------------
// K0b: omega[b,k,h,i] = angle_init - sum_{k'<k} asum[b,k',h,i]  (fp64 carry),
// omega[b,K,h,i] = final angle.  One CTA per (b,h); threads over (i, segment of K).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kCT) angle_prefix_kernel(FwdParams a) {
  __shared__ double s_tot[kCT];
  const m3b_layer_params& p = a.prm;
  const int H = p.H, nh2 = p.N / 2, K = a.K;
  const int b = blockIdx.x / H, h = blockIdx.x % H;
  const int nseg = kCT / nh2;
  const int i = threadIdx.x % nh2, seg = threadIdx.x / nh2;
  const bool act = seg < nseg;
  const int per = (K + nseg - 1) / nseg;
  const int klo = act ? min(K, seg * per) : K, khi = act ? min(K, klo + per) : K;
  const float* src = a.asum + ((int64_t)b * K * H + h) * nh2 + i;
  double tot = 0.0;
  for (int k = klo; k < khi; ++k) tot += (double)src[(int64_t)k * H * nh2];
  s_tot[threadIdx.x] = tot;
  __syncthreads();
  if (!act) return;
  double acc = 0.0;
  for (int s = 0; s < seg; ++s) acc += s_tot[s * nh2 + i];
  const double init = a.angle_init ? (double)a.angle_init[((int64_t)b * H + h) * nh2 + i] : 0.0;
  float* dst = a.omega + ((int64_t)b * (K + 1) * H + h) * nh2 + i;
  for (int k = klo; k < khi; ++k) {
    dst[(int64_t)k * H * nh2] = (float)(init - acc);
    acc += (double)src[(int64_t)k * H * nh2];
  }
  if (seg == nseg - 1) {
    dst[(int64_t)K * H * nh2] = (float)(init - acc);
    if (a.angle_final) a.angle_final[((int64_t)b * H + h) * nh2 + i] = (float)(init - acc);
  }
}

// Common prologue of the two tensor-core chunk kernels.
template <typename TA, int R>
__device__ void chunk_prologue(const FwdParams& a, uint8_t* sm, int b, int k, int h, int g, bool out_kernel) {
  constexpr int RP = rp_of(R);
  using PL = Plan<RP, TA>;
  constexpr int L = PL::L;
  float* rmsv = reinterpret_cast<float*>(sm + PL::rmsv);
  for (int s = threadIdx.x; s < L; s += kCT) {
    const int64_t t = (int64_t)k * L + s;
    float rb = 0.f, rc = 0.f;
    if (t < a.T) {
      const float* src = a.rms + (((int64_t)b * a.T + t) * a.prm.G + g) * 2;
      rb = src[0];
      rc = src[1];
    }
    rmsv[2 * s] = rb;
    rmsv[2 * s + 1] = rc;
  }
  chunk_params<TA, RP>(a, sm, h, g, out_kernel);
  chunk_scalars<TA, RP>(a, sm, b, k, h);  // ends with __syncthreads
  if (a.prm.complex_ssm) chunk_angles<TA, RP>(a, sm, b, k, h);
  chunk_stage_xz<TA, RP>(a, sm, b, k, h, out_kernel);
}

// ---------------------------------------------------------------------------
// K2: chunk increments S'_k[p,n] = sum_{(s,q)} B^[(s,q),n] * w_s x_r[s,p,q]
// D (TMEM lanes = n, columns = p) = A (B^ tile read MN-major) x B (wX^T, K-major)
// ---------------------------------------------------------------------------
template <typename TA, typename TS, int R>
__global__ void __launch_bounds__(kCT, 1) chunk_state_kernel(FwdParams a) {
  constexpr int RP = rp_of(R);
  using PL = Plan<RP, TA>;
  constexpr int L = PL::L;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  const m3b_layer_params& p = a.prm;
  const int h = blockIdx.x, k = blockIdx.y, b = blockIdx.z;
  const int g = h / (p.H / p.G);
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
  chunk_prologue<TA, R>(a, sm, b, k, h, g, false);
  const float* cum2 = reinterpret_cast<const float*>(sm + PL::cum2);
  const float* gam = reinterpret_cast<const float*>(sm + PL::gam);
  const float* bpr = reinterpret_cast<const float*>(sm + PL::bpr);
  float* wgt = reinterpret_cast<float*>(sm + PL::wgt);
  for (int s = threadIdx.x; s < L; s += kCT) wgt[s] = exp2f(cum2[L - 1] - cum2[s]) * (gam[s] + bpr[s + 1]);
  if (threadIdx.x == 0) {
    a.decay[((int64_t)b * a.K + k) * p.H + h] = exp2f(cum2[L - 1]);
    if (k == 0) a.coef0[(int64_t)b * p.H + h] = bpr[0];
  }
  __syncthreads();
  chunk_produce_bc<TA, R, true, false, PL::F32>(a, sm, b, k, g);  // fp32: B^ transposed (K-major A)
  if constexpr (PL::F32) __syncthreads();  // the angles (in the X tile region) have been read
  chunk_produce_x<TA, RP, true>(a, sm, b, k, h);
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  if (threadIdx.x == 0) {
    if constexpr (PL::F32) {
      constexpr uint32_t idesc = idesc_tf32(128, kPP, /*a_mn=*/false, /*b_mn=*/false);
#pragma unroll
      for (int kk = 0; kk < 16; ++kk)
        umma_tf32(tbase, kmajor_desc_b(sm + PL::tileB, 128, kk * 32), kmajor_desc_b(sm + PL::tileX, kPP, kk * 32),
                  idesc, kk > 0 ? 1u : 0u);
    } else {
      constexpr uint32_t idesc = idesc_bf16(128, kPP, /*a_mn=*/true, /*b_mn=*/false);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk)
        umma_bf16(tbase, mnmajor_desc(sm + PL::tileB, 128, kk * 16), kmajor_desc(sm + PL::tileX, kPP, kk * 16),
                  idesc, kk > 0 ? 1u : 0u);
    }
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
    if (n < p.N) {
      TS* out = reinterpret_cast<TS*>(a.sstate) + (((int64_t)b * a.K + k) * p.H + h) * (int64_t)p.P * p.N + n;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int pp = 32 * half + j;
        if (pp < p.P) io<TS>::st(out + (int64_t)pp * p.N, v[j]);
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

// ---------------------------------------------------------------------------
// K14: intra-chunk + inter-chunk output with the D skip, gate and MIMO down.
// TMEM columns: [0,128) S = C^ B^T, [128,192) Y = P X, [192,256) Yi = C^ H'^T.
// ---------------------------------------------------------------------------
template <typename TA, typename TS, int R>
__global__ void __launch_bounds__(kCT, 1) chunk_out_kernel(FwdParams a) {
  constexpr int RP = rp_of(R);
  using PL = Plan<RP, TA>;
  constexpr int L = PL::L;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  const m3b_layer_params& p = a.prm;
  const int h = blockIdx.x, k = blockIdx.y, b = blockIdx.z;
  const int g = h / (p.H / p.G);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + PL::bars);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + PL::taddr);
  if (warp == 0) {
    tmem_alloc(tslot, 256);
    tmem_relinquish();
  }
  if (threadIdx.x == 32) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    fence_mbar_init();
  }
  chunk_prologue<TA, R>(a, sm, b, k, h, g, true);
  const float* cum2 = reinterpret_cast<const float*>(sm + PL::cum2);
  const float* gam = reinterpret_cast<const float*>(sm + PL::gam);
  const float* bpr = reinterpret_cast<const float*>(sm + PL::bpr);
  float* wgt = reinterpret_cast<float*>(sm + PL::wgt);
  for (int s = threadIdx.x; s < L; s += kCT) wgt[s] = gam[s] + bpr[s + 1];
  // H'_k tile: row p, column n
  {
    uint8_t* tH = sm + PL::tileH;
    const TS* hs = reinterpret_cast<const TS*>(a.hstate) + (((int64_t)b * a.K + k) * p.H + h) * (int64_t)p.P * p.N;
    for (int u = threadIdx.x; u < kPP * (kNS / 8); u += kCT) {
      const int pp = u / (kNS / 8), c = u % (kNS / 8);
      float v[8];
      if (pp < p.P && c * 8 < p.N) {
        load8<TS>(hs + (int64_t)pp * p.N + c * 8, v);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = 0.f;
      }
      tile_store8<TA>(tH, pp, c, kPP, v);
    }
  }
  __syncthreads();
  chunk_produce_bc<TA, R, true, true>(a, sm, b, k, g);
  if constexpr (PL::F32) __syncthreads();  // the angles (in the X tile region) have been read
  chunk_produce_x<TA, RP, false>(a, sm, b, k, h);
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  if (threadIdx.x == 0) {
    if constexpr (PL::F32) {
      constexpr uint32_t id_s = idesc_tf32(128, 128, false, false);
      constexpr uint32_t id_o = idesc_tf32(128, kPP, false, false);
#pragma unroll
      for (int kk = 0; kk < 16; ++kk)
        umma_tf32(tbase, kmajor_desc_b(sm + PL::tileC, 128, kk * 32), kmajor_desc_b(sm + PL::tileB, 128, kk * 32),
                  id_s, kk > 0 ? 1u : 0u);
#pragma unroll
      for (int kk = 0; kk < 16; ++kk)
        umma_tf32(tbase + 192, kmajor_desc_b(sm + PL::tileC, 128, kk * 32),
                  kmajor_desc_b(sm + PL::tileH, kPP, kk * 32), id_o, kk > 0 ? 1u : 0u);
    } else {
      constexpr uint32_t id_s = idesc_bf16(128, 128, false, false);
      constexpr uint32_t id_o = idesc_bf16(128, kPP, false, false);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk)
        umma_bf16(tbase, kmajor_desc(sm + PL::tileC, 128, kk * 16), kmajor_desc(sm + PL::tileB, 128, kk * 16), id_s,
                  kk > 0 ? 1u : 0u);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk)
        umma_bf16(tbase + 192, kmajor_desc(sm + PL::tileC, 128, kk * 16), kmajor_desc(sm + PL::tileH, kPP, kk * 16),
                  id_o, kk > 0 ? 1u : 0u);
    }
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
    // decay mask: P[m, (s,q)] = S * exp(cum_t - cum_s) * (s<t ? gamma_s + (1-lam_{s+1})dt_{s+1} : gamma_s), s <= t
    uint8_t* tP = sm + PL::tileB;
    const float ct = cum2[t];
#pragma unroll
    for (int g2 = 0; g2 < 2; ++g2) {
      const int c0 = 64 * half + 32 * g2;
      float v[32];
      tmem_ld32(trow + c0, v);
#pragma unroll
      for (int j = 0; j < 32; j += RP) {
        const int s = (c0 + j) / RP;
        float w = 0.f;
        if (s <= t) w = exp2f(ct - cum2[s]) * (s < t ? wgt[s] : gam[s]);
#pragma unroll
        for (int q = 0; q < RP; ++q) v[j + q] *= w;
      }
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        float v8[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) v8[e] = v[8 * cc + e];
        tile_store8<TA>(tP, m, c0 / 8 + cc, 128, v8);
      }
    }
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (ok && threadIdx.x == 0) {
    if constexpr (PL::F32) {
      constexpr uint32_t id_o = idesc_tf32(128, kPP, false, false);
#pragma unroll
      for (int kk = 0; kk < 16; ++kk)
        umma_tf32(tbase + 128, kmajor_desc_b(sm + PL::tileB, 128, kk * 32),
                  kmajor_desc_b(sm + PL::tileX, kPP, kk * 32), id_o, kk > 0 ? 1u : 0u);
    } else {
      constexpr uint32_t id_o = idesc_bf16(128, kPP, false, false);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk)
        umma_bf16(tbase + 128, kmajor_desc(sm + PL::tileB, 128, kk * 16), kmajor_desc(sm + PL::tileX, kPP, kk * 16),
                  id_o, kk > 0 ? 1u : 0u);
    }
    umma_commit(&bar[1]);
  }
  if (ok) {
    ok = mbar_wait(&bar[1], 0);
  }
  __syncwarp();
  ok = __syncthreads_and(ok);
  tc_fence_after();
  if (ok) {
    const float* xs = reinterpret_cast<const float*>(sm + PL::xs);
    const float* zs = reinterpret_cast<const float*>(sm + PL::zs);
    const float* mx = reinterpret_cast<const float*>(sm + PL::mx);
    const float* mz = reinterpret_cast<const float*>(sm + PL::mz);
    const float* md = reinterpret_cast<const float*>(sm + PL::md);
    float Y[32], Yi[32];
    tmem_ld32(trow + 128 + 32 * half, Y);
    tmem_ld32(trow + 192 + 32 * half, Yi);
    const float ec = exp2f(cum2[t]);
    const float Dh = ldf(p.D, h, p.param_dtype);
    float acc[32];
    const int64_t tok0 = (int64_t)k * L + t;
    const TA* prow = reinterpret_cast<const TA*>(a.proj) + ((int64_t)b * a.T + (tok0 < a.T ? tok0 : 0)) * a.proj_stride;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int pp = 32 * half + j;
      float xv, zv;
      if constexpr (PL::F32) {  // x and z of this row straight from the projection
        const bool okp = pp < p.P && tok0 < a.T;
        xv = okp ? io<TA>::ld(prow + (int64_t)p.H * p.P + (int64_t)h * p.P + pp) : 0.f;
        zv = okp ? io<TA>::ld(prow + (int64_t)h * p.P + pp) : 0.f;
      } else {
        xv = xs[t * PL::XS + pp];
        zv = zs[t * PL::XS + pp];
      }
      const float xr = xv * mx[pp * RP + r];
      const float zz = zv * mz[pp * RP + r];
      acc[j] = (Y[j] + ec * Yi[j] + Dh * xr) * silu_f(zz) * md[pp * RP + r];
    }
#pragma unroll
    for (int o = 1; o < RP; o <<= 1) {
#pragma unroll
      for (int j = 0; j < 32; ++j) acc[j] += __shfl_xor_sync(0xffffffffu, acc[j], o);
    }
    const int64_t tok = (int64_t)k * L + t;
    if (tok < a.T) {
      constexpr int W = 32 / RP;
      TA* yo = reinterpret_cast<TA*>(a.y) + ((int64_t)b * a.T + tok) * ((int64_t)p.H * p.P) + (int64_t)h * p.P;
#pragma unroll
      for (int rr = 0; rr < RP; ++rr) {
        if (rr != r) continue;
#pragma unroll
        for (int c8 = 0; c8 < W / 8; ++c8) {
          const int p0 = 32 * half + rr * W + c8 * 8;
          if (p0 + 8 <= p.P) {
            float o8[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) o8[e] = acc[rr * W + c8 * 8 + e];
            store8<TA>(yo + p0, o8);
          } else {
#pragma unroll
            for (int e = 0; e < 8; ++e)
              if (p0 + e < p.P) io<TA>::st(yo + p0 + e, acc[rr * W + c8 * 8 + e]);
          }
        }
      }
    }
  } else if (threadIdx.x == 0) {
    record_error(a.err, M3B_ERR_TIMEOUT);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, 256);
  }
}

// ---------------------------------------------------------------------------
// prefill prev_BX = sum_r B^_{T-1}[n,r] x_r[T-1,p,r]  (mamba3/mamba3.py:248-250), fp32.
// ---------------------------------------------------------------------------
template <typename TA>
__global__ void __launch_bounds__(kCT) last_bx_kernel(FwdParams a, const float* angle_last, float* prev_bx,
                                                       float* prev_b, float* prev_x) {
  __shared__ float sB[kNS * 8];
  __shared__ float sX[kPP * 8];
  const m3b_layer_params& p = a.prm;
  const int H = p.H, P = p.P, N = p.N, R = p.R, NR = N * R, pd = p.param_dtype;
  const int b = blockIdx.x / H, h = blockIdx.x % H, g = h / (H / p.G);
  const int64_t t = a.T - 1;
  const TA* row = reinterpret_cast<const TA*>(a.proj) + ((int64_t)b * a.T + t) * a.proj_stride;
  const float rb = a.rms[(((int64_t)b * a.T + t) * p.G + g) * 2];
  for (int e = threadIdx.x; e < NR; e += kCT)
    sB[e] = fmaf(io<TA>::ld(row + 2 * H * P + g * NR + e) * rb, ldf(p.B_norm_w, e, pd),
                 ldf(p.B_bias, (int64_t)g * NR + e, pd));
  for (int e = threadIdx.x; e < P * R; e += kCT)
    sX[e] = io<TA>::ld(row + H * P + h * P + e / R) * ldf(p.mimo_x, (int64_t)h * P * R + e, pd);
  __syncthreads();
  if (p.complex_ssm) {
    const float* ang = angle_last + ((int64_t)b * H + h) * (N / 2);
    for (int i = threadIdx.x; i < N / 2; i += kCT) {
      float sn, cs;
      sincosf(ang[i], &sn, &cs);
      for (int r = 0; r < R; ++r) {
        const float b0 = sB[(2 * i) * R + r], b1 = sB[(2 * i + 1) * R + r];
        sB[(2 * i) * R + r] = b0 * cs - b1 * sn;
        sB[(2 * i + 1) * R + r] = b0 * sn + b1 * cs;
      }
    }
    __syncthreads();
  }
  if (prev_b) {  // compact form: the last token's B^ (N, R) and x_r (P, R)
    const int64_t bh = (int64_t)b * H + h;
    for (int e = threadIdx.x; e < NR; e += kCT) prev_b[bh * NR + e] = sB[e];
    for (int e = threadIdx.x; e < P * R; e += kCT) prev_x[bh * P * R + e] = sX[e];
  }
  if (!prev_bx) return;
  float* out = prev_bx + ((int64_t)b * H + h) * (int64_t)P * N;
  for (int e = threadIdx.x; e < P * N; e += kCT) {
    const int pp = e / N, n = e % N;
    float acc = 0.f;
    for (int r = 0; r < R; ++r) acc = fmaf(sB[n * R + r], sX[pp * R + r], acc);
    out[e] = acc;
  }
}

// ---------------------------------------------------------------------------
// host orchestration
// ---------------------------------------------------------------------------
namespace {

struct WsLayout {
  size_t rms, asum, omega, sstate, hstate, decay, coef0, angle_last, ho_h, ho_ang, ho_flag, total;
  bool fused;
  int kp;  // fused path: chunks per sequence part (K: sequences are not cut)
};

size_t up256(size_t x) { return (x + 255) & ~size_t(255); }

// The fused sequential kernel takes bf16 activations; fp32 activations always run the
// chunk-parallel kernels, whose fp32 operand tiles feed kind::tf32 MMAs (fp32-level accuracy).
bool use_fused(const m3b_layer_fwd_args* a) {
  if (a->algo == 2 || a->act_dtype != M3B_BF16) return false;
  return fused_supported(a->prm);
}

// Chunks per part when the fused kernel cuts sequences into parts: equal-length sequences fill
// ceil(nseq / nsm) rounds of the persistent grid, so e.g. 384 sequences on 148 SMs leave the
// last round 40 % occupied; parts of K / np chunks make nseq * np jobs and fill the rounds
// better; a job start costs about a chunk's time, a part's state hand-off a quarter more.  A part cannot start
// before the previous part of its sequence has finished, so the time of a cut is modelled by
// walking the static job order (job j on CTA j % grid, after the CTA's previous job and after
// job j - nseq); with fewer sequences than SMs the parts of a sequence would only wait on one
// another, and the model keeps whole sequences.  The number of parts np divides K; cutting must
// save at least 1 % of the modelled time.
int choose_kp_uncached(int64_t nseq, int K, int nsm) {
  constexpr double kSwitch = 1.0;    // start of any job (new sequence or part), in chunk times
  constexpr double kHandoff = 0.25;  // extra for a part that loads its predecessor's state
  std::vector<double> cta_free, fin;
  auto cost = [&](int np) {
    const int64_t jobs = nseq * np;
    const int64_t grid = jobs < nsm ? jobs : nsm;
    const double len = (double)(K / np) + kSwitch + (np > 1 ? kHandoff : 0.0);
    cta_free.assign((size_t)grid, 0.0);
    fin.assign((size_t)jobs, 0.0);
    double span = 0.0;
    for (int64_t j = 0; j < jobs; ++j) {
      double start = cta_free[(size_t)(j % grid)];
      if (j >= nseq && fin[(size_t)(j - nseq)] > start) start = fin[(size_t)(j - nseq)];
      fin[(size_t)j] = start + len;
      cta_free[(size_t)(j % grid)] = fin[(size_t)j];
      if (fin[(size_t)j] > span) span = fin[(size_t)j];
    }
    return span;
  };
  const double base = cost(1);
  int best = 1;
  double best_cost = base;
  for (int np = 2; np <= 64 && np <= K; ++np) {
    if (K % np != 0) continue;
    const double c = cost(np);
    if (c < best_cost) {
      best_cost = c;
      best = np;
    }
  }
  return best_cost <= 0.99 * base ? K / best : K;
}

// choose_kp, remembered per (sequences, chunks, SMs): the model walks every job once
int choose_kp(int64_t nseq, int K, int nsm) {
  static std::mutex mu;
  static std::map<std::tuple<int64_t, int, int>, int> memo;
  const auto key = std::make_tuple(nseq, K, nsm);
  {
    std::lock_guard<std::mutex> lk(mu);
    const auto it = memo.find(key);
    if (it != memo.end()) return it->second;
  }
  const int kp = choose_kp_uncached(nseq, K, nsm);
  std::lock_guard<std::mutex> lk(mu);
  memo[key] = kp;
  return kp;
}

WsLayout ws_layout(const m3b_layer_fwd_args* a, int L, bool allow_parts = true) {
  const m3b_layer_params& p = a->prm;
  const int64_t B = a->batch, T = a->seqlen, K = (T + L - 1) / L;
  const size_t ssz = (a->act_dtype == M3B_BF16) ? 2 : 4;
  const bool cx = p.complex_ssm != 0;
  WsLayout w{};
  size_t o = 0;
  w.fused = use_fused(a);
  w.kp = (int)K;
  w.rms = o; o += up256((size_t)B * T * p.G * 2 * 4);
  w.angle_last = o; o += up256((size_t)B * p.H * (p.N / 2) * 4);
  if (w.fused) {
    if (allow_parts) w.kp = choose_kp(B * p.H, (int)K, num_sms());
    if (w.kp < K) {
      const size_t nseq = (size_t)B * p.H;
      w.ho_h = o; o += up256(nseq * p.P * p.N * 4);
      w.ho_ang = o; o += up256(nseq * 64 * 8);
      w.ho_flag = o; o += up256(nseq * 2 * 4);
    }
    w.total = o;
    return w;
  }
  w.asum = o; o += cx ? up256((size_t)B * K * p.H * (p.N / 2) * 4) : 0;
  w.omega = o; o += cx ? up256((size_t)B * (K + 1) * p.H * (p.N / 2) * 4) : 0;
  w.sstate = o; o += up256((size_t)B * K * p.H * p.P * p.N * ssz);
  w.hstate = o; o += up256((size_t)B * K * p.H * p.P * p.N * ssz);
  w.decay = o; o += up256((size_t)B * K * p.H * 4);
  w.coef0 = o; o += up256((size_t)B * p.H * 4);
  w.total = o;
  return w;
}

// Opt a kernel into more than 48 KB of dynamic shared memory, once per (kernel, device).
int ensure_smem(const void* kernel, int bytes) {
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

template <typename TA, typename TS, int R, typename Mark>
int run_chunks(FwdParams& fp, const m3b_layer_fwd_args* a, cudaStream_t st, Mark& mark) {
  constexpr int RP = rp_of(R);
  using PL = Plan<RP, TA>;
  const m3b_layer_params& p = a->prm;
  int rc;
  dim3 grid((unsigned)p.H, (unsigned)fp.K, (unsigned)fp.B);
  mark(2);
  if ((rc = ensure_smem((const void*)chunk_state_kernel<TA, TS, R>, PL::bytes)) != M3B_OK) return rc;
  chunk_state_kernel<TA, TS, R><<<grid, kCT, PL::bytes, st>>>(fp);
  if ((rc = check_launch("chunk_state")) != M3B_OK) return rc;
  ScanLaunch s{fp.decay,
               fp.sstate,
               a->h_init,
               a->prev_bx_init,
               a->prev_bx_init ? fp.coef0 : nullptr,
               fp.hstate,
               a->h_final,
               fp.B,
               fp.K,
               p.H,
               (int64_t)p.P * p.N,
               io<TS>::code};
  mark(3);
  if ((rc = launch_scan(s, st)) != M3B_OK) return rc;
  mark(4);
  if ((rc = ensure_smem((const void*)chunk_out_kernel<TA, TS, R>, PL::bytes)) != M3B_OK) return rc;
  chunk_out_kernel<TA, TS, R><<<grid, kCT, PL::bytes, st>>>(fp);
  return check_launch("chunk_out");
}

template <typename TA, typename TS, typename Mark>
int run_rank(FwdParams& fp, const m3b_layer_fwd_args* a, cudaStream_t st, Mark& mark) {
  switch (a->prm.R) {
    case 1: return run_chunks<TA, TS, 1>(fp, a, st, mark);
    case 2: return run_chunks<TA, TS, 2>(fp, a, st, mark);
    case 3: return run_chunks<TA, TS, 3>(fp, a, st, mark);
    case 4: return run_chunks<TA, TS, 4>(fp, a, st, mark);
    default: return fail(M3B_ERR_UNSUPPORTED, "layer_fwd: mimo_rank %d not built (1..4)", a->prm.R);
  }
}

template <typename TA, typename TS>
int layer_fwd_t(const m3b_layer_fwd_args* a, uint8_t* ws, const WsLayout& w, int L, cudaStream_t st) {
  const m3b_layer_params& p = a->prm;
  FwdParams fp{};
  fp.prm = p;
  fp.proj = a->proj;
  fp.proj_stride = a->proj_stride;
  fp.dt_scale = a->dt_scale;
  fp.B = a->batch;
  fp.T = a->seqlen;
  fp.L = L;
  fp.K = (int)((a->seqlen + L - 1) / L);
  fp.rms = reinterpret_cast<float*>(ws + w.rms);
  fp.asum = reinterpret_cast<float*>(ws + w.asum);
  fp.omega = reinterpret_cast<float*>(ws + w.omega);
  fp.angle_init = a->angle_init;
  fp.angle_final = reinterpret_cast<float*>(ws + w.angle_last);
  fp.sstate = ws + w.sstate;
  fp.hstate = ws + w.hstate;
  fp.decay = reinterpret_cast<float*>(ws + w.decay);
  fp.coef0 = reinterpret_cast<float*>(ws + w.coef0);
  fp.y = a->y;
  fp.err = a->err;
  int rc;
  auto mark = [&](int i) {
    if (a->stage_events) cudaEventRecord(static_cast<cudaEvent_t>(a->stage_events[i]), st);
  };
  float* angle_last = reinterpret_cast<float*>(ws + w.angle_last);
  // the fused path needs only the 1/rms rows from the pre-pass: a caller that has them (the input
  // projection's epilogue, m3b_in_proj) skips it
  const bool rms_given = w.fused && a->rms_in != nullptr;
  if (rms_given) fp.rms = const_cast<float*>(a->rms_in);
  mark(0);
  if (w.fused) fp.asum = nullptr;
  if (!rms_given) {
    prep_kernel<TA><<<dim3((unsigned)fp.K, (unsigned)fp.B), kCT, 0, st>>>(fp);
    if ((rc = check_launch("prep")) != M3B_OK) return rc;
  }
  if (w.fused) {
    mark(1);
    mark(2);
    mark(3);
    mark(4);
    FusedParams f{};
    f.prm = p;
    f.proj = a->proj;
    f.proj_stride = a->proj_stride;
    f.dt_scale = a->dt_scale;
    f.B = fp.B;
    f.T = fp.T;
    f.K = fp.K;
    f.L = fp.L;
    f.rms = fp.rms;
    f.h_init = a->h_init;
    f.angle_init = a->angle_init;
    f.prev_bx_init = a->prev_bx_init;
    f.y = a->y;
    f.h_final = a->h_final;
    f.angle_last = angle_last;
    f.err = a->err;
    f.wait_ns = a->wait_limit_ns > 0 ? (uint64_t)a->wait_limit_ns : kWaitLimitNs;
    f.state_only = a->state_only != 0;
    f.KP = w.kp;
    if (w.kp < fp.K) {
      f.ho_h = reinterpret_cast<float*>(ws + w.ho_h);
      f.ho_ang = reinterpret_cast<double*>(ws + w.ho_ang);
      f.ho_flag = reinterpret_cast<int*>(ws + w.ho_flag);
    }
    if ((rc = launch_fused(f, st, a->act_dtype == M3B_BF16)) != M3B_OK) return rc;
    if (a->angle_final) {
      const cudaError_t e = cudaMemcpyAsync(a->angle_final, angle_last, (size_t)fp.B * p.H * (p.N / 2) * 4,
                                            cudaMemcpyDeviceToDevice, st);
      if (e != cudaSuccess) return fail(M3B_ERR_CUDA, "angle_final: %s", cudaGetErrorString(e));
    }
    mark(5);
    if (a->prev_bx_final || a->prev_b_final) {
      last_bx_kernel<TA><<<(unsigned)(fp.B * p.H), kCT, 0, st>>>(fp, angle_last, a->prev_bx_final, a->prev_b_final,
                                                                 a->prev_x_final);
      if ((rc = check_launch("last_bx")) != M3B_OK) return rc;
    }
    mark(6);
    return M3B_OK;
  }
  mark(1);
  if (p.complex_ssm) {
    angle_prefix_kernel<<<(unsigned)(fp.B * p.H), kCT, 0, st>>>(fp);
    if ((rc = check_launch("angle_prefix")) != M3B_OK) return rc;
    if (a->angle_final) {
      const cudaError_t e = cudaMemcpyAsync(a->angle_final, angle_last, (size_t)fp.B * p.H * (p.N / 2) * 4,
                                            cudaMemcpyDeviceToDevice, st);
      if (e != cudaSuccess) return fail(M3B_ERR_CUDA, "angle_final: %s", cudaGetErrorString(e));
    }
  } else if (a->angle_final) {
    const size_t bytes = (size_t)fp.B * p.H * (p.N / 2) * 4;
    const cudaError_t e = a->angle_init
                              ? cudaMemcpyAsync(a->angle_final, a->angle_init, bytes, cudaMemcpyDeviceToDevice, st)
                              : cudaMemsetAsync(a->angle_final, 0, bytes, st);
    if (e != cudaSuccess) return fail(M3B_ERR_CUDA, "angle_final: %s", cudaGetErrorString(e));
  }
  if ((rc = run_rank<TA, TS>(fp, a, st, mark)) != M3B_OK) return rc;
  mark(5);
  if (a->prev_bx_final || a->prev_b_final) {
    last_bx_kernel<TA><<<(unsigned)(fp.B * p.H), kCT, 0, st>>>(fp, angle_last, a->prev_bx_final, a->prev_b_final,
                                                               a->prev_x_final);
    if ((rc = check_launch("last_bx")) != M3B_OK) return rc;
  }
  mark(6);
  return M3B_OK;
}

int validate(const m3b_layer_fwd_args* a) {
  const m3b_layer_params& p = a->prm;
  if (!a->proj || !a->y) return fail(M3B_ERR_INVALID_ARG, "layer_fwd: null proj/y");
  if (p.H <= 0 || p.P <= 0 || p.N <= 0 || p.R <= 0 || p.G <= 0 || p.H % p.G != 0)
    return fail(M3B_ERR_INVALID_ARG, "layer_fwd: bad dims H=%d P=%d N=%d R=%d G=%d", p.H, p.P, p.N, p.R, p.G);
  if (p.P > kPP || p.P % 8 != 0) return fail(M3B_ERR_UNSUPPORTED, "layer_fwd: headdim %d (need P %% 8 == 0, P <= 64)", p.P);
  if (p.N > kNS || p.N % 8 != 0) return fail(M3B_ERR_UNSUPPORTED, "layer_fwd: d_state %d (need N %% 8 == 0, N <= 128)", p.N);
  if (p.R > 4) return fail(M3B_ERR_UNSUPPORTED, "layer_fwd: mimo_rank %d > 4", p.R);
  if (a->act_dtype != M3B_BF16 && a->act_dtype != M3B_F32)
    return fail(M3B_ERR_UNSUPPORTED, "layer_fwd: act dtype must be bf16 or f32");
  const int esz = a->act_dtype == M3B_BF16 ? 2 : 4;
  if (!aligned16(a->proj) || ((a->proj_stride * esz) & 15) != 0 || !aligned16(a->y))
    return fail(M3B_ERR_ALIGNMENT, "layer_fwd: proj / y need 16-byte aligned rows");
  if ((a->h_init && !aligned16(a->h_init)) || (a->prev_bx_init && !aligned16(a->prev_bx_init)) ||
      (a->h_final && !aligned16(a->h_final)))
    return fail(M3B_ERR_ALIGNMENT, "layer_fwd: state buffers must be 16-byte aligned");
  if (a->batch > 65535) return fail(M3B_ERR_UNSUPPORTED, "layer_fwd: batch > 65535");
  if (a->rms_in && (reinterpret_cast<uintptr_t>(a->rms_in) & 7u) != 0)
    return fail(M3B_ERR_ALIGNMENT, "layer_fwd: rms_in must be 8-byte aligned");
  return M3B_OK;
}

}  // namespace

size_t layer_fwd_workspace(const m3b_layer_fwd_args* a) {
  if (validate(a) != M3B_OK) return 0;
  return ws_layout(a, 128 / rp_of(a->prm.R)).total;
}

size_t layer_fwd_workspace_min(const m3b_layer_fwd_args* a) {
  if (validate(a) != M3B_OK) return 0;
  return ws_layout(a, 128 / rp_of(a->prm.R), false).total;
}

int layer_fwd(const m3b_layer_fwd_args* a, void* ws, size_t ws_bytes, cudaStream_t st) {
  int rc = validate(a);
  if (rc != M3B_OK) return rc;
  if (a->batch <= 0 || a->seqlen <= 0) return M3B_OK;
  const int L = 128 / rp_of(a->prm.R);
  WsLayout w = ws_layout(a, L);
  if (ws_bytes < w.total) w = ws_layout(a, L, false);  // a smaller workspace: whole sequences per CTA
  if (!ws || ws_bytes < w.total) return fail(M3B_ERR_WORKSPACE, "layer_fwd: need %zu workspace bytes", w.total);
  if ((a->seqlen + L - 1) / L > 65535) return fail(M3B_ERR_UNSUPPORTED, "layer_fwd: too many chunks");
  uint8_t* base = static_cast<uint8_t*>(ws);
  if (a->act_dtype == M3B_BF16) return layer_fwd_t<__nv_bfloat16, __nv_bfloat16>(a, base, w, L, st);
  return layer_fwd_t<float, float>(a, base, w, L, st);
}

}  // namespace m3b
