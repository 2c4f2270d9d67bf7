// B / C preparation of the layer (mamba3/mamba3.py:203-232) for the training path, forward and
// backward.  Per token row (b, t), group g, head h (group g = h / (H / G)), pair k (n = 2k, 2k+1)
// and rank r:
//   Bn[g, n, r] = Bf[g, n, r] * rsqrt(mean_{n,r} Bf[g]^2 + eps) * wB[n, r] + bB[g, n, r]   (RMSNorm + bias)
//   phi[t, h, k] = -sum_{t' <= t} dt[t', h] theta[t', k]                                  (rotate)
//   B_g[t, h, 2k, r]   = Bn[g, 2k, r] cos phi - Bn[g, 2k+1, r] sin phi
//   B_g[t, h, 2k+1, r] = Bn[g, 2k, r] sin phi + Bn[g, 2k+1, r] cos phi                    (C alike)
//   B_b[t] = B_g[t - 1], B_b[0] = 0                                                         (shift)
// The torch formulation writes and re-reads (B, T, H, N, R) tensors a dozen times each way (the
// head broadcast, cos / sin, the pair stack, the pad, and their backward with sums over heads
// and over (batch, token)); here the forward is one pass that writes B_g, B_b and C once, and the
// backward one pass over their gradients, plus small passes for the angle's reverse prefix sum
// and the parameter gradients.  fp32 arithmetic; the angle prefix runs over 64-token chunks
// (chunk sums first, then each chunk from its start angle).  Every sum has a fixed order (no
// atomics): results are bitwise reproducible.
#include <type_traits>

#include "common.cuh"
#include "launch.h"

namespace m3b {

namespace {

constexpr int kBcThreads = 256;
constexpr int kBcWarps = kBcThreads / 32;
constexpr int kBcChunk = 64;  // tokens per CTA
constexpr int kBcMaxJ = 8;    // (head, pair) angles per thread: H * N / 2 <= 2048

struct BcParams {
  int64_t B, T, bc_stride, th_stride;
  int H, G, N, R, K, NR, GNR, HK, hpg, nchunks;
  int rotate, shift, dt_dtype;
  float eps;
  const void *Bf, *Cf, *theta, *dt, *wB, *bB, *wC, *bC;
  void *B_g, *B_b, *C;
  const void *dB_g, *dB_b, *dC;
  void *dBf, *dCf, *dtheta, *ddt, *dwB, *dbB, *dwC, *dbC;
  float* S;      // (B, nchunks, HK) chunk sums of dt * theta
  float* D;      // (B, nchunks, HK) chunk sums of dphi
  float* dphi;   // (B, T, HK)
  float* part;   // (B, nchunks, 4, GNR) parameter-gradient partials: wB, bB, wC, bC
};

__device__ __forceinline__ float bc_warp_sum(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

// S[b, c, j] = sum over the tokens of chunk c of dt[t, h] theta[t, k]   (j = h K + k)
template <typename T>
__global__ void __launch_bounds__(kBcThreads) bc_chunk_sums(BcParams p) {
  const int c = blockIdx.x;
  const int64_t b = blockIdx.y;
  const int64_t t0 = (int64_t)c * kBcChunk, t1 = t0 + kBcChunk < p.T ? t0 + kBcChunk : p.T;
  const T* th = static_cast<const T*>(p.theta);
  for (int j = threadIdx.x; j < p.HK; j += kBcThreads) {
    const int h = j / p.K, k = j - h * p.K;
    float s = 0.f;
    for (int64_t t = t0; t < t1; ++t) {
      const int64_t row = b * p.T + t;
      s = fmaf(ldf(p.dt, row * p.H + h, p.dt_dtype), io<T>::ld(th + row * p.th_stride + k), s);
    }
    p.S[(b * p.nchunks + c) * p.HK + j] = s;
  }
}

// the shared part of both passes: the raw rows of token `row` into shared memory and the inverse
// RMS of each group (B groups at inv[0, G), C groups at inv[G, 2G))
template <typename T>
__device__ __forceinline__ void bc_load_rows(const BcParams& p, int64_t row, float* xB, float* xC, float* inv) {
  const T* Bf = static_cast<const T*>(p.Bf) + row * p.bc_stride;
  const T* Cf = static_cast<const T*>(p.Cf) + row * p.bc_stride;
  for (int e = threadIdx.x; e < p.GNR; e += kBcThreads) {
    xB[e] = io<T>::ld(Bf + e);
    xC[e] = io<T>::ld(Cf + e);
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int gi = warp; gi < 2 * p.G; gi += kBcWarps) {
    const float* x = gi < p.G ? xB + gi * p.NR : xC + (gi - p.G) * p.NR;
    float s = 0.f;
    for (int e = lane; e < p.NR; e += 32) s = fmaf(x[e], x[e], s);
    s = bc_warp_sum(s);
    if (lane == 0) inv[gi] = rsqrtf(s / (float)p.NR + p.eps);
  }
  __syncthreads();
}

// parameters into shared memory as floats
template <typename T>
__device__ __forceinline__ void bc_load_params(const BcParams& p, float* wB, float* bB, float* wC, float* bC) {
  for (int e = threadIdx.x; e < p.NR; e += kBcThreads) {
    wB[e] = io<T>::ld(static_cast<const T*>(p.wB) + e);
    wC[e] = io<T>::ld(static_cast<const T*>(p.wC) + e);
  }
  for (int e = threadIdx.x; e < p.GNR; e += kBcThreads) {
    bB[e] = io<T>::ld(static_cast<const T*>(p.bB) + e);
    bC[e] = io<T>::ld(static_cast<const T*>(p.bC) + e);
  }
}

// the angles of this thread's (head, pair) slots at the start of chunk c: -sum of the earlier
// chunks' sums, in chunk order
__device__ __forceinline__ void bc_start_angles(const BcParams& p, int64_t b, int c, float (&phi)[kBcMaxJ]) {
#pragma unroll
  for (int i = 0; i < kBcMaxJ; ++i) {
    const int j = threadIdx.x + i * kBcThreads;
    float s = 0.f;
    if (p.rotate && j < p.HK)
      for (int cc = 0; cc < c; ++cc) s += p.S[(b * p.nchunks + cc) * p.HK + j];
    phi[i] = -s;
  }
}

// 2 RV consecutive outputs of one (head, pair) slot, as one store of 2 RV elements (the slot's
// offset is a multiple of 2 RV elements: aligned for the vector)
template <typename T, int RV>
__device__ __forceinline__ void bc_store_slot(T* dst, const float (&v)[2 * RV]) {
  if constexpr (std::is_same<T, float>::value) {
    if constexpr (RV == 1) {
      *reinterpret_cast<float2*>(dst) = make_float2(v[0], v[1]);
    } else {
#pragma unroll
      for (int q = 0; q < RV / 2; ++q)
        reinterpret_cast<float4*>(dst)[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    }
  } else {
    uint32_t w[RV];
#pragma unroll
    for (int q = 0; q < RV; ++q) {
      if constexpr (std::is_same<T, __nv_bfloat16>::value) {
        __nv_bfloat162 x = __floats2bfloat162_rn(v[2 * q], v[2 * q + 1]);
        w[q] = *reinterpret_cast<uint32_t*>(&x);
      } else {
        __half2 x = __floats2half2_rn(v[2 * q], v[2 * q + 1]);
        w[q] = *reinterpret_cast<uint32_t*>(&x);
      }
    }
    if constexpr (RV == 1) *reinterpret_cast<uint32_t*>(dst) = w[0];
    else if constexpr (RV == 2) *reinterpret_cast<uint2*>(dst) = make_uint2(w[0], w[1]);
    else *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// RV: the rank R at compile time (1, 2, 4: vector stores), or 0 (R at run time, scalar stores)
template <typename T, int RV>
__global__ void __launch_bounds__(kBcThreads) bc_fwd_kernel(BcParams p) {
  extern __shared__ float4 bc_smem4[];
  float* xB = reinterpret_cast<float*>(bc_smem4);
  float* xC = xB + p.GNR;
  float* bB = xC + p.GNR;
  float* bC = bB + p.GNR;
  float* wB = bC + p.GNR;
  float* wC = wB + p.NR;
  float* inv = wC + p.NR;  // 2G
  const int c = blockIdx.x;
  const int64_t b = blockIdx.y;
  const int64_t t0 = (int64_t)c * kBcChunk, t1 = t0 + kBcChunk < p.T ? t0 + kBcChunk : p.T;
  const T* th = static_cast<const T*>(p.theta);
  T* Bg = static_cast<T*>(p.B_g);
  T* Bb = static_cast<T*>(p.B_b);
  T* Co = static_cast<T*>(p.C);
  bc_load_params<T>(p, wB, bB, wC, bC);
  float phi[kBcMaxJ];
  bc_start_angles(p, b, c, phi);
  const int R = p.R, NR = p.NR;
  for (int64_t t = t0; t < t1; ++t) {
    const int64_t row = b * p.T + t;
    bc_load_rows<T>(p, row, xB, xC, inv);
#pragma unroll
    for (int i = 0; i < kBcMaxJ; ++i) {
      const int j = threadIdx.x + i * kBcThreads;
      if (j >= p.HK) break;
      const int h = j / p.K, k = j - h * p.K, g = h / p.hpg;
      float cs = 1.f, sn = 0.f;
      if (p.rotate) {
        phi[i] -= ldf(p.dt, row * p.H + h, p.dt_dtype) * io<T>::ld(th + row * p.th_stride + k);
        sincosf(phi[i], &sn, &cs);
      }
      const int64_t o = (row * p.H + h) * NR;
      const float iB = inv[g], iC = inv[p.G + g];
      if constexpr (RV > 0) {
        float vb[2 * RV], vc[2 * RV];
#pragma unroll
        for (int r = 0; r < RV; ++r) {
          const int e0 = 2 * k * RV + r, e1 = e0 + RV;
          const float a0 = xB[g * NR + e0] * iB * wB[e0] + bB[g * NR + e0];
          const float a1 = xB[g * NR + e1] * iB * wB[e1] + bB[g * NR + e1];
          vb[r] = a0 * cs - a1 * sn;
          vb[RV + r] = a0 * sn + a1 * cs;
          const float q0 = xC[g * NR + e0] * iC * wC[e0] + bC[g * NR + e0];
          const float q1 = xC[g * NR + e1] * iC * wC[e1] + bC[g * NR + e1];
          vc[r] = q0 * cs - q1 * sn;
          vc[RV + r] = q0 * sn + q1 * cs;
        }
        const int64_t so = o + 2 * k * RV;
        bc_store_slot<T, RV>(Bg + so, vb);
        bc_store_slot<T, RV>(Co + so, vc);
        if (p.shift) {
          if (t + 1 < p.T) bc_store_slot<T, RV>(Bb + so + (int64_t)p.H * NR, vb);
          if (t == 0) {
            float zero[2 * RV];
#pragma unroll
            for (int q = 0; q < 2 * RV; ++q) zero[q] = 0.f;
            bc_store_slot<T, RV>(Bb + so, zero);
          }
        }
        continue;
      }
      for (int r = 0; r < R; ++r) {
        const int e0 = 2 * k * R + r, e1 = e0 + R;
        const float a0 = xB[g * NR + e0] * iB * wB[e0] + bB[g * NR + e0];
        const float a1 = xB[g * NR + e1] * iB * wB[e1] + bB[g * NR + e1];
        const float o0 = a0 * cs - a1 * sn, o1 = a0 * sn + a1 * cs;
        io<T>::st(Bg + o + e0, o0);
        io<T>::st(Bg + o + e1, o1);
        if (p.shift) {
          if (t + 1 < p.T) {
            io<T>::st(Bb + o + (int64_t)p.H * NR + e0, o0);
            io<T>::st(Bb + o + (int64_t)p.H * NR + e1, o1);
          }
          if (t == 0) {
            io<T>::st(Bb + o + e0, 0.f);
            io<T>::st(Bb + o + e1, 0.f);
          }
        }
        const float q0 = xC[g * NR + e0] * iC * wC[e0] + bC[g * NR + e0];
        const float q1 = xC[g * NR + e1] * iC * wC[e1] + bC[g * NR + e1];
        io<T>::st(Co + o + e0, q0 * cs - q1 * sn);
        io<T>::st(Co + o + e1, q0 * sn + q1 * cs);
      }
    }
    __syncthreads();  // the rows are read before the next token overwrites them
  }
}

// Backward, one CTA per (chunk, batch row), tokens in order:
//   dB_r[t] = dB_g[t] + dB_b[t + 1]; through the rotation: dphi = sum_r (g1 o0 - g0 o1) over B
//   and C, dBn = R(-phi) dB_r; summed over the heads of each group (in head order); RMSNorm
//   backward: dx = inv (dy w) - x inv^3 / NR * sum(dy w x); dw += dy x inv, dbias += dy.
template <typename T>
__global__ void __launch_bounds__(kBcThreads) bc_bwd_kernel(BcParams p) {
  extern __shared__ float4 bc_smem4[];
  const int GNR = p.GNR, NR = p.NR, R = p.R, HNR = p.H * p.NR;
  float* xB = reinterpret_cast<float*>(bc_smem4);
  float* xC = xB + GNR;
  float* bB = xC + GNR;
  float* bC = bB + GNR;
  float* gwB = bC + GNR;
  float* gwC = gwB + GNR;
  float* acc = gwC + GNR;  // 4 x GNR: dwB, dbB, dwC, dbC partials of this CTA
  float* dpB = acc + 4 * GNR;
  float* dpC = dpB + HNR;
  float* wB = dpC + HNR;
  float* wC = wB + NR;
  float* inv = wC + NR;    // 2G
  float* sred = inv + 2 * p.G;  // 2G: sums of dy w x per group
  const int c = blockIdx.x;
  const int64_t b = blockIdx.y;
  const int64_t t0 = (int64_t)c * kBcChunk, t1 = t0 + kBcChunk < p.T ? t0 + kBcChunk : p.T;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const T* th = static_cast<const T*>(p.theta);
  const T* dBg = static_cast<const T*>(p.dB_g);
  const T* dBb = static_cast<const T*>(p.dB_b);
  const T* dCo = static_cast<const T*>(p.dC);
  bc_load_params<T>(p, wB, bB, wC, bC);
  for (int e = tid; e < 4 * GNR; e += kBcThreads) acc[e] = 0.f;
  float phi[kBcMaxJ], dsum[kBcMaxJ];
  bc_start_angles(p, b, c, phi);
#pragma unroll
  for (int i = 0; i < kBcMaxJ; ++i) dsum[i] = 0.f;
  for (int64_t t = t0; t < t1; ++t) {
    const int64_t row = b * p.T + t;
    bc_load_rows<T>(p, row, xB, xC, inv);
#pragma unroll
    for (int i = 0; i < kBcMaxJ; ++i) {
      const int j = tid + i * kBcThreads;
      if (j >= p.HK) break;
      const int h = j / p.K, k = j - h * p.K, g = h / p.hpg;
      float cs = 1.f, sn = 0.f;
      if (p.rotate) {
        phi[i] -= ldf(p.dt, row * p.H + h, p.dt_dtype) * io<T>::ld(th + row * p.th_stride + k);
        sincosf(phi[i], &sn, &cs);
      }
      const int64_t o = (row * p.H + h) * NR;
      const float iB = inv[g], iC = inv[p.G + g];
      float dph = 0.f;
      for (int r = 0; r < R; ++r) {
        const int e0 = 2 * k * R + r, e1 = e0 + R;
        float g0 = io<T>::ld(dBg + o + e0), g1 = io<T>::ld(dBg + o + e1);
        if (p.shift && t + 1 < p.T) {
          g0 += io<T>::ld(dBb + o + HNR + e0);
          g1 += io<T>::ld(dBb + o + HNR + e1);
        }
        const float a0 = xB[g * NR + e0] * iB * wB[e0] + bB[g * NR + e0];
        const float a1 = xB[g * NR + e1] * iB * wB[e1] + bB[g * NR + e1];
        dph += g1 * (a0 * cs - a1 * sn) - g0 * (a0 * sn + a1 * cs);
        dpB[h * NR + e0] = g0 * cs + g1 * sn;
        dpB[h * NR + e1] = g1 * cs - g0 * sn;
        const float u0 = io<T>::ld(dCo + o + e0), u1 = io<T>::ld(dCo + o + e1);
        const float q0 = xC[g * NR + e0] * iC * wC[e0] + bC[g * NR + e0];
        const float q1 = xC[g * NR + e1] * iC * wC[e1] + bC[g * NR + e1];
        dph += u1 * (q0 * cs - q1 * sn) - u0 * (q0 * sn + q1 * cs);
        dpC[h * NR + e0] = u0 * cs + u1 * sn;
        dpC[h * NR + e1] = u1 * cs - u0 * sn;
      }
      if (p.rotate) {
        p.dphi[row * p.HK + j] = dph;
        dsum[i] += dph;
      }
    }
    __syncthreads();
    // sums over the heads of each group; parameter partials; dy w and its products with x
    for (int e = tid; e < GNR; e += kBcThreads) {
      const int g = e / NR, en = e - g * NR;
      float yb = 0.f, yc = 0.f;
      for (int h = g * p.hpg; h < (g + 1) * p.hpg; ++h) {
        yb += dpB[h * NR + en];
        yc += dpC[h * NR + en];
      }
      acc[e] = fmaf(yb, xB[e] * inv[g], acc[e]);
      acc[GNR + e] += yb;
      acc[2 * GNR + e] = fmaf(yc, xC[e] * inv[p.G + g], acc[2 * GNR + e]);
      acc[3 * GNR + e] += yc;
      gwB[e] = yb * wB[en];
      gwC[e] = yc * wC[en];
    }
    __syncthreads();
    for (int gi = warp; gi < 2 * p.G; gi += kBcWarps) {
      const float* x = gi < p.G ? xB + gi * NR : xC + (gi - p.G) * NR;
      const float* gw = gi < p.G ? gwB + gi * NR : gwC + (gi - p.G) * NR;
      float s = 0.f;
      for (int e = lane; e < NR; e += 32) s = fmaf(gw[e], x[e], s);
      s = bc_warp_sum(s);
      if (lane == 0) sred[gi] = s;
    }
    __syncthreads();
    T* dBf = static_cast<T*>(p.dBf) + row * GNR;
    T* dCf = static_cast<T*>(p.dCf) + row * GNR;
    for (int e = tid; e < GNR; e += kBcThreads) {
      const int g = e / NR;
      const float ib = inv[g], ic = inv[p.G + g];
      io<T>::st(dBf + e, ib * gwB[e] - xB[e] * (ib * ib * ib) * (sred[g] / (float)NR));
      io<T>::st(dCf + e, ic * gwC[e] - xC[e] * (ic * ic * ic) * (sred[p.G + g] / (float)NR));
    }
    __syncthreads();  // rows, dp and gw are rewritten by the next token
  }
  float* part = p.part + (b * p.nchunks + c) * 4 * GNR;
  for (int e = tid; e < 4 * GNR; e += kBcThreads) part[e] = acc[e];
  if (p.rotate) {
#pragma unroll
    for (int i = 0; i < kBcMaxJ; ++i) {
      const int j = tid + i * kBcThreads;
      if (j < p.HK) p.D[(b * p.nchunks + c) * p.HK + j] = dsum[i];
    }
  }
}

// The angle's reverse prefix sum: du[t, j] = -sum_{t' >= t} dphi[t', j] (chunk sums of the later
// chunks first, in chunk order, then this chunk's tokens in reverse), and its two products:
// ddt[t, h] = sum_k du theta[t, k], dtheta[t, k] = sum_h du dt[t, h].
template <typename T>
__global__ void __launch_bounds__(kBcThreads) bc_angle_bwd(BcParams p) {
  extern __shared__ float4 bc_smem4[];
  float* du = reinterpret_cast<float*>(bc_smem4);  // HK
  float* dtv = du + p.HK;                           // H
  float* thv = dtv + p.H;                           // K
  const int c = blockIdx.x;
  const int64_t b = blockIdx.y;
  const int64_t t0 = (int64_t)c * kBcChunk, t1 = t0 + kBcChunk < p.T ? t0 + kBcChunk : p.T;
  const int tid = threadIdx.x;
  const T* th = static_cast<const T*>(p.theta);
  float a[kBcMaxJ];
#pragma unroll
  for (int i = 0; i < kBcMaxJ; ++i) {
    const int j = tid + i * kBcThreads;
    float s = 0.f;
    if (j < p.HK)
      for (int cc = p.nchunks - 1; cc > c; --cc) s += p.D[(b * p.nchunks + cc) * p.HK + j];
    a[i] = s;
  }
  for (int64_t t = t1 - 1; t >= t0; --t) {
    const int64_t row = b * p.T + t;
#pragma unroll
    for (int i = 0; i < kBcMaxJ; ++i) {
      const int j = tid + i * kBcThreads;
      if (j < p.HK) {
        a[i] += p.dphi[row * p.HK + j];
        du[j] = -a[i];
      }
    }
    for (int h = tid; h < p.H; h += kBcThreads) dtv[h] = ldf(p.dt, row * p.H + h, p.dt_dtype);
    for (int k = tid; k < p.K; k += kBcThreads) thv[k] = io<T>::ld(th + row * p.th_stride + k);
    __syncthreads();
    for (int h = tid; h < p.H; h += kBcThreads) {
      float s = 0.f;
      for (int k = 0; k < p.K; ++k) s = fmaf(du[h * p.K + k], thv[k], s);
      stf(p.ddt, row * p.H + h, p.dt_dtype, s);
    }
    for (int k = tid; k < p.K; k += kBcThreads) {
      float s = 0.f;
      for (int h = 0; h < p.H; ++h) s = fmaf(du[h * p.K + k], dtv[h], s);
      io<T>::st(static_cast<T*>(p.dtheta) + row * p.K + k, s);
    }
    __syncthreads();
  }
}

// parameter gradients: the CTA partials summed over (batch row, chunk), the weights also over
// the groups.  A CTA takes 32 elements; its 8 warps sum the partials q = warp (mod 8), each in
// q order, and the 8 warp sums are added in warp order: a fixed order for every launch.
constexpr int kBcSumSegs = kBcWarps;
template <typename T>
__global__ void __launch_bounds__(kBcThreads) bc_param_sums(BcParams p) {
  __shared__ float red[kBcSumSegs][4][32];
  const int lane = threadIdx.x & 31, seg = threadIdx.x >> 5;
  const int e = blockIdx.x * 32 + lane;
  const int64_t nparts = p.B * p.nchunks;
  float sbB = 0.f, sbC = 0.f, swB = 0.f, swC = 0.f;
  if (e < p.GNR) {
    for (int64_t q = seg; q < nparts; q += kBcSumSegs) {
      const float* pq = p.part + q * 4 * p.GNR;
      sbB += pq[p.GNR + e];
      sbC += pq[3 * p.GNR + e];
      if (e < p.NR)
        for (int g = 0; g < p.G; ++g) {
          swB += pq[g * p.NR + e];
          swC += pq[2 * p.GNR + g * p.NR + e];
        }
    }
  }
  red[seg][0][lane] = sbB;
  red[seg][1][lane] = sbC;
  red[seg][2][lane] = swB;
  red[seg][3][lane] = swC;
  __syncthreads();
  if (seg != 0 || e >= p.GNR) return;
  float s[4] = {0.f, 0.f, 0.f, 0.f};
  for (int w = 0; w < kBcSumSegs; ++w)
#pragma unroll
    for (int k = 0; k < 4; ++k) s[k] += red[w][k][lane];
  io<T>::st(static_cast<T*>(p.dbB) + e, s[0]);
  io<T>::st(static_cast<T*>(p.dbC) + e, s[1]);
  if (e < p.NR) {
    io<T>::st(static_cast<T*>(p.dwB) + e, s[2]);
    io<T>::st(static_cast<T*>(p.dwC) + e, s[3]);
  }
}

size_t fwd_smem(const BcParams& p) { return ((size_t)4 * p.GNR + 2 * p.NR + 2 * p.G) * sizeof(float); }
size_t bwd_smem(const BcParams& p) {
  return ((size_t)10 * p.GNR + 2 * (size_t)p.H * p.NR + 2 * p.NR + 4 * p.G) * sizeof(float);
}

struct BcLayout {
  size_t S, D, dphi, part, total;
};

BcLayout bc_layout(const m3b_bc_args* a, bool bwd) {
  auto up = [](size_t x) { return (x + 255) & ~(size_t)255; };
  const size_t nch = (size_t)((a->seqlen + kBcChunk - 1) / kBcChunk);
  const size_t hk = (size_t)a->H * (a->N / 2);
  const size_t gnr = (size_t)a->G * a->N * a->R;
  BcLayout w{};
  w.S = 0;
  size_t off = a->rotate ? up((size_t)a->batch * nch * hk * sizeof(float)) : 0;
  if (bwd) {
    w.D = off;
    off += a->rotate ? up((size_t)a->batch * nch * hk * sizeof(float)) : 0;
    w.dphi = off;
    off += a->rotate ? up((size_t)a->batch * a->seqlen * hk * sizeof(float)) : 0;
    w.part = off;
    off += up((size_t)a->batch * nch * 4 * gnr * sizeof(float));
  }
  w.total = off;
  return w;
}

int bc_validate(const m3b_bc_args* a, bool bwd) {
  if (!a) return fail(M3B_ERR_INVALID_ARG, "bc_prep: null args");
  if (a->batch < 0 || a->seqlen < 0 || a->H <= 0 || a->G <= 0 || a->N <= 0 || a->R <= 0 || a->H % a->G != 0)
    return fail(M3B_ERR_INVALID_ARG, "bc_prep: bad dims");
  if (a->N % 2 != 0) return fail(M3B_ERR_INVALID_ARG, "bc_prep: N must be even");
  if ((int64_t)a->H * (a->N / 2) > (int64_t)kBcMaxJ * kBcThreads)
    return fail(M3B_ERR_UNSUPPORTED, "bc_prep: H * N / 2 above %d", kBcMaxJ * kBcThreads);
  if (a->dtype != M3B_F32 && a->dtype != M3B_BF16 && a->dtype != M3B_F16)
    return fail(M3B_ERR_UNSUPPORTED, "bc_prep: dtype");
  if (a->dt_dtype != M3B_F32 && a->dt_dtype != M3B_BF16 && a->dt_dtype != M3B_F16)
    return fail(M3B_ERR_UNSUPPORTED, "bc_prep: dt dtype");
  const int64_t gnr = (int64_t)a->G * a->N * a->R;
  if ((a->bc_stride != 0 && a->bc_stride < gnr) || (a->theta_stride != 0 && a->theta_stride < a->N / 2))
    return fail(M3B_ERR_INVALID_ARG, "bc_prep: row stride below the row width");
  if ((a->seqlen + kBcChunk - 1) / kBcChunk > 65535 * 1024LL || a->batch > 65535)
    return fail(M3B_ERR_UNSUPPORTED, "bc_prep: too many tokens");
  if (!a->wB || !a->bB || !a->wC || !a->bC) return fail(M3B_ERR_INVALID_ARG, "bc_prep: null parameter");
  if (bwd && (!a->dwB || !a->dbB || !a->dwC || !a->dbC))
    return fail(M3B_ERR_INVALID_ARG, "bc_prep: null parameter gradient");
  if (a->batch * a->seqlen > 0) {
    if (!a->Bf || !a->Cf || (a->rotate && (!a->theta || !a->dt)))
      return fail(M3B_ERR_INVALID_ARG, "bc_prep: null input");
    if (!bwd && (!a->B_g || !a->C || (a->shift && !a->B_b))) return fail(M3B_ERR_INVALID_ARG, "bc_prep: null output");
    if (bwd && (!a->dB_g || !a->dC || (a->shift && !a->dB_b) || !a->dBf || !a->dCf ||
                (a->rotate && (!a->dtheta || !a->ddt))))
      return fail(M3B_ERR_INVALID_ARG, "bc_prep: null gradient");
  }
  return M3B_OK;
}

BcParams bc_params(const m3b_bc_args* a, void* ws, bool bwd) {
  BcParams p{};
  p.B = a->batch;
  p.T = a->seqlen;
  p.H = a->H;
  p.G = a->G;
  p.N = a->N;
  p.R = a->R;
  p.K = a->N / 2;
  p.NR = a->N * a->R;
  p.GNR = a->G * p.NR;
  p.HK = a->H * p.K;
  p.hpg = a->H / a->G;
  p.bc_stride = a->bc_stride ? a->bc_stride : p.GNR;
  p.th_stride = a->theta_stride ? a->theta_stride : p.K;
  p.nchunks = (int)((a->seqlen + kBcChunk - 1) / kBcChunk);
  p.rotate = a->rotate != 0;
  p.shift = a->shift != 0;
  p.dt_dtype = a->dt_dtype;
  p.eps = a->eps;
  p.Bf = a->Bf;
  p.Cf = a->Cf;
  p.theta = a->theta;
  p.dt = a->dt;
  p.wB = a->wB;
  p.bB = a->bB;
  p.wC = a->wC;
  p.bC = a->bC;
  p.B_g = a->B_g;
  p.B_b = a->B_b;
  p.C = a->C;
  p.dB_g = a->dB_g;
  p.dB_b = a->dB_b;
  p.dC = a->dC;
  p.dBf = a->dBf;
  p.dCf = a->dCf;
  p.dtheta = a->dtheta;
  p.ddt = a->ddt;
  p.dwB = a->dwB;
  p.dbB = a->dbB;
  p.dwC = a->dwC;
  p.dbC = a->dbC;
  const BcLayout w = bc_layout(a, bwd);
  uint8_t* base = static_cast<uint8_t*>(ws);
  p.S = reinterpret_cast<float*>(base + w.S);
  if (bwd) {
    p.D = reinterpret_cast<float*>(base + w.D);
    p.dphi = reinterpret_cast<float*>(base + w.dphi);
    p.part = reinterpret_cast<float*>(base + w.part);
  }
  return p;
}

template <typename T>
int bc_run_t(const BcParams& p, bool bwd, cudaStream_t st) {
  const dim3 grid((unsigned)p.nchunks, (unsigned)p.B);
  int rc;
  if (p.rotate) {
    bc_chunk_sums<T><<<grid, kBcThreads, 0, st>>>(p);
    if ((rc = check_launch("bc_chunk_sums")) != M3B_OK) return rc;
  }
  if (!bwd) {
    const size_t smem = fwd_smem(p);
    auto launch = [&](auto kern) {
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      kern<<<grid, kBcThreads, smem, st>>>(p);
    };
    // vector stores need 16-byte aligned output buffers (each slot is then aligned as well)
    const bool al = aligned16(p.B_g) && aligned16(p.C) && (!p.shift || aligned16(p.B_b));
    switch (al ? p.R : 0) {
      case 1: launch(bc_fwd_kernel<T, 1>); break;
      case 2: launch(bc_fwd_kernel<T, 2>); break;
      case 4: launch(bc_fwd_kernel<T, 4>); break;
      default: launch(bc_fwd_kernel<T, 0>); break;
    }
    return check_launch("bc_fwd");
  }
  const size_t smem = bwd_smem(p);
  cudaFuncSetAttribute(bc_bwd_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  bc_bwd_kernel<T><<<grid, kBcThreads, smem, st>>>(p);
  if ((rc = check_launch("bc_bwd")) != M3B_OK) return rc;
  if (p.rotate) {
    const size_t s2 = ((size_t)p.HK + p.H + p.K) * sizeof(float);
    bc_angle_bwd<T><<<grid, kBcThreads, s2, st>>>(p);
    if ((rc = check_launch("bc_angle_bwd")) != M3B_OK) return rc;
  }
  bc_param_sums<T><<<(unsigned)((p.GNR + 31) / 32), kBcThreads, 0, st>>>(p);
  return check_launch("bc_param_sums");
}

int bc_run(const m3b_bc_args* a, bool bwd, void* ws, size_t ws_bytes, cudaStream_t st) {
  int rc = bc_validate(a, bwd);
  if (rc != M3B_OK) return rc;
  const BcLayout w = bc_layout(a, bwd);
  if (a->batch * a->seqlen == 0) {
    if (!bwd) return M3B_OK;
    // no tokens: zero parameter gradients
    const size_t es = a->dtype == M3B_F32 ? 4 : 2;
    const size_t nr = (size_t)a->N * a->R, gnr = nr * a->G;
    if (cudaMemsetAsync(a->dwB, 0, nr * es, st) != cudaSuccess || cudaMemsetAsync(a->dwC, 0, nr * es, st) != cudaSuccess ||
        cudaMemsetAsync(a->dbB, 0, gnr * es, st) != cudaSuccess || cudaMemsetAsync(a->dbC, 0, gnr * es, st) != cudaSuccess)
      return fail(M3B_ERR_CUDA, "bc_prep: memset");
    return M3B_OK;
  }
  if (w.total > 0 && (!ws || ws_bytes < w.total))
    return fail(M3B_ERR_WORKSPACE, "bc_prep: need %zu workspace bytes", w.total);
  const BcParams p = bc_params(a, ws, bwd);
  const size_t smem = bwd ? bwd_smem(p) : fwd_smem(p);
  if (smem > 200 * 1024) return fail(M3B_ERR_UNSUPPORTED, "bc_prep: rows too wide for shared memory");
  switch (a->dtype) {
    case M3B_F32: return bc_run_t<float>(p, bwd, st);
    case M3B_BF16: return bc_run_t<__nv_bfloat16>(p, bwd, st);
    default: return bc_run_t<__half>(p, bwd, st);
  }
}

}  // namespace

}  // namespace m3b

extern "C" size_t m3b_bc_fwd_workspace(const m3b_bc_args* a) {
  if (m3b::bc_validate(a, false) != M3B_OK) return 0;
  return m3b::bc_layout(a, false).total;
}

extern "C" size_t m3b_bc_bwd_workspace(const m3b_bc_args* a) {
  if (m3b::bc_validate(a, true) != M3B_OK) return 0;
  return m3b::bc_layout(a, true).total;
}

extern "C" int m3b_bc_fwd(const m3b_bc_args* a, void* workspace, size_t workspace_bytes, void* stream) {
  m3b::clear_error();
  return m3b::bc_run(a, false, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

extern "C" int m3b_bc_bwd(const m3b_bc_args* a, void* workspace, size_t workspace_bytes, void* stream) {
  m3b::clear_error();
  return m3b::bc_run(a, true, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}
