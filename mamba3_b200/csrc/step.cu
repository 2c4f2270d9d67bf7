// O(1) decode step: the SSM core of KulaMamba.step (mamba3/mamba3.py:278-316).
//
// One CTA per (batch, head).  The CTA first builds, in shared memory, the
// token's per-head operands: dt / decay / trapezoid weights, the B and C rows
// after joint N*R RMSNorm + bias (mamba3/mamba3.py:174-177), rotated by the
// advanced angle (mamba3/mamba3.py:182-188), the MIMO-expanded x and the gate
// silu(z * mimo_z) * mimo_down.  It then streams the (P, N) fp32 state once:
// each thread reads 16-byte vectors of h and prev_BX, forms
//   BX  = sum_r B^[n,r] x_r[p,r]                      (mamba3/mamba3.py:298)
//   h'  = dA h + gamma BX + beta prev_BX              (mamba3/mamba3.py:304-306)
//   y_r += C^[n,r] h'                                 (mamba3/mamba3.py:309)
// writes h' and BX back (16-byte vectors), and reduces y_r over n with warp
// shuffles.  The epilogue adds D x_r, applies the gate and sums the ranks
// (mamba3/mamba3.py:310-316).  State traffic is the minimum of the reference
// layout: read h + prev_BX, write h + BX.
#include "common.cuh"
#include "launch.h"

namespace m3b {

constexpr int kStepThreads = 256;
constexpr int kStepMaxN = 256;
constexpr int kStepMaxP = 256;

// ROW32: N = 128, so the 32 float4 of one state row are the 32 lanes of one warp (R a power of
// two, so that the readout's reduce-scatter halves evenly).
// COMPACT: the previous token is kept as its rotated B^ (N, R) and MIMO x (P, R) instead of the
// (P, N) product prev_BX, which the state loop rebuilds on the fly: half the state traffic.
template <typename TA, int R, bool ROW32, bool COMPACT>
__global__ void __launch_bounds__(kStepThreads, COMPACT ? 4 : 2) step_kernel(m3b_step_args a) {
  const m3b_layer_params& prm = a.prm;
  const int H = prm.H, P = prm.P, N = prm.N, G = prm.G;
  const int b = blockIdx.x / H;
  const int h = blockIdx.x - b * H;
  const int g = h / (H / G);
  const int tid = threadIdx.x;
  const int NR = N * R;
  const int pd = prm.param_dtype;

  // B^ / C^ rank-major ([r][n]) so the state loop reads 4 consecutive n as one float4
  __shared__ __align__(16) float sB[kStepMaxN * R];
  __shared__ __align__(16) float sC[kStepMaxN * R];
  __shared__ float sXr[kStepMaxP * R];
  __shared__ float sGate[kStepMaxP * R];
  __shared__ float sY[kStepMaxP * R];
  __shared__ float sRed[2][kStepThreads / 32];
  __shared__ float sScal[4];  // dA, gamma, beta, dt
  // COMPACT: previous token's B^ (rank-major) and x_r
  __shared__ __align__(16) float sPB[COMPACT ? kStepMaxN * R : 4];
  __shared__ float sPX[COMPACT ? kStepMaxP * R : 4];

  // The first batch of the (P, N) state is requested before anything else: its HBM latency
  // then overlaps the per-token operand preparation below.
  const int64_t sbase = ((int64_t)b * H + h) * (int64_t)P * N;
  const float4* h4 = reinterpret_cast<const float4*>(a.h + sbase);
  const float4* p4 = COMPACT ? nullptr : reinterpret_cast<const float4*>(a.prev_bx + sbase);
  const int nvec = P * N / 4;
  constexpr int BATCH = 8;
  float4 hv[BATCH], pv[COMPACT ? 1 : BATCH];
  auto load_batch = [&](int f0) {
#pragma unroll
    for (int u = 0; u < BATCH; ++u) {
      const int f = f0 + u * kStepThreads + tid;
      if (f < nvec) {
        hv[u] = __ldcs(h4 + f);
        if constexpr (!COMPACT) pv[u] = __ldcs(p4 + f);
      }
    }
  };
  load_batch(0);
  if constexpr (COMPACT) {
    const int64_t bh = (int64_t)b * H + h;
    for (int e = tid; e < N * R; e += kStepThreads) {  // (n, r), r fastest
      const int n = e / R, r = e - (e / R) * R;
      sPB[r * N + n] = a.prev_b[bh * N * R + e];
    }
    for (int e = tid; e < P * R; e += kStepThreads) sPX[e] = a.prev_x[bh * P * R + e];
  }

  const TA* row = reinterpret_cast<const TA*>(a.proj) + (int64_t)b * a.proj_stride;
  const int HP = H * P;
  const int offB = 2 * HP + g * NR;
  const int offC = 2 * HP + G * NR + g * NR;
  const int offDt = 2 * HP + 2 * G * NR;
  const int offLam = offDt + H;
  const int offTh = offLam + (prm.trapezoidal ? H : 0);

  // --- every global load of the prologue, issued together (one round trip): the raw B / C
  // entries of this thread with their norm weights and biases, the angle pair and theta, x and
  // z of channel p = tid with the MIMO weights, the head's scalars
  constexpr int EPT = R;  // B / C entries per thread (N * R <= 256 * R)
  float bv[EPT], cv[EPT], wb[EPT], wc[EPT], bbv[EPT], bcv[EPT];
#pragma unroll
  for (int k = 0; k < EPT; ++k) {
    const int e = tid + k * kStepThreads;
    bv[k] = cv[k] = wb[k] = wc[k] = bbv[k] = bcv[k] = 0.f;
    if (e < NR) {
      bv[k] = io<TA>::ld(row + offB + e);
      cv[k] = io<TA>::ld(row + offC + e);
      wb[k] = ldf(prm.B_norm_w, e, pd);
      wc[k] = ldf(prm.C_norm_w, e, pd);
      bbv[k] = ldf(prm.B_bias, (int64_t)g * NR + e, pd);
      bcv[k] = ldf(prm.C_bias, (int64_t)g * NR + e, pd);
    }
  }
  const int64_t abase = ((int64_t)b * H + h) * (N / 2);
  float ang = 0.f, th = 0.f;
  if (tid < N / 2) {
    ang = ldf(a.angle, abase + tid, a.angle_dtype);
    if (prm.complex_ssm) th = io<TA>::ld(row + offTh + tid);
  }
  float xv = 0.f, zv = 0.f, mxv[R], mzv[R], mdv[R];
#pragma unroll
  for (int r = 0; r < R; ++r) mxv[r] = mzv[r] = mdv[r] = 0.f;
  if (tid < P) {
    xv = io<TA>::ld(row + HP + h * P + tid);
    zv = io<TA>::ld(row + h * P + tid);
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int64_t q = ((int64_t)h * P + tid) * R + r;
      mxv[r] = ldf(prm.mimo_x, q, pd);
      mzv[r] = ldf(prm.mimo_z, q, pd);
      mdv[r] = ldf(prm.mimo_down, q, pd);
    }
  }
  float dt_raw = 0.f, lam_raw = 0.f, dtb = 0.f, alog = 0.f, dts = 1.f;
  if (tid == 0) {
    dt_raw = io<TA>::ld(row + offDt + h);
    if (prm.trapezoidal) lam_raw = io<TA>::ld(row + offLam + h);
    dtb = ldf(prm.dt_bias, h, pd);
    alog = ldf(prm.A_log, h, pd);
    if (a.dt_scale) dts = io<TA>::ld(reinterpret_cast<const TA*>(a.dt_scale) + (int64_t)b * H + h);
  }
  const float Dh = ldf(prm.D, h, pd);

  // --- sums of squares of the raw B / C rows (joint N*R RMSNorm), the head's scalars
  float sb = 0.f, sc = 0.f;
#pragma unroll
  for (int k = 0; k < EPT; ++k) {
    sb = fmaf(bv[k], bv[k], sb);
    sc = fmaf(cv[k], cv[k], sc);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    sb += __shfl_xor_sync(0xffffffffu, sb, o);
    sc += __shfl_xor_sync(0xffffffffu, sc, o);
  }
  if ((tid & 31) == 0) {
    sRed[0][tid >> 5] = sb;
    sRed[1][tid >> 5] = sc;
  }
  if (tid == 0) {
    const float dt = softplus_f(dt_raw + dtb) * dts;
    const float A = -expf(alog);
    const float dA = expf(A * dt);
    float gamma = dt, beta = 0.f;
    if (prm.trapezoidal) {
      const float lam = sigmoid_f(lam_raw);
      gamma = lam * dt;
      beta = (1.f - lam) * dt * dA;
    }
    sScal[0] = dA;
    sScal[1] = gamma;
    sScal[2] = beta;
    sScal[3] = dt;
  }
  // MIMO-expanded x and the gate of channel p = tid
  if (tid < P) {
#pragma unroll
    for (int r = 0; r < R; ++r) {
      sXr[tid * R + r] = xv * mxv[r];
      sGate[tid * R + r] = silu_f(zv * mzv[r]) * mdv[r];
      sY[tid * R + r] = 0.f;
    }
  }
  __syncthreads();
  float tb = 0.f, tc = 0.f;
#pragma unroll
  for (int w = 0; w < kStepThreads / 32; ++w) {
    tb += sRed[0][w];
    tc += sRed[1][w];
  }
  const float rb = rsqrtf(tb / (float)NR + prm.norm_eps);
  const float rc = rsqrtf(tc / (float)NR + prm.norm_eps);
#pragma unroll
  for (int k = 0; k < EPT; ++k) {
    const int e = tid + k * kStepThreads;
    if (e < NR) {
      const int n = e / R, r = e - (e / R) * R;  // proj holds (n, r) with r fastest
      sB[r * N + n] = fmaf(bv[k] * rb, wb[k], bbv[k]);
      sC[r * N + n] = fmaf(cv[k] * rc, wc[k], bcv[k]);
    }
  }
  __syncthreads();
  const float dt = sScal[3];
  // --- RoPE advance and rotation of the (2i, 2i+1) pairs; pair i belongs to thread i
  if (tid < N / 2) {
    const int i = tid;
    if (prm.complex_ssm) {
      ang -= dt * th;
      float s, c;
      sincosf(ang, &s, &c);
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const float b0 = sB[r * N + 2 * i], b1 = sB[r * N + 2 * i + 1];
        sB[r * N + 2 * i] = b0 * c - b1 * s;
        sB[r * N + 2 * i + 1] = b0 * s + b1 * c;
        const float c0 = sC[r * N + 2 * i], c1 = sC[r * N + 2 * i + 1];
        sC[r * N + 2 * i] = c0 * c - c1 * s;
        sC[r * N + 2 * i + 1] = c0 * s + c1 * c;
      }
    }
    a.angle_out[abase + i] = ang;
  }
  __syncthreads();

  // --- stream the state: float4 f covers (p, n0..n0+3)
  const float dA = sScal[0], gamma = sScal[1], beta = sScal[2];
  float4* ho4 = reinterpret_cast<float4*>(a.h_out + sbase);
  float4* bo4 = COMPACT ? nullptr : reinterpret_cast<float4*>(a.bx_out + sbase);
  const int gsz = N / 4;                                     // lanes per state row
  const bool pow2 = (gsz & (gsz - 1)) == 0;
  const int lane = tid & 31, wid = tid >> 5;
  for (int f0 = 0; f0 < nvec; f0 += kStepThreads * BATCH) {
    if (f0 > 0) load_batch(f0);
    float part[BATCH][R];  // ROW32: this lane's partial y of row p_u, rank r
#pragma unroll
    for (int u = 0; u < BATCH; ++u) {
      const int f = f0 + u * kStepThreads + tid;
      const bool ok = f < nvec;
      const int p = ROW32 ? (f >> 5) : (ok ? (4 * f) / N : 0);
      const int n0 = ROW32 ? 4 * lane : (ok ? (4 * f) - p * N : 0);
      float yr[R];
#pragma unroll
      for (int r = 0; r < R; ++r) yr[r] = 0.f;
      if (ok) {
        const float hin[4] = {hv[u].x, hv[u].y, hv[u].z, hv[u].w};
        float pin[4];
        if constexpr (COMPACT) {  // prev_BX[p, n] = sum_r prev_B[n, r] prev_x[p, r]
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) pin[jj] = 0.f;
#pragma unroll
          for (int r = 0; r < R; ++r) {
            const float4 q4 = *reinterpret_cast<const float4*>(sPB + r * N + n0);
            const float px = sPX[p * R + r];
            pin[0] = fmaf(q4.x, px, pin[0]);
            pin[1] = fmaf(q4.y, px, pin[1]);
            pin[2] = fmaf(q4.z, px, pin[2]);
            pin[3] = fmaf(q4.w, px, pin[3]);
          }
        } else {
          pin[0] = pv[u].x, pin[1] = pv[u].y, pin[2] = pv[u].z, pin[3] = pv[u].w;
        }
        float hn[4], bx[4];
        float bq[R][4], cq[R][4], xq[R];
#pragma unroll
        for (int r = 0; r < R; ++r) {
          const float4 b4 = *reinterpret_cast<const float4*>(sB + r * N + n0);
          const float4 c4 = *reinterpret_cast<const float4*>(sC + r * N + n0);
          bq[r][0] = b4.x, bq[r][1] = b4.y, bq[r][2] = b4.z, bq[r][3] = b4.w;
          cq[r][0] = c4.x, cq[r][1] = c4.y, cq[r][2] = c4.z, cq[r][3] = c4.w;
          xq[r] = sXr[p * R + r];
        }
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          float cur = 0.f;
#pragma unroll
          for (int r = 0; r < R; ++r) cur = fmaf(bq[r][jj], xq[r], cur);
          bx[jj] = cur;
          hn[jj] = fmaf(dA, hin[jj], fmaf(gamma, cur, beta * pin[jj]));
#pragma unroll
          for (int r = 0; r < R; ++r) yr[r] = fmaf(cq[r][jj], hn[jj], yr[r]);
        }
        __stcs(ho4 + f, make_float4(hn[0], hn[1], hn[2], hn[3]));
        if constexpr (!COMPACT) __stcs(bo4 + f, make_float4(bx[0], bx[1], bx[2], bx[3]));
      }
      if constexpr (ROW32) {
#pragma unroll
        for (int r = 0; r < R; ++r) part[u][r] = yr[r];
        continue;
      }
      // reduce over the lanes that share row p (N/4 consecutive lanes when N/4 is a power of 2)
      if (pow2) {
        const int lim = gsz < 32 ? gsz : 32;
        for (int o = 1; o < lim; o <<= 1) {
#pragma unroll
          for (int r = 0; r < R; ++r) yr[r] += __shfl_xor_sync(0xffffffffu, yr[r], o);
        }
        if (ok && ((tid & 31) % lim) == 0) {
#pragma unroll
          for (int r = 0; r < R; ++r) atomicAdd(&sY[p * R + r], yr[r]);
        }
      } else if (ok) {
#pragma unroll
        for (int r = 0; r < R; ++r) atomicAdd(&sY[p * R + r], yr[r]);
      }
    }
    if constexpr (ROW32) {
      // Every lane of a warp covers row p_u = f0/32 + 8u + warp: one warp-wide reduce-scatter of
      // the BATCH*R partials.  Each halving step keeps the lower or upper half by one lane bit;
      // once a single value is left the remaining steps add it across the other bits.
      constexpr int NV = BATCH * R;
      float v[NV];
#pragma unroll
      for (int u = 0; u < BATCH; ++u)
#pragma unroll
        for (int r = 0; r < R; ++r) v[u * R + r] = part[u][r];
      int idx = 0;
#pragma unroll
      for (int s = 0; s < 5; ++s) {
        const int mask = 16 >> s;
        const int cnt = NV >> s;
        const bool upper = (lane & mask) != 0;
        if (cnt >= 2) {
          const int half = cnt / 2;
#pragma unroll
          for (int i = 0; i < half; ++i) {
            const float send = upper ? v[i] : v[i + half];
            const float keep = upper ? v[i + half] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, mask);
          }
          if (upper) idx += half;
        } else {
          v[0] += __shfl_xor_sync(0xffffffffu, v[0], mask);
        }
      }
      // lanes that differ only in the bits of the plain-add steps hold the same total
      constexpr int dup = NV >= 32 ? 1 : 32 / NV;
      const int u = idx / R, r = idx - (idx / R) * R;
      const int fw = f0 + u * kStepThreads + wid * 32;  // first float4 of this warp at batch u
      if ((lane & (dup - 1)) == 0 && fw < nvec) sY[(fw >> 5) * R + r] = v[0];
    }
  }
  __syncthreads();
  if constexpr (COMPACT) {  // this token's B^ and x_r are the next step's previous token
    const int64_t bh = (int64_t)b * H + h;
    for (int e = tid; e < N * R; e += kStepThreads) {
      const int n = e / R, r = e - (e / R) * R;
      a.prev_b_out[bh * N * R + e] = sB[r * N + n];
    }
    for (int e = tid; e < P * R; e += kStepThreads) a.prev_x_out[bh * P * R + e] = sXr[e];
  }
  // --- readout + D, gate, MIMO down
  TA* yo = reinterpret_cast<TA*>(a.y) + (int64_t)b * HP + (int64_t)h * P;
  for (int p = tid; p < P; p += kStepThreads) {
    float acc = 0.f;
#pragma unroll
    for (int r = 0; r < R; ++r) acc = fmaf(sY[p * R + r] + Dh * sXr[p * R + r], sGate[p * R + r], acc);
    io<TA>::st(yo + p, acc);
  }
}

template <typename TA>
static int launch_step_t(const m3b_step_args* a, cudaStream_t st) {
  const unsigned grid = (unsigned)(a->batch * a->prm.H);
  const bool row32 = a->prm.N == 128;
  const bool compact = a->prev_b != nullptr;
#define M3B_STEP_ROW(RR, CP)                                                                            \
  if (row32 && (RR & (RR - 1)) == 0) step_kernel<TA, RR, (RR & (RR - 1)) == 0, CP><<<grid, kStepThreads, 0, st>>>(*a); \
  else step_kernel<TA, RR, false, CP><<<grid, kStepThreads, 0, st>>>(*a);
#define M3B_STEP_CASE(RR)                   \
  case RR:                                  \
    if (compact) { M3B_STEP_ROW(RR, true) } \
    else { M3B_STEP_ROW(RR, false) }        \
    break;
  switch (a->prm.R) {
    M3B_STEP_CASE(1)
    M3B_STEP_CASE(2)
    M3B_STEP_CASE(3)
    M3B_STEP_CASE(4)
    default: return fail(M3B_ERR_UNSUPPORTED, "step: mimo_rank %d not built (1..4)", a->prm.R);
  }
#undef M3B_STEP_CASE
#undef M3B_STEP_ROW
  return check_launch("step");
}

int launch_step(const m3b_step_args* a, cudaStream_t st) {
  const m3b_layer_params& p = a->prm;
  const bool compact = a->prev_b != nullptr;
  if (!a->proj || !a->h || !a->angle || !a->h_out || !a->angle_out || !a->y)
    return fail(M3B_ERR_INVALID_ARG, "step: null pointer");
  if (compact ? (!a->prev_x || !a->prev_b_out || !a->prev_x_out) : (!a->prev_bx || !a->bx_out))
    return fail(M3B_ERR_INVALID_ARG, "step: null previous-token state (%s form)", compact ? "compact" : "prev_BX");
  if (p.H <= 0 || p.P <= 0 || p.N <= 0 || p.R <= 0 || p.G <= 0 || p.H % p.G != 0)
    return fail(M3B_ERR_INVALID_ARG, "step: bad dims H=%d P=%d N=%d R=%d G=%d", p.H, p.P, p.N, p.R, p.G);
  if (p.N % 4 != 0 || p.N > kStepMaxN || p.P > kStepMaxP)
    return fail(M3B_ERR_UNSUPPORTED, "step: needs N %% 4 == 0, N <= %d, P <= %d", kStepMaxN, kStepMaxP);
  if (!aligned16(a->h) || !aligned16(a->h_out) ||
      (!compact && (!aligned16(a->prev_bx) || !aligned16(a->bx_out))))
    return fail(M3B_ERR_ALIGNMENT, "step: state buffers must be 16-byte aligned");
  if (a->batch <= 0) return M3B_OK;
  if (a->batch * p.H > 0x7fffffffLL) return fail(M3B_ERR_INVALID_ARG, "step: batch*H too large");
  switch (a->act_dtype) {
    case M3B_F32: return launch_step_t<float>(a, st);
    case M3B_BF16: return launch_step_t<__nv_bfloat16>(a, st);
    case M3B_F16: return launch_step_t<__half>(a, st);
    default: return fail(M3B_ERR_INVALID_ARG, "step: bad act dtype %d", a->act_dtype);
  }
}

}  // namespace m3b
