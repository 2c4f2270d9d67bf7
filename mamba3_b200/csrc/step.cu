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

template <typename TA, int R>
__global__ void __launch_bounds__(kStepThreads) step_kernel(m3b_step_args a) {
  const m3b_layer_params& prm = a.prm;
  const int H = prm.H, P = prm.P, N = prm.N, G = prm.G;
  const int b = blockIdx.x / H;
  const int h = blockIdx.x - b * H;
  const int g = h / (H / G);
  const int tid = threadIdx.x;
  const int NR = N * R;
  const int pd = prm.param_dtype;

  __shared__ float sB[kStepMaxN * R];
  __shared__ float sC[kStepMaxN * R];
  __shared__ float sXr[kStepMaxP * R];
  __shared__ float sGate[kStepMaxP * R];
  __shared__ float sY[kStepMaxP * R];
  __shared__ float sRed[2][kStepThreads / 32];
  __shared__ float sScal[4];  // dA, gamma, beta, dt

  const TA* row = reinterpret_cast<const TA*>(a.proj) + (int64_t)b * a.proj_stride;
  const int HP = H * P;
  const int offB = 2 * HP + g * NR;
  const int offC = 2 * HP + G * NR + g * NR;
  const int offDt = 2 * HP + 2 * G * NR;
  const int offLam = offDt + H;
  const int offTh = offLam + (prm.trapezoidal ? H : 0);

  // --- raw B / C rows of group g and their sums of squares
  float sb = 0.f, sc = 0.f;
  for (int e = tid; e < NR; e += kStepThreads) {
    const float bv = io<TA>::ld(row + offB + e);
    const float cv = io<TA>::ld(row + offC + e);
    sB[e] = bv;
    sC[e] = cv;
    sb += bv * bv;
    sc += cv * cv;
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
    float dt = softplus_f(io<TA>::ld(row + offDt + h) + ldf(prm.dt_bias, h, pd));
    if (a.dt_scale) dt *= io<TA>::ld(reinterpret_cast<const TA*>(a.dt_scale) + (int64_t)b * H + h);
    const float A = -expf(ldf(prm.A_log, h, pd));
    const float dA = expf(A * dt);
    float gamma = dt, beta = 0.f;
    if (prm.trapezoidal) {
      const float lam = sigmoid_f(io<TA>::ld(row + offLam + h));
      gamma = lam * dt;
      beta = (1.f - lam) * dt * dA;
    }
    sScal[0] = dA;
    sScal[1] = gamma;
    sScal[2] = beta;
    sScal[3] = dt;
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
  // normalise + bias, in place
  for (int e = tid; e < NR; e += kStepThreads) {
    sB[e] = sB[e] * rb * ldf(prm.B_norm_w, e, pd) + ldf(prm.B_bias, (int64_t)g * NR + e, pd);
    sC[e] = sC[e] * rc * ldf(prm.C_norm_w, e, pd) + ldf(prm.C_bias, (int64_t)g * NR + e, pd);
  }
  __syncthreads();
  const float dt = sScal[3];
  // --- RoPE advance and rotation of the (2i, 2i+1) pairs
  const int64_t abase = ((int64_t)b * H + h) * (N / 2);
  for (int i = tid; i < N / 2; i += kStepThreads) {
    float ang = ldf(a.angle, abase + i, a.angle_dtype);
    if (prm.complex_ssm) {
      ang -= dt * io<TA>::ld(row + offTh + i);
      float s, c;
      sincosf(ang, &s, &c);
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const float b0 = sB[(2 * i) * R + r], b1 = sB[(2 * i + 1) * R + r];
        sB[(2 * i) * R + r] = b0 * c - b1 * s;
        sB[(2 * i + 1) * R + r] = b0 * s + b1 * c;
        const float c0 = sC[(2 * i) * R + r], c1 = sC[(2 * i + 1) * R + r];
        sC[(2 * i) * R + r] = c0 * c - c1 * s;
        sC[(2 * i + 1) * R + r] = c0 * s + c1 * c;
      }
    }
    a.angle_out[abase + i] = ang;
  }
  // --- MIMO x, gate
  for (int p = tid; p < P; p += kStepThreads) {
    const float xv = io<TA>::ld(row + HP + h * P + p);
    const float zv = io<TA>::ld(row + h * P + p);
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int64_t q = ((int64_t)h * P + p) * R + r;
      sXr[p * R + r] = xv * ldf(prm.mimo_x, q, pd);
      sGate[p * R + r] = silu_f(zv * ldf(prm.mimo_z, q, pd)) * ldf(prm.mimo_down, q, pd);
      sY[p * R + r] = 0.f;
    }
  }
  __syncthreads();

  // --- stream the state: float4 f covers (p, n0..n0+3)
  const float dA = sScal[0], gamma = sScal[1], beta = sScal[2];
  const int64_t sbase = ((int64_t)b * H + h) * (int64_t)P * N;
  const float4* h4 = reinterpret_cast<const float4*>(a.h + sbase);
  const float4* p4 = reinterpret_cast<const float4*>(a.prev_bx + sbase);
  float4* ho4 = reinterpret_cast<float4*>(a.h_out + sbase);
  float4* bo4 = reinterpret_cast<float4*>(a.bx_out + sbase);
  const int nvec = P * N / 4;
  const int gsz = N / 4;                                     // lanes per state row
  const bool pow2 = (gsz & (gsz - 1)) == 0;
  constexpr int BATCH = 8;
  for (int f0 = 0; f0 < nvec; f0 += kStepThreads * BATCH) {
    float4 hv[BATCH], pv[BATCH];
#pragma unroll
    for (int u = 0; u < BATCH; ++u) {
      const int f = f0 + u * kStepThreads + tid;
      if (f < nvec) {
        hv[u] = __ldcs(h4 + f);
        pv[u] = __ldcs(p4 + f);
      }
    }
#pragma unroll
    for (int u = 0; u < BATCH; ++u) {
      const int f = f0 + u * kStepThreads + tid;
      const bool ok = f < nvec;
      const int p = ok ? (4 * f) / N : 0;
      const int n0 = ok ? (4 * f) - p * N : 0;
      float yr[R];
#pragma unroll
      for (int r = 0; r < R; ++r) yr[r] = 0.f;
      if (ok) {
        const float hin[4] = {hv[u].x, hv[u].y, hv[u].z, hv[u].w};
        const float pin[4] = {pv[u].x, pv[u].y, pv[u].z, pv[u].w};
        float hn[4], bx[4];
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          const int n = n0 + jj;
          float cur = 0.f;
#pragma unroll
          for (int r = 0; r < R; ++r) cur = fmaf(sB[n * R + r], sXr[p * R + r], cur);
          bx[jj] = cur;
          hn[jj] = fmaf(dA, hin[jj], fmaf(gamma, cur, beta * pin[jj]));
#pragma unroll
          for (int r = 0; r < R; ++r) yr[r] = fmaf(sC[n * R + r], hn[jj], yr[r]);
        }
        __stcs(ho4 + f, make_float4(hn[0], hn[1], hn[2], hn[3]));
        __stcs(bo4 + f, make_float4(bx[0], bx[1], bx[2], bx[3]));
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
  }
  __syncthreads();
  // --- readout + D, gate, MIMO down
  const float Dh = ldf(prm.D, h, pd);
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
  switch (a->prm.R) {
    case 1: step_kernel<TA, 1><<<grid, kStepThreads, 0, st>>>(*a); break;
    case 2: step_kernel<TA, 2><<<grid, kStepThreads, 0, st>>>(*a); break;
    case 3: step_kernel<TA, 3><<<grid, kStepThreads, 0, st>>>(*a); break;
    case 4: step_kernel<TA, 4><<<grid, kStepThreads, 0, st>>>(*a); break;
    default: return fail(M3B_ERR_UNSUPPORTED, "step: mimo_rank %d not built (1..4)", a->prm.R);
  }
  return check_launch("step");
}

int launch_step(const m3b_step_args* a, cudaStream_t st) {
  const m3b_layer_params& p = a->prm;
  if (!a->proj || !a->h || !a->prev_bx || !a->angle || !a->h_out || !a->bx_out || !a->angle_out || !a->y)
    return fail(M3B_ERR_INVALID_ARG, "step: null pointer");
  if (p.H <= 0 || p.P <= 0 || p.N <= 0 || p.R <= 0 || p.G <= 0 || p.H % p.G != 0)
    return fail(M3B_ERR_INVALID_ARG, "step: bad dims H=%d P=%d N=%d R=%d G=%d", p.H, p.P, p.N, p.R, p.G);
  if (p.N % 4 != 0 || p.N > kStepMaxN || p.P > kStepMaxP)
    return fail(M3B_ERR_UNSUPPORTED, "step: needs N %% 4 == 0, N <= %d, P <= %d", kStepMaxN, kStepMaxP);
  if (!aligned16(a->h) || !aligned16(a->prev_bx) || !aligned16(a->h_out) || !aligned16(a->bx_out))
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
