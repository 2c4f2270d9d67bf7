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
#include <map>
#include <mutex>

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

// ---------------------------------------------------------------------------
// Two-kernel decode step for d_state 128, headdim <= 64 (a multiple of 8), mimo_rank 1, 2 or 4
// (the decode configurations), used when the caller passes a workspace:
//   step_prep_kernel   one warp per (batch, head): the token's operands -- the advanced angle's
//                      cos / sin, x_r, the gate, dA / gamma / beta and D -- into the workspace,
//                      the new angle; the warp of a group's first head also writes the group's
//                      RMSNorm-ed (+ weight, bias) B and C rows, shared by the group's heads.
//   step_stream_kernel persistent CTAs walk the (batch, head) items; the fp32 state of the next
//                      item, its operands, its group's normalised B / C rows and its
//                      previous-token state arrive by bulk copies into the other half of a
//                      two-slot shared-memory ring while the current item is computed, so the
//                      loop has no global-load latency of its own and the state streams at HBM
//                      rate.  Each thread rotates the B^ / C^ entries of its four state columns
//                      in registers.  Stores go straight from registers.
// Same arithmetic as step_kernel.
// ---------------------------------------------------------------------------
constexpr int kStreamN = 128, kStreamPMax = 64;

// operand block of one (batch, head) item, fp32: cos / sin of the advanced angle per pair
// (interleaved), x_r and the gate (PMAX x R each, p-major), then dA, gamma, beta, D.  The
// workspace holds batch x H of these, then per (batch row, group) the normalised B and C rows
// (N R each, (n, r) order as in the projection).
template <int R>
struct OpBlock {
  static constexpr int Cs = 0, Xr = kStreamN, Gate = Xr + kStreamPMax * R;
  static constexpr int Scal = Gate + kStreamPMax * R;
  static constexpr int floats = Scal + 4;
  static constexpr int bytes = floats * 4;
  static constexpr int bc_floats = 2 * kStreamN * R;  // one group's B and C rows
  static_assert(bytes % 16 == 0, "operand blocks are copied in 16-byte units");
};

template <typename TA, int R>
__global__ void __launch_bounds__(256) step_prep_kernel(m3b_step_args a, float* ws, int nitems) {
  // one warp per (batch, head) item; the warp of a group's first head also writes the group's
  // normalised B / C rows.  Every load is issued before the first store (the workspace may alias
  // nothing, but the compiler cannot know that), so an item costs about one memory round trip.
  using OB = OpBlock<R>;
  constexpr int N = kStreamN, NR = N * R;
  constexpr int PC = kStreamPMax / 32;          // channels per lane
  constexpr int Q = NR >= 256 ? NR / 256 : 1;   // 8-entry runs of the B / C rows per lane
  constexpr int RUN = NR >= 256 ? 8 : 4;
  const m3b_layer_params& prm = a.prm;
  const int H = prm.H, P = prm.P, G = prm.G, pd = prm.param_dtype;
  const int lane = threadIdx.x & 31;
  // the streaming kernel may start now: it loads the state (which this kernel does not touch)
  // and waits for this grid's completion before it reads the operand blocks
  pdl_launch_dependents();
  const int item = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (item >= nitems) return;
  const int b = item / H, h = item - b * H, hpg = H / G, g = h / hpg;
  const bool leader = h % hpg == 0;
  const TA* row = reinterpret_cast<const TA*>(a.proj) + (int64_t)b * a.proj_stride;
  const int HP = H * P;
  const int offDt = 2 * HP + 2 * G * NR, offLam = offDt + H, offTh = offLam + (prm.trapezoidal ? H : 0);
  const int offB = 2 * HP + g * NR, offC = 2 * HP + G * NR + g * NR;
  // ---- loads
  const float dt_raw = io<TA>::ld(row + offDt + h);
  const float lam_raw = prm.trapezoidal ? io<TA>::ld(row + offLam + h) : 0.f;
  const float dts = a.dt_scale ? io<TA>::ld(reinterpret_cast<const TA*>(a.dt_scale) + item) : 1.f;
  const float dtb = ldf(prm.dt_bias, h, pd), alog = ldf(prm.A_log, h, pd), Dh = ldf(prm.D, h, pd);
  const int64_t abase = (int64_t)item * (N / 2);
  float ang[2], th[2];
#pragma unroll
  for (int k = 0; k < 2; ++k) {  // pairs lane and lane + 32
    ang[k] = ldf(a.angle, abase + lane + 32 * k, a.angle_dtype);
    th[k] = prm.complex_ssm ? io<TA>::ld(row + offTh + lane + 32 * k) : 0.f;
  }
  float xv[PC], zv[PC], mx[PC][R], mz[PC][R], md[PC][R];
#pragma unroll
  for (int k = 0; k < PC; ++k) {
    const int p = lane + 32 * k;
    const bool on = p < P;
    xv[k] = on ? io<TA>::ld(row + HP + h * P + p) : 0.f;
    zv[k] = on ? io<TA>::ld(row + h * P + p) : 0.f;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int64_t q = ((int64_t)h * P + p) * R + r;
      mx[k][r] = on ? ldf(prm.mimo_x, q, pd) : 0.f;
      mz[k][r] = on ? ldf(prm.mimo_z, q, pd) : 0.f;
      md[k][r] = on ? ldf(prm.mimo_down, q, pd) : 0.f;
    }
  }
  // the group's raw B / C rows (leader warps): entries RUN lane + 256 j .. + RUN - 1
  float bv[Q][RUN], cv[Q][RUN];
  if (leader) {
#pragma unroll
    for (int j = 0; j < Q; ++j) {
      const int e0 = RUN * lane + 256 * j;
      if constexpr (RUN == 8) {
        load8<TA>(row + offB + e0, bv[j]);
        load8<TA>(row + offC + e0, cv[j]);
      } else {
#pragma unroll
        for (int e = 0; e < RUN; ++e) {
          bv[j][e] = io<TA>::ld(row + offB + e0 + e);
          cv[j][e] = io<TA>::ld(row + offC + e0 + e);
        }
      }
    }
  }
  // ---- compute and store
  float* ob = ws + (int64_t)item * OB::floats;
  const float dt = softplus_f(dt_raw + dtb) * dts;
  if (lane == 0) {
    const float dA = expf(-expf(alog) * dt);
    float gamma = dt, beta = 0.f;
    if (prm.trapezoidal) {
      const float lam = sigmoid_f(lam_raw);
      gamma = lam * dt;
      beta = (1.f - lam) * dt * dA;
    }
    *reinterpret_cast<float4*>(ob + OB::Scal) = make_float4(dA, gamma, beta, Dh);
  }
  // the advanced angle of pairs lane, lane + 32 and its cos / sin
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int i = lane + 32 * k;
    float a_ = ang[k], sn = 0.f, cs = 1.f;
    if (prm.complex_ssm) {
      a_ -= dt * th[k];
      sincosf(a_, &sn, &cs);
    }
    a.angle_out[abase + i] = a_;
    *reinterpret_cast<float2*>(ob + OB::Cs + 2 * i) = make_float2(cs, sn);
  }
  // x_r and the gate of channels lane, lane + 32
#pragma unroll
  for (int k = 0; k < PC; ++k) {
    const int p = lane + 32 * k;
    if (p < P) {
#pragma unroll
      for (int r = 0; r < R; ++r) {
        ob[OB::Xr + p * R + r] = xv[k] * mx[k][r];
        ob[OB::Gate + p * R + r] = silu_f(zv[k] * mz[k][r]) * md[k][r];
      }
    }
  }
  if (!leader) return;
  // the group's joint N R RMSNorm of B and C, + weight and bias
  float sb = 0.f, sc = 0.f;
#pragma unroll
  for (int j = 0; j < Q; ++j)
#pragma unroll
    for (int e = 0; e < RUN; ++e) {
      sb = fmaf(bv[j][e], bv[j][e], sb);
      sc = fmaf(cv[j][e], cv[j][e], sc);
    }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    sb += __shfl_xor_sync(0xffffffffu, sb, o);
    sc += __shfl_xor_sync(0xffffffffu, sc, o);
  }
  const float rb = rsqrtf(sb / (float)NR + prm.norm_eps), rc = rsqrtf(sc / (float)NR + prm.norm_eps);
  float* dst = ws + (int64_t)nitems * OB::floats + ((int64_t)b * G + g) * OB::bc_floats;
  // the norm weights and biases: one more round trip for these warps only
  float wb[Q][RUN], wc[Q][RUN], bb[Q][RUN], bc[Q][RUN];
#pragma unroll
  for (int j = 0; j < Q; ++j) {
    const int e0 = RUN * lane + 256 * j;
    if constexpr (RUN == 8) {
      ldf8(prm.B_norm_w, e0, pd, wb[j]);
      ldf8(prm.C_norm_w, e0, pd, wc[j]);
      ldf8(prm.B_bias, (int64_t)g * NR + e0, pd, bb[j]);
      ldf8(prm.C_bias, (int64_t)g * NR + e0, pd, bc[j]);
    } else {
#pragma unroll
      for (int e = 0; e < RUN; ++e) {
        wb[j][e] = ldf(prm.B_norm_w, e0 + e, pd);
        wc[j][e] = ldf(prm.C_norm_w, e0 + e, pd);
        bb[j][e] = ldf(prm.B_bias, (int64_t)g * NR + e0 + e, pd);
        bc[j][e] = ldf(prm.C_bias, (int64_t)g * NR + e0 + e, pd);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < Q; ++j) {
    const int e0 = RUN * lane + 256 * j;
    float ob8[RUN], oc8[RUN];
#pragma unroll
    for (int e = 0; e < RUN; ++e) {
      ob8[e] = fmaf(bv[j][e] * rb, wb[j][e], bb[j][e]);
      oc8[e] = fmaf(cv[j][e] * rc, wc[j][e], bc[j][e]);
    }
#pragma unroll
    for (int e = 0; e < RUN; e += 4) {
      *reinterpret_cast<float4*>(dst + e0 + e) = make_float4(ob8[e], ob8[e + 1], ob8[e + 2], ob8[e + 3]);
      *reinterpret_cast<float4*>(dst + NR + e0 + e) = make_float4(oc8[e], oc8[e + 1], oc8[e + 2], oc8[e + 3]);
    }
  }
}

template <int R, bool COMPACT>
struct StreamPlan {
  static constexpr int N = kStreamN, PMAX = kStreamPMax;
  static constexpr int st = PMAX * N * 4;                              // h (and prev_BX) bytes
  static constexpr int ob = (COMPACT ? 1 : 2) * st;                    // operand block
  static constexpr int bc = ob + OpBlock<R>::bytes;                    // the group's B / C rows
  static constexpr int pb = bc + OpBlock<R>::bc_floats * 4;            // COMPACT: previous B^ (N, R)
  static constexpr int px = pb + N * R * 4;                            // COMPACT: previous x_r (P, R)
  static constexpr int slot_used = COMPACT ? px + PMAX * R * 4 : pb;
  static constexpr int slot = (slot_used + 127) / 128 * 128;     // 128-byte aligned slots
  static_assert(slot >= slot_used, "a slot holds everything copied into it");
  static constexpr int sY = 2 * slot;                                  // PMAX x R
  static constexpr int bars = sY + PMAX * R * 4;                       // 2 mbarriers
  static constexpr int bytes = bars + 16;
};

template <typename TA, int R, bool COMPACT>
__global__ void __launch_bounds__(kStepThreads, COMPACT ? 3 : 1)
    step_stream_kernel(m3b_step_args a, const float* ws, int nitems, uint64_t wait_ns) {
  using SP = StreamPlan<R, COMPACT>;
  using OB = OpBlock<R>;
  extern __shared__ __align__(128) uint8_t ssm[];
  constexpr int N = kStreamN;
  const m3b_layer_params& prm = a.prm;
  const int H = prm.H, P = prm.P;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  float* sY = reinterpret_cast<float*>(ssm + SP::sY);
  uint64_t* bars = reinterpret_cast<uint64_t*>(ssm + SP::bars);
  const int nvec = P * N / 4;
  const uint32_t sbytes = (uint32_t)(P * N * 4);
  const uint32_t pbytes = (uint32_t)(N * R * 4), xbytes = (uint32_t)(P * R * 4);
  const uint32_t bcbytes = (uint32_t)(OB::bc_floats * 4);
  const float* wbc = ws + (int64_t)nitems * OB::floats;  // the (batch row, group) B / C rows
  const int hpg = H / prm.G;
  if (tid == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    fence_mbar_init();
  }
  __syncthreads();
  auto bulk = [](void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
  };
  // bulk copies of item `it` into slot `sl` (thread 0): state, operand block, previous token.
  // parts: 1 = the state and previous token (with the slot's expected byte count), 2 = the
  // operand block and the group's B / C rows, 3 = both.
  auto issue = [&](int it, int sl, int parts) {
    uint8_t* d = ssm + sl * SP::slot;
    uint64_t* bar = &bars[sl];
    const int64_t sbase = (int64_t)it * P * N;
    if (parts & 1) {
      mbar_arrive_expect_tx(bar, (COMPACT ? sbytes + pbytes + xbytes : 2 * sbytes) + (uint32_t)OB::bytes + bcbytes);
      bulk(d, a.h + sbase, sbytes, bar);
      if constexpr (COMPACT) {
        bulk(d + SP::pb, a.prev_b + (int64_t)it * N * R, pbytes, bar);
        bulk(d + SP::px, a.prev_x + (int64_t)it * P * R, xbytes, bar);
      } else {
        bulk(d + SP::st, a.prev_bx + sbase, sbytes, bar);
      }
    }
    if (parts & 2) {
      const int ib = it / H, ig = (it - ib * H) / hpg;
      bulk(d + SP::bc, wbc + ((int64_t)ib * prm.G + ig) * OB::bc_floats, bcbytes, bar);
      bulk(d + SP::ob, ws + (int64_t)it * OB::floats, (uint32_t)OB::bytes, bar);
    }
  };
  const int stride = (int)gridDim.x;
  // The first item's state and previous-token copies do not depend on the preparation kernel
  // before this one (programmatic dependent launch): they start before the wait for it; the
  // operand block and B / C rows it writes are copied after.
  if (tid == 0 && (int)blockIdx.x < nitems) issue((int)blockIdx.x, 0, 1);
  pdl_wait_primary();
  if (tid == 0 && (int)blockIdx.x < nitems) issue((int)blockIdx.x, 0, 2);
  int k = 0;
  for (int item = (int)blockIdx.x; item < nitems; item += stride, ++k) {
    const int sl = k & 1;
    const bool pending = item + stride < nitems;
    // the next item streams into the other slot (released by the barrier ending the last item)
    if (tid == 0 && pending) issue(item + stride, sl ^ 1, 3);
    bool ok = mbar_wait(&bars[sl], (k >> 1) & 1, wait_ns);
    ok = __syncthreads_and(ok);
    if (!ok) {
      // a copy that never completed: the copy into the other slot must land before leaving
      if (tid == 0 && pending) mbar_wait(&bars[sl ^ 1], ((k + 1) >> 1) & 1, wait_ns);
      break;
    }
    const uint8_t* d = ssm + sl * SP::slot;
    const float* obs = reinterpret_cast<const float*>(d + SP::ob);
    const float* sBn = reinterpret_cast<const float*>(d + SP::bc);  // normalised B, then C, (n, r) order
    const float* sCn = sBn + N * R;
    const float* sXr = obs + OB::Xr;
    const float dA = obs[OB::Scal + 0], gamma = obs[OB::Scal + 1], beta = obs[OB::Scal + 2];
    const float4* hs4 = reinterpret_cast<const float4*>(d);
    const float4* ps4 = reinterpret_cast<const float4*>(d + SP::st);
    const float* spb = reinterpret_cast<const float*>(d + SP::pb);  // (n, r) order
    const float* spx = reinterpret_cast<const float*>(d + SP::px);
    float4* ho4 = reinterpret_cast<float4*>(a.h_out + (int64_t)item * P * N);
    float4* bo4 = COMPACT ? nullptr : reinterpret_cast<float4*>(a.bx_out + (int64_t)item * P * N);
    constexpr int BATCH = 8;  // float4 f = u * 256 + tid: row p = 8 u + warp, columns 4 lane ..
    float part[BATCH][R];
    const int n0 = 4 * lane;
    // this thread's four state columns n0 .. n0 + 3 (pairs n0 / 2 and n0 / 2 + 1) are the same for
    // all its rows: their normalised B / C entries (and previous B^) are read from shared memory
    // once per item and rotated here by the head's angle: (x0 c - x1 s, x0 s + x1 c)
    float bq[R][4], cq[R][4], pbv[COMPACT ? 4 * R : 1];
    {
      const float4 cs4 = *reinterpret_cast<const float4*>(obs + OB::Cs + n0);  // c0, s0, c1, s1
      float bn[4 * R], cn[4 * R];
#pragma unroll
      for (int q = 0; q < R; ++q) {
        const float4 b4 = reinterpret_cast<const float4*>(sBn + n0 * R)[q];
        const float4 c4 = reinterpret_cast<const float4*>(sCn + n0 * R)[q];
        bn[4 * q] = b4.x, bn[4 * q + 1] = b4.y, bn[4 * q + 2] = b4.z, bn[4 * q + 3] = b4.w;
        cn[4 * q] = c4.x, cn[4 * q + 1] = c4.y, cn[4 * q + 2] = c4.z, cn[4 * q + 3] = c4.w;
      }
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const float b0 = bn[r], b1 = bn[R + r], b2 = bn[2 * R + r], b3 = bn[3 * R + r];
        const float c0 = cn[r], c1 = cn[R + r], c2 = cn[2 * R + r], c3 = cn[3 * R + r];
        bq[r][0] = b0 * cs4.x - b1 * cs4.y;
        bq[r][1] = b0 * cs4.y + b1 * cs4.x;
        bq[r][2] = b2 * cs4.z - b3 * cs4.w;
        bq[r][3] = b2 * cs4.w + b3 * cs4.z;
        cq[r][0] = c0 * cs4.x - c1 * cs4.y;
        cq[r][1] = c0 * cs4.y + c1 * cs4.x;
        cq[r][2] = c2 * cs4.z - c3 * cs4.w;
        cq[r][3] = c2 * cs4.w + c3 * cs4.z;
      }
    }
    if constexpr (COMPACT) {
#pragma unroll
      for (int q = 0; q < R; ++q) {
        const float4 v4 = reinterpret_cast<const float4*>(spb + n0 * R)[q];
        pbv[4 * q] = v4.x, pbv[4 * q + 1] = v4.y, pbv[4 * q + 2] = v4.z, pbv[4 * q + 3] = v4.w;
      }
    }
#pragma unroll
    for (int u = 0; u < BATCH; ++u) {
      const int f = u * kStepThreads + tid;
      const int p = f >> 5;
      float yr[R];
#pragma unroll
      for (int r = 0; r < R; ++r) yr[r] = 0.f;
      if (f < nvec) {
        const float4 h4 = hs4[f];
        const float hin[4] = {h4.x, h4.y, h4.z, h4.w};
        float pin[4];
        if constexpr (COMPACT) {  // prev_BX[p, n] = sum_r prev_B[n, r] prev_x[p, r]
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            float acc = 0.f;
#pragma unroll
            for (int r = 0; r < R; ++r) acc = fmaf(pbv[jj * R + r], spx[p * R + r], acc);
            pin[jj] = acc;
          }
        } else {
          const float4 p4 = ps4[f];
          pin[0] = p4.x, pin[1] = p4.y, pin[2] = p4.z, pin[3] = p4.w;
        }
        float hn[4], bx[4], xq[R];
#pragma unroll
        for (int r = 0; r < R; ++r) xq[r] = sXr[p * R + r];
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
#pragma unroll
      for (int r = 0; r < R; ++r) part[u][r] = yr[r];
    }
    // y_r of row p = 8 u + warp: one warp-wide reduce-scatter of the BATCH * R partials (each
    // halving step keeps the lower or upper half by one lane bit; a single value left is then
    // added across the remaining bits)
    constexpr int NV = BATCH * R;
    float v[NV];
#pragma unroll
    for (int u = 0; u < BATCH; ++u)
#pragma unroll
      for (int r = 0; r < R; ++r) v[u * R + r] = part[u][r];
    int idx = 0;
#pragma unroll
    for (int st = 0; st < 5; ++st) {
      const int mask = 16 >> st;
      const int cnt = NV >> st;
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
    constexpr int dup = NV >= 32 ? 1 : 32 / NV;
    {
      const int u = idx / R, r = idx - (idx / R) * R;
      const int fw = u * kStepThreads + wid * 32;
      if ((lane & (dup - 1)) == 0 && fw < nvec) sY[(fw >> 5) * R + r] = v[0];
    }
    __syncthreads();
    const int b = item / H, h = item - (item / H) * H;
    if constexpr (COMPACT) {  // this token's B^ and x_r are the next step's previous token
      if (wid == 0) {  // warp 0 holds all N columns' rotated B^: (n, r) entries n0 .. n0 + 3
        float4* pbo = reinterpret_cast<float4*>(a.prev_b_out + (int64_t)item * N * R + n0 * R);
#pragma unroll
        for (int q = 0; q < R; ++q) {
          float v4[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int e = 4 * q + k;  // entry (n0 + e / R, e % R)
            v4[k] = bq[e % R][e / R];
          }
          pbo[q] = make_float4(v4[0], v4[1], v4[2], v4[3]);
        }
      }
      for (int e = tid; e < P * R; e += kStepThreads) a.prev_x_out[(int64_t)item * P * R + e] = sXr[e];
    }
    if (tid < P) {  // readout + D, gate, MIMO down
      const float* sG = obs + OB::Gate;
      const float Dh = obs[OB::Scal + 3];
      float acc = 0.f;
#pragma unroll
      for (int r = 0; r < R; ++r) acc = fmaf(sY[tid * R + r] + Dh * sXr[tid * R + r], sG[tid * R + r], acc);
      io<TA>::st(reinterpret_cast<TA*>(a.y) + (int64_t)b * H * P + (int64_t)h * P + tid, acc);
    }
    __syncthreads();  // the slot and sY are free for the next items
  }
}

// The two-kernel path covers d_state 128, headdim <= 64 (a multiple of 8), mimo_rank 1, 2, 4.
static bool stream_ok(const m3b_step_args* a) {
  const m3b_layer_params& p = a->prm;
  const int esz = a->act_dtype == M3B_F32 ? 4 : 2;
  // the prep's vector loads of the B / C rows: 16-byte aligned projection rows
  const bool rows16 = aligned16(a->proj) && (a->proj_stride * esz) % 16 == 0 && (2 * p.H * p.P) % 8 == 0 &&
                      aligned16(p.B_norm_w) && aligned16(p.C_norm_w) && aligned16(p.B_bias) && aligned16(p.C_bias);
  return p.N == kStreamN && p.P <= kStreamPMax && p.P % 8 == 0 && (p.R == 1 || p.R == 2 || p.R == 4) && rows16 &&
         a->batch * p.H <= 0x7fffffffLL;
}

static size_t stream_ws_bytes(const m3b_step_args* a) {
  const int R = a->prm.R;
  const size_t ob = R == 1 ? OpBlock<1>::bytes : R == 2 ? OpBlock<2>::bytes : OpBlock<4>::bytes;
  const size_t bc = (size_t)2 * kStreamN * R * 4;
  return (size_t)a->batch * a->prm.H * ob + (size_t)a->batch * a->prm.G * bc;
}

template <typename TA, int R, bool COMPACT>
static int launch_stream_t(const m3b_step_args* a, float* ws, cudaStream_t st) {
  using SP = StreamPlan<R, COMPACT>;
  const void* fn = (const void*)step_stream_kernel<TA, R, COMPACT>;
  static std::mutex mu;
  static std::map<int, int> per_sm;  // resident CTAs per SM, per device
  int dev = 0;
  cudaGetDevice(&dev);
  int occ = 0;
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = per_sm.find(dev);
    if (it == per_sm.end()) {
      cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, SP::bytes);
      if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, fn, kStepThreads, SP::bytes);
      if (e != cudaSuccess) return fail(M3B_ERR_CUDA, "step (stream): %s", cudaGetErrorString(e));
      per_sm[dev] = occ;
    } else {
      occ = it->second;
    }
  }
  if (occ < 1) return fail(M3B_ERR_UNSUPPORTED, "step (stream): kernel does not fit an SM");
  const int nitems = (int)(a->batch * a->prm.H);
  step_prep_kernel<TA, R><<<(unsigned)((nitems + 7) / 8), 256, 0, st>>>(*a, ws, nitems);
  int rc = check_launch("step (prep)");
  if (rc != M3B_OK) return rc;
  const int cap = num_sms() * occ;
  const int grid = nitems < cap ? nitems : cap;
  // programmatic dependent launch: the streaming kernel starts while the preparation finishes
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kStepThreads);
  cfg.dynamicSmemBytes = SP::bytes;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  const uint64_t lim = kWaitLimitNs;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, step_stream_kernel<TA, R, COMPACT>, *a, (const float*)ws, nitems, lim);
  if (e != cudaSuccess) return fail(M3B_ERR_CUDA, "step (stream): %s", cudaGetErrorString(e));
  return check_launch("step (stream)");
}

template <typename TA>
static int launch_stream(const m3b_step_args* a, float* ws, cudaStream_t st) {
  const bool compact = a->prev_b != nullptr;
  switch (a->prm.R) {
    case 1: return compact ? launch_stream_t<TA, 1, true>(a, ws, st) : launch_stream_t<TA, 1, false>(a, ws, st);
    case 2: return compact ? launch_stream_t<TA, 2, true>(a, ws, st) : launch_stream_t<TA, 2, false>(a, ws, st);
    default: return compact ? launch_stream_t<TA, 4, true>(a, ws, st) : launch_stream_t<TA, 4, false>(a, ws, st);
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

size_t step_workspace(const m3b_step_args* a) {
  if (!a || !stream_ok(a) || a->batch <= 0) return 0;
  return stream_ws_bytes(a);
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
  if (a->workspace && stream_ok(a)) {
    if (a->workspace_bytes < stream_ws_bytes(a))
      return fail(M3B_ERR_WORKSPACE, "step: need %zu workspace bytes", stream_ws_bytes(a));
    if (!aligned16(a->workspace) || (a->prev_b && (!aligned16(a->prev_b) || !aligned16(a->prev_x))))
      return fail(M3B_ERR_ALIGNMENT, "step: workspace and previous-token buffers must be 16-byte aligned");
    float* ws = static_cast<float*>(a->workspace);
    switch (a->act_dtype) {
      case M3B_F32: return launch_stream<float>(a, ws, st);
      case M3B_BF16: return launch_stream<__nv_bfloat16>(a, ws, st);
      case M3B_F16: return launch_stream<__half>(a, ws, st);
      default: return fail(M3B_ERR_INVALID_ARG, "step: bad act dtype %d", a->act_dtype);
    }
  }
  switch (a->act_dtype) {
    case M3B_F32: return launch_step_t<float>(a, st);
    case M3B_BF16: return launch_step_t<__nv_bfloat16>(a, st);
    case M3B_F16: return launch_step_t<__half>(a, st);
    default: return fail(M3B_ERR_INVALID_ARG, "step: bad act dtype %d", a->act_dtype);
  }
}

}  // namespace m3b
