// Backward of chunked_ssd on pre-processed tensors (the gradients of mamba3/ssd.py:118-244,
// which the reference obtains from torch autograd through _IntraChunkFn, mamba3/ssd.py:27-115,
// and SSDScanFn, mamba3/scan.py:65-140).
//
// The chunked forward is the token recurrence (per batch row b and head h; chunking only
// regroups it):
//   h_t = a_t h_{t-1} + dt_t Xt_t Bt_t^T,  a_t = exp(A dt_t),  h_{-1} = h_init,
//   y_t = h_t C_t + D x_raw_t,             h_final = h_{T-1}
// with Xt = [x_g | x_b] (P x RI), Bt = [B_g | B_b] (N x RI), C (N x R).  Its gradients, with
// G_t = dL/dh_t = a_{t+1} G_{t+1} + dy_t C_t^T (G_T = dh_final, a_T = 1):
//   dXt_t = dt_t G_t Bt_t,  dBt_t = dt_t G_t^T Xt_t,  dC_t = h_t^T dy_t,
//   dx_raw = D dy,  dD = sum dy . x_raw,  dh_init = a_0 G_0,
//   ddt_t = fr_t + A m_t,  dA = sum_t dt_t m_t,
// where fr_t = <G_t, Xt_t Bt_t^T> and m_t = a_t <G_t, h_{t-1}>.  m_t needs h_{t-1} and G_t
// together, but satisfies a scalar recurrence: <G_t, h_t> = m_{t+1} + e_t with
// e_t = <dy_t, h_t C_t> = <C_t, dC_t>, and <G_t, h_t> = m_t + dt_t fr_t, so
//   m_t = m_{t+1} + e_t - dt_t fr_t,  m_T = <dh_final, h_final>:
// a suffix sum of per-token scalars from the two sweeps.
//
// Design: one CTA per (batch row, head) walks the tokens twice with the P x N state in
// shared memory (rows padded to N + 1 floats: column walks are conflict free): a forward
// sweep (h, dC, e_t, dx_raw, dD) and a reverse sweep (G, dXt, dBt, fr_t, dh_init), then the
// suffix sum gives ddt and this row's share of dA.  Each token's operands are staged in a
// double-buffered shared-memory slot loaded one token ahead; per-token scalars go to the
// workspace as per-warp partial sums, added in warp order, and the (b, h) shares of dA / dD
// are added over b in order by a second kernel: no atomics, bitwise reproducible.  fp32
// arithmetic throughout; gradients are stored in the dtypes of their inputs.
#include "chunk.cuh"
#include "launch.h"

namespace m3b {

namespace {

constexpr int kBwdThreads = 256;
constexpr int kBwdWarps = kBwdThreads / 32;
constexpr int kMaxRI = 16;  // 2 R with R <= 8

struct BwdParams {
  int64_t B, T;
  int H, P, N, R, RI;
  const void *x_g, *x_b, *B_g, *B_b, *C, *x_raw, *dt, *A, *D, *dy;
  int dt_dtype, ad_dtype;
  const float* h_init;
  const float* dh_final;
  void *dx_g, *dx_b, *dB_g, *dB_b, *dC, *dx_raw, *ddt;
  float* dh_init;
  float* ew;   // (B*H, T, kBwdWarps) per-warp partials of e_t
  float* fw;   // (B*H, T, kBwdWarps) per-warp partials of fr_t
  float* dA_bh;  // (B, H)
  float* dD_bh;  // (B, H)
  float* mT_bh;   // (B, H) <dh_final, h_final>, from the tiled kernel's forward-sweep CTAs
  float* dDf_bh;  // (B, H) sum dy . x_raw, likewise
};

// One token's operands in shared memory (floats): Xt [p][j], Bt^T [j][n], C^T [q][n], dy [p][q]
struct Slot {
  float* x;
  float* bt;
  float* ct;
  float* dy;
  float* sc;  // dt, a
};

__host__ __device__ inline int slot_floats(int P, int N, int R, int RI) {
  return ((P * RI + RI * N + R * N + P * R + 4) + 3) & ~3;
}

__device__ __forceinline__ Slot slot_at(float* base, int P, int N, int R, int RI) {
  Slot s;
  s.x = base;
  s.bt = s.x + P * RI;
  s.ct = s.bt + RI * N;
  s.dy = s.ct + R * N;
  s.sc = s.dy + P * R;
  return s;
}

template <typename T>
__device__ __forceinline__ void load_slot(const BwdParams& a, const Slot& s, int64_t b, int h, int64_t t,
                                          float Aval) {
  const int P = a.P, N = a.N, R = a.R, RI = a.RI;
  const int64_t row = (b * a.T + t) * a.H + h;
  const T* xg = static_cast<const T*>(a.x_g) + row * P * R;
  const T* xb = a.x_b ? static_cast<const T*>(a.x_b) + row * P * R : nullptr;
  const T* bg = static_cast<const T*>(a.B_g) + row * N * R;
  const T* bb = a.B_b ? static_cast<const T*>(a.B_b) + row * N * R : nullptr;
  const T* cc = static_cast<const T*>(a.C) + row * N * R;
  const T* gy = static_cast<const T*>(a.dy) + row * P * R;
  for (int e = threadIdx.x; e < P * R; e += kBwdThreads) {
    const int p = e / R, r = e - p * R;
    s.x[p * RI + r] = io<T>::ld(xg + e);
    if (xb) s.x[p * RI + R + r] = io<T>::ld(xb + e);
    s.dy[e] = io<T>::ld(gy + e);
  }
  for (int e = threadIdx.x; e < N * R; e += kBwdThreads) {
    const int n = e / R, r = e - n * R;
    s.bt[r * N + n] = io<T>::ld(bg + e);
    if (bb) s.bt[(R + r) * N + n] = io<T>::ld(bb + e);
    s.ct[r * N + n] = io<T>::ld(cc + e);
  }
  if (threadIdx.x == 0) {
    const float dtv = ldf(a.dt, row, a.dt_dtype);
    s.sc[0] = dtv;
    s.sc[1] = expf(Aval * dtv);
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

// Suffix pass shared by the backward kernels: m_t = m_{t+1} + e_t - dt_t fr_t (m_T = mT) from the
// per-warp partials ew / fw, then ddt_t = fr_t + A m_t and this (b, h)'s shares of dA and dD.
// suf: >= kBwdThreads floats of shared memory, red: >= kBwdWarps; both free for reuse here.
__device__ void bwd_finish(const BwdParams& a, int64_t bh, int64_t b, int h, float Aval, float mT, float dD_acc,
                           const float* ew, const float* fw, float* suf, float* red) {
  const int64_t TT = a.T;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // thread i owns tokens [i*seg, (i+1)*seg); the per-warp partials of e_t, fr_t are visible
  // (written before the last barrier of the reverse sweep, or the forward sweep's)
  const int64_t seg = (TT + kBwdThreads - 1) / kBwdThreads;
  const int64_t t0 = tid * seg, t1 = t0 + seg < TT ? t0 + seg : TT;
  auto tok = [&](int64_t t, float& e, float& f, float& dtv) {
    e = 0.f;
    f = 0.f;
    for (int w = 0; w < kBwdWarps; ++w) {
      e += ew[t * kBwdWarps + w];
      f += fw[t * kBwdWarps + w];
    }
    dtv = ldf(a.dt, (b * TT + t) * a.H + h, a.dt_dtype);
  };
  float local = 0.f;
  for (int64_t t = t0; t < t1; ++t) {
    float e, f, dtv;
    tok(t, e, f, dtv);
    local += e - dtv * f;
  }
  suf[tid] = local;
  __syncthreads();
  if (tid == 0) {  // exclusive suffix sums of the segment sums, in segment order
    float acc = mT;
    for (int i = kBwdThreads - 1; i >= 0; --i) {
      const float v = suf[i];
      suf[i] = acc;
      acc += v;
    }
  }
  __syncthreads();
  float m = suf[tid];
  float dA_acc = 0.f;
  for (int64_t t = t1 - 1; t >= t0; --t) {
    float e, f, dtv;
    tok(t, e, f, dtv);
    m += e - dtv * f;
    const int64_t row = (b * TT + t) * a.H + h;
    const float g = f + Aval * m;
    if (a.dt_dtype == M3B_F32) static_cast<float*>(a.ddt)[row] = g;
    else if (a.dt_dtype == M3B_BF16) static_cast<__nv_bfloat16*>(a.ddt)[row] = __float2bfloat16_rn(g);
    else static_cast<__half*>(a.ddt)[row] = __float2half_rn(g);
    dA_acc = fmaf(dtv, m, dA_acc);
  }
  __syncthreads();
  dA_acc = warp_sum(dA_acc);
  dD_acc = warp_sum(dD_acc);
  if (lane == 0) {
    red[warp] = dA_acc;
    suf[warp] = dD_acc;
  }
  __syncthreads();
  if (tid == 0) {
    float sa = 0.f, sd = 0.f;
    for (int w = 0; w < kBwdWarps; ++w) {
      sa += red[w];
      sd += suf[w];
    }
    a.dA_bh[bh] = sa;
    a.dD_bh[bh] = sd;
  }
}

template <typename T>
__global__ void __launch_bounds__(kBwdThreads) ssd_bwd_kernel(BwdParams a) {
  extern __shared__ float4 smem4[];
  float* sm = reinterpret_cast<float*>(smem4);
  const int P = a.P, N = a.N, R = a.R, RI = a.RI;
  const int NS = N + 1;  // padded row of the state
  const int64_t bh = blockIdx.x;
  const int64_t b = bh / a.H;
  const int h = (int)(bh - b * a.H);
  const int64_t TT = a.T;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  float* S = sm;  // [P][N+1]: h in the forward sweep, G in the reverse sweep
  const int sf = slot_floats(P, N, R, RI);
  float* slots = S + ((P * NS + 3) & ~3);
  float* red = slots + (2 * sf > kBwdThreads ? 2 * sf : kBwdThreads);  // [kBwdWarps] block reductions
  auto slot = [&](int64_t t) { return slot_at(slots + (t & 1) * sf, P, N, R, RI); };
  const float Aval = ldf(a.A, h, a.ad_dtype);
  const float Dval = ldf(a.D, h, a.ad_dtype);
  const int64_t state_base = bh * (int64_t)P * N;
  float* ew = a.ew + bh * TT * kBwdWarps;
  float* fw = a.fw + bh * TT * kBwdWarps;

  // ---------------- forward sweep: h_t, dC_t, e_t, dx_raw, dD ----------------
  for (int e = tid; e < P * N; e += kBwdThreads) {
    const int p = e / N, n = e - p * N;
    S[p * NS + n] = a.h_init ? a.h_init[state_base + e] : 0.f;
  }
  float dD_acc = 0.f;
  if (TT > 0) load_slot<T>(a, slot(0), b, h, 0, Aval);
  __syncthreads();
  for (int64_t t = 0; t < TT; ++t) {
    const Slot s = slot(t);
    const float dtv = s.sc[0], av = s.sc[1];
    // h_t = a_t h_{t-1} + dt_t Xt Bt^T
    for (int e = tid; e < P * N; e += kBwdThreads) {
      const int p = e / N, n = e - p * N;
      float u = 0.f;
      for (int j = 0; j < RI; ++j) u = fmaf(s.x[p * RI + j], s.bt[j * N + n], u);
      S[p * NS + n] = fmaf(av, S[p * NS + n], dtv * u);
    }
    // dx_raw = D dy and dD (this slot's dy; x_raw straight from global memory)
    {
      const int64_t row = (b * TT + t) * a.H + h;
      const T* xr = static_cast<const T*>(a.x_raw) + row * P * R;
      T* dxr = static_cast<T*>(a.dx_raw) + row * P * R;
      for (int e = tid; e < P * R; e += kBwdThreads) {
        const float g = s.dy[e];
        dD_acc = fmaf(g, io<T>::ld(xr + e), dD_acc);
        io<T>::st(dxr + e, Dval * g);
      }
    }
    __syncthreads();
    if (t + 1 < TT) load_slot<T>(a, slot(t + 1), b, h, t + 1, Aval);
    // dC_t[n, q] = sum_p h_t[p, n] dy_t[p, q];  e_t = <C_t, dC_t>
    {
      const int64_t row = (b * TT + t) * a.H + h;
      T* dc = static_cast<T*>(a.dC) + row * N * R;
      float e_acc = 0.f;
      for (int o = tid; o < N * R; o += kBwdThreads) {
        const int q = o / N, n = o - q * N;
        float v = 0.f;
        for (int p = 0; p < P; ++p) v = fmaf(S[p * NS + n], s.dy[p * R + q], v);
        io<T>::st(dc + (int64_t)n * R + q, v);
        e_acc = fmaf(s.ct[q * N + n], v, e_acc);
      }
      e_acc = warp_sum(e_acc);
      if (lane == 0) ew[t * kBwdWarps + warp] = e_acc;
    }
    __syncthreads();
  }
  // h_final = h_{T-1};  m_T = <dh_final, h_final>
  float mT = 0.f;
  {
    float acc = 0.f;
    if (a.dh_final)
      for (int e = tid; e < P * N; e += kBwdThreads) {
        const int p = e / N, n = e - p * N;
        acc = fmaf(a.dh_final[state_base + e], S[p * NS + n], acc);
      }
    acc = warp_sum(acc);
    if (lane == 0) red[warp] = acc;
    __syncthreads();
    for (int w = 0; w < kBwdWarps; ++w) mT += red[w];
    __syncthreads();
  }

  // ---------------- reverse sweep: G_t, dXt_t, dBt_t, fr_t, dh_init ----------------
  for (int e = tid; e < P * N; e += kBwdThreads) {
    const int p = e / N, n = e - p * N;
    S[p * NS + n] = a.dh_final ? a.dh_final[state_base + e] : 0.f;
  }
  if (TT > 0) load_slot<T>(a, slot(TT - 1), b, h, TT - 1, Aval);
  __syncthreads();
  float a_next = 1.f;  // a_{t+1} (1 past the last token)
  for (int64_t t = TT - 1; t >= 0; --t) {
    const Slot s = slot(t);
    const float dtv = s.sc[0], av = s.sc[1];
    // G_t = a_{t+1} G_{t+1} + dy_t C_t^T
    for (int e = tid; e < P * N; e += kBwdThreads) {
      const int p = e / N, n = e - p * N;
      float u = 0.f;
      for (int q = 0; q < R; ++q) u = fmaf(s.dy[p * R + q], s.ct[q * N + n], u);
      S[p * NS + n] = fmaf(a_next, S[p * NS + n], u);
    }
    __syncthreads();
    if (t > 0) load_slot<T>(a, slot(t - 1), b, h, t - 1, Aval);
    const int64_t row = (b * TT + t) * a.H + h;
    // dXt[p, j] = dt_t sum_n G_t[p, n] Bt[n, j]
    for (int o = tid; o < P * RI; o += kBwdThreads) {
      const int j = o / P, p = o - j * P;
      float v = 0.f;
      for (int n = 0; n < N; ++n) v = fmaf(S[p * NS + n], s.bt[j * N + n], v);
      v *= dtv;
      if (j < R) io<T>::st(static_cast<T*>(a.dx_g) + row * P * R + (int64_t)p * R + j, v);
      else io<T>::st(static_cast<T*>(a.dx_b) + row * P * R + (int64_t)p * R + (j - R), v);
    }
    // E[n, j] = sum_p G_t[p, n] Xt[p, j];  dBt = dt_t E;  fr_t = <Bt, E>
    float f_acc = 0.f;
    for (int o = tid; o < N * RI; o += kBwdThreads) {
      const int j = o / N, n = o - j * N;
      float v = 0.f;
      for (int p = 0; p < P; ++p) v = fmaf(S[p * NS + n], s.x[p * RI + j], v);
      f_acc = fmaf(s.bt[j * N + n], v, f_acc);
      v *= dtv;
      if (j < R) io<T>::st(static_cast<T*>(a.dB_g) + row * N * R + (int64_t)n * R + j, v);
      else io<T>::st(static_cast<T*>(a.dB_b) + row * N * R + (int64_t)n * R + (j - R), v);
    }
    f_acc = warp_sum(f_acc);
    if (lane == 0) fw[t * kBwdWarps + warp] = f_acc;
    a_next = av;
    __syncthreads();
  }
  // dh_init = a_0 G_0
  if (a.dh_init)
    for (int e = tid; e < P * N; e += kBwdThreads) {
      const int p = e / N, n = e - p * N;
      a.dh_init[state_base + e] = a_next * S[p * NS + n];
    }

  bwd_finish(a, bh, b, h, Aval, mT, dD_acc, ew, fw, slots, red);
}

// ---------------------------------------------------------------------------------------------
// Register-tiled variant (P <= 64, N <= 128, R <= 4): the same two sweeps with the state held
// in registers, each sweep in its own CTA (the sweeps share nothing but per-token scalars):
// CTAs [0, B*H) walk the tokens in reverse (G, the larger share of the work, scheduled first),
// CTAs [B*H, 2*B*H) walk them forward (h), and ssd_bwd_finish_kernel runs the suffix pass.  Thread (pb, nb) owns rows p = 4 pb + i (i < 4) and columns n = 8 nb + k
// (k < 8) of h / G; lanes carry nbl = lane & 7 and pbl = lane >> 3, warps nbh = warp & 1 and
// pbh = warp >> 1 (nb = nbl + 8 nbh, pb = pbl + 4 pbh).  Per token the sums over n (dX) and
// over p (dB, dC) are reduce-scattered across the lanes of a warp with shuffles and finished
// across warps in shared memory, one barrier per token.  Token operands are fetched into
// registers one token ahead and stored into a three-deep ring of shared-memory slots.
constexpr int kTilePairs = 5;  // operand element pairs one thread fetches per token (<= 2560 / 2 / 256)

template <int R, int RI>
struct TPlan {
  static constexpr int JB = RI > 4 ? 4 : RI;  // j block of one reduction pass
  static constexpr int NJ = RI / JB;
  static constexpr int VX = 4 * JB < 8 ? 8 : 4 * JB;  // dX partials per thread and pass (padded)
  static constexpr int VE = 8 * JB;                    // dB partials per thread and pass
  static constexpr int VC = 8 * R;                     // dC partials per thread
  // one slot: Xt [64][RI], Bt^T [RI][128], C^T [R][128], dy [64][R], x_raw [64][R], dt, a
  static constexpr int sx = 0, sbt = sx + 64 * RI, sct = sbt + RI * 128, sdy = sct + R * 128,
                       sxr = sdy + 64 * R, ssc = sxr + 64 * R, slot = (ssc + 4 + 31) & ~31;
  static constexpr int redx = 2 * 16 * NJ * VX;  // [nbh][pb][jb][VX]
  static constexpr int rede = 4 * 16 * NJ * VE;  // [pbh][nb][jb][VE]
  static constexpr int redc = 4 * 16 * VC;       // [pbh][nb][VC]
  static constexpr int red = (redx + rede > redc ? redx + rede : redc);
  static constexpr int floats = 3 * slot + 2 * red + 32;
};

// v[0..V) summed over the 2^NB lanes that differ in lane bits lo .. lo+NB-1; afterwards this lane
// holds the sums of V >> NB consecutive values, v[0 ..) = global values [returned offset ..).
template <int V, int NB>
__device__ __forceinline__ int reduce_scatter(float (&v)[V], int lane, int lo) {
  int off = 0;
#pragma unroll
  for (int r = 0; r < NB; ++r) {
    const int bit = 1 << (lo + r);
    const bool up = (lane & bit) != 0;
    const int half = V >> (r + 1);
#pragma unroll
    for (int i = 0; i < half; ++i) {
      const float send = up ? v[i] : v[half + i];
      const float keep = up ? v[half + i] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, bit);
    }
    off += up ? half : 0;
  }
  return off;
}

// raw storage of two consecutive elements: one 32-bit word for bf16, two floats for fp32
template <typename T>
struct PairT;
template <>
struct PairT<__nv_bfloat16> {
  using type = uint32_t;
  static __device__ __forceinline__ type ld(const __nv_bfloat16* p) { return __ldg(reinterpret_cast<const unsigned*>(p)); }
  static __device__ __forceinline__ float lo(type w) { return __uint_as_float(w << 16); }
  static __device__ __forceinline__ float hi(type w) { return __uint_as_float(w & 0xffff0000u); }
};
template <>
struct PairT<float> {
  using type = float2;
  static __device__ __forceinline__ type ld(const float* p) { return __ldg(reinterpret_cast<const float2*>(p)); }
  static __device__ __forceinline__ float lo(type w) { return w.x; }
  static __device__ __forceinline__ float hi(type w) { return w.y; }
};

template <typename T>
struct TokFetch {
  typename PairT<T>::type w[kTilePairs];
  float dt;
};

// the operands of token `row` (flat (b, t, h) index): Xt, Bt, C, dy and, in the forward sweep,
// x_raw; as registers (fetch: element pairs, every segment has an even length) and then into a
// slot (store)
template <typename T, int R, int RI>
__device__ __forceinline__ void tile_fetch(const BwdParams& a, int64_t row, bool with_xr, TokFetch<T>& f) {
  using PT = PairT<T>;
  const int P = a.P, N = a.N;
  const int PR = P * R, NR = N * R;
  const bool beta = RI == 2 * R;
  const int s0 = PR, s1 = s0 + (beta ? PR : 0), s2 = s1 + NR, s3 = s2 + (beta ? NR : 0), s4 = s3 + NR, s5 = s4 + PR,
            s6 = s5 + (with_xr ? PR : 0);
  const int64_t rp = row * PR, rn = row * NR;
#pragma unroll
  for (int u = 0; u < kTilePairs; ++u) {
    const int e = 2 * (threadIdx.x + kBwdThreads * u);
    typename PT::type v{};
    if (e < s0) v = PT::ld(static_cast<const T*>(a.x_g) + rp + e);
    else if (e < s1) v = PT::ld(static_cast<const T*>(a.x_b) + rp + (e - s0));
    else if (e < s2) v = PT::ld(static_cast<const T*>(a.B_g) + rn + (e - s1));
    else if (e < s3) v = PT::ld(static_cast<const T*>(a.B_b) + rn + (e - s2));
    else if (e < s4) v = PT::ld(static_cast<const T*>(a.C) + rn + (e - s3));
    else if (e < s5) v = PT::ld(static_cast<const T*>(a.dy) + rp + (e - s4));
    else if (e < s6) v = PT::ld(static_cast<const T*>(a.x_raw) + rp + (e - s5));
    f.w[u] = v;
  }
  f.dt = threadIdx.x == 0 ? ldf(a.dt, row, a.dt_dtype) : 0.f;
}

template <typename T, int R, int RI>
__device__ __forceinline__ void tile_store(const BwdParams& a, float* slot, bool with_xr, const TokFetch<T>& f,
                                           float Aval) {
  using TP = TPlan<R, RI>;
  using PT = PairT<T>;
  const int P = a.P, N = a.N;
  const int PR = P * R, NR = N * R;
  const bool beta = RI == 2 * R;
  const int s0 = PR, s1 = s0 + (beta ? PR : 0), s2 = s1 + NR, s3 = s2 + (beta ? NR : 0), s4 = s3 + NR, s5 = s4 + PR,
            s6 = s5 + (with_xr ? PR : 0);
  // element e of a segment -> its slot position
  auto put = [&](int e, float v) {
    if (e < s0) slot[TP::sx + (e / R) * RI + e % R] = v;
    else if (e < s1) slot[TP::sx + ((e - s0) / R) * RI + R + (e - s0) % R] = v;
    else if (e < s2) slot[TP::sbt + ((e - s1) % R) * 128 + (e - s1) / R] = v;
    else if (e < s3) slot[TP::sbt + (R + (e - s2) % R) * 128 + (e - s2) / R] = v;
    else if (e < s4) slot[TP::sct + ((e - s3) % R) * 128 + (e - s3) / R] = v;
    else if (e < s5) slot[TP::sdy + (e - s4)] = v;
    else if (e < s6) slot[TP::sxr + (e - s5)] = v;
  };
#pragma unroll
  for (int u = 0; u < kTilePairs; ++u) {
    const int e = 2 * (threadIdx.x + kBwdThreads * u);
    if (e < s6) {
      put(e, PT::lo(f.w[u]));
      put(e + 1, PT::hi(f.w[u]));
    }
  }
  if (threadIdx.x == 0) {
    slot[TP::ssc] = f.dt;
    slot[TP::ssc + 1] = expf(Aval * f.dt);
  }
}

template <typename T, int R, int RI>
__global__ void __launch_bounds__(kBwdThreads, 2) ssd_bwd_tiled_kernel(BwdParams a) {
  using TP = TPlan<R, RI>;
  constexpr int JB = TP::JB, NJ = TP::NJ, VX = TP::VX, VE = TP::VE, VC = TP::VC;
  extern __shared__ float4 smem4[];
  float* sm = reinterpret_cast<float*>(smem4);
  const int P = a.P, N = a.N;
  const int64_t nbhs = a.B * a.H;
  const bool rev_role = (int64_t)blockIdx.x < nbhs;
  const int64_t bh = rev_role ? (int64_t)blockIdx.x : (int64_t)blockIdx.x - nbhs;
  const int64_t b = bh / a.H;
  const int h = (int)(bh - b * a.H);
  const int64_t TT = a.T;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nbl = lane & 7, pbl = lane >> 3, nbh = warp & 1, pbh = warp >> 1;
  const int nb = nbl + 8 * nbh, pb = pbl + 4 * pbh;
  const int p0 = 4 * pb, n0 = 8 * nb;
  float* slots = sm;                       // 3 x TP::slot
  float* redbuf = sm + 3 * TP::slot;       // 2 x TP::red
  float* red = redbuf + 2 * TP::red;       // 32 floats
  auto slot = [&](int64_t t) { return slots + (int)(t % 3) * TP::slot; };
  const float Aval = ldf(a.A, h, a.ad_dtype);
  const float Dval = ldf(a.D, h, a.ad_dtype);
  const int64_t state_base = bh * (int64_t)P * N;
  float* ew = a.ew + bh * TT * kBwdWarps;
  float* fw = a.fw + bh * TT * kBwdWarps;
  // rows / columns past P / N stay zero in every slot
  for (int e = tid; e < 3 * TP::slot; e += kBwdThreads) slots[e] = 0.f;
  auto ok_pk = [&](int i, int k) { return p0 + i < P && n0 + k < N; };

  float st[4][8];
  // token operands are fetched two tokens ahead into two register sets that trade roles every
  // token (so a set is stored one full token after its loads were issued)
  TokFetch<T> fa, fb;
  __syncthreads();  // slots zeroed
  if (!rev_role) {
  // ---------------- forward sweep: h_t, dC_t, e_t, dx_raw, dD ----------------
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int k = 0; k < 8; ++k)
      st[i][k] = a.h_init && ok_pk(i, k) ? a.h_init[state_base + (int64_t)(p0 + i) * N + n0 + k] : 0.f;
  float dD_acc = 0.f;
  if (TT > 0) {
    tile_fetch<T, R, RI>(a, (b * TT) * a.H + h, true, fa);
    tile_store<T, R, RI>(a, slot(0), true, fa, Aval);
  }
  if (TT > 1) tile_fetch<T, R, RI>(a, (b * TT + 1) * a.H + h, true, fa);
  __syncthreads();
  // token t; fcur holds token t + 1 (stored here), fnext receives token t + 2
  auto fwd_tok = [&](int64_t t, TokFetch<T>& fcur, TokFetch<T>& fnext) {
    if (t + 2 < TT) tile_fetch<T, R, RI>(a, (b * TT + t + 2) * a.H + h, true, fnext);
    const float* sl = slot(t);
    const float dtv = sl[TP::ssc], av = sl[TP::ssc + 1];
    // h_t = a_t h_{t-1} + dt_t Xt Bt^T
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int k = 0; k < 8; ++k) st[i][k] *= av;
#pragma unroll
    for (int j = 0; j < RI; ++j) {
      float bv[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) bv[k] = sl[TP::sbt + j * 128 + n0 + k];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float xv = dtv * sl[TP::sx + (p0 + i) * RI + j];
#pragma unroll
        for (int k = 0; k < 8; ++k) st[i][k] = fmaf(xv, bv[k], st[i][k]);
      }
    }
    // dC partials over this thread's rows: pc[k R + q] = sum_i h[i][k] dy[p0 + i][q]
    float pc[VC];
#pragma unroll
    for (int e = 0; e < VC; ++e) pc[e] = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
      for (int q = 0; q < R; ++q) {
        const float g = sl[TP::sdy + (p0 + i) * R + q];
#pragma unroll
        for (int k = 0; k < 8; ++k) pc[k * R + q] = fmaf(st[i][k], g, pc[k * R + q]);
      }
    }
    const int offc = reduce_scatter<VC, 2>(pc, lane, 3);
    float* rc = redbuf + (int)(t & 1) * TP::red + (pbh * 16 + nb) * VC + offc;
#pragma unroll
    for (int e = 0; e < VC / 4; ++e) rc[e] = pc[e];
    if (t + 1 < TT) tile_store<T, R, RI>(a, slot(t + 1), true, fcur, Aval);
    __syncthreads();
    // dC_t, e_t = <C_t, dC_t>; dx_raw = D dy, dD
    const int64_t row = (b * TT + t) * a.H + h;
    const float* rcs = redbuf + (int)(t & 1) * TP::red;
    float e_acc = 0.f;
    for (int o = tid; o < N * R; o += kBwdThreads) {
      const int n = o / R, q = o - n * R;
      const int idx = (n & 7) * R + q, nbo = n >> 3;
      const float v = rcs[(0 * 16 + nbo) * VC + idx] + rcs[(1 * 16 + nbo) * VC + idx] +
                      rcs[(2 * 16 + nbo) * VC + idx] + rcs[(3 * 16 + nbo) * VC + idx];
      io<T>::st(static_cast<T*>(a.dC) + row * N * R + o, v);
      e_acc = fmaf(sl[TP::sct + q * 128 + n], v, e_acc);
    }
    for (int o = tid; o < P * R; o += kBwdThreads) {
      const float g = sl[TP::sdy + o];
      dD_acc = fmaf(g, sl[TP::sxr + o], dD_acc);
      io<T>::st(static_cast<T*>(a.dx_raw) + row * P * R + o, Dval * g);
    }
    e_acc = warp_sum(e_acc);
    if (lane == 0) ew[t * kBwdWarps + warp] = e_acc;
  };
  for (int64_t t = 0; t < TT; t += 2) {
    fwd_tok(t, fa, fb);
    if (t + 1 < TT) fwd_tok(t + 1, fb, fa);
  }
  // m_T = <dh_final, h_final> and this (b, h)'s share of dD, for the suffix pass
  {
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float g = a.dh_final && ok_pk(i, k) ? a.dh_final[state_base + (int64_t)(p0 + i) * N + n0 + k] : 0.f;
        acc = fmaf(g, st[i][k], acc);
      }
    acc = warp_sum(acc);
    dD_acc = warp_sum(dD_acc);
    __syncthreads();  // the last token's reads of the slots and reductions are done
    if (lane == 0) {
      red[warp] = acc;
      red[kBwdWarps + warp] = dD_acc;
    }
    __syncthreads();
    if (tid == 0) {
      float mT = 0.f, dD = 0.f;
      for (int w = 0; w < kBwdWarps; ++w) {
        mT += red[w];
        dD += red[kBwdWarps + w];
      }
      a.mT_bh[bh] = mT;
      a.dDf_bh[bh] = dD;
    }
  }
  return;
  }

  // ---------------- reverse sweep: G_t, dXt_t, dBt_t, fr_t, dh_init ----------------
  // G_T = dh_final
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int k = 0; k < 8; ++k)
      st[i][k] = a.dh_final && ok_pk(i, k) ? a.dh_final[state_base + (int64_t)(p0 + i) * N + n0 + k] : 0.f;
  if (TT > 0) {
    tile_fetch<T, R, RI>(a, (b * TT + TT - 1) * a.H + h, false, fa);
    tile_store<T, R, RI>(a, slot(TT - 1), false, fa, Aval);
  }
  if (TT > 1) tile_fetch<T, R, RI>(a, (b * TT + TT - 2) * a.H + h, false, fa);
  __syncthreads();
  float a_next = 1.f;  // a_{t+1} (1 past the last token)
  // token t; fcur holds token t - 1 (stored here), fnext receives token t - 2
  auto rev_tok = [&](int64_t t, TokFetch<T>& fcur, TokFetch<T>& fnext) {
    if (t > 1) tile_fetch<T, R, RI>(a, (b * TT + t - 2) * a.H + h, false, fnext);
    const float* sl = slot(t);
    const float dtv = sl[TP::ssc], av = sl[TP::ssc + 1];
    // G_t = a_{t+1} G_{t+1} + dy_t C_t^T
    {
      float ct[R][8];
#pragma unroll
      for (int q = 0; q < R; ++q)
#pragma unroll
        for (int k = 0; k < 8; ++k) ct[q][k] = sl[TP::sct + q * 128 + n0 + k];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float g[R];
#pragma unroll
        for (int q = 0; q < R; ++q) g[q] = sl[TP::sdy + (p0 + i) * R + q];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          float u = 0.f;
#pragma unroll
          for (int q = 0; q < R; ++q) u = fmaf(g[q], ct[q][k], u);
          st[i][k] = fmaf(a_next, st[i][k], u);
        }
      }
    }
    float* rb = redbuf + (int)(t & 1) * TP::red;
#pragma unroll
    for (int jb = 0; jb < NJ; ++jb) {
      // dX partials over this thread's columns: px[i JB + jj] = sum_k G[i][k] Bt[jb JB + jj][n0 + k]
      float px[VX];
#pragma unroll
      for (int e = 0; e < VX; ++e) px[e] = 0.f;
#pragma unroll
      for (int jj = 0; jj < JB; ++jj) {
        float bv[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) bv[k] = sl[TP::sbt + (jb * JB + jj) * 128 + n0 + k];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int k = 0; k < 8; ++k) px[i * JB + jj] = fmaf(st[i][k], bv[k], px[i * JB + jj]);
      }
      const int offx = reduce_scatter<VX, 3>(px, lane, 0);
      float* rx = rb + ((nbh * 16 + pb) * NJ + jb) * VX + offx;
#pragma unroll
      for (int e = 0; e < VX / 8; ++e) rx[e] = px[e];
      // dB partials over this thread's rows: pe[k JB + jj] = sum_i G[i][k] Xt[p0 + i][jb JB + jj]
      float pe[VE];
#pragma unroll
      for (int e = 0; e < VE; ++e) pe[e] = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
#pragma unroll
        for (int jj = 0; jj < JB; ++jj) {
          const float xv = sl[TP::sx + (p0 + i) * RI + jb * JB + jj];
#pragma unroll
          for (int k = 0; k < 8; ++k) pe[k * JB + jj] = fmaf(st[i][k], xv, pe[k * JB + jj]);
        }
      }
      const int offe = reduce_scatter<VE, 2>(pe, lane, 3);
      float* re = rb + TP::redx + ((pbh * 16 + nb) * NJ + jb) * VE + offe;
#pragma unroll
      for (int e = 0; e < VE / 4; ++e) re[e] = pe[e];
    }
    if (t > 0) tile_store<T, R, RI>(a, slot(t - 1), false, fcur, Aval);
    a_next = av;
    __syncthreads();
    // dXt = dt sum over the two column halves; E = sum over the four row quarters, dBt = dt E
    const int64_t row = (b * TT + t) * a.H + h;
    for (int o = tid; o < P * RI; o += kBwdThreads) {
      const int p = o / RI, j = o - p * RI;
      const int jb = j / JB, idx = (p & 3) * JB + (j - jb * JB), pbo = p >> 2;
      const float v = dtv * (rb[((0 * 16 + pbo) * NJ + jb) * VX + idx] + rb[((1 * 16 + pbo) * NJ + jb) * VX + idx]);
      if (j < R) io<T>::st(static_cast<T*>(a.dx_g) + row * P * R + (int64_t)p * R + j, v);
      else io<T>::st(static_cast<T*>(a.dx_b) + row * P * R + (int64_t)p * R + (j - R), v);
    }
    float f_acc = 0.f;
    for (int o = tid; o < N * RI; o += kBwdThreads) {
      const int n = o / RI, j = o - n * RI;
      const int jb = j / JB, idx = (n & 7) * JB + (j - jb * JB), nbo = n >> 3;
      const float* re = rb + TP::redx;
      const float v = re[((0 * 16 + nbo) * NJ + jb) * VE + idx] + re[((1 * 16 + nbo) * NJ + jb) * VE + idx] +
                      re[((2 * 16 + nbo) * NJ + jb) * VE + idx] + re[((3 * 16 + nbo) * NJ + jb) * VE + idx];
      f_acc = fmaf(sl[TP::sbt + j * 128 + n], v, f_acc);
      if (j < R) io<T>::st(static_cast<T*>(a.dB_g) + row * N * R + (int64_t)n * R + j, dtv * v);
      else io<T>::st(static_cast<T*>(a.dB_b) + row * N * R + (int64_t)n * R + (j - R), dtv * v);
    }
    f_acc = warp_sum(f_acc);
    if (lane == 0) fw[t * kBwdWarps + warp] = f_acc;
  };
  for (int64_t t = TT - 1; t >= 0; t -= 2) {
    rev_tok(t, fa, fb);
    if (t >= 1) rev_tok(t - 1, fb, fa);
  }
  // dh_init = a_0 G_0
  if (a.dh_init) {
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (ok_pk(i, k)) a.dh_init[state_base + (int64_t)(p0 + i) * N + n0 + k] = a_next * st[i][k];
  }
}

// the suffix pass after the tiled kernel's two sweeps, one CTA per (batch row, head)
__global__ void __launch_bounds__(kBwdThreads) ssd_bwd_finish_kernel(BwdParams a) {
  __shared__ float suf[kBwdThreads];
  __shared__ float red[kBwdWarps];
  const int64_t bh = blockIdx.x;
  const int64_t b = bh / a.H;
  const int h = (int)(bh - b * a.H);
  const float dD = threadIdx.x == 0 ? a.dDf_bh[bh] : 0.f;
  bwd_finish(a, bh, b, h, ldf(a.A, h, a.ad_dtype), a.mT_bh[bh], dD, a.ew + bh * a.T * kBwdWarps,
             a.fw + bh * a.T * kBwdWarps, suf, red);
}

// dA[h] = sum_b dA_bh[b, h], dD likewise, in b order
__global__ void ssd_bwd_head_sums(const float* __restrict__ dA_bh, const float* __restrict__ dD_bh,
                                  float* __restrict__ dA, float* __restrict__ dD, int64_t B, int H) {
  const int h = blockIdx.x * blockDim.x + threadIdx.x;
  if (h >= H) return;
  float sa = 0.f, sd = 0.f;
  for (int64_t b = 0; b < B; ++b) {
    sa += dA_bh[b * H + h];
    sd += dD_bh[b * H + h];
  }
  dA[h] = sa;
  dD[h] = sd;
}

struct BwdLayout {
  size_t ew, fw, dA, dD, mT, dDf, total;
};

BwdLayout bwd_layout(const m3b_ssd_bwd_args* a) {
  auto up = [](size_t x) { return (x + 255) & ~(size_t)255; };
  BwdLayout w{};
  const size_t bh = (size_t)a->batch * a->H;
  const size_t tok = bh * (size_t)a->seqlen * kBwdWarps * sizeof(float);
  w.ew = 0;
  w.fw = up(tok);
  w.dA = w.fw + up(tok);
  w.dD = w.dA + up(bh * sizeof(float));
  w.mT = w.dD + up(bh * sizeof(float));
  w.dDf = w.mT + up(bh * sizeof(float));
  w.total = w.dDf + up(bh * sizeof(float));
  return w;
}

int bvalidate(const m3b_ssd_bwd_args* a) {
  if (!a->A || !a->D || !a->dA || !a->dD) return fail(M3B_ERR_INVALID_ARG, "chunked_ssd_bwd: null pointer");
  // per-token tensors may be empty (NULL) when there are no tokens
  if (a->seqlen > 0 && (!a->x_g || !a->B_g || !a->C || !a->x_raw || !a->dt || !a->dy || !a->dx_g || !a->dB_g ||
                        !a->dC || !a->dx_raw || !a->ddt))
    return fail(M3B_ERR_INVALID_ARG, "chunked_ssd_bwd: null pointer");
  if ((a->x_b == nullptr) != (a->B_b == nullptr) || (a->x_b == nullptr) != (a->dx_b == nullptr) ||
      (a->x_b == nullptr) != (a->dB_b == nullptr))
    return fail(M3B_ERR_INVALID_ARG, "chunked_ssd_bwd: x_b, B_b, dx_b, dB_b must all be given or all be NULL");
  if (a->batch < 0 || a->seqlen < 0 || a->H <= 0 || a->P <= 0 || a->N <= 0 || a->R <= 0)
    return fail(M3B_ERR_INVALID_ARG, "chunked_ssd_bwd: bad dims");
  if (a->P > 256 || a->N > 256 || a->R > kMaxRI / 2)
    return fail(M3B_ERR_UNSUPPORTED, "chunked_ssd_bwd: needs P <= 256, N <= 256, R <= 8");
  if (a->dtype != M3B_BF16 && a->dtype != M3B_F32) return fail(M3B_ERR_UNSUPPORTED, "chunked_ssd_bwd: dtype");
  if (a->dt_dtype != M3B_F32 && a->dt_dtype != M3B_BF16 && a->dt_dtype != M3B_F16)
    return fail(M3B_ERR_UNSUPPORTED, "chunked_ssd_bwd: dt dtype");
  if (a->batch * a->H > 0x3fffffffLL) return fail(M3B_ERR_UNSUPPORTED, "chunked_ssd_bwd: batch * H too large");
  return M3B_OK;
}

template <typename T, int R, int RI>
int launch_tiled(const BwdParams& p, unsigned grid, cudaStream_t st) {
  const int smem = TPlan<R, RI>::floats * (int)sizeof(float);
  const cudaError_t e =
      cudaFuncSetAttribute(ssd_bwd_tiled_kernel<T, R, RI>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return fail(M3B_ERR_CUDA, "chunked_ssd_bwd: %s", cudaGetErrorString(e));
  ssd_bwd_tiled_kernel<T, R, RI><<<2 * grid, kBwdThreads, smem, st>>>(p);
  const int rc = check_launch("chunked_ssd_bwd");
  if (rc != M3B_OK) return rc;
  ssd_bwd_finish_kernel<<<grid, kBwdThreads, 0, st>>>(p);
  return check_launch("chunked_ssd_bwd_finish");
}

size_t bwd_smem(const m3b_ssd_bwd_args* a) {
  const int RI = a->x_b ? 2 * a->R : a->R;
  const size_t st = ((size_t)a->P * (a->N + 1) + 3) & ~(size_t)3;
  size_t sl = 2 * (size_t)slot_floats(a->P, a->N, a->R, RI);
  if (sl < kBwdThreads) sl = kBwdThreads;  // the suffix-sum pass reuses the slots
  return (st + sl + kBwdWarps) * sizeof(float);
}

}  // namespace

}  // namespace m3b

extern "C" size_t m3b_chunked_ssd_bwd_workspace(const m3b_ssd_bwd_args* a) {
  if (!a || m3b::bvalidate(a) != M3B_OK) return 0;
  const size_t base = m3b::bwd_layout(a).total;
  return a->algo == 0 && m3b::bwd_tc_ok(a) ? base + m3b::bwd_tc_workspace(a) : base;
}

extern "C" int m3b_chunked_ssd_bwd(const m3b_ssd_bwd_args* a, void* ws, size_t ws_bytes, void* stream) {
  using namespace m3b;
  clear_error();
  if (!a) return fail(M3B_ERR_INVALID_ARG, "chunked_ssd_bwd: null args");
  int rc = bvalidate(a);
  if (rc != M3B_OK) return rc;
  if (a->batch == 0) {  // no tokens: the per-head gradients are zero, not left unwritten
    const cudaStream_t st0 = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaSuccess;
    if (a->dA) e = cudaMemsetAsync(a->dA, 0, sizeof(float) * (size_t)a->H, st0);
    if (e == cudaSuccess && a->dD) e = cudaMemsetAsync(a->dD, 0, sizeof(float) * (size_t)a->H, st0);
    if (e != cudaSuccess) return fail(M3B_ERR_CUDA, "chunked_ssd_bwd: %s", cudaGetErrorString(e));
    return M3B_OK;
  }
  const BwdLayout w = bwd_layout(a);
  const bool tc = a->algo == 0 && bwd_tc_ok(a);
  const size_t need = tc ? w.total + bwd_tc_workspace(a) : w.total;
  if (!ws || ws_bytes < need) return fail(M3B_ERR_WORKSPACE, "chunked_ssd_bwd: need %zu workspace bytes", need);
  if (a->algo != 0 && a->algo != 1) return fail(M3B_ERR_INVALID_ARG, "chunked_ssd_bwd: algo %d", a->algo);
  const bool tiled = a->P <= 64 && a->N <= 128 && (a->R == 1 || a->R == 2 || a->R == 4);
  const size_t smem = tiled ? 0 : bwd_smem(a);
  if (smem > 227 * 1024) return fail(M3B_ERR_UNSUPPORTED, "chunked_ssd_bwd: state too large for shared memory");
  uint8_t* base = static_cast<uint8_t*>(ws);
  BwdParams p{};
  p.B = a->batch;
  p.T = a->seqlen;
  p.H = a->H;
  p.P = a->P;
  p.N = a->N;
  p.R = a->R;
  p.RI = a->x_b ? 2 * a->R : a->R;
  p.x_g = a->x_g;
  p.x_b = a->x_b;
  p.B_g = a->B_g;
  p.B_b = a->B_b;
  p.C = a->C;
  p.x_raw = a->x_raw;
  p.dt = a->dt;
  p.A = a->A;
  p.D = a->D;
  p.dy = a->dy;
  p.dt_dtype = a->dt_dtype;
  p.ad_dtype = a->ad_dtype;
  p.h_init = a->h_init;
  p.dh_final = a->dh_final;
  p.dx_g = a->dx_g;
  p.dx_b = a->dx_b;
  p.dB_g = a->dB_g;
  p.dB_b = a->dB_b;
  p.dC = a->dC;
  p.dx_raw = a->dx_raw;
  p.ddt = a->ddt;
  p.dh_init = a->dh_init;
  p.ew = reinterpret_cast<float*>(base + w.ew);
  p.fw = reinterpret_cast<float*>(base + w.fw);
  p.dA_bh = reinterpret_cast<float*>(base + w.dA);
  p.dD_bh = reinterpret_cast<float*>(base + w.dD);
  p.mT_bh = reinterpret_cast<float*>(base + w.mT);
  p.dDf_bh = reinterpret_cast<float*>(base + w.dDf);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned grid = (unsigned)(a->batch * a->H);
  if (tc) {
    // chunk-level products on tensor cores, then the same suffix pass on their per-token partials
    if ((rc = bwd_tc_run(a, base + w.total, p.fw, p.ew, p.mT_bh, p.dDf_bh, st)) != M3B_OK) return rc;
    ssd_bwd_finish_kernel<<<grid, kBwdThreads, 0, st>>>(p);
    if ((rc = check_launch("chunked_ssd_bwd_finish")) != M3B_OK) return rc;
  } else if (tiled) {
    const bool f32 = a->dtype == M3B_F32, beta = a->x_b != nullptr;
    switch (a->R * 2 + (beta ? 1 : 0)) {
      case 2: rc = f32 ? launch_tiled<float, 1, 1>(p, grid, st) : launch_tiled<__nv_bfloat16, 1, 1>(p, grid, st); break;
      case 3: rc = f32 ? launch_tiled<float, 1, 2>(p, grid, st) : launch_tiled<__nv_bfloat16, 1, 2>(p, grid, st); break;
      case 4: rc = f32 ? launch_tiled<float, 2, 2>(p, grid, st) : launch_tiled<__nv_bfloat16, 2, 2>(p, grid, st); break;
      case 5: rc = f32 ? launch_tiled<float, 2, 4>(p, grid, st) : launch_tiled<__nv_bfloat16, 2, 4>(p, grid, st); break;
      case 8: rc = f32 ? launch_tiled<float, 4, 4>(p, grid, st) : launch_tiled<__nv_bfloat16, 4, 4>(p, grid, st); break;
      default: rc = f32 ? launch_tiled<float, 4, 8>(p, grid, st) : launch_tiled<__nv_bfloat16, 4, 8>(p, grid, st); break;
    }
    if (rc != M3B_OK) return rc;
  } else if (a->dtype == M3B_F32) {
    cudaFuncSetAttribute(ssd_bwd_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    ssd_bwd_kernel<float><<<grid, kBwdThreads, smem, st>>>(p);
  } else {
    cudaFuncSetAttribute(ssd_bwd_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    ssd_bwd_kernel<__nv_bfloat16><<<grid, kBwdThreads, smem, st>>>(p);
  }
  if ((rc = check_launch("chunked_ssd_bwd")) != M3B_OK) return rc;
  ssd_bwd_head_sums<<<(a->H + 127) / 128, 128, 0, st>>>(p.dA_bh, p.dD_bh, a->dA, a->dD, a->batch, a->H);
  return check_launch("chunked_ssd_bwd_head_sums");
}
