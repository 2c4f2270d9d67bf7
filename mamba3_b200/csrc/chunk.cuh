// Shared pieces of the chunked layer-forward kernels: launch parameters, the
// shared-memory plan of a chunk CTA and the operand producers that build the
// tensor-core tiles of one (batch, chunk, head) work item.
//
// Formulation (equivalent to mamba3/ssd.py:118-244 fed by mamba3/mamba3.py:198-232).
// Per head, with u_s = sum_r B^_s[:,r] x_r[s,:,r]^T (a rank-R P x N matrix), the
// trapezoidal recurrence h_s = dA_s h_{s-1} + gamma_s u_s + beta_s u_{s-1} folds,
// because beta_{s+1} = (1-lam_{s+1}) dt_{s+1} dA_{s+1} and dA_{s+1} is exactly the
// decay between s and s+1, into one weight per (t, s):
//     W[t,s] = exp(cum_t - cum_s) * (gamma_s + [s<t] (1-lam_{s+1}) dt_{s+1}),  s <= t
// so the intra-chunk output is  y_t = sum_{s<=t} W[t,s] C^_t . u_s  -- rank R on
// both sides instead of the reference's rank-2R concatenation.  The beta term of
// a chunk's first token (which reads the previous chunk's last token) is carried
// by the inter-chunk state: the scan runs on H'_k = h_{chunk start} +
// (1-lam_0) dt_0 u_{-1}, whose chunk increment is
//     S'_k = sum_s w_s u_s,  w_s = exp(cum_last - cum_s) (gamma_s + (1-lam_{s+1}) dt_{s+1})
// (token L of a chunk is the next chunk's first token; zero past the sequence).
// The inter-chunk output is exp(cum_t) C^_t . H'_k and h_final = H'_K.
// Exponents are always of non-positive differences (segsum form), never the
// reference's exp(-cum) factoring (mamba3/ssd.py:44), so no chunk overflows.
//
// Internal chunk length L = 128 / RP, RP = mimo_rank rounded up to a power of 2,
// so every tile is 128 rows (t, r) x 128 columns (s, q); padded ranks, padded
// state columns (N < 128) and padded tokens (T not a multiple of L) are zeros.
#pragma once

#include "common.cuh"
#include "launch.h"

namespace m3b {

constexpr int kCT = 256;       // threads per chunk CTA
constexpr int kNS = 128;       // state dim as seen by the tiles (N <= 128, zero padded)
constexpr int kPP = 64;        // head dim as seen by the tiles (P <= 64, zero padded)
constexpr float kLog2e = 1.4426950408889634f;

struct FwdParams {
  m3b_layer_params prm;
  const void* proj;
  int64_t proj_stride;
  const void* dt_scale;      // (B,T,H) or null
  int64_t B, T;
  int K, L;
  float* rms;                // (B,T,G,2): 1/rms of B, C per token and group
  float* asum;               // (B,K,H,N/2): per-chunk sum of dt*theta
  float* omega;              // (B,K+1,H,N/2): angle before chunk k (k=K: final angle)
  const float* angle_init;   // (B,H,N/2) or null
  float* angle_final;        // (B,H,N/2) or null
  void* sstate;              // (B,K,H,P,N) chunk increments S'
  void* hstate;              // (B,K,H,P,N) scanned H'
  float* decay;              // (B,K,H)
  float* coef0;              // (B,H): (1-lam_0) dt_0 of the first token
  void* y;                   // (B,T,H*P)
  int* err;
};

struct FusedParams {
  m3b_layer_params prm;
  const void* proj;
  int64_t proj_stride;
  const void* dt_scale;
  int64_t B, T;
  int K, L;
  const float* rms;
  const float* h_init;
  const float* angle_init;
  const float* prev_bx_init;
  void* y;
  float* h_final;
  float* angle_last;  // (B,H,N/2): angle after the last token (always written)
  int* err;
  uint64_t wait_ns;   // limit of every device-side wait (the caller's, or kWaitLimitNs)
  bool state_only;    // y not needed: the kernel may skip the outputs (TMA path)
  // Sequences cut into parts of KP chunks (KP == K: whole sequences).  Part q > 0 of sequence s
  // starts from the state part q - 1 hands over: H in ho_h[s] (P x N fp32, h_final layout), the
  // angles in ho_ang[s] (64 doubles); ho_flag[2 s] / [2 s + 1] count the parts whose angles / H
  // are written (zeroed before the launch).
  int KP;
  float* ho_h;
  double* ho_ang;
  int* ho_flag;
};

// Fused sequential path (fused.cu): supported shapes and launcher.
bool fused_supported(const m3b_layer_params& p);
int launch_fused(const FusedParams& fp, cudaStream_t st, bool bf16);

__host__ __device__ constexpr int rp_of(int R) { return R <= 1 ? 1 : R <= 2 ? 2 : R <= 4 ? 4 : 8; }

// dt of token row `row`, head h: softplus(dt_raw + dt_bias) * dt_scale (mamba3/mamba3.py:200-202).
template <typename TA>
__device__ __forceinline__ float token_dt(const FwdParams& a, const TA* row, int64_t bt, int h) {
  const m3b_layer_params& p = a.prm;
  const int offDt = 2 * p.H * p.P + 2 * p.G * p.N * p.R;
  float dt = softplus_f(io<TA>::ld(row + offDt + h) + ldf(p.dt_bias, h, p.param_dtype));
  if (a.dt_scale) dt *= io<TA>::ld(reinterpret_cast<const TA*>(a.dt_scale) + bt * p.H + h);
  return dt;
}

// Shared-memory plan of one chunk CTA (byte offsets from a 1024-aligned base).  The tensor-core
// operand tiles hold bf16 for 16-bit activations (kind::f16 MMAs) and fp32 words for fp32
// activations (kind::tf32 MMAs: 10 mantissa bits instead of 7, so fp32 models keep fp32-level
// accuracy).  fp32 tiles double the tile bytes, so that variant does not stage x and z (it reads
// them from global memory, where the chunk's rows are L2-resident) and keeps the angles in the X
// tile's region until the X tile is built.
template <int RP, typename TA = __nv_bfloat16>
struct Plan {
  static constexpr int L = 128 / RP;
  static constexpr int E = (int)sizeof(TA) == 4 ? 4 : 2;  // operand tile element bytes
  static constexpr bool F32 = E == 4;
  static constexpr int XS = kPP + 4;                 // fp32 row stride of the staged x / z tiles
  static constexpr int tileC = 0;                    // 128 x 128 (K-major SW128)
  static constexpr int tileB = tileC + 128 * 128 * E;  // 128 x 128; reused for P = mask(S)
  static constexpr int tileX = tileB + 128 * 128 * E;  // 64 x 128
  static constexpr int tileH = tileX + 64 * 128 * E;   // 64 x 128
  static constexpr int xs = tileH + 64 * 128 * E;      // L x XS fp32 (bf16 tiles only)
  static constexpr int zs = xs + (F32 ? 0 : L * XS * 4);  // L x XS fp32 (bf16 tiles only)
  static constexpr int phi_own = zs + (F32 ? 0 : L * XS * 4);
  static constexpr int phi = F32 ? tileX : phi_own;  // L x 64 fp32 angles
  static constexpr int cum2 = phi_own + (F32 ? 0 : L * 64 * 4);  // (L+1) fp32: log2e * inclusive cumsum of A dt
  static constexpr int dtv = cum2 + (L + 1) * 4;     // (L+1) dt
  static constexpr int gam = dtv + (L + 1) * 4;      // (L+1) gamma
  static constexpr int bpr = gam + (L + 1) * 4;      // (L+1) (1-lam) dt
  static constexpr int wgt = bpr + (L + 1) * 4;      // L chunk-state weights
  static constexpr int rmsv = wgt + L * 4;           // L x 2
  static constexpr int nwB = rmsv + L * 8;           // N*R fp32 (B norm weight)
  static constexpr int nwC = nwB + kNS * 8 * 4;
  static constexpr int biB = nwC + kNS * 8 * 4;
  static constexpr int biC = biB + kNS * 8 * 4;
  static constexpr int mx = biC + kNS * 8 * 4;       // kPP x RP
  static constexpr int mz = mx + kPP * RP * 4;
  static constexpr int md = mz + kPP * RP * 4;
  static constexpr int bars = (md + kPP * RP * 4 + 15) & ~15;  // 4 mbarriers
  static constexpr int taddr = bars + 32;
  static constexpr int total = taddr + 16;
  static constexpr int bytes = total + 1024;         // + alignment slack
  static_assert(bytes <= 227 * 1024, "chunk CTA shared memory exceeds 227 KB");
  static_assert(L % 32 == 0, "chunk length must be a multiple of 32");
  static_assert(!F32 || L * 64 * 4 <= 64 * 128 * E, "fp32 plan: the angles fit the X tile region");
};

// fp32 -> the nearest tf32 value (10 mantissa bits, ties away from zero), as an fp32 word.  The
// tensor core reads only the upper 19 bits of a tf32 operand, i.e. it would truncate an fp32
// word; rounding first halves the error and removes its bias towards zero.
__device__ __forceinline__ uint32_t tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}

// Byte offset of fp32 element (row, col) in a K-major SW128 tile of `rows` rows (128-byte column
// blocks of 32 elements).
__device__ __forceinline__ uint32_t sw128_offset_f32(int row, int col, int rows) {
  const int cb = col >> 5, c16 = (col & 31) >> 2;
  return (uint32_t)(cb * rows * 128 + (row >> 3) * 1024 + (row & 7) * 128 + ((c16 ^ (row & 7)) << 4) +
                    ((col & 3) << 2));
}

// Store 8 consecutive fp32 values (columns [8 c8, 8 c8 + 8) of `row`) into an operand tile of
// element type TA's tile format: one 16-byte chunk of bf16, or two of tf32-rounded fp32.
template <typename TA>
__device__ __forceinline__ void tile_store8(uint8_t* tile, int row, int c8, int rows, const float (&v)[8]) {
  if constexpr (sizeof(TA) == 4) {
    sw128_store_chunk(tile, row, 2 * c8, rows, make_uint4(tf32_rna(v[0]), tf32_rna(v[1]), tf32_rna(v[2]), tf32_rna(v[3])));
    sw128_store_chunk(tile, row, 2 * c8 + 1, rows,
                      make_uint4(tf32_rna(v[4]), tf32_rna(v[5]), tf32_rna(v[6]), tf32_rna(v[7])));
  } else {
    uint4 o;
    o.x = pack_bf16x2(v[0], v[1]);
    o.y = pack_bf16x2(v[2], v[3]);
    o.z = pack_bf16x2(v[4], v[5]);
    o.w = pack_bf16x2(v[6], v[7]);
    sw128_store_chunk(tile, row, c8, rows, o);
  }
}

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// Per-token scalars of the chunk (tokens 0..L, token L = next chunk's first token):
// dt, gamma, (1-lam) dt and the log2e-scaled inclusive cumsum of A*dt.
template <typename TA, int RP>
__device__ void chunk_scalars(const FwdParams& a, uint8_t* sm, int b, int k, int h) {
  using PL = Plan<RP, TA>;
  constexpr int L = PL::L;
  const m3b_layer_params& p = a.prm;
  float* cum2 = reinterpret_cast<float*>(sm + PL::cum2);
  float* dtv = reinterpret_cast<float*>(sm + PL::dtv);
  float* gam = reinterpret_cast<float*>(sm + PL::gam);
  float* bpr = reinterpret_cast<float*>(sm + PL::bpr);
  const int64_t t0 = (int64_t)k * L;
  const TA* base = reinterpret_cast<const TA*>(a.proj) + (int64_t)b * a.T * a.proj_stride;
  const int offLam = 2 * p.H * p.P + 2 * p.G * p.N * p.R + p.H;
  const float A = -expf(ldf(p.A_log, h, p.param_dtype));
  for (int s = threadIdx.x; s <= L; s += kCT) {
    const int64_t t = t0 + s;
    float dt = 0.f, g = 0.f, bp = 0.f;
    if (t < a.T) {
      const TA* row = base + t * a.proj_stride;
      dt = token_dt<TA>(a, row, (int64_t)b * a.T + t, h);
      if (p.trapezoidal) {
        const float lam = sigmoid_f(io<TA>::ld(row + offLam + h));
        g = lam * dt;
        bp = (1.f - lam) * dt;
      } else {
        g = dt;
      }
    }
    dtv[s] = dt;
    gam[s] = g;
    bpr[s] = bp;
  }
  __syncthreads();
  // inclusive cumsum of A*dt over s < L by warp 0 (L/32 elements per lane)
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

// phi[s][i] = omega_k[i] - sum_{s'<=s} dt_s' theta_s'[i]   (mamba3/mamba3.py:160-162)
// All (s, i) products are loaded in one coalesced pass, then each i is scanned in
// nseg segments in parallel (segment totals combined in shared memory).
template <typename TA, int RP>
__device__ void chunk_angles(const FwdParams& a, uint8_t* sm, int b, int k, int h) {
  using PL = Plan<RP, TA>;
  constexpr int L = PL::L;
  const m3b_layer_params& p = a.prm;
  const int nh2 = p.N / 2;
  const float* dtv = reinterpret_cast<const float*>(sm + PL::dtv);
  float* phi = reinterpret_cast<float*>(sm + PL::phi);
  // segment totals (<= kCT floats); the H'-tile region is not in use during the prologue
  float* segtot = reinterpret_cast<float*>(sm + PL::tileH);
  const int64_t t0 = (int64_t)k * L;
  const int offTh = 2 * p.H * p.P + 2 * p.G * p.N * p.R + p.H + (p.trapezoidal ? p.H : 0);
  const TA* base = reinterpret_cast<const TA*>(a.proj) + (int64_t)b * a.T * a.proj_stride + offTh;
  const int nt = (int)((a.T - t0) < L ? (a.T - t0) : L);
  for (int e = threadIdx.x; e < L * nh2; e += kCT) {
    const int s = e / nh2, i = e - s * nh2;
    phi[s * 64 + i] = s < nt ? dtv[s] * io<TA>::ld(base + (t0 + s) * a.proj_stride + i) : 0.f;
  }
  __syncthreads();
  int nseg = 1;
  while (nseg * 2 * nh2 <= kCT && nseg * 2 <= L && nseg * 2 <= 32) nseg *= 2;
  const int seglen = L / nseg;
  const int i = threadIdx.x % nh2, seg = threadIdx.x / nh2;
  const bool act = seg < nseg;
  float run = 0.f;
  if (act) {
    for (int s = seg * seglen; s < (seg + 1) * seglen; ++s) {
      run += phi[s * 64 + i];
      phi[s * 64 + i] = run;
    }
    segtot[seg * nh2 + i] = run;
  }
  __syncthreads();
  if (act) {
    const float om = a.omega[(((int64_t)b * (a.K + 1) + k) * p.H + h) * nh2 + i];
    float off = 0.f;
    for (int q = 0; q < seg; ++q) off += segtot[q * nh2 + i];
    for (int s = seg * seglen; s < (seg + 1) * seglen; ++s) phi[s * 64 + i] = om - (off + phi[s * 64 + i]);
  }
  __syncthreads();
}

// sin/cos of an unbounded angle: Cody-Waite reduction by 2*pi (2*pi split into its fp32
// value and the fp32 remainder), then the hardware approximations on [-pi, pi].
__device__ __forceinline__ void sincos_reduced(float x, float* s, float* c) {
  const float kq = rintf(x * 0.15915494309189535f);
  float r = fmaf(-kq, 6.28318548202514648f, x);
  r = fmaf(-kq, -1.7484555314695172e-7f, r);
  __sincosf(r, s, c);
}

// Layer parameters used by the producers / epilogue, staged in fp32.
template <typename TA, int RP>
__device__ void chunk_params(const FwdParams& a, uint8_t* sm, int h, int g, bool need_z) {
  using PL = Plan<RP, TA>;
  const m3b_layer_params& p = a.prm;
  const int NR = p.N * p.R, pd = p.param_dtype;
  float* nwB = reinterpret_cast<float*>(sm + PL::nwB);
  float* nwC = reinterpret_cast<float*>(sm + PL::nwC);
  float* biB = reinterpret_cast<float*>(sm + PL::biB);
  float* biC = reinterpret_cast<float*>(sm + PL::biC);
  for (int e = threadIdx.x; e < NR; e += kCT) {
    nwB[e] = ldf(p.B_norm_w, e, pd);
    nwC[e] = ldf(p.C_norm_w, e, pd);
    biB[e] = ldf(p.B_bias, (int64_t)g * NR + e, pd);
    biC[e] = ldf(p.C_bias, (int64_t)g * NR + e, pd);
  }
  float* mx = reinterpret_cast<float*>(sm + PL::mx);
  float* mz = reinterpret_cast<float*>(sm + PL::mz);
  float* md = reinterpret_cast<float*>(sm + PL::md);
  for (int e = threadIdx.x; e < kPP * RP; e += kCT) {
    const int pp = e / RP, r = e % RP;
    float vx = 0.f, vz = 0.f, vd = 0.f;
    if (pp < p.P && r < p.R) {
      const int64_t q = ((int64_t)h * p.P + pp) * p.R + r;
      vx = ldf(p.mimo_x, q, pd);
      if (need_z) {
        vz = ldf(p.mimo_z, q, pd);
        vd = ldf(p.mimo_down, q, pd);
      }
    }
    mx[e] = vx;
    mz[e] = vz;
    md[e] = vd;
  }
}

// Stage x (and z) of the chunk's tokens for head h as fp32 [L][XS].
template <typename TA, int RP>
__device__ void chunk_stage_xz(const FwdParams& a, uint8_t* sm, int b, int k, int h, bool need_z) {
  using PL = Plan<RP, TA>;
  constexpr int L = PL::L;
  if constexpr (PL::F32) return;  // fp32 tiles read x and z from the projection where they use them
  const m3b_layer_params& p = a.prm;
  float* xs = reinterpret_cast<float*>(sm + PL::xs);
  float* zs = reinterpret_cast<float*>(sm + PL::zs);
  const int64_t t0 = (int64_t)k * L;
  const TA* base = reinterpret_cast<const TA*>(a.proj) + (int64_t)b * a.T * a.proj_stride;
  const int HP = p.H * p.P;
  const int npc = kPP / 8;
  for (int u = threadIdx.x; u < L * npc; u += kCT) {
    const int s = u / npc, pc = u % npc;
    float v[8], w[8];
    const int64_t t = t0 + s;
    if (t < a.T && pc * 8 < p.P) {
      const TA* row = base + t * a.proj_stride;
      load8<TA>(row + HP + h * p.P + pc * 8, v);
      if (need_z) load8<TA>(row + h * p.P + pc * 8, w);
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = w[e] = 0.f;
    }
    float4* xd = reinterpret_cast<float4*>(xs + s * PL::XS + pc * 8);
    xd[0] = make_float4(v[0], v[1], v[2], v[3]);
    xd[1] = make_float4(v[4], v[5], v[6], v[7]);
    if (need_z) {
      float4* zd = reinterpret_cast<float4*>(zs + s * PL::XS + pc * 8);
      zd[0] = make_float4(w[0], w[1], w[2], w[3]);
      zd[1] = make_float4(w[4], w[5], w[6], w[7]);
    }
  }
}

// Normalised (+bias), rotated B^ and/or C^ rows of the chunk into K-major tiles:
// row (s*RP + r), column n.  (mamba3/mamba3.py:151-166)
// B_T: B^ goes in transposed (row n, column s*RP + r), the K-major A operand of the chunk-state
// GEMM on fp32 tiles (kind::tf32 operands are read K-major here).
template <typename TA, int R, bool WANT_B, bool WANT_C, bool B_T = false>
__device__ void chunk_produce_bc(const FwdParams& a, uint8_t* sm, int b, int k, int g) {
  constexpr int RP = rp_of(R);
  using PL = Plan<RP, TA>;
  constexpr int L = PL::L;
  const m3b_layer_params& p = a.prm;
  const int NR = p.N * R;
  const float* nwB = reinterpret_cast<const float*>(sm + PL::nwB);
  const float* nwC = reinterpret_cast<const float*>(sm + PL::nwC);
  const float* biB = reinterpret_cast<const float*>(sm + PL::biB);
  const float* biC = reinterpret_cast<const float*>(sm + PL::biC);
  const float* rmsv = reinterpret_cast<const float*>(sm + PL::rmsv);
  const float* phi = reinterpret_cast<const float*>(sm + PL::phi);
  uint8_t* tB = sm + PL::tileB;
  uint8_t* tC = sm + PL::tileC;
  const int64_t t0 = (int64_t)k * L;
  const TA* base = reinterpret_cast<const TA*>(a.proj) + (int64_t)b * a.T * a.proj_stride;
  const int offB = 2 * p.H * p.P + g * NR;
  const int offC = 2 * p.H * p.P + p.G * NR + g * NR;
  constexpr int NC = kNS / 8;  // 16-byte column chunks per row
  for (int u = threadIdx.x; u < L * NC; u += kCT) {
    const int s = u / NC, c = u % NC;
    const int64_t t = t0 + s;
    const bool valid = (t < a.T) && (c * 8 < p.N);
    float vb[8 * R], vc[8 * R];
    if (valid) {
      const TA* row = base + t * a.proj_stride;
      const float rb = rmsv[2 * s], rc = rmsv[2 * s + 1];
      // 8 state columns x R ranks are contiguous: (n, r) at n*R + r
#pragma unroll
      for (int j = 0; j < R; ++j) {
        float tmp[8];
        if (WANT_B) {
          load8<TA>(row + offB + c * 8 * R + j * 8, tmp);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int idx = c * 8 * R + j * 8 + e;
            vb[j * 8 + e] = fmaf(tmp[e] * rb, nwB[idx], biB[idx]);
          }
        }
        if (WANT_C) {
          load8<TA>(row + offC + c * 8 * R + j * 8, tmp);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int idx = c * 8 * R + j * 8 + e;
            vc[j * 8 + e] = fmaf(tmp[e] * rc, nwC[idx], biC[idx]);
          }
        }
      }
      if (p.complex_ssm) {
#pragma unroll
        for (int pr = 0; pr < 4; ++pr) {
          float sn, cs;
          sincos_reduced(phi[s * 64 + c * 4 + pr], &sn, &cs);
#pragma unroll
          for (int r = 0; r < R; ++r) {
            const int e0 = (2 * pr) * R + r, e1 = (2 * pr + 1) * R + r;
            if (WANT_B) {
              const float b0 = vb[e0], b1 = vb[e1];
              vb[e0] = b0 * cs - b1 * sn;
              vb[e1] = b0 * sn + b1 * cs;
            }
            if (WANT_C) {
              const float c0 = vc[e0], c1 = vc[e1];
              vc[e0] = c0 * cs - c1 * sn;
              vc[e1] = c0 * sn + c1 * cs;
            }
          }
        }
      }
    }
    if constexpr (B_T) {
      static_assert(sizeof(TA) == 4 && !WANT_C, "transposed B^ tiles: fp32 state kernel only");
      // row n = 8 c + e, columns s*RP .. s*RP + RP - 1 (4, 8 or 16 aligned bytes)
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        uint32_t w[RP];
#pragma unroll
        for (int r = 0; r < RP; ++r) w[r] = (valid && r < R) ? tf32_rna(vb[e * R + (r < R ? r : 0)]) : 0u;
        uint8_t* dst = tB + sw128_offset_f32(c * 8 + e, s * RP, 128);
        if constexpr (RP == 4) *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
        else if constexpr (RP == 2) *reinterpret_cast<uint2*>(dst) = make_uint2(w[0], w[1]);
        else *reinterpret_cast<uint32_t*>(dst) = w[0];
      }
    } else {
#pragma unroll
      for (int r = 0; r < RP; ++r) {
        float ob[8], oc[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          ob[e] = (valid && r < R) ? vb[e * R + (r < R ? r : 0)] : 0.f;
          oc[e] = (valid && r < R) ? vc[e * R + (r < R ? r : 0)] : 0.f;
        }
        if (WANT_B) tile_store8<TA>(tB, s * RP + r, c, 128, ob);
        if (WANT_C) tile_store8<TA>(tC, s * RP + r, c, 128, oc);
      }
    }
  }
}

// X^T tile: row p, column (s*RP + q) = x[s,p] * mimo_x[p,q] (* w_s when WEIGHTED).  (mamba3/mamba3.py:210)
// x comes from the staged fp32 rows (bf16 tiles) or straight from the projection (fp32 tiles).
template <typename TA, int RP, bool WEIGHTED>
__device__ void chunk_produce_x(const FwdParams& a, uint8_t* sm, int b, int k, int h) {
  using PL = Plan<RP, TA>;
  constexpr int L = PL::L;
  const float* xs = reinterpret_cast<const float*>(sm + PL::xs);
  const float* mx = reinterpret_cast<const float*>(sm + PL::mx);
  const float* wgt = reinterpret_cast<const float*>(sm + PL::wgt);
  uint8_t* tX = sm + PL::tileX;
  const m3b_layer_params& p = a.prm;
  const int64_t t0 = (int64_t)k * L;
  const TA* xg = reinterpret_cast<const TA*>(a.proj) + (int64_t)b * a.T * a.proj_stride + (int64_t)p.H * p.P +
                 (int64_t)h * p.P;
  for (int u = threadIdx.x; u < kPP * 16; u += kCT) {
    const int pp = u % kPP, cc = u / kPP;
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int col = cc * 8 + e;
      const int s = col / RP, q = col % RP;
      float xv;
      if constexpr (PL::F32) {
        xv = (t0 + s < a.T && pp < p.P) ? io<TA>::ld(xg + (t0 + s) * a.proj_stride + pp) : 0.f;
      } else {
        xv = xs[s * PL::XS + pp];
      }
      float val = xv * mx[pp * RP + q];
      if (WEIGHTED) val *= wgt[s];
      v[e] = val;
    }
    tile_store8<TA>(tX, pp, cc, kPP, v);
  }
}

}  // namespace m3b
