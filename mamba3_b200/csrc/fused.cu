// Fused sequential SSD layer kernel: one persistent CTA per SM walks whole (batch, head)
// sequences chunk by chunk, so the inter-chunk state never leaves the SM.
//
// Roles (416 threads):
//   warps 0-3  epilogue: decay mask S -> P, running-state bookkeeping (TMEM <-> SMEM),
//              output y = P X + e^cum C^ H'^T + D x, gate, MIMO down, h_final
//   warps 4-11 producers: per chunk, token scalars, angle prefix + RoPE on B/C, MIMO x tiles,
//              into one of two shared-memory stages
//   warp 12    tcgen05 issue (one thread) + TMEM allocation
// Per chunk g (stage s = g % 2), with the running state H (fp32, TMEM lanes n x cols p):
//   MMA:  S  = C^ B^T                         (TMEM [0,128))
//         Yi = C^ H'_g^T   (H' bf16 tile)     (TMEM [256 + 64 (g%2), ...))
//         H += B^^T (w X)  (H already scaled by the chunk decay)   (TMEM [384,448))
//         Y  = P X         (P = mask(S))      (TMEM [128 + 64 (g%2), ...))
//   epilogue: mask(g); state(g+1): H'_{g+1} = H -> bf16 tile, H *= d_{g+1}; output(g)
// The algebra (weights W, w, the first-token beta term carried by H') is in chunk.cuh.
// Every wait is bounded; on a timeout one leader thread per role raises a shared abort flag
// that its role reads after a named barrier, so every role leaves its loop uniformly.
#include <mutex>
#include <set>
#include <utility>

#include "chunk.cuh"

namespace m3b {

constexpr int kFusedThreads = 13 * 32;
constexpr int kEpiThreads = 128;
constexpr int kProdThreads = 256;
constexpr int kMmaWarp = 12;
constexpr uint32_t kColS = 0, kColY = 128, kColYi = 256, kColH = 384;
constexpr int kBarProd = 1, kBarEpi = 2;

// Optional per-phase timestamps of CTA 0 for pipeline analysis: build with -DM3B_TIMELINE and
// read them with m3b_timeline_read(); compiled out otherwise.
#ifdef M3B_TIMELINE
__device__ unsigned long long g_m3b_timeline[64 * 16];
#define M3B_TL(g, slot)                                                              \
  do {                                                                               \
    if (blockIdx.x == 0 && (g) < 64) g_m3b_timeline[(g)*16 + (slot)] = globaltimer_ns(); \
  } while (0)
#else
#define M3B_TL(g, slot) \
  do {                  \
  } while (0)
#endif

template <int RP>
struct FPlan {
  static constexpr int L = 128 / RP;
  static constexpr int kStage = 98304;
  static constexpr int tC = 0, tB = 32768, tX = 65536, tW = 81920;  // offsets inside a stage
  static constexpr int tileH = 2 * kStage;                           // 128 rows (n) x 64 cols (p)
  static constexpr int NA = L + 1;
  static constexpr int scalStride = ((8 * NA * 4) + 15) & ~15;       // cum2 dtv gam bpr wst gb rmsB rmsC
  static constexpr int scal = tileH + 16384;
  static constexpr int omega = scal + 2 * scalStride;                // 2 x 64 doubles (by chunk parity)
  static constexpr int segt = omega + 128 * 8;                       // 256 floats
  static constexpr int nrm = segt + 256 * 4;                         // B/C norm weight, bias: 4 x N*R fp32
  static constexpr int mxs = nrm + 4 * kNS * RP * 4;                 // mimo_x: kPP x RP fp32
  static constexpr int seqp = mxs + kPP * RP * 4;                    // A, dt_bias of the producers' sequence
  static constexpr int epar = seqp + 16;                             // mimo_z, mimo_down (epilogue)
  static constexpr int bars = epar + 2 * kPP * RP * 4;               // 8 mbarriers
  static constexpr int misc = bars + 64;                             // taddr, abort
  static constexpr int bytes = misc + 16 + 1024;
  static_assert(bytes <= 227 * 1024, "fused CTA shared memory exceeds 227 KB");
};

enum { BAR_FULL0 = 0, BAR_FULL1 = 1, BAR_EMPTY0 = 2, BAR_EMPTY1 = 3, BAR_SMMA = 4, BAR_YMMA = 5, BAR_HREADY = 6,
       BAR_PREADY = 7 };

// CTA c walks sequences (batch, head) = c, c + stride, c + 2 stride, ... of nseq_total,
// each chunk by chunk; g numbers the chunks of all its sequences.
struct Sched {
  int K, H, nseq_total, stride;
  __device__ int count() const { return (nseq_total - (int)blockIdx.x + stride - 1) / stride; }
  __device__ void at(int g, int& seq, int& b, int& h, int& k) const {
    const int j = g / K;
    k = g - j * K;
    seq = (int)blockIdx.x + j * stride;
    b = seq / H;
    h = seq - b * H;
  }
};

// One leader waits on the mbarrier; the role's named barrier then releases the others.
// Returns false (for every thread of the role) once any wait of this CTA has timed out.
__device__ __forceinline__ bool role_wait(uint64_t* bar, uint32_t parity, bool leader, int bar_id, int nthreads,
                                          volatile int* abort_flag, int* err) {
  if (leader && !*abort_flag) {
    if (!mbar_wait(bar, parity)) {
      *abort_flag = 1;
      record_error(err, M3B_ERR_TIMEOUT);
    }
  }
  __syncwarp();  // the leader's lanes reconverge before the aligned barrier
  named_bar(bar_id, nthreads);
  return *abort_flag == 0;
}

// 2R consecutive activations (the (2i, 2i+1) x R block of a B or C row), kept packed in
// registers between the load and its use so a whole batch of loads can be in flight.
template <typename TA, int R>
struct PairRaw {
  static constexpr int W = sizeof(TA) == 2 ? R : 2 * R;  // 32-bit words
  uint32_t w[W];
  __device__ __forceinline__ void load(const TA* p) {
    if constexpr (W == 1) {
      w[0] = __ldg(reinterpret_cast<const unsigned int*>(p));
    } else if constexpr (W == 2) {
      const uint2 t = __ldg(reinterpret_cast<const uint2*>(p));
      w[0] = t.x;
      w[1] = t.y;
    } else {
#pragma unroll
      for (int i = 0; i < W / 4; ++i) {
        const uint4 t = __ldg(reinterpret_cast<const uint4*>(p) + i);
        w[4 * i] = t.x;
        w[4 * i + 1] = t.y;
        w[4 * i + 2] = t.z;
        w[4 * i + 3] = t.w;
      }
    }
  }
  __device__ __forceinline__ void zero() {
#pragma unroll
    for (int i = 0; i < W; ++i) w[i] = 0u;
  }
  __device__ __forceinline__ float get(int e) const {  // element e of the 2R
    if constexpr (sizeof(TA) == 2) {
      const uint32_t x = w[e >> 1];
      return __uint_as_float((e & 1) ? (x & 0xffff0000u) : (x << 16));
    } else {
      return __uint_as_float(w[e]);
    }
  }
};

// 8 consecutive activations, packed (16 B for 16-bit types, 32 B for fp32).
template <typename TA>
struct Raw8 {
  static constexpr int W = sizeof(TA) == 2 ? 4 : 8;
  uint32_t w[W];
  __device__ __forceinline__ void load(const TA* p) {
#pragma unroll
    for (int i = 0; i < W / 4; ++i) {
      const uint4 t = __ldg(reinterpret_cast<const uint4*>(p) + i);
      w[4 * i] = t.x;
      w[4 * i + 1] = t.y;
      w[4 * i + 2] = t.z;
      w[4 * i + 3] = t.w;
    }
  }
  __device__ __forceinline__ void zero() {
#pragma unroll
    for (int i = 0; i < W; ++i) w[i] = 0u;
  }
  __device__ __forceinline__ float get(int e) const {
    if constexpr (sizeof(TA) == 2) {
      const uint32_t x = w[e >> 1];
      return __uint_as_float((e & 1) ? (x & 0xffff0000u) : (x << 16));
    } else {
      return __uint_as_float(w[e]);
    }
  }
};

template <typename TA, int R>
__global__ void __launch_bounds__(kFusedThreads, 1) ssd_fused_kernel(FusedParams a, Sched sc) {
  constexpr int RP = rp_of(R);
  using PL = FPlan<RP>;
  constexpr int L = PL::L;
  constexpr int NA = PL::NA;
  constexpr int SEGMAX = L / 4;          // longest token segment of one producer thread (N/2 <= 64)
  constexpr int XU = L / 32;             // x-tile units per producer thread (L * 8 / 256)
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  const m3b_layer_params& p = a.prm;
  const int H = p.H, P = p.P, N = p.N, NR = N * R;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + PL::bars);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + PL::misc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + PL::misc + 4);
  double* omega = reinterpret_cast<double*>(sm + PL::omega);
  float* segt = reinterpret_cast<float*>(sm + PL::segt);
  const int G = sc.count() * sc.K;

  if (warp == kMmaWarp) {
    tmem_alloc(tslot, 512);
    tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(&bars[BAR_FULL0], 1);
    mbar_init(&bars[BAR_FULL1], 1);
    mbar_init(&bars[BAR_EMPTY0], kEpiThreads);
    mbar_init(&bars[BAR_EMPTY1], kEpiThreads);
    mbar_init(&bars[BAR_SMMA], 1);
    mbar_init(&bars[BAR_YMMA], 1);
    mbar_init(&bars[BAR_HREADY], 1);
    mbar_init(&bars[BAR_PREADY], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  // the operand tiles start zeroed: columns n >= N of tileC stay zero for the whole kernel
  // (tileB is rewritten by P every chunk, so the producers zero those columns per chunk)
  for (int e = tid; e < (2 * PL::kStage + 16384) / 16; e += kFusedThreads)
    reinterpret_cast<uint4*>(sm)[e] = make_uint4(0, 0, 0, 0);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;

  const TA* proj = reinterpret_cast<const TA*>(a.proj);
  const int HP = H * P;
  const int offB = 2 * HP, offC = offB + p.G * NR, offDt = offC + p.G * NR;
  const int offLam = offDt + H, offTh = offLam + (p.trapezoidal ? H : 0);

  if (warp >= 4 && warp < 12) {
    // =============================== producers ===============================
    const int ptid = tid - 128;
    const int nh2 = N / 2;
    int nseg = 1;
    while (nseg * 2 * nh2 <= kProdThreads && nseg * 2 <= L) nseg *= 2;
    const int seglen = L / nseg;  // <= SEGMAX
    const bool bc_act = ptid < nh2 * nseg;
    const int pi = ptid % nh2, seg = ptid / nh2;
    const int pc = ptid & 7;  // x-tile p-chunk
    float* nwB = reinterpret_cast<float*>(sm + PL::nrm);
    float* nwC = nwB + kNS * RP;
    float* nbB = nwC + kNS * RP;
    float* nbC = nbB + kNS * RP;
    float* mxs = reinterpret_cast<float*>(sm + PL::mxs);
    for (int g = 0; g < G; ++g) {
      const int s = g & 1;
      int seq, b, h, k;
      sc.at(g, seq, b, h, k);
      const int grp = h / (H / p.G);
      const int64_t t0 = (int64_t)k * L;
      const TA* rowbase = proj + (int64_t)b * a.T * a.proj_stride;
      if (k == 0) {  // per-sequence parameters (every producer passed the last barrier of chunk g-1)
        const int pd = p.param_dtype;
        for (int e = ptid; e < NR; e += kProdThreads) {
          nwB[e] = ldf(p.B_norm_w, e, pd);
          nwC[e] = ldf(p.C_norm_w, e, pd);
          nbB[e] = ldf(p.B_bias, (int64_t)grp * NR + e, pd);
          nbC[e] = ldf(p.C_bias, (int64_t)grp * NR + e, pd);
        }
        for (int e = ptid; e < kPP * RP; e += kProdThreads) {
          const int pp = e / RP, q = e % RP;
          mxs[e] = (pp < P && q < R) ? ldf(p.mimo_x, ((int64_t)h * P + pp) * R + q, pd) : 0.f;
        }
        if (ptid < nh2)
          omega[(g & 1) * 64 + ptid] = a.angle_init ? (double)a.angle_init[((int64_t)b * H + h) * nh2 + ptid] : 0.0;
        if (ptid == 0) {
          float* sp = reinterpret_cast<float*>(sm + PL::seqp);
          sp[0] = -expf(ldf(p.A_log, h, pd));
          sp[1] = ldf(p.dt_bias, h, pd);
        }
        named_bar(kBarProd, kProdThreads);  // the sequence's parameters are read below
      }
      if (ptid == 0) M3B_TL(g, 0);
      if (g >= 2 && !role_wait(&bars[BAR_EMPTY0 + s], ((g >> 1) - 1) & 1, ptid == 0, kBarProd, kProdThreads,
                               abort_flag, a.err))
        break;
      if (ptid == 0) M3B_TL(g, 1);
      uint8_t* st = sm + s * PL::kStage;
      float* scal = reinterpret_cast<float*>(sm + PL::scal + s * PL::scalStride);
      float* cum2 = scal;
      float* dtv = scal + NA;
      float* gam = scal + 2 * NA;
      float* bpr = scal + 3 * NA;
      float* wst = scal + 4 * NA;
      float* gbw = scal + 5 * NA;
      float* rmsB = scal + 6 * NA;
      float* rmsC = scal + 7 * NA;
      // L2 prefetch of the projection rows the next chunk reads (B|C, x, z, dt|lam|theta)
      if (g + 1 < G && ptid < 4 * L) {
        int seqn, bn, hn, kn;
        sc.at(g + 1, seqn, bn, hn, kn);
        const int64_t tn = (int64_t)kn * L + (ptid >> 2);
        if (tn < a.T) {
          const TA* row = proj + ((int64_t)bn * a.T + tn) * a.proj_stride;
          const int part = ptid & 3;
          const int esz = (int)sizeof(TA);
          if (part == 0) prefetch_l2(row + offB, (uint32_t)(2 * p.G * NR * esz) & ~15u);
          else if (part == 1) prefetch_l2(row + HP + hn * P, (uint32_t)(P * esz) & ~15u);
          else if (part == 2) prefetch_l2(row + hn * P, (uint32_t)(P * esz) & ~15u);
          else {
            const int64_t span = (int64_t)a.proj_stride - offDt;  // dt | lam | theta to the row end
            const uint32_t bytes = (uint32_t)((span * esz) & ~int64_t(15));
            if (bytes > 0 && ((offDt * esz) & 15) == 0) prefetch_l2(row + offDt, bytes < 4096u ? bytes : 4096u);
          }
        }
      }
      // (0) every global load of this chunk, issued together: x rows, theta and the B/C rows of
      // my segment, the token scalars.  One round trip covers the scalar and prefix phases.
      Raw8<TA> xr[XU];
#pragma unroll
      for (int jj = 0; jj < XU; ++jj) {
        const int j = (ptid + kProdThreads * jj) >> 3;
        const int64_t t = t0 + j;
        if (t < a.T && pc * 8 < P) xr[jj].load(rowbase + t * a.proj_stride + HP + h * P + pc * 8);
        else xr[jj].zero();
      }
      const TA* thp = rowbase + offTh + pi;
      float th[SEGMAX];
#pragma unroll
      for (int jj = 0; jj < SEGMAX; ++jj) {
        const int64_t t = t0 + seg * seglen + jj;
        th[jj] = (bc_act && p.complex_ssm && jj < seglen && t < a.T) ? io<TA>::ld(thp + t * a.proj_stride) : 0.f;
      }
      const TA* pB = rowbase + offB + grp * NR + 2 * pi * R;
      const TA* pC = rowbase + offC + grp * NR + 2 * pi * R;
      PairRaw<TA, R> vb[SEGMAX], vc[SEGMAX];
#pragma unroll
      for (int jj = 0; jj < SEGMAX; ++jj) {
        const int64_t t = t0 + seg * seglen + jj;
        if (bc_act && jj < seglen && t < a.T) {
          vb[jj].load(pB + t * a.proj_stride);
          vc[jj].load(pC + t * a.proj_stride);
        } else {
          vb[jj].zero();
          vc[jj].zero();
        }
      }
      float dt_raw = 0.f, lam_raw = 0.f, rb = 0.f, rc = 0.f;
      const bool tok_act = ptid <= L && t0 + ptid < a.T;
      if (tok_act) {
        const TA* row = rowbase + (t0 + ptid) * a.proj_stride;
        dt_raw = io<TA>::ld(row + offDt + h);
        if (p.trapezoidal) lam_raw = io<TA>::ld(row + offLam + h);
        if (ptid < L) {
          const float* rr = a.rms + (((int64_t)b * a.T + t0 + ptid) * p.G + grp) * 2;
          rb = rr[0];
          rc = rr[1];
        }
      }
      // (1) token scalars (token L is the next chunk's first token)
      if (ptid <= L) {
        float dt = 0.f, gmm = 0.f, bp = 0.f;
        if (tok_act) {
          dt = softplus_f(dt_raw + reinterpret_cast<const float*>(sm + PL::seqp)[1]);
          if (a.dt_scale)
            dt *= io<TA>::ld(reinterpret_cast<const TA*>(a.dt_scale) + ((int64_t)b * a.T + t0 + ptid) * H + h);
          if (p.trapezoidal) {
            const float lam = sigmoid_f(lam_raw);
            gmm = lam * dt;
            bp = (1.f - lam) * dt;
          } else {
            gmm = dt;
          }
        }
        dtv[ptid] = dt;
        gam[ptid] = gmm;
        bpr[ptid] = bp;
        if (ptid < L) {
          rmsB[ptid] = rb;
          rmsC[ptid] = rc;
        }
      }
      named_bar(kBarProd, kProdThreads);
      if (ptid == 0) M3B_TL(g, 2);
      if (ptid < 32) {
        constexpr int PER = L / 32;
        const float A = reinterpret_cast<const float*>(sm + PL::seqp)[0];
        float v[PER];
        float run = 0.f;
#pragma unroll
        for (int e = 0; e < PER; ++e) {
          run += A * dtv[ptid * PER + e];
          v[e] = run;
        }
        float incl = run;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const float nb = __shfl_up_sync(0xffffffffu, incl, o);
          if (ptid >= o) incl += nb;
        }
        const float excl = incl - run;
#pragma unroll
        for (int e = 0; e < PER; ++e) cum2[ptid * PER + e] = (v[e] + excl) * kLog2e;
      }
      // (2a) sum of dt * theta over my segment (dtv is visible: barrier above)
      float segsum = 0.f;
#pragma unroll
      for (int jj = 0; jj < SEGMAX; ++jj)
        if (jj < seglen) segsum = fmaf(dtv[seg * seglen + jj], th[jj], segsum);
      if (bc_act) segt[seg * nh2 + pi] = segsum;
      named_bar(kBarProd, kProdThreads);
      if (ptid < L) {
        const float gw = gam[ptid] + bpr[ptid + 1];
        gbw[ptid] = gw;
        wst[ptid] = exp2f(cum2[L - 1] - cum2[ptid]) * gw;
      }
      // (2b) rotated, normalised B^ / C^ entries of pair i for the tokens of my segment
      if (bc_act) {
        float off = 0.f;
        for (int q = 0; q < seg; ++q) off += segt[q * nh2 + pi];
        const double om = omega[(g & 1) * 64 + pi];
        float run = off;
        float wb0[RP], wb1[RP], bb0[RP], bb1[RP], wc0[RP], wc1[RP], bc0[RP], bc1[RP];
#pragma unroll
        for (int r = 0; r < RP; ++r) {
          const int i0 = 2 * pi * R + (r < R ? r : 0), i1 = i0 + R;  // flat (n, r) of n = 2i, 2i+1
          wb0[r] = nwB[i0];
          wb1[r] = nwB[i1];
          bb0[r] = nbB[i0];
          bb1[r] = nbB[i1];
          wc0[r] = nwC[i0];
          wc1[r] = nwC[i1];
          bc0[r] = nbC[i0];
          bc1[r] = nbC[i1];
        }
#pragma unroll
        for (int jj = 0; jj < SEGMAX; ++jj) {
          if (jj >= seglen) break;
          const int j = seg * seglen + jj;
          const bool valid = t0 + j < a.T;
          float cs = 1.f, sn = 0.f;
          if (p.complex_ssm) {
            run = fmaf(dtv[j], th[jj], run);
            sincos_reduced((float)(om - (double)run), &sn, &cs);
          }
          const float rbj = rmsB[j], rcj = rmsC[j];
          if (ptid == 0 && jj == 4) M3B_TL(g, 15);
#pragma unroll
          for (int r = 0; r < RP; ++r) {
            uint32_t ob = 0, oc = 0;
            if (r < R && valid) {
              const float b0 = fmaf(vb[jj].get(r) * rbj, wb0[r], bb0[r]);
              const float b1 = fmaf(vb[jj].get(R + r) * rbj, wb1[r], bb1[r]);
              const float c0 = fmaf(vc[jj].get(r) * rcj, wc0[r], bc0[r]);
              const float c1 = fmaf(vc[jj].get(R + r) * rcj, wc1[r], bc1[r]);
              ob = pack_bf16x2(b0 * cs - b1 * sn, b0 * sn + b1 * cs);
              oc = pack_bf16x2(c0 * cs - c1 * sn, c0 * sn + c1 * cs);
            }
            const uint32_t o = sw128_offset(j * RP + r, 2 * pi, 128);
            *reinterpret_cast<uint32_t*>(st + PL::tB + o) = ob;
            *reinterpret_cast<uint32_t*>(st + PL::tC + o) = oc;
          }
        }
        if (seg == nseg - 1) {
          // angle after this chunk = before - (off + own segment sum); the next chunk reads the other slot
          const double nom = p.complex_ssm ? om - (double)(off + segsum) : om;
          omega[((g + 1) & 1) * 64 + pi] = nom;
          if (k == sc.K - 1) a.angle_last[((int64_t)b * H + h) * nh2 + pi] = (float)nom;
        }
      }
      if (N < kNS) {  // zero columns [N, 128) of the B tile (P of an earlier chunk lives there)
        const int c0 = N / 8;
        const int ncz = kNS / 8 - c0;
        for (int u = ptid; u < 128 * ncz; u += kProdThreads)
          sw128_store_chunk(st + PL::tB, u / ncz, c0 + u % ncz, 128, make_uint4(0, 0, 0, 0));
      }
      if (ptid == 0) M3B_TL(g, 3);
      named_bar(kBarProd, kProdThreads);  // wst ready
      // (3) X and w X tiles from the prefetched x rows: row (s*RP + q), column p
#pragma unroll
      for (int jj = 0; jj < XU; ++jj) {
        const int j = (ptid + kProdThreads * jj) >> 3;
        const float w = wst[j];
#pragma unroll
        for (int q = 0; q < RP; ++q) {
          float v[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) v[e] = xr[jj].get(e) * mxs[(pc * 8 + e) * RP + q];
          uint4 o1, o2;
          o1.x = pack_bf16x2(v[0], v[1]);
          o1.y = pack_bf16x2(v[2], v[3]);
          o1.z = pack_bf16x2(v[4], v[5]);
          o1.w = pack_bf16x2(v[6], v[7]);
          o2.x = pack_bf16x2(v[0] * w, v[1] * w);
          o2.y = pack_bf16x2(v[2] * w, v[3] * w);
          o2.z = pack_bf16x2(v[4] * w, v[5] * w);
          o2.w = pack_bf16x2(v[6] * w, v[7] * w);
          sw128_store_chunk(st + PL::tX, j * RP + q, pc, 128, o1);
          sw128_store_chunk(st + PL::tW, j * RP + q, pc, 128, o2);
        }
      }
      fence_async_smem();
      named_bar(kBarProd, kProdThreads);
      if (ptid == 0) mbar_arrive(&bars[BAR_FULL0 + s]);
      if (ptid == 0) M3B_TL(g, 4);
    }
  } else if (warp == kMmaWarp) {
    // =============================== MMA issue ===============================
    if (lane == 0) {
      constexpr uint32_t idS = idesc_bf16(128, 128, false, false);
      constexpr uint32_t idYi = idesc_bf16(128, kPP, false, true);
      constexpr uint32_t idH = idesc_bf16(128, kPP, true, true);
      constexpr uint32_t idY = idesc_bf16(128, kPP, false, true);
      uint8_t* tileH = sm + PL::tileH;
      for (int g = 0; g < G; ++g) {
        const int s = g & 1;
        uint8_t* st = sm + s * PL::kStage;
        if (*abort_flag) break;
        if (!mbar_wait(&bars[BAR_FULL0 + s], (g >> 1) & 1)) {
          *abort_flag = 1;
          record_error(a.err, M3B_ERR_TIMEOUT);
          break;
        }
        tc_fence_after();
        M3B_TL(g, 5);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_bf16(tbase + kColS, kmajor_desc(st + PL::tC, 128, kk * 16), kmajor_desc(st + PL::tB, 128, kk * 16),
                    idS, kk > 0 ? 1u : 0u);
        if (!mbar_wait(&bars[BAR_HREADY], g & 1)) {
          *abort_flag = 1;
          record_error(a.err, M3B_ERR_TIMEOUT);
          break;
        }
        tc_fence_after();
        M3B_TL(g, 6);
        const uint32_t cyi = kColYi + 64 * (g & 1);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_bf16(tbase + cyi, kmajor_desc(st + PL::tC, 128, kk * 16), mnmajor_desc(tileH, 128, kk * 16), idYi,
                    kk > 0 ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_bf16(tbase + kColH, mnmajor_desc(st + PL::tB, 128, kk * 16), mnmajor_desc(st + PL::tW, 128, kk * 16),
                    idH, 1u);
        umma_commit(&bars[BAR_SMMA]);
        if (!mbar_wait(&bars[BAR_PREADY], g & 1)) {
          *abort_flag = 1;
          record_error(a.err, M3B_ERR_TIMEOUT);
          break;
        }
        tc_fence_after();
        M3B_TL(g, 7);
        const uint32_t cy = kColY + 64 * (g & 1);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_bf16(tbase + cy, kmajor_desc(st + PL::tB, 128, kk * 16), mnmajor_desc(st + PL::tX, 128, kk * 16), idY,
                    kk > 0 ? 1u : 0u);
        umma_commit(&bars[BAR_YMMA]);
      }
    }
    __syncwarp();  // reconverge before the CTA-wide barrier below
  } else if (warp < 4) {
    // =============================== epilogue ===============================
    const int m = tid;  // TMEM lane = tile row (t, r)
    const int t = m / RP, r = m % RP;
    const uint32_t trow = tbase + ((uint32_t)(32 * warp) << 16);
    uint8_t* tileH = sm + PL::tileH;
    float* emz = reinterpret_cast<float*>(sm + PL::epar);  // mimo_z, mimo_down of the current sequence
    float* emd = emz + kPP * RP;
    const bool lead = m == 0;
    // H'_0 of the sequence starting at chunk gs -> bf16 tile row n = m, and H = d * H'_0 in TMEM
    auto state_init = [&](int gs) -> bool {
      int seq, b, h, k;
      sc.at(gs, seq, b, h, k);
      const int s2 = gs & 1;
      if (!role_wait(&bars[BAR_FULL0 + s2], (gs >> 1) & 1, lead, kBarEpi, kEpiThreads, abort_flag, a.err))
        return false;
      const float* scal = reinterpret_cast<const float*>(sm + PL::scal + s2 * PL::scalStride);
      const float d = exp2f(scal[L - 1]);
      const float c0 = scal[3 * NA];  // (1-lam_0) dt_0
      const int64_t base = ((int64_t)b * H + h) * (int64_t)P * N;
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        float hv[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int pp = 32 * hf + e;
          float v = 0.f;
          if (m < N && pp < P) {
            if (a.h_init) v = a.h_init[base + (int64_t)pp * N + m];
            if (a.prev_bx_init) v = fmaf(c0, a.prev_bx_init[base + (int64_t)pp * N + m], v);
          }
          hv[e] = v;
        }
#pragma unroll
        for (int c8 = 0; c8 < 4; ++c8) {
          uint4 o;
          o.x = pack_bf16x2(hv[8 * c8 + 0], hv[8 * c8 + 1]);
          o.y = pack_bf16x2(hv[8 * c8 + 2], hv[8 * c8 + 3]);
          o.z = pack_bf16x2(hv[8 * c8 + 4], hv[8 * c8 + 5]);
          o.w = pack_bf16x2(hv[8 * c8 + 6], hv[8 * c8 + 7]);
          sw128_store_chunk(tileH, m, 4 * hf + c8, 128, o);
        }
#pragma unroll
        for (int e = 0; e < 32; ++e) hv[e] *= d;
        tmem_st32(trow + kColH + 32 * hf, hv);
      }
      // this sequence's gate parameters (the previous sequence's last output is complete)
      const int pd = p.param_dtype;
      for (int e = m; e < kPP * RP; e += kEpiThreads) {
        const int pp = e / RP, q = e % RP;
        const bool okp = pp < P && q < R;
        emz[e] = okp ? ldf(p.mimo_z, ((int64_t)h * P + pp) * R + q, pd) : 0.f;
        emd[e] = okp ? ldf(p.mimo_down, ((int64_t)h * P + pp) * R + q, pd) : 0.f;
      }
      return true;
    };
    auto write_h_final = [&](int glast) {
      if (!a.h_final) return;
      int seq, b, h, k;
      sc.at(glast, seq, b, h, k);
      const int64_t base = ((int64_t)b * H + h) * (int64_t)P * N;
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        float v[32];
        tmem_ld32(trow + kColH + 32 * hf, v);
        if (m < N) {
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const int pp = 32 * hf + e;
            if (pp < P) a.h_final[base + (int64_t)pp * N + m] = v[e];
          }
        }
      }
    };
    bool ok = G > 0 && state_init(0);
    if (ok) {
      fence_async_smem();
      tc_fence_before();
      named_bar(kBarEpi, kEpiThreads);
      if (lead) mbar_arrive(&bars[BAR_HREADY]);
    }
    for (int g = 0; ok && g < G; ++g) {
      const int s = g & 1;
      int seq, b, h, k;
      sc.at(g, seq, b, h, k);
      uint8_t* st = sm + s * PL::kStage;
      const float* scal = reinterpret_cast<const float*>(sm + PL::scal + s * PL::scalStride);
      const float* cum2 = scal;
      const float* gam = scal + 2 * NA;
      const float* gbw = scal + 5 * NA;
      // z of this chunk's row (t, r), prefetched while the tensor core works
      const int64_t tok = (int64_t)k * L + t;
      const bool row_ok = tok < a.T && r < R;
      Raw8<TA> zr[8];
      {
        const TA* zrow = proj + ((int64_t)b * a.T + (tok < a.T ? tok : 0)) * a.proj_stride + (int64_t)h * P;
#pragma unroll
        for (int c8 = 0; c8 < 8; ++c8) {
          if (row_ok && c8 * 8 < P) zr[c8].load(zrow + c8 * 8);
          else zr[c8].zero();
        }
      }
      if (!(ok = role_wait(&bars[BAR_SMMA], g & 1, lead, kBarEpi, kEpiThreads, abort_flag, a.err))) break;
      tc_fence_after();
      if (lead) M3B_TL(g, 8);
      // ---- mask: P[m, (s,q)] = S * exp(cum_t - cum_s) * (s<t ? gamma_s + (1-lam_{s+1})dt_{s+1} : gamma_s)
      {
        const float ct = cum2[t];
#pragma unroll
        for (int c32 = 0; c32 < 4; ++c32) {
          float v[32];
          tmem_ld32(trow + kColS + 32 * c32, v);
          if (lead && c32 == 0) M3B_TL(g, 13);
#pragma unroll
          for (int jj = 0; jj < 32; jj += RP) {
            const int sj = (32 * c32 + jj) / RP;
            const float e = ex2_fast(fminf(ct - cum2[sj], 0.f));
            const float w = sj < t ? e * gbw[sj] : (sj == t ? gam[sj] : 0.f);
#pragma unroll
            for (int q = 0; q < RP; ++q) v[jj + q] *= w;
          }
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) {
            uint4 o;
            o.x = pack_bf16x2(v[8 * cc + 0], v[8 * cc + 1]);
            o.y = pack_bf16x2(v[8 * cc + 2], v[8 * cc + 3]);
            o.z = pack_bf16x2(v[8 * cc + 4], v[8 * cc + 5]);
            o.w = pack_bf16x2(v[8 * cc + 6], v[8 * cc + 7]);
            sw128_store_chunk(st + PL::tB, m, 4 * c32 + cc, 128, o);
          }
          if (lead && c32 == 0) M3B_TL(g, 14);
        }
      }
      fence_async_smem();
      tc_fence_before();
      named_bar(kBarEpi, kEpiThreads);
      if (lead) mbar_arrive(&bars[BAR_PREADY]);
      if (lead) M3B_TL(g, 9);
      // ---- output of chunk g (x_r comes from the X tile of this stage)
      if (!(ok = role_wait(&bars[BAR_YMMA], g & 1, lead, kBarEpi, kEpiThreads, abort_flag, a.err))) break;
      tc_fence_after();
      if (lead) M3B_TL(g, 10);
      {
        const float ec = exp2f(cum2[t]);
        const float Dh = ldf(p.D, h, p.param_dtype);
        TA* yo = reinterpret_cast<TA*>(a.y) + ((int64_t)b * a.T + tok) * HP + (int64_t)h * P;
        const uint32_t cy = kColY + 64 * (g & 1), cyi = kColYi + 64 * (g & 1);
#pragma unroll
        for (int qq = 0; qq < 4; ++qq) {
          float Y[16], Yi[16];
          tmem_ld16(trow + cy + 16 * qq, Y);
          tmem_ld16(trow + cyi + 16 * qq, Yi);
          float acc[16];
#pragma unroll
          for (int hc = 0; hc < 2; ++hc) {
            const int c8 = 2 * qq + hc;
            const uint4 xq = *reinterpret_cast<const uint4*>(st + PL::tX + sw128_offset(m, c8 * 8, 128));
            const uint32_t xw[4] = {xq.x, xq.y, xq.z, xq.w};
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const int pp = c8 * 8 + e;
              const float xr = __uint_as_float((e & 1) ? (xw[e >> 1] & 0xffff0000u) : (xw[e >> 1] << 16));
              const float zz = zr[c8].get(e) * emz[pp * RP + r];
              acc[8 * hc + e] = (Y[8 * hc + e] + ec * Yi[8 * hc + e] + Dh * xr) * silu_fast(zz) * emd[pp * RP + r];
            }
          }
#pragma unroll
          for (int o = 1; o < RP; o <<= 1) {
#pragma unroll
            for (int e = 0; e < 16; ++e) acc[e] += __shfl_xor_sync(0xffffffffu, acc[e], o);
          }
          if (tok < a.T) {
            constexpr int W = 16 / RP;  // outputs written by each of the RP lanes of a token
#pragma unroll
            for (int rr = 0; rr < RP; ++rr) {
              if (rr != r) continue;
              const int p0 = 16 * qq + rr * W;
              if constexpr (W == 16) {
                if (p0 + 16 <= P) {
                  float o8[8];
#pragma unroll
                  for (int e = 0; e < 8; ++e) o8[e] = acc[e];
                  store8<TA>(yo + p0, o8);
#pragma unroll
                  for (int e = 0; e < 8; ++e) o8[e] = acc[8 + e];
                  store8<TA>(yo + p0 + 8, o8);
                  continue;
                }
              } else if constexpr (W == 8) {
                if (p0 + 8 <= P) {
                  float o8[8];
#pragma unroll
                  for (int e = 0; e < 8; ++e) o8[e] = acc[rr * W + e];
                  store8<TA>(yo + p0, o8);
                  continue;
                }
              }
#pragma unroll
              for (int e = 0; e < W; ++e)
                if (p0 + e < P) io<TA>::st(yo + p0 + e, acc[rr * W + e]);
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&bars[BAR_EMPTY0 + s]);
      if (lead) M3B_TL(g, 11);
      // ---- state for chunk g+1: H'_{g+1} -> bf16 tile, H *= d_{g+1}
      if (g + 1 < G) {
        int seq1, b1, h1, k1;
        sc.at(g + 1, seq1, b1, h1, k1);
        if (k1 == 0) {
          write_h_final(g);
          if (!(ok = state_init(g + 1))) break;
        } else {
          const int s1 = (g + 1) & 1;
          if (!(ok = role_wait(&bars[BAR_FULL0 + s1], ((g + 1) >> 1) & 1, lead, kBarEpi, kEpiThreads, abort_flag,
                               a.err)))
            break;
          const float* scal1 = reinterpret_cast<const float*>(sm + PL::scal + s1 * PL::scalStride);
          const float d = exp2f(scal1[L - 1]);
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {
            float v[32];
            tmem_ld32(trow + kColH + 32 * hf, v);
#pragma unroll
            for (int c8 = 0; c8 < 4; ++c8) {
              uint4 o;
              o.x = pack_bf16x2(v[8 * c8 + 0], v[8 * c8 + 1]);
              o.y = pack_bf16x2(v[8 * c8 + 2], v[8 * c8 + 3]);
              o.z = pack_bf16x2(v[8 * c8 + 4], v[8 * c8 + 5]);
              o.w = pack_bf16x2(v[8 * c8 + 6], v[8 * c8 + 7]);
              sw128_store_chunk(tileH, m, 4 * hf + c8, 128, o);
            }
#pragma unroll
            for (int e = 0; e < 32; ++e) v[e] *= d;
            tmem_st32(trow + kColH + 32 * hf, v);
          }
        }
        fence_async_smem();
        tc_fence_before();
        named_bar(kBarEpi, kEpiThreads);
        if (lead) mbar_arrive(&bars[BAR_HREADY]);
        if (lead) M3B_TL(g, 12);
      } else {
        write_h_final(g);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
namespace {
int ensure_smem_f(const void* kernel, int bytes) {
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

template <typename TA, int R>
int launch_fused_t(const FusedParams& fp, cudaStream_t st) {
  constexpr int RP = rp_of(R);
  using PL = FPlan<RP>;
  const int nseq_total = (int)(fp.B * fp.prm.H);
  const int nsm = num_sms();
  const int grid = nseq_total < nsm ? nseq_total : nsm;
  int rc;
  if ((rc = ensure_smem_f((const void*)ssd_fused_kernel<TA, R>, PL::bytes)) != M3B_OK) return rc;
  cudaFuncAttributes fa{};
  if (cudaFuncGetAttributes(&fa, (const void*)ssd_fused_kernel<TA, R>) == cudaSuccess &&
      fa.maxThreadsPerBlock < kFusedThreads)
    return fail(M3B_ERR_UNSUPPORTED, "ssd_fused: %d registers/thread allow only %d threads per block (need %d)",
                fa.numRegs, fa.maxThreadsPerBlock, kFusedThreads);
  const Sched sc{fp.K, fp.prm.H, nseq_total, grid};
  ssd_fused_kernel<TA, R><<<grid, kFusedThreads, PL::bytes, st>>>(fp, sc);
  return check_launch("ssd_fused");
}
}  // namespace

#ifdef M3B_TIMELINE
extern "C" M3B_API int m3b_timeline_read(unsigned long long* host, int n) {
  return cudaMemcpyFromSymbol(host, g_m3b_timeline, sizeof(unsigned long long) * (n < 1024 ? n : 1024)) ==
                 cudaSuccess
             ? 0
             : 3;
}
#endif

bool fused_supported(const m3b_layer_params& p) {
  const int nh2 = p.N / 2;
  return p.N <= kNS && p.P <= kPP && (nh2 & (nh2 - 1)) == 0 && nh2 >= 1 && (p.R == 1 || p.R == 2 || p.R == 4);
}

int launch_fused(const FusedParams& fp, cudaStream_t st, bool bf16) {
  switch (fp.prm.R) {
    case 1: return bf16 ? launch_fused_t<__nv_bfloat16, 1>(fp, st) : launch_fused_t<float, 1>(fp, st);
    case 2: return bf16 ? launch_fused_t<__nv_bfloat16, 2>(fp, st) : launch_fused_t<float, 2>(fp, st);
    case 4: return bf16 ? launch_fused_t<__nv_bfloat16, 4>(fp, st) : launch_fused_t<float, 4>(fp, st);
    default: return fail(M3B_ERR_UNSUPPORTED, "ssd_fused: mimo_rank %d", fp.prm.R);
  }
}

}  // namespace m3b
