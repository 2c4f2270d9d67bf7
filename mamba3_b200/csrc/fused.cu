// Fused sequential SSD layer kernel: one persistent CTA per SM walks whole (batch, head)
// sequences chunk by chunk, so the inter-chunk state never leaves the SM.
//
// Roles (512 threads, 128 registers each):
//   warps 0-7   epilogue (TMEM lane quadrant = warp % 4, column half = warp / 4):
//               decay mask S -> P (kept in TMEM), output y = P X + e^cum C^ H'^T + D x with gate
//               and MIMO down,
//               running-state bookkeeping (TMEM <-> bf16 tile), MIMO x tiles X and W, h_final.
//               Its leader issues the GEMMs that depend on the running state and on P, and
//               hands each shared-memory stage back to the producers (with the TMA copies of
//               the chunk two ahead) as soon as the last GEMM that reads the stage has completed,
//               before the output of that chunk is written.
//   warps 8-15  producers: per chunk, token scalars, angle prefix + RoPE + norm of B/C into one
//               of two shared-memory stages; their leader issues S = C^ B^T.
// Per chunk g (stage s = g % 2), with the running state H (fp32, TMEM lanes n x columns p):
//   producer leader:  S_g = C^ B^T                            -> TMEM S[g%2] (128 columns)
//   epilogue leader:  Yi_g = C^ H'_g^T, H += B^^T W           -> Yi, H          (after state(g))
//                     Y_g = P X, P read from TMEM             -> Y
//   epilogue:         mask(g), [stage s handed over], output(g), state(g+1): H'_{g+1} = H -> bf16
//                     tile, H *= d_{g+1}, X and W tiles of chunk g+1
// The algebra (weights W, w, the first-token beta term carried by H') is in chunk.cuh.
// Every wait is bounded.  In the chunk loops each thread waits on the GEMM / stage mbarriers
// itself (own_wait) and keeps its own timeout flag; the role ORs the flags at its next named
// barrier (barrier_or, bar.red.or), so all its threads leave the loop together.  Job starts wait
// through the role's leader and a shared abort flag read after a named barrier (role_wait).  The
// other role then times out on the mbarrier this role no longer completes, and leaves too.
#include <cuda.h>

#include <mutex>
#include <set>
#include <utility>

#include "chunk.cuh"
#include "tmap.h"

namespace m3b {

constexpr int kFusedThreads = 16 * 32;
constexpr int kEpiThreads = 256;
constexpr int kProdThreads = 256;
// TMEM columns: S[g%2] at 128 (g%2); Yi at 256; Y at 320; H at 384; the masked score tile P (bf16,
// two per column) at 448.  Yi and Y have one buffer each: a chunk's GEMMs that write them are
// issued only after the previous chunk's output has read them.
constexpr uint32_t kColS = 0, kColYi = 256, kColY = 320, kColH = 384, kColP = 448;
constexpr int kBarProd = 1, kBarEpi = 2;

// Optional per-phase timestamps of CTA 0 for pipeline analysis: build with -DM3B_TIMELINE and
// read them with m3b_timeline_read(); compiled out otherwise.
#ifdef M3B_TIMELINE
__device__ unsigned long long g_m3b_timeline[64 * 16];
#define M3B_TL(g, slot)                                                                   \
  do {                                                                                    \
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
  static constexpr int NA = (L + 1 + 3) & ~3;  // per-token scalar arrays: L + 1 entries, 16-byte rows
  static constexpr int scalStride = ((8 * NA * 4) + 15) & ~15;       // cum2 dtv gam bpr wst gb rmsB rmsC
  static constexpr int scal = tileH + 16384;
  static constexpr int omega = scal + 2 * scalStride;                // 2 x 64 doubles (by chunk parity)
  static constexpr int segt = omega + 128 * 8;                       // 256 floats
  static constexpr int nrm = segt + 256 * 4;  // B/C norm weight, bias: 4 x N*R fp32 (register path);
                                               // packed bf16 pairs, 16 B per (pair, rank pair) (TMA)
  static constexpr int mxs = nrm + 4 * kNS * RP * 4;                 // mimo_x (epilogue): kPP x RP fp32
  static_assert(RP * 64 * 16 <= 4 * kNS * RP * 4, "packed bf16 norm pairs (TMA path) fit the norm region");
  static constexpr int seqp = mxs + kPP * RP * 4;                    // A, dt_bias of the producers' sequence
  static constexpr int epar = seqp + 16;                             // mimo_z, mimo_down (epilogue)
  static constexpr int bars = epar + 2 * kPP * RP * 4;               // 9 mbarriers
  static constexpr int misc = bars + 128;                            // taddr, abort flags
  static constexpr int bytes = misc + 16 + 1024;
  static_assert(bytes <= 227 * 1024, "fused CTA shared memory exceeds 227 KB");
};

enum { BAR_FULL0 = 0, BAR_FULL1 = 1, BAR_SDONE0 = 4, BAR_SDONE1 = 5, BAR_HDONE = 6, BAR_YDONE = 7,
       BAR_STAGE0 = 8, BAR_STAGE1 = 9 };

// Position of one chunk: job, part of the sequence, sequence index, batch row, head, group,
// chunk within the sequence (k) and within the part (kk).
struct ChunkPos {
  int job, part, seq, b, h, grp, k, kk;
};

// Every sequence (batch, head) is cut into nparts parts of KP chunks (K = nparts KP); job j is
// part j / nseq_total of sequence j % nseq_total, so all first parts come before all second
// parts.  CTA c walks jobs c, c + stride, c + 2 stride, ... chunk by chunk; g numbers the chunks
// of all its jobs.  The predecessor of job j (part - 1 of the same sequence) is job j - nseq_total,
// which a CTA took in an earlier round.  The roles step a ChunkPos cursor along g (divisions
// only when a new job starts).
struct Sched {
  int K, H, nseq_total, stride, heads_per_group, KP, nparts;
  __device__ int count() const { return (nseq_total * nparts - (int)blockIdx.x + stride - 1) / stride; }
  __device__ void set_job(ChunkPos& c, int job) const {
    c.job = job;
    c.part = job / nseq_total;
    c.seq = job - c.part * nseq_total;
    c.b = c.seq / H;
    c.h = c.seq - c.b * H;
    c.grp = c.h / heads_per_group;
    c.k = c.part * KP;
    c.kk = 0;
  }
  __device__ ChunkPos first() const {
    ChunkPos c;
    set_job(c, (int)blockIdx.x);
    return c;
  }
  __device__ void advance(ChunkPos& c) const {
    if (++c.kk == KP) {
      set_job(c, c.job + stride);
    } else {
      ++c.k;
    }
  }
  __device__ ChunkPos ahead(ChunkPos c, int n) const {
    for (int i = 0; i < n; ++i) advance(c);
    return c;
  }
};

// One leader waits on the mbarrier; the role's named barrier then releases the others.
// Returns false (for every thread of the role) once any wait of this CTA has timed out.
__device__ __forceinline__ bool role_wait(uint64_t* bar, uint32_t parity, bool leader, int bar_id, int nthreads,
                                          volatile int* abort_flag, int* err, uint64_t lim) {
  if (leader && !*abort_flag) {
    if (!mbar_wait(bar, parity, lim)) {
      *abort_flag = 1;
      record_error(err, M3B_ERR_TIMEOUT);
    }
  }
  __syncwarp();  // the leader's lanes reconverge before the aligned barrier
  named_bar(bar_id, nthreads);
  return *abort_flag == 0;
}

// Every thread of a role waits on the mbarrier itself, with no role barrier after it, so each warp
// goes on as soon as the phase completes.  A timeout is kept in the thread's own `timed_out`
// (later waits are then skipped) and the role acts on it at its next barrier_or.
__device__ __forceinline__ void own_wait(uint64_t* bar, uint32_t parity, bool& timed_out, int* err, uint64_t lim) {
  if (!timed_out && !mbar_wait(bar, parity, lim)) {
    timed_out = true;
    record_error(err, M3B_ERR_TIMEOUT);
  }
}

// Named barrier that also ORs one flag over its threads (bar.red.or): every thread gets the same
// result, computed at the barrier itself.
__device__ __forceinline__ bool barrier_or(int id, int n, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred pi, po;\n\t"
      "setp.ne.u32 pi, %1, 0;\n\t"
      "bar.red.or.pred po, %2, %3, pi;\n\t"
      "selp.u32 %0, 1, 0, po;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)v), "r"(id), "r"(n)
      : "memory");
  return r != 0;
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
  __device__ __forceinline__ void load_shared(const uint8_t* p) {
    if constexpr (W == 1) {
      w[0] = *reinterpret_cast<const uint32_t*>(p);
    } else if constexpr (W == 2) {
      const uint2 t = *reinterpret_cast<const uint2*>(p);
      w[0] = t.x;
      w[1] = t.y;
    } else {
#pragma unroll
      for (int i = 0; i < W / 4; ++i) {
        const uint4 t = reinterpret_cast<const uint4*>(p)[i];
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
  // elements (e, e+1) of the 2R as a float pair (e even)
  __device__ __forceinline__ float2 pair(int e) const {
    if constexpr (sizeof(TA) == 2) return bf2_to_f2(w[e >> 1]);
    else return make_float2(__uint_as_float(w[e]), __uint_as_float(w[e + 1]));
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
  // elements (e, e+1) as a float pair (e even)
  __device__ __forceinline__ float2 pair(int e) const {
    if constexpr (sizeof(TA) == 2) return bf2_to_f2(w[e >> 1]);
    else return make_float2(__uint_as_float(w[e]), __uint_as_float(w[e + 1]));
  }
};

__device__ __forceinline__ void st_pack_chunk(uint8_t* tile, int row, int c8, const float (&v)[8]) {
  uint4 o;
  o.x = pack_bf16x2(v[0], v[1]);
  o.y = pack_bf16x2(v[2], v[3]);
  o.z = pack_bf16x2(v[4], v[5]);
  o.w = pack_bf16x2(v[6], v[7]);
  sw128_store_chunk(tile, row, c8, 128, o);
}

// TMA: bf16 activations, N = 128 and 16-byte aligned projection rows.  The raw B / C rows and
// theta of a chunk then arrive by tensor-memory-accelerator copies straight into the stage's
// B / C / W tiles, and each producer warp rewrites its tokens in place; otherwise every
// producer thread loads its raw values from global memory into registers.
// SO (state only, TMA path): the caller needs the final state but not y, so C^, S, the mask,
// P'W, C^H'^T and the output are skipped; what remains is B^, W and H += B^^T W per chunk.
template <typename TA, int R, bool TMA, bool SO>
__global__ void __launch_bounds__(kFusedThreads, 1)
    ssd_fused_kernel(FusedParams a, Sched sc, const __grid_constant__ CUtensorMap tm_bc,
                     const __grid_constant__ CUtensorMap tm_th) {
  static_assert(!TMA || sizeof(TA) == 2, "the TMA producer path stages bf16 rows");
  static_assert(!SO || TMA, "the state-only variant is built on the TMA path");
  constexpr bool N128 = TMA;
  constexpr int RP = rp_of(R);
  using PL = FPlan<RP>;
  constexpr int L = PL::L;
  constexpr int NA = PL::NA;
  constexpr int SEGMAX = L / 4;  // longest token segment of one producer thread (N/2 <= 64)
  constexpr int XU = L / 32;     // X / W tile units (8 columns of one token) per epilogue thread
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  const m3b_layer_params& p = a.prm;
  const int H = p.H, P = p.P, N = p.N, NR = N * R;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + PL::bars);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + PL::misc);
  volatile int* prod_abort = reinterpret_cast<volatile int*>(sm + PL::misc + 4);
  volatile int* epi_abort = reinterpret_cast<volatile int*>(sm + PL::misc + 8);
  double* omega = reinterpret_cast<double*>(sm + PL::omega);
  float* segt = reinterpret_cast<float*>(sm + PL::segt);
  const int G = sc.count() * sc.KP;

  if (warp == 0) {
    tmem_alloc(tslot, 512);
    tmem_relinquish();
  }
  if (tid == 32) {
    mbar_init(&bars[BAR_FULL0], 1);
    mbar_init(&bars[BAR_FULL1], 1);
    mbar_init(&bars[BAR_SDONE0], 1);
    mbar_init(&bars[BAR_SDONE1], 1);
    mbar_init(&bars[BAR_HDONE], 1);
    mbar_init(&bars[BAR_YDONE], 1);
    mbar_init(&bars[BAR_STAGE0], 1);
    mbar_init(&bars[BAR_STAGE1], 1);
    *prod_abort = 0;
    *epi_abort = 0;
    fence_mbar_init();
  }
  // the operand tiles start zeroed: columns n >= N of tileC and tileB stay zero for the whole kernel
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

  // Stage gg % 2 is handed to the producers for chunk gg through STAGE[gg % 2].  On the TMA path
  // the hand-over also starts the copies of the chunk's raw B / C halves (n < 64 | n >= 64 ->
  // tile blocks 0 | 1; token j's half lands on the bytes of tile rows j*RP .. j*RP+RP-1) and of
  // theta (-> the W tile, built only after theta has been consumed), counted as transaction
  // bytes of the same phase.  The producers hand chunks 0 and 1 to themselves; the epilogue
  // leader hands chunk g + 2 over once the last GEMMs that read chunk g's stage (its state GEMMs
  // and Y = P'W; in the state-only variant the state GEMM) have completed.
  auto issue_stage = [&](const ChunkPos& c, int gg) {
    uint64_t* bar = &bars[BAR_STAGE0 + (gg & 1)];
    if constexpr (TMA) {
      uint8_t* stg = sm + (gg & 1) * PL::kStage;
      constexpr uint32_t kHalf = 16384;
      mbar_arrive_expect_tx(bar, (SO ? 2 : 4) * kHalf + (p.complex_ssm ? (uint32_t)L * 128u : 0u));
      const int xb = offB + c.grp * NR, xc = offC + c.grp * NR, ti = c.k * L;
      tma_load_3d(stg + PL::tB, &tm_bc, xb, ti, c.b, bar);
      tma_load_3d(stg + PL::tB + kHalf, &tm_bc, xb + NR / 2, ti, c.b, bar);
      if constexpr (!SO) {
        tma_load_3d(stg + PL::tC, &tm_bc, xc, ti, c.b, bar);
        tma_load_3d(stg + PL::tC + kHalf, &tm_bc, xc + NR / 2, ti, c.b, bar);
      }
      if (p.complex_ssm) tma_load_3d(stg + PL::tW, &tm_th, offTh, ti, c.b, bar);
    } else {
      mbar_arrive(bar);
    }
  };

  if (warp >= 8) {
    // =============================== producers ===============================
    volatile int* abort_flag = prod_abort;
    bool ptmo = false;  // this thread's own bounded waits (own_wait) timed out
    const int ptid = tid - kEpiThreads;
    const int nh2 = N / 2;
    int nseg = 1;
    while (nseg * 2 * nh2 <= kProdThreads && nseg * 2 <= L) nseg *= 2;
    const int seglen = N128 ? SEGMAX : L / nseg;  // N = 128: nseg = 4
    const bool bc_act = ptid < nh2 * nseg;
    const int pi = ptid % nh2, seg = ptid / nh2;
    float* nwB = reinterpret_cast<float*>(sm + PL::nrm);
    float* nwC = nwB + kNS * RP;
    float* nbB = nwC + kNS * RP;
    float* nbC = nbB + kNS * RP;
    const float* sp = reinterpret_cast<const float*>(sm + PL::seqp);
    constexpr uint32_t idS = idesc_bf16(128, 128, false, false);
    ChunkPos pos = sc.first();
    if (ptid == 0) {
      if (G > 0) issue_stage(pos, 0);
      if (G > 1) issue_stage(sc.ahead(pos, 1), 1);
    }
    // raw token scalars of chunk gg for token ptid (0..L; token L is the next chunk's first),
    // loaded one chunk ahead of their use
    struct TokRaw {
      float dt, lam, rb, rc, dts;
      bool ok;
      bool pre;            // sdt / sgam / sbp below already hold the token scalars
      float sdt, sgam, sbp;
    };
    // dt = softplus(dt_raw + dt_bias) * dt_scale; gamma = lam dt; (1 - lam) dt (trapezoid)
    auto tok_scalars = [&](TokRaw& tr) {
      float dt = 0.f, gmm = 0.f, bp = 0.f;
      if (tr.ok) {
        dt = softplus_fast(tr.dt + sp[1]) * tr.dts;
        if (p.trapezoidal) {
          const float lam = sigmoid_fast(tr.lam);
          gmm = lam * dt;
          bp = (1.f - lam) * dt;
        } else {
          gmm = dt;
        }
      }
      tr.sdt = dt;
      tr.sgam = gmm;
      tr.sbp = bp;
      tr.pre = true;
    };
    auto load_tok = [&](const ChunkPos& c, TokRaw& tr) {
      const int bb = c.b, hh = c.h, gr = c.grp;
      const int64_t tt = (int64_t)c.k * L + ptid;
      tr.dt = tr.lam = tr.rb = tr.rc = 0.f;
      tr.dts = 1.f;
      tr.ok = ptid <= L && tt < a.T;
      tr.pre = false;
      if (tr.ok) {
        const TA* row = proj + ((int64_t)bb * a.T + tt) * a.proj_stride;
        tr.dt = io<TA>::ld(row + offDt + hh);
        if (p.trapezoidal) tr.lam = io<TA>::ld(row + offLam + hh);
        if (a.dt_scale) tr.dts = io<TA>::ld(reinterpret_cast<const TA*>(a.dt_scale) + ((int64_t)bb * a.T + tt) * H + hh);
        if (ptid < L) {
          const float2 rr = *reinterpret_cast<const float2*>(a.rms + (((int64_t)bb * a.T + tt) * p.G + gr) * 2);
          tr.rb = rr.x;
          tr.rc = rr.y;
        }
      }
    };
    TokRaw nxt;
    if (G > 0) load_tok(pos, nxt);
    for (int g = 0; g < G; ++g, sc.advance(pos)) {
      const int s = g & 1;
      const int b = pos.b, h = pos.h, k = pos.k, grp = pos.grp;
      const ChunkPos pnext = sc.ahead(pos, 1);
      const int64_t t0 = (int64_t)k * L;
      const TA* rowbase = proj + (int64_t)b * a.T * a.proj_stride;
      if (pos.kk == 0) {  // a new job: its sequence's parameters (every producer passed chunk g-1's last barrier)
        const int pd = p.param_dtype;
        if constexpr (TMA) {
          // the norm weights / biases of pair ptid as the packed bf16 pairs the rotation multiplies
          // with, converted once per job; quad q of pair i at 16-byte slot q * 64 + i
          if (ptid < nh2) {
            uint4* hq = reinterpret_cast<uint4*>(sm + PL::nrm) + ptid;
            const int64_t gb = (int64_t)grp * NR;
            auto pk = [&](const void* base, int64_t i) { return pack_bf16x2(ldf(base, i, pd), ldf(base, i + 1, pd)); };
            if constexpr (R % 2 == 0) {
#pragma unroll
              for (int rp = 0; rp < R / 2; ++rp) {
                const int i0 = 2 * ptid * R + 2 * rp, i1 = i0 + R;  // (n = 2i | 2i+1, ranks 2rp, 2rp+1)
                hq[(2 * rp) * 64] = make_uint4(pk(p.B_norm_w, i0), pk(p.B_norm_w, i1), pk(p.B_bias, gb + i0),
                                               pk(p.B_bias, gb + i1));
                hq[(2 * rp + 1) * 64] = make_uint4(pk(p.C_norm_w, i0), pk(p.C_norm_w, i1), pk(p.C_bias, gb + i0),
                                                   pk(p.C_bias, gb + i1));
              }
            } else {
              const int i0 = 2 * ptid;  // (n = 2i, 2i+1) of the single rank
              hq[0] = make_uint4(pk(p.B_norm_w, i0), pk(p.B_bias, gb + i0), pk(p.C_norm_w, i0), pk(p.C_bias, gb + i0));
            }
          }
        } else {
          for (int e = ptid; e < NR; e += kProdThreads) {
            nwB[e] = ldf(p.B_norm_w, e, pd);
            nwC[e] = ldf(p.C_norm_w, e, pd);
            nbB[e] = ldf(p.B_bias, (int64_t)grp * NR + e, pd);
            nbC[e] = ldf(p.C_bias, (int64_t)grp * NR + e, pd);
          }
        }
        if (pos.part == 0) {
          if (ptid < nh2)
            omega[(g & 1) * 64 + ptid] = a.angle_init ? (double)a.angle_init[((int64_t)b * H + h) * nh2 + ptid] : 0.0;
        } else {
          // the angles after the previous part of this sequence (another CTA, an earlier round)
          if (ptid == 0 && !*abort_flag && !flag_wait_geq(a.ho_flag + 2 * pos.seq, pos.part, a.wait_ns)) {
            *abort_flag = 1;
            record_error(a.err, M3B_ERR_TIMEOUT);
          }
          __syncwarp();
          named_bar(kBarProd, kProdThreads);
          if (*abort_flag) break;
          if (ptid < nh2) omega[(g & 1) * 64 + ptid] = __ldcg(a.ho_ang + (int64_t)pos.seq * 64 + ptid);
        }
        if (ptid == 0) {
          float* spw = reinterpret_cast<float*>(sm + PL::seqp);
          spw[0] = -expf(ldf(p.A_log, h, pd));
          spw[1] = ldf(p.dt_bias, h, pd);
        }
        named_bar(kBarProd, kProdThreads);  // the sequence's parameters are read below
      }
      if (ptid == 0) M3B_TL(g, 0);
      // the stage is free (and on the TMA path its raw rows have landed); every thread waits
      // itself, and a timeout is acted on at the barrier after the token scalars
      own_wait(&bars[BAR_STAGE0 + s], (g >> 1) & 1, ptmo, a.err, a.wait_ns);
      if (ptid == 0) M3B_TL(g, 1);
      uint8_t* st = sm + s * PL::kStage;
      const TokRaw cur = nxt;
      if (g + 1 < G) load_tok(pnext, nxt);
      float* scal = reinterpret_cast<float*>(sm + PL::scal + s * PL::scalStride);
      float* cum2 = scal;
      float* dtv = scal + NA;
      float* gam = scal + 2 * NA;
      float* bpr = scal + 3 * NA;
      float* wst = scal + 4 * NA;
      float* gbw = scal + 5 * NA;
      float* rmsB = scal + 6 * NA;
      float* rmsC = scal + 7 * NA;
      // register path: L2 prefetch of the projection rows the next chunk reads (the TMA path
      // starts its copies a chunk ahead, and the epilogue loads x and z ahead of use)
      if (!TMA && g + 1 < G && ptid < 4 * L) {
        const int bn = pnext.b, hn = pnext.h, kn = pnext.k;
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
      // (0) register path: the raw theta, B and C values of my segment, issued together
      constexpr int SEGR = TMA ? 1 : SEGMAX;  // register-staged tokens (the TMA path reads shared memory)
      float th[SEGR];
      PairRaw<TA, R> vb[SEGR], vc[SEGR];
      if constexpr (!TMA) {
        const TA* thp = rowbase + offTh + pi;
#pragma unroll
        for (int jj = 0; jj < SEGMAX; ++jj) {
          const int64_t t = t0 + seg * seglen + jj;
          th[jj] = (bc_act && p.complex_ssm && jj < seglen && t < a.T) ? io<TA>::ld(thp + t * a.proj_stride) : 0.f;
        }
        const TA* pB = rowbase + offB + grp * NR + 2 * pi * R;
        const TA* pC = rowbase + offC + grp * NR + 2 * pi * R;
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
      }
      // theta of (token j of the chunk, my pair) from the TMA-staged W tile
      const __nv_bfloat16* ths = reinterpret_cast<const __nv_bfloat16*>(st + PL::tW) + pi;
      auto theta = [&](int jj) -> float {
        if constexpr (TMA) return p.complex_ssm ? __bfloat162float(ths[(seg * SEGMAX + jj) * 64]) : 0.f;
        else return th[jj];
      };
      if (ptid == 0) M3B_TL(g, 5);
      // (1) token scalars (token L is the next chunk's first token); within a sequence they were
      // computed at the end of the previous chunk
      if (ptid <= L) {
        TokRaw c2 = cur;
        if (!c2.pre) tok_scalars(c2);
        dtv[ptid] = c2.sdt;
        gam[ptid] = c2.sgam;
        bpr[ptid] = c2.sbp;
        if (ptid < L) {
          rmsB[ptid] = cur.rb;
          rmsC[ptid] = cur.rc;
        }
      }
      if (ptid == 0) M3B_TL(g, 6);
      if (barrier_or(kBarProd, kProdThreads, ptmo)) {  // scalars written (or a stage wait timed out)
        *abort_flag = 1;
        break;
      }
      if (ptid == 0) M3B_TL(g, 2);
      if (ptid < 32) {
        constexpr int PER = L / 32;
        const float A = sp[0];
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
      float pre[SEGMAX];  // running dt * theta sum of my segment, per token
#pragma unroll
      for (int jj = 0; jj < SEGMAX; ++jj) {
        if (N128 || jj < seglen) segsum = fmaf(dtv[seg * seglen + jj], theta(jj), segsum);
        pre[jj] = segsum;
      }
      if (bc_act) segt[seg * nh2 + pi] = segsum;
      named_bar(kBarProd, kProdThreads);
      if (ptid == 0) M3B_TL(g, 7);
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
        const float omf = (float)om;
        float run = off;
        // norm weight / bias of (n = 2i + e, r) as r-pairs (R even) or n-pairs (R = 1)
        float2 wB0[RP / 2 + 1], wB1[RP / 2 + 1], bB0[RP / 2 + 1], bB1[RP / 2 + 1];
        float2 wC0[RP / 2 + 1], wC1[RP / 2 + 1], bC0[RP / 2 + 1], bC1[RP / 2 + 1];
        if constexpr (TMA) {
          // (packed bf16 pairs below)
        } else if constexpr (R % 2 == 0) {
#pragma unroll
          for (int rp = 0; rp < R / 2; ++rp) {
            const int i0 = 2 * pi * R + 2 * rp, i1 = i0 + R;
            wB0[rp] = make_float2(nwB[i0], nwB[i0 + 1]);
            wB1[rp] = make_float2(nwB[i1], nwB[i1 + 1]);
            bB0[rp] = make_float2(nbB[i0], nbB[i0 + 1]);
            bB1[rp] = make_float2(nbB[i1], nbB[i1 + 1]);
            wC0[rp] = make_float2(nwC[i0], nwC[i0 + 1]);
            wC1[rp] = make_float2(nwC[i1], nwC[i1 + 1]);
            bC0[rp] = make_float2(nbC[i0], nbC[i0 + 1]);
            bC1[rp] = make_float2(nbC[i1], nbC[i1 + 1]);
          }
        } else {
          wB0[0] = make_float2(nwB[2 * pi], nwB[2 * pi + 1]);
          bB0[0] = make_float2(nbB[2 * pi], nbB[2 * pi + 1]);
          wC0[0] = make_float2(nwC[2 * pi], nwC[2 * pi + 1]);
          bC0[0] = make_float2(nbC[2 * pi], nbC[2 * pi + 1]);
        }
        // TMA path (bf16 rows): norm and rotation in packed bf16 arithmetic straight on the raw
        // bf16 pairs, as the reference computes them for a bf16 model; weights / biases as pairs
        __nv_bfloat162 hwB0[RP / 2 + 1], hwB1[RP / 2 + 1], hbB0[RP / 2 + 1], hbB1[RP / 2 + 1];
        __nv_bfloat162 hwC0[RP / 2 + 1], hwC1[RP / 2 + 1], hbC0[RP / 2 + 1], hbC1[RP / 2 + 1];
        if constexpr (TMA) {
          const uint4* hq = reinterpret_cast<const uint4*>(sm + PL::nrm) + pi;
          auto h2 = [](uint32_t w) { return *reinterpret_cast<const __nv_bfloat162*>(&w); };
          if constexpr (R % 2 == 0) {
#pragma unroll
            for (int rp = 0; rp < R / 2; ++rp) {
              const uint4 qb = hq[(2 * rp) * 64], qc = hq[(2 * rp + 1) * 64];
              hwB0[rp] = h2(qb.x);
              hwB1[rp] = h2(qb.y);
              hbB0[rp] = h2(qb.z);
              hbB1[rp] = h2(qb.w);
              hwC0[rp] = h2(qc.x);
              hwC1[rp] = h2(qc.y);
              hbC0[rp] = h2(qc.z);
              hbC1[rp] = h2(qc.w);
            }
          } else {
            const uint4 q = hq[0];
            hwB0[0] = h2(q.x);
            hbB0[0] = h2(q.y);
            hwC0[0] = h2(q.z);
            hbC0[0] = h2(q.w);
          }
        }
        // raw (2i, 2i+1) x R blocks: registers, or shared memory (TMA path), where the whole warp
        // reads a group of TG tokens before any lane overwrites them with tile entries
        constexpr int TG = TMA ? 4 : 1;
        // Rows of tokens past T come out as the rotated bias: harmless, since their C^ rows only
        // reach outputs that are not stored, their S columns are masked for every stored row,
        // and their X / W rows are zero.
        PairRaw<TA, R> grb[TG], grc[TG];
        float4 dt4, rb4, rc4;  // the group's dt and rms of B / C (TMA path)
#pragma unroll
        for (int jj = 0; jj < SEGMAX; ++jj) {
          if (!N128 && jj >= seglen) break;
          const int j = seg * seglen + jj;
          if constexpr (TMA) {
            static_assert(TG == 4, "the TMA path reads the group's token scalars as float4");
            if (jj % TG == 0) {
#pragma unroll
              for (int u = 0; u < TG; ++u) {
                const uint8_t* src = st + (pi >> 5) * 16384 + (j + u) * (RP * 128) + (pi & 31) * (R * 4);
                grb[u].load_shared(src + PL::tB);
                grc[u].load_shared(src + PL::tC);
              }
              dt4 = *reinterpret_cast<const float4*>(dtv + j);
              rb4 = *reinterpret_cast<const float4*>(rmsB + j);
              rc4 = *reinterpret_cast<const float4*>(rmsC + j);
              __syncwarp();
            }
          }
          auto comp = [](const float4& v, int i) { return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w; };
          const float dtj = TMA ? comp(dt4, jj % 4) : dtv[j];
          const float rbv = TMA ? comp(rb4, jj % 4) : rmsB[j];
          const float rcv = TMA ? comp(rc4, jj % 4) : rmsC[j];
          const PairRaw<TA, R>& rawb = [&]() -> const PairRaw<TA, R>& {
            if constexpr (TMA) return grb[jj % TG];
            else return vb[jj];
          }();
          const PairRaw<TA, R>& rawc = [&]() -> const PairRaw<TA, R>& {
            if constexpr (TMA) return grc[jj % TG];
            else return vc[jj];
          }();
          float cs = 1.f, sn = 0.f;
          if (p.complex_ssm) {
            run = off + pre[jj];
            sincos_reduced(omf - run, &sn, &cs);
          }
          const float2 rbj = make_float2(rbv, rbv), rcj = make_float2(rcv, rcv);
          uint32_t ob[RP], oc[RP];
          auto as_h2 = [](uint32_t w) { return *reinterpret_cast<const __nv_bfloat162*>(&w); };
          auto as_u = [](__nv_bfloat162 v) { return *reinterpret_cast<const uint32_t*>(&v); };
          if constexpr (TMA && R % 2 == 0) {
            const __nv_bfloat162 rb2 = __float2bfloat162_rn(rbv), rc2 = __float2bfloat162_rn(rcv);
            const __nv_bfloat162 c2 = __float2bfloat162_rn(cs), s2 = __float2bfloat162_rn(sn);
            const __nv_bfloat162 ns2 = __hneg2(s2);
#pragma unroll
            for (int rp = 0; rp < R / 2; ++rp) {
              // words: n = 2i (ranks 2rp, 2rp+1) and n = 2i+1 (same ranks)
              const __nv_bfloat162 b0 = __hfma2(__hmul2(as_h2(rawb.w[rp]), hwB0[rp]), rb2, hbB0[rp]);
              const __nv_bfloat162 b1 = __hfma2(__hmul2(as_h2(rawb.w[R / 2 + rp]), hwB1[rp]), rb2, hbB1[rp]);
              const __nv_bfloat162 be = __hfma2(b1, ns2, __hmul2(b0, c2)), bo = __hfma2(b1, c2, __hmul2(b0, s2));
              ob[2 * rp] = as_u(__lows2bfloat162(be, bo));
              ob[2 * rp + 1] = as_u(__highs2bfloat162(be, bo));
              if constexpr (!SO) {
                const __nv_bfloat162 c0 = __hfma2(__hmul2(as_h2(rawc.w[rp]), hwC0[rp]), rc2, hbC0[rp]);
                const __nv_bfloat162 c1 = __hfma2(__hmul2(as_h2(rawc.w[R / 2 + rp]), hwC1[rp]), rc2, hbC1[rp]);
                const __nv_bfloat162 ce = __hfma2(c1, ns2, __hmul2(c0, c2)), co = __hfma2(c1, c2, __hmul2(c0, s2));
                oc[2 * rp] = as_u(__lows2bfloat162(ce, co));
                oc[2 * rp + 1] = as_u(__highs2bfloat162(ce, co));
              } else {
                oc[2 * rp] = oc[2 * rp + 1] = 0u;
              }
            }
          } else if constexpr (TMA) {
            // R = 1: the word is (n = 2i, 2i+1); (x0 c - x1 s, x0 s + x1 c) = x1 (-s, c) + x0 (c, s)
            const __nv_bfloat162 rb2 = __float2bfloat162_rn(rbv), rc2 = __float2bfloat162_rn(rcv);
            const __nv_bfloat162 ncs = __floats2bfloat162_rn(-sn, cs), csn = __floats2bfloat162_rn(cs, sn);
            const __nv_bfloat162 bv = __hfma2(__hmul2(as_h2(rawb.w[0]), hwB0[0]), rb2, hbB0[0]);
            ob[0] = as_u(__hfma2(__high2bfloat162(bv), ncs, __hmul2(__low2bfloat162(bv), csn)));
            const __nv_bfloat162 cv = __hfma2(__hmul2(as_h2(rawc.w[0]), hwC0[0]), rc2, hbC0[0]);
            oc[0] = as_u(__hfma2(__high2bfloat162(cv), ncs, __hmul2(__low2bfloat162(cv), csn)));
          } else if constexpr (R % 2 == 0) {
            const float2 c2 = make_float2(cs, cs), s2 = make_float2(sn, sn), ns2 = make_float2(-sn, -sn);
#pragma unroll
            for (int rp = 0; rp < R / 2; ++rp) {
              // x0 = element n = 2i, x1 = n = 2i+1, both for ranks (2 rp, 2 rp + 1)
              const float2 b0 = fma2(rawb.pair(2 * rp), mul2(rbj, wB0[rp]), bB0[rp]);
              const float2 b1 = fma2(rawb.pair(R + 2 * rp), mul2(rbj, wB1[rp]), bB1[rp]);
              const float2 c0 = fma2(rawc.pair(2 * rp), mul2(rcj, wC0[rp]), bC0[rp]);
              const float2 c1 = fma2(rawc.pair(R + 2 * rp), mul2(rcj, wC1[rp]), bC1[rp]);
              const float2 be = fma2(b1, ns2, mul2(b0, c2)), bo = fma2(b1, c2, mul2(b0, s2));
              const float2 ce = fma2(c1, ns2, mul2(c0, c2)), co = fma2(c1, c2, mul2(c0, s2));
              ob[2 * rp] = pack_bf16x2(be.x, bo.x);
              ob[2 * rp + 1] = pack_bf16x2(be.y, bo.y);
              oc[2 * rp] = pack_bf16x2(ce.x, co.x);
              oc[2 * rp + 1] = pack_bf16x2(ce.y, co.y);
            }
#pragma unroll
            for (int r = R; r < RP; ++r) ob[r] = oc[r] = 0u;
          } else {
            // R = 1: the pair (n = 2i, 2i+1) is one float2
            const float2 bv = fma2(rawb.pair(0), mul2(rbj, wB0[0]), bB0[0]);
            const float2 cv = fma2(rawc.pair(0), mul2(rcj, wC0[0]), bC0[0]);
            // (x0 c - x1 s, x0 s + x1 c) = x1 * (-s, c) + x0 * (c, s)
            const float2 ncs = make_float2(-sn, cs), csn = make_float2(cs, sn);
            const float2 be = fma2(make_float2(bv.y, bv.y), ncs, mul2(make_float2(bv.x, bv.x), csn));
            const float2 ce = fma2(make_float2(cv.y, cv.y), ncs, mul2(make_float2(cv.x, cv.x), csn));
            ob[0] = pack_bf16x2(be.x, be.y);
            oc[0] = pack_bf16x2(ce.x, ce.y);
#pragma unroll
            for (int r = 1; r < RP; ++r) ob[r] = oc[r] = 0u;
          }
#pragma unroll
          for (int r = 0; r < RP; ++r) {
            const uint32_t o = sw128_offset(j * RP + r, 2 * pi, 128);
            *reinterpret_cast<uint32_t*>(st + PL::tB + o) = ob[r];
            if constexpr (!SO) *reinterpret_cast<uint32_t*>(st + PL::tC + o) = oc[r];
          }
        }
        if (seg == nseg - 1) {
          // angle after this chunk = before - (off + own segment sum); the next chunk reads the other slot
          const double nom = p.complex_ssm ? om - (double)(off + segsum) : om;
          omega[((g + 1) & 1) * 64 + pi] = nom;
          if (k == sc.K - 1) {
            a.angle_last[((int64_t)b * H + h) * nh2 + pi] = (float)nom;
          } else if (pos.kk == sc.KP - 1) {  // end of a part: hand the angles to the next part
            a.ho_ang[(int64_t)pos.seq * 64 + pi] = nom;
            __threadfence();
          }
        }
      }
      if (ptid == 0) M3B_TL(g, 3);
      // the next chunk's token scalars, while the other warps finish their rotations (its raw
      // values were requested at the start of this chunk; same sequence, so same dt_bias)
      if (ptid <= L && g + 1 < G && pnext.kk != 0) tok_scalars(nxt);
      fence_async_smem();
      named_bar(kBarProd, kProdThreads);  // B^, C^ tiles and the token scalars (wst, gbw) complete
      if (ptid == 0 && pos.kk == sc.KP - 1 && pos.part + 1 < sc.nparts)
        st_release_gpu(a.ho_flag + 2 * pos.seq, pos.part + 1);  // this part's angles are written
      if (ptid == 0) {
        mbar_arrive(&bars[BAR_FULL0 + s]);
        if constexpr (!SO) {
          // S_g = C^ B^T into S[g%2] (free: the epilogue released this stage before handing it over)
          tc_fence_after();
          const uint32_t cs0 = kColS + 128 * s;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            umma_bf16(tbase + cs0, kmajor_desc(st + PL::tC, 128, kk * 16), kmajor_desc(st + PL::tB, 128, kk * 16),
                      idS, kk > 0 ? 1u : 0u);
          umma_commit(&bars[BAR_SDONE0 + s]);
        }
        M3B_TL(g, 4);
      }
    }
  } else {
    // =============================== epilogue ===============================
    volatile int* abort_flag = epi_abort;
    bool tmo = false;  // this thread's own bounded waits (own_wait) timed out
    const int lq = warp & 3, ch = warp >> 2;  // TMEM lane quadrant, column half
    const int m = 32 * lq + lane;             // TMEM lane = tile row (t, r)
    const int t = m / RP, r = m % RP;
    const uint32_t trow = tbase + ((uint32_t)(32 * lq) << 16);
    uint8_t* tileH = sm + PL::tileH;
    // mimo_z, mimo_down, mimo_x of the current sequence, rank-major: [q][p]
    float* emz = reinterpret_cast<float*>(sm + PL::epar);
    float* emd = emz + kPP * RP;
    float* emx = reinterpret_cast<float*>(sm + PL::mxs);
    const bool lead = tid == 0;
    const int xpc = tid & 7;  // X / W tiles: this thread's 8-column chunk of p
    // x of chunk gg, rows j = (tid + 256 u) / 8 (loaded a chunk ahead of the X / W tiles)
    auto load_x = [&](const ChunkPos& c, Raw8<TA> (&xr)[XU]) {
      const TA* xb = proj + (int64_t)c.b * a.T * a.proj_stride + HP + (int64_t)c.h * P + xpc * 8;
#pragma unroll
      for (int u = 0; u < XU; ++u) {
        const int64_t tt = (int64_t)c.k * L + ((tid + kEpiThreads * u) >> 3);
        if (tt < a.T && xpc * 8 < P) xr[u].load(xb + tt * a.proj_stride);
        else xr[u].zero();
      }
    };
    // X (rows (s, q) = x_s * mimo_x[:, q]) and W = wst_s X tiles of chunk gg; its token scalars
    // are in place (FULL of gg has completed) and mimo_x is the current sequence's
    auto build_xw = [&](int gg, const Raw8<TA> (&xr)[XU]) {
      uint8_t* stg = sm + (gg & 1) * PL::kStage;
      const float* wsg = reinterpret_cast<const float*>(sm + PL::scal + (gg & 1) * PL::scalStride) + 4 * NA;
#pragma unroll
      for (int u = 0; u < XU; ++u) {
        const int j = (tid + kEpiThreads * u) >> 3;
        const float2 w2 = make_float2(wsg[j], wsg[j]);
#pragma unroll
        for (int q = 0; q < RP; ++q) {
          const float4* mx4 = reinterpret_cast<const float4*>(emx + q * kPP + xpc * 8);
          const float4 ma = mx4[0], mb = mx4[1];
          const float2 mxp[4] = {make_float2(ma.x, ma.y), make_float2(ma.z, ma.w), make_float2(mb.x, mb.y),
                                 make_float2(mb.z, mb.w)};
          uint4 ox, ow;
          uint32_t* oxw = reinterpret_cast<uint32_t*>(&ox);
          uint32_t* oww = reinterpret_cast<uint32_t*>(&ow);
#pragma unroll
          for (int e2 = 0; e2 < 4; ++e2) {
            const float2 v = mul2(xr[u].pair(2 * e2), mxp[e2]);
            const float2 vw = mul2(v, w2);
            oxw[e2] = pack_bf16x2(v.x, v.y);
            oww[e2] = pack_bf16x2(vw.x, vw.y);
          }
          if constexpr (!SO) sw128_store_chunk(stg + PL::tX, j * RP + q, xpc, 128, ox);
          sw128_store_chunk(stg + PL::tW, j * RP + q, xpc, 128, ow);
        }
      }
    };
    constexpr uint32_t idO = idesc_bf16(128, kPP, false, true);  // Yi and Y: B operand MN-major
    constexpr uint32_t idH = idesc_bf16(128, kPP, true, true);   // H: A and B MN-major
    // leader: Yi_g = C^ H'^T and H += B^^T (w X) for chunk g, then commit HDONE
    auto issue_state_mma = [&](int g) {
      const int s = g & 1;
      uint8_t* st = sm + s * PL::kStage;
      tc_fence_after();
      if constexpr (!SO) {
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_bf16(tbase + kColYi, kmajor_desc(st + PL::tC, 128, kk * 16), mnmajor_desc(tileH, 128, kk * 16), idO,
                    kk > 0 ? 1u : 0u);
      }
#pragma unroll
      for (int kk = 0; kk < 8; ++kk)
        umma_bf16(tbase + kColH, mnmajor_desc(st + PL::tB, 128, kk * 16), mnmajor_desc(st + PL::tW, 128, kk * 16),
                  idH, 1u);
      umma_commit(&bars[BAR_HDONE]);
    };
    // H'_0 of the job starting at chunk gs -> bf16 tile row n = m, and H = d * H'_0 in TMEM.  A first
    // part starts from h_init (+ (1-lam_0) dt_0 prev_bx_init); a later part from the state the
    // previous part of its sequence handed over (the beta term of its first token is in it)
    auto state_init = [&](const ChunkPos& c, int gs) -> bool {
      const int b = c.b, h = c.h;
      const int s2 = gs & 1;
      // this sequence's gate parameters (one entry per thread), requested before the waits below
      static_assert(kPP * 4 <= kEpiThreads, "one gate parameter entry per epilogue thread");
      const int pd = p.param_dtype;
      const int gpp = tid / RP, gq = tid % RP;
      const bool gok = tid < kPP * RP && gpp < P && gq < R;
      const int64_t gi = ((int64_t)h * P + gpp) * R + gq;
      const float gmz = gok ? ldf(p.mimo_z, gi, pd) : 0.f;
      const float gmd = gok ? ldf(p.mimo_down, gi, pd) : 0.f;
      const float gmx = gok ? ldf(p.mimo_x, gi, pd) : 0.f;
      if (c.part > 0 && lead && !*abort_flag && !flag_wait_geq(a.ho_flag + 2 * c.seq + 1, c.part, a.wait_ns)) {
        *abort_flag = 1;
        record_error(a.err, M3B_ERR_TIMEOUT);
      }
      if (!role_wait(&bars[BAR_FULL0 + s2], (gs >> 1) & 1, lead, kBarEpi, kEpiThreads, abort_flag, a.err, a.wait_ns))
        return false;
      const float* scal = reinterpret_cast<const float*>(sm + PL::scal + s2 * PL::scalStride);
      const float d = exp2f(scal[L - 1]);
      const float c0 = scal[3 * NA];  // (1-lam_0) dt_0
      const int64_t o = ((int64_t)b * H + h) * (int64_t)P * N + (int64_t)(32 * ch) * N + m;
      const float* hsrc = m < N ? (c.part > 0 ? a.ho_h : a.h_init) : nullptr;
      const float* bxsrc = m < N && c.part == 0 ? a.prev_bx_init : nullptr;
      // eight columns at a time: their loads are in flight together, and few registers are live
#pragma unroll
      for (int c8 = 0; c8 < 4; ++c8) {
        float v8[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const bool okp = 32 * ch + 8 * c8 + e < P;
          v8[e] = hsrc && okp ? __ldcg(hsrc + o + (int64_t)(8 * c8 + e) * N) : 0.f;
        }
        if (bxsrc) {
#pragma unroll
          for (int e = 0; e < 8; ++e)
            if (32 * ch + 8 * c8 + e < P) v8[e] = fmaf(c0, bxsrc[o + (int64_t)(8 * c8 + e) * N], v8[e]);
        }
        st_pack_chunk(tileH, m, 4 * ch + c8, v8);
#pragma unroll
        for (int e = 0; e < 8; ++e) v8[e] *= d;
        tmem_st8_nowait(trow + kColH + 32 * ch + 8 * c8, v8);
      }
      tmem_wait_st();
      // the gate parameters into shared memory (the previous sequence's last output is complete)
      if (tid < kPP * RP) {
        emz[gq * kPP + gpp] = 0.5f * gmz;  // halved: the output takes silu(2a) with a = z mimo_z / 2
        emd[gq * kPP + gpp] = gmd;
        emx[gq * kPP + gpp] = gmx;
      }
      named_bar(kBarEpi, kEpiThreads);  // mimo_x is read by the X / W tiles below
      return true;
    };
    // the state after the last chunk of job c: h_final after a sequence's last part, otherwise
    // handed to the sequence's next part (written, then flagged)
    auto write_h_final = [&](const ChunkPos& c) {
      const bool handoff = c.part + 1 < sc.nparts;
      float* dst = handoff ? a.ho_h : a.h_final;
      if (dst) {
        const int64_t base = ((int64_t)c.b * H + c.h) * (int64_t)P * N;
        float v[32];
        tmem_ld32(trow + kColH + 32 * ch, v);
        if (m < N) {
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const int pp = 32 * ch + e;
            if (pp < P) dst[base + (int64_t)pp * N + m] = v[e];
          }
        }
      }
      if (handoff) {
        __threadfence();
        named_bar(kBarEpi, kEpiThreads);
        if (lead) st_release_gpu(a.ho_flag + 2 * c.seq + 1, c.part + 1);
      }
    };
    // The blocks of P above the block diagonal (column block > this warp's lane quadrant) are zero
    // in every chunk: stored once here, never rewritten.
    if constexpr (!SO) {
      uint32_t z16[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) z16[e] = 0u;
#pragma unroll
      for (int c32 = 0; c32 < 2; ++c32)
        if (2 * ch + c32 > lq) tmem_st16_nowait(trow + kColP + 16 * (2 * ch + c32), z16);
      tmem_wait_st();
    }
    Raw8<TA> xn[XU];  // x of the next chunk
    ChunkPos pos = sc.first();
    if (G > 0) load_x(pos, xn);
    bool ok = G > 0 && state_init(pos, 0);
    if (ok) {
      build_xw(0, xn);
      fence_async_smem();
      tc_fence_before();
      named_bar(kBarEpi, kEpiThreads);
      if (lead) issue_state_mma(0);
    }
    for (int g = 0; ok && g < G; ++g, sc.advance(pos)) {
      const int s = g & 1;
      const int b = pos.b, h = pos.h, k = pos.k;
      const ChunkPos pnext = sc.ahead(pos, 1);
      uint8_t* st = sm + s * PL::kStage;
      const float* scal = reinterpret_cast<const float*>(sm + PL::scal + s * PL::scalStride);
      const float* cum2 = scal;
      const float* gam = scal + 2 * NA;
      const float* gbw = scal + 5 * NA;
      const uint32_t cs0 = kColS + 128 * s;
      if (g + 1 < G) load_x(pnext, xn);
      if constexpr (TMA && !SO) {  // z of the next chunk into L2 (its loads below are a chunk later)
        if (lead && g + 1 < G) tma_prefetch_3d(&tm_th, pnext.h * P, pnext.k * L, pnext.b);
      }
      if constexpr (SO) {
        // state only: the H update of chunk g must be complete before the stage is handed
        // over and before state(g+1) reads H
        if (lead && !*abort_flag) {
          if (!mbar_wait(&bars[BAR_HDONE], g & 1, a.wait_ns)) {
            *abort_flag = 1;
            record_error(a.err, M3B_ERR_TIMEOUT);
          } else if (g + 2 < G) {
            issue_stage(sc.ahead(pnext, 1), g + 2);
          }
        }
        __syncwarp();
        named_bar(kBarEpi, kEpiThreads);
        if (*abort_flag) {
          ok = false;
          break;
        }
        tc_fence_after();
      } else {
        // z of this thread's row (t, r) and column half, prefetched while the tensor core works
        const int64_t tok = (int64_t)k * L + t;
        const bool row_ok = tok < a.T && r < R;
        Raw8<TA> zr[4];
        {
          const TA* zrow = proj + ((int64_t)b * a.T + (tok < a.T ? tok : 0)) * a.proj_stride + (int64_t)h * P + 32 * ch;
#pragma unroll
          for (int c8 = 0; c8 < 4; ++c8) {
            if (row_ok && 32 * ch + c8 * 8 < P) zr[c8].load(zrow + c8 * 8);
            else zr[c8].zero();
          }
        }
        // S_g (producer) must be complete before the mask reads it; the state GEMMs of chunk g
        // (issued at the end of the previous chunk) keep running meanwhile.  Every thread waits
        // itself (no role barrier); a timeout is acted on after the barrier that ends the mask.
        own_wait(&bars[BAR_SDONE0 + s], (g >> 1) & 1, tmo, a.err, a.wait_ns);
        tc_fence_after();
        if (lead) M3B_TL(g, 8);
        // ---- mask.  The intra-chunk weight of (token t, source s <= t) is
        //   w(t, s) = 2^(cum_t - cum_s) * (s < t ? gamma_s + (1-lam_{s+1}) dt_{s+1} : gamma_s).
        // Separable form (the chunk's decay range cum_0 - cum_{L-1} <= kSepRange): for s < t,
        // w = e_t * wst_s with e_t = 2^(cum_t - cum_{L-1}) and wst_s the state-update weight, so
        // Y = diag(e) * P' * W with P' = S masked (s < t: S; s = t: S gamma_t / gbw_t; s > t: 0)
        // and W the chunk-state tile: no per-element exponentials.  Otherwise P = S * w, Y = P X.
        // Column block blk (32 columns) of warp quadrant lq lies below (blk < lq), on (blk == lq)
        // or above (blk > lq) the block diagonal, for every lane alike.
        // Everything the output needs from this stage (scalars, the thread's x_r row of the X tile)
        // is read here: the stage goes back to the producers before the output is written.
        constexpr float kSepRange = 64.f;
        const float c_last = cum2[L - 1];
        const bool sep = cum2[0] - c_last <= kSepRange;
        const float Dh = ldf(p.D, h, p.param_dtype);
        const float ct = cum2[t];
        const float ec = exp2f(ct);
        const float et = sep ? exp2f(ct - c_last) : 1.f;
        {
          const float gwt = gbw[t];
          const float rat = gwt > 0.f ? gam[t] / gwt : 0.f;
#pragma unroll
          for (int c32 = 0; c32 < 2; ++c32) {
            const int blk = 2 * ch + c32;
            const int c0 = 32 * blk;
            if (blk > lq) continue;  // above the block diagonal: stays zero (stored once at kernel start)
            float v[32];
            {
              tmem_ld32(trow + cs0 + c0, v);
              if (lead && c32 == 0) M3B_TL(g, 13);
              if (sep) {
                if (blk == lq) {
#pragma unroll
                  for (int jj = 0; jj < 32; jj += RP) {
                    const int sj = (c0 + jj) / RP;
                    const float f = sj < t ? 1.f : (sj == t ? rat : 0.f);
#pragma unroll
                    for (int q = 0; q < RP; ++q) v[jj + q] *= f;
                  }
                }
              } else {
#pragma unroll
                for (int jj = 0; jj < 32; jj += RP) {
                  const int sj = (c0 + jj) / RP;
                  const float e = ex2_fast(fminf(ct - cum2[sj], 0.f));
                  const float w = sj < t ? e * gbw[sj] : (sj == t ? gam[sj] : 0.f);
#pragma unroll
                  for (int q = 0; q < RP; ++q) v[jj + q] *= w;
                }
              }
            }
            // row m of P, columns (s, q) of this block: bf16 pairs into TMEM (16 columns)
            uint32_t pw[16];
#pragma unroll
            for (int e = 0; e < 16; ++e) pw[e] = pack_bf16x2(v[2 * e], v[2 * e + 1]);
            tmem_st16_nowait(trow + kColP + 16 * blk, pw);
            if (lead && c32 == 0) M3B_TL(g, 14);
          }
        }
        // x_r of this thread's row (t, r) and column half, for D x (the X tile goes back with the stage)
        uint4 xq[4];
#pragma unroll
        for (int c8 = 0; c8 < 4; ++c8)
          xq[c8] = *reinterpret_cast<const uint4*>(st + PL::tX + sw128_offset(m, 32 * ch + c8 * 8, 128));
        tmem_wait_st();
        tc_fence_before();
        if (barrier_or(kBarEpi, kEpiThreads, tmo)) {  // a wait of this chunk timed out
          *abort_flag = 1;
          ok = false;
          break;
        }
        if (lead) {
          // Y_g = P' W (separable) or P X into Y (the previous chunk's output has read it); A = P
          // from TMEM, K = (s, q) in 8 columns per instruction
          tc_fence_after();
          const uint8_t* yb = st + (sep ? PL::tW : PL::tX);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            umma_bf16_ts(tbase + kColY, tbase + kColP + 8 * kk, mnmajor_desc(yb, 128, kk * 16), idO, kk > 0 ? 1u : 0u);
          umma_commit(&bars[BAR_YDONE]);
          M3B_TL(g, 9);
        }
        // The state GEMMs of chunk g (Yi_g, the H update; committed to HDONE) and Y_g (YDONE) are
        // the last readers of stage s: once both have completed, the stage goes to the producers
        // for chunk g + 2 (with its TMA copies) while this chunk's output is written.  Every thread
        // waits itself; a timeout is acted on after the next role barrier (the state of chunk g+1).
        own_wait(&bars[BAR_HDONE], g & 1, tmo, a.err, a.wait_ns);
        own_wait(&bars[BAR_YDONE], g & 1, tmo, a.err, a.wait_ns);
        if (lead && !tmo && g + 2 < G) issue_stage(sc.ahead(pnext, 1), g + 2);
        tc_fence_after();
        if (lead) M3B_TL(g, 10);
        // ---- output of chunk g: y = e_t Y + e^cum_t Yi + D x_r, gate, MIMO down
        {
          const float2 et2 = make_float2(et, et), ec2 = make_float2(ec, ec), D2 = make_float2(Dh, Dh);
          TA* yo = reinterpret_cast<TA*>(a.y) + ((int64_t)b * a.T + tok) * HP + (int64_t)h * P;
#pragma unroll
          for (int qq = 0; qq < 2; ++qq) {
            // 16 columns of Y and of Yi in flight at once, combined right away
            uint32_t yraw[16], yiraw[16];
            tmem_ld16_async(trow + kColY + 32 * ch + 16 * qq, yraw);
            tmem_ld16_async(trow + kColYi + 32 * ch + 16 * qq, yiraw);
            tmem_wait_ld(yraw, yiraw);
            float acc[16];
#pragma unroll
            for (int hc = 0; hc < 2; ++hc) {
              const int c8 = 2 * qq + hc;  // chunk within this column half
              const int p8 = 32 * ch + c8 * 8;
              const uint32_t xw[4] = {xq[c8].x, xq[c8].y, xq[c8].z, xq[c8].w};
              const float4* mz4 = reinterpret_cast<const float4*>(emz + r * kPP + p8);
              const float4* md4 = reinterpret_cast<const float4*>(emd + r * kPP + p8);
              const float4 za = mz4[0], zb = mz4[1], da = md4[0], db = md4[1];
              const float2 mzp[4] = {make_float2(za.x, za.y), make_float2(za.z, za.w), make_float2(zb.x, zb.y),
                                     make_float2(zb.z, zb.w)};
              const float2 mdp[4] = {make_float2(da.x, da.y), make_float2(da.z, da.w), make_float2(db.x, db.y),
                                     make_float2(db.z, db.w)};
#pragma unroll
              for (int e2 = 0; e2 < 4; ++e2) {
                const int i = 8 * hc + 2 * e2;
                const float2 ys = fma2(et2, make_float2(__uint_as_float(yraw[i]), __uint_as_float(yraw[i + 1])),
                                       mul2(ec2, make_float2(__uint_as_float(yiraw[i]), __uint_as_float(yiraw[i + 1]))));
                const float2 yv = fma2(D2, bf2_to_f2(xw[e2]), ys);
                // silu(z mz) md with a = z mz / 2: a md (1 + tanh a)
                const float2 o = mul2(yv, silu2a_mul2(mul2(zr[c8].pair(2 * e2), mzp[e2]), mdp[e2]));
                acc[i] = o.x;
                acc[i + 1] = o.y;
              }
            }
            // sum over the RP lanes (t, r) of a token, reduce-scatter style: each halving step
            // keeps the half picked by one bit of r, so lane r ends with columns [r W, r W + W)
            constexpr int W = 16 / RP;  // outputs written by each of the RP lanes of a token
#pragma unroll
            for (int o = RP / 2, w = 8; o >= 1; o >>= 1, w >>= 1) {
              const bool up = (r & o) != 0;
#pragma unroll
              for (int e = 0; e < w; ++e) {
                const float send = up ? acc[e] : acc[e + w];
                const float keep = up ? acc[e + w] : acc[e];
                acc[e] = keep + __shfl_xor_sync(0xffffffffu, send, o);
              }
            }
            if (tok < a.T) {
              const int p0 = 32 * ch + 16 * qq + r * W;
              if (p0 + W <= P) {
                if constexpr (W >= 8) {
#pragma unroll
                  for (int h8 = 0; h8 < W / 8; ++h8) {
                    float o8[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) o8[e] = acc[8 * h8 + e];
                    store8<TA>(yo + p0 + 8 * h8, o8);
                  }
                } else if constexpr (W == 4 && sizeof(TA) == 2) {
                  uint2 o4;
                  o4.x = pack_bf16x2(acc[0], acc[1]);
                  o4.y = pack_bf16x2(acc[2], acc[3]);
                  *reinterpret_cast<uint2*>(yo + p0) = o4;
                } else {
#pragma unroll
                  for (int e = 0; e < W; ++e) io<TA>::st(yo + p0 + e, acc[e]);
                }
              } else {
#pragma unroll
                for (int e = 0; e < W; ++e)
                  if (p0 + e < P) io<TA>::st(yo + p0 + e, acc[e]);
              }
            }
          }
        }
      }
      if (lead) M3B_TL(g, 11);
      // ---- state for chunk g+1: H'_{g+1} -> bf16 tile, H *= d_{g+1}; then Yi_{g+1}, H += ...
      if (g + 1 < G) {
        if (pnext.kk == 0) {  // a new job starts with chunk g+1
          write_h_final(pos);
          if (!(ok = state_init(pnext, g + 1))) break;
        } else {
          const int s1 = (g + 1) & 1;
          // every thread waits itself; a timeout is acted on after the barrier below
          own_wait(&bars[BAR_FULL0 + s1], ((g + 1) >> 1) & 1, tmo, a.err, a.wait_ns);
          const float* scal1 = reinterpret_cast<const float*>(sm + PL::scal + s1 * PL::scalStride);
          const float d = exp2f(scal1[L - 1]);
          float v[32];
          tmem_ld32(trow + kColH + 32 * ch, v);
          if constexpr (!SO) {  // H' for C^H'^T (not issued in state-only mode)
#pragma unroll
            for (int c8 = 0; c8 < 4; ++c8) {
              float v8[8];
#pragma unroll
              for (int e = 0; e < 8; ++e) v8[e] = v[8 * c8 + e];
              st_pack_chunk(tileH, m, 4 * ch + c8, v8);
            }
          }
#pragma unroll
          for (int e = 0; e < 32; ++e) v[e] *= d;
          tmem_st32(trow + kColH + 32 * ch, v);
        }
        build_xw(g + 1, xn);
        fence_async_smem();
        tc_fence_before();
        if (barrier_or(kBarEpi, kEpiThreads, tmo)) {  // a wait of this chunk timed out
          *abort_flag = 1;
          ok = false;
          break;
        }
        if (lead) {
          issue_state_mma(g + 1);
          M3B_TL(g, 12);
        }
      } else {
        write_h_final(pos);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
// cuTensorMapEncodeTiled from the driver the runtime is bound to (no link-time libcuda dependency).
EncodeTiledFn encode_tiled() {
  static const EncodeTiledFn fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &f, 12000, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      f = nullptr;
    return reinterpret_cast<EncodeTiledFn>(f);
  }();
  return fn;
}

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


// 3-D bf16 map over the projection (columns, tokens, batch rows) with box (box0, box1, 1); tokens
// past T read as zeros.  False when the driver refuses the encoding.
bool make_proj_map(CUtensorMap* m, const FusedParams& fp, uint32_t box0, uint32_t box1) {
  const EncodeTiledFn enc = encode_tiled();
  if (!enc) return false;
  const cuuint64_t dims[3] = {(cuuint64_t)fp.proj_stride, (cuuint64_t)fp.T, (cuuint64_t)fp.B};
  const cuuint64_t strides[2] = {(cuuint64_t)fp.proj_stride * 2, (cuuint64_t)fp.proj_stride * 2 * (cuuint64_t)fp.T};
  const cuuint32_t box[3] = {box0, box1, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(fp.proj), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The TMA producer path needs N = 128 and 16-byte aligned rows and column offsets of B, C and theta.
bool tma_layout_ok(const FusedParams& fp) {
  const m3b_layer_params& p = fp.prm;
  const int64_t HP = (int64_t)p.H * p.P, NR = (int64_t)p.N * p.R;
  const int64_t offB = 2 * HP, offTh = offB + 2 * p.G * NR + p.H + (p.trapezoidal ? p.H : 0);
  return p.N == 128 && (reinterpret_cast<uintptr_t>(fp.proj) & 15) == 0 && fp.proj_stride % 8 == 0 &&
         offB % 8 == 0 && (!p.complex_ssm || offTh % 8 == 0) && fp.T < (int64_t(1) << 31);
}

template <typename TA, int R, bool TMA, bool SO>
int launch_fused_t(const FusedParams& fp, cudaStream_t st, const CUtensorMap& tm_bc, const CUtensorMap& tm_th) {
  constexpr int RP = rp_of(R);
  using PL = FPlan<RP>;
  const int nseq_total = (int)(fp.B * fp.prm.H);
  const int nsm = num_sms();
  const void* fn = (const void*)ssd_fused_kernel<TA, R, TMA, SO>;
  int rc;
  if ((rc = ensure_smem_f(fn, PL::bytes)) != M3B_OK) return rc;
  cudaFuncAttributes fa{};
  if (cudaFuncGetAttributes(&fa, fn) == cudaSuccess && fa.maxThreadsPerBlock < kFusedThreads)
    return fail(M3B_ERR_UNSUPPORTED, "ssd_fused: %d registers/thread allow only %d threads per block (need %d)",
                fa.numRegs, fa.maxThreadsPerBlock, kFusedThreads);
  const int KP = fp.KP > 0 && fp.K % fp.KP == 0 ? fp.KP : fp.K;
  const int nparts = fp.K / KP;
  const int njobs = nseq_total * nparts;
  const int grid = njobs < nsm ? njobs : nsm;
  if (nparts > 1) {
    if (!fp.ho_h || !fp.ho_ang || !fp.ho_flag) return fail(M3B_ERR_INVALID_ARG, "ssd_fused: hand-off buffers missing");
    const cudaError_t e = cudaMemsetAsync(fp.ho_flag, 0, sizeof(int) * 2 * (size_t)nseq_total, st);
    if (e != cudaSuccess) return fail(M3B_ERR_CUDA, "ssd_fused: %s", cudaGetErrorString(e));
  }
  const Sched sc{fp.K, fp.prm.H, nseq_total, grid, fp.prm.H / fp.prm.G, KP, nparts};
  ssd_fused_kernel<TA, R, TMA, SO><<<grid, kFusedThreads, PL::bytes, st>>>(fp, sc, tm_bc, tm_th);
  return check_launch("ssd_fused");
}

template <typename TA, int R>
int launch_fused_r(const FusedParams& fp, cudaStream_t st) {
  CUtensorMap tm_bc{}, tm_th{};
  if constexpr (sizeof(TA) == 2) {
    constexpr int L = 128 / rp_of(R);
    if (tma_layout_ok(fp) && make_proj_map(&tm_bc, fp, 64 * R, L) && make_proj_map(&tm_th, fp, 64, L))
      return fp.state_only ? launch_fused_t<TA, R, true, true>(fp, st, tm_bc, tm_th)
                           : launch_fused_t<TA, R, true, false>(fp, st, tm_bc, tm_th);
  }
  return launch_fused_t<TA, R, false, false>(fp, st, tm_bc, tm_th);
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
  if (!bf16) return fail(M3B_ERR_UNSUPPORTED, "ssd_fused: bf16 activations only (fp32 runs the tf32 chunk path)");
  switch (fp.prm.R) {
    case 1: return launch_fused_r<__nv_bfloat16, 1>(fp, st);
    case 2: return launch_fused_r<__nv_bfloat16, 2>(fp, st);
    case 4: return launch_fused_r<__nv_bfloat16, 4>(fp, st);
    default: return fail(M3B_ERR_UNSUPPORTED, "ssd_fused: mimo_rank %d", fp.prm.R);
  }
}

}  // namespace m3b
