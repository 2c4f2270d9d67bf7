// Cross-shard fold of the sequence-parallel prefill: the exact state entering shard `upto` from
// the affine summaries of shards 0 .. upto-1 (every rank's summary, as one all_gather left them).
//
// A shard run from the zero state ends in (S, PB, Om); with Lam = sum A dt over the shard and
// c0 = (1 - lam) dt of its first token, the state after it is affine in the state before it:
//   h' = e^Lam (h + c0 pb) + Rot(a) S,   a' = a + Om,   pb' = Rot(a) PB
// (Rot(a) turns the (2i, 2i+1) columns of a (P, N) state by the angle a_i).  Unrolled from the
// zero state, with a_g = sum_{j<g} Om_j and pb_g = Rot(a_{g-1}) PB_{g-1} (zero for g = 0):
//   h = sum_{g<upto} e^{sum_{g<j<upto} Lam_j} (e^{Lam_g} c0_g pb_g + Rot(a_g) S_g).
// One thread per (batch, head, p, column pair i) walks the shards in order; the angle prefix is
// summed in double (the layer kernels carry the running angle in double too) and each rotation
// uses the double-precision sine and cosine, so the fold adds no angle rounding of its own.
#include "common.cuh"
#include "launch.h"

namespace m3b {

namespace {

constexpr int kFoldThreads = 256;

__global__ void __launch_bounds__(kFoldThreads) seqpar_fold_kernel(m3b_seqpar_fold_args a) {
  const int nh2 = a.N / 2;
  const int64_t PN = (int64_t)a.P * a.N, BH = a.batch * a.H;
  const int64_t total = BH * a.P * nh2;
  const int64_t oPB = BH * PN, oOm = 2 * BH * PN, oLam = oOm + BH * nh2, oC0 = oLam + BH;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int i = (int)(idx % nh2);
    const int64_t rest = idx / nh2;
    const int p = (int)(rest % a.P);
    const int64_t bh = rest / a.P;
    const int64_t e = bh * PN + (int64_t)p * a.N + 2 * i;  // element (p, 2i) of this (batch, head)
    double lam_all = 0.0;
    for (int g = 0; g < a.upto; ++g) lam_all += a.summaries[(int64_t)g * a.rank_stride + oLam + bh];
    double ang = 0.0, lam_pre = 0.0;
    float h0 = 0.f, h1 = 0.f, pb0 = 0.f, pb1 = 0.f;  // pb: previous shard's PB in the global frame
    for (int g = 0; g < a.upto; ++g) {
      const float* s = a.summaries + (int64_t)g * a.rank_stride;
      double sn, cs;
      sincos(ang, &sn, &cs);
      const float c = (float)cs, sf = (float)sn;
      const float s0 = s[e], s1 = s[e + 1];
      const float lam = s[oLam + bh], c0 = s[oC0 + bh];
      lam_pre += lam;
      const float w = (float)exp(lam_all - lam_pre);  // e^{sum over the later shards}
      const float k = expf(lam) * c0;
      h0 += w * (k * pb0 + (s0 * c - s1 * sf));
      h1 += w * (k * pb1 + (s0 * sf + s1 * c));
      const float q0 = s[oPB + e], q1 = s[oPB + e + 1];
      pb0 = q0 * c - q1 * sf;
      pb1 = q0 * sf + q1 * c;
      ang += (double)s[oOm + bh * nh2 + i];
    }
    reinterpret_cast<float2*>(a.h + e)[0] = make_float2(h0, h1);
    reinterpret_cast<float2*>(a.prev_bx + e)[0] = make_float2(pb0, pb1);
    if (p == 0) a.angle[bh * nh2 + i] = (float)ang;
  }
}

}  // namespace

}  // namespace m3b

extern "C" M3B_API int m3b_seqpar_fold(const m3b_seqpar_fold_args* a, void* stream) {
  using namespace m3b;
  clear_error();
  if (!a) return fail(M3B_ERR_INVALID_ARG, "seqpar_fold: null args");
  if (a->batch < 0 || a->H <= 0 || a->P <= 0 || a->N <= 0 || a->N % 2 != 0 || a->upto < 0)
    return fail(M3B_ERR_INVALID_ARG, "seqpar_fold: bad dims batch=%lld H=%d P=%d N=%d upto=%d",
                (long long)a->batch, a->H, a->P, a->N, a->upto);
  const int64_t BH = a->batch * a->H, PN = (int64_t)a->P * a->N;
  const int64_t need = 2 * BH * PN + BH * (a->N / 2) + 2 * BH;
  if (a->upto > 0 && (!a->summaries || a->rank_stride < need))
    return fail(M3B_ERR_INVALID_ARG, "seqpar_fold: summaries missing or rank_stride %lld < summary size %lld",
                (long long)a->rank_stride, (long long)need);
  if (!a->h || !a->angle || !a->prev_bx) return fail(M3B_ERR_INVALID_ARG, "seqpar_fold: null output");
  if ((reinterpret_cast<uintptr_t>(a->h) | reinterpret_cast<uintptr_t>(a->prev_bx)) & 7u)
    return fail(M3B_ERR_ALIGNMENT, "seqpar_fold: h and prev_bx must be 8-byte aligned");
  const int64_t total = BH * a->P * (a->N / 2);
  if (total == 0) return M3B_OK;
  const int64_t cap = (int64_t)num_sms() * 8;
  const int64_t blocks = (total + kFoldThreads - 1) / kFoldThreads;
  seqpar_fold_kernel<<<(unsigned)(blocks < cap ? blocks : cap), kFoldThreads, 0, (cudaStream_t)stream>>>(*a);
  return check_launch("seqpar_fold");
}
