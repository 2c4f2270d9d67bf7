// Inter-chunk state scan (memory-bound).
//
//   h_states[:,0]   = h_init (+ coef * bx)          (zero when absent)
//   h_states[:,k+1] = decay[:,k] * h_states[:,k] + h_chunk[:,k]
//   h_final         = decay[:,K-1] * h_states[:,K-1] + h_chunk[:,K-1]
//
// Semantics of the reference scan (mamba3/scan.py:34-44, mamba3/csrc/scan.cu:10-50).
// Design: each thread owns VPT 8-element vectors of one (batch, head) state and
// walks the K chunks sequentially with an fp32 carry; the loads of the next U
// chunks are issued before the carry chain consumes them, every access is a
// 16-byte vector and consecutive threads touch consecutive vectors.  The decay
// scalar of a (batch, head, chunk) is shared by the whole block (broadcast load).
#include "common.cuh"
#include "launch.h"

namespace m3b {

template <typename T, int VPT>
__global__ void __launch_bounds__(256) scan_fwd_vec_kernel(const float* __restrict__ decay,
                                                           const T* __restrict__ hc,
                                                           const float* __restrict__ h_init,
                                                           const float* __restrict__ init_bx,
                                                           const float* __restrict__ init_coef,
                                                           T* __restrict__ hs, float* __restrict__ h_final,
                                                           int64_t K, int64_t H, int64_t PN) {
  constexpr int U = 4;
  const int64_t bh = blockIdx.x;
  const int64_t b = bh / H, h = bh - b * H;
  const int64_t kstride = H * PN;
  const float* dptr = decay + b * K * H + h;
  float c[VPT][8];
  int64_t j[VPT];
  bool act[VPT];
#pragma unroll
  for (int v = 0; v < VPT; ++v) {
    j[v] = ((int64_t)(blockIdx.y * VPT + v) * blockDim.x + threadIdx.x) * 8;
    act[v] = j[v] < PN;
#pragma unroll
    for (int i = 0; i < 8; ++i) c[v][i] = 0.f;
    if (act[v] && h_init) load8<float>(h_init + bh * PN + j[v], c[v]);
    if (act[v] && init_bx) {
      float bx[8];
      load8<float>(init_bx + bh * PN + j[v], bx);
      const float cf = init_coef[bh];
#pragma unroll
      for (int i = 0; i < 8; ++i) c[v][i] = fmaf(cf, bx[i], c[v][i]);
    }
  }
  const int64_t base = (b * K * H + h) * PN;
  for (int64_t k0 = 0; k0 < K; k0 += U) {
    float x[U][VPT][8];
    float d[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t k = k0 + u;
      d[u] = (k < K) ? __ldg(dptr + k * H) : 0.f;
#pragma unroll
      for (int v = 0; v < VPT; ++v)
        if (k < K && act[v]) load8<T>(hc + base + k * kstride + j[v], x[u][v]);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t k = k0 + u;
      if (k < K) {
#pragma unroll
        for (int v = 0; v < VPT; ++v) {
          if (!act[v]) continue;
          store8<T>(hs + base + k * kstride + j[v], c[v]);
#pragma unroll
          for (int i = 0; i < 8; ++i) c[v][i] = fmaf(d[u], c[v][i], x[u][v][i]);
        }
      }
    }
  }
  if (h_final) {
#pragma unroll
    for (int v = 0; v < VPT; ++v)
      if (act[v]) store8<float>(h_final + bh * PN + j[v], c[v]);
  }
}

// Any PN / alignment: one element per thread.
template <typename T>
__global__ void __launch_bounds__(256) scan_fwd_scalar_kernel(const float* __restrict__ decay,
                                                              const T* __restrict__ hc,
                                                              const float* __restrict__ h_init,
                                                              const float* __restrict__ init_bx,
                                                              const float* __restrict__ init_coef,
                                                              T* __restrict__ hs, float* __restrict__ h_final,
                                                              int64_t K, int64_t H, int64_t PN) {
  const int64_t bh = blockIdx.x;
  const int64_t b = bh / H, h = bh - b * H;
  const int64_t j = (int64_t)blockIdx.y * blockDim.x + threadIdx.x;
  if (j >= PN) return;
  float c = h_init ? h_init[bh * PN + j] : 0.f;
  if (init_bx) c = fmaf(init_coef[bh], init_bx[bh * PN + j], c);
  const int64_t base = (b * K * H + h) * PN + j;
  for (int64_t k = 0; k < K; ++k) {
    io<T>::st(hs + base + k * H * PN, c);
    c = fmaf(decay[(b * K + k) * H + h], c, io<T>::ld(hc + base + k * H * PN));
  }
  if (h_final) h_final[bh * PN + j] = c;
}

template <typename T>
static int launch_scan_t(const ScanLaunch& s, cudaStream_t st) {
  const int64_t BH = s.B * s.H;
  const bool vec_ok = (s.PN % 8 == 0) && aligned16(s.h_chunk) && aligned16(s.h_states) &&
                      aligned16(s.h_init) && aligned16(s.h_final) && aligned16(s.init_bx);
  if (vec_ok) {
    const int64_t nvec = s.PN / 8;
    // Two vectors per thread when one per thread would exceed one wave of resident threads.
    const int64_t resident = (int64_t)num_sms() * 2048;
    const bool two = BH * nvec > resident;
    const int vpt = two ? 2 : 1;
    const int64_t per_block = 256 * vpt;
    dim3 grid((unsigned)BH, (unsigned)((nvec + per_block - 1) / per_block));
    if (two)
      scan_fwd_vec_kernel<T, 2><<<grid, 256, 0, st>>>(s.decay, (const T*)s.h_chunk, s.h_init, s.init_bx,
                                                      s.init_coef, (T*)s.h_states, s.h_final, s.K, s.H, s.PN);
    else
      scan_fwd_vec_kernel<T, 1><<<grid, 256, 0, st>>>(s.decay, (const T*)s.h_chunk, s.h_init, s.init_bx,
                                                      s.init_coef, (T*)s.h_states, s.h_final, s.K, s.H, s.PN);
  } else {
    dim3 grid((unsigned)BH, (unsigned)((s.PN + 255) / 256));
    scan_fwd_scalar_kernel<T><<<grid, 256, 0, st>>>(s.decay, (const T*)s.h_chunk, s.h_init, s.init_bx,
                                                    s.init_coef, (T*)s.h_states, s.h_final, s.K, s.H, s.PN);
  }
  return check_launch("scan_fwd");
}

int launch_scan(const ScanLaunch& s, cudaStream_t st) {
  if (s.B <= 0 || s.K <= 0 || s.H <= 0 || s.PN <= 0) return M3B_OK;
  if (s.B * s.H > 0x7fffffffLL) return fail(M3B_ERR_INVALID_ARG, "scan: B*H too large");
  switch (s.dtype) {
    case M3B_F32: return launch_scan_t<float>(s, st);
    case M3B_BF16: return launch_scan_t<__nv_bfloat16>(s, st);
    default: return fail(M3B_ERR_INVALID_ARG, "scan: dtype must be f32 or bf16");
  }
}

}  // namespace m3b
