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

// VEC consecutive elements <-> VEC floats (VEC = 8: one 16- or 32-byte vector; VEC = 1: scalar)
template <typename T, int VEC>
__device__ __forceinline__ void ldv(const T* p, float (&v)[VEC]) {
  if constexpr (VEC == 8) load8<T>(p, v);
  else v[0] = io<T>::ld(p);
}
template <typename T, int VEC>
__device__ __forceinline__ void stv(T* p, const float (&v)[VEC]) {
  if constexpr (VEC == 8) store8<T>(p, v);
  else io<T>::st(p, v[0]);
}

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

// ---------------------------------------------------------------------------------------------
// Backward of the scan (semantics of mamba3/scan.py:47-62 and mamba3/csrc/scan.cu:52-126).
// With the carry g_{K-1} = grad_h[K-1] and g_k = grad_h[k] + decay[k] * g_{k+1} (k = K-2 .. 0):
//   d_chunk[k] = g_{k+1}, d_decay[k] = sum_j g_{k+1}[j] h_states[k][j]   (k < K-1; both 0 at K-1)
//   d_h_init   = g_0.
// Design: the forward's layout walked in reverse.  Block (bh, y) owns VPT vectors of VEC
// elements of one (batch, head) state; the loads of the next U chunks are issued before the
// carry chain consumes them.  d_decay is a sum over the whole state: each warp reduces its
// lanes with shuffles, the U per-chunk warp sums of a group meet in shared memory (double
// buffered, one barrier per group) and are added in warp order; with several blocks per
// state (gridDim.y > 1) every block writes its partial to part[y] and scan_bwd_reduce adds
// the partials in y order -- no atomics, so the result is bitwise reproducible.
template <typename T, int VEC, int VPT>
__global__ void __launch_bounds__(256) scan_bwd_kernel(const float* __restrict__ decay,
                                                       const T* __restrict__ hs, const T* __restrict__ gh,
                                                       T* __restrict__ dc, float* __restrict__ d_decay,
                                                       float* __restrict__ part, float* __restrict__ d_h_init,
                                                       int64_t K, int64_t H, int64_t PN) {
  constexpr int U = VPT == 2 ? 2 : 4;  // chunks whose loads are in flight together
  constexpr int NW = 256 / 32;
  __shared__ float red[2][U][NW];
  const int64_t bh = blockIdx.x;
  const int64_t b = bh / H, h = bh - b * H;
  const int64_t kstride = H * PN;
  const int64_t base = (b * K * H + h) * PN;
  const float* dptr = decay + b * K * H + h;
  // d_decay of (b, k, h) goes to d_decay directly (one block per state) or to this block's partials
  float* dout = gridDim.y == 1 ? d_decay + b * K * H + h : part + (int64_t)blockIdx.y * (gridDim.x * K) + b * K * H + h;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float g[VPT][VEC];
  int64_t j[VPT];
  bool act[VPT];
#pragma unroll
  for (int v = 0; v < VPT; ++v) {
    j[v] = ((int64_t)(blockIdx.y * VPT + v) * blockDim.x + threadIdx.x) * VEC;
    act[v] = j[v] < PN;
#pragma unroll
    for (int i = 0; i < VEC; ++i) g[v][i] = 0.f;
    if (act[v]) {
      const int64_t o = base + (K - 1) * kstride + j[v];
      ldv<T, VEC>(gh + o, g[v]);
      float z[VEC];
#pragma unroll
      for (int i = 0; i < VEC; ++i) z[i] = 0.f;
      stv<T, VEC>(dc + o, z);
    }
  }
  if (threadIdx.x == 0) dout[(K - 1) * H] = 0.f;
  int grp = 0;
  for (int64_t k0 = K - 2; k0 >= 0; k0 -= U, ++grp) {
    float xg[U][VPT][VEC], xh[U][VPT][VEC];
    float d[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t k = k0 - u;
      d[u] = k >= 0 ? __ldg(dptr + k * H) : 0.f;
#pragma unroll
      for (int v = 0; v < VPT; ++v) {
        if (k >= 0 && act[v]) {
          ldv<T, VEC>(gh + base + k * kstride + j[v], xg[u][v]);
          ldv<T, VEC>(hs + base + k * kstride + j[v], xh[u][v]);
        }
      }
    }
    float acc[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t k = k0 - u;
      acc[u] = 0.f;
      if (k >= 0) {
#pragma unroll
        for (int v = 0; v < VPT; ++v) {
          if (!act[v]) continue;
          stv<T, VEC>(dc + base + k * kstride + j[v], g[v]);
#pragma unroll
          for (int i = 0; i < VEC; ++i) {
            acc[u] = fmaf(g[v][i], xh[u][v][i], acc[u]);
            g[v][i] = fmaf(d[u], g[v][i], xg[u][v][i]);
          }
        }
      }
    }
    float* rb = &red[grp & 1][0][0];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      float s = acc[u];
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
      if (lane == 0) rb[u * NW + warp] = s;
    }
    __syncthreads();
    if (threadIdx.x < U && k0 - (int64_t)threadIdx.x >= 0) {
      float s = 0.f;
#pragma unroll
      for (int w = 0; w < NW; ++w) s += rb[threadIdx.x * NW + w];
      dout[(k0 - threadIdx.x) * H] = s;
    }
  }
  if (d_h_init) {
#pragma unroll
    for (int v = 0; v < VPT; ++v)
      if (act[v]) {
        float o[VEC];
#pragma unroll
        for (int i = 0; i < VEC; ++i) o[i] = g[v][i];
        stv<float, VEC>(d_h_init + bh * PN + j[v], o);
      }
  }
}

// d_decay[i] = sum over y of part[y][i], in y order
__global__ void __launch_bounds__(256) scan_bwd_reduce(const float* __restrict__ part, float* __restrict__ d_decay,
                                                       int64_t n, int nsplit) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float s = 0.f;
  for (int y = 0; y < nsplit; ++y) s += part[(int64_t)y * n + i];
  d_decay[i] = s;
}

namespace {
struct BwdShape {
  bool vec;
  int vpt;
  int64_t nsplit;
};
BwdShape bwd_shape(const ScanBwdLaunch& s) {
  BwdShape r{};
  r.vec = (s.PN % 8 == 0) && aligned16(s.h_states) && aligned16(s.grad_h) && aligned16(s.d_chunk) &&
          aligned16(s.d_h_init);
  const int64_t BH = s.B * s.H;
  if (r.vec) {
    const int64_t nvec = s.PN / 8;
    r.vpt = BH * nvec > (int64_t)num_sms() * 2048 ? 2 : 1;
    r.nsplit = (nvec + 256 * r.vpt - 1) / (256 * r.vpt);
  } else {
    r.vpt = 1;
    r.nsplit = (s.PN + 255) / 256;
  }
  return r;
}
}  // namespace

size_t scan_bwd_workspace(const ScanBwdLaunch& s) {
  if (s.B <= 0 || s.K <= 0 || s.H <= 0 || s.PN <= 0) return 0;
  const BwdShape r = bwd_shape(s);
  return r.nsplit > 1 ? (size_t)(r.nsplit * s.B * s.K * s.H) * sizeof(float) : 0;
}

template <typename T>
static int launch_scan_bwd_t(const ScanBwdLaunch& s, float* part, cudaStream_t st) {
  const BwdShape r = bwd_shape(s);
  const int64_t BH = s.B * s.H;
  dim3 grid((unsigned)BH, (unsigned)r.nsplit);
  const T* hs = static_cast<const T*>(s.h_states);
  const T* gh = static_cast<const T*>(s.grad_h);
  T* dc = static_cast<T*>(s.d_chunk);
  if (r.vec && r.vpt == 2)
    scan_bwd_kernel<T, 8, 2><<<grid, 256, 0, st>>>(s.decay, hs, gh, dc, s.d_decay, part, s.d_h_init, s.K, s.H, s.PN);
  else if (r.vec)
    scan_bwd_kernel<T, 8, 1><<<grid, 256, 0, st>>>(s.decay, hs, gh, dc, s.d_decay, part, s.d_h_init, s.K, s.H, s.PN);
  else
    scan_bwd_kernel<T, 1, 1><<<grid, 256, 0, st>>>(s.decay, hs, gh, dc, s.d_decay, part, s.d_h_init, s.K, s.H, s.PN);
  if (int rc = check_launch("scan_bwd")) return rc;
  if (r.nsplit > 1) {
    const int64_t n = s.B * s.K * s.H;
    scan_bwd_reduce<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(part, s.d_decay, n, (int)r.nsplit);
    return check_launch("scan_bwd_reduce");
  }
  return M3B_OK;
}

int launch_scan_bwd(const ScanBwdLaunch& s, void* ws, size_t ws_bytes, cudaStream_t st) {
  if (s.B <= 0 || s.K <= 0 || s.H <= 0 || s.PN <= 0) return M3B_OK;
  if (s.B * s.H > 0x7fffffffLL) return fail(M3B_ERR_INVALID_ARG, "scan_bwd: B*H too large");
  const size_t need = scan_bwd_workspace(s);
  if (need > 0 && (ws == nullptr || ws_bytes < need))
    return fail(M3B_ERR_INVALID_ARG, "scan_bwd: workspace of %zu bytes needed, %zu given", need, ws_bytes);
  if (need > 0 && !aligned16(ws)) return fail(M3B_ERR_INVALID_ARG, "scan_bwd: workspace must be 16-byte aligned");
  float* part = static_cast<float*>(ws);
  switch (s.dtype) {
    case M3B_F32: return launch_scan_bwd_t<float>(s, part, st);
    case M3B_BF16: return launch_scan_bwd_t<__nv_bfloat16>(s, part, st);
    default: return fail(M3B_ERR_INVALID_ARG, "scan_bwd: dtype must be f32 or bf16");
  }
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
