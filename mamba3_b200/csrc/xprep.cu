// MIMO expansion and trapezoid weights of x (mamba3/mamba3.py:218-230) for the training path,
// forward and backward.  Per token row (b, t), head h, channel p and rank r:
//   x_raw[t, h, p, r] = xf[t, h, p] mx[h, p, r]
//   lam[t, h] = sigmoid(lam_raw[t, h]),  sb[t, h] = (1 - lam) exp(A[h] dt[t, h])
//   x_g[t] = x_raw[t] lam[t],  x_b[t] = x_raw[t - 1] sb[t],  x_b[0] = 0           (trapezoid)
// Backward, with dx_r[t] = dx_raw[t] + dx_g[t] lam[t] + dx_b[t + 1] sb[t + 1]:
//   dxf = sum_r dx_r mx,  dmx = sum over rows of dx_r xf,
//   dlam = sum_{p,r} dx_g x_raw - e sum_{p,r} dx_b[t] x_raw[t - 1]  (e = exp(A dt)),
//   dlam_raw = dlam lam (1 - lam),  with ds = sum_{p,r} dx_b x_raw[t-1] (1 - lam) e:
//   ddt = ds A,  dA = sum over rows of ds dt.
// A CTA covers whole heads (floor(256 / P) of them, one thread per channel) and a chunk of 64
// rows; the sums over (p, r) of a row run by warp shuffles and shared memory (or, when P is not
// a multiple of 32, in channel order by one thread per head), the sums over rows per chunk and
// then over chunks in chunk order: no atomics, bitwise reproducible.  fp32
// arithmetic; torch builds these with a dozen broadcast passes over (B, T, H, P, R) tensors.
#include "common.cuh"
#include "launch.h"

namespace m3b {

namespace {

constexpr int kXThreads = 256;
constexpr int kXRows = 64;

struct XParams {
  int64_t rows, T, xs, ls;  // rows = batch * seqlen; row strides of xf and lam_raw
  int H, P, R, C, hpc, cpb, nrc;
  int trap, dtype, dt_dtype, a_dtype;
  const void *xf, *mx, *lam, *dt, *A;
  void *x_raw, *x_g, *x_b;
  const void *dx_raw, *dx_g, *dx_b;
  void *dxf, *dmx, *dlam, *ddt, *dA;
  float* pmx;  // (nrc, C * R)
  float* pA;   // (nrc, H)
};

__device__ __forceinline__ float x_sigm(float u) { return 1.f / (1.f + expf(-u)); }

template <typename T, int R>
__global__ void __launch_bounds__(kXThreads) xprep_fwd_kernel(XParams p) {
  const int tid = threadIdx.x;
  const int c = blockIdx.x * p.cpb + tid;
  if (tid >= p.cpb || c >= p.C) return;
  const int h = c / p.P;
  float m[R];
#pragma unroll
  for (int r = 0; r < R; ++r) m[r] = io<T>::ld(static_cast<const T*>(p.mx) + (int64_t)c * R + r);
  const T* xf = static_cast<const T*>(p.xf);
  const T* lr = static_cast<const T*>(p.lam);
  const float Ah = p.trap ? ldf(p.A, h, p.a_dtype) : 0.f;
  const int64_t r0 = (int64_t)blockIdx.y * kXRows, r1 = r0 + kXRows < p.rows ? r0 + kXRows : p.rows;
  int64_t t = r0 % p.T;
  float xprev = (p.trap && t > 0) ? io<T>::ld(xf + (r0 - 1) * p.xs + c) : 0.f;
  for (int64_t row = r0; row < r1; ++row) {
    const float x = io<T>::ld(xf + row * p.xs + c);
    const int64_t o = (row * p.C + c) * R;
#pragma unroll
    for (int r = 0; r < R; ++r) io<T>::st(static_cast<T*>(p.x_raw) + o + r, x * m[r]);
    if (p.trap) {
      const float lam = x_sigm(io<T>::ld(lr + row * p.ls + h));
      const float sb = (1.f - lam) * expf(Ah * ldf(p.dt, row * p.H + h, p.dt_dtype));
#pragma unroll
      for (int r = 0; r < R; ++r) {
        io<T>::st(static_cast<T*>(p.x_g) + o + r, x * m[r] * lam);
        io<T>::st(static_cast<T*>(p.x_b) + o + r, t == 0 ? 0.f : xprev * m[r] * sb);
      }
    }
    xprev = x;
    if (++t == p.T) t = 0;
  }
}

template <typename T, int R>
__global__ void __launch_bounds__(kXThreads) xprep_bwd_kernel(XParams p) {
  __shared__ float sl[kXThreads], ss[kXThreads];
  const int tid = threadIdx.x;
  const int c = blockIdx.x * p.cpb + tid;
  const bool active = tid < p.cpb && c < p.C;
  const int h = active ? c / p.P : 0;
  const T* xf = static_cast<const T*>(p.xf);
  const T* lr = static_cast<const T*>(p.lam);
  const T* dxr_in = static_cast<const T*>(p.dx_raw);
  const T* dxg_in = static_cast<const T*>(p.dx_g);
  const T* dxb_in = static_cast<const T*>(p.dx_b);
  float m[R], gm[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    m[r] = active ? io<T>::ld(static_cast<const T*>(p.mx) + (int64_t)c * R + r) : 0.f;
    gm[r] = 0.f;
  }
  // per-head finishing thread: head hl = tid of this CTA's heads
  const int hf = blockIdx.x * p.hpc + tid;
  const bool fin = p.trap && tid < p.hpc && hf < p.H;
  const float Ah = p.trap ? ldf(p.A, active ? h : 0, p.a_dtype) : 0.f;
  const float Af = fin ? ldf(p.A, hf, p.a_dtype) : 0.f;
  float accA = 0.f;
  const int64_t r0 = (int64_t)blockIdx.y * kXRows, r1 = r0 + kXRows < p.rows ? r0 + kXRows : p.rows;
  int64_t t = r0 % p.T;
  float xprev = (active && p.trap && t > 0) ? io<T>::ld(xf + (r0 - 1) * p.xs + c) : 0.f;
  for (int64_t row = r0; row < r1; ++row) {
    float x = 0.f, gl = 0.f, gs = 0.f;
    if (active) {
      x = io<T>::ld(xf + row * p.xs + c);
      const int64_t o = (row * p.C + c) * R;
      float lam = 0.f, sbn = 0.f;
      const bool nxt = p.trap && t + 1 < p.T;
      if (p.trap) lam = x_sigm(io<T>::ld(lr + row * p.ls + h));
      if (nxt) {
        const float ln = x_sigm(io<T>::ld(lr + (row + 1) * p.ls + h));
        sbn = (1.f - ln) * expf(Ah * ldf(p.dt, (row + 1) * p.H + h, p.dt_dtype));
      }
      float dxf = 0.f;
#pragma unroll
      for (int r = 0; r < R; ++r) {
        float d = io<T>::ld(dxr_in + o + r);
        if (p.trap) {
          const float dg = io<T>::ld(dxg_in + o + r);
          d = fmaf(dg, lam, d);
          gl = fmaf(dg, m[r], gl);
          if (nxt) d = fmaf(io<T>::ld(dxb_in + o + (int64_t)p.C * R + r), sbn, d);
          if (t > 0) gs = fmaf(io<T>::ld(dxb_in + o + r), m[r], gs);
        }
        dxf = fmaf(d, m[r], dxf);
        gm[r] = fmaf(d, x, gm[r]);
      }
      io<T>::st(static_cast<T*>(p.dxf) + row * p.C + c, dxf);
    }
    if (p.trap) {
      // per head: the sums over its P channels -- by warp shuffles when whole warps fall in a
      // head (P a multiple of 32; then the warp sums in warp order), else one thread in channel order
      const bool by_warp = p.P % 32 == 0;
      int q0 = tid * p.P, q1 = (tid + 1) * p.P;
      if (by_warp) {
        float u = gl * x, v = gs * xprev;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
          u += __shfl_xor_sync(0xffffffffu, u, off);
          v += __shfl_xor_sync(0xffffffffu, v, off);
        }
        if ((tid & 31) == 0) {
          sl[tid >> 5] = u;
          ss[tid >> 5] = v;
        }
        q0 = tid * (p.P / 32);
        q1 = (tid + 1) * (p.P / 32);
      } else {
        sl[tid] = gl * x;
        ss[tid] = gs * xprev;
      }
      __syncthreads();
      if (fin) {
        float DL = 0.f, DS = 0.f;
        for (int q = q0; q < q1; ++q) {
          DL += sl[q];
          DS += ss[q];
        }
        const float lam = x_sigm(io<T>::ld(lr + row * p.ls + hf));
        const float dtv = ldf(p.dt, row * p.H + hf, p.dt_dtype);
        const float e = expf(Af * dtv);
        io<T>::st(static_cast<T*>(p.dlam) + row * p.H + hf, (DL - DS * e) * lam * (1.f - lam));
        const float ds = DS * (1.f - lam) * e;
        stf(p.ddt, row * p.H + hf, p.dt_dtype, ds * Af);
        accA = fmaf(ds, dtv, accA);
      }
      __syncthreads();
    }
    xprev = x;
    if (++t == p.T) t = 0;
  }
  if (active) {
#pragma unroll
    for (int r = 0; r < R; ++r) p.pmx[(int64_t)blockIdx.y * p.C * R + (int64_t)c * R + r] = gm[r];
  }
  if (fin) p.pA[(int64_t)blockIdx.y * p.H + hf] = accA;
}

// out[e] = sum over q < nq of part[q * ne + e]: a CTA takes 32 elements, its 8 warps sum the q
// of their residue (mod 8) in q order, and the warp sums are added in warp order
__global__ void __launch_bounds__(kXThreads) xprep_colsum(const float* __restrict__ part, int64_t nq, int ne,
                                                          void* out, int dtype) {
  __shared__ float red[kXThreads / 32][32];
  const int lane = threadIdx.x & 31, seg = threadIdx.x >> 5;
  const int e = blockIdx.x * 32 + lane;
  float s = 0.f;
  if (e < ne)
    for (int64_t q = seg; q < nq; q += kXThreads / 32) s += part[q * ne + e];
  red[seg][lane] = s;
  __syncthreads();
  if (seg != 0 || e >= ne) return;
  float v = 0.f;
  for (int w = 0; w < kXThreads / 32; ++w) v += red[w][lane];
  stf(out, e, dtype, v);
}

struct XLayout {
  size_t pmx, pA, total;
};

XLayout x_layout(const m3b_xprep_args* a) {
  auto up = [](size_t x) { return (x + 255) & ~(size_t)255; };
  const size_t rows = (size_t)a->batch * a->seqlen;
  const size_t nrc = (rows + kXRows - 1) / kXRows;
  XLayout w{};
  w.pmx = 0;
  w.pA = up(nrc * (size_t)a->H * a->P * a->R * sizeof(float));
  w.total = w.pA + (a->trapezoidal ? up(nrc * (size_t)a->H * sizeof(float)) : 0);
  return w;
}

int x_validate(const m3b_xprep_args* a, bool bwd) {
  if (!a) return fail(M3B_ERR_INVALID_ARG, "xprep: null args");
  if (a->batch < 0 || a->seqlen < 0 || a->H <= 0 || a->P <= 0 || a->R <= 0)
    return fail(M3B_ERR_INVALID_ARG, "xprep: bad dims");
  if (a->P > kXThreads || a->R > 4) return fail(M3B_ERR_UNSUPPORTED, "xprep: needs P <= 256, R <= 4");
  for (int d : {a->dtype, a->dt_dtype, a->a_dtype})
    if (d != M3B_F32 && d != M3B_BF16 && d != M3B_F16) return fail(M3B_ERR_UNSUPPORTED, "xprep: dtype");
  const int64_t C = (int64_t)a->H * a->P;
  if ((a->x_stride != 0 && a->x_stride < C) || (a->lam_stride != 0 && a->lam_stride < a->H))
    return fail(M3B_ERR_INVALID_ARG, "xprep: row stride below the row width");
  const int64_t rows = a->batch * a->seqlen;
  if ((rows + kXRows - 1) / kXRows > 65535) return fail(M3B_ERR_UNSUPPORTED, "xprep: more than %d rows", 65535 * kXRows);
  if (!a->mimo_x || (bwd && !a->dmimo_x)) return fail(M3B_ERR_INVALID_ARG, "xprep: null parameter");
  if (a->trapezoidal && (!a->A || (bwd && !a->dA))) return fail(M3B_ERR_INVALID_ARG, "xprep: null A");
  if (rows > 0) {
    if (!a->xf || (a->trapezoidal && (!a->lam_raw || !a->dt))) return fail(M3B_ERR_INVALID_ARG, "xprep: null input");
    if (!bwd && (!a->x_raw || (a->trapezoidal && (!a->x_g || !a->x_b))))
      return fail(M3B_ERR_INVALID_ARG, "xprep: null output");
    if (bwd && (!a->dx_raw || !a->dxf || (a->trapezoidal && (!a->dx_g || !a->dx_b || !a->dlam_raw || !a->ddt))))
      return fail(M3B_ERR_INVALID_ARG, "xprep: null gradient");
  }
  return M3B_OK;
}

template <typename T, int R>
int x_run_t(const XParams& p, bool bwd, cudaStream_t st) {
  const dim3 grid((unsigned)((p.H + p.hpc - 1) / p.hpc), (unsigned)p.nrc);
  if (!bwd) {
    xprep_fwd_kernel<T, R><<<grid, kXThreads, 0, st>>>(p);
    return check_launch("xprep_fwd");
  }
  xprep_bwd_kernel<T, R><<<grid, kXThreads, 0, st>>>(p);
  int rc = check_launch("xprep_bwd");
  if (rc != M3B_OK) return rc;
  xprep_colsum<<<(unsigned)((p.C * R + 31) / 32), kXThreads, 0, st>>>(p.pmx, p.nrc, p.C * R, p.dmx, p.dtype);
  if ((rc = check_launch("xprep_colsum")) != M3B_OK) return rc;
  if (p.trap) {
    xprep_colsum<<<(unsigned)((p.H + 31) / 32), kXThreads, 0, st>>>(p.pA, p.nrc, p.H, p.dA, p.a_dtype);
    rc = check_launch("xprep_colsum");
  }
  return rc;
}

template <typename T>
int x_dispatch(const XParams& p, bool bwd, cudaStream_t st) {
  switch (p.R) {
    case 1: return x_run_t<T, 1>(p, bwd, st);
    case 2: return x_run_t<T, 2>(p, bwd, st);
    case 3: return x_run_t<T, 3>(p, bwd, st);
    default: return x_run_t<T, 4>(p, bwd, st);
  }
}

int x_run(const m3b_xprep_args* a, bool bwd, void* ws, size_t ws_bytes, cudaStream_t st) {
  int rc = x_validate(a, bwd);
  if (rc != M3B_OK) return rc;
  const int64_t rows = a->batch * a->seqlen;
  const size_t es = [](int d) { return d == M3B_F32 ? (size_t)4 : (size_t)2; }(a->dtype);
  if (rows == 0) {
    if (!bwd) return M3B_OK;
    // no tokens: zero parameter gradients
    if (cudaMemsetAsync(a->dmimo_x, 0, (size_t)a->H * a->P * a->R * es, st) != cudaSuccess ||
        (a->trapezoidal && cudaMemsetAsync(a->dA, 0, (size_t)a->H * (a->a_dtype == M3B_F32 ? 4 : 2), st) != cudaSuccess))
      return fail(M3B_ERR_CUDA, "xprep: memset");
    return M3B_OK;
  }
  const XLayout w = x_layout(a);
  if (bwd && (!ws || ws_bytes < w.total)) return fail(M3B_ERR_WORKSPACE, "xprep_bwd: need %zu workspace bytes", w.total);
  XParams p{};
  p.rows = rows;
  p.T = a->seqlen;
  p.H = a->H;
  p.P = a->P;
  p.R = a->R;
  p.C = a->H * a->P;
  p.xs = a->x_stride ? a->x_stride : p.C;
  p.ls = a->lam_stride ? a->lam_stride : a->H;
  p.hpc = kXThreads / a->P;
  p.cpb = p.hpc * a->P;
  p.nrc = (int)((rows + kXRows - 1) / kXRows);
  p.trap = a->trapezoidal != 0;
  p.dtype = a->dtype;
  p.dt_dtype = a->dt_dtype;
  p.a_dtype = a->a_dtype;
  p.xf = a->xf;
  p.mx = a->mimo_x;
  p.lam = a->lam_raw;
  p.dt = a->dt;
  p.A = a->A;
  p.x_raw = a->x_raw;
  p.x_g = a->x_g;
  p.x_b = a->x_b;
  p.dx_raw = a->dx_raw;
  p.dx_g = a->dx_g;
  p.dx_b = a->dx_b;
  p.dxf = a->dxf;
  p.dmx = a->dmimo_x;
  p.dlam = a->dlam_raw;
  p.ddt = a->ddt;
  p.dA = a->dA;
  p.pmx = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + w.pmx);
  p.pA = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + w.pA);
  switch (a->dtype) {
    case M3B_F32: return x_dispatch<float>(p, bwd, st);
    case M3B_BF16: return x_dispatch<__nv_bfloat16>(p, bwd, st);
    default: return x_dispatch<__half>(p, bwd, st);
  }
}

}  // namespace

}  // namespace m3b

extern "C" size_t m3b_xprep_bwd_workspace(const m3b_xprep_args* a) {
  if (m3b::x_validate(a, true) != M3B_OK) return 0;
  return m3b::x_layout(a).total;
}

extern "C" int m3b_xprep_fwd(const m3b_xprep_args* a, void* stream) {
  m3b::clear_error();
  return m3b::x_run(a, false, nullptr, 0, static_cast<cudaStream_t>(stream));
}

extern "C" int m3b_xprep_bwd(const m3b_xprep_args* a, void* workspace, size_t workspace_bytes, void* stream) {
  m3b::clear_error();
  return m3b::x_run(a, true, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}
