// Gate and MIMO down-projection of the layer (mamba3/mamba3.py:234-238) as used by the
// training path, forward and backward, for rows of (H*P) channels with R ranks each:
//   out[c]   = sum_r y[c,r] * silu(z[c] * mz[c,r]) * md[c,r]            (c = (h, p))
//   dy[c,r]  = dout[c] * silu(u_r) * md[c,r]                            (u_r = z[c] mz[c,r])
//   dz[c]    = sum_r dout[c] y[c,r] md[c,r] silu'(u_r) mz[c,r]
//   dmz[c,r] = sum over rows of dout[c] y[c,r] md[c,r] silu'(u_r) z[c]
//   dmd[c,r] = sum over rows of dout[c] y[c,r] silu(u_r)
// silu'(u) = s (1 + u (1 - s)), s = sigmoid(u).  fp32 arithmetic; the parameter gradients are
// summed per row chunk into partials and the partials in chunk order (no atomics).  In torch
// these are broadcast products and sums over the rank or (batch, token) dimensions, a dozen
// passes over (B, T, H, P, R) tensors.
#include "common.cuh"
#include "launch.h"

namespace m3b {

namespace {

constexpr int kGateThreads = 256;
constexpr int kGateRows = 128;  // rows per chunk of the backward

__device__ __forceinline__ float sigm(float u) { return 1.f / (1.f + expf(-u)); }

template <typename T, int R>
__global__ void __launch_bounds__(kGateThreads) gate_fwd_kernel(const T* __restrict__ y, const T* __restrict__ z,
                                                                const T* __restrict__ mz, const T* __restrict__ md,
                                                                T* __restrict__ out, int64_t rows, int64_t zs, int C) {
  const int c = blockIdx.x * kGateThreads + threadIdx.x;
  if (c >= C) return;
  float wz[R], wd[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    wz[r] = io<T>::ld(mz + (int64_t)c * R + r);
    wd[r] = io<T>::ld(md + (int64_t)c * R + r);
  }
  for (int64_t row = blockIdx.y; row < rows; row += gridDim.y) {
    const int64_t i = row * C + c;
    const float zv = io<T>::ld(z + row * zs + c);
    float acc = 0.f;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const float u = zv * wz[r];
      acc = fmaf(io<T>::ld(y + i * R + r) * (u * sigm(u)), wd[r], acc);
    }
    io<T>::st(out + i, acc);
  }
}

template <typename T, int R>
__global__ void __launch_bounds__(kGateThreads) gate_bwd_kernel(const T* __restrict__ y, const T* __restrict__ z,
                                                                const T* __restrict__ mz, const T* __restrict__ md,
                                                                const T* __restrict__ dout, T* __restrict__ dy,
                                                                T* __restrict__ dz, float* __restrict__ part,
                                                                int64_t rows, int64_t zs, int C) {
  const int c = blockIdx.x * kGateThreads + threadIdx.x;
  if (c >= C) return;
  float wz[R], wd[R], gz[R], gd[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    wz[r] = io<T>::ld(mz + (int64_t)c * R + r);
    wd[r] = io<T>::ld(md + (int64_t)c * R + r);
    gz[r] = gd[r] = 0.f;
  }
  const int64_t r0 = (int64_t)blockIdx.y * kGateRows;
  const int64_t r1 = r0 + kGateRows < rows ? r0 + kGateRows : rows;
  for (int64_t row = r0; row < r1; ++row) {
    const int64_t i = row * C + c;
    const float zv = io<T>::ld(z + row * zs + c), g = io<T>::ld(dout + i);
    float dzv = 0.f;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const float yv = io<T>::ld(y + i * R + r);
      const float u = zv * wz[r], s = sigm(u), si = u * s;
      const float ds = s * (1.f + u * (1.f - s));  // silu'(u)
      io<T>::st(dy + i * R + r, g * si * wd[r]);
      const float t = g * yv * wd[r] * ds;
      dzv = fmaf(t, wz[r], dzv);
      gz[r] = fmaf(t, zv, gz[r]);
      gd[r] = fmaf(g * yv, si, gd[r]);
    }
    io<T>::st(dz + i, dzv);
  }
  float* pc = part + ((int64_t)blockIdx.y * C + c) * 2 * R;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    pc[r] = gz[r];
    pc[R + r] = gd[r];
  }
}

// dmz / dmd = sums of the chunk partials in chunk order
template <typename T, int R>
__global__ void gate_param_sums(const float* __restrict__ part, T* __restrict__ dmz, T* __restrict__ dmd,
                                int64_t nchunks, int C) {
  const int e = blockIdx.x * blockDim.x + threadIdx.x;  // (c, r)
  if (e >= C * R) return;
  const int c = e / R, r = e - c * R;
  float sz = 0.f, sd = 0.f;
  for (int64_t k = 0; k < nchunks; ++k) {
    const float* pc = part + (k * C + c) * 2 * R;
    sz += pc[r];
    sd += pc[R + r];
  }
  io<T>::st(dmz + e, sz);
  io<T>::st(dmd + e, sd);
}

int64_t zstride(const m3b_gate_args* a) { return a->z_stride ? a->z_stride : a->channels; }

template <typename T, int R>
int gate_fwd_t(const m3b_gate_args* a, cudaStream_t st) {
  const int C = a->channels;
  const int64_t ychunks = a->rows < 4096 ? a->rows : 4096;
  dim3 grid((unsigned)((C + kGateThreads - 1) / kGateThreads), (unsigned)(ychunks > 0 ? ychunks : 1));
  gate_fwd_kernel<T, R><<<grid, kGateThreads, 0, st>>>(
      static_cast<const T*>(a->y), static_cast<const T*>(a->z), static_cast<const T*>(a->mimo_z),
      static_cast<const T*>(a->mimo_down), static_cast<T*>(a->out), a->rows, zstride(a), C);
  return check_launch("gate_fwd");
}

template <typename T, int R>
int gate_bwd_t(const m3b_gate_args* a, float* part, cudaStream_t st) {
  const int C = a->channels;
  const int64_t nchunks = (a->rows + kGateRows - 1) / kGateRows;
  if (nchunks > 65535)  // one grid row per chunk of rows; gridDim.y is at most 65535
    return fail(M3B_ERR_UNSUPPORTED, "gate_bwd: %lld rows exceed %lld (65535 chunks of %d rows)",
                (long long)a->rows, 65535LL * kGateRows, kGateRows);
  if (nchunks > 0) {
    dim3 grid((unsigned)((C + kGateThreads - 1) / kGateThreads), (unsigned)nchunks);
    gate_bwd_kernel<T, R><<<grid, kGateThreads, 0, st>>>(
        static_cast<const T*>(a->y), static_cast<const T*>(a->z), static_cast<const T*>(a->mimo_z),
        static_cast<const T*>(a->mimo_down), static_cast<const T*>(a->dout), static_cast<T*>(a->dy),
        static_cast<T*>(a->dz), part, a->rows, zstride(a), C);
    const int rc = check_launch("gate_bwd");
    if (rc != M3B_OK) return rc;
  }
  gate_param_sums<T, R><<<(unsigned)((C * R + 255) / 256), 256, 0, st>>>(
      part, static_cast<T*>(a->d_mimo_z), static_cast<T*>(a->d_mimo_down), nchunks, C);
  return check_launch("gate_param_sums");
}

template <int R>
int gate_dispatch(const m3b_gate_args* a, bool bwd, float* part, cudaStream_t st) {
  switch (a->dtype) {
    case M3B_F32: return bwd ? gate_bwd_t<float, R>(a, part, st) : gate_fwd_t<float, R>(a, st);
    case M3B_BF16: return bwd ? gate_bwd_t<__nv_bfloat16, R>(a, part, st) : gate_fwd_t<__nv_bfloat16, R>(a, st);
    case M3B_F16: return bwd ? gate_bwd_t<__half, R>(a, part, st) : gate_fwd_t<__half, R>(a, st);
    default: return fail(M3B_ERR_INVALID_ARG, "gate: dtype");
  }
}

int gate_run(const m3b_gate_args* a, bool bwd, void* ws, size_t ws_bytes, cudaStream_t st) {
  if (!a) return fail(M3B_ERR_INVALID_ARG, "gate: null args");
  if (a->rows < 0 || a->channels <= 0 || (a->z_stride != 0 && a->z_stride < a->channels))
    return fail(M3B_ERR_INVALID_ARG, "gate: bad shape");
  // per-row operands may be null when there are no rows; the parameter gradients are then zeros
  const bool has_rows = a->rows > 0;
  if (!a->mimo_z || !a->mimo_down || (bwd && (!a->d_mimo_z || !a->d_mimo_down)))
    return fail(M3B_ERR_INVALID_ARG, "gate: null pointer");
  if (has_rows && (!a->y || !a->z || (bwd ? (!a->dout || !a->dy || !a->dz) : !a->out)))
    return fail(M3B_ERR_INVALID_ARG, "gate: null pointer");
  if (!has_rows && !bwd) return M3B_OK;
  if ((a->rows + kGateRows - 1) / kGateRows > 0x7fffffffLL) return fail(M3B_ERR_UNSUPPORTED, "gate: too many rows");
  if (bwd) {
    const size_t need = (size_t)((a->rows + kGateRows - 1) / kGateRows) * a->channels * 2 * a->R * sizeof(float);
    if (has_rows && (!ws || ws_bytes < need)) return fail(M3B_ERR_WORKSPACE, "gate_bwd: need %zu workspace bytes", need);
  }
  float* part = static_cast<float*>(ws);
  switch (a->R) {
    case 1: return gate_dispatch<1>(a, bwd, part, st);
    case 2: return gate_dispatch<2>(a, bwd, part, st);
    case 3: return gate_dispatch<3>(a, bwd, part, st);
    case 4: return gate_dispatch<4>(a, bwd, part, st);
    default: return fail(M3B_ERR_UNSUPPORTED, "gate: mimo_rank %d (1..4)", a->R);
  }
}

}  // namespace

}  // namespace m3b

extern "C" size_t m3b_gate_bwd_workspace(const m3b_gate_args* a) {
  if (!a || a->rows <= 0 || a->channels <= 0 || a->R <= 0) return 0;
  return (size_t)((a->rows + m3b::kGateRows - 1) / m3b::kGateRows) * a->channels * 2 * a->R * sizeof(float);
}

extern "C" int m3b_gate_fwd(const m3b_gate_args* a, void* stream) {
  m3b::clear_error();
  return m3b::gate_run(a, false, nullptr, 0, static_cast<cudaStream_t>(stream));
}

extern "C" int m3b_gate_bwd(const m3b_gate_args* a, void* workspace, size_t workspace_bytes, void* stream) {
  m3b::clear_error();
  return m3b::gate_run(a, true, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}
