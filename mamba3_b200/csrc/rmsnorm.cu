// RMSNorm of the blocks around the SSM layer (mamba3/mamba3.py:19-35, used by
// mamba3/block.py:53,70,96-103 and the LM's final norm):
//   y = (x * rsqrt(mean(x^2) + eps)) * weight
// with the reference's rounding: the mean of squares in fp32, the scale rounded to the
// activation dtype, then two products in that dtype (each rounded once).
//
// x and y may be the same buffer (each lane reads its elements before writing them).
// Design: one warp per row; each lane owns d / 256 16-byte vectors (d % 8 == 0, bf16) or
// d / 32 scalars (any d), so the row is read once, reduced with shuffles, and written once.
// In torch the same norm is six kernels with an fp32 copy of the activations; at config-2
// size (64 x 2048 rows of 768) those took ~0.9 ms per norm against ~0.07 ms of traffic here.
#include <type_traits>

#include "common.cuh"
#include "launch.h"

namespace m3b {

namespace {

constexpr int kNormThreads = 256;
constexpr int kNormRowsPerBlock = kNormThreads / 32;
constexpr int kNormMaxVecPerLane = 8;  // d <= 2048 on the vector path

// a * b rounded to T (what one torch multiply of two T tensors stores)
template <typename T>
__device__ __forceinline__ float mul_rt(float a, float b) {
  if constexpr (std::is_same<T, float>::value) {
    return a * b;
  } else if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    return __bfloat162float(__float2bfloat16_rn(a * b));
  } else {
    return __half2float(__float2half_rn(a * b));
  }
}

template <typename T>
__device__ __forceinline__ float to_t(float a) {
  if constexpr (std::is_same<T, float>::value) return a;
  else if constexpr (std::is_same<T, __nv_bfloat16>::value) return __bfloat162float(__float2bfloat16_rn(a));
  else return __half2float(__float2half_rn(a));
}

// 16-bit activations, d % 8 == 0, 16-byte aligned rows: VPL vectors of 8 per lane
template <typename T, int VPL>
__global__ void __launch_bounds__(kNormThreads) rmsnorm_vec_kernel(const T* x, const T* __restrict__ w, T* y,
                                                                    int64_t rows, int d,
                                                                    float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kNormRowsPerBlock + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int nvec = d / 8;
  const T* xr = x + row * d;
  float v[VPL][8];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < VPL; ++k) {
    const int c = lane + 32 * k;
    if (c < nvec) {
      load8<T>(xr + 8 * c, v[k]);
#pragma unroll
      for (int e = 0; e < 8; ++e) ss = fmaf(v[k][e], v[k][e], ss);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float rms = to_t<T>(rsqrtf(ss / (float)d + eps));
  T* yr = y + row * d;
#pragma unroll
  for (int k = 0; k < VPL; ++k) {
    const int c = lane + 32 * k;
    if (c < nvec) {
      float wv[8], o[8];
      load8<T>(w + 8 * c, wv);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = mul_rt<T>(mul_rt<T>(v[k][e], rms), wv[e]);
      store8<T>(yr + 8 * c, o);
    }
  }
}

// The residual step before a norm, fused: x_out = x + h * scale (the product rounded to T, then
// the sum, as m3b_scaled_add stores it), y = RMSNorm(x_out) exactly as rmsnorm_vec_kernel computes
// it from the stored x_out (same lanes, same order of the sums).  x_out may alias x.
template <typename T, int VPL>
__global__ void __launch_bounds__(kNormThreads) add_rmsnorm_vec_kernel(const T* x, const T* h, float scale,
                                                                        const T* __restrict__ w, T* x_out, T* y,
                                                                        int64_t rows, int d, float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kNormRowsPerBlock + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int nvec = d / 8;
  const T* xr = x + row * d;
  const T* hr = h + row * d;
  T* xo = x_out + row * d;
  float v[VPL][8];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < VPL; ++k) {
    const int c = lane + 32 * k;
    if (c < nvec) {
      float hv[8];
      load8<T>(xr + 8 * c, v[k]);
      load8<T>(hr + 8 * c, hv);
#pragma unroll
      for (int e = 0; e < 8; ++e) v[k][e] = to_t<T>(v[k][e] + to_t<T>(hv[e] * scale));
      store8<T>(xo + 8 * c, v[k]);
#pragma unroll
      for (int e = 0; e < 8; ++e) ss = fmaf(v[k][e], v[k][e], ss);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float rms = to_t<T>(rsqrtf(ss / (float)d + eps));
  T* yr = y + row * d;
#pragma unroll
  for (int k = 0; k < VPL; ++k) {
    const int c = lane + 32 * k;
    if (c < nvec) {
      float wv[8], o[8];
      load8<T>(w + 8 * c, wv);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = mul_rt<T>(mul_rt<T>(v[k][e], rms), wv[e]);
      store8<T>(yr + 8 * c, o);
    }
  }
}

// any d / alignment / dtype: scalars, two passes over the row
template <typename T>
__global__ void __launch_bounds__(kNormThreads) rmsnorm_scalar_kernel(const T* x, const T* __restrict__ w,
                                                                       T* y,
                                                                       int64_t rows, int d, float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kNormRowsPerBlock + (threadIdx.x >> 5);
  if (row >= rows) return;
  const T* xr = x + row * d;
  float ss = 0.f;
  for (int c = lane; c < d; c += 32) {
    const float v = io<T>::ld(xr + c);
    ss = fmaf(v, v, ss);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float rms = to_t<T>(rsqrtf(ss / (float)d + eps));
  T* yr = y + row * d;
  for (int c = lane; c < d; c += 32)
    io<T>::st(yr + c, mul_rt<T>(mul_rt<T>(io<T>::ld(xr + c), rms), io<T>::ld(w + c)));
}

template <typename T>
int launch_norm_t(const void* x, const void* w, void* y, int64_t rows, int d, float eps, cudaStream_t st) {
  const unsigned grid = (unsigned)((rows + kNormRowsPerBlock - 1) / kNormRowsPerBlock);
  const T* xt = static_cast<const T*>(x);
  const T* wt = static_cast<const T*>(w);
  T* yt = static_cast<T*>(y);
  const bool vec = sizeof(T) == 2 && d % 8 == 0 && d / 8 <= 32 * kNormMaxVecPerLane && aligned16(x) &&
                   aligned16(w) && aligned16(y);
  if (vec) {
    const int vpl = (d / 8 + 31) / 32;
    if (vpl <= 1) rmsnorm_vec_kernel<T, 1><<<grid, kNormThreads, 0, st>>>(xt, wt, yt, rows, d, eps);
    else if (vpl <= 3) rmsnorm_vec_kernel<T, 3><<<grid, kNormThreads, 0, st>>>(xt, wt, yt, rows, d, eps);
    else rmsnorm_vec_kernel<T, kNormMaxVecPerLane><<<grid, kNormThreads, 0, st>>>(xt, wt, yt, rows, d, eps);
  } else {
    rmsnorm_scalar_kernel<T><<<grid, kNormThreads, 0, st>>>(xt, wt, yt, rows, d, eps);
  }
  return check_launch("rmsnorm");
}

template <typename T>
int launch_add_norm_t(const void* x, const void* h, float scale, const void* w, void* xo, void* y, int64_t rows,
                      int d, float eps, cudaStream_t st) {
  const unsigned grid = (unsigned)((rows + kNormRowsPerBlock - 1) / kNormRowsPerBlock);
  const T* xt = static_cast<const T*>(x);
  const T* ht = static_cast<const T*>(h);
  const T* wt = static_cast<const T*>(w);
  T* xot = static_cast<T*>(xo);
  T* yt = static_cast<T*>(y);
  const int vpl = (d / 8 + 31) / 32;
  if (vpl <= 1) add_rmsnorm_vec_kernel<T, 1><<<grid, kNormThreads, 0, st>>>(xt, ht, scale, wt, xot, yt, rows, d, eps);
  else if (vpl <= 3) add_rmsnorm_vec_kernel<T, 3><<<grid, kNormThreads, 0, st>>>(xt, ht, scale, wt, xot, yt, rows, d, eps);
  else add_rmsnorm_vec_kernel<T, kNormMaxVecPerLane><<<grid, kNormThreads, 0, st>>>(xt, ht, scale, wt, xot, yt, rows, d, eps);
  return check_launch("add_rmsnorm");
}

}  // namespace

}  // namespace m3b

extern "C" int m3b_add_rmsnorm(const void* x, const void* h, float scale, const void* weight, void* x_out, void* y,
                               int64_t rows, int32_t d, float eps, int32_t dtype, void* stream) {
  using namespace m3b;
  clear_error();
  if (rows < 0 || d <= 0) return fail(M3B_ERR_INVALID_ARG, "add_rmsnorm: bad shape");
  if (rows == 0) return M3B_OK;  // nothing to touch: the pointers may be null
  if (!x || !h || !weight || !x_out || !y) return fail(M3B_ERR_INVALID_ARG, "add_rmsnorm: null pointer");
  if (dtype != M3B_BF16 && dtype != M3B_F16) return fail(M3B_ERR_UNSUPPORTED, "add_rmsnorm: 16-bit dtypes only");
  if (d % 8 != 0 || d / 8 > 32 * kNormMaxVecPerLane)
    return fail(M3B_ERR_UNSUPPORTED, "add_rmsnorm: d must be a multiple of 8, at most %d", 256 * kNormMaxVecPerLane);
  if (!aligned16(x) || !aligned16(h) || !aligned16(weight) || !aligned16(x_out) || !aligned16(y))
    return fail(M3B_ERR_ALIGNMENT, "add_rmsnorm: 16-byte aligned rows required");
  if (rows == 0) return M3B_OK;
  if ((rows + kNormRowsPerBlock - 1) / kNormRowsPerBlock > 0x7fffffffLL)
    return fail(M3B_ERR_UNSUPPORTED, "add_rmsnorm: too many rows");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == M3B_BF16) return launch_add_norm_t<__nv_bfloat16>(x, h, scale, weight, x_out, y, rows, d, eps, st);
  return launch_add_norm_t<__half>(x, h, scale, weight, x_out, y, rows, d, eps, st);
}

extern "C" int m3b_rmsnorm(const void* x, const void* weight, void* y, int64_t rows, int32_t d, float eps,
                           int32_t dtype, void* stream) {
  using namespace m3b;
  clear_error();
  if (rows < 0 || d <= 0) return fail(M3B_ERR_INVALID_ARG, "rmsnorm: bad shape");
  if (rows == 0) return M3B_OK;  // nothing to touch: the pointers may be null
  if (!x || !weight || !y) return fail(M3B_ERR_INVALID_ARG, "rmsnorm: null pointer");
  if ((rows + kNormRowsPerBlock - 1) / kNormRowsPerBlock > 0x7fffffffLL)
    return fail(M3B_ERR_UNSUPPORTED, "rmsnorm: too many rows");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case M3B_F32: return launch_norm_t<float>(x, weight, y, rows, d, eps, st);
    case M3B_BF16: return launch_norm_t<__nv_bfloat16>(x, weight, y, rows, d, eps, st);
    case M3B_F16: return launch_norm_t<__half>(x, weight, y, rows, d, eps, st);
    default: return fail(M3B_ERR_INVALID_ARG, "rmsnorm: dtype");
  }
}
