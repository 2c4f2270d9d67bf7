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

}  // namespace

}  // namespace m3b

extern "C" int m3b_rmsnorm(const void* x, const void* weight, void* y, int64_t rows, int32_t d, float eps,
                           int32_t dtype, void* stream) {
  using namespace m3b;
  clear_error();
  if (!x || !weight || !y) return fail(M3B_ERR_INVALID_ARG, "rmsnorm: null pointer");
  if (rows < 0 || d <= 0) return fail(M3B_ERR_INVALID_ARG, "rmsnorm: bad shape");
  if (rows == 0) return M3B_OK;
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
