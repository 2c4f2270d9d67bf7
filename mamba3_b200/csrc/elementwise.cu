// Two element-wise steps of the blocks around the SSM layer, each one pass instead of torch's
// two kernels (with the reference's rounding: every torch op stores its result in the
// activation dtype, so each intermediate is rounded once here as well):
//   swiglu_act:  out = silu(g) * u                 (mamba3/block.py:16-26, SwiGLU.forward)
//   scaled_add:  out = x + h * scale               (mamba3/block.py:79-107, the residuals)
// 16-byte vectors when the element count is a multiple of 8 and the buffers are aligned.
// Outputs may alias inputs (every element is read before it is written, by the same thread).
#include <type_traits>

#include "common.cuh"
#include "launch.h"

namespace m3b {

namespace {

constexpr int kEwThreads = 256;

template <typename T>
__device__ __forceinline__ float rnd(float a) {
  if constexpr (std::is_same<T, float>::value) return a;
  else if constexpr (std::is_same<T, __nv_bfloat16>::value) return __bfloat162float(__float2bfloat16_rn(a));
  else return __half2float(__float2half_rn(a));
}

struct SwigluOp {
  template <typename T>
  __device__ __forceinline__ float operator()(float g, float u, float) const {
    const float s = rnd<T>(g / (1.f + expf(-g)));
    return s * u;
  }
};

struct ScaledAddOp {
  template <typename T>
  __device__ __forceinline__ float operator()(float x, float h, float scale) const {
    return x + rnd<T>(h * scale);
  }
};

template <typename T, typename Op, bool VEC>
__global__ void __launch_bounds__(kEwThreads) ew2_kernel(const T* a, const T* b, T* out, int64_t n, float scale) {
  const Op op;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  if constexpr (VEC) {
    const int64_t nv = n / 8;
    for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < nv; v += stride) {
      float av[8], bv[8], o[8];
      load8<T>(a + 8 * v, av);
      load8<T>(b + 8 * v, bv);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = op.template operator()<T>(av[e], bv[e], scale);
      store8<T>(out + 8 * v, o);
    }
  } else {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
      io<T>::st(out + i, op.template operator()<T>(io<T>::ld(a + i), io<T>::ld(b + i), scale));
  }
}

// silu(g) * u over rows of one GEMM output [g (f) | u (f)] (the gate and up projections of the
// SwiGLU computed as one GEMM): out (rows, f).  16-byte vectors, f % 8 == 0.
template <typename T>
__global__ void __launch_bounds__(kEwThreads) swiglu_rows_kernel(const T* gu, T* out, int64_t rows, int f) {
  const SwigluOp op;
  const int fv = f / 8;
  const int64_t nv = rows * fv;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < nv; v += stride) {
    const int64_t r = v / fv;
    const int c = (int)(v - r * fv);
    float gv[8], uv[8], o[8];
    load8<T>(gu + r * 2 * f + 8 * c, gv);
    load8<T>(gu + r * 2 * f + f + 8 * c, uv);
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = op.template operator()<T>(gv[e], uv[e], 0.f);
    store8<T>(out + r * f + 8 * c, o);
  }
}

template <typename T, typename Op>
int launch_ew2(const void* a, const void* b, void* out, int64_t n, float scale, cudaStream_t st, const char* what) {
  const bool vec = n % 8 == 0 && aligned16(a) && aligned16(b) && aligned16(out);
  const int64_t units = vec ? n / 8 : n;
  int64_t blocks = (units + kEwThreads - 1) / kEwThreads;
  const int64_t cap = (int64_t)num_sms() * 16;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  const T* at = static_cast<const T*>(a);
  const T* bt = static_cast<const T*>(b);
  T* ot = static_cast<T*>(out);
  if (vec) ew2_kernel<T, Op, true><<<(unsigned)blocks, kEwThreads, 0, st>>>(at, bt, ot, n, scale);
  else ew2_kernel<T, Op, false><<<(unsigned)blocks, kEwThreads, 0, st>>>(at, bt, ot, n, scale);
  return check_launch(what);
}

template <typename Op>
int dispatch_ew2(const void* a, const void* b, void* out, int64_t n, float scale, int32_t dtype, void* stream,
                 const char* what) {
  if (n < 0) return fail(M3B_ERR_INVALID_ARG, "%s: negative size", what);
  if (n == 0) return M3B_OK;  // nothing to touch: the pointers may be null
  if (!a || !b || !out) return fail(M3B_ERR_INVALID_ARG, "%s: null pointer", what);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case M3B_F32: return launch_ew2<float, Op>(a, b, out, n, scale, st, what);
    case M3B_BF16: return launch_ew2<__nv_bfloat16, Op>(a, b, out, n, scale, st, what);
    case M3B_F16: return launch_ew2<__half, Op>(a, b, out, n, scale, st, what);
    default: return fail(M3B_ERR_INVALID_ARG, "%s: dtype", what);
  }
}

}  // namespace

}  // namespace m3b

extern "C" int m3b_swiglu_act(const void* g, const void* u, void* out, int64_t n, int32_t dtype, void* stream) {
  m3b::clear_error();
  return m3b::dispatch_ew2<m3b::SwigluOp>(g, u, out, n, 0.f, dtype, stream, "swiglu_act");
}

extern "C" int m3b_scaled_add(const void* x, const void* h, float scale, void* out, int64_t n, int32_t dtype,
                              void* stream) {
  m3b::clear_error();
  return m3b::dispatch_ew2<m3b::ScaledAddOp>(x, h, out, n, scale, dtype, stream, "scaled_add");
}

extern "C" int m3b_swiglu_rows(const void* gu, void* out, int64_t rows, int32_t f, int32_t dtype, void* stream) {
  using namespace m3b;
  clear_error();
  if (rows < 0 || f <= 0) return fail(M3B_ERR_INVALID_ARG, "swiglu_rows: bad shape");
  if (rows == 0) return M3B_OK;  // nothing to touch: the pointers may be null
  if (!gu || !out) return fail(M3B_ERR_INVALID_ARG, "swiglu_rows: null pointer");
  if (f % 8 != 0 || !aligned16(gu) || !aligned16(out))
    return fail(M3B_ERR_UNSUPPORTED, "swiglu_rows: f must be a multiple of 8 and the rows 16-byte aligned");
  if (rows == 0) return M3B_OK;
  const int64_t units = rows * (f / 8);
  int64_t blocks = (units + kEwThreads - 1) / kEwThreads;
  const int64_t cap = (int64_t)num_sms() * 16;
  if (blocks > cap) blocks = cap;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case M3B_F32:
      swiglu_rows_kernel<float><<<(unsigned)blocks, kEwThreads, 0, st>>>(static_cast<const float*>(gu),
                                                                         static_cast<float*>(out), rows, f);
      break;
    case M3B_BF16:
      swiglu_rows_kernel<__nv_bfloat16><<<(unsigned)blocks, kEwThreads, 0, st>>>(
          static_cast<const __nv_bfloat16*>(gu), static_cast<__nv_bfloat16*>(out), rows, f);
      break;
    case M3B_F16:
      swiglu_rows_kernel<__half><<<(unsigned)blocks, kEwThreads, 0, st>>>(static_cast<const __half*>(gu),
                                                                        static_cast<__half*>(out), rows, f);
      break;
    default: return fail(M3B_ERR_INVALID_ARG, "swiglu_rows: dtype");
  }
  return check_launch("swiglu_rows");
}
