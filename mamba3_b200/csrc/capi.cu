// extern "C" entry points of libmamba3_b200 (declared in include/mamba3_b200.h)
// and the host-side error plumbing shared by the launchers.
#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "launch.h"

namespace m3b {

static thread_local char g_last_error[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

void clear_error() { g_last_error[0] = 0; }

int check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(M3B_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return M3B_OK;
}

int num_sms() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

}  // namespace m3b

extern "C" {

const char* m3b_strerror(int status) {
  switch (status) {
    case M3B_OK: return "ok";
    case M3B_ERR_INVALID_ARG: return "invalid argument";
    case M3B_ERR_UNSUPPORTED: return "unsupported configuration";
    case M3B_ERR_CUDA: return "CUDA error";
    case M3B_ERR_ALIGNMENT: return "misaligned pointer";
    case M3B_ERR_TIMEOUT: return "device wait timed out";
    case M3B_ERR_WORKSPACE: return "workspace missing or too small";
    default: return "unknown status";
  }
}

const char* m3b_last_error(void) { return m3b::g_last_error; }

int m3b_abi_version(void) { return M3B_ABI_VERSION; }

int m3b_copy_rows_async(void* dst, size_t dst_pitch, const void* src, size_t src_pitch, size_t row_bytes,
                        size_t rows, void* stream) {
  if (!dst || !src || row_bytes > dst_pitch || row_bytes > src_pitch)
    return m3b::fail(M3B_ERR_INVALID_ARG, "copy_rows: null pointer or row wider than its pitch");
  if (rows == 0 || row_bytes == 0) return M3B_OK;
  const cudaError_t e = cudaMemcpy2DAsync(dst, dst_pitch, src, src_pitch, row_bytes, rows, cudaMemcpyDefault,
                                          static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return m3b::fail(M3B_ERR_CUDA, "copy_rows: %s", cudaGetErrorString(e));
  return M3B_OK;
}

int m3b_scan_fwd(const m3b_scan_args* a, void* stream) {
  m3b::g_last_error[0] = 0;
  if (!a || !a->decay || !a->h_chunk || !a->h_states)
    return m3b::fail(M3B_ERR_INVALID_ARG, "scan_fwd: null pointer");
  if (a->B < 0 || a->K < 0 || a->H < 0 || a->PN < 0) return m3b::fail(M3B_ERR_INVALID_ARG, "scan_fwd: negative dim");
  m3b::ScanLaunch s{a->decay, a->h_chunk, a->h_init, nullptr, nullptr, a->h_states, a->h_final,
                    a->B, a->K, a->H, a->PN, a->dtype};
  return m3b::launch_scan(s, static_cast<cudaStream_t>(stream));
}

static m3b::ScanBwdLaunch scan_bwd_launch(const m3b_scan_bwd_args* a) {
  return m3b::ScanBwdLaunch{a->decay, a->h_states, a->grad_h, a->d_chunk, a->d_decay, a->d_h_init,
                            a->B, a->K, a->H, a->PN, a->dtype};
}

size_t m3b_scan_bwd_workspace(const m3b_scan_bwd_args* a) { return a ? m3b::scan_bwd_workspace(scan_bwd_launch(a)) : 0; }

int m3b_scan_bwd(const m3b_scan_bwd_args* a, void* workspace, size_t workspace_bytes, void* stream) {
  m3b::g_last_error[0] = 0;
  if (!a || !a->decay || !a->h_states || !a->grad_h || !a->d_chunk || !a->d_decay)
    return m3b::fail(M3B_ERR_INVALID_ARG, "scan_bwd: null pointer");
  if (a->B < 0 || a->K < 0 || a->H < 0 || a->PN < 0) return m3b::fail(M3B_ERR_INVALID_ARG, "scan_bwd: negative dim");
  return m3b::launch_scan_bwd(scan_bwd_launch(a), workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

size_t m3b_step_workspace(const m3b_step_args* a) { return m3b::step_workspace(a); }

int m3b_step(const m3b_step_args* a, void* stream) {
  m3b::g_last_error[0] = 0;
  if (!a) return m3b::fail(M3B_ERR_INVALID_ARG, "step: null args");
  return m3b::launch_step(a, static_cast<cudaStream_t>(stream));
}

size_t m3b_layer_fwd_workspace(const m3b_layer_fwd_args* a) { return a ? m3b::layer_fwd_workspace(a) : 0; }

int m3b_layer_fwd(const m3b_layer_fwd_args* a, void* workspace, size_t workspace_bytes, void* stream) {
  m3b::g_last_error[0] = 0;
  if (!a) return m3b::fail(M3B_ERR_INVALID_ARG, "layer_fwd: null args");
  return m3b::layer_fwd(a, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
