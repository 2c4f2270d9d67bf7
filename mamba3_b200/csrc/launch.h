// Host-side internals shared by the launchers (not part of the C ABI).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/mamba3_b200.h"

namespace m3b {

// Record a failure detail for m3b_last_error() and return `code`.
int fail(int code, const char* fmt, ...);
// Clear the calling thread's m3b_last_error() detail (at the start of an entry point).
void clear_error();
// cudaGetLastError() after a launch -> M3B_OK or M3B_ERR_CUDA (with detail).
int check_launch(const char* what);
// Number of SMs of the current device (cached per device).
int num_sms();

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

struct ScanLaunch {
  const float* decay;
  const void* h_chunk;
  const float* h_init;
  const float* init_bx;    // optional: h_states[0] += init_coef[b,h] * init_bx
  const float* init_coef;  // (B,H)
  void* h_states;
  float* h_final;
  int64_t B, K, H, PN;
  int dtype;
};
int launch_scan(const ScanLaunch& s, cudaStream_t st);

struct ScanBwdLaunch {
  const float* decay;
  const void* h_states;
  const void* grad_h;
  void* d_chunk;
  float* d_decay;
  float* d_h_init;
  int64_t B, K, H, PN;
  int dtype;
};
size_t scan_bwd_workspace(const ScanBwdLaunch& s);
int launch_scan_bwd(const ScanBwdLaunch& s, void* ws, size_t ws_bytes, cudaStream_t st);

int launch_step(const m3b_step_args* a, cudaStream_t st);
size_t step_workspace(const m3b_step_args* a);
int layer_fwd(const m3b_layer_fwd_args* a, void* ws, size_t ws_bytes, cudaStream_t st);
size_t layer_fwd_workspace(const m3b_layer_fwd_args* a);
// The least workspace layer_fwd accepts (it then runs whole sequences per CTA).
size_t layer_fwd_workspace_min(const m3b_layer_fwd_args* a);

// chunked_ssd backward on tensor cores (ssd_general.cu): applicable shapes, extra workspace, and
// the run that writes every gradient but ddt / dA / dD plus the per-token partials fw / ew
// ((batch H, T, 8) floats), m_T = <dh_final, h_final> and sum dy . x_raw per (batch, head).
bool bwd_tc_ok(const m3b_ssd_bwd_args* a);
size_t bwd_tc_workspace(const m3b_ssd_bwd_args* a);
int bwd_tc_run(const m3b_ssd_bwd_args* a, void* ws, float* fw, float* ew, float* mT, float* dDf, cudaStream_t st);

}  // namespace m3b
