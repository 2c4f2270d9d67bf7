/*
 * mamba3_b200 -- C ABI of the B200 (sm_100a) Mamba-3 SSD kernels.
 *
 * Conventions (every entry point):
 *  - Arguments are plain device pointers, element counts and dtype codes; no
 *    framework types cross this boundary.  `stream` is a cudaStream_t.
 *  - The caller owns every buffer, outputs and workspace included; the library
 *    never allocates or frees device memory.
 *  - Calls are asynchronous on `stream` and return M3B_OK or an m3b_status code;
 *    they never abort the process.  m3b_last_error() gives a detail message for
 *    the calling thread's last failure.
 *  - Launches are reentrant and thread-safe for distinct streams; the only
 *    process-wide state is a one-time kernel attribute setup per device.
 *  - Optional `err` pointers name a device int that kernels set (first error
 *    wins) when a bounded on-device wait expires; read it after synchronising.
 *
 * Shapes use the reference's layouts: activations (batch, seqlen, ...),
 * states (batch, H, P, N), angles (batch, H, N/2).  H = heads, P = headdim,
 * N = d_state, R = mimo_rank, G = ngroups.
 */
#ifndef MAMBA3_B200_H
#define MAMBA3_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define M3B_ABI_VERSION 8

#if defined(__GNUC__)
#define M3B_API __attribute__((visibility("default")))
#else
#define M3B_API
#endif

typedef enum m3b_dtype { M3B_F32 = 0, M3B_BF16 = 1, M3B_F16 = 2 } m3b_dtype;

typedef enum m3b_status {
  M3B_OK = 0,
  M3B_ERR_INVALID_ARG = 1,  /* null pointer, bad shape or dtype */
  M3B_ERR_UNSUPPORTED = 2,  /* valid request this build does not implement */
  M3B_ERR_CUDA = 3,         /* CUDA runtime / launch error */
  M3B_ERR_ALIGNMENT = 4,    /* a pointer lacks the required 16-byte alignment */
  M3B_ERR_TIMEOUT = 5,      /* a bounded device wait expired (reported via `err`) */
  M3B_ERR_WORKSPACE = 6     /* workspace missing or too small */
} m3b_status;

/* Status code -> static string. */
M3B_API const char* m3b_strerror(int status);
/* Detail message of the calling thread's last failed call ("" if none). */
M3B_API const char* m3b_last_error(void);
/* M3B_ABI_VERSION of the loaded library. */
M3B_API int m3b_abi_version(void);

/* ------------------------------------------------------------------------
 * Inter-chunk scan.
 * Replaces the reference's pybind entry `scan_forward(decay, h_chunk, h_init)`
 * (mamba3/csrc/scan.cu:128-166; called from mamba3/scan.py:80 in SSDScanFn.forward,
 * mamba3/scan.py:65-100).  h_states[:,0] = h_init (or 0);
 * h_states[:,k+1] = decay[:,k] * h_states[:,k] + h_chunk[:,k], carried in fp32.
 * Optionally also h_final = decay[:,K-1]*h_states[:,K-1] + h_chunk[:,K-1] (fp32),
 * the value mamba3/ssd.py:235-242 derives from the scan.
 * ------------------------------------------------------------------------ */
typedef struct m3b_scan_args {
  const float* decay;     /* (B,K,H) */
  const void* h_chunk;    /* (B,K,H,PN), `dtype` */
  const float* h_init;    /* (B,H,PN) or NULL */
  void* h_states;         /* (B,K,H,PN), `dtype` (may not alias h_chunk) */
  float* h_final;         /* (B,H,PN) or NULL */
  int64_t B, K, H, PN;
  int32_t dtype;          /* M3B_F32 or M3B_BF16 */
} m3b_scan_args;
M3B_API int m3b_scan_fwd(const m3b_scan_args* a, void* stream);

/* ------------------------------------------------------------------------
 * Inter-chunk scan, backward.
 * Replaces the reference's pybind entry `scan_backward(decay, h_states, grad_h, has_h_init)`
 * (mamba3/csrc/scan.cu:168-211, kernel :52-126; called from mamba3/scan.py:102-118 in
 * SSDScanFn.backward; torch loop mamba3/scan.py:47-62).  With the fp32 carry
 * g_{K-1} = grad_h[:,K-1], g_k = grad_h[:,k] + decay[:,k] * g_{k+1}:
 *   d_chunk[:,k] = g_{k+1} and d_decay[:,k] = sum_j g_{k+1}[j] * h_states[:,k,j] for k < K-1,
 *   d_chunk[:,K-1] = 0, d_decay[:,K-1] = 0, d_h_init = g_0 (when d_h_init != NULL).
 * d_decay is summed in a fixed order: results are bitwise reproducible run to run.
 * m3b_scan_bwd_workspace gives the caller-owned workspace size (0 when none is needed;
 * 16-byte aligned otherwise).
 * ------------------------------------------------------------------------ */
typedef struct m3b_scan_bwd_args {
  const float* decay;     /* (B,K,H) */
  const void* h_states;   /* (B,K,H,PN), `dtype` (the forward's exclusive states) */
  const void* grad_h;     /* (B,K,H,PN), `dtype` */
  void* d_chunk;          /* (B,K,H,PN), `dtype` (may not alias the inputs) */
  float* d_decay;         /* (B,K,H) */
  float* d_h_init;        /* (B,H,PN) or NULL */
  int64_t B, K, H, PN;
  int32_t dtype;          /* M3B_F32 or M3B_BF16 */
} m3b_scan_bwd_args;
M3B_API size_t m3b_scan_bwd_workspace(const m3b_scan_bwd_args* a);
M3B_API int m3b_scan_bwd(const m3b_scan_bwd_args* a, void* workspace, size_t workspace_bytes, void* stream);

/* Parameters of one KulaMamba layer (names and shapes of mamba3/mamba3.py:95-111). */
typedef struct m3b_layer_params {
  int32_t H, P, N, R, G;
  int32_t trapezoidal;    /* use_trapezoidal */
  int32_t complex_ssm;    /* use_complex_ssm (data-dependent RoPE on B/C) */
  int32_t param_dtype;    /* dtype of every pointer below */
  float norm_eps;         /* B_norm / C_norm eps (1e-5 in the reference) */
  const void* A_log;      /* (H) */
  const void* D;          /* (H) */
  const void* dt_bias;    /* (H) */
  const void* B_norm_w;   /* (N*R) */
  const void* C_norm_w;   /* (N*R) */
  const void* B_bias;     /* (G,N,R) */
  const void* C_bias;     /* (G,N,R) */
  const void* mimo_x;     /* (H,P,R) */
  const void* mimo_z;     /* (H,P,R) */
  const void* mimo_down;  /* (H,P,R) */
} m3b_layer_params;

/* The input projection row of one token, as split by mamba3/mamba3.py:125-140:
 * [ z (H*P) | x (H*P) | B (G*N*R) | C (G*N*R) | dt (H) | lam (H, if trapezoidal) |
 *   theta (N/2, if complex_ssm) ], `proj_stride` elements between tokens. */

/* ------------------------------------------------------------------------
 * O(1) decode step.
 * Replaces the SSM core of KulaMamba.step (mamba3/mamba3.py:278-316): everything
 * between in_proj and out_proj -- softplus dt, decay, B/C RMSNorm + bias, RoPE
 * advance of the angle state, MIMO x, the fp32 trapezoidal state update
 * h = dA*h + gamma*B^x + beta*prev_BX, readout C^.h + D*x, gate and MIMO-down.
 * State buffers may be updated in place (h_out == h, bx_out == prev_bx,
 * angle_out == angle when angle is fp32).
 * ------------------------------------------------------------------------ */
typedef struct m3b_step_args {
  m3b_layer_params prm;
  int64_t batch;
  const void* proj;       /* (batch, proj_stride), act_dtype */
  int64_t proj_stride;
  int32_t act_dtype;
  const void* dt_scale;   /* (batch, H) act_dtype, or NULL */
  const float* h;         /* (batch,H,P,N) */
  const float* prev_bx;   /* (batch,H,P,N) */
  const void* angle;      /* (batch,H,N/2), angle_dtype */
  int32_t angle_dtype;
  float* h_out;           /* (batch,H,P,N) */
  float* bx_out;          /* (batch,H,P,N): this token's B^x (next step's prev_BX) */
  float* angle_out;       /* (batch,H,N/2) fp32 */
  void* y;                /* (batch, H*P) act_dtype: gated MIMO-down output, input of out_proj */
  /* Compact previous-token state (no reference counterpart; opt-in): when prev_b is not NULL
   * the previous token is given as its rotated B^ (batch,H,N,R) and MIMO x (batch,H,P,R) fp32,
   * prev_BX = sum_r prev_b[n,r] prev_x[p,r] is rebuilt inside the kernel, prev_bx / bx_out
   * are not used, and this token's B^ / x_r are written to prev_b_out / prev_x_out (may alias
   * prev_b / prev_x): half the state bytes per step. */
  const float* prev_b;
  const float* prev_x;
  float* prev_b_out;
  float* prev_x_out;
  /* Optional workspace (no reference counterpart) of m3b_step_workspace() bytes, 16-byte
   * aligned: with it, d_state 128 / headdim <= 64 / mimo_rank 1, 2 or 4 run as two kernels --
   * per-(batch, head) operand preparation, then persistent CTAs that stream the state through a
   * shared-memory ring by bulk copies.  NULL: one kernel, no workspace.  Same results. */
  void* workspace;
  size_t workspace_bytes;
} m3b_step_args;
/* Workspace bytes of the streaming decode step for these arguments (0: not applicable). */
M3B_API size_t m3b_step_workspace(const m3b_step_args* a);
M3B_API int m3b_step(const m3b_step_args* a, void* stream);

/* ------------------------------------------------------------------------
 * Layer forward / prefill (parallel, chunked).
 * Replaces KulaMamba._forward_impl between in_proj and out_proj
 * (mamba3/mamba3.py:198-238) including chunked_ssd (mamba3/ssd.py:118-244) and,
 * when requested, the prefill state of mamba3/mamba3.py:241-256.
 * It may also continue from an inference state (h_init, angle_init, prev_bx_init),
 * which the reference does not offer; with all three NULL it is the reference's
 * computation from a zero state.
 * ------------------------------------------------------------------------ */
typedef struct m3b_layer_fwd_args {
  m3b_layer_params prm;
  int64_t batch, seqlen;
  const void* proj;          /* (batch, seqlen, proj_stride), act_dtype */
  int64_t proj_stride;
  int32_t act_dtype;         /* M3B_BF16 or M3B_F32 */
  const void* dt_scale;      /* (batch, seqlen, H) act_dtype, or NULL */
  const float* h_init;       /* (batch,H,P,N) or NULL */
  const float* angle_init;   /* (batch,H,N/2) or NULL */
  const float* prev_bx_init; /* (batch,H,P,N) or NULL */
  void* y;                   /* (batch, seqlen, H*P) act_dtype */
  float* h_final;            /* (batch,H,P,N) or NULL */
  float* angle_final;        /* (batch,H,N/2) or NULL */
  float* prev_bx_final;      /* (batch,H,P,N) or NULL */
  int* err;                  /* device int or NULL */
  /* NULL, or M3B_LAYER_FWD_STAGES + 1 cudaEvent_t: event i is recorded on `stream` before
   * stage i (prep, angle prefix, chunk state, scan, chunk output, prefill prev_BX) and the
   * last one after the final stage, so callers can time each kernel. */
  void* const* stage_events;
  /* 0: automatic; 1: fused sequential kernel (one persistent CTA per SM walks whole
   * (batch, head) sequences, state kept on chip); 2: chunk-parallel kernels (chunk
   * states in HBM + scan). Same results up to fp32 rounding. */
  int32_t algo;
  /* 1: the caller needs only h_final / angle_final / prev_bx_final; y must still be a valid
   * buffer, but the fused path may leave it unwritten and skips the output work. */
  int32_t state_only;
  /* Optional compact final previous-token state (see m3b_step_args.prev_b): the last token's
   * rotated B^ (batch,H,N,R) and MIMO x (batch,H,P,R), fp32. */
  float* prev_b_final;
  float* prev_x_final;
  /* Limit in nanoseconds of every device-side wait of this call (0: the library's 2 s).  A wait
   * that runs out records M3B_ERR_TIMEOUT in `err` and the kernel returns early. */
  int64_t wait_limit_ns;
  /* Optional (batch*seqlen, G, 2) fp32: the 1/rms of every group's B and C row per token, as
   * m3b_in_proj writes it.  When given (bf16 activations), the fused path reads it instead of
   * making its own pass over the projection's B / C columns. */
  const float* rms_in;
} m3b_layer_fwd_args;
#define M3B_LAYER_FWD_STAGES 6

/* ------------------------------------------------------------------------
 * Input projection with the layer's per-token prologue in its epilogue.
 * Replaces `proj = self.in_proj(x)` (mamba3/mamba3.py:197, an nn.Linear) and the
 * layer forward's own pass over the projection's B / C columns that B_norm /
 * C_norm need (mamba3/mamba3.py:200-204): proj = x W^T (+ bias), bf16 operands
 * and output, fp32 accumulation on the tensor cores; with `rms` given, the same
 * epilogue also writes 1/rms of every group's B and C row of each token (the
 * rms_in of m3b_layer_fwd_args).
 * ------------------------------------------------------------------------ */
typedef struct m3b_in_proj_args {
  int64_t rows;           /* tokens: batch * seqlen */
  int32_t d_model;        /* multiple of 8 */
  int32_t d_proj;         /* output columns, multiple of 8 */
  const void* x;          /* (rows, x_stride) bf16, 16-byte aligned */
  int64_t x_stride;       /* elements, multiple of 8 */
  const void* weight;     /* (d_proj, d_model) bf16, row-contiguous (the nn.Linear weight) */
  const void* bias;       /* (d_proj) bf16, or NULL */
  void* proj;             /* (rows, proj_stride) bf16, 16-byte aligned */
  int64_t proj_stride;    /* elements, multiple of 8 */
  /* H, P, N, R, G and norm_eps place and normalise B and C in the projection row (only read
   * when rms is given; the parameter pointers are not read) */
  m3b_layer_params prm;
  float* rms;             /* (rows, G, 2) fp32, or NULL */
  int* err;               /* device int or NULL */
  int64_t wait_limit_ns;  /* limit of every device-side wait (0: the library's 2 s) */
} m3b_in_proj_args;
M3B_API int m3b_in_proj(const m3b_in_proj_args* a, void* stream);

/* ------------------------------------------------------------------------
 * Allocation-free layer forward (no counterpart in the reference).
 * For callers that cannot allocate device memory where they run the layer --
 * e.g. a plugin hosted by another runtime that owns the allocator and hands it
 * only input and output buffers.  Same arguments and results as m3b_layer_fwd,
 * but the workspace is a static device array of M3B_NOALLOC_SCRATCH_BYTES that
 * every GPU loading the library holds until exit; larger problems fail with
 * M3B_ERR_WORKSPACE.  All calls share that array: calls that overlap on the GPU
 * race and must be serialised by the caller.  The first call on a device looks
 * the array's address up; make it before any stream capture.  Calls no
 * allocating routine.
 * ------------------------------------------------------------------------ */
#define M3B_NOALLOC_SCRATCH_BYTES ((size_t)32 << 20)
M3B_API int m3b_layer_fwd_noalloc(const m3b_layer_fwd_args* a, void* stream);

/* ---------------------------------------------------------------------------
 * Strided copy of `rows` rows of `row_bytes` bytes between host and device
 * memory (either direction, or device to device) on `stream`, one call per
 * block of rows: the piece-wise host streaming of KulaMamba.forward_host
 * (no reference counterpart) moves a (batch, token range) slab of a
 * (batch, seqlen, d_model) host tensor with it.  Pitches are in bytes; host
 * memory should be pinned for the copy to be asynchronous.
 * ------------------------------------------------------------------------ */
M3B_API int m3b_copy_rows_async(void* dst, size_t dst_pitch, const void* src, size_t src_pitch, size_t row_bytes,
                                size_t rows, void* stream);
/* Bytes of device workspace m3b_layer_fwd uses for these arguments on the current device.
 * With enough (batch, head) sequences the fused kernel cuts them into parts handed from CTA to
 * CTA, and this size includes the hand-off buffers; given less (but at least what the same
 * call needs without them), m3b_layer_fwd keeps whole sequences per CTA instead. */
M3B_API size_t m3b_layer_fwd_workspace(const m3b_layer_fwd_args* a);
M3B_API int m3b_layer_fwd(const m3b_layer_fwd_args* a, void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * chunked_ssd on pre-processed tensors.
 * Replaces the reference's chunked_ssd(x_g, x_b, B_g, B_b, C, dt, A, D, x_raw,
 * chunk_size, h_init, return_final_state) (mamba3/ssd.py:118-244): the input of token s
 * is dt_s * sum_q [x_g|x_b][s,:,q] [B_g|B_b][s,:,q]^T (x_b / B_b may be NULL: Euler),
 * y = intra-chunk + inter-chunk readout + D * x_raw, h_final in fp32.  All tensors are
 * contiguous; the per-chunk length is the library's own (results do not depend on it).
 * ------------------------------------------------------------------------ */
typedef struct m3b_ssd_args {
  int64_t batch, seqlen;
  int32_t H, P, N, R;
  int32_t dtype;             /* of x_g, x_b, B_g, B_b, C, x_raw and y: M3B_BF16 or M3B_F32 */
  const void* x_g;           /* (batch,seqlen,H,P,R) */
  const void* x_b;           /* (batch,seqlen,H,P,R) or NULL */
  const void* B_g;           /* (batch,seqlen,H,N,R) */
  const void* B_b;           /* (batch,seqlen,H,N,R) or NULL (NULL iff x_b is NULL) */
  const void* C;             /* (batch,seqlen,H,N,R) */
  const void* x_raw;         /* (batch,seqlen,H,P,R) */
  const void* dt;            /* (batch,seqlen,H), dt_dtype */
  int32_t dt_dtype;
  const void* A;             /* (H), ad_dtype (A = -exp(A_log), negative) */
  const void* D;             /* (H), ad_dtype */
  int32_t ad_dtype;
  const float* h_init;       /* (batch,H,P,N) or NULL */
  void* y;                   /* (batch,seqlen,H,P,R), dtype */
  float* h_final;            /* (batch,H,P,N) or NULL */
  int* err;                  /* device int or NULL */
} m3b_ssd_args;
M3B_API size_t m3b_chunked_ssd_workspace(const m3b_ssd_args* a);
M3B_API int m3b_chunked_ssd(const m3b_ssd_args* a, void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * Backward of chunked_ssd: the gradients torch autograd gives the reference through
 * _IntraChunkFn (mamba3/ssd.py:27-115), SSDScanFn (mamba3/scan.py:65-140) and the torch
 * ops of chunked_ssd (mamba3/ssd.py:118-244), for the same inputs as m3b_ssd_args plus the
 * output gradients dy (and dh_final when h_final was used).  fp32 arithmetic; gradients
 * in the dtypes of their inputs (ddt in dt_dtype; dA, dD per head and dh_init in fp32).
 * Deterministic: no atomics, every sum in a fixed order.
 * ------------------------------------------------------------------------ */
typedef struct m3b_ssd_bwd_args {
  int64_t batch, seqlen;
  int32_t H, P, N, R;
  int32_t dtype;             /* of x_g, x_b, B_g, B_b, C, x_raw, dy and their gradients */
  const void* x_g;           /* (batch,seqlen,H,P,R) */
  const void* x_b;           /* (batch,seqlen,H,P,R) or NULL (Euler) */
  const void* B_g;           /* (batch,seqlen,H,N,R) */
  const void* B_b;           /* (batch,seqlen,H,N,R) or NULL (NULL iff x_b is NULL) */
  const void* C;             /* (batch,seqlen,H,N,R) */
  const void* x_raw;         /* (batch,seqlen,H,P,R) */
  const void* dt;            /* (batch,seqlen,H), dt_dtype */
  int32_t dt_dtype;
  const void* A;             /* (H), ad_dtype */
  const void* D;             /* (H), ad_dtype */
  int32_t ad_dtype;
  const float* h_init;       /* (batch,H,P,N) or NULL */
  const void* dy;            /* (batch,seqlen,H,P,R), dtype */
  const float* dh_final;     /* (batch,H,P,N) or NULL */
  void* dx_g;                /* (batch,seqlen,H,P,R), dtype */
  void* dx_b;                /* (batch,seqlen,H,P,R) or NULL (NULL iff x_b is NULL) */
  void* dB_g;                /* (batch,seqlen,H,N,R) */
  void* dB_b;                /* (batch,seqlen,H,N,R) or NULL (NULL iff x_b is NULL) */
  void* dC;                  /* (batch,seqlen,H,N,R) */
  void* dx_raw;              /* (batch,seqlen,H,P,R) */
  void* ddt;                 /* (batch,seqlen,H), dt_dtype */
  float* dA;                 /* (H) */
  float* dD;                 /* (H) */
  float* dh_init;            /* (batch,H,P,N) or NULL */
  /* 0: chunk-level products on tensor cores where they apply (bf16, N <= 128 and P <= 64 both
   * multiples of 8, mimo_rank 1, 2 or 4, 16-byte aligned per-token tensors), else the token
   * sweeps; 1: always the token sweeps (fp32 CUDA cores).  No counterpart in the reference. */
  int32_t algo;
} m3b_ssd_bwd_args;
M3B_API size_t m3b_chunked_ssd_bwd_workspace(const m3b_ssd_bwd_args* a);
M3B_API int m3b_chunked_ssd_bwd(const m3b_ssd_bwd_args* a, void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * Cross-shard fold of the sequence-parallel prefill (no counterpart in the reference, which
 * runs one sequence on one device; it replaces the h_init chaining of mamba3/ssd.py:118-131
 * across devices).  Rank g's summary of its token range, run from the zero state, is one fp32
 * block [S (batch,H,P,N) | PB (batch,H,P,N) | Om (batch,H,N/2) | Lam (batch,H) | c0 (batch,H)]:
 * final state, final prev_BX, final angle, sum of A dt, and (1 - lam) dt of its first token.
 * `summaries` holds the blocks of ranks 0, 1, ... rank_stride floats apart (an all_gather
 * output).  Writes the exact state entering rank `upto`'s range:
 *   h = sum_{g<upto} exp(sum_{g<j<upto} Lam_j) (exp(Lam_g) c0_g pb_g + Rot(a_g) S_g),
 *   angle = a_upto, prev_bx = Rot(a_{upto-1}) PB_{upto-1}    (a_g = sum_{j<g} Om_j,
 * pb_g = Rot(a_{g-1}) PB_{g-1}, Rot(a) turning the (2i, 2i+1) columns by a_i); upto = 0 gives
 * the zero state.  h and prev_bx 8-byte aligned.
 * ------------------------------------------------------------------------ */
typedef struct m3b_seqpar_fold_args {
  const float* summaries;
  int64_t rank_stride;
  int32_t upto;
  int64_t batch;
  int32_t H, P, N;
  float* h;
  float* angle;
  float* prev_bx;
} m3b_seqpar_fold_args;
M3B_API int m3b_seqpar_fold(const m3b_seqpar_fold_args* a, void* stream);

/* ------------------------------------------------------------------------
 * RMSNorm of the blocks around the layer (mamba3/mamba3.py:19-35; used by
 * mamba3/block.py:53,70,81-103 and KulaMambaLM's final norm): for each of `rows` rows of d
 * contiguous elements, y = (x * rsqrt(mean(x^2) + eps)) * weight, the mean in fp32, the
 * scale and both products rounded to `dtype` as the reference's torch ops store them.
 * x, weight (d) and y share `dtype` (M3B_F32, M3B_BF16 or M3B_F16); y may alias x.
 * ------------------------------------------------------------------------ */
M3B_API int m3b_rmsnorm(const void* x, const void* weight, void* y, int64_t rows, int32_t d, float eps,
                        int32_t dtype, void* stream);
/* The residual step that precedes each norm of the blocks (mamba3/block.py:79-107: x + h * scale
 * feeding the next RMSNorm), in one pass: x_out = x + h * scale rounded as m3b_scaled_add stores
 * it, and y = RMSNorm(x_out) with `weight`, bit for bit what m3b_scaled_add then m3b_rmsnorm give.
 * 16-bit dtypes (M3B_BF16, M3B_F16), d % 8 == 0 and d <= 2048, 16-byte aligned rows; x_out may
 * alias x. */
M3B_API int m3b_add_rmsnorm(const void* x, const void* h, float scale, const void* weight, void* x_out, void* y,
                            int64_t rows, int32_t d, float eps, int32_t dtype, void* stream);

/* ------------------------------------------------------------------------
 * Gate and MIMO down-projection of the layer (mamba3/mamba3.py:234-238) for the training path,
 * forward and backward, over `rows` rows of `channels` = H*P channels with R ranks:
 *   out[c] = sum_r y[c,r] silu(z[c] mimo_z[c,r]) mimo_down[c,r]
 * y (rows, channels, R), z (rows, channels; rows z_stride elements apart, 0 = channels),
 * out / dout / dz (rows, channels), mimo_z / mimo_down and their gradients (channels, R), all
 * of `dtype` and otherwise contiguous.  The backward gives dy, dz and the
 * parameter gradients (summed over the rows in a fixed order; caller-owned workspace of
 * m3b_gate_bwd_workspace bytes).  With rows == 0 the per-row pointers may be null and the
 * backward writes zero parameter gradients.
 * ------------------------------------------------------------------------ */
typedef struct m3b_gate_args {
  int64_t rows, z_stride;
  int32_t channels, R, dtype;
  const void* y;
  const void* z;
  const void* mimo_z;
  const void* mimo_down;
  void* out;              /* forward */
  const void* dout;       /* backward: */
  void* dy;
  void* dz;
  void* d_mimo_z;
  void* d_mimo_down;
} m3b_gate_args;
M3B_API int m3b_gate_fwd(const m3b_gate_args* a, void* stream);
M3B_API size_t m3b_gate_bwd_workspace(const m3b_gate_args* a);
M3B_API int m3b_gate_bwd(const m3b_gate_args* a, void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * B / C preparation of the layer for the training path (mamba3/mamba3.py:203-232), forward and
 * backward: RMSNorm over each group's N*R values + bias, broadcast of the G groups to the H
 * heads, the data-dependent rotation of (n = 2k, 2k+1) pairs by
 * phi[t, h, k] = -sum_{t' <= t} dt[t', h] theta[t', k]  (rotate != 0), and B_b[t] = B_g[t-1],
 * B_b[0] = 0  (shift != 0, the trapezoidal rule's previous-token B).
 * Bf, Cf (batch, seqlen, G*N*R) and theta (batch, seqlen, N/2): rows bc_stride / theta_stride
 * elements apart (0 = contiguous), so column slices of the input projection pass as they are;
 * dt (batch, seqlen, H) contiguous, of dt_dtype; wB / wC (N*R) and bB / bC (G, N, R) the norm
 * weights and biases.  Forward outputs B_g, B_b, C: (batch, seqlen, H, N, R).  Backward inputs
 * their gradients (dB_b unused without shift); outputs dBf, dCf (batch, seqlen, G*N*R) and
 * dtheta (batch, seqlen, N/2) contiguous, ddt (batch, seqlen, H) of dt_dtype (rotate only), and
 * the parameter gradients.  Activations and parameters share `dtype`; fp32 arithmetic; the
 * sums over heads, tokens and batch rows run in a fixed order.  Needs H*N/2 <= 2048.
 * Caller-owned workspaces of m3b_bc_fwd_workspace / m3b_bc_bwd_workspace bytes (the backward's
 * holds one fp32 angle gradient per (token, head, pair) when rotating).
 * ------------------------------------------------------------------------ */
typedef struct m3b_bc_args {
  int64_t batch, seqlen;
  int32_t H, G, N, R;
  int32_t rotate, shift;
  int32_t dtype, dt_dtype;
  float eps;
  int64_t bc_stride, theta_stride;
  const void* Bf;
  const void* Cf;
  const void* theta;
  const void* dt;
  const void* wB;
  const void* bB;
  const void* wC;
  const void* bC;
  void* B_g;            /* forward outputs */
  void* B_b;
  void* C;
  const void* dB_g;     /* backward inputs */
  const void* dB_b;
  const void* dC;
  void* dBf;            /* backward outputs */
  void* dCf;
  void* dtheta;
  void* ddt;
  void* dwB;
  void* dbB;
  void* dwC;
  void* dbC;
} m3b_bc_args;
M3B_API size_t m3b_bc_fwd_workspace(const m3b_bc_args* a);
M3B_API int m3b_bc_fwd(const m3b_bc_args* a, void* workspace, size_t workspace_bytes, void* stream);
M3B_API size_t m3b_bc_bwd_workspace(const m3b_bc_args* a);
M3B_API int m3b_bc_bwd(const m3b_bc_args* a, void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * MIMO expansion and trapezoid weights of x for the training path (mamba3/mamba3.py:218-230),
 * forward and backward:
 *   x_raw[t,h,p,r] = xf[t,h,p] mimo_x[h,p,r];  with trapezoidal != 0, lam = sigmoid(lam_raw),
 *   x_g[t] = x_raw[t] lam[t],  x_b[t] = x_raw[t-1] (1 - lam[t]) exp(A dt[t]),  x_b[0] = 0.
 * xf (batch, seqlen, H*P) and lam_raw (batch, seqlen, H): rows x_stride / lam_stride elements
 * apart (0 = contiguous), so column slices of the input projection pass as they are; dt
 * (batch, seqlen, H) contiguous of dt_dtype; A (H) of a_dtype (A = -exp(A_log)); mimo_x
 * (H, P, R).  Outputs (batch, seqlen, H, P, R).  The backward takes the gradients of x_raw,
 * x_g, x_b and gives dxf (batch, seqlen, H*P) contiguous, dmimo_x, and with trapezoidal
 * dlam_raw (batch, seqlen, H), ddt (dt's share through the weights) and dA.  Needs P <= 256,
 * R <= 4; fp32 arithmetic; fixed-order sums; caller-owned workspace of
 * m3b_xprep_bwd_workspace bytes for the backward.
 * ------------------------------------------------------------------------ */
typedef struct m3b_xprep_args {
  int64_t batch, seqlen;
  int32_t H, P, R, trapezoidal;
  int32_t dtype, dt_dtype, a_dtype;
  int64_t x_stride, lam_stride;
  const void* xf;
  const void* mimo_x;
  const void* lam_raw;
  const void* dt;
  const void* A;
  void* x_raw;          /* forward outputs */
  void* x_g;
  void* x_b;
  const void* dx_raw;   /* backward inputs */
  const void* dx_g;
  const void* dx_b;
  void* dxf;            /* backward outputs */
  void* dmimo_x;
  void* dlam_raw;
  void* ddt;
  void* dA;
} m3b_xprep_args;
M3B_API int m3b_xprep_fwd(const m3b_xprep_args* a, void* stream);
M3B_API size_t m3b_xprep_bwd_workspace(const m3b_xprep_args* a);
M3B_API int m3b_xprep_bwd(const m3b_xprep_args* a, void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * Element-wise steps of the blocks, one pass each, results rounded to `dtype` as the
 * reference's torch ops store them; n elements, out may alias an input.
 *   m3b_swiglu_act: out = silu(g) * u   (SwiGLU.forward, mamba3/block.py:16-26)
 *   m3b_scaled_add: out = x + h * scale (the residuals of mamba3/block.py:79-107)
 * ------------------------------------------------------------------------ */
M3B_API int m3b_swiglu_act(const void* g, const void* u, void* out, int64_t n, int32_t dtype, void* stream);
/* m3b_swiglu_rows: the same activation when the gate and up projections come from one GEMM with
 * the two weights stacked: gu (rows, 2f) = [g | u] per row, out (rows, f); f % 8 == 0, 16-byte
 * aligned rows. */
M3B_API int m3b_swiglu_rows(const void* gu, void* out, int64_t rows, int32_t f, int32_t dtype, void* stream);
M3B_API int m3b_scaled_add(const void* x, const void* h, float scale, void* out, int64_t n, int32_t dtype,
                           void* stream);

/* ------------------------------------------------------------------------
 * Tensor-core self-test (diagnostic; no counterpart in the reference).
 * D (128 x 64, fp32) = A (128 x 128 bf16, row-major) x B (64 x 128 bf16, row-major)^T,
 * staged through the same shared-memory layouts and UMMA descriptors as the chunk
 * kernels: mode 0 reads A K-major, mode 1 stages A transposed and reads it MN-major,
 * mode 2 stages B transposed and reads it MN-major.  Mode 3 takes fp32 A and B on
 * kind::tf32, both K-major (the tiles of the fp32 chunk kernels).  Mode 6 holds A in tensor
 * memory (bf16, two per 32-bit column), as the fused kernel holds its masked score tile.
 * ------------------------------------------------------------------------ */
M3B_API int m3b_selftest_umma(const void* A, const void* B, float* D, int mode, int* err, void* stream);

/* ------------------------------------------------------------------------
 * Bounded-wait self-test (diagnostic; no counterpart in the reference).
 * One thread runs the library's bounded wait on a condition for at most limit_ns
 * (0 < limit_ns <= 1 s): mode 0 waits for *flag >= target (the acquire-load flag wait the
 * fused layer kernel uses when one CTA hands a sequence part to another), mode 1 for phase 0
 * of a shared-memory mbarrier that nothing arrives on (the kernels' pipeline waits).  A wait
 * that runs out records M3B_ERR_TIMEOUT in *err (first error wins) and the kernel returns, so
 * a caller can check that an expired wait surfaces as a status and leaves the context usable.
 * ------------------------------------------------------------------------ */
M3B_API int m3b_selftest_wait(const int* flag, int target, int mode, int64_t limit_ns, int* err, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MAMBA3_B200_H */
