/*
 * vlak_b200.h -- C ABI of the B200 (sm_100a) kernels that sit behind the
 * torch.ops.vlak operators.
 *
 * Every entry point takes plain device pointers, sizes, element strides and a
 * CUDA stream handle (a cudaStream_t passed as void*; NULL = legacy default
 * stream), and returns an int status (0 = VLAK_OK). No torch types cross this
 * boundary. Launches are asynchronous on the given stream; nothing here
 * synchronizes the device. On a nonzero status, vlak_last_error_message()
 * holds a one-line description (thread-local).
 *
 * Inputs are borrowed for the duration of the launch; outputs are written in
 * place and owned by the caller. None of the entry points allocates device
 * memory (the first attention launch allocates one 4-byte pinned host word,
 * see vlak_device_error_poll).
 */
#ifndef VLAK_B200_H_
#define VLAK_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define VLAK_ABI_VERSION 1

#if defined(__GNUC__)
#define VLAK_API __attribute__((visibility("default")))
#else
#define VLAK_API
#endif

/* status codes */
enum {
  VLAK_OK = 0,
  VLAK_ERR_INVALID_ARGUMENT = 1, /* a shape / size / parameter contract is violated */
  VLAK_ERR_ALIGNMENT = 2,        /* a base address or stride breaks 16-byte alignment */
  VLAK_ERR_UNSUPPORTED_DTYPE = 3,
  VLAK_ERR_CUDA = 4,             /* a CUDA runtime / driver call failed */
  VLAK_ERR_DEVICE_TIMEOUT = 5,   /* a bounded device-side wait ran out */
  VLAK_ERR_UNSUPPORTED_DEVICE = 6 /* the current device is not sm_100 */
};

/* element types */
enum { VLAK_F32 = 0, VLAK_F16 = 1, VLAK_BF16 = 2, VLAK_F64 = 3, VLAK_I32 = 4, VLAK_I64 = 5 };

/* Library identity and diagnostics. */
VLAK_API int vlak_abi_version(void);
VLAK_API const char* vlak_status_string(int status);
VLAK_API const char* vlak_last_error_message(void);

/*
 * Device error reporting. Kernels whose waits are bounded (the attention
 * kernels) record a failed wait instead of hanging: VLAK_ERR_DEVICE_TIMEOUT,
 * sticky until read, and that launch's output is incomplete.
 *  - The status goes to a pinned, device-mapped host word of the process
 *    (4 bytes, allocated once by the first attention launch that is not being
 *    stream-captured; shared by all devices).
 *  - A launch made before that word exists (the first call of the process
 *    inside a stream capture) records into a per-device word instead.
 * vlak_device_error_poll() reads the host word without synchronizing
 * anything: it sees the failures of kernels that have finished, copies the
 * status to *code (0 = none) and clears it. The torch ops call it on entry
 * and raise RuntimeError when it is set. Replaces nothing in the reference,
 * which checks only cudaGetLastError after each launch
 * (kernels/attention/fused_attention.cu:594-596).
 */
VLAK_API int vlak_device_error_poll(int* code);

/* Synchronous form: reads and clears the per-device word of the current
 * device (a blocking copy, so call it between steps, not inside a stream
 * capture) and the host word; *code is the status found (0 = none). */
VLAK_API int vlak_device_error_read(int* code);

/* ------------------------------------------------------------------------
 * Row softmax over the last dimension of a contiguous [rows, cols] tensor.
 *
 * Replaces softmax_lastdim (kernels/softmax/softmax_kernels.cu:255-297) behind
 * the schema vlak::softmax(Tensor x, int version=4) -> Tensor
 * (kernels/softmax/softmax_kernels.cu:303-305).
 *   x, y     : device pointers, rows*cols elements each, row-major, no padding
 *   dtype    : VLAK_F32 / VLAK_F16 / VLAK_BF16 / VLAK_F64 (math is fp32 in
 *              all cases, as in the reference's AT_DISPATCH body)
 *   version  : 0..4 selects the algorithm family (0 thread-per-row,
 *              1 warp-per-row, 2 block-per-row 3-pass, 3 block-per-row
 *              online 2-pass, 4 register-resident single read); any other
 *              value behaves as 4, as in the reference dispatcher.
 * rows == 0 or cols == 0 is a no-op. A row whose entries are all -inf
 * produces NaN, as torch.softmax does.
 * ---------------------------------------------------------------------- */
VLAK_API int vlak_softmax_fwd(const void* x, void* y, int64_t rows, int64_t cols,
                     int dtype, int version, void* stream);

/* The version "auto" resolves to, restating _auto_version
 * (kernels/softmax/__init__.py:26-37): cols > 2048 -> 4; rows >= 32 -> 1;
 * else 4. */
VLAK_API int vlak_softmax_auto_version(int64_t rows, int64_t cols);

/* ------------------------------------------------------------------------
 * GQA-native fused attention, head_dim 64, bf16 in / bf16 out, fp32 accumulate.
 *
 * Replaces the host functions fused_attention_gqa
 * (kernels/attention/fused_attention.cu:603-669) and fused_attention_gqa_v4
 * (kernels/attention/fused_attention_v4.cu:278-331) behind the schemas
 * vlak::fused_attention_gqa / vlak::fused_attention_gqa_v4
 * (fused_attention.cu:671-676, fused_attention_v4.cu:333-336).
 *
 * Logical shapes: q (B, M, H, 64), k and v (B, N, Hkv, 64), o (B, M, H, 64).
 * Strides are in ELEMENTS for dims (0, 1, 2); dim 3 (head_dim) must be
 * contiguous. Query head h reads kv head h / (H / Hkv).
 *
 * Mask (analytic, no tensor):
 *   visible(r, c) = c < P ? (c < dead_start || c >= dead_end)
 *                         : c <= (N - M) + r
 * with P = prefix_len >= 0 ? prefix_len : N. scale <= 0 selects 1/sqrt(64).
 * A query row with no visible key is written as exact zeros.
 *
 * Contract (checked before anything is launched; violations return
 * VLAK_ERR_INVALID_ARGUMENT / VLAK_ERR_ALIGNMENT):
 *   H % Hkv == 0, H / Hkv <= 128, 0 <= dead_start <= dead_end <= P <= N,
 *   every pointer 16-byte aligned, every stride a multiple of 8 elements.
 * B == 0 or M == 0 is a no-op; N == 0 writes zeros.
 * ---------------------------------------------------------------------- */
typedef struct {
  const void* q;
  const void* k;
  const void* v;
  void* o;
  int64_t B, M, N, H, Hkv;
  int64_t q_stride[3]; /* (b, m, h) element strides of q */
  int64_t k_stride[3]; /* (b, n, h_kv) element strides of k */
  int64_t v_stride[3]; /* (b, n, h_kv) element strides of v */
  int64_t o_stride[3]; /* (b, m, h) element strides of o */
  double scale;
  int64_t prefix_len;
  int64_t dead_start;
  int64_t dead_end;
} vlak_attn_gqa_args;

/* vlak::fused_attention_gqa (reference v3 contract). */
VLAK_API int vlak_attn_gqa_fwd(const vlak_attn_gqa_args* args, void* stream);

/* vlak::fused_attention_gqa_v4 (reference v4 contract). Same arguments and
 * results as vlak_attn_gqa_fwd; both run the tcgen05 kernel. */
VLAK_API int vlak_attn_gqa_v4_fwd(const vlak_attn_gqa_args* args, void* stream);

/* Resolve the analytic-mask parameters exactly as the launch does
 * (P = -1 -> N, scale <= 0 -> 1/8) and validate the contract without
 * touching the device. Returns the status the launch would return for these
 * arguments; writes the resolved values when the pointers are non-NULL. */
VLAK_API int vlak_attn_gqa_check(const vlak_attn_gqa_args* args, int64_t* prefix_out,
                        float* scale_out);

/* GQA attention with a per-sample length mask (varlen prefix attention, the
 * reference's C4 site, which it leaves on SDPA; no counterpart kernel there,
 * new schema vlak::fused_attention_gqa_varlen). Same arguments as
 * vlak_attn_gqa_fwd; prefix_len / dead_start / dead_end are ignored.
 *   lengths       : device array of B lengths, VLAK_I32 or VLAK_I64
 *   visible(r, c) = c < L_b && r < L_b, with L_b clamped to [0, N];
 *   rows r >= L_b are written as zeros. */
VLAK_API int vlak_attn_gqa_varlen_fwd(const vlak_attn_gqa_args* args, const void* lengths,
                                      int lengths_dtype, void* stream);

/* GQA attention with a bool mask (B, M, N) broadcast over heads, on the
 * tensor cores. Serves the bf16 tensor-mask path of vlak::fused_attention
 * (the reference's v2, kernels/attention/fused_attention.cu:555-577).
 * Same arguments as vlak_attn_gqa_fwd; the analytic fields are ignored.
 *   mask           : device bytes, nonzero = attend; keys contiguous
 *   mask_stride_b/m: byte strides of dims b and m (0 broadcasts) */
VLAK_API int vlak_attn_gqa_masked_fwd(const vlak_attn_gqa_args* args, const void* mask,
                                      int64_t mask_stride_b, int64_t mask_stride_m,
                                      void* stream);

/* Key-split variants for small batches. No counterpart in the reference,
 * whose v3 launches one CTA per (b, head, 32- or 64-row query tile) however
 * few that makes (kernels/attention/fused_attention.cu:646-663). When the
 * query blocks fill
 * less than half of the GPU, these split each block's keys across CTAs and
 * merge the partial results with a second kernel on `stream`; they need a
 * device workspace of vlak_attn_gqa_workspace_size bytes, 256-byte aligned,
 * owned by the caller and not used by anything else until the work on
 * `stream` has finished. A NULL or smaller workspace runs unsplit. Results
 * match the unsplit calls within bf16 rounding (each split's O / l is held
 * in bf16 before the merge). */
/* Workspace bytes a _ws call with these arguments uses on the current
 * device (0 when it would not split). Validates like vlak_attn_gqa_check. */
VLAK_API int vlak_attn_gqa_workspace_size(const vlak_attn_gqa_args* args, int64_t* bytes);
/* vlak_attn_gqa_fwd with a workspace (also serves _v4). */
VLAK_API int vlak_attn_gqa_fwd_ws(const vlak_attn_gqa_args* args, void* workspace,
                                  int64_t workspace_bytes, void* stream);
/* vlak_attn_gqa_varlen_fwd with a workspace. */
VLAK_API int vlak_attn_gqa_varlen_fwd_ws(const vlak_attn_gqa_args* args, const void* lengths,
                                         int lengths_dtype, void* workspace,
                                         int64_t workspace_bytes, void* stream);
/* vlak_attn_gqa_masked_fwd with a workspace. */
VLAK_API int vlak_attn_gqa_masked_fwd_ws(const vlak_attn_gqa_args* args, const void* mask,
                                         int64_t mask_stride_b, int64_t mask_stride_m,
                                         void* workspace, int64_t workspace_bytes,
                                         void* stream);

/* vlak_attn_gqa_fwd that allocates nothing. No counterpart in the reference.
 * For callers that must not allocate device memory per call: a control loop
 * that reserves all of its memory at start-up (cudaMalloc synchronizes the
 * device and can stall the loop for milliseconds), or a host calling through
 * a C FFI without a pool allocator to hand out a workspace. Small batches
 * still split their keys across CTAs; the split scratch is a static 8 MiB
 * device buffer of this library, one per device.
 *  - The first call on a device looks up that buffer's address
 *    (cudaGetSymbolAddress); make the first call before any stream capture.
 *  - A problem whose split scratch would exceed 8 MiB (see
 *    vlak_attn_gqa_workspace_size) is rejected with VLAK_ERR_INVALID_ARGUMENT;
 *    use vlak_attn_gqa_fwd_ws for it.
 *  - Every call on a device shares the buffer: calls whose GPU work overlaps
 *    (different streams) race on it and corrupt each other's results; keep
 *    them ordered on one stream. No part of it has to start at zero: a call
 *    writes every entry its merge reads.
 *  - It does not set up the host error word either: a failed wait is
 *    reported there only if an earlier call of another entry point created
 *    it, else in the per-device word (vlak_device_error_read). */
VLAK_API int vlak_attn_gqa_fwd_noalloc(const vlak_attn_gqa_args* args, void* stream);

/* Non-GQA attention on the CUDA cores with fp32 math: the v1 path of
 * vlak::fused_attention for fp32 / fp16 / fp64 inputs (replaces
 * fused_attention_warp_row and its host branch,
 * kernels/attention/fused_attention.cu:28-79, :578-592).
 *   q, o : (B, H, M, 64) contiguous; k, v : (B, H, N, 64) contiguous
 *   dtype: VLAK_F32 / VLAK_F16 / VLAK_BF16 / VLAK_F64
 *   mask : optional bool (B, M, N) contiguous, broadcast over heads (NULL = none)
 *   scale: <= 0 selects 1/sqrt(64)
 * A row with no visible key is written as zeros. */
VLAK_API int vlak_attn_fwd(const void* q, const void* k, const void* v, void* o, int dtype,
                           int64_t B, int64_t H, int64_t M, int64_t N, const void* mask,
                           double scale, void* stream);

/* Self-test of the bounded device waits. No counterpart in the reference:
 * a test hook for the failure path that replaces a hang. Launches, on
 * `stream`, one kernel that waits on a barrier nothing completes; after the
 * 1 s wait limit it records VLAK_ERR_DEVICE_TIMEOUT as a failed attention
 * wait would (read it with vlak_device_error_poll or vlak_device_error_read)
 * and returns, leaving the context usable. */
VLAK_API int vlak_selftest_wait_timeout(void* stream);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* VLAK_B200_H_ */
