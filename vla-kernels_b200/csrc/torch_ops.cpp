// torch.ops.vlak registration for the B200 build: the reference's operator
// schemas, byte for byte, with CUDA implementations that validate, allocate the
// output through the caching allocator and call the C ABI of libvlak_b200.so on
// the current stream. No CUDA code lives here.
//
// Schemas: kernels/softmax/softmax_kernels.cu:303-305,
//          kernels/attention/fused_attention.cu:671-676,
//          kernels/attention/fused_attention_v4.cu:333-336;
// plus two additive schemas with no counterpart in the reference:
// fused_attention_gqa_varlen (per-sample lengths) and device_error (the
// synchronous check of the bounded-wait error words).

#include <ATen/ATen.h>
#include <c10/cuda/CUDAFunctions.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include <algorithm>
#include <optional>

#include "vlak_b200.h"

namespace {

void check_status(int status, const char* op) {
  TORCH_CHECK(status == VLAK_OK, op, ": ", vlak_last_error_message(), " (",
              vlak_status_string(status), ")");
}

// Every op first reads the host-mapped error word (no device
// synchronization): a bounded wait that ran out in an attention kernel which
// has finished since is raised here, on the caller's next op, instead of
// going unnoticed. The word is cleared by the read, so the following call
// runs normally.
void raise_pending_device_error(const char* op) {
  int code = VLAK_OK;
  vlak_device_error_poll(&code);
  TORCH_CHECK(code == VLAK_OK, op, ": an earlier vlak kernel gave up a bounded device wait (",
              vlak_status_string(code), "); the output of that call is incomplete");
}

// vlak::device_error(): the synchronous check. Waits for the device, then
// reads and clears the error words; returns the status found (0 = none).
int64_t device_error() {
  int code = VLAK_OK;
  c10::cuda::device_synchronize();
  check_status(vlak_device_error_read(&code), "vlak::device_error");
  return code;
}

int dtype_code(at::ScalarType t) {
  switch (t) {
    case at::kFloat: return VLAK_F32;
    case at::kHalf: return VLAK_F16;
    case at::kBFloat16: return VLAK_BF16;
    case at::kDouble: return VLAK_F64;
    default: return -1;
  }
}

// kernels/softmax/softmax_kernels.cu:255-297
at::Tensor softmax_lastdim(const at::Tensor& x_in, int64_t version) {
  raise_pending_device_error("vlak::softmax");
  TORCH_CHECK(x_in.is_cuda(), "input must be CUDA");
  TORCH_CHECK(x_in.dim() == 2, "expected a 2D [rows, cols] tensor");
  const int dt = dtype_code(x_in.scalar_type());
  TORCH_CHECK(dt >= 0, "softmax_lastdim: unsupported dtype ", x_in.scalar_type());
  c10::cuda::CUDAGuard guard(x_in.device());
  at::Tensor x = x_in.contiguous();
  at::Tensor y = at::empty_like(x, at::MemoryFormat::Contiguous);
  const int st = vlak_softmax_fwd(x.data_ptr(), y.data_ptr(), x.size(0), x.size(1), dt,
                                  static_cast<int>(version),
                                  c10::cuda::getCurrentCUDAStream().stream());
  check_status(st, "softmax kernel launch failed");
  return y;
}

vlak_attn_gqa_args gqa_args(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                            double scale, int64_t prefix_len, int64_t dead_start,
                            int64_t dead_end, const char* op) {
  // kernels/attention/fused_attention.cu:606-626
  TORCH_CHECK(q.is_cuda() && q.dim() == 4 && k.dim() == 4 && v.dim() == 4,
              "expected 4D CUDA tensors (B, seq, heads, 64)");
  TORCH_CHECK(k.is_cuda() && v.is_cuda() && k.device() == q.device() && v.device() == q.device(),
              "q, k and v must be on the same CUDA device");
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && k.scalar_type() == at::kBFloat16 &&
                  v.scalar_type() == at::kBFloat16,
              op, " is bf16-only");
  TORCH_CHECK(q.size(3) == 64 && k.size(3) == 64 && v.size(3) == 64, "head_dim must be 64");
  TORCH_CHECK(q.stride(3) == 1 && k.stride(3) == 1 && v.stride(3) == 1,
              "head_dim must be the contiguous dim");
  const int64_t B = q.size(0), M = q.size(1), H = q.size(2);
  const int64_t N = k.size(1), Hkv = k.size(2);
  TORCH_CHECK(k.size(0) == B && v.size(0) == B && v.size(1) == N && v.size(2) == Hkv &&
                  k.sizes() == v.sizes(),
              "k/v shape mismatch");
  TORCH_CHECK(Hkv > 0 && H % Hkv == 0, "query heads must be a multiple of kv heads");
  vlak_attn_gqa_args a{};
  a.q = q.data_ptr();
  a.k = k.data_ptr();
  a.v = v.data_ptr();
  a.B = B; a.M = M; a.N = N; a.H = H; a.Hkv = Hkv;
  for (int d = 0; d < 3; ++d) {
    a.q_stride[d] = q.stride(d);
    a.k_stride[d] = k.stride(d);
    a.v_stride[d] = v.stride(d);
  }
  a.scale = scale;
  a.prefix_len = prefix_len;
  a.dead_start = dead_start;
  a.dead_end = dead_end;
  return a;
}

// Key-split workspace for small batches, from the caching allocator on the
// current stream (its memory is reused only by work queued after this call
// on that stream). Undefined when the launch will not split.
at::Tensor split_workspace(const vlak_attn_gqa_args& a, const at::Tensor& like) {
  int64_t bytes = 0;
  check_status(vlak_attn_gqa_workspace_size(&a, &bytes), "fused_attention workspace size");
  if (bytes == 0) return at::Tensor();
  return at::empty({bytes}, like.options().dtype(at::kByte));
}
void* ws_ptr(const at::Tensor& ws) { return ws.defined() ? ws.data_ptr() : nullptr; }
int64_t ws_bytes(const at::Tensor& ws) { return ws.defined() ? ws.numel() : 0; }

at::Tensor run_gqa(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, double scale,
                   int64_t prefix_len, int64_t dead_start, int64_t dead_end, bool v4) {
  raise_pending_device_error(v4 ? "vlak::fused_attention_gqa_v4" : "vlak::fused_attention_gqa");
  const char* op = v4 ? "v4" : "v3";
  vlak_attn_gqa_args a = gqa_args(q, k, v, scale, prefix_len, dead_start, dead_end, op);
  c10::cuda::CUDAGuard guard(q.device());
  // validate before allocating so contract errors surface without side effects
  check_status(vlak_attn_gqa_check(&a, nullptr, nullptr),
               v4 ? "fused_attention_gqa_v4" : "fused_attention_gqa");
  at::Tensor o = at::empty({a.B, a.M, a.H, 64}, q.options());
  a.o = o.data_ptr();
  a.o_stride[0] = o.stride(0);
  a.o_stride[1] = o.stride(1);
  a.o_stride[2] = o.stride(2);
  void* stream = c10::cuda::getCurrentCUDAStream().stream();
  // v3 and v4 share one kernel; the workspace variant serves both
  const at::Tensor ws = split_workspace(a, q);
  const int st = vlak_attn_gqa_fwd_ws(&a, ws_ptr(ws), ws_bytes(ws), stream);
  check_status(st, v4 ? "fused_attention_gqa_v4 launch failed" : "fused_attention_gqa launch failed");
  return o;
}

at::Tensor fused_attention_gqa(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                               double scale, int64_t prefix_len, int64_t dead_start,
                               int64_t dead_end) {
  return run_gqa(q, k, v, scale, prefix_len, dead_start, dead_end, false);
}

at::Tensor fused_attention_gqa_v4(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                                  double scale, int64_t prefix_len, int64_t dead_start,
                                  int64_t dead_end) {
  return run_gqa(q, k, v, scale, prefix_len, dead_start, dead_end, true);
}

// kernels/attention/fused_attention.cu:525-598: (B, H, M, 64) layout, no GQA.
// bf16 runs on the tensor cores (the reference's v2): analytic prefix mask
// when prefix_len >= 0 (it wins over attn_mask, as there), else the bool
// mask, else unmasked. fp32 / fp16 / fp64 run on the CUDA cores (v1), which
// take no analytic mask.
at::Tensor fused_attention(const at::Tensor& q_in, const at::Tensor& k_in, const at::Tensor& v_in,
                           double scale, const std::optional<at::Tensor>& attn_mask,
                           int64_t prefix_len) {
  raise_pending_device_error("vlak::fused_attention");
  TORCH_CHECK(q_in.is_cuda() && q_in.dim() == 4, "expected 4D CUDA (B,H,M,D)");
  TORCH_CHECK(q_in.size(3) == 64, "this kernel is specialized to head_dim 64");
  TORCH_CHECK(k_in.dim() == 4 && v_in.dim() == 4 && k_in.size(3) == 64 && v_in.size(3) == 64,
              "k/v head_dim 64");
  TORCH_CHECK(k_in.size(2) == v_in.size(2), "k/v length mismatch");
  TORCH_CHECK(k_in.size(0) == q_in.size(0) && k_in.size(1) == q_in.size(1) &&
                  v_in.size(0) == q_in.size(0) && v_in.size(1) == q_in.size(1),
              "k/v must be (B, H, N, 64) with the batch and heads of q");
  TORCH_CHECK(k_in.device() == q_in.device() && v_in.device() == q_in.device(),
              "q, k and v must be on the same CUDA device");
  TORCH_CHECK(k_in.scalar_type() == q_in.scalar_type() && v_in.scalar_type() == q_in.scalar_type(),
              "q, k and v must have the same dtype");
  const int dt = dtype_code(q_in.scalar_type());
  TORCH_CHECK(dt >= 0, "fused_attention: unsupported dtype ", q_in.scalar_type());
  c10::cuda::CUDAGuard guard(q_in.device());
  at::Tensor q = q_in.contiguous(), k = k_in.contiguous(), v = v_in.contiguous();
  const int64_t B = q.size(0), H = q.size(1), M = q.size(2), N = k.size(2);
  at::Tensor o = at::empty_like(q, at::MemoryFormat::Contiguous);
  at::Tensor mask;
  if (attn_mask.has_value()) {
    mask = attn_mask->contiguous();
    TORCH_CHECK(mask.scalar_type() == at::kBool, "attn_mask must be bool");
    TORCH_CHECK(mask.dim() == 3 && mask.size(0) == B && mask.size(1) == M && mask.size(2) == N,
                "attn_mask must be (B, M, N)");
    TORCH_CHECK(mask.device() == q.device(), "attn_mask must be on the device of q");
  }
  if (B * H * M == 0) return o;
  void* stream = c10::cuda::getCurrentCUDAStream().stream();
  if (dt == VLAK_BF16) {
    vlak_attn_gqa_args a{};
    a.q = q.data_ptr(); a.k = k.data_ptr(); a.v = v.data_ptr(); a.o = o.data_ptr();
    a.B = B; a.M = M; a.N = N; a.H = H; a.Hkv = H;
    // (B, H, seq, 64) seen as (B, seq, H, 64): strides of dims (b, seq, h)
    const at::Tensor* ts[4] = {&q, &k, &v, &o};
    int64_t* st[4] = {a.q_stride, a.k_stride, a.v_stride, a.o_stride};
    for (int i = 0; i < 4; ++i) {
      st[i][0] = ts[i]->stride(0);
      st[i][1] = ts[i]->stride(2);
      st[i][2] = ts[i]->stride(1);
    }
    a.scale = scale;
    a.prefix_len = -1;
    int status;
    if (prefix_len >= 0) a.prefix_len = std::min(prefix_len, N);  // a prefix past N shows every key
    const at::Tensor ws = split_workspace(a, q);
    if (mask.defined() && prefix_len < 0) {
      status = vlak_attn_gqa_masked_fwd_ws(&a, mask.data_ptr(), M * N, N, ws_ptr(ws), ws_bytes(ws),
                                           stream);
    } else {
      status = vlak_attn_gqa_fwd_ws(&a, ws_ptr(ws), ws_bytes(ws), stream);
    }
    check_status(status, "fused_attention launch failed");
    return o;
  }
  TORCH_CHECK(prefix_len < 0, "analytic prefix mask requires the bf16 tensor-core path");
  const int status = vlak_attn_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), dt, B,
                                   H, M, N, mask.defined() ? mask.data_ptr() : nullptr, scale,
                                   stream);
  check_status(status, "fused_attention launch failed");
  return o;
}

// Per-sample-length GQA attention (new schema; the reference leaves this
// site, the C4 prefix attention, on SDPA with a materialised mask).
at::Tensor fused_attention_gqa_varlen(const at::Tensor& q, const at::Tensor& k,
                                      const at::Tensor& v, const at::Tensor& lengths_in,
                                      double scale) {
  raise_pending_device_error("vlak::fused_attention_gqa_varlen");
  vlak_attn_gqa_args a = gqa_args(q, k, v, scale, -1, 0, 0, "fused_attention_gqa_varlen");
  TORCH_CHECK(lengths_in.is_cuda() && lengths_in.device() == q.device(),
              "lengths must be on the device of q");
  TORCH_CHECK(lengths_in.dim() == 1 && lengths_in.size(0) == a.B, "lengths must be (B,)");
  TORCH_CHECK(lengths_in.scalar_type() == at::kInt || lengths_in.scalar_type() == at::kLong,
              "lengths must be int32 or int64");
  c10::cuda::CUDAGuard guard(q.device());
  at::Tensor lengths = lengths_in.contiguous();
  check_status(vlak_attn_gqa_check(&a, nullptr, nullptr), "fused_attention_gqa_varlen");
  at::Tensor o = at::empty({a.B, a.M, a.H, 64}, q.options());
  a.o = o.data_ptr();
  a.o_stride[0] = o.stride(0);
  a.o_stride[1] = o.stride(1);
  a.o_stride[2] = o.stride(2);
  const at::Tensor ws = split_workspace(a, q);
  const int st = vlak_attn_gqa_varlen_fwd_ws(
      &a, lengths.data_ptr(), lengths.scalar_type() == at::kLong ? VLAK_I64 : VLAK_I32, ws_ptr(ws),
      ws_bytes(ws), c10::cuda::getCurrentCUDAStream().stream());
  check_status(st, "fused_attention_gqa_varlen launch failed");
  return o;
}

}  // namespace

TORCH_LIBRARY_FRAGMENT(vlak, m) {
  m.def(
      "fused_attention(Tensor q, Tensor k, Tensor v, float scale=-1., "
      "Tensor? attn_mask=None, int prefix_len=-1) -> Tensor");
  m.def(
      "fused_attention_gqa_varlen(Tensor q, Tensor k, Tensor v, Tensor lengths, "
      "float scale=-1.) -> Tensor");
  m.def("softmax(Tensor x, int version=4) -> Tensor");
  m.def("device_error() -> int");
  m.def(
      "fused_attention_gqa(Tensor q, Tensor k, Tensor v, float scale=-1., "
      "int prefix_len=-1, int dead_start=0, int dead_end=0) -> Tensor");
  m.def(
      "fused_attention_gqa_v4(Tensor q, Tensor k, Tensor v, float scale=-1., "
      "int prefix_len=-1, int dead_start=0, int dead_end=0) -> Tensor");
}

TORCH_LIBRARY_IMPL(vlak, CompositeExplicitAutograd, m) {
  m.impl("device_error", &device_error);
}

TORCH_LIBRARY_IMPL(vlak, CUDA, m) {
  m.impl("softmax", &softmax_lastdim);
  m.impl("fused_attention_gqa", &fused_attention_gqa);
  m.impl("fused_attention_gqa_v4", &fused_attention_gqa_v4);
  m.impl("fused_attention", &fused_attention);
  m.impl("fused_attention_gqa_varlen", &fused_attention_gqa_varlen);
}
