// torch.ops.vlak registration for the B200 build: the reference's operator
// schemas, byte for byte, with CUDA implementations that validate, allocate the
// output through the caching allocator and call the C ABI of libvlak_b200.so on
// the current stream. No CUDA code lives here.
//
// Schemas: kernels/softmax/softmax_kernels.cu:303-305,
//          kernels/attention/fused_attention.cu:671-676,
//          kernels/attention/fused_attention_v4.cu:333-336.

#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include "vlak_b200.h"

namespace {

void check_status(int status, const char* op) {
  TORCH_CHECK(status == VLAK_OK, op, ": ", vlak_last_error_message(), " (",
              vlak_status_string(status), ")");
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

at::Tensor run_gqa(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, double scale,
                   int64_t prefix_len, int64_t dead_start, int64_t dead_end, bool v4) {
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
  const int st = v4 ? vlak_attn_gqa_v4_fwd(&a, stream) : vlak_attn_gqa_fwd(&a, stream);
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

}  // namespace

TORCH_LIBRARY_FRAGMENT(vlak, m) {
  m.def("softmax(Tensor x, int version=4) -> Tensor");
  m.def(
      "fused_attention_gqa(Tensor q, Tensor k, Tensor v, float scale=-1., "
      "int prefix_len=-1, int dead_start=0, int dead_end=0) -> Tensor");
  m.def(
      "fused_attention_gqa_v4(Tensor q, Tensor k, Tensor v, float scale=-1., "
      "int prefix_len=-1, int dead_start=0, int dead_end=0) -> Tensor");
}

TORCH_LIBRARY_IMPL(vlak, CUDA, m) {
  m.impl("softmax", &softmax_lastdim);
  m.impl("fused_attention_gqa", &fused_attention_gqa);
  m.impl("fused_attention_gqa_v4", &fused_attention_gqa_v4);
}
