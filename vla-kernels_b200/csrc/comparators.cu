// Library comparators for the row softmax (benchmark bars, not the product
// path): the vendor softmax of cuDNN and a block-per-row softmax built on
// CUB's BlockReduce. They restate what the reference's comparator extension
// provides (kernels/softmax/softmax_baselines.cu:23-55 and :57-117, exposed as
// softmax_cudnn / softmax_cub by kernels/softmax/__init__.py:78-114), behind
// the C ABI of include/vlak_comparators.h. Built into their own library,
// libvlak_comparators.so, so the product library does not depend on cuDNN.

#include <cub/block/block_reduce.cuh>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cudnn.h>
#include <math.h>
#include <stdint.h>

#include <mutex>
#include <string>

#include "../../include/vlak_comparators.h"

namespace {

thread_local std::string t_error;

int fail(int status, const std::string& msg) {
  t_error = msg;
  return status;
}

template <typename T> __device__ __forceinline__ float to_f(T v) { return static_cast<float>(v); }
template <> __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
template <> __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
template <typename T> __device__ __forceinline__ T from_f(float v) { return static_cast<T>(v); }
template <> __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }

struct MaxOp {
  __device__ __forceinline__ float operator()(float a, float b) const { return fmaxf(a, b); }
};

// One block per row: the row max and the sum of exponentials each come from
// one cub::BlockReduce over the threads' strided partials, then a third pass
// writes exp(x - max) / sum. fp32 arithmetic whatever the storage type.
template <typename T, int kThreads>
__global__ void __launch_bounds__(kThreads) softmax_cub_rows(const T* __restrict__ x,
                                                             T* __restrict__ y, int64_t cols) {
  using Reduce = cub::BlockReduce<float, kThreads>;
  __shared__ typename Reduce::TempStorage tmp;
  __shared__ float row_max, row_inv;
  const T* xr = x + static_cast<int64_t>(blockIdx.x) * cols;
  T* yr = y + static_cast<int64_t>(blockIdx.x) * cols;

  float m = -INFINITY;
  for (int64_t c = threadIdx.x; c < cols; c += kThreads) m = fmaxf(m, to_f(xr[c]));
  m = Reduce(tmp).Reduce(m, MaxOp());
  if (threadIdx.x == 0) row_max = m;
  __syncthreads();
  m = row_max;

  float s = 0.f;
  for (int64_t c = threadIdx.x; c < cols; c += kThreads) s += expf(to_f(xr[c]) - m);
  __syncthreads();  // tmp is reused
  s = Reduce(tmp).Sum(s);
  if (threadIdx.x == 0) row_inv = 1.f / s;
  __syncthreads();
  const float inv = row_inv;
  for (int64_t c = threadIdx.x; c < cols; c += kThreads) yr[c] = from_f<T>(expf(to_f(xr[c]) - m) * inv);
}

// One cuDNN handle per (device, host thread), bound to the caller's stream
// at each call.
int cudnn_handle(cudnnHandle_t* out) {
  constexpr int kMaxDev = 64;
  thread_local cudnnHandle_t handles[kMaxDev] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev)
    return fail(VLAK_CMP_ERR_CUDA, "cudaGetDevice failed");
  if (!handles[dev]) {
    cudnnStatus_t s = cudnnCreate(&handles[dev]);
    if (s != CUDNN_STATUS_SUCCESS) return fail(VLAK_CMP_ERR_CUDNN, cudnnGetErrorString(s));
  }
  *out = handles[dev];
  return VLAK_CMP_OK;
}

}  // namespace

extern "C" const char* vlak_cmp_last_error_message(void) { return t_error.c_str(); }

extern "C" int vlak_softmax_cub_fwd(const void* x, void* y, int64_t rows, int64_t cols, int dtype,
                                    void* stream) {
  t_error.clear();
  if (rows < 0 || cols < 0) return fail(VLAK_CMP_ERR_INVALID_ARGUMENT, "negative size");
  if (rows == 0 || cols == 0) return VLAK_CMP_OK;
  if (rows > INT32_MAX) return fail(VLAK_CMP_ERR_INVALID_ARGUMENT, "too many rows");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  constexpr int kThreads = 256;
  const dim3 grid(static_cast<unsigned>(rows));
  switch (dtype) {
    case VLAK_CMP_F32:
      softmax_cub_rows<float, kThreads><<<grid, kThreads, 0, s>>>(
          static_cast<const float*>(x), static_cast<float*>(y), cols);
      break;
    case VLAK_CMP_F16:
      softmax_cub_rows<__half, kThreads><<<grid, kThreads, 0, s>>>(
          static_cast<const __half*>(x), static_cast<__half*>(y), cols);
      break;
    case VLAK_CMP_BF16:
      softmax_cub_rows<__nv_bfloat16, kThreads><<<grid, kThreads, 0, s>>>(
          static_cast<const __nv_bfloat16*>(x), static_cast<__nv_bfloat16*>(y), cols);
      break;
    default:
      return fail(VLAK_CMP_ERR_UNSUPPORTED_DTYPE, "dtype must be f32, f16 or bf16");
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(VLAK_CMP_ERR_CUDA, cudaGetErrorString(e));
  return VLAK_CMP_OK;
}

extern "C" int vlak_softmax_cudnn_fwd(const void* x, void* y, int64_t rows, int64_t cols,
                                      int dtype, void* stream) {
  t_error.clear();
  if (rows < 0 || cols < 0) return fail(VLAK_CMP_ERR_INVALID_ARGUMENT, "negative size");
  if (rows == 0 || cols == 0) return VLAK_CMP_OK;
  if (rows > INT32_MAX || cols > INT32_MAX) return fail(VLAK_CMP_ERR_INVALID_ARGUMENT, "size exceeds 2^31-1");
  cudnnDataType_t dt;
  switch (dtype) {
    case VLAK_CMP_F32: dt = CUDNN_DATA_FLOAT; break;
    case VLAK_CMP_F16: dt = CUDNN_DATA_HALF; break;
    case VLAK_CMP_BF16: dt = CUDNN_DATA_BFLOAT16; break;
    default: return fail(VLAK_CMP_ERR_UNSUPPORTED_DTYPE, "dtype must be f32, f16 or bf16");
  }
  cudnnHandle_t h;
  int st = cudnn_handle(&h);
  if (st != VLAK_CMP_OK) return st;
  cudnnStatus_t s = cudnnSetStream(h, static_cast<cudaStream_t>(stream));
  if (s != CUDNN_STATUS_SUCCESS) return fail(VLAK_CMP_ERR_CUDNN, cudnnGetErrorString(s));
  // the [rows, cols] matrix as an NCHW tensor (rows, cols, 1, 1); softmax
  // over C, H, W of each instance n is the row softmax
  cudnnTensorDescriptor_t d;
  s = cudnnCreateTensorDescriptor(&d);
  if (s != CUDNN_STATUS_SUCCESS) return fail(VLAK_CMP_ERR_CUDNN, cudnnGetErrorString(s));
  s = cudnnSetTensor4dDescriptor(d, CUDNN_TENSOR_NCHW, dt, static_cast<int>(rows),
                                 static_cast<int>(cols), 1, 1);
  if (s == CUDNN_STATUS_SUCCESS) {
    const float one = 1.f, zero = 0.f;  // scaling factors are float for every data type here
    s = cudnnSoftmaxForward(h, CUDNN_SOFTMAX_ACCURATE, CUDNN_SOFTMAX_MODE_INSTANCE, &one, d, x,
                            &zero, d, y);
  }
  cudnnDestroyTensorDescriptor(d);
  if (s != CUDNN_STATUS_SUCCESS) return fail(VLAK_CMP_ERR_CUDNN, cudnnGetErrorString(s));
  return VLAK_CMP_OK;
}
