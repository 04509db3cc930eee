// Non-GQA fused attention on the CUDA cores, for the element types the
// tensor-core kernel does not take (fp32, fp16, fp64; bf16 is accepted too).
//
// Contract (the reference's v1 path of vlak::fused_attention,
// kernels/attention/fused_attention.cu:28-79 kernel, :525-598 host):
//   q (B, H, M, 64), k and v (B, H, N, 64), o (B, H, M, 64), all contiguous;
//   optional bool mask (B, M, N) broadcast over heads (true = attend);
//   scores, softmax and P.V in fp32, output rounded to the input type.
// Difference by design: a row with no visible key is written as zeros (the
// reference divides 0 by a zero row sum and produces NaN there).
//
// B200 design: one CTA per block of 8 query rows of one (b, h), one warp per
// row. 64-key tiles of K and V are staged in shared memory as fp32 (K rows
// padded to 65 words, so the 32 lanes reading 32 different keys hit 32
// different banks) and shared by the CTA's 8 rows. Lane l scores keys l and
// l + 32 of the tile against the row's query (held in registers), the warp
// reduces the tile max and sum with shuffles, and lane l accumulates output
// dims l and l + 32 with the tile's probabilities broadcast by shuffle.

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "vlak_device.cuh"
#include "vlak_internal.h"

namespace vlak {
namespace {

constexpr int kRowsPerCta = 8;  // one warp per query row
constexpr int kTile = 64;       // keys per shared-memory tile
constexpr int kD = 64;          // head dim
constexpr int kKPitch = kD + 1; // padded K row (words)

template <typename T> __device__ __forceinline__ float to_f(T v);
template <> __device__ __forceinline__ float to_f<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f<double>(double v) { return static_cast<float>(v); }
template <> __device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <typename T> __device__ __forceinline__ T from_f(float v);
template <> __device__ __forceinline__ float from_f<float>(float v) { return v; }
template <> __device__ __forceinline__ double from_f<double>(float v) { return v; }
template <> __device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

template <typename T>
__global__ void __launch_bounds__(32 * kRowsPerCta)
attention_rows_simt(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                    T* __restrict__ o, const uint8_t* __restrict__ mask, int H, int M, int N,
                    float scale) {
  __shared__ float ks[kTile * kKPitch];
  __shared__ float vs[kTile * kD];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.y;
  const int b = bh / H;
  const int m = blockIdx.x * kRowsPerCta + warp;
  const bool row_ok = m < M;
  const T* kb = k + static_cast<size_t>(bh) * N * kD;
  const T* vb = v + static_cast<size_t>(bh) * N * kD;
  const uint8_t* mrow = (mask && row_ok) ? mask + (static_cast<size_t>(b) * M + m) * N : nullptr;

  float qr[kD];
  {
    const T* qp = q + (static_cast<size_t>(bh) * M + (row_ok ? m : 0)) * kD;
#pragma unroll
    for (int d = 0; d < kD; ++d) qr[d] = to_f(qp[d]) * scale;
  }
  float m_run = -INFINITY, l_run = 0.f, o0 = 0.f, o1 = 0.f;

  for (int n0 = 0; n0 < N; n0 += kTile) {
    __syncthreads();  // the previous tile is no longer read
    for (int i = threadIdx.x; i < kTile * kD; i += 32 * kRowsPerCta) {
      const int key = i / kD, d = i % kD;
      const bool in = n0 + key < N;
      ks[key * kKPitch + d] = in ? to_f(kb[static_cast<size_t>(n0 + key) * kD + d]) : 0.f;
      vs[key * kD + d] = in ? to_f(vb[static_cast<size_t>(n0 + key) * kD + d]) : 0.f;
    }
    __syncthreads();
    if (!row_ok) continue;

    // scores of keys n0 + lane and n0 + lane + 32
    float s[2];
    bool vis[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int key = lane + 32 * h;
      const float* kr = ks + key * kKPitch;
      float acc = 0.f;
#pragma unroll
      for (int d = 0; d < kD; ++d) acc = fmaf(qr[d], kr[d], acc);
      vis[h] = (n0 + key < N) && (!mrow || mrow[n0 + key] != 0);
      s[h] = vis[h] ? acc : -INFINITY;
    }
    const float tmax = warp_max(fmaxf(s[0], s[1]));
    const float m_new = fmaxf(m_run, tmax);
    if (m_new == -INFINITY) continue;  // nothing visible so far
    const float alpha = expf(m_run - m_new);  // 0 while m_run is -inf
    const float p0 = vis[0] ? expf(s[0] - m_new) : 0.f;
    const float p1 = vis[1] ? expf(s[1] - m_new) : 0.f;
    l_run = l_run * alpha + warp_sum(p0 + p1);
    o0 *= alpha;
    o1 *= alpha;
#pragma unroll 8
    for (int j = 0; j < 32; ++j) {
      const float pa = __shfl_sync(kFullMask, p0, j);
      const float pb = __shfl_sync(kFullMask, p1, j);
      o0 = fmaf(pa, vs[j * kD + lane], o0);
      o1 = fmaf(pa, vs[j * kD + lane + 32], o1);
      o0 = fmaf(pb, vs[(j + 32) * kD + lane], o0);
      o1 = fmaf(pb, vs[(j + 32) * kD + lane + 32], o1);
    }
    m_run = m_new;
  }
  if (!row_ok) return;
  const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
  T* orow = o + (static_cast<size_t>(bh) * M + m) * kD;
  orow[lane] = from_f<T>(o0 * inv);
  orow[lane + 32] = from_f<T>(o1 * inv);
}

template <typename T>
cudaError_t launch(const void* q, const void* k, const void* v, void* o, const void* mask,
                   int B, int H, int M, int N, float scale, cudaStream_t st) {
  const dim3 grid((M + kRowsPerCta - 1) / kRowsPerCta, B * H);
  attention_rows_simt<T><<<grid, 32 * kRowsPerCta, 0, st>>>(
      static_cast<const T*>(q), static_cast<const T*>(k), static_cast<const T*>(v),
      static_cast<T*>(o), static_cast<const uint8_t*>(mask), H, M, N, scale);
  return cudaGetLastError();
}

}  // namespace
}  // namespace vlak

extern "C" int vlak_attn_fwd(const void* q, const void* k, const void* v, void* o, int dtype,
                             int64_t B, int64_t H, int64_t M, int64_t N, const void* mask,
                             double scale, void* stream) {
  using namespace vlak;
  clear_error();
  if (B < 0 || H < 0 || M < 0 || N < 0)
    return set_error(VLAK_ERR_INVALID_ARGUMENT, "fused_attention: negative size");
  if (B * H > 65535 || M > INT32_MAX || N > INT32_MAX)
    return set_error(VLAK_ERR_INVALID_ARGUMENT, "fused_attention: B*H must be at most 65535");
  if (dtype != VLAK_F32 && dtype != VLAK_F16 && dtype != VLAK_BF16 && dtype != VLAK_F64)
    return set_error(VLAK_ERR_UNSUPPORTED_DTYPE, "fused_attention: unsupported dtype");
  if (B == 0 || H == 0 || M == 0) return VLAK_OK;
  if (!q || !o || (N > 0 && (!k || !v)))
    return set_error(VLAK_ERR_INVALID_ARGUMENT, "fused_attention: null tensor pointer");
  const float sc = scale > 0 ? static_cast<float>(scale) : 0.125f;  // 1/sqrt(64)
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int b = static_cast<int>(B), h = static_cast<int>(H), m = static_cast<int>(M),
            n = static_cast<int>(N);
  cudaError_t e;
  switch (dtype) {
    case VLAK_F32: e = launch<float>(q, k, v, o, mask, b, h, m, n, sc, st); break;
    case VLAK_F16: e = launch<__half>(q, k, v, o, mask, b, h, m, n, sc, st); break;
    case VLAK_BF16: e = launch<__nv_bfloat16>(q, k, v, o, mask, b, h, m, n, sc, st); break;
    default: e = launch<double>(q, k, v, o, mask, b, h, m, n, sc, st); break;
  }
  if (e != cudaSuccess) return set_cuda_error("fused_attention launch failed", e);
  return VLAK_OK;
}
