// Row softmax over the last dimension of a contiguous [rows, cols] tensor, for
// sm_100a. fp32 math for every element type.
//
// The reference dispatcher (kernels/softmax/softmax_kernels.cu:255-297) selects
// one of five algorithm families with an integer `version`; the same numbers
// select the same families here, each re-designed for B200's HBM3e:
//   0  one thread per row, scalar, three passes   (ladder baseline, :19-33)
//   1  one warp per row; the row is held in registers as 16-byte vectors and
//      read once; rows wider than the register budget stream twice  (:36-56)
//   2  one block per row, three vectorised passes (safe softmax)     (:59-87)
//   3  one block per row, online (max, sum) pass + write pass        (:101-139)
//   4  register-resident single read: one warp per row while the row fits a
//      warp's registers, else one block per row; beyond the block budget the
//      online two-pass stream                                     (:149-248)
//
// Every global access of versions 1-4 is a 16-byte vector. A row that does not
// start on a 16-byte boundary is split into a scalar head (< 8 elements), a
// vector body and a scalar tail. When x and y disagree modulo 16 bytes (an
// offset view), all versions fall back to the scalar online kernel.
//
// fp32 / fp64 (computed in fp32 like the reference's dispatch body): x - max
// is formed in fp32 exactly as torch does, exp is the accurate expf and the
// normalisation multiplies by the IEEE-rounded reciprocal of the row sum, which
// keeps the fp32 result within 1e-6 relative of the exact value. fp16 / bf16:
// exp2 on the MUFU unit.
// A row of all -inf yields NaN, as torch.softmax does.

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include <type_traits>

#include "vlak_device.cuh"
#include "vlak_internal.h"

namespace vlak {
namespace {

constexpr float kLog2e = 1.4426950408889634f;

// exp(x - m) at the precision each element type needs
template <typename T> __device__ __forceinline__ float exp_shift(float x, float m) {
  return ex2((x - m) * kLog2e);
}
template <> __device__ __forceinline__ float exp_shift<float>(float x, float m) {
  return expf(x - m);
}
template <> __device__ __forceinline__ float exp_shift<double>(float x, float m) {
  return expf(x - m);
}
// e / s as e times the row's reciprocal. `inv` is 1.f / s, an IEEE-rounded
// division done once per row, so the result is within about one ulp of the
// correctly rounded quotient (the fp32 bar is 1e-6 relative) at the cost of
// one multiply per element instead of a division.
template <typename T> __device__ __forceinline__ float normalize(float e, float s, float inv) {
  return e * inv;
}

// Segmentation of one row into scalar head, 16-byte body, scalar tail.
struct RowSeg {
  int head, nvec, tail;
};
template <typename T> __device__ __forceinline__ RowSeg row_seg(const T* p, int n) {
  constexpr int V = Elem<T>::kVec;
  const int mis = static_cast<int>(reinterpret_cast<uintptr_t>(p) & 15u);
  RowSeg s;
  s.head = mis ? min(n, (16 - mis) / static_cast<int>(sizeof(T))) : 0;
  s.nvec = (n - s.head) / V;
  s.tail = n - s.head - s.nvec * V;
  return s;
}

// Reductions over the threads that share one row.
struct WarpGroup {
  __device__ __forceinline__ float max(float v) const { return warp_max(v); }
  __device__ __forceinline__ float sum(float v) const { return warp_sum(v); }
};
// LPR consecutive lanes of a warp (LPR = 8 or 16): shuffles stay inside the
// lane group and name only its lanes, so a group whose row lies past the end
// of the tensor may return early.
template <int LPR> struct SubWarpGroup {
  unsigned mask;
  __device__ __forceinline__ float max(float v) const {
#pragma unroll
    for (int o = LPR / 2; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(mask, v, o));
    return v;
  }
  __device__ __forceinline__ float sum(float v) const {
#pragma unroll
    for (int o = LPR / 2; o > 0; o >>= 1) v += __shfl_xor_sync(mask, v, o);
    return v;
  }
};
// Whole block; two separate slots so max and sum need one barrier each.
template <int NT> struct BlockGroup {
  float* smax;
  float* ssum;
  __device__ __forceinline__ float reduce(float v, float* slot, bool is_max) const {
    v = is_max ? warp_max(v) : warp_sum(v);
    const int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) slot[w] = v;
    __syncthreads();
    float r = slot[0];
#pragma unroll
    for (int i = 1; i < NT / 32; ++i) r = is_max ? fmaxf(r, slot[i]) : r + slot[i];
    return r;
  }
  __device__ __forceinline__ float max(float v) const { return reduce(v, smax, true); }
  __device__ __forceinline__ float sum(float v) const { return reduce(v, ssum, false); }
};

// Register-resident row: the row is read from HBM exactly once. `t` is the
// thread's index within the NT threads that own the row; thread t holds body
// vectors t, t+NT, ... (at most RV of them), head element t and tail element t.
template <typename T, int RV, int NT, class Group>
__device__ __forceinline__ void row_softmax_reg(const T* __restrict__ xr, T* __restrict__ yr,
                                                int n, int t, const Group& grp) {
  using E = Elem<T>;
  constexpr int V = E::kVec;
  const RowSeg sg = row_seg(xr, n);
  float v[RV][V];
  float hv = -INFINITY, tv = -INFINITY;
  const char* xb = reinterpret_cast<const char*>(xr + sg.head);
#pragma unroll
  for (int i = 0; i < RV; ++i) {
    const int vi = t + i * NT;
    if (vi < sg.nvec) {
      E::unpack(ld_stream16(xb + static_cast<size_t>(vi) * 16), v[i]);
    } else {
#pragma unroll
      for (int j = 0; j < V; ++j) v[i][j] = -INFINITY;
    }
  }
  if (t < sg.head) hv = E::to_f(xr[t]);
  if (t < sg.tail) tv = E::to_f(xr[sg.head + sg.nvec * V + t]);

  float m = fmaxf(hv, tv);
#pragma unroll
  for (int i = 0; i < RV; ++i)
#pragma unroll
    for (int j = 0; j < V; ++j) m = fmaxf(m, v[i][j]);
  m = grp.max(m);

  float s = 0.f;
  if constexpr (sizeof(T) == 2) {
    // element pairs through the f32x2 FMA pipe: exp2(x log2e - m log2e); an
    // all -inf row gives NaN (as torch), a -inf element 0
    const float nb = -m * kLog2e;
    const uint64_t sc2 = f2_pack(kLog2e, kLog2e), nb2 = f2_pack(nb, nb);
    uint64_t s2 = f2_pack(0.f, 0.f);
#pragma unroll
    for (int i = 0; i < RV; ++i)
#pragma unroll
      for (int j = 0; j < V; j += 2) {
        float x0, x1;
        f2_unpack(f2_fma(f2_pack(v[i][j], v[i][j + 1]), sc2, nb2), x0, x1);
        v[i][j] = ex2(x0);
        v[i][j + 1] = ex2(x1);
        s2 = f2_add(s2, f2_pack(v[i][j], v[i][j + 1]));
      }
    float s0, s1;
    f2_unpack(s2, s0, s1);
    s = s0 + s1;
  } else {
#pragma unroll
    for (int i = 0; i < RV; ++i)
#pragma unroll
      for (int j = 0; j < V; ++j) {
        v[i][j] = exp_shift<T>(v[i][j], m);
        s += v[i][j];
      }
  }
  if (t < sg.head) { hv = exp_shift<T>(hv, m); s += hv; }
  if (t < sg.tail) { tv = exp_shift<T>(tv, m); s += tv; }
  s = grp.sum(s);
  const float inv = 1.f / s;

  char* yb = reinterpret_cast<char*>(yr + sg.head);
#pragma unroll
  for (int i = 0; i < RV; ++i) {
    const int vi = t + i * NT;
    if (vi < sg.nvec) {
      float o[V];
      if constexpr (sizeof(T) == 2) {
        const uint64_t inv2 = f2_pack(inv, inv);
#pragma unroll
        for (int j = 0; j < V; j += 2)
          f2_unpack(f2_mul(f2_pack(v[i][j], v[i][j + 1]), inv2), o[j], o[j + 1]);
      } else {
#pragma unroll
        for (int j = 0; j < V; ++j) o[j] = normalize<T>(v[i][j], s, inv);
      }
      st_stream16(yb + static_cast<size_t>(vi) * 16, E::pack(o));
    }
  }
  if (t < sg.head) yr[t] = E::from_f(normalize<T>(hv, s, inv));
  if (t < sg.tail) yr[sg.head + sg.nvec * V + t] = E::from_f(normalize<T>(tv, s, inv));
}

// Packed max of the eight 2-byte elements of a 16-byte vector pair-wise with
// an accumulator of four element pairs (exact; NaN handling as fmaxf).
template <typename T> struct Pair2;
template <> struct Pair2<__half> {
  using P = __half2;
  __device__ __forceinline__ static P neg_inf() { return __half2half2(__ushort_as_half(0xFC00u)); }
  __device__ __forceinline__ static P max(P a, P b) { return __hmax2(a, b); }
  __device__ __forceinline__ static float hmax(P a) {
    const float2 f = __half22float2(a);
    return fmaxf(f.x, f.y);
  }
};
template <> struct Pair2<__nv_bfloat16> {
  using P = __nv_bfloat162;
  __device__ __forceinline__ static P neg_inf() {
    return __bfloat162bfloat162(__ushort_as_bfloat16(0xFF80u));
  }
  __device__ __forceinline__ static P max(P a, P b) { return __hmax2(a, b); }
  __device__ __forceinline__ static float hmax(P a) {
    const float2 f = __bfloat1622float2(a);
    return fmaxf(f.x, f.y);
  }
};

// exp values of a row in (0, 1], held as pairs of the row's own 2-byte type
// between the sum and the output pass. fp16 rows keep f16 pairs (11
// significant bits; below 2^-14 an absolute error under 2^-25, which is also
// where fp16 outputs lose their own precision). bf16 rows keep bf16 pairs:
// 8 significant bits but bf16's 8-bit exponent, so tail probabilities far
// below 2^-24 survive, as they do in torch.softmax.
__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ void unpack_f16x2(uint32_t u, float& lo, float& hi) {
  asm("{\n\t.reg .f16 l, h;\n\tmov.b32 {l, h}, %2;\n\tcvt.f32.f16 %0, l;\n\tcvt.f32.f16 %1, h;\n\t}"
      : "=f"(lo), "=f"(hi) : "r"(u));
}
template <typename T>
__device__ __forceinline__ uint32_t pack_exp2(float lo, float hi) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
  } else {
    return pack_f16x2(lo, hi);
  }
}
template <typename T>
__device__ __forceinline__ void unpack_exp2(uint32_t u, float& lo, float& hi) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    lo = __uint_as_float(u << 16);  // bf16 -> f32 is a 16-bit shift
    hi = __uint_as_float(u & 0xffff0000u);
  } else {
    unpack_f16x2(u, lo, hi);
  }
}

// Register-resident row for 2-byte element types: the row stays in registers
// as the raw 16-byte vectors (4 registers per 8 elements, half the footprint
// of fp32 copies), so a 32768-column row fits 512 threads x 8 vectors at
// under 64 registers and two rows share an SM. The max runs on packed pairs;
// the sum pass evaluates each exp once and keeps it in the same registers as
// a pair of the row's type (pack_exp2), so the output pass only scales by
// 1 / sum: one MUFU operation per element, which is what bounds wide rows at
// full HBM rate. The outputs are the rounded exps times the fp32 reciprocal,
// rounded to the output type (fp16: within 2^-11 + one output ulp relative;
// bf16: within 2^-9 + one output ulp).
template <typename T, int RV, int NT, class Group>
__device__ __forceinline__ void row_softmax_reg_packed(const T* __restrict__ xr,
                                                       T* __restrict__ yr, int n, int t,
                                                       const Group& grp) {
  using E = Elem<T>;
  using H = Pair2<T>;
  using P = typename H::P;
  constexpr int V = E::kVec;
  const RowSeg sg = row_seg(xr, n);
  uint4 raw[RV];
  float hv = -INFINITY, tv = -INFINITY;
  const char* xb = reinterpret_cast<const char*>(xr + sg.head);
#pragma unroll
  for (int i = 0; i < RV; ++i) {
    const int vi = t + i * NT;
    if (vi < sg.nvec) raw[i] = ld_stream16(xb + static_cast<size_t>(vi) * 16);
  }
  if (t < sg.head) hv = E::to_f(xr[t]);
  if (t < sg.tail) tv = E::to_f(xr[sg.head + sg.nvec * V + t]);

  P pm[4] = {H::neg_inf(), H::neg_inf(), H::neg_inf(), H::neg_inf()};
#pragma unroll
  for (int i = 0; i < RV; ++i) {
    if (t + i * NT < sg.nvec) {
      const uint32_t w[4] = {raw[i].x, raw[i].y, raw[i].z, raw[i].w};
#pragma unroll
      for (int k = 0; k < 4; ++k) pm[k] = H::max(pm[k], *reinterpret_cast<const P*>(&w[k]));
    }
  }
  float m = fmaxf(fmaxf(H::hmax(H::max(pm[0], pm[1])), H::hmax(H::max(pm[2], pm[3]))),
                  fmaxf(hv, tv));
  m = grp.max(m);

  // Blocks of under 512 threads take pairs of elements through the f32x2 FMA
  // pipe, exp2(x log2e - m log2e), which saves issue slots where the kernel is
  // instruction-bound (4096 columns: 0.91 -> 1.00 of HBM). The 512-thread
  // blocks sit at the 64-register cap of two blocks per SM, where the paired
  // form measured slower, and keep the scalar form. Either way an all -inf
  // row gives NaN, as torch does, and a -inf element gives 0.
  constexpr bool kPairs = NT < 512;
  float s = 0.f;
  const float nb = -m * kLog2e;
  const uint64_t sc2 = f2_pack(kLog2e, kLog2e), nb2 = f2_pack(nb, nb);
  uint64_t s2 = f2_pack(0.f, 0.f);
#pragma unroll
  for (int i = 0; i < RV; ++i) {
    if (t + i * NT < sg.nvec) {
      float f[V];
      E::unpack(raw[i], f);
      uint32_t w[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        float e0, e1;
        if constexpr (kPairs) {
          float x0, x1;
          f2_unpack(f2_fma(f2_pack(f[2 * k], f[2 * k + 1]), sc2, nb2), x0, x1);
          e0 = ex2(x0);
          e1 = ex2(x1);
          s2 = f2_add(s2, f2_pack(e0, e1));
        } else {
          e0 = exp_shift<T>(f[2 * k], m);
          e1 = exp_shift<T>(f[2 * k + 1], m);
          s += e0 + e1;
        }
        w[k] = pack_exp2<T>(e0, e1);
      }
      raw[i] = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
  if constexpr (kPairs) {
    float s0, s1;
    f2_unpack(s2, s0, s1);
    s = s0 + s1;
  }
  if (t < sg.head) { hv = exp_shift<T>(hv, m); s += hv; }
  if (t < sg.tail) { tv = exp_shift<T>(tv, m); s += tv; }
  s = grp.sum(s);
  const float inv = 1.f / s;

  char* yb = reinterpret_cast<char*>(yr + sg.head);
  const uint64_t inv2 = f2_pack(inv, inv);
#pragma unroll
  for (int i = 0; i < RV; ++i) {
    const int vi = t + i * NT;
    if (vi < sg.nvec) {
      const uint32_t w[4] = {raw[i].x, raw[i].y, raw[i].z, raw[i].w};
      float f[V];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        float a, b;
        unpack_exp2<T>(w[k], a, b);
        if constexpr (kPairs) {
          f2_unpack(f2_mul(f2_pack(a, b), inv2), f[2 * k], f[2 * k + 1]);
        } else {
          f[2 * k] = a * inv;
          f[2 * k + 1] = b * inv;
        }
      }
      st_stream16(yb + static_cast<size_t>(vi) * 16, E::pack(f));
    }
  }
  if (t < sg.head) yr[t] = E::from_f(hv * inv);
  if (t < sg.tail) yr[sg.head + sg.nvec * V + t] = E::from_f(tv * inv);
}

// Online (max, sum) over this thread's share of the row, one 16-byte vector
// at a time; then a group merge. Returns the row's (m, l).
__device__ __forceinline__ void ml_update(float& m, float& l, float x) {
  // x is a new element; exp(-inf - -inf) cannot occur because m starts at
  // -inf only while l == 0 and the guarded form below keeps l finite
  const float mn = fmaxf(m, x);
  if (mn == -INFINITY) return;
  l = l * expf(m - mn) + expf(x - mn);
  m = mn;
}

template <typename T, int NT, bool kVector, class Group>
__device__ __forceinline__ void row_softmax_stream(const T* __restrict__ xr, T* __restrict__ yr,
                                                   int n, int t, const Group& grp,
                                                   bool three_pass) {
  using E = Elem<T>;
  constexpr int V = E::kVec;
  RowSeg sg;
  if (kVector) {
    sg = row_seg(xr, n);
  } else {
    sg.head = 0; sg.nvec = 0; sg.tail = n;
  }
  const char* xb = reinterpret_cast<const char*>(xr + sg.head);
  const int tail0 = sg.head + sg.nvec * V;
  float m, s;
  if (three_pass) {
    // pass 1: max
    float mx = -INFINITY;
    for (int vi = t; vi < sg.nvec; vi += NT) {
      float f[V];
      E::unpack(ld_stream16(xb + static_cast<size_t>(vi) * 16), f);
#pragma unroll
      for (int j = 0; j < V; ++j) mx = fmaxf(mx, f[j]);
    }
    for (int i = t; i < sg.head; i += NT) mx = fmaxf(mx, E::to_f(xr[i]));
    for (int i = t; i < sg.tail; i += NT) mx = fmaxf(mx, E::to_f(xr[tail0 + i]));
    m = grp.max(mx);
    // pass 2: sum
    float acc = 0.f;
    for (int vi = t; vi < sg.nvec; vi += NT) {
      float f[V];
      E::unpack(ld_stream16(xb + static_cast<size_t>(vi) * 16), f);
#pragma unroll
      for (int j = 0; j < V; ++j) acc += exp_shift<T>(f[j], m);
    }
    for (int i = t; i < sg.head; i += NT) acc += exp_shift<T>(E::to_f(xr[i]), m);
    for (int i = t; i < sg.tail; i += NT) acc += exp_shift<T>(E::to_f(xr[tail0 + i]), m);
    s = grp.sum(acc);
  } else {
    float ml = -INFINITY, ll = 0.f;
    for (int vi = t; vi < sg.nvec; vi += NT) {
      float f[V];
      E::unpack(ld_stream16(xb + static_cast<size_t>(vi) * 16), f);
      float vm = f[0];
#pragma unroll
      for (int j = 1; j < V; ++j) vm = fmaxf(vm, f[j]);
      const float mn = fmaxf(ml, vm);
      if (mn != -INFINITY) {
        float part = 0.f;
#pragma unroll
        for (int j = 0; j < V; ++j) part += exp_shift<T>(f[j], mn);
        ll = ll * exp_shift<T>(ml, mn) + part;
        ml = mn;
      }
    }
    for (int i = t; i < sg.head; i += NT) ml_update(ml, ll, E::to_f(xr[i]));
    for (int i = t; i < sg.tail; i += NT) ml_update(ml, ll, E::to_f(xr[tail0 + i]));
    // the row max, then every thread's partial sum rescaled to it
    m = grp.max(ml);
    const float scaled = (ml == -INFINITY) ? 0.f : ll * exp_shift<T>(ml, m);
    s = grp.sum(scaled);
  }
  // NaN for an all -inf row (m = -inf), matching torch
  if (m == -INFINITY) { m = NAN; }
  const float inv = 1.f / s;
  char* yb = reinterpret_cast<char*>(yr + sg.head);
  for (int vi = t; vi < sg.nvec; vi += NT) {
    float f[V];
    E::unpack(ld_stream16(xb + static_cast<size_t>(vi) * 16), f);
#pragma unroll
    for (int j = 0; j < V; ++j) f[j] = normalize<T>(exp_shift<T>(f[j], m), s, inv);
    st_stream16(yb + static_cast<size_t>(vi) * 16, E::pack(f));
  }
  for (int i = t; i < sg.head; i += NT)
    yr[i] = E::from_f(normalize<T>(exp_shift<T>(E::to_f(xr[i]), m), s, inv));
  for (int i = t; i < sg.tail; i += NT)
    yr[tail0 + i] = E::from_f(normalize<T>(exp_shift<T>(E::to_f(xr[tail0 + i]), m), s, inv));
}

// ---- kernels ---------------------------------------------------------------

// v0: one thread per row, three scalar passes
template <typename T>
__global__ void softmax_thread_row(const T* __restrict__ x, T* __restrict__ y, int64_t rows,
                                   int cols) {
  using E = Elem<T>;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (row >= rows) return;
  const T* xr = x + row * cols;
  T* yr = y + row * cols;
  float m = -INFINITY;
  for (int c = 0; c < cols; ++c) m = fmaxf(m, E::to_f(xr[c]));
  if (m == -INFINITY) m = NAN;
  // one thread sums the whole row serially: a double accumulator keeps the
  // fp32 result within the same 1e-6 relative bound as the tree reductions
  double acc = 0.0;
  for (int c = 0; c < cols; ++c) acc += exp_shift<T>(E::to_f(xr[c]), m);
  const float s = static_cast<float>(acc);
  const float inv = 1.f / s;
  for (int c = 0; c < cols; ++c) yr[c] = E::from_f(normalize<T>(exp_shift<T>(E::to_f(xr[c]), m), s, inv));
}

// v1 / v4-narrow: one warp per row, register resident
template <typename T, int RV>
__global__ void __launch_bounds__(256) softmax_warp_reg(const T* __restrict__ x, T* __restrict__ y,
                                                        int64_t rows, int cols) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  row_softmax_reg<T, RV, 32>(x + row * cols, y + row * cols, cols, threadIdx.x & 31, WarpGroup{});
}

// The same for narrow rows with LPR (8 or 16) lanes per row: a warp owns
// 32 / LPR rows, and a row's vectors fill its lanes' RV slots far better than
// a whole warp would (a 291-column bf16 row is about 37 vectors: 40 slots at
// LPR 8 against 64 at LPR 32), which the narrow, issue-bound case needs.
template <typename T, int RV, int LPR>
__global__ void __launch_bounds__(256) softmax_subwarp_reg(const T* __restrict__ x,
                                                           T* __restrict__ y, int64_t rows,
                                                           int cols) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5)) *
                          (32 / LPR) + lane / LPR;
  if (row >= rows) return;
  const unsigned mask = ((1u << LPR) - 1u) << (lane & ~(LPR - 1));
  row_softmax_reg<T, RV, LPR>(x + row * cols, y + row * cols, cols, lane & (LPR - 1),
                              SubWarpGroup<LPR>{mask});
}

template <typename T, int RV, int LPR>
cudaError_t launch_subwarp(const T* x, T* y, int64_t rows, int cols, cudaStream_t st) {
  const int64_t per_block = 8 * (32 / LPR);
  const int64_t blocks = (rows + per_block - 1) / per_block;
  softmax_subwarp_reg<T, RV, LPR><<<static_cast<unsigned>(blocks), 256, 0, st>>>(x, y, rows, cols);
  return cudaGetLastError();
}

// v1 for rows wider than a warp's registers: online pass + write pass
template <typename T, bool kVector>
__global__ void __launch_bounds__(256) softmax_warp_stream(const T* __restrict__ x,
                                                           T* __restrict__ y, int64_t rows,
                                                           int cols) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  row_softmax_stream<T, 32, kVector>(x + row * cols, y + row * cols, cols, threadIdx.x & 31,
                                     WarpGroup{}, false);
}

// v2 (three_pass) / v3 / v4-stream: one block per row, streaming
template <typename T, int NT, bool kVector>
__global__ void __launch_bounds__(NT) softmax_block_stream(const T* __restrict__ x,
                                                           T* __restrict__ y, int cols,
                                                           int three_pass) {
  __shared__ float smax[NT / 32], ssum[NT / 32];
  const int64_t row = blockIdx.x;
  row_softmax_stream<T, NT, kVector>(x + row * cols, y + row * cols, cols, threadIdx.x,
                                     BlockGroup<NT>{smax, ssum}, three_pass != 0);
}

// v4 wide rows: one block per row, register resident
template <typename T, int NT, int RV>
__global__ void __launch_bounds__(NT) softmax_block_reg(const T* __restrict__ x, T* __restrict__ y,
                                                        int cols) {
  __shared__ float smax[NT / 32], ssum[NT / 32];
  const int64_t row = blockIdx.x;
  row_softmax_reg<T, RV, NT>(x + row * cols, y + row * cols, cols, threadIdx.x,
                             BlockGroup<NT>{smax, ssum});
}

// v4 wide rows, 2-byte types: one block per row, row held as raw vectors
template <typename T, int NT, int RV>
__global__ void __launch_bounds__(NT) softmax_block_reg_packed(const T* __restrict__ x,
                                                               T* __restrict__ y, int cols) {
  __shared__ float smax[NT / 32], ssum[NT / 32];
  const int64_t row = blockIdx.x;
  row_softmax_reg_packed<T, RV, NT>(x + row * cols, y + row * cols, cols, threadIdx.x,
                                    BlockGroup<NT>{smax, ssum});
}

// ---- launch logic ------------------------------------------------------------

constexpr int kWarpRowsPerBlock = 8;  // 256-thread blocks of warp-per-row kernels

template <typename T>
cudaError_t launch_warp_reg(const T* x, T* y, int64_t rows, int cols, int rv, cudaStream_t st) {
  const int64_t blocks = (rows + kWarpRowsPerBlock - 1) / kWarpRowsPerBlock;
  const dim3 g(static_cast<unsigned>(blocks)), b(32 * kWarpRowsPerBlock);
  switch (rv) {
    case 1: softmax_warp_reg<T, 1><<<g, b, 0, st>>>(x, y, rows, cols); break;
    case 2: softmax_warp_reg<T, 2><<<g, b, 0, st>>>(x, y, rows, cols); break;
    case 4: softmax_warp_reg<T, 4><<<g, b, 0, st>>>(x, y, rows, cols); break;
    default: softmax_warp_reg<T, 8><<<g, b, 0, st>>>(x, y, rows, cols); break;
  }
  return cudaGetLastError();
}

template <typename T, bool kVector>
cudaError_t launch_block_stream(const T* x, T* y, int64_t rows, int cols, bool three_pass,
                                cudaStream_t st) {
  constexpr int V = kVector ? Elem<T>::kVec : 1;
  const int units = cols / V + 1;
  const dim3 g(static_cast<unsigned>(rows));
  if (units <= 512) {
    softmax_block_stream<T, 128, kVector><<<g, 128, 0, st>>>(x, y, cols, three_pass);
  } else if (units <= 4096) {
    softmax_block_stream<T, 256, kVector><<<g, 256, 0, st>>>(x, y, cols, three_pass);
  } else {
    softmax_block_stream<T, 512, kVector><<<g, 512, 0, st>>>(x, y, cols, three_pass);
  }
  return cudaGetLastError();
}

// Block-per-row register budget: RV 16-byte vectors per thread.
template <typename T>
bool launch_block_reg(const T* x, T* y, int64_t rows, int cols, cudaStream_t st,
                      cudaError_t* err) {
  constexpr int V = Elem<T>::kVec;
  const int nvec = cols / V;  // upper bound on the body of any row
  const dim3 g(static_cast<unsigned>(rows));
#define VLAK_TRY_BLOCK_REG(NT_, RV_)                                      \
  if (nvec <= (NT_) * (RV_)) {                                            \
    softmax_block_reg<T, NT_, RV_><<<g, NT_, 0, st>>>(x, y, cols);        \
    *err = cudaGetLastError();                                            \
    return true;                                                          \
  }
#define VLAK_TRY_BLOCK_REG_PACKED(NT_, RV_)                               \
  if (nvec <= (NT_) * (RV_)) {                                            \
    softmax_block_reg_packed<T, NT_, RV_><<<g, NT_, 0, st>>>(x, y, cols); \
    *err = cudaGetLastError();                                            \
    return true;                                                          \
  }
  if constexpr (sizeof(T) == 2) {
    // Raw-vector rows: few threads per row and two or more rows resident per
    // SM keep the loads of one row in flight while another reduces (bf16,
    // 8192 rows, L2 flushed: 32768 cols 512x8 6.2 TB/s vs 3.6 TB/s for fp32
    // copies at 1024x4; 16384 cols 256x8 6.2 TB/s; 4096 cols 128x4 5.0 TB/s).
    VLAK_TRY_BLOCK_REG_PACKED(128, 2)
    VLAK_TRY_BLOCK_REG_PACKED(128, 4)
    VLAK_TRY_BLOCK_REG_PACKED(256, 4)
    VLAK_TRY_BLOCK_REG_PACKED(256, 8)
    VLAK_TRY_BLOCK_REG_PACKED(512, 8)
    VLAK_TRY_BLOCK_REG_PACKED(1024, 8)
  } else {
    VLAK_TRY_BLOCK_REG(128, 2)
    VLAK_TRY_BLOCK_REG(128, 4)
    VLAK_TRY_BLOCK_REG(256, 4)
    VLAK_TRY_BLOCK_REG(512, 4)
    VLAK_TRY_BLOCK_REG(1024, 4)
    VLAK_TRY_BLOCK_REG(1024, 8)
  }
#undef VLAK_TRY_BLOCK_REG
#undef VLAK_TRY_BLOCK_REG_PACKED
  return false;
}

template <typename T>
cudaError_t dispatch(const T* x, T* y, int64_t rows, int cols, int version, cudaStream_t st) {
  constexpr int V = Elem<T>::kVec;
  const bool vec_ok = (reinterpret_cast<uintptr_t>(x) & 15u) == (reinterpret_cast<uintptr_t>(y) & 15u);
  if (version == 0) {
    const int64_t blocks = (rows + 127) / 128;
    softmax_thread_row<T><<<static_cast<unsigned>(blocks), 128, 0, st>>>(x, y, rows, cols);
    return cudaGetLastError();
  }
  if (!vec_ok) {
    // x and y misaligned relative to each other: scalar online stream
    return launch_block_stream<T, false>(x, y, rows, cols, version == 2, st);
  }
  const int nvec = cols / V;
  // largest body a warp keeps in registers: 8 vectors per lane
  const int warp_rv = nvec <= 32 ? 1 : nvec <= 64 ? 2 : nvec <= 128 ? 4 : nvec <= 256 ? 8 : 0;
  // Narrow rows (versions 1 and 4): a lane group of 8 or 16 per row with as
  // many vector slots as the row needs (the +1 covers a row whose head and
  // tail make one more partial vector).
  if (version == 1 || (version != 2 && version != 3 && nvec <= 128)) {
    const int need = nvec + 1;
    if (need <= 16) return launch_subwarp<T, 2, 8>(x, y, rows, cols, st);
    if (need <= 32) return launch_subwarp<T, 4, 8>(x, y, rows, cols, st);
    if (need <= 40) return launch_subwarp<T, 5, 8>(x, y, rows, cols, st);
    if (need <= 64) return launch_subwarp<T, 8, 8>(x, y, rows, cols, st);
    if (need <= 128) return launch_subwarp<T, 8, 16>(x, y, rows, cols, st);
  }
  if (version == 1) {
    if (warp_rv) return launch_warp_reg<T>(x, y, rows, cols, warp_rv, st);
    const int64_t blocks = (rows + kWarpRowsPerBlock - 1) / kWarpRowsPerBlock;
    softmax_warp_stream<T, true><<<static_cast<unsigned>(blocks), 32 * kWarpRowsPerBlock, 0, st>>>(
        x, y, rows, cols);
    return cudaGetLastError();
  }
  if (version == 2 || version == 3) {
    return launch_block_stream<T, true>(x, y, rows, cols, version == 2, st);
  }
  // version 4 (and any other value, as the reference's else-branch)
  if (nvec <= 128) return launch_warp_reg<T>(x, y, rows, cols, warp_rv ? warp_rv : 4, st);
  cudaError_t err = cudaSuccess;
  if (launch_block_reg<T>(x, y, rows, cols, st, &err)) return err;
  return launch_block_stream<T, true>(x, y, rows, cols, false, st);
}

}  // namespace
}  // namespace vlak

extern "C" int vlak_softmax_auto_version(int64_t rows, int64_t cols) {
  // kernels/softmax/__init__.py:26-37
  if (cols > 2048) return 4;
  if (rows >= 32) return 1;
  return 4;
}

extern "C" int vlak_softmax_fwd(const void* x, void* y, int64_t rows, int64_t cols, int dtype,
                                int version, void* stream) {
  using namespace vlak;
  clear_error();
  if (rows < 0 || cols < 0) return set_error(VLAK_ERR_INVALID_ARGUMENT, "softmax: negative size");
  if (rows == 0 || cols == 0) return VLAK_OK;
  if (cols > INT32_MAX) return set_error(VLAK_ERR_INVALID_ARGUMENT, "softmax: cols exceeds 2^31-1");
  if (rows > INT32_MAX) return set_error(VLAK_ERR_INVALID_ARGUMENT, "softmax: rows exceeds 2^31-1");
  if (x == nullptr || y == nullptr) return set_error(VLAK_ERR_INVALID_ARGUMENT, "softmax: null pointer");
  const size_t esz = dtype == VLAK_F64 ? 8 : dtype == VLAK_F32 ? 4 : 2;
  if ((reinterpret_cast<uintptr_t>(x) % esz) || (reinterpret_cast<uintptr_t>(y) % esz))
    return set_error(VLAK_ERR_ALIGNMENT, "softmax: pointer not aligned to its element size");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int c = static_cast<int>(cols);
  cudaError_t err;
  switch (dtype) {
    case VLAK_F32:
      err = dispatch<float>(static_cast<const float*>(x), static_cast<float*>(y), rows, c, version, st);
      break;
    case VLAK_F16:
      err = dispatch<__half>(static_cast<const __half*>(x), static_cast<__half*>(y), rows, c, version, st);
      break;
    case VLAK_BF16:
      err = dispatch<__nv_bfloat16>(static_cast<const __nv_bfloat16*>(x),
                                    static_cast<__nv_bfloat16*>(y), rows, c, version, st);
      break;
    case VLAK_F64:
      err = dispatch<double>(static_cast<const double*>(x), static_cast<double*>(y), rows, c, version, st);
      break;
    default:
      return set_error(VLAK_ERR_UNSUPPORTED_DTYPE,
                       "softmax: dtype must be float32, float64, float16 or bfloat16");
  }
  if (err != cudaSuccess) return set_cuda_error("softmax kernel launch failed", err);
  return VLAK_OK;
}
