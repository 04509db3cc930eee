// GQA-native fused attention for sm_100a: tcgen05 tensor cores with TMEM
// accumulators, TMA-staged Q/K/V, analytic prefix / dead-band / staircase mask.
//
// Contract (the reference's v3/v4 host functions,
// kernels/attention/fused_attention.cu:603-669 and fused_attention_v4.cu:278-331):
//   q (B, M, H, 64), k/v (B, N, Hkv, 64) at arbitrary strides with head_dim
//   innermost, bf16; o (B, M, H, 64) bf16; query head h reads kv head h / G;
//   visible(r, c) = c < P ? (c < ds || c >= de) : c <= (N - M) + r
//   (reference mask predicate: fused_attention.cu:378-398, :437-445).
// Difference by design: a query row with no visible key is written as exact
// zeros (the reference v3 produces NaN there, v4 leaves the row unwritten).
//
// Work decomposition. One work item = (b, kv head, block of query positions).
// The G query heads of a kv head share K/V, so an item stacks its rows as
// r = m_local * G + g (the order in which q stores them) into up to two
// 128-row M-tiles; K/V are read once per item and reused by all G heads.
// Items are distributed over a persistent grid of one CTA per SM.
//
// Roles inside a CTA (12 warps = 3 warpgroups):
//   warps 0-3   softmax for M-tile 0, one TMEM lane (query row) per thread
//   warps 4-7   softmax for M-tile 1
//   warps 8-9   idle
//   warp 10     TMA producer: Q tiles (double-buffered across items) and
//               64-key K/V chunks through an 8-stage ring.
//   warp 11     TMEM allocator and MMA issuer (one elected lane):
//               S_t = Q_t K_c^T  (SS MMA, M=128, N=chunk width, K=64)
//               O_t (+)= P_t V_c (TS MMA: P from TMEM, V from smem, N=64)
// Keys are processed in 64-key chunks; S and P are double-buffered, so the
// MMA warp computes S two chunks ahead while softmax turns the current chunk
// into P. A softmax thread reads its row of a chunk's S from TMEM once
// (2 x 32 columns).
//
// Tensor memory (512 columns x 128 lanes, fp32 cells), per M-tile t at 256 t:
//   [0,64) [64,128) S buffers   [128,160) [160,192) P buffers   [192,256) O
// P holds bf16 pairs (two keys per 32-bit column), the A-operand layout of
// the TS MMA.
//
// Online softmax in the exp2 domain with a lazily updated row max: the
// reference max only moves (and O / l are rescaled in TMEM) when a new chunk's
// max exceeds it by more than 8 (a factor 256), so P stays <= 256 in bf16 and
// rescales are rare.
//
// Every mbarrier wait is bounded (1 s); on expiry the kernel records
// VLAK_ERR_DEVICE_TIMEOUT in the device error word, drains its own TMA and
// MMA work, frees TMEM and exits.

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include <algorithm>
#include <atomic>
#include <cstring>

#include "vlak_device.cuh"
#include "vlak_internal.h"

namespace vlak {

// Device error word of this library (see vlak_device_error_read).
__device__ int g_device_error = 0;

namespace {

__device__ __forceinline__ void record_device_error(int code) {
  atomicCAS(&g_device_error, 0, code);
}

constexpr uint64_t kWaitLimitNs = 1000ull * 1000ull * 1000ull;  // 1 s per wait

// Bounded parity wait; `abort_flag` (shared) short-circuits the other
// waiters of the CTA once one of them has given up. kMode selects the probe:
// 0 try_wait with a suspend-time hint (a waiting warp yields its issue slots),
// 1 try_wait with the hardware's own time limit, 2 test_wait (pure polling,
// lowest wake-up latency, for waits on the critical hand-off path).
template <int kMode = 0>
__device__ __forceinline__ bool probe(uint64_t* bar, uint32_t parity) {
  if (kMode == 2) return mbar_test_wait(bar, parity);
  if (kMode == 1) return mbar_try_wait(bar, parity);
  return mbar_try_wait_suspend(bar, parity, 20000u);
}
template <int kMode = 0>
__device__ __forceinline__ bool bounded_wait(uint64_t* bar, uint32_t parity,
                                             volatile int* abort_flag,
                                             bool honour_abort = true) {
  // the elapsed time is checked every 64 probes
  if (probe<kMode>(bar, parity)) return true;
  uint64_t t0;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  for (uint32_t it = 1;; ++it) {
    if (probe<kMode>(bar, parity)) return true;
    if ((it & 63u) == 0) {
      if (honour_abort && *abort_flag) return false;
      uint64_t t;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
      if (t - t0 > kWaitLimitNs) {
        record_device_error(VLAK_ERR_DEVICE_TIMEOUT);
        *abort_flag = 1;
        return false;
      }
    }
  }
}

// Waits on the chunk hand-off path use try_wait without a hint (measured
// about 2 % faster on the C5 workload than the hinted form).
constexpr int kWaitMma = 1;      // MMA warp: P ready, K/V ready
constexpr int kWaitSoftmax = 1;  // softmax warps: S ready

constexpr int kThreads = 384;   // 3 warpgroups
// control warps sit on SM sub-partitions 2 and 3: sub-partition 0 also hosts
// the softmax warp of the second M-tile's first lane quarter
constexpr int kWarpProducer = 10, kWarpMma = 11;
// Key pairs whose exp2 runs on the FMA pipe instead of MUFU: bit (k % 8) of
// the mask selects pair k of a 32-key group (full groups only).
#ifndef VLAK_POLY_MASK
#define VLAK_POLY_MASK 0x88u
#endif
constexpr uint32_t kPolyMask = VLAK_POLY_MASK;
constexpr int kChunk = 64;      // keys per K/V chunk (S tile width)
constexpr int kStages = 8;      // K/V ring depth (chunks)
constexpr int kRowBytes = 128;  // 64 bf16 per row
constexpr int kTileBytes = 128 * kRowBytes;        // one 128-row Q tile
constexpr int kChunkBytes = kChunk * kRowBytes;    // one 64-key K (or V) chunk
constexpr int kQBytes = 2 * 2 * kTileBytes;        // 2 buffers x 2 M-tiles
constexpr int kKVBytes = kStages * kChunkBytes;    // K ring (V ring the same)
constexpr int kOBytes = 2 * kTileBytes;            // output staging, one tile per M-tile
constexpr int kSmemData = kQBytes + 2 * kKVBytes + kOBytes;  // 224 KB
constexpr int kBarrierBytes = 512;
constexpr int kSmemBytes = kSmemData + kBarrierBytes + 1024;  // + alignment slack

// Tensor memory, per M-tile t (base 256 t): S double buffer [0,64) [64,128),
// P double buffer [128,160) [160,192) (bf16 pairs), O [192,256).
constexpr uint32_t kTileCols = 256, kColS = 0, kColP = 128, kColO = 192;
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleThreshold = 8.f;  // log2 units

struct __align__(64) Params {
  CUtensorMap tm_q;  // dims (64, H, M, B), box (64, G, MT, 1)
  CUtensorMap tm_k;  // dims (64, Hkv, N, B), box (64, 1, 64, 1)
  CUtensorMap tm_v;
  CUtensorMap tm_o;  // dims (64, H, M, B) of o, box (64, G, MT, 1): tile stores
  __nv_bfloat16* o;
  long long o_sb, o_sm, o_sh;  // element strides of o
  int B, M, N, H, Hkv, G;
  int MT;       // query positions per M-tile
  int tiles;    // M-tiles per item (1 or 2)
  int n_mblk;   // query-position blocks per (b, kv head)
  int num_items;
  int P, ds, de;
  float scale_log2;  // softmax scale * log2(e)
  // mask mode 1: per-sample lengths (B,), int32 or int64, in device memory
  const void* lengths;
  int lengths_i64;
  // mask mode 2: bool (B, M, N) broadcast over heads, keys contiguous
  const uint8_t* mask;
  long long mask_sb, mask_sm;  // byte strides of dims b and m
  int mask_words;              // rows start 4-byte aligned: four keys per load
};

// Mask modes (a template parameter of the kernel, uniform per launch):
//   0 analytic: visible(r, c) = c < P ? (c < ds || c >= de) : c <= (N - M) + r
//   1 per-sample length L_b: visible(r, c) = c < L_b && r < L_b (L_b clamped
//     to [0, N]); rows r >= L_b have no visible key and are written as zeros
//   2 bool mask (B, M, N): visible(r, c) = mask[b, r, c] != 0
constexpr int kMaskAnalytic = 0, kMaskLength = 1, kMaskBool = 2;

struct Barriers {
  uint64_t q_full[2], q_empty[2];
  uint64_t kv_full[kStages], kv_empty[kStages];
  // S and P are double-buffered per tile; each buffer has its own pair of
  // barriers, so no barrier ever runs two phases ahead of its waiter
  uint64_t s_full[2][2];  // [tile][buffer]
  uint64_t p_full[2];     // [buffer]: every softmax warp of the item's tiles arrives
  uint64_t pv_done[2], o_full[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
};

static_assert(sizeof(Barriers) <= kBarrierBytes, "barrier block overflows its region");

struct Item {
  int b, kvh, m0;  // m0: first query position of the item
  int tiles_active;
  int L;           // mask mode 1: length of sample b
};

template <int kMode>
__device__ __forceinline__ Item decode_item(const Params& p, int item) {
  Item it;
  const int mblk = item % p.n_mblk;
  const int bk = item / p.n_mblk;
  it.kvh = bk % p.Hkv;
  it.b = bk / p.Hkv;
  it.m0 = mblk * p.tiles * p.MT;
  it.tiles_active = (p.tiles == 2 && it.m0 + p.MT < p.M) ? 2 : 1;
  it.L = 0;
  if (kMode == kMaskLength) {
    const long long len = p.lengths_i64 ? static_cast<const long long*>(p.lengths)[it.b]
                                        : static_cast<const int*>(p.lengths)[it.b];
    it.L = static_cast<int>(min(max(len, 0LL), static_cast<long long>(p.N)));
  }
  return it;
}

// Whether key chunk c has a visible key for some row of the item (every role
// evaluates this identically, so all agree on the item's live chunks). A bool
// mask is not inspected here: every chunk of its items is processed.
template <int kMode>
__device__ __forceinline__ bool chunk_live(const Params& p, const Item& it, int c) {
  const int c0 = c * kChunk;
  if (kMode == kMaskBool) return true;
  if (kMode == kMaskLength) return c0 < it.L && it.m0 < it.L;
  const int width = min(kChunk, p.N - c0);
  const int m_hi = min(p.M, it.m0 + it.tiles_active * p.MT) - 1;
  const int e2_hi = max(p.P, min(p.N, p.N - p.M + m_hi + 1));
  return (c0 < p.ds) || (c0 + width > p.de && c0 < e2_hi);
}
template <int kMode>
__device__ __forceinline__ int next_live(const Params& p, const Item& it, int c, int n_chunks) {
  for (; c < n_chunks; ++c)
    if (chunk_live<kMode>(p, it, c)) return c;
  return -1;
}

// Bits of keys g0 .. g0+31 of one bool-mask row (bit i set when key g0 + i is
// below N and its mask byte is nonzero).
__device__ __forceinline__ uint32_t mask_bits32(const Params& p, const uint8_t* row, int g0) {
  uint32_t vm = 0u;
  if (p.mask_words && g0 + 32 <= p.N) {
    const uint32_t* w = reinterpret_cast<const uint32_t*>(row + g0);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      // one byte per key -> bytes 0x01 / 0x00 -> four bits gathered by a
      // multiply (the partial products of distinct bytes never overlap)
      const uint32_t b = __vcmpne4(__ldg(w + i), 0u) & 0x01010101u;
      vm |= ((b * 0x01020408u) >> 24) << (4 * i);
    }
  } else {
    const int n = min(32, p.N - g0);
    for (int i = 0; i < n; ++i) vm |= (__ldg(row + g0 + i) != 0 ? 1u : 0u) << i;
  }
  return vm;
}
__device__ __forceinline__ int chunk_cols(const Params& p, int c) {
  const int width = min(kChunk, p.N - c * kChunk);
  return (width + 15) & ~15;  // MMA N must be a multiple of 16
}

template <int kMode>
__global__ void __launch_bounds__(kThreads, 1)
gqa_attention_sm100(const __grid_constant__ Params p) {
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment for the 128-byte-swizzled operand tiles
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint8_t* q_smem = smem;                      // [2 buf][2 tile][128 x 128 B]
  uint8_t* k_smem = smem + kQBytes;            // [stage][64 x 128 B]
  uint8_t* v_smem = k_smem + kKVBytes;
  uint8_t* o_smem = v_smem + kKVBytes;         // [tile][128 x 128 B], 128B-swizzled
  Barriers* bars = reinterpret_cast<Barriers*>(smem + kSmemData);
  volatile int* abort_flag = &bars->abort_flag;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->q_full[i], 1);
      mbar_init(&bars->q_empty[i], 1);
      for (int b = 0; b < 2; ++b) mbar_init(&bars->s_full[i][b], 1);
      mbar_init(&bars->p_full[i], 8);  // one arrival per softmax warp of both tiles
      mbar_init(&bars->pv_done[i], 1);
      mbar_init(&bars->o_full[i], 1);
    }
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&bars->kv_full[i], 1);
      mbar_init(&bars->kv_empty[i], 1);
    }
    mbar_init(&bars->drain, 1);
    bars->abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kWarpMma) {
    tmem_alloc(&bars->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  // Q rows that no TMA box covers feed only discarded rows; clear them once so
  // they hold finite values.
  for (int i = threadIdx.x; i < kQBytes / 16; i += kThreads)
    reinterpret_cast<uint4*>(q_smem)[i] = make_uint4(0, 0, 0, 0);
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  const int n_chunks = (p.N + kChunk - 1) / kChunk;

  if (warp == kWarpProducer) {
    // ------------------------------------------------------------ producer
    // The whole warp runs this loop (converged); one elected lane issues.
    if (lane == 0) {
      prefetch_tmap(&p.tm_q);
      prefetch_tmap(&p.tm_k);
      prefetch_tmap(&p.tm_v);
      prefetch_tmap(&p.tm_o);
    }
    __syncwarp();
    uint32_t qi = 0, kv = 0;
    // per full barrier: bit i of *_used = armed at least once, bit i of
    // *_par = parity of its most recently armed phase (registers, no arrays)
    uint32_t q_used = 0, q_par = 0, kv_used = 0, kv_par = 0;
    bool ok = true;
    for (int item = blockIdx.x; ok && item < p.num_items; item += gridDim.x, ++qi) {
      const Item it = decode_item<kMode>(p, item);
      const int qs = qi & 1;
      if (!__all_sync(kFullMask, bounded_wait(&bars->q_empty[qs], ((qi >> 1) & 1) ^ 1, abort_flag))) {
        ok = false;
        break;
      }
      const uint32_t qbytes = static_cast<uint32_t>(it.tiles_active * p.G * p.MT * kRowBytes);
      mbar_arrive_expect_tx_elect(&bars->q_full[qs], qbytes);
      q_par = (q_used & (1u << qs)) ? (q_par ^ (1u << qs)) : q_par;
      q_used |= 1u << qs;
      for (int t = 0; t < it.tiles_active; ++t)
        tma_load_4d_elect(q_smem + (qs * 2 + t) * kTileBytes, &p.tm_q, &bars->q_full[qs], 0,
                          it.kvh * p.G, it.m0 + t * p.MT, it.b);
      for (int c = next_live<kMode>(p, it, 0, n_chunks); c >= 0; c = next_live<kMode>(p, it, c + 1, n_chunks)) {
        const int s = kv % kStages;
        if (!__all_sync(kFullMask, bounded_wait(&bars->kv_empty[s], ((kv / kStages) & 1) ^ 1, abort_flag))) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx_elect(&bars->kv_full[s], 2 * kChunkBytes);
        kv_par = (kv_used & (1u << s)) ? (kv_par ^ (1u << s)) : kv_par;
        kv_used |= 1u << s;
        tma_load_4d_elect(k_smem + s * kChunkBytes, &p.tm_k, &bars->kv_full[s], 0, it.kvh, c * kChunk, it.b);
        tma_load_4d_elect(v_smem + s * kChunkBytes, &p.tm_v, &bars->kv_full[s], 0, it.kvh, c * kChunk, it.b);
        ++kv;
      }
    }
    // never leave the CTA with copies in flight: wait for the last phase
    // armed on every full barrier (bounded, independent of the abort flag)
    for (int i = 0; i < 2; ++i)
      if (q_used & (1u << i)) bounded_wait(&bars->q_full[i], (q_par >> i) & 1u, abort_flag, false);
    for (int s = 0; s < kStages; ++s)
      if (kv_used & (1u << s)) bounded_wait(&bars->kv_full[s], (kv_par >> s) & 1u, abort_flag, false);
    __syncwarp();
  } else if (warp == kWarpMma) {
    // ------------------------------------------------------------ MMA issuer
    // Per item, chunk j of tile t:  S_t(j) -> buffer j%2 (issued two chunks
    // ahead), then, once softmax has turned it into P_t(j) (buffer j%2),
    // O_t (+)= P_t(j) V(j). Issue order per chunk: PV_t(j) then S_t(j+2), so
    // the commit of S_t(j+2) also covers PV_t(j) (same thread, in order).
    // The whole warp runs the loop (converged); one elected lane issues.
    {
      uint32_t qi = 0, kv = 0, pph = 0;  // bit b: parity expected on p_full[b]
      bool ok = true;
      for (int item = blockIdx.x; ok && item < p.num_items; item += gridDim.x, ++qi) {
        const Item it = decode_item<kMode>(p, item);
        const int qs = qi & 1;
        if (!__all_sync(kFullMask, bounded_wait(&bars->q_full[qs], (qi >> 1) & 1, abort_flag))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t q_base = smem_u32(q_smem + qs * 2 * kTileBytes);
        // Each burst below is straight-line code: both tiles and all K-steps
        // unrolled, absent ones predicated off inside the issuing asm.
        const uint32_t two = it.tiles_active == 2 ? 1u : 0u;
        auto issue_s = [&](int c, int j, uint32_t en) {  // S_t(j) for every active tile
          const int s = (kv + j) % kStages;
          const uint32_t idesc = idesc_bf16_f32(128, chunk_cols(p, c), false);
          const uint32_t b0 = smem_u32(k_smem + s * kChunkBytes);
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            const uint32_t on = (t == 0 ? 1u : two) & en;
            const uint32_t a0 = q_base + t * kTileBytes;
            const uint32_t d = tmem + t * kTileCols + kColS + (j & 1) * kChunk;
#pragma unroll
            for (int k = 0; k < 4; ++k)  // head_dim 64 = 4 x K16, 32 B apart in a swizzled row
              umma_ss_elect(d, sdesc_sw128(a0 + 32 * k), sdesc_sw128(b0 + 32 * k), idesc, k > 0, on);
            umma_commit_elect(&bars->s_full[t][j & 1], on);
          }
        };
        auto issue_pv = [&](int c, int j) {  // O_t (+)= P_t(j) V(j) for every active tile
          const int s = (kv + j) % kStages;
          const int nk = chunk_cols(p, c) / 16;  // 16 keys = 8 packed columns of P, 2 KB of V
          const uint32_t idesc = idesc_bf16_f32(128, 64, true);
          const uint32_t b0 = smem_u32(v_smem + s * kChunkBytes);
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            const uint32_t on = t == 0 ? 1u : two;
            const uint32_t a = tmem + t * kTileCols + kColP + (j & 1) * (kChunk / 2);
            const uint32_t d = tmem + t * kTileCols + kColO;
#pragma unroll
            for (int k = 0; k < 4; ++k)
              umma_ts_elect(d, a + 8 * k, sdesc_sw128(b0 + 2048 * k), idesc, (j > 0 || k > 0) ? 1u : 0u,
                            (k < nk) ? on : 0u);
            umma_commit_elect(&bars->pv_done[t], on);
          }
        };
        auto wait_kv = [&](int j) {
          const uint32_t n = kv + j;
          if (!__all_sync(kFullMask, bounded_wait<kWaitMma>(&bars->kv_full[n % kStages], (n / kStages) & 1, abort_flag)))
            return false;
          tc_fence_after();
          return true;
        };
        auto wait_p = [&](int j) {
          const uint32_t bit = 1u << (j & 1);
          if (!__all_sync(kFullMask, bounded_wait<kWaitMma>(&bars->p_full[j & 1], (pph & bit) ? 1u : 0u, abort_flag)))
            return false;
          pph ^= bit;
          tc_fence_after();
          return true;
        };
        int cur = next_live<kMode>(p, it, 0, n_chunks);
        int nxt = cur >= 0 ? next_live<kMode>(p, it, cur + 1, n_chunks) : -1;
        int j = 0;
        if (cur >= 0) {
          if (!wait_kv(0)) { ok = false; break; }
          issue_s(cur, 0, 1u);
        }
        if (nxt >= 0) {
          if (!wait_kv(1)) { ok = false; break; }
          issue_s(nxt, 1, 1u);
        }
        while (cur >= 0) {
          const int nn = nxt >= 0 ? next_live<kMode>(p, it, nxt + 1, n_chunks) : -1;  // chunk j+2
          // both waits first (both tiles' P, the K/V two chunks ahead), then
          // one branch-free burst: PV of every tile, then the S two chunks ahead
          if (!wait_p(j)) { ok = false; break; }
          if (nn >= 0 && !wait_kv(j + 2)) { ok = false; break; }
          const int cs = nn >= 0 ? nn : cur;  // any valid chunk when S is off
          issue_pv(cur, j);
          issue_s(cs, j + 2, nn >= 0 ? 1u : 0u);
          umma_commit_elect(&bars->kv_empty[(kv + j) % kStages]);
          cur = nxt;
          nxt = nn;
          ++j;
        }
        if (!ok) break;
        umma_commit_elect(&bars->o_full[0]);
        umma_commit_elect(&bars->o_full[1], two);
        umma_commit_elect(&bars->q_empty[qs]);
        kv += j;
      }
      // every issued MMA must complete before TMEM is released
      umma_commit_elect(&bars->drain);
      bounded_wait(&bars->drain, 0, abort_flag, false);
    }
    __syncwarp();  // reconverge before the CTA-wide barrier and the dealloc
  } else if (warp < 8) {
    // ------------------------------------------------------------ softmax
    const int t = warp >> 2;                // M-tile of this group
    const int quarter = warp & 3;           // TMEM lane quarter this warp may access
    const int row = quarter * 32 + lane;    // TMEM lane = row within the tile
    const uint32_t tbase = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + t * kTileCols;
    const uint32_t tO = tbase + kColO;
    const int m_local = row / p.G;
    uint32_t sph = 0, oph = 0, pv_seen = 0;  // sph bit b: parity on s_full[t][b]; pv_seen: P.V products so far
    bool ok = true;

    for (int item = blockIdx.x; ok && item < p.num_items; item += gridDim.x) {
      const Item it = decode_item<kMode>(p, item);
      if (t >= it.tiles_active) continue;
      const int m_first = it.m0 + t * p.MT;        // first query position of this tile
      const int m = m_first + m_local;
      const bool valid = (m_local < p.MT) && (m < p.M);
      // a warp whose rows are all invalid skips the arithmetic
      const int warp_first_m = m_first + (quarter * 32) / p.G;
      const bool warp_active = ((quarter * 32) / p.G < p.MT) && (warp_first_m < p.M);
      // this row's visible set [0, ds) U [de, e2) (mask modes 0 and 1) or its
      // bool-mask row (mode 2)
      const int rds = kMode == kMaskAnalytic ? p.ds : 0;
      const int rde = kMode == kMaskAnalytic ? p.de : 0;
      const int e2 = kMode == kMaskAnalytic ? max(p.P, min(p.N, p.N - p.M + m + 1))
                     : kMode == kMaskLength ? (m < it.L ? it.L : 0) : 0;
      const uint8_t* mrow = nullptr;
      if (kMode == kMaskBool && valid)
        mrow = p.mask + static_cast<long long>(it.b) * p.mask_sb + static_cast<long long>(m) * p.mask_sm;
      float m_run = -INFINITY, l_run = 0.f;
      int j = 0;
      for (int c = next_live<kMode>(p, it, 0, n_chunks); c >= 0; c = next_live<kMode>(p, it, c + 1, n_chunks), ++j) {
        // warp-uniform outcome: the TMEM accesses below are warp-collective
        if (!__all_sync(kFullMask, bounded_wait<kWaitSoftmax>(&bars->s_full[t][j & 1], (sph >> (j & 1)) & 1u, abort_flag))) {
          ok = false;
          break;
        }
        sph ^= 1u << (j & 1);
        tc_fence_after();
        if (warp_active) {
          const int c0 = c * kChunk;
          const int ncols = chunk_cols(p, c);
          const uint32_t tS = tbase + kColS + (j & 1) * kChunk;
          const uint32_t tP = tbase + kColP + (j & 1) * (kChunk / 2);
          // S of this chunk in one batch and one wait; columns past the chunk
          // width fail the visibility test (they lie at or past N >= e2). The
          // mask is applied where a value is used; S is never rewritten.
          float sv[kChunk / 32][32];
#pragma unroll
          for (int gq = 0; gq < kChunk / 32; ++gq) tmem_ld32(tS + 32 * gq, sv[gq]);
          // Warp-uniform class of each 32-key group: every valid row of the
          // warp sees all 32 keys (no mask arithmetic) or none of them (no
          // exp); otherwise each row's visible keys as a bit mask. Rows past
          // the tile or past M do not vote (their outputs are discarded), so
          // the analytic and the bool-mask form of one mask classify alike.
          uint32_t vmask[kChunk / 32];
          uint32_t full_bits = 0, none_bits = 0;
#pragma unroll
          for (int gq = 0; gq < kChunk / 32; ++gq) {
            const int g0 = c0 + 32 * gq;
            const bool in_chunk = 32 * gq < ncols;
            auto low = [](int n) -> uint32_t {
              return n <= 0 ? 0u : n >= 32 ? 0xffffffffu : ((1u << n) - 1u);
            };
            bool full, none;
            uint32_t vm = 0u;
            if (kMode == kMaskBool) {
              if (in_chunk && mrow != nullptr) vm = mask_bits32(p, mrow, g0);
              full = !valid || (in_chunk && vm == 0xffffffffu);
              none = !valid || vm == 0u;
            } else {
              full = !valid || (in_chunk && ((g0 + 32 <= rds) || (g0 >= rde && g0 + 32 <= e2)));
              none = !valid || !in_chunk || ((g0 >= rds) && (g0 + 32 <= rde || g0 >= e2));
            }
            full_bits |= (__all_sync(kFullMask, full) ? 1u : 0u) << gq;
            none_bits |= (__all_sync(kFullMask, none) ? 1u : 0u) << gq;
            if (kMode != kMaskBool && !(((full_bits | none_bits) >> gq) & 1u))
              vm = valid ? (low(rds - g0) | (low(e2 - g0) & ~low(rde - g0))) : 0u;
            vmask[gq] = vm;
          }
          tmem_wait_ld();
          // row max with four independent accumulators (short dependency chains)
          float mxa[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
          for (int gq = 0; gq < kChunk / 32; ++gq) {
            if ((none_bits >> gq) & 1u) continue;
            if ((full_bits >> gq) & 1u) {
#pragma unroll
              for (int i = 0; i < 32; i += 2)
                mxa[(i >> 1) & 3] = fmax3(mxa[(i >> 1) & 3], sv[gq][i], sv[gq][i + 1]);
            } else {
              const uint32_t vm = vmask[gq];
#pragma unroll
              for (int i = 0; i < 32; i += 2)
                mxa[(i >> 1) & 3] = fmax3(mxa[(i >> 1) & 3],
                                          ((vm >> i) & 1u) ? sv[gq][i] : -INFINITY,
                                          ((vm >> (i + 1)) & 1u) ? sv[gq][i + 1] : -INFINITY);
            }
          }
          const float mx = fmax3(fmaxf(mxa[0], mxa[1]), mxa[2], mxa[3]);
          const float mz = mx * p.scale_log2;  // -inf stays -inf (scale > 0)
          // The reference max moves only when this chunk's max exceeds it by
          // more than the threshold; O and l are then rescaled by alpha (after
          // P is written, so S is no longer live).
          bool need = false;
          float alpha = 1.f;
          if (j == 0) {
            m_run = mz;
          } else {
            need = mz > m_run + kRescaleThreshold;
            if (need) {
              alpha = ex2(m_run - mz);
              m_run = mz;
            }
          }
          // P = exp2(s * scale_log2 - mref) as bf16 pairs into TMEM. Key pairs
          // go through the f32x2 FMA pipe; exps run on MUFU except for the pairs
          // kPolyMask selects, which use the FMA-pipe polynomial (full groups
          // only, where no -inf occurs).
          const float nref = (m_run == -INFINITY) ? 0.f : -m_run;
          const uint64_t sl2 = f2_pack(p.scale_log2, p.scale_log2);
          const uint64_t nr2 = f2_pack(nref, nref);
          uint64_t acc[4] = {0ull, 0ull, 0ull, 0ull};  // four (+0.f, +0.f) pairs
#pragma unroll
          for (int gq = 0; gq < kChunk / 32; ++gq) {
            if (32 * gq >= ncols) continue;
            uint32_t pk[16];
            if ((none_bits >> gq) & 1u) {
#pragma unroll
              for (int i = 0; i < 16; ++i) pk[i] = 0u;
            } else if ((full_bits >> gq) & 1u) {
#pragma unroll
              for (int k = 0; k < 16; ++k) {
                const uint64_t x = f2_fma(f2_pack(sv[gq][2 * k], sv[gq][2 * k + 1]), sl2, nr2);
                uint64_t e;
                float x0, x1;
                f2_unpack(x, x0, x1);
                if ((kPolyMask >> (k & 7)) & 1u) {
                  e = f2_exp2_poly(f2_pack(fmaxf(x0, -126.f), fmaxf(x1, -126.f)));
                } else {
                  e = f2_pack(ex2(x0), ex2(x1));
                }
                acc[k & 3] = f2_add(acc[k & 3], e);
                float e0, e1;
                f2_unpack(e, e0, e1);
                pk[k] = pack_bf16x2(e0, e1);
              }
            } else {
              const uint32_t vm = vmask[gq];
#pragma unroll
              for (int k = 0; k < 16; ++k) {
                const uint64_t x = f2_fma(f2_pack(sv[gq][2 * k], sv[gq][2 * k + 1]), sl2, nr2);
                float x0, x1;
                f2_unpack(x, x0, x1);
                const float e0 = ((vm >> (2 * k)) & 1u) ? ex2(x0) : 0.f;
                const float e1 = ((vm >> (2 * k + 1)) & 1u) ? ex2(x1) : 0.f;
                acc[k & 3] = f2_add(acc[k & 3], f2_pack(e0, e1));
                pk[k] = pack_bf16x2(e0, e1);
              }
            }
            tmem_st16(tP + 16 * gq, pk);
          }
          float acc0, acc1;
          f2_unpack(f2_add(f2_add(acc[0], acc[1]), f2_add(acc[2], acc[3])), acc0, acc1);
          const float lsum = acc0 + acc1;
          l_run = l_run * alpha + lsum;
          tmem_wait_st();
          if (__any_sync(kFullMask, need)) {
            // O_t must hold the previous P.V of this tile before it is scaled
            if (!__all_sync(kFullMask, bounded_wait(&bars->pv_done[t], (pv_seen - 1) & 1, abort_flag))) {
              ok = false;
              break;
            }
            tc_fence_after();
#pragma unroll
            for (int half = 0; half < 2; ++half) {
              float o[32];
              tmem_ld32(tO + 32 * half, o);
              tmem_wait_ld();
#pragma unroll
              for (int i = 0; i < 32; ++i) o[i] *= alpha;
              tmem_st32f(tO + 32 * half, o);
            }
            tmem_wait_st();
          }
        }
        ++pv_seen;
        tc_fence_before();
        // eight arrivals complete a phase; with one active tile its warps
        // arrive for the absent ones too
        mbar_arrive_elect(&bars->p_full[j & 1], it.tiles_active == 2 ? 1u : 2u);
      }
      if (!ok) break;
      // epilogue: O / l -> bf16 rows, staged in shared memory (128B-swizzled,
      // the layout of the output tensor map) and written by one TMA store
      if (!__all_sync(kFullMask, bounded_wait(&bars->o_full[t], oph, abort_flag))) { ok = false; break; }
      oph ^= 1;
      tc_fence_after();
      uint8_t* stage = o_smem + t * kTileBytes;
      const bool leader = (quarter == 0 && lane == 0);
      // the previous store from this staging tile must have read it
      if (leader) bulk_wait_read0();
      named_barrier(1 + t, 128);
      if (warp_active) {
        const bool any = (j > 0) && (l_run > 0.f);
        const float inv = any ? 1.f / l_run : 0.f;
        uint8_t* srow = stage + row * kRowBytes;
#pragma unroll
        for (int half = 0; half < 2; ++half) {  // 32 columns of O at a time
          float o[32];
          if (j > 0) {
            tmem_ld32(tO + 32 * half, o);
            tmem_wait_ld();
          }
          if (valid) {
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              uint32_t w[4];
#pragma unroll
              for (int e = 0; e < 4; ++e)
                w[e] = any ? pack_bf16x2(o[v * 8 + 2 * e] * inv, o[v * 8 + 2 * e + 1] * inv) : 0u;
              const int cv = half * 4 + v;  // 16-byte chunk of the 128-byte row
              *reinterpret_cast<uint4*>(srow + ((cv ^ (row & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
            }
          }
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      named_barrier(1 + t, 128);
      if (leader) {
        tma_store_4d(&p.tm_o, stage, 0, it.kvh * p.G, m_first, it.b);
        bulk_commit_group();
      }
    }
    // stores must finish reading shared memory before the CTA exits
    if (quarter == 0 && lane == 0) bulk_wait_all0();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kWarpMma) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// Zero-fill of o for N == 0 (every row fully masked).
__global__ void zero_rows(__nv_bfloat16* o, long long o_sb, long long o_sm, long long o_sh, int B,
                          int M, int H) {
  const long long rows = static_cast<long long>(B) * M * H;
  for (long long r = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; r < rows;
       r += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long h = r % H, bm = r / H, m = bm % M, b = bm / M;
    uint4* row = reinterpret_cast<uint4*>(o + b * o_sb + m * o_sm + h * o_sh);
#pragma unroll
    for (int v = 0; v < 8; ++v) row[v] = make_uint4(0, 0, 0, 0);
  }
}

int encode_map(CUtensorMap* map, const void* base, int64_t d1, int64_t d2, int64_t d3,
               int64_t s1, int64_t s2, int64_t s3, uint32_t box1, uint32_t box2,
               const char* name) {
  EncodeTiledFn enc = encode_tiled_fn();
  if (!enc) return set_error(VLAK_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  // a size-1 dimension is never stepped over; give it a harmless stride
  auto fix = [](int64_t size, int64_t stride_bytes, int64_t fallback) {
    return size == 1 ? fallback : stride_bytes;
  };
  const int64_t b1 = fix(d1, s1 * 2, 128);
  const int64_t b2 = fix(d2, s2 * 2, b1 * d1);
  const int64_t b3 = fix(d3, s3 * 2, b2 * d2);
  cuuint64_t dims[4] = {64, static_cast<cuuint64_t>(d1), static_cast<cuuint64_t>(d2),
                        static_cast<cuuint64_t>(d3)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(b1), static_cast<cuuint64_t>(b2),
                           static_cast<cuuint64_t>(b3)};
  cuuint32_t box[4] = {64, box1, box2, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_errorf(VLAK_ERR_INVALID_ARGUMENT,
                      "fused_attention_gqa: cannot describe %s to TMA (CUresult %d); strides "
                      "must be multiples of 8 elements and the layout addressable",
                      name, static_cast<int>(r));
  return VLAK_OK;
}

}  // namespace

// Validation shared by the launch and vlak_attn_gqa_check. Mirrors the
// TORCH_CHECKs of fused_attention.cu:608-633 (shape, GQA ratio, alignment,
// prefix / dead-band order) with the same acceptance set.
static int validate(const vlak_attn_gqa_args* a, int64_t* P_out, float* scale_out) {
  if (!a) return set_error(VLAK_ERR_INVALID_ARGUMENT, "fused_attention_gqa: null arguments");
  if (a->B < 0 || a->M < 0 || a->N < 0 || a->H <= 0 || a->Hkv <= 0)
    return set_error(VLAK_ERR_INVALID_ARGUMENT, "fused_attention_gqa: sizes must be non-negative and heads positive");
  if (a->H % a->Hkv != 0)
    return set_error(VLAK_ERR_INVALID_ARGUMENT, "query heads must be a multiple of kv heads");
  if (a->H / a->Hkv > 128)
    return set_error(VLAK_ERR_INVALID_ARGUMENT, "fused_attention_gqa: at most 128 query heads per kv head");
  if (a->B > INT32_MAX || a->M > INT32_MAX || a->N > INT32_MAX || a->H > INT32_MAX)
    return set_error(VLAK_ERR_INVALID_ARGUMENT, "fused_attention_gqa: size exceeds 2^31-1");
  const int64_t P = a->prefix_len >= 0 ? a->prefix_len : a->N;
  if (P > a->N) return set_error(VLAK_ERR_INVALID_ARGUMENT, "prefix_len exceeds kv length");
  if (!(0 <= a->dead_start && a->dead_start <= a->dead_end && a->dead_end <= P))
    return set_error(VLAK_ERR_INVALID_ARGUMENT, "dead band must satisfy 0 <= ds <= de <= prefix_len");
  const void* ptrs[4] = {a->q, a->k, a->v, a->o};
  const int64_t* strides[4] = {a->q_stride, a->k_stride, a->v_stride, a->o_stride};
  for (int i = 0; i < 4; ++i) {
    if (reinterpret_cast<uintptr_t>(ptrs[i]) % 16 != 0)
      return set_error(VLAK_ERR_ALIGNMENT, "strides/base must keep 16B alignment for cp.async");
    for (int d = 0; d < 3; ++d)
      if (strides[i][d] % 8 != 0)
        return set_error(VLAK_ERR_ALIGNMENT, "strides/base must keep 16B alignment for cp.async");
  }
  if (P_out) *P_out = P;
  if (scale_out) *scale_out = a->scale > 0 ? static_cast<float>(a->scale) : 0.125f;
  return VLAK_OK;
}

// Mask beyond the analytic form: per-sample lengths (mode 1) or a bool mask
// (mode 2). The analytic fields of the arguments are ignored for those modes.
struct MaskSpec {
  int mode = kMaskAnalytic;
  const void* lengths = nullptr;
  int lengths_dtype = VLAK_I32;
  const void* mask = nullptr;
  int64_t mask_sb = 0, mask_sm = 0;
};

template <int kMode>
static cudaError_t launch_mode(const Params& prm, int grid, cudaStream_t cs, int device) {
  // one-time per (device, mode) opt-in to the large dynamic shared-memory carve-out
  static std::atomic<int> ready[64];
  if (ready[device].load() == 0) {
    cudaError_t e = cudaFuncSetAttribute(gqa_attention_sm100<kMode>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return e;
    ready[device].store(1);
  }
  gqa_attention_sm100<kMode><<<grid, kThreads, kSmemBytes, cs>>>(prm);
  return cudaGetLastError();
}

static int launch_gqa(const vlak_attn_gqa_args* a_in, void* stream, const MaskSpec& ms = MaskSpec()) {
  using namespace vlak;
  clear_error();
  if (!a_in) return set_error(VLAK_ERR_INVALID_ARGUMENT, "fused_attention_gqa: null arguments");
  vlak_attn_gqa_args args = *a_in;
  const vlak_attn_gqa_args* a = &args;
  if (ms.mode != kMaskAnalytic) {
    args.prefix_len = -1;
    args.dead_start = args.dead_end = 0;
  }
  int64_t P = 0;
  float scale = 0.f;
  int st = validate(a, &P, &scale);
  if (st != VLAK_OK) return st;
  if (ms.mode == kMaskLength) {
    if (!ms.lengths && a->B > 0) return set_error(VLAK_ERR_INVALID_ARGUMENT, "lengths must not be null");
    if (ms.lengths_dtype != VLAK_I32 && ms.lengths_dtype != VLAK_I64)
      return set_error(VLAK_ERR_UNSUPPORTED_DTYPE, "lengths must be int32 or int64");
    if (reinterpret_cast<uintptr_t>(ms.lengths) % (ms.lengths_dtype == VLAK_I64 ? 8 : 4))
      return set_error(VLAK_ERR_ALIGNMENT, "lengths must be aligned to its element size");
  } else if (ms.mode == kMaskBool) {
    if (!ms.mask && a->B > 0 && a->M > 0 && a->N > 0)
      return set_error(VLAK_ERR_INVALID_ARGUMENT, "attn_mask must not be null");
    if (ms.mask_sb < 0 || ms.mask_sm < 0)
      return set_error(VLAK_ERR_INVALID_ARGUMENT, "attn_mask strides must be non-negative");
  }
  if (a->B == 0 || a->M == 0) return VLAK_OK;
  // with no keys only o is touched; empty k / v may carry null pointers
  if (!a->o || (a->N > 0 && (!a->q || !a->k || !a->v)))
    return set_error(VLAK_ERR_INVALID_ARGUMENT, "fused_attention_gqa: null tensor pointer");
  cudaStream_t cs = static_cast<cudaStream_t>(stream);
  DeviceInfo dev;
  st = current_device_info(&dev);
  if (st != VLAK_OK) return st;
  if (dev.cc_major != 10)
    return set_errorf(VLAK_ERR_UNSUPPORTED_DEVICE,
                      "fused_attention_gqa: needs an sm_100 device (found sm_%d%d)", dev.cc_major,
                      dev.cc_minor);
  auto* o = static_cast<__nv_bfloat16*>(a->o);
  if (a->N == 0) {
    const long long rows = a->B * a->M * a->H;
    const int blocks = static_cast<int>(std::min<long long>((rows + 255) / 256, 4096));
    zero_rows<<<blocks, 256, 0, cs>>>(o, a->o_stride[0], a->o_stride[1], a->o_stride[2],
                                      static_cast<int>(a->B), static_cast<int>(a->M),
                                      static_cast<int>(a->H));
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? VLAK_OK : set_cuda_error("fused_attention_gqa zero fill", e);
  }

  Params prm;
  memset(&prm, 0, sizeof(prm));
  const int G = static_cast<int>(a->H / a->Hkv);
  const int M = static_cast<int>(a->M);
  prm.B = static_cast<int>(a->B);
  prm.M = M;
  prm.N = static_cast<int>(a->N);
  prm.H = static_cast<int>(a->H);
  prm.Hkv = static_cast<int>(a->Hkv);
  prm.G = G;
  prm.MT = std::min(128 / G, M);
  prm.tiles = M > prm.MT ? 2 : 1;
  prm.n_mblk = (M + prm.tiles * prm.MT - 1) / (prm.tiles * prm.MT);
  const long long items = static_cast<long long>(prm.B) * prm.Hkv * prm.n_mblk;
  if (items > INT32_MAX) return set_error(VLAK_ERR_INVALID_ARGUMENT, "fused_attention_gqa: too many work items");
  prm.num_items = static_cast<int>(items);
  prm.P = static_cast<int>(P);
  prm.ds = static_cast<int>(a->dead_start);
  prm.de = static_cast<int>(a->dead_end);
  prm.scale_log2 = scale * 1.4426950408889634f;
  prm.o = o;
  prm.o_sb = a->o_stride[0];
  prm.o_sm = a->o_stride[1];
  prm.o_sh = a->o_stride[2];
  prm.lengths = ms.lengths;
  prm.lengths_i64 = ms.lengths_dtype == VLAK_I64 ? 1 : 0;
  prm.mask = static_cast<const uint8_t*>(ms.mask);
  prm.mask_sb = ms.mask_sb;
  prm.mask_sm = ms.mask_sm;
  prm.mask_words = (reinterpret_cast<uintptr_t>(ms.mask) % 4 == 0 && ms.mask_sb % 4 == 0 &&
                    ms.mask_sm % 4 == 0) ? 1 : 0;

  st = encode_map(&prm.tm_q, a->q, a->H, a->M, a->B, a->q_stride[2], a->q_stride[1],
                  a->q_stride[0], static_cast<uint32_t>(G), static_cast<uint32_t>(prm.MT), "q");
  if (st != VLAK_OK) return st;
  st = encode_map(&prm.tm_k, a->k, a->Hkv, a->N, a->B, a->k_stride[2], a->k_stride[1],
                  a->k_stride[0], 1, kChunk, "k");
  if (st != VLAK_OK) return st;
  st = encode_map(&prm.tm_v, a->v, a->Hkv, a->N, a->B, a->v_stride[2], a->v_stride[1],
                  a->v_stride[0], 1, kChunk, "v");
  if (st != VLAK_OK) return st;
  st = encode_map(&prm.tm_o, a->o, a->H, a->M, a->B, a->o_stride[2], a->o_stride[1],
                  a->o_stride[0], static_cast<uint32_t>(G), static_cast<uint32_t>(prm.MT), "o");
  if (st != VLAK_OK) return st;

  if (dev.device >= 64) return set_error(VLAK_ERR_CUDA, "device ordinal out of range");
  const int grid = static_cast<int>(std::min<long long>(items, dev.sm_count));
  cudaError_t e = ms.mode == kMaskLength ? launch_mode<kMaskLength>(prm, grid, cs, dev.device)
                  : ms.mode == kMaskBool ? launch_mode<kMaskBool>(prm, grid, cs, dev.device)
                                         : launch_mode<kMaskAnalytic>(prm, grid, cs, dev.device);
  if (e != cudaSuccess) return set_cuda_error("fused_attention_gqa launch failed", e);
  return VLAK_OK;
}

namespace {

// Self-test of the bounded-wait machinery: one thread waits on an mbarrier
// that nothing arrives on. The wait runs out after its limit, records
// VLAK_ERR_DEVICE_TIMEOUT in the device error word and the kernel returns
// normally, so the context stays usable.
__global__ void wait_timeout_selftest() {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) bounded_wait(&bar, 0, &abort_flag);
}

}  // namespace

int selftest_wait_timeout(void* stream) {
  clear_error();
  wait_timeout_selftest<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error("wait_timeout_selftest launch failed", e);
  return VLAK_OK;
}

}  // namespace vlak

extern "C" int vlak_selftest_wait_timeout(void* stream) {
  return vlak::selftest_wait_timeout(stream);
}

extern "C" int vlak_attn_gqa_check(const vlak_attn_gqa_args* args, int64_t* prefix_out,
                                   float* scale_out) {
  vlak::clear_error();
  return vlak::validate(args, prefix_out, scale_out);
}

extern "C" int vlak_attn_gqa_fwd(const vlak_attn_gqa_args* args, void* stream) {
  return vlak::launch_gqa(args, stream);
}

extern "C" int vlak_attn_gqa_v4_fwd(const vlak_attn_gqa_args* args, void* stream) {
  return vlak::launch_gqa(args, stream);
}

extern "C" int vlak_attn_gqa_varlen_fwd(const vlak_attn_gqa_args* args, const void* lengths,
                                        int lengths_dtype, void* stream) {
  vlak::MaskSpec ms;
  ms.mode = vlak::kMaskLength;
  ms.lengths = lengths;
  ms.lengths_dtype = lengths_dtype;
  return vlak::launch_gqa(args, stream, ms);
}

extern "C" int vlak_attn_gqa_masked_fwd(const vlak_attn_gqa_args* args, const void* mask,
                                        int64_t mask_stride_b, int64_t mask_stride_m,
                                        void* stream) {
  vlak::MaskSpec ms;
  ms.mode = vlak::kMaskBool;
  ms.mask = mask;
  ms.mask_sb = mask_stride_b;
  ms.mask_sm = mask_stride_m;
  return vlak::launch_gqa(args, stream, ms);
}

extern "C" int vlak_device_error_read(int* code) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, vlak::g_device_error, sizeof(int));
  if (e != cudaSuccess) return vlak::set_cuda_error("vlak_device_error_read", e);
  const int zero = 0;
  e = cudaMemcpyToSymbol(vlak::g_device_error, &zero, sizeof(int));
  if (e != cudaSuccess) return vlak::set_cuda_error("vlak_device_error_read", e);
  if (code) *code = v;
  return VLAK_OK;
}
