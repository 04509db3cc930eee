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
// Items are distributed over a persistent grid of two CTAs per SM; the two
// CTAs' chunk pipelines are independent and fill each other's stalls.
//
// Roles inside a CTA (10 warps):
//   warps 0-3   softmax for M-tile 0, one TMEM lane (query row) per thread
//   warps 4-7   softmax for M-tile 1
//   warp 8      TMA producer: Q tiles into two buffers (items alternate) and
//               64-key K/V chunks through a 3-stage ring
//   warp 9      TMEM allocator and MMA issuer (one elected lane):
//               S_t = Q_t K_c^T  (SS MMA, M=128, N=chunk width, K=64)
//               O_t (+)= P_t V_c (TS MMA: P from TMEM, V from smem, N=64)
// Narrow layout (8 warps, 128 registers), when M-tile 1 never holds more than
// 32 rows (one query block; the expert self-attention's 8 positions x 3
// heads): warps 0-3 softmax for M-tile 0, warp 4 producer, warp 5 MMA issuer,
// and warp 6 or 7 softmax for M-tile 1, whose rows are loaded with a small
// TMA box into TMEM lane quarter 2 or 3 (one per CTA of an SM).
// Keys are processed in 64-key chunks. Softmax writes P over the columns of S
// it has read; the MMA warp then issues P.V and, behind it in issue order,
// the next chunk's S into the same columns.
//
// Tensor memory (256 columns x 128 lanes per CTA, fp32 cells), per M-tile t
// at 128 t: [0,64) S, with P (bf16 pairs, two keys per 32-bit column, the
// A-operand layout of the TS MMA) over its first 32 columns; [64,128) O.
//
// Output. When an item's O is final, its softmax warps write the bf16 rows
// into the item's Q buffer (no longer read by then) and one thread per tile
// stores the tile with a TMA tensor store; the buffer goes back to the
// producer once the store has read it.
//
// Online softmax in the exp2 domain with a lazily updated row max: the
// reference max only moves (and O / l are rescaled in TMEM) when a new
// group's max exceeds it by more than 8 (a factor 256), so P stays <= 256 in
// bf16 and rescales are rare.
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
#include <mutex>

#include "vlak_device.cuh"
#include "vlak_internal.h"

namespace vlak {

// Device error word of this library (see vlak_device_error_read). Used when
// a launch has no host-mapped error word (see host_error_word).
__device__ int g_device_error = 0;

namespace {

// Records a failed wait where the host can see it: in the process's
// host-mapped error word when the launch has one (read without any device
// synchronization by vlak_device_error_poll, which the torch ops call on
// entry), else in the device error word.
__device__ __forceinline__ void publish_device_error(int* host_err, int code) {
  if (host_err != nullptr) {
    *reinterpret_cast<volatile int*>(host_err) = code;
    __threadfence_system();
  } else {
    atomicCAS(&g_device_error, 0, code);
  }
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
        // reported by the CTA's thread 0 once every role has drained
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

// Two CTAs share each SM (each 10 warps, or 8 in the narrow layout below; 256
// TMEM columns; 113 KB of shared memory): the two CTAs' chunk pipelines are
// independent, so one CTA's softmax warps compute while the other's wait on
// TMEM loads, barrier hand-offs or the tensor pipe.
constexpr int kCtasPerSm = 2;
// Warp layout. The full one gives each M-tile four softmax warps. The narrow
// one serves problems whose second M-tile never holds more than 32 rows (one
// query block, e.g. the expert self-attention: 8 positions x 3 heads = 24
// rows in TMEM lanes 0-31): one warp covers that tile, and with 7 warps per
// CTA the register cap of two CTAs per SM rises from 96 to 144.
// In the narrow layout the second tile's rows go to TMEM lane quarter 2 in
// one of an SM's two CTAs and quarter 3 in the other (the CTAs own TMEM
// columns [0, 256) and [256, 512)), served by warp 6 or 7: no SM
// sub-partition then runs more than three softmax warps. The other of
// warps 6 / 7 has no role.
template <bool kNarrow> struct WarpLayout {
  static constexpr int kThreads = kNarrow ? 256 : 320;
  static constexpr int kWarpProducer = kNarrow ? 4 : 8;
  static constexpr int kWarpMma = kNarrow ? 5 : 9;
  static constexpr int kTile1Warps = kNarrow ? 1 : 4;
};
// first TMEM lane (= row of the tile) of the narrow second tile
__device__ __forceinline__ int narrow_tile1_row0(uint32_t tmem) {
  return 64 + 32 * static_cast<int>((tmem >> 8) & 1u);
}
// Key pairs whose exp2 runs on the FMA pipe instead of MUFU: bit (k % 8) of
// the mask selects pair k of a 32-key group (full groups only). With two CTAs
// per SM the MUFU pipe runs at about a fifth of its rate, so all pairs use it
// (measured 1 % faster than moving a quarter of them to the polynomial).
#ifndef VLAK_POLY_MASK
#define VLAK_POLY_MASK 0x00u
#endif
constexpr uint32_t kPolyMask = VLAK_POLY_MASK;
constexpr int kChunk = 64;      // keys per K/V chunk (S tile width)
constexpr int kStages = 3;      // K/V ring depth (chunks) per CTA
constexpr int kRowBytes = 128;  // 64 bf16 per row
constexpr int kTileBytes = 128 * kRowBytes;        // one 128-row Q tile
constexpr int kChunkBytes = kChunk * kRowBytes;    // one 64-key K (or V) chunk
constexpr int kQBytes = 2 * kTileBytes;            // the 2 M-tiles of one item
constexpr int kKVBytes = kStages * kChunkBytes;    // K ring (V ring the same)
// Two Q buffers (items alternate between them). A finished item's buffer
// then stages its O rows for the TMA store.
constexpr int kSmemData = 2 * kQBytes + 2 * kKVBytes;  // 112 KB
constexpr int kBarrierBytes = 256;
// The operand tiles need 1024-byte alignment and the dynamic shared memory
// base is only guaranteed 16-byte aligned. The barrier block goes into the
// alignment gap when the gap has room for it and after the data otherwise,
// so 1008 bytes of slack cover every base alignment: two CTAs then fit in an
// SM's 228 KB (each CTA also has 1 KB reserved by the system).
constexpr int kSmemSlack = 1008;
constexpr int kSmemBytes = kSmemData + kSmemSlack;
static_assert(kBarrierBytes + 240 <= kSmemSlack, "barrier block does not fit the slack");
static_assert(kCtasPerSm * (kSmemBytes + 1024) <= 228 * 1024, "two CTAs must share an SM");

// Tensor memory (256 columns per CTA), per M-tile t at 128 t: S [0,64) and O
// [64,128). P (bf16 pairs, two keys per 32-bit column) is written over the
// first 32 columns of S, which the softmax has already read; the next chunk's
// S is issued behind the P.V product that reads P (MMAs of one thread execute
// in issue order).
constexpr uint32_t kTileCols = 128, kColS = 0, kColO = 64;
constexpr uint32_t kTmemCols = 256;
constexpr float kRescaleThreshold = 8.f;  // log2 units

struct __align__(64) Params {
  CUtensorMap tm_q;  // dims (64, H, M, B), box (64, G, MT, 1)
  CUtensorMap tm_k;  // dims (64, Hkv, N, B), box (64, 1, 64, 1)
  CUtensorMap tm_v;
  CUtensorMap tm_o;  // dims (64, H, M, B), box (64, G, MT, 1), TMA stores of O
  // narrow layout: the second M-tile's M - MT positions (box (64, G, M - MT, 1))
  CUtensorMap tm_q1, tm_o1;
  // Key splits (splits > 1): split s of a query block covers chunks
  // [s * split_chunks, (s + 1) * split_chunks) and writes O / l in bf16 to the
  // partials (dims (64, H, M, splits * B), box as tm_o) and (reference max,
  // row sum) to part_ml; a combine kernel then writes o.
  CUtensorMap tm_part;
  float2* part_ml;
  int splits, split_chunks, n_chunks;
  __nv_bfloat16* o;
  long long o_sb, o_sm, o_sh;  // element strides of o
  int B, M, N, H, Hkv, G;
  int MT;       // query positions per M-tile
  int tiles;    // M-tiles per item (1 or 2)
  int n_mblk;   // query-position blocks per (b, kv head)
  int num_items;
  int P, ds, de;
  float scale_log2;  // softmax scale * log2(e)
  int* host_err;     // host-mapped error word of the process, or nullptr
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
  uint64_t q_full[2], q_empty[2];  // [Q buffer]
  // K (and V) of a stage landed. The split kernel, whose items are a few
  // chunks long, gives V its own barrier so that an item's first S product
  // waits for K alone; in the unsplit kernel both land on k_full (one probe
  // fewer per chunk on the MMA warp's chain).
  uint64_t k_full[kStages], v_full[kStages], kv_empty[kStages];
  uint64_t s_full[2];   // [tile]: S of the chunk is in TMEM
  uint64_t p_full[2];   // [tile]: the tile's 4 softmax warps wrote P
  uint64_t pv_done[2];  // [tile]: P.V of the chunk completed
  uint64_t o_full[2];   // [tile]: O of the item is final
  uint64_t o_staged[2]; // [tile]: the tile's 4 softmax warps wrote O to smem
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
};

static_assert(sizeof(Barriers) <= kBarrierBytes, "barrier block overflows its region");

struct Item {
  int b, kvh, m0;  // m0: first query position of the item
  int tiles_active;
  int L;           // mask mode 1: length of sample b
  int split;       // key split of the item
  int c_begin, c_end;  // key chunks [c_begin, c_end) of the split
};

template <int kMode, bool kSplit>
__device__ __forceinline__ Item decode_item(const Params& p, int item) {
  Item it;
  it.split = kSplit ? item % p.splits : 0;
  const int qblk = kSplit ? item / p.splits : item;
  it.c_begin = kSplit ? it.split * p.split_chunks : 0;
  it.c_end = kSplit ? min(p.n_chunks, it.c_begin + p.split_chunks) : p.n_chunks;
  const int mblk = qblk % p.n_mblk;
  const int bk = qblk / p.n_mblk;
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

// The item's live key chunks -- those holding a visible key for some row of
// the item -- as two intervals [a0, a1) U [b0, b1) (either may be empty).
// Every role computes them once per item from the same arithmetic, so all
// roles agree on the chunk sequence; finding the next chunk is then a couple
// of compares, off the per-chunk critical path of the softmax and MMA warps.
//  - analytic mask: chunk c is live iff 64c < ds, or its keys reach past de
//    and it starts before e2_hi (the end of the item's last row's staircase):
//    [0, ceil(ds / 64)) and [de / 64, ceil(e2_hi / 64)), the second empty when
//    de >= N (no key lies past de);
//  - per-sample length L: [0, ceil(L / 64)) when the item's first row is
//    below L, else nothing;
//  - bool mask: every chunk (the mask is not inspected here).
// A split intersects them with its chunk range [c_begin, c_end).
struct LiveSet {
  int a0, a1, b0, b1;
};
template <int kMode, bool kSplit>
__device__ __forceinline__ LiveSet live_set(const Params& p, const Item& it) {
  LiveSet s{0, 0, 0, 0};
  if (kMode == kMaskBool) {
    s.a1 = p.n_chunks;
  } else if (kMode == kMaskLength) {
    s.a1 = it.m0 < it.L ? (it.L + kChunk - 1) / kChunk : 0;
  } else {
    s.a1 = min(p.n_chunks, (p.ds + kChunk - 1) / kChunk);
    if (p.de < p.N) {
      const int m_hi = min(p.M, it.m0 + it.tiles_active * p.MT) - 1;
      const int e2_hi = max(p.P, min(p.N, p.N - p.M + m_hi + 1));
      s.b0 = p.de / kChunk;
      s.b1 = min(p.n_chunks, (e2_hi + kChunk - 1) / kChunk);
    }
  }
  if (kSplit) {
    s.a0 = max(s.a0, it.c_begin);
    s.a1 = min(s.a1, it.c_end);
    s.b0 = max(s.b0, it.c_begin);
    s.b1 = min(s.b1, it.c_end);
  }
  return s;
}
// First live chunk at or after c, or -1.
__device__ __forceinline__ int live_next(const LiveSet& s, int c) {
  if (c < s.a1 && s.a0 < s.a1) return max(c, s.a0);
  if (c < s.b1 && s.b0 < s.b1) return max(c, s.b0);
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

template <int kMode, bool kSplit, bool kNarrow>
__global__ void __launch_bounds__(WarpLayout<kNarrow>::kThreads, kCtasPerSm)
gqa_attention_sm100(const __grid_constant__ Params p) {
  using WL = WarpLayout<kNarrow>;
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment for the 128-byte-swizzled operand tiles; the barrier
  // block sits in the alignment gap when it fits there
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t gap = ((raw_addr + 1023u) & ~1023u) - raw_addr;
  uint8_t* smem = smem_raw + gap;
  uint8_t* q_smem = smem;                      // [Q buffer][tile][128 x 128 B]
  uint8_t* k_smem = smem + 2 * kQBytes;        // [stage][64 x 128 B]
  uint8_t* v_smem = k_smem + kKVBytes;
  Barriers* bars = reinterpret_cast<Barriers*>(gap >= kBarrierBytes ? smem_raw : smem + kSmemData);
  volatile int* abort_flag = &bars->abort_flag;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->q_full[i], 1);
      // one arrival per M-tile once its O has been read out of the buffer
      // (tile 0 arrives twice for a one-tile item)
      mbar_init(&bars->q_empty[i], 2);
      mbar_init(&bars->o_staged[i], i == 0 ? 4 : WL::kTile1Warps);  // one arrival per softmax warp of the tile
      mbar_init(&bars->s_full[i], 1);
      mbar_init(&bars->p_full[i], i == 0 ? 4 : WL::kTile1Warps);  // one arrival per softmax warp of the tile
      mbar_init(&bars->pv_done[i], 1);
      mbar_init(&bars->o_full[i], 1);
    }
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&bars->k_full[i], 1);
      mbar_init(&bars->v_full[i], 1);
      mbar_init(&bars->kv_empty[i], 1);
    }
    mbar_init(&bars->drain, 1);
    bars->abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == WL::kWarpMma) {
    tmem_alloc(&bars->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  // Q rows that no TMA box covers feed only discarded rows; clear them once so
  // they hold finite values.
  for (int i = threadIdx.x; i < 2 * kQBytes / 16; i += WL::kThreads)
    reinterpret_cast<uint4*>(q_smem)[i] = make_uint4(0, 0, 0, 0);
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  // the merge kernel that follows a split launch may be scheduled from now
  // on; it waits for this grid's completion before reading anything
  if (kSplit) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  const int t1_row0 = kNarrow ? narrow_tile1_row0(tmem) : 0;  // narrow: row offset of tile 1
  const bool softmax_warp = kNarrow ? (warp < 4 || warp == 4 + t1_row0 / 32) : (warp < 8);
  if (warp == WL::kWarpProducer) {
    // ------------------------------------------------------------ producer
    // The whole warp runs this loop (converged); one elected lane issues.
    if (lane == 0) {
      prefetch_tmap(&p.tm_q);
      prefetch_tmap(&p.tm_k);
      prefetch_tmap(&p.tm_v);
    }
    __syncwarp();
    uint32_t qi = 0, kv = 0, q_armed = 0;
    // per K/V stage (its K and V barriers are armed together): bit i of
    // kv_used = armed at least once, bit i of kv_par = parity of its most
    // recently armed phase (registers, no arrays)
    uint32_t kv_used = 0, kv_par = 0;
    bool ok = true;
    for (int item = blockIdx.x; ok && item < p.num_items; item += gridDim.x) {
      const Item it = decode_item<kMode, kSplit>(p, item);
      const LiveSet ls = live_set<kMode, kSplit>(p, it);
      // an item with no live chunk is written as zeros by the softmax warps
      // alone: no Q, no K/V, no barrier phase
      if (live_next(ls, 0) < 0) continue;
      // Q buffer qi & 1 is free once the O rows that item qi - 2 staged in
      // it have been stored
      const uint32_t qb = qi & 1;
      if (!__all_sync(kFullMask, bounded_wait(&bars->q_empty[qb], ((qi >> 1) & 1) ^ 1, abort_flag))) {
        ok = false;
        break;
      }
      const uint32_t qbytes = static_cast<uint32_t>(
          (kNarrow ? p.G * p.MT + (it.tiles_active - 1) * p.G * (p.M - p.MT)
                   : it.tiles_active * p.G * p.MT) * kRowBytes);
      mbar_arrive_expect_tx_elect(&bars->q_full[qb], qbytes);
      ++q_armed;
      tma_load_4d_elect(q_smem + qb * kQBytes, &p.tm_q, &bars->q_full[qb], 0, it.kvh * p.G, it.m0,
                        it.b);
      if (it.tiles_active == 2) {
        if (kNarrow)
          tma_load_4d_elect(q_smem + qb * kQBytes + kTileBytes + t1_row0 * kRowBytes, &p.tm_q1,
                            &bars->q_full[qb], 0, it.kvh * p.G, it.m0 + p.MT, it.b);
        else
          tma_load_4d_elect(q_smem + qb * kQBytes + kTileBytes, &p.tm_q, &bars->q_full[qb], 0,
                            it.kvh * p.G, it.m0 + p.MT, it.b);
      }
      for (int c = live_next(ls, 0); c >= 0; c = live_next(ls, c + 1)) {
        const int s = kv % kStages;
        if (!__all_sync(kFullMask, bounded_wait(&bars->kv_empty[s], ((kv / kStages) & 1) ^ 1, abort_flag))) {
          ok = false;
          break;
        }
        kv_par = (kv_used & (1u << s)) ? (kv_par ^ (1u << s)) : kv_par;
        kv_used |= 1u << s;
        uint64_t* v_bar = kSplit ? &bars->v_full[s] : &bars->k_full[s];
        mbar_arrive_expect_tx_elect(&bars->k_full[s], kSplit ? kChunkBytes : 2 * kChunkBytes);
        tma_load_4d_elect(k_smem + s * kChunkBytes, &p.tm_k, &bars->k_full[s], 0, it.kvh, c * kChunk, it.b);
        if (kSplit) mbar_arrive_expect_tx_elect(v_bar, kChunkBytes);
        tma_load_4d_elect(v_smem + s * kChunkBytes, &p.tm_v, v_bar, 0, it.kvh, c * kChunk, it.b);
        ++kv;
      }
      ++qi;
    }
    // never leave the CTA with copies in flight: wait for the last phase
    // armed on every full barrier (bounded, independent of the abort flag)
    // buffer b was armed (q_armed + 1 - b) / 2 times
    for (uint32_t b = 0; b < 2; ++b) {
      const uint32_t uses = (q_armed + 1 - b) / 2;
      if (uses > 0) bounded_wait(&bars->q_full[b], (uses - 1) & 1, abort_flag, false);
    }
    for (int s = 0; s < kStages; ++s) {
      if (kv_used & (1u << s)) {
        bounded_wait(&bars->k_full[s], (kv_par >> s) & 1u, abort_flag, false);
        if (kSplit) bounded_wait(&bars->v_full[s], (kv_par >> s) & 1u, abort_flag, false);
      }
    }
    __syncwarp();
  } else if (warp == WL::kWarpMma) {
    // ------------------------------------------------------------ MMA issuer
    // Per item and chunk j of tile t: S_t(j) = Q_t K(j)^T into the tile's S
    // columns; once softmax has written P_t(j) over them, O_t (+)= P_t(j) V(j)
    // and, right behind it in issue order, S_t(j+1) over the same columns.
    // The whole warp runs the loop (converged); one elected lane issues.
    {
      uint32_t qi = 0, kv = 0;
      uint32_t pph = 0;  // bit t: parity expected on p_full[t]
      bool ok = true;
      for (int item = blockIdx.x; ok && item < p.num_items; item += gridDim.x) {
        const Item it = decode_item<kMode, kSplit>(p, item);
        const bool two = it.tiles_active == 2;
        const LiveSet ls = live_set<kMode, kSplit>(p, it);
        if (live_next(ls, 0) < 0) continue;  // zeros, written by softmax
        if (!__all_sync(kFullMask, bounded_wait(&bars->q_full[qi & 1], (qi >> 1) & 1, abort_flag))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t q_base = smem_u32(q_smem + (qi & 1) * kQBytes);
        auto issue_s = [&](int t, int c, int j) {  // four K16 steps, 32 B apart in a swizzled row
          const int s = (kv + j) % kStages;
          const uint32_t idesc = idesc_bf16_f32(128, chunk_cols(p, c), false);
          const uint32_t a0 = q_base + t * kTileBytes;
          const uint32_t b0 = smem_u32(k_smem + s * kChunkBytes);
          const uint32_t d = tmem + t * kTileCols + kColS;
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_ss_elect(d, sdesc_sw128(a0 + 32 * k), sdesc_sw128(b0 + 32 * k), idesc, k > 0);
          umma_commit_elect(&bars->s_full[t]);
        };
        auto issue_pv = [&](int t, int c, int j) {  // 16 keys = 8 packed columns of P, 2 KB of V
          const int s = (kv + j) % kStages;
          const int nk = chunk_cols(p, c) / 16;
          const uint32_t idesc = idesc_bf16_f32(128, 64, true);
          const uint32_t b0 = smem_u32(v_smem + s * kChunkBytes);
          const uint32_t a = tmem + t * kTileCols + kColS;
          const uint32_t d = tmem + t * kTileCols + kColO;
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_ts_elect(d, a + 8 * k, sdesc_sw128(b0 + 2048 * k), idesc,
                          (j > 0 || k > 0) ? 1u : 0u, k < nk ? 1u : 0u);
          umma_commit_elect(&bars->pv_done[t]);
        };
        auto wait_kv = [&](uint64_t* full, int j) {  // K or V of chunk j landed
          const uint32_t n = kv + j;
          if (!__all_sync(kFullMask, bounded_wait<kWaitMma>(&full[n % kStages], (n / kStages) & 1, abort_flag)))
            return false;
          tc_fence_after();
          return true;
        };
        auto wait_p = [&](int t) {
          const uint32_t bit = 1u << t;
          if (!__all_sync(kFullMask, bounded_wait<kWaitMma>(&bars->p_full[t], (pph & bit) ? 1u : 0u, abort_flag)))
            return false;
          pph ^= bit;
          tc_fence_after();
          return true;
        };
        int cur = live_next(ls, 0);
        int j = 0;
        // S of chunk 0 is issued after the previous item's last P.V, which
        // read P from the same columns; tcgen05.mma operations of one thread
        // execute in issue order, so no completion wait is needed in between.
        if (!wait_kv(bars->k_full, 0)) { ok = false; break; }
        issue_s(0, cur, 0);
        if (two) issue_s(1, cur, 0);
        while (cur >= 0) {
          const int nxt = live_next(ls, cur + 1);
          // per tile: P of chunk j ready -> O += P V(j), then S of chunk j+1
          // over the S/P columns (in issue order after the product reading P)
          if (!wait_p(0)) { ok = false; break; }
          if (kSplit && !wait_kv(bars->v_full, j)) { ok = false; break; }
          issue_pv(0, cur, j);
          if (nxt >= 0) {
            if (!wait_kv(bars->k_full, j + 1)) { ok = false; break; }
            issue_s(0, nxt, j + 1);
          } else {
            // tile 0's O is final once its last P.V completes: its epilogue
            // need not wait for tile 1's last P
            umma_commit_elect(&bars->o_full[0]);
          }
          if (two) {
            if (!wait_p(1)) { ok = false; break; }
            issue_pv(1, cur, j);
            if (nxt >= 0) issue_s(1, nxt, j + 1);
          }
          umma_commit_elect(&bars->kv_empty[(kv + j) % kStages]);  // K and V of chunk j read
          cur = nxt;
          ++j;
        }
        if (!ok) break;
        // one o_full phase per item with live chunks and tile; each follows
        // the softmax warps' arrivals on p_full, so no phase can run ahead
        umma_commit_elect(&bars->o_full[1], two ? 1u : 0u);
        kv += j;
        ++qi;
      }
      // every issued MMA must complete before TMEM is released
      umma_commit_elect(&bars->drain);
      bounded_wait(&bars->drain, 0, abort_flag, false);
    }
    __syncwarp();  // reconverge before the CTA-wide barrier and the dealloc
  } else if (softmax_warp) {
    // ------------------------------------------------------------ softmax
    // Warp w owns TMEM lane quarter w % 4 (32 query rows) of M-tile w / 4.
    // A chunk's 64 keys are handled as two 32-key groups: load, max, exp,
    // P store per group, so a thread holds 32 scores at a time.
    const int t = warp < 4 ? 0 : 1;
    const int quarter = warp & 3;
    // the warp that stores the tile's O and hands its Q buffer back: quarter
    // 0, or the narrow second tile's only warp
    const bool leader = quarter == 0 || (kNarrow && t == 1);
    const int row = quarter * 32 + lane;    // TMEM lane = row within the tile
    const uint32_t tbase = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + t * kTileCols;
    const uint32_t tS = tbase + kColS;      // S; P (bf16 pairs) over its first 32 columns
    const uint32_t tO = tbase + kColO;
    // the tile's rows start at TMEM lane 0, or at t1_row0 for the narrow
    // second tile
    const int row_rel = row - (t == 1 ? t1_row0 : 0);
    const int m_local = row_rel >= 0 ? row_rel / p.G : p.MT;  // p.MT: no row here
    const int g = row_rel >= 0 ? row_rel - m_local * p.G : 0;
    uint32_t sph = 0, oph = 0, pv_seen = 0;  // pv_seen: this tile's P.V products so far
    uint32_t qi = 0;    // items with live chunks so far; item qi uses Q buffer qi & 1
    // Quarter-0 warps: the Q buffer whose staged O rows this tile's last TMA
    // store reads, (buffer + 1) | (q_empty arrivals << 2), or 0. The buffer is
    // handed back to the producer one chunk later, when the store has long
    // finished reading it, or at once when the warp has no chunk to process.
    uint32_t pend = 0;
    auto release = [&]() {
      if (lane == 0) {
        bulk_wait_read0();
        mbar_arrive_count(&bars->q_empty[(pend & 3u) - 1u], pend >> 2);
      }
      pend = 0;
    };
    bool ok = true;

    for (int item = blockIdx.x; ok && item < p.num_items; item += gridDim.x) {
      const Item it = decode_item<kMode, kSplit>(p, item);
      const LiveSet ls = live_set<kMode, kSplit>(p, it);
      const bool live = live_next(ls, 0) >= 0;
      const uint32_t qb = qi & 1;
      qi += live ? 1u : 0u;
      if (pend != 0 && (t >= it.tiles_active || !live)) release();
      if (t >= it.tiles_active) continue;
      const int m_first = it.m0 + t * p.MT;        // first query position of this tile
      const int m = m_first + m_local;
      const bool valid = (m_local < p.MT) && (m < p.M);
      // a warp whose rows are all invalid skips the arithmetic
      const bool warp_active = __any_sync(kFullMask, valid);
      // this row's visible set [0, ds) U [de, e2) (mask modes 0 and 1) or its
      // bool-mask row (mode 2)
      const int rds = kMode == kMaskAnalytic ? p.ds : 0;
      const int rde = kMode == kMaskAnalytic ? p.de : 0;
      const int e2 = kMode == kMaskAnalytic ? max(p.P, min(p.N, p.N - p.M + m + 1))
                     : kMode == kMaskLength ? (m < it.L ? it.L : 0) : 0;
      const uint8_t* mrow = nullptr;
      if (kMode == kMaskBool && valid)
        mrow = p.mask + static_cast<long long>(it.b) * p.mask_sb + static_cast<long long>(m) * p.mask_sm;
      // this thread's (b, m, h) row in the split partials (computed where
      // used, so it is not live across the chunk loop)
      auto part_row = [&]() {
        return ((static_cast<long long>(it.split) * p.B + it.b) * p.M + m) * p.H + it.kvh * p.G + g;
      };
      if (!live) {
        // no key visible to any row of the item: zeros, no barrier phase (a
        // split records an empty partial, which the combine skips)
        if (valid && kSplit) {
          p.part_ml[part_row()] = make_float2(-INFINITY, 0.f);
        } else if (valid) {
          __nv_bfloat16* orow = p.o + static_cast<long long>(it.b) * p.o_sb +
                                static_cast<long long>(m) * p.o_sm +
                                static_cast<long long>(it.kvh * p.G + g) * p.o_sh;
#pragma unroll
          for (int v = 0; v < 8; ++v) reinterpret_cast<uint4*>(orow)[v] = make_uint4(0, 0, 0, 0);
        }
        continue;
      }
      float m_run = -INFINITY, l_run = 0.f;
      int j = 0;
      for (int c = live_next(ls, 0); c >= 0; c = live_next(ls, c + 1), ++j) {
        // warp-uniform outcome: the TMEM accesses below are warp-collective
        if (!__all_sync(kFullMask, bounded_wait<kWaitSoftmax>(&bars->s_full[t], sph, abort_flag))) {
          ok = false;
          break;
        }
        sph ^= 1u;
        tc_fence_after();
        if (warp_active) {
          const int c0 = c * kChunk;
          const int ncols = chunk_cols(p, c);
          float alpha_o = 1.f, alpha_p = 1.f;  // this chunk's rescale factors (O, first group's P)
          // The narrow layout has the registers to load both groups' scores
          // at once (one TMEM round trip per chunk instead of two).
          float sv2[kNarrow ? kChunk / 32 : 1][32];
          if constexpr (kNarrow) {
            tmem_ld32(tS, sv2[0]);
            tmem_ld32(tS + 32, sv2[1]);
            tmem_wait_ld();
          }
#pragma unroll
          for (int gq = 0; gq < kChunk / 32; ++gq) {
            const int g0 = c0 + 32 * gq;
            const bool in_chunk = 32 * gq < ncols;
            // Warp-uniform class of the 32-key group: every valid row of the
            // warp sees all 32 keys (no mask arithmetic) or none of them (no
            // exp); otherwise each row's visible keys as a bit mask. Rows past
            // the tile or past M do not vote (their outputs are discarded), so
            // the analytic and the bool-mask form of one mask classify alike.
            auto low = [](int n) -> uint32_t {
              return n <= 0 ? 0u : n >= 32 ? 0xffffffffu : ((1u << n) - 1u);
            };
            bool full_l, none_l;
            uint32_t vm = 0u;
            if (kMode == kMaskBool) {
              if (in_chunk && mrow != nullptr) vm = mask_bits32(p, mrow, g0);
              full_l = !valid || (in_chunk && vm == 0xffffffffu);
              none_l = !valid || vm == 0u;
            } else {
              full_l = !valid || (in_chunk && ((g0 + 32 <= rds) || (g0 >= rde && g0 + 32 <= e2)));
              none_l = !valid || !in_chunk || ((g0 >= rds) && (g0 + 32 <= rde || g0 >= e2));
            }
            const bool full = __all_sync(kFullMask, full_l);
            const bool none = __all_sync(kFullMask, none_l);
            if (kMode != kMaskBool && !full && !none)
              vm = valid ? (low(rds - g0) | (low(e2 - g0) & ~low(rde - g0))) : 0u;
            float (&sv)[32] = sv2[kNarrow ? gq : 0];
            float mx = -INFINITY;
            if (!none) {
              if constexpr (!kNarrow) {
                tmem_ld32(tS + 32 * gq, sv);
                tmem_wait_ld();
              }
              // group max with four independent accumulators
              float mxa[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
              if (full) {
#pragma unroll
                for (int i = 0; i < 32; i += 2)
                  mxa[(i >> 1) & 3] = fmax3(mxa[(i >> 1) & 3], sv[i], sv[i + 1]);
              } else {
#pragma unroll
                for (int i = 0; i < 32; i += 2)
                  mxa[(i >> 1) & 3] = fmax3(mxa[(i >> 1) & 3], ((vm >> i) & 1u) ? sv[i] : -INFINITY,
                                            ((vm >> (i + 1)) & 1u) ? sv[i + 1] : -INFINITY);
              }
              mx = fmax3(fmaxf(mxa[0], mxa[1]), mxa[2], mxa[3]);
            }
            const float mz = mx * p.scale_log2;  // -inf stays -inf (scale > 0)
            // The reference max moves only when a group's max exceeds it by
            // more than the threshold; O, l and the P already written for this
            // chunk are then rescaled by alpha (below, once the scores are dead).
            float alpha = 1.f;
            if (j == 0 && gq == 0) {
              m_run = mz;
            } else if (mz > m_run + kRescaleThreshold) {
              alpha = ex2(m_run - mz);
              m_run = mz;
            }
            if (!in_chunk) continue;  // (no keys: alpha is 1)
            // P = exp2(s * scale_log2 - mref) as bf16 pairs over the group's
            // first 16 columns of S. Key pairs go through the f32x2 FMA pipe;
            // exps run on MUFU except for the pairs kPolyMask selects, which
            // use the FMA-pipe polynomial (full groups only, where no -inf
            // occurs).
            const float nref = (m_run == -INFINITY) ? 0.f : -m_run;
            const uint64_t sl2 = f2_pack(p.scale_log2, p.scale_log2);
            const uint64_t nr2 = f2_pack(nref, nref);
            uint64_t acc[2] = {0ull, 0ull};  // two (+0.f, +0.f) pairs
            uint32_t pk[16];
            if (none) {
#pragma unroll
              for (int i = 0; i < 16; ++i) pk[i] = 0u;
            } else if (full) {
#pragma unroll
              for (int k = 0; k < 16; ++k) {
                const uint64_t x = f2_fma(f2_pack(sv[2 * k], sv[2 * k + 1]), sl2, nr2);
                uint64_t e;
                float x0, x1;
                f2_unpack(x, x0, x1);
                if ((kPolyMask >> (k & 7)) & 1u) {
                  e = f2_exp2_poly(f2_pack(fmaxf(x0, -126.f), fmaxf(x1, -126.f)));
                } else {
                  e = f2_pack(ex2(x0), ex2(x1));
                }
                acc[k & 1] = f2_add(acc[k & 1], e);
                float e0, e1;
                f2_unpack(e, e0, e1);
                pk[k] = pack_bf16x2(e0, e1);
              }
            } else {
#pragma unroll
              for (int k = 0; k < 16; ++k) {
                const uint64_t x = f2_fma(f2_pack(sv[2 * k], sv[2 * k + 1]), sl2, nr2);
                float x0, x1;
                f2_unpack(x, x0, x1);
                const float e0 = ((vm >> (2 * k)) & 1u) ? ex2(x0) : 0.f;
                const float e1 = ((vm >> (2 * k + 1)) & 1u) ? ex2(x1) : 0.f;
                acc[k & 1] = f2_add(acc[k & 1], f2_pack(e0, e1));
                pk[k] = pack_bf16x2(e0, e1);
              }
            }
            tmem_st16(tS + 16 * gq, pk);
            float acc0, acc1;
            f2_unpack(f2_add(acc[0], acc[1]), acc0, acc1);
            l_run = l_run * alpha + (acc0 + acc1);
            alpha_o *= alpha;
            if (gq > 0) alpha_p = alpha;
          }
          // Rare: the reference max moved within the chunk. O (P.V of chunks
          // 0 .. j-1) is rescaled by the product of the chunk's factors and
          // the first group's P by the second group's factor; the scores are
          // no longer live here.
          if (__any_sync(kFullMask, alpha_o != 1.f)) {
            if (__any_sync(kFullMask, alpha_p != 1.f)) {
              tmem_wait_st();  // the first group's P store has landed
              float pf[16];
              tmem_ld16(tS, pf);
              tmem_wait_ld();
              uint32_t pw[16];
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                const uint32_t w = __float_as_uint(pf[i]);
                pw[i] = pack_bf16x2(__uint_as_float(w << 16) * alpha_p,
                                    __uint_as_float(w & 0xffff0000u) * alpha_p);
              }
              tmem_st16(tS, pw);
            }
            if (j > 0) {
              if (!__all_sync(kFullMask, bounded_wait(&bars->pv_done[t], (pv_seen - 1) & 1, abort_flag))) {
                ok = false;
                break;
              }
              tc_fence_after();
#pragma unroll 1
              for (int q4 = 0; q4 < 4; ++q4) {  // 16 columns at a time keeps the registers low
                float o[16];
                tmem_ld16(tO + 16 * q4, o);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 16; ++i) o[i] *= alpha_o;
                tmem_st16f(tO + 16 * q4, o);
              }
            }
          }
          tmem_wait_st();
        }
        ++pv_seen;
        tc_fence_before();
        mbar_arrive_elect(&bars->p_full[t], 1u);
        if (pend != 0) release();
      }
      if (!ok) break;
      // Epilogue: O / l -> bf16 rows staged in this item's Q buffer (dead once
      // O is final: every MMA of the item has completed), in the 128-byte
      // swizzled layout of the Q / O tensor maps, then one TMA store per tile.
      // Per-thread global stores of whole rows (one 128-byte line per lane)
      // flood the SM's memory pipeline and stall the barrier waits behind it.
      if (!__all_sync(kFullMask, bounded_wait(&bars->o_full[t], oph, abort_flag))) { ok = false; break; }
      oph ^= 1;
      tc_fence_after();
      uint8_t* stage = q_smem + qb * kQBytes + t * kTileBytes;
      if (warp_active) {
        const bool any = (j > 0) && (l_run > 0.f);
        const float inv = any ? 1.f / l_run : 0.f;
#pragma unroll 1
        for (int q4 = 0; q4 < 4; ++q4) {  // 16 columns of O at a time
          float o[16];
          if (j > 0) {
            tmem_ld16(tO + 16 * q4, o);
            tmem_wait_ld();
          }
          if (valid) {
#pragma unroll
            for (int v = 0; v < 2; ++v) {
              uint32_t w[4];
#pragma unroll
              for (int e = 0; e < 4; ++e)
                w[e] = any ? pack_bf16x2(o[v * 8 + 2 * e] * inv, o[v * 8 + 2 * e + 1] * inv) : 0u;
              const uint32_t chunk = static_cast<uint32_t>(2 * q4 + v) ^ static_cast<uint32_t>(row & 7);
              st_shared_v4(stage + row * kRowBytes + chunk * 16, w[0], w[1], w[2], w[3]);
            }
          }
        }
      }
      if (kSplit && valid) p.part_ml[part_row()] = make_float2(m_run, l_run);
      fence_proxy_async_smem();
      mbar_arrive_elect(&bars->o_staged[t], 1u);
      if (leader) {
        // o_staged completes one phase per item of the tile, like o_full
        if (!__all_sync(kFullMask, bounded_wait(&bars->o_staged[t], oph ^ 1u, abort_flag))) {
          ok = false;
          break;
        }
        if (lane == 0) {
          if (kNarrow && t == 1)  // the tile's rows start at t1_row0
            tma_store_4d(&p.tm_o1, stage + t1_row0 * kRowBytes, 0, it.kvh * p.G, m_first,
                         kSplit ? it.split * p.B + it.b : it.b);
          else if (kSplit)
            tma_store_4d(&p.tm_part, stage, 0, it.kvh * p.G, m_first, it.split * p.B + it.b);
          else
            tma_store_4d(&p.tm_o, stage, 0, it.kvh * p.G, m_first, it.b);
          bulk_commit_group();
        }
        pend = (qb + 1u) | ((t == 0 && it.tiles_active == 1 ? 2u : 1u) << 2);
      }
      // the next item's first P.V overwrites O once this tile's softmax warps
      // arrive on p_full, after these loads
      tc_fence_before();
    }
    // the TMA stores of this warp's last items complete before the CTA exits
    if (leader && lane == 0) bulk_wait_all0();
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && *abort_flag) publish_device_error(p.host_err, VLAK_ERR_DEVICE_TIMEOUT);
  if (warp == WL::kWarpMma) {
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

// Merge of the key splits: eight threads per row of o, eight bf16 each. Split
// s of a row holds O_s / l_s (bf16) and (m_s, l_s): its rows' probabilities
// are 2^(x - m_s) and l_s their sum, so the whole row's sum is
// sum_s l_s 2^(m_s - m*) (any common m*) and O = sum_s w_s (O_s / l_s) /
// sum_s w_s with w_s = l_s 2^(m_s - m*). Splits with l_s = 0 saw no visible
// key and are skipped; a row with none left is written as zeros.
// The kernel is a chain of L2 round trips, so the loads of kCombineBatch
// splits are issued together: with at most that many splits every (m_s, l_s)
// and partial row is in flight at once (one round trip), otherwise one round
// trip for the maximum per batch and one for the sums. The sums run over s in
// ascending order whatever the batching.
constexpr int kCombineBatch = 8;
__global__ void __launch_bounds__(256) combine_splits(const __nv_bfloat16* __restrict__ part,
                                                      const float2* __restrict__ ml,
                                                      __nv_bfloat16* o, long long o_sb, long long o_sm,
                                                      long long o_sh, int B, int M, int H, int splits) {
  // launched as a programmatic dependent of the attention kernel: wait for
  // that grid to complete and its partials to be visible
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const long long rows = static_cast<long long>(B) * M * H;
  const long long tid = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  const long long r = tid >> 3;
  const int q = static_cast<int>(tid & 7);
  if (r >= rows) return;
  float2 v[kCombineBatch];
  uint4 u[kCombineBatch];
  auto load_ml = [&](int s0) {
#pragma unroll
    for (int i = 0; i < kCombineBatch; ++i)
      v[i] = s0 + i < splits ? ml[(s0 + i) * rows + r] : make_float2(-INFINITY, 0.f);
  };
  auto load_part = [&](int s0) {
#pragma unroll
    for (int i = 0; i < kCombineBatch; ++i)
      u[i] = s0 + i < splits
                 ? *reinterpret_cast<const uint4*>(part + ((s0 + i) * rows + r) * 64 + q * 8)
                 : make_uint4(0, 0, 0, 0);
  };
  float mx = -INFINITY;
  auto batch_max = [&]() {
#pragma unroll
    for (int i = 0; i < kCombineBatch; ++i)
      if (v[i].y > 0.f) mx = fmaxf(mx, v[i].x);
  };
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  float wsum = 0.f;
  auto accumulate = [&]() {
#pragma unroll
    for (int i = 0; i < kCombineBatch; ++i) {
      if (!(v[i].y > 0.f)) continue;
      const float w = exp2f(v[i].x - mx) * v[i].y;
      wsum += w;
      const uint32_t uw[4] = {u[i].x, u[i].y, u[i].z, u[i].w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        acc[2 * e] += w * __uint_as_float(uw[e] << 16);
        acc[2 * e + 1] += w * __uint_as_float(uw[e] & 0xffff0000u);
      }
    }
  };
  if (splits <= kCombineBatch) {
    load_ml(0);
    load_part(0);
    batch_max();
    accumulate();
  } else {
    for (int s0 = 0; s0 < splits; s0 += kCombineBatch) {
      load_ml(s0);
      batch_max();
    }
    for (int s0 = 0; s0 < splits; s0 += kCombineBatch) {
      load_ml(s0);
      load_part(s0);
      accumulate();
    }
  }
  const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
  const long long h = r % H, bm = r / H, m = bm % M, b = bm / M;
  uint32_t w[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) w[e] = pack_bf16x2(acc[2 * e] * inv, acc[2 * e + 1] * inv);
  *reinterpret_cast<uint4*>(o + b * o_sb + m * o_sm + h * o_sh + q * 8) = make_uint4(w[0], w[1], w[2], w[3]);
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
  // The reference requires this for its cp.async tiles; the same condition
  // is what TMA tensor maps need here (16-byte base and byte strides).
  const void* ptrs[4] = {a->q, a->k, a->v, a->o};
  const int64_t* strides[4] = {a->q_stride, a->k_stride, a->v_stride, a->o_stride};
  constexpr const char* kAlignMsg = "strides/base must keep 16B alignment (TMA tensor maps)";
  for (int i = 0; i < 4; ++i) {
    if (reinterpret_cast<uintptr_t>(ptrs[i]) % 16 != 0) return set_error(VLAK_ERR_ALIGNMENT, kAlignMsg);
    for (int d = 0; d < 3; ++d)
      if (strides[i][d] % 8 != 0) return set_error(VLAK_ERR_ALIGNMENT, kAlignMsg);
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
  void* workspace = nullptr;  // key-split partials (nullptr: never split)
  int64_t workspace_bytes = 0;
  bool no_alloc = false;      // never set up the host error word here
};

// Query tiling of an item: MT query positions per M-tile, 1 or 2 M-tiles per
// item, n_mblk query blocks per (b, kv head).
struct Tiling {
  int G, MT, tiles, n_mblk, n_chunks;
};
static Tiling tiling_of(const vlak_attn_gqa_args* a) {
  Tiling t;
  t.G = static_cast<int>(a->H / a->Hkv);
  const int M = static_cast<int>(a->M);
  t.MT = std::min(128 / t.G, M);
  t.tiles = M > t.MT ? 2 : 1;
  t.n_mblk = (M + t.tiles * t.MT - 1) / (t.tiles * t.MT);
  t.n_chunks = static_cast<int>((a->N + kChunk - 1) / kChunk);
  return t;
}

// Key splits. When the query blocks fill less than half of the CTA slots
// (small batches, few heads), each block's keys are split into up to
// n_chunks contiguous ranges processed by separate items, enough to fill the
// slots; a second kernel merges the splits.
// Workspace: splits * B * M * H rows of 128 bytes (bf16 O / l), then 8 bytes
// per row (m, l), the first part rounded up to 256 bytes.
struct SplitPlan {
  int splits = 1, split_chunks = 1;
  int64_t part_bytes = 0, bytes = 0;
};
static SplitPlan plan_splits(const vlak_attn_gqa_args* a, const Tiling& t, int sm_count) {
  SplitPlan sp;
  sp.split_chunks = std::max(t.n_chunks, 1);
  const long long base = static_cast<long long>(a->B) * a->Hkv * t.n_mblk;
  const long long slots = static_cast<long long>(sm_count) * kCtasPerSm;
  // The merge costs about as much as three chunk steps of one CTA, so a
  // split must shorten the chain by at least four chunks.
  if (t.n_chunks < 5 || base <= 0 || 2 * base > slots) return sp;
  const int want = static_cast<int>(std::min<long long>(t.n_chunks, (slots + base - 1) / base));
  sp.split_chunks = (t.n_chunks + want - 1) / want;
  sp.splits = (t.n_chunks + sp.split_chunks - 1) / sp.split_chunks;
  if (sp.splits < 2) {
    sp.splits = 1;
    sp.split_chunks = t.n_chunks;
    return sp;
  }
  const long long rows = static_cast<long long>(a->B) * a->M * a->H;
  sp.part_bytes = (sp.splits * rows * 128 + 255) / 256 * 256;
  sp.bytes = sp.part_bytes + sp.splits * rows * 8;
  return sp;
}

template <int kMode, bool kSplit, bool kNarrow>
static cudaError_t launch_variant(const Params& prm, int grid, cudaStream_t cs, int device) {
  // one-time per (device, variant) opt-in to the large dynamic shared-memory carve-out
  static std::atomic<int> ready[64];
  if (ready[device].load() == 0) {
    cudaError_t e = cudaFuncSetAttribute(gqa_attention_sm100<kMode, kSplit, kNarrow>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return e;
    ready[device].store(1);
  }
  gqa_attention_sm100<kMode, kSplit, kNarrow>
      <<<grid, WarpLayout<kNarrow>::kThreads, kSmemBytes, cs>>>(prm);
  return cudaGetLastError();
}
template <int kMode>
static cudaError_t launch_mode(const Params& prm, int grid, cudaStream_t cs, int device) {
  // the narrow warp layout when the second M-tile holds at most 32 rows
  // (analytic mask only: the sites of the other modes never qualify)
  if constexpr (kMode == kMaskAnalytic) {
    if (prm.tiles == 2 && prm.n_mblk == 1 && (prm.M - prm.MT) * prm.G <= 32)
      return prm.splits > 1 ? launch_variant<kMode, true, true>(prm, grid, cs, device)
                            : launch_variant<kMode, false, true>(prm, grid, cs, device);
  }
  return prm.splits > 1 ? launch_variant<kMode, true, false>(prm, grid, cs, device)
                        : launch_variant<kMode, false, false>(prm, grid, cs, device);
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
  const Tiling tl = tiling_of(a);
  const int G = tl.G;
  prm.B = static_cast<int>(a->B);
  prm.M = static_cast<int>(a->M);
  prm.N = static_cast<int>(a->N);
  prm.H = static_cast<int>(a->H);
  prm.Hkv = static_cast<int>(a->Hkv);
  prm.G = G;
  prm.MT = tl.MT;
  prm.tiles = tl.tiles;
  prm.n_mblk = tl.n_mblk;
  prm.n_chunks = tl.n_chunks;
  SplitPlan sp;
  if (ms.workspace) {
    if (reinterpret_cast<uintptr_t>(ms.workspace) % 256 != 0)
      return set_error(VLAK_ERR_ALIGNMENT, "fused_attention_gqa: workspace must be 256-byte aligned");
    sp = plan_splits(a, tl, dev.sm_count);
    if (sp.splits > 1 && ms.workspace_bytes < sp.bytes) sp = SplitPlan();  // too small: no split
  }
  prm.splits = sp.splits;
  prm.split_chunks = sp.splits > 1 ? sp.split_chunks : tl.n_chunks;
  const long long items = static_cast<long long>(prm.B) * prm.Hkv * prm.n_mblk * prm.splits;
  if (items > INT32_MAX) return set_error(VLAK_ERR_INVALID_ARGUMENT, "fused_attention_gqa: too many work items");
  prm.num_items = static_cast<int>(items);
  prm.P = static_cast<int>(P);
  prm.ds = static_cast<int>(a->dead_start);
  prm.de = static_cast<int>(a->dead_end);
  prm.scale_log2 = scale * 1.4426950408889634f;
  prm.host_err = host_error_word(cs, !ms.no_alloc);
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
  st = encode_map(&prm.tm_o, a->o, a->H, a->M, a->B, a->o_stride[2], a->o_stride[1],
                  a->o_stride[0], static_cast<uint32_t>(G), static_cast<uint32_t>(prm.MT), "o");
  if (st != VLAK_OK) return st;
  // narrow layout: one query block whose second M-tile holds <= 32 rows
  const bool narrow = ms.mode == kMaskAnalytic && prm.tiles == 2 && prm.n_mblk == 1 &&
                      (prm.M - prm.MT) * G <= 32;
  if (narrow) {
    const uint32_t n1 = static_cast<uint32_t>(prm.M - prm.MT);
    st = encode_map(&prm.tm_q1, a->q, a->H, a->M, a->B, a->q_stride[2], a->q_stride[1],
                    a->q_stride[0], static_cast<uint32_t>(G), n1, "q");
    if (st != VLAK_OK) return st;
    if (ms.workspace && sp.splits > 1)
      st = encode_map(&prm.tm_o1, ms.workspace, a->H, a->M, a->B * sp.splits, 64, a->H * 64,
                      a->M * a->H * 64, static_cast<uint32_t>(G), n1, "workspace");
    else
      st = encode_map(&prm.tm_o1, a->o, a->H, a->M, a->B, a->o_stride[2], a->o_stride[1],
                      a->o_stride[0], static_cast<uint32_t>(G), n1, "o");
    if (st != VLAK_OK) return st;
  }
  if (sp.splits > 1) {
    const int64_t H = a->H;
    st = encode_map(&prm.tm_part, ms.workspace, H, a->M, a->B * sp.splits, 64, H * 64,
                    a->M * H * 64, static_cast<uint32_t>(G), static_cast<uint32_t>(prm.MT),
                    "workspace");
    if (st != VLAK_OK) return st;
    prm.part_ml = reinterpret_cast<float2*>(static_cast<uint8_t*>(ms.workspace) + sp.part_bytes);
  }
  st = encode_map(&prm.tm_k, a->k, a->Hkv, a->N, a->B, a->k_stride[2], a->k_stride[1],
                  a->k_stride[0], 1, kChunk, "k");
  if (st != VLAK_OK) return st;
  st = encode_map(&prm.tm_v, a->v, a->Hkv, a->N, a->B, a->v_stride[2], a->v_stride[1],
                  a->v_stride[0], 1, kChunk, "v");
  if (st != VLAK_OK) return st;

  if (dev.device >= 64) return set_error(VLAK_ERR_CUDA, "device ordinal out of range");
  const int grid = static_cast<int>(std::min<long long>(items, static_cast<long long>(dev.sm_count) * kCtasPerSm));

  cudaError_t e = ms.mode == kMaskLength ? launch_mode<kMaskLength>(prm, grid, cs, dev.device)
                  : ms.mode == kMaskBool ? launch_mode<kMaskBool>(prm, grid, cs, dev.device)
                                         : launch_mode<kMaskAnalytic>(prm, grid, cs, dev.device);
  if (e != cudaSuccess) return set_cuda_error("fused_attention_gqa launch failed", e);
  if (sp.splits > 1) {
    const long long threads = static_cast<long long>(a->B) * a->M * a->H * 8;
    // programmatic dependent launch: the merge grid is scheduled while the
    // attention grid drains and waits on the device for its completion
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>((threads + 255) / 256));
    cfg.blockDim = dim3(256);
    cfg.stream = cs;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, combine_splits, static_cast<const __nv_bfloat16*>(ms.workspace),
                           static_cast<const float2*>(prm.part_ml), o,
                           static_cast<long long>(a->o_stride[0]),
                           static_cast<long long>(a->o_stride[1]),
                           static_cast<long long>(a->o_stride[2]), prm.B, prm.M, prm.H, sp.splits);
    if (e != cudaSuccess) return set_cuda_error("fused_attention_gqa split combine failed", e);
  }
  return VLAK_OK;
}

static int workspace_size(const vlak_attn_gqa_args* a, int64_t* bytes) {
  clear_error();
  if (!bytes) return set_error(VLAK_ERR_INVALID_ARGUMENT, "workspace size: null output");
  *bytes = 0;
  int st = validate(a, nullptr, nullptr);
  if (st != VLAK_OK) return st;
  if (a->B == 0 || a->M == 0 || a->N == 0) return VLAK_OK;
  DeviceInfo dev;
  st = current_device_info(&dev);
  if (st != VLAK_OK) return st;
  *bytes = plan_splits(a, tiling_of(a), dev.sm_count).bytes;
  return VLAK_OK;
}

namespace {

// Self-test of the bounded-wait machinery: one thread waits on an mbarrier
// that nothing arrives on. The wait runs out after its limit, records
// VLAK_ERR_DEVICE_TIMEOUT in the device error word and the kernel returns
// normally, so the context stays usable.
__global__ void wait_timeout_selftest(int* host_err) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0 && !bounded_wait(&bar, 0, &abort_flag))
    publish_device_error(host_err, VLAK_ERR_DEVICE_TIMEOUT);
}

}  // namespace

int selftest_wait_timeout(void* stream) {
  clear_error();
  cudaStream_t cs = static_cast<cudaStream_t>(stream);
  wait_timeout_selftest<<<1, 32, 0, cs>>>(host_error_word(cs));
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

extern "C" int vlak_attn_gqa_workspace_size(const vlak_attn_gqa_args* args, int64_t* bytes) {
  return vlak::workspace_size(args, bytes);
}

extern "C" int vlak_attn_gqa_fwd_ws(const vlak_attn_gqa_args* args, void* workspace,
                                    int64_t workspace_bytes, void* stream) {
  vlak::MaskSpec ms;
  ms.workspace = workspace;
  ms.workspace_bytes = workspace_bytes;
  return vlak::launch_gqa(args, stream, ms);
}

extern "C" int vlak_attn_gqa_varlen_fwd_ws(const vlak_attn_gqa_args* args, const void* lengths,
                                           int lengths_dtype, void* workspace,
                                           int64_t workspace_bytes, void* stream) {
  vlak::MaskSpec ms;
  ms.mode = vlak::kMaskLength;
  ms.lengths = lengths;
  ms.lengths_dtype = lengths_dtype;
  ms.workspace = workspace;
  ms.workspace_bytes = workspace_bytes;
  return vlak::launch_gqa(args, stream, ms);
}

extern "C" int vlak_attn_gqa_masked_fwd_ws(const vlak_attn_gqa_args* args, const void* mask,
                                           int64_t mask_stride_b, int64_t mask_stride_m,
                                           void* workspace, int64_t workspace_bytes,
                                           void* stream) {
  vlak::MaskSpec ms;
  ms.mode = vlak::kMaskBool;
  ms.mask = mask;
  ms.mask_sb = mask_stride_b;
  ms.mask_sm = mask_stride_m;
  ms.workspace = workspace;
  ms.workspace_bytes = workspace_bytes;
  return vlak::launch_gqa(args, stream, ms);
}

// ---------------------------------------------------------------------------
// Allocation-free GQA attention. For callers that must not allocate device
// memory per call: a robot-control loop that reserves all of its memory at
// start-up and treats an allocation inside the loop as a latency fault
// (cudaMalloc synchronizes the device and can take milliseconds), or a host
// reaching the library through a C FFI (Go, Java, plain C) that has no pool
// allocator to draw a workspace from. The key-split scratch then comes from
// this file's static device buffer instead of a caller workspace.
namespace vlak {
namespace {

constexpr int64_t kNoAllocScratchBytes = int64_t(8) << 20;  // 8 MiB per device
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of the static scratch on the current device, looked up once
// per device (with that device current) on its first call.
int noalloc_scratch(void** out) {
  constexpr int kMaxDev = 64;
  static std::mutex mu;
  static void* addr[kMaxDev] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_cuda_error("cudaGetDevice", e);
  if (dev < 0 || dev >= kMaxDev) return set_error(VLAK_ERR_CUDA, "device ordinal out of range");
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return set_cuda_error("fused_attention_gqa_noalloc: scratch address", e);
    addr[dev] = p;
  }
  *out = addr[dev];
  return VLAK_OK;
}

}  // namespace
}  // namespace vlak

extern "C" int vlak_attn_gqa_fwd_noalloc(const vlak_attn_gqa_args* args, void* stream) {
  using namespace vlak;
  int64_t need = 0;
  int st = workspace_size(args, &need);  // validates the arguments too
  if (st != VLAK_OK) return st;
  if (need > kNoAllocScratchBytes)
    return set_errorf(VLAK_ERR_INVALID_ARGUMENT,
                      "fused_attention_gqa_noalloc: this problem needs %lld bytes of key-split "
                      "scratch, more than the %lld-byte static buffer; call vlak_attn_gqa_fwd_ws "
                      "with a workspace instead",
                      static_cast<long long>(need), static_cast<long long>(kNoAllocScratchBytes));
  MaskSpec ms;
  ms.no_alloc = true;
  if (need > 0) {
    st = noalloc_scratch(&ms.workspace);
    if (st != VLAK_OK) return st;
    ms.workspace_bytes = kNoAllocScratchBytes;
  }
  return launch_gqa(args, stream, ms);
}

extern "C" int vlak_device_error_read(int* code) {
  vlak::clear_error();
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, vlak::g_device_error, sizeof(int));
  if (e != cudaSuccess) return vlak::set_cuda_error("vlak_device_error_read", e);
  const int zero = 0;
  e = cudaMemcpyToSymbol(vlak::g_device_error, &zero, sizeof(int));
  if (e != cudaSuccess) return vlak::set_cuda_error("vlak_device_error_read", e);
  // the host-mapped word of the process (cleared as well)
  int h = 0;
  vlak_device_error_poll(&h);
  if (code) *code = v != 0 ? v : h;
  return VLAK_OK;
}
