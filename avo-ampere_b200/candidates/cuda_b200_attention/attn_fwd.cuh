// BF16 attention forward for sm_100a (B200), head_dim 128.
//
// Replaces the candidate kernel behind `attention(q, k, v, causal)` of the AVO
// candidate contract (candidates/cuda_mma_attention/attention_kernel.cu:22-171 in
// the reference, a 16x16 WMMA kernel).  The math is the same softmax(QK^T*scale)V
// with an optional lower-triangular mask (query i sees keys <= i,
// candidates/cuda_naive_attention/attention_kernel.cu:28) and the online-softmax
// recurrence of candidates/cuda_tiled_attention/attention_kernel.cu:84-99; the
// structure is Blackwell-native and shares nothing with the reference kernels:
//
//   * the grid is persistent, one CTA per SM; a work item is 256 query rows of one
//     (batch, head) as two 128-row Q tiles, and CTA c takes one item per wave,
//     walking the waves in alternating directions (longest causal items first);
//   * warp 8 streams Q and the K and V tiles (128 keys x 128 dims, bf16) with TMA:
//     K_j and V_j alternate in a 4-slot shared-memory ring, mbarrier-tracked, and
//     the next item's Q is loaded as soon as the current item's last S has read Q;
//   * warp 9 issues tcgen05.mma: S_i = Q_i K_j^T into TMEM, then O_i += P_i V_j
//     with P_i read straight from TMEM (bf16, in S_i's columns 64-127); it waits only on
//     hardware named barriers (warp 10 performs the mbarrier waits for it);
//   * warps 0-3 and 4-7 are two softmax warpgroups, one per Q tile, one thread
//     per query row: tcgen05.ld of the S row, max, exp2 with scale*log2(e) folded
//     into one FFMA, row sum, tcgen05.st of P.  The running max is only raised
//     when it grows by more than 2^15 ("conditional rescale"), so O in TMEM is
//     rescaled rarely; the two groups ping-pong against the tensor core;
//   * causal tiles above the diagonal are never loaded or multiplied;
//   * the epilogue scales O by 1/l and writes each row straight from registers as
//     whole 32-byte sectors, while the MMA warp already computes the next item's
//     first S tiles; LSE (natural log) goes out as coalesced fp32.
//
// Every mbarrier wait is bounded by a wall-clock watchdog: on expiry the CTA sets
// a status bit, stops issuing work, drains its in-flight copies and MMAs, frees
// TMEM and returns.  Nothing traps.
#pragma once

#include <cuda_bf16.h>
#include <math_constants.h>

#include <type_traits>

#include "schedule.cuh"
#include "sm100_ptx.cuh"

// Optional per-tile timeline hooks (role, tile, event) for development builds; they
// compile to nothing unless a build defines AVO_TRACE_HOOK before including this file.
#ifndef AVO_TRACE_HOOK
#define AVO_TRACE_HOOK(role, tile, event)
#endif

namespace avo_b200 {

constexpr int kHeadDim = 128;
constexpr int kBlockM = 128;                   // rows per Q tile (one M=128 accumulator)
constexpr int kQTiles = 2;                     // Q tiles per work item
constexpr int kRowsPerCta = kBlockM * kQTiles; // 256 query rows per work item
constexpr int kBlockN = 128;                   // keys per K/V tile
constexpr int kStages = 4;                     // K/V ring depth
constexpr int kTileBytes = 128 * kHeadDim * 2; // 32 KiB: 128 rows x 128 bf16
constexpr int kHalfBytes = kTileBytes / 2;     // one 64-column, 128B-swizzled half
constexpr int kLoadWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kWaitWarp = 10;
// Named barriers: 0 = __syncthreads, 3 = waiter -> MMA warp release (64 threads),
// 4 + 2*tile + half = P half of a Q tile published, 8 + tile = the tile's O read out by
// its epilogue (for both: the tile's 4 softmax warps arrive, the MMA warp syncs; 160
// threads).
constexpr uint32_t kBarMmaHandoff = 3;
constexpr uint32_t kBarPHalf = 4;
constexpr uint32_t kBarOFree = 8;
constexpr uint32_t kBarSlot = 10;              // 10 + tile: the tile's 4 softmax warps (split pieces)
constexpr uint32_t kPHalfThreads = 128 + 32;
constexpr int kThreads = 384;                  // 3 warpgroups: softmax 0, softmax 1, load/MMA/waiter
// Register split (setmaxnreg): launched at 168 per thread (384 x 168 = 64512), the
// load/MMA warpgroup drops to 72 and each softmax warpgroup rises to 216:
// 2 x 128 x 216 + 128 x 72 = 64512 (no spills in either role; measured on B200 against
// 208/88 and 224/56: equal on non-causal work, faster on causal).
constexpr uint32_t kRegsLaunch = 168;
constexpr uint32_t kRegsSoftmax = 216;
constexpr uint32_t kRegsOther = 72;
static_assert(2 * 128 * kRegsSoftmax + 128 * kRegsOther <= kThreads * kRegsLaunch, "register split");
constexpr uint32_t kTmemCols = 512;            // S0 | S1 | O0 | O1, 128 columns each
// log2 units: the running max (and O, l with it) moves only when a tile's max exceeds it by
// more than 2^15, so P = 2^(s*scale - m) stays below 2^15: exact in bf16 (8 exponent bits),
// inside the FMA-pipe exp2's input range, and the fp32 O accumulator could only overflow for
// |V| above ~1e28.  Measured on B200 with k x3 (B1 H16 S16384): at 2^8, 4.2 % of warp-tiles
// after the first took the rescale path and, as a group's P hand-off waits for all four of
// its warps, ~16 % of group-tiles stalled on it (+15 % cycles per launch); at 2^15, none.
constexpr float kRescaleThreshold = 15.0f;
// FMA-pipe exp2 share: 1 of every 8 pairs (measured on B200: 1/8 beat 0/8 by 4-7 % and
// 3/8 by ~4 %; 2/8 is within noise of it).
constexpr int kEmuPairsPer8 = 1;
constexpr int kSumAcc = 8;                     // independent packed row-sum accumulators

constexpr uint32_t kWaitSuspendNs = 200000;   // try_wait suspend hint while draining

// Device status bits (OR-ed into the caller's status word).
constexpr int kStatusWatchdog = 1;  // a pipeline wait exceeded the watchdog; outputs invalid
constexpr int kStatusDrain = 2;     // draining in-flight copies/MMAs exceeded the watchdog

// Shared-memory layout, offsets from a 1024-byte aligned base.
constexpr int kSmemQ = 0;
constexpr int kSmemRing = kSmemQ + kQTiles * kTileBytes;
constexpr int kSmemBars = kSmemRing + kStages * kTileBytes;
enum : int {
  BAR_Q = 0,
  BAR_Q_EMPTY = 1,  // the current item's last S MMAs have read Q
  BAR_KV_FULL = 2,
  BAR_KV_EMPTY = BAR_KV_FULL + kStages,
  BAR_S_FULL = BAR_KV_EMPTY + kStages,
  BAR_O_DONE = BAR_S_FULL + kQTiles,
  BAR_DRAIN = BAR_O_DONE + kQTiles,
  NUM_BARS = BAR_DRAIN + 1
};
constexpr int kSmemTmemSlot = kSmemBars + NUM_BARS * 8;
constexpr int kSmemAbort = kSmemTmemSlot + 4;
// Per softmax warp: its schedule walker's state (4 ints) and current unit (8 ints), kept
// here across a unit's tile loop so they hold no registers there.
constexpr int kSmemWalk = (kSmemAbort + 4 + 15) / 16 * 16;
constexpr int kWalkInts = 16;
constexpr int kSmemUsed = kSmemWalk + 8 * kWalkInts * 4;
constexpr int kSmemBytes = kSmemUsed + 1024;  // slack for the manual 1024-byte alignment
static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");

struct AttnParams {
  sched::Plan plan;             // work units of every CTA (schedule.cuh)
  float* lse;                   // [num_bh, lse_head_stride] natural-log LSE, or null
  int* status;                  // device status word, or null
  long long lse_head_stride;    // elements between consecutive heads of lse
  long long q_pos0;             // sequence position of local query row 0 (mask only)
  long long kv_pos0;            // sequence position of local key row 0 (mask only)
  unsigned long long watchdog_ns;
  int seq_q;
  int seq_kv;
  int num_bh;
  void* o;                      // bf16 output rows, [num_bh, o_head_stride]
  int o_sector_aligned;         // o and o_head_stride * 2 bytes are multiples of 32
  long long o_head_stride;      // elements between consecutive heads of o
  int causal;                   // key position > query position is masked
  float scale_log2;             // softmax_scale * log2(e)
  int test_skip_load;           // test hook: K/V copy index the producer never issues, or -1
  // Split pieces (stream-K plans only; null otherwise).  Per CTA, per segment parity, per
  // Q tile: one slot of 128 rows: unnormalised O (fp32, 16 pieces of 8 values per row,
  // piece-major so that a warp's stores are contiguous), the row max m and sum l, and a
  // flag (1 = the slot holds a continuation piece not yet merged, 0 = free).
  float* part_o;
  float* part_ml;
  int* part_flag;
};

// Scratch of one slot (CTA, segment parity, Q tile).
constexpr int kSlotO = 16 * kBlockM * 8;  // floats
constexpr int kSlotMl = 2 * kBlockM;       // floats
__host__ __device__ constexpr long long slot_index(int cta, int parity, int tile) {
  return (static_cast<long long>(cta) * 2 + parity) * kQTiles + tile;
}

struct Watch {
  volatile int* abort;
  int* status;
  unsigned long long limit_ns;
};

// Waits for completion of phase `parity` of `bar`.  Returns false (and raises the
// CTA abort flag plus the watchdog status bit) if the limit passes first, or at
// once if another thread of the CTA already aborted.
// The clock and the abort flag are read only every 64 probes, so a waiting warp
// spends its issue slots on try_wait alone.
__device__ __forceinline__ bool wait_phase(uint32_t bar, uint32_t parity, const Watch& w) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  while (true) {
#pragma unroll 1
    for (int probe = 0; probe < 64; ++probe)
      if (mbar_try_wait(bar, parity)) return true;
    if (*w.abort) return false;
    if (global_timer_ns() - t0 > w.limit_ns) {
      *w.abort = 1;
      if (w.status != nullptr) atomicOr(w.status, kStatusWatchdog);
      return false;
    }
  }
}

// Bounded wait used only to drain work that is already in flight; ignores the abort flag.
// Its limit never drops below kDrainFloorNs, whatever the pipeline watchdog is set to:
// copies and MMAs in flight land within microseconds, and a CTA must not exit while a
// TMA copy can still write its shared memory.
constexpr unsigned long long kDrainFloorNs = 100000000ull;  // 100 ms
__device__ __forceinline__ void drain_phase(uint32_t bar, uint32_t parity, const Watch& w) {
  const uint64_t t0 = global_timer_ns();
  const unsigned long long limit = w.limit_ns > kDrainFloorNs ? w.limit_ns : kDrainFloorNs;
  while (!mbar_try_wait_sleep(bar, parity, kWaitSuspendNs)) {
    if (global_timer_ns() - t0 > limit) {
      if (w.status != nullptr) atomicOr(w.status, kStatusDrain);
      return;
    }
  }
}

// S = Q K^T for one 128x128 tile: 8 MMAs of K=16 along head_dim.  Both operands are
// K-major, 128B-swizzled, stored as two 64-column halves of 128 rows.
__device__ __forceinline__ void issue_qk(uint32_t d_tmem, uint32_t q_lo, uint32_t k_lo, uint32_t desc_hi) {
  constexpr uint32_t idesc = idesc_bf16_f32(kBlockM, kBlockN, 0, 0);
#pragma unroll
  for (int kk = 0; kk < kHeadDim / 16; ++kk) {
    const uint32_t off = ((kk >> 2) * kHalfBytes + (kk & 3) * 32) >> 4;
    mma_ss_lo(d_tmem, q_lo + off, k_lo + off, desc_hi, idesc, kk > 0 ? 1u : 0u);
  }
}

// O += P V over keys [64*half, 64*half + 64): P (128 rows x keys, bf16) from TMEM,
// V (keys x 128 dims) from shared memory as an MN-major operand: dims contiguous, the
// two 64-dim halves 16 KiB apart (leading byte offset), 8-key groups 1024 B apart
// (stride byte offset); v_lo = smem_desc_lo(V tile, 16 KiB).
__device__ __forceinline__ void issue_pv_half(uint32_t d_tmem, uint32_t p_tmem, uint32_t v_lo, uint32_t desc_hi,
                                              int half, uint32_t accumulate) {
  constexpr uint32_t idesc = idesc_bf16_f32(kBlockM, kHeadDim, 0, 1);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int kk = half * 4 + q;
    mma_ts_lo(d_tmem, p_tmem + kk * 8, v_lo + ((kk * 16 * 128) >> 4), desc_hi, idesc,
              (accumulate | (kk > 0 ? 1u : 0u)));
  }
}

__device__ __forceinline__ float u2f(uint32_t x) { return __uint_as_float(x); }
__device__ __forceinline__ uint32_t f2u(float x) { return __float_as_uint(x); }

// P for 64 keys (two 32-column chunks of S): x = s*scale - m by packed FMA, p = 2^x,
// row sums accumulated in packed pairs, P packed to bf16x2 and stored to TMEM at tP a
// quarter (16 keys, 8 columns) at a time, so only 8 packed registers are ever live.
// kEmuPairsPer8 of every 8 pairs go through the FMA-pipe exp2 (exp2_poly_x2) to
// offload the MUFU unit; the split is fixed at compile time, so the whole half is one
// straight-line block in which MUFU and FMA chains interleave.  A masked (-inf) score
// gives exactly 0 on the MUFU path and 2^-125 on the FMA path: negligible against any
// row that sees a key (the row sum is >= 1), and a row that sees none is zeroed in
// the epilogue.
__device__ __forceinline__ void exp_half(const uint32_t (&sa)[32], const uint32_t (&sb)[32],
                                         uint64_t scale2, uint64_t neg_m2, uint64_t (&sum2)[kSumAcc],
                                         uint32_t tP) {
  uint32_t pk[8];
#pragma unroll
  for (int cc = 0; cc < 2; ++cc) {
    const uint32_t (&sc)[32] = cc == 0 ? sa : sb;
#pragma unroll
    for (int e = 0; e < 32; e += 2) {
      const uint64_t x2 = f2_fma(f2_pack(u2f(sc[e]), u2f(sc[e + 1])), scale2, neg_m2);
      float x0, x1, p0, p1;
      f2_unpack(x2, x0, x1);
      if (((e >> 1) & 7) < kEmuPairsPer8) {
        exp2_poly_x2(f2_pack(fmaxf(x0, -125.f), fmaxf(x1, -125.f)), p0, p1);
      } else {
        p0 = ex2_approx(x0);
        p1 = ex2_approx(x1);
      }
      sum2[(e >> 1) % kSumAcc] = f2_add(sum2[(e >> 1) % kSumAcc], f2_pack(p0, p1));
      pk[(e >> 1) & 7] = pack_bf16x2(p0, p1);
      if (((e >> 1) & 7) == 7) {
        const int q = cc * 16 + (e >> 1) - 7;
        tmem_st8(tP + q, pk[0], pk[1], pk[2], pk[3], pk[4], pk[5], pk[6], pk[7]);
      }
    }
  }
}

// exp_half over keys 0-63 with the row max over all 128 scores (raw, unscaled) folded
// into the same straight-line block: every pair step also folds two score pairs into
// four running maxima, so the independent max3 work fills the gaps between dependent
// MUFU operations.  Measured on B200 with one warp per SM sub-partition: 565 cycles
// for this half in one block, about 840 when a branch split the exps from a separate
// max loop (the scheduler cannot interleave across basic blocks).
__device__ __forceinline__ float exp_half_max(const uint32_t (&s)[4][32], uint64_t scale2, uint64_t neg_m2,
                                              uint64_t (&sum2)[kSumAcc], uint32_t tP) {
  uint32_t pk[8];
  float mx[4];  // four running maxima (eight measured 0.5 % slower: more live registers)
#pragma unroll
  for (int e = 0; e < 4; ++e) mx[e] = -CUDART_INF_F;
#pragma unroll
  for (int q = 0; q < 32; ++q) {
    const int cc = q >> 4, e = (q & 15) * 2;
    const uint64_t x2 = f2_fma(f2_pack(u2f(s[cc][e]), u2f(s[cc][e + 1])), scale2, neg_m2);
    float x0, x1, p0, p1;
    f2_unpack(x2, x0, x1);
    if ((q & 7) < kEmuPairsPer8) {
      exp2_poly_x2(f2_pack(fmaxf(x0, -125.f), fmaxf(x1, -125.f)), p0, p1);
    } else {
      p0 = ex2_approx(x0);
      p1 = ex2_approx(x1);
    }
    sum2[(q & 15) % kSumAcc] = f2_add(sum2[(q & 15) % kSumAcc], f2_pack(p0, p1));
    pk[q & 7] = pack_bf16x2(p0, p1);
    if ((q & 7) == 7) tmem_st8(tP + q - 7, pk[0], pk[1], pk[2], pk[3], pk[4], pk[5], pk[6], pk[7]);
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int pr = 2 * q + r, c = pr >> 4, ee = (pr & 15) * 2;
      mx[pr & 3] = fmax3(mx[pr & 3], u2f(s[c][ee]), u2f(s[c][ee + 1]));
    }
  }
  return fmaxf(fmax3(mx[0], mx[1], mx[2]), mx[3]);
}

// Flags of split-piece slots (cta_lo..cta_hi, parity, tile): poll with acquire semantics
// until each holds `want`, bounded by the watchdog.  Lane k polls CTAs cta_lo + k,
// cta_lo + k + 32, ..., so the polls of all pieces are in flight together.
__device__ __forceinline__ bool wait_flags(const int* flags, int cta_lo, int cta_hi, int parity, int tile, int want,
                                           const Watch& w) {
  bool ok = true;
  for (int c = cta_lo + static_cast<int>(threadIdx.x & 31); ok && c <= cta_hi; c += 32) {
    const int* flag = flags + slot_index(c, parity, tile);
    if (ld_acquire_gpu(flag) == want) continue;
    const uint64_t t0 = global_timer_ns();
    while (true) {
      if (ld_acquire_gpu(flag) == want) break;
      if (*w.abort) { ok = false; break; }
      if (global_timer_ns() - t0 > w.limit_ns) {
        *w.abort = 1;
        if (w.status != nullptr) atomicOr(w.status, kStatusWatchdog);
        ok = false;
        break;
      }
      __nanosleep(64);
    }
  }
  const bool all = __all_sync(0xffffffffu, ok);
  __threadfence();  // every lane's later reads of the slots are ordered after the acquires
  return all;
}

// Online merge of a continuation piece's row (max mc, sum lc) into (m, l), log2 units.
__device__ __forceinline__ void merge_ml(float& m, float& l, float mc, float lc) {
  if (mc == -CUDART_INF_F || !(lc > 0.f)) return;
  const float mn = fmaxf(m, mc);
  l = (m == -CUDART_INF_F ? 0.f : l * ex2_approx(m - mn)) + lc * ex2_approx(mc - mn);
  m = mn;
}

// Persistent: each CTA walks its unit sequence (schedule.cuh).  Every role walks the same
// sequence and derives all mbarrier phases from running counters (tiles, ring positions,
// Q loads), so the pipeline flows from one unit into the next: the producer loads the
// next unit's Q as soon as the current unit's last S MMAs have read Q, and the MMA warp
// computes the next unit's first S tiles while the softmax warpgroups finish the current
// unit's epilogue.
// The kTable plan's item lists ride in the parameter block of their own instantiation, so
// launches of the other plans carry no 25 KB table.
template <bool kWithTable>
struct TableParam {
  int unused;
};
template <>
struct TableParam<true> {
  sched::Table t;
};

template <bool kWithTable>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ AttnParams p,
                    const __grid_constant__ TableParam<kWithTable> tab) {
  const sched::Table* table = nullptr;
  if constexpr (kWithTable) table = &tab.t;
  extern __shared__ uint8_t smem_dyn[];
  const uint32_t raw = smem_addr(smem_dyn);
  uint8_t* smem = smem_dyn + ((1024u - (raw & 1023u)) & 1023u);
  const uint32_t sbase = smem_addr(smem);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  auto bar = [&](int idx) -> uint32_t { return sbase + kSmemBars + idx * 8; };
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kSmemAbort);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kSmemTmemSlot);
  const Watch watch{abort_flag, p.status, p.watchdog_ns};

  if (threadIdx.x == 0) {
    mbar_init(bar(BAR_Q), 1);
    mbar_init(bar(BAR_Q_EMPTY), 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar(BAR_KV_FULL + s), 1);
      mbar_init(bar(BAR_KV_EMPTY + s), 1);
    }
    for (int i = 0; i < kQTiles; ++i) {
      mbar_init(bar(BAR_S_FULL + i), 1);
      mbar_init(bar(BAR_O_DONE + i), 1);
    }
    mbar_init(bar(BAR_DRAIN), 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == kLoadWarp && lane == 0) {
    prefetch_tensormap(&tm_q);
    prefetch_tensormap(&tm_k);
    prefetch_tensormap(&tm_v);
  }
  if (warp == kMmaWarp) {
    tmem_alloc(smem_addr(tmem_slot), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Everything above touches only this CTA's shared memory, TMEM and the parameter block,
  // so it may overlap the previous launch in the stream when the launch allows it; every
  // global-memory access below (the Q/K/V loads, O/LSE stores, status word, workspace)
  // comes after the wait.  The next launch may then start its own set-up on free
  // multiprocessors: this grid is persistent, at most one CTA per multiprocessor, all
  // resident from the start, so nothing of it waits for a multiprocessor.
  grid_dependency_wait();
  grid_launch_dependents();

  const uint32_t sQ = sbase + kSmemQ;
  const uint32_t sRing = sbase + kSmemRing;

  if (warp < 2 * 4) {
    regs_increase<kRegsSoftmax>();
    // ------------------------------------------------------------ softmax warpgroups
    const int i = warp >> 2;          // Q tile of this warpgroup
    const int wq = warp & 3;          // TMEM lane quarter of this warp
    const int t = threadIdx.x & 127;  // row within the Q tile
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    const uint32_t tS = tmem + lane_off + i * kBlockN;
    const uint32_t tO = tmem + lane_off + 2 * kBlockN + i * kHeadDim;
    const float scale = p.scale_log2;
    bool ok = true;
    // ph bit 0: parity of the tiles of earlier units (the S_FULL phase base); bit 1: parity
    // of the earlier units with work (the O_DONE phase).
    uint32_t ph = 0;
    // This warp's walker state and current unit live in shared memory (volatile reads),
    // so the tile loop carries only n_tiles and the two key limits in registers.
    volatile int* wst = reinterpret_cast<volatile int*>(smem + kSmemWalk) + warp * kWalkInts;
    if (lane == 0) {
      wst[0] = 0;
      wst[1] = 0;
      wst[2] = -1;
      wst[3] = 0;
    }
    __syncwarp();
    while (true) {
      int n_tiles, row_keys, warp_keys;
      {
        sched::Walker walk(p.plan, static_cast<int>(blockIdx.x), wst[0], wst[1], wst[2], wst[3], table);
        sched::Unit u;
        const bool more = walk.next(u);
        __syncwarp();
        if (lane == 0) {
          int saved[4];
          walk.save(saved);
          wst[0] = saved[0];
          wst[1] = saved[1];
          wst[2] = saved[2];
          wst[3] = saved[3];
          wst[4] = u.bh;
          wst[5] = u.q0;
          wst[6] = u.t0;
          wst[7] = u.t1;
          wst[8] = u.kind;
          wst[9] = u.seg;
          wst[10] = u.cont_lo;
          wst[11] = u.cont_hi;
        }
        __syncwarp();
        if (!more) break;
        n_tiles = u.t1 - u.t0;
        // Visible keys as local key counts in [0, seq_kv]: this row sees keys [0, row_keys);
        // every row of this warp sees at least the first warp_keys.  Key counts are relative
        // to the unit's first tile.
        row_keys = p.seq_kv;
        warp_keys = p.seq_kv;
        if (p.causal) {
          const long long rk = p.q_pos0 + u.q0 + i * kBlockM + t - p.kv_pos0 + 1;
          const long long wk = p.q_pos0 + u.q0 + i * kBlockM + wq * 32 - p.kv_pos0 + 1;
          row_keys = static_cast<int>(max(0LL, min(static_cast<long long>(p.seq_kv), rk)));
          warp_keys = static_cast<int>(max(0LL, min(static_cast<long long>(p.seq_kv), wk)));
        }
        row_keys -= u.t0 * kBlockN;
        warp_keys -= u.t0 * kBlockN;
      }

      float m = -CUDART_INF_F;  // running max, log2 units (already scaled)
      float l = 0.f;            // running sum of exp2(s*scale - m)

      int j = 0;
      for (; ok && j < n_tiles; ++j) {
        ok = __all_sync(0xffffffffu, wait_phase(bar(BAR_S_FULL + i), (ph ^ j) & 1u, watch));
        if (!ok) break;
        AVO_TRACE_HOOK(i, j, 0);
        tc_fence_after();
        uint32_t s[4][32];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32(tS + c * 32, s[c]);
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_wait_ld(s[c]);
        AVO_TRACE_HOOK(i, j, 1);

        const int key_base = j * kBlockN;
        if (key_base + kBlockN > warp_keys) {  // the tile has keys some row of this warp masks
          const int lim = row_keys - key_base;
#pragma unroll
          for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int e = 0; e < 32; ++e)
              if (c * 32 + e >= lim) s[c][e] = f2u(-CUDART_INF_F);
        }

        // Speculative P for keys 0-63 against the running max, computed side by side
        // with the row max over all 128 scores (independent instruction streams).  The
        // running max only moves when the tile max exceeds it by more than 2^15, so the
        // speculation almost always stands; when it does not (first tile, rare jumps)
        // the half is recomputed with the new max, giving exactly the values a
        // max-first order would.  An overflow of the speculative exp2 implies a move.
        const uint64_t scale2 = f2_pack(scale, scale);
        uint64_t neg_m2 = f2_pack((m == -CUDART_INF_F) ? 0.f : -m, (m == -CUDART_INF_F) ? 0.f : -m);
        uint64_t sum2[kSumAcc];
#pragma unroll
        for (int q = 0; q < kSumAcc; ++q) sum2[q] = f2_pack(0.f, 0.f);
        // P goes to S columns 64-127 (keys 64-127's scores are already in registers, and
        // the rescale path re-reads only columns 0-63), a quarter at a time as computed.
        // Measured on B200: 4-15 % faster than holding 32 packed registers for one store
        // per half into columns 0-63.
        const uint32_t tP = tS + 64;
        const float mt = exp_half_max(s, scale2, neg_m2, sum2, tP);
        const float m_new = fmaxf(m, mt * scale);
        const bool grow = m_new > m + kRescaleThreshold;
        AVO_TRACE_HOOK(i, j, 2);

        if (__any_sync(0xffffffffu, grow)) {
          float factor = 1.f;
          if (grow) {
            factor = ex2_approx(m - m_new);
            l *= factor;
            m = m_new;
          }
          const float neg_m = (m == -CUDART_INF_F) ? 0.f : -m;
          neg_m2 = f2_pack(neg_m, neg_m);
#pragma unroll
          for (int q = 0; q < kSumAcc; ++q) sum2[q] = f2_pack(0.f, 0.f);
          // Scores 0-63 again, from TMEM (S stays intact there until P is stored): then
          // the registers of s[0] and s[1] need not outlive the speculative pass, which
          // is the softmax warps' register peak.
          uint32_t s01[2][32];
          tmem_ld32(tS, s01[0]);
          tmem_ld32(tS + 32, s01[1]);
          tmem_wait_ld(s01[0]);
          tmem_wait_ld(s01[1]);
          if (key_base + kBlockN > warp_keys) {
            const int lim = row_keys - key_base;
#pragma unroll
            for (int c = 0; c < 2; ++c)
#pragma unroll
              for (int e = 0; e < 32; ++e)
                if (c * 32 + e >= lim) s01[c][e] = f2u(-CUDART_INF_F);
          }
          exp_half(s01[0], s01[1], scale2, neg_m2, sum2, tP);
          if (j > 0) {
            // O holds P V summed over tiles < j relative to the old max; rescale this
            // row in TMEM before any part of P_j is published.  Those MMAs are complete:
            // the S_j commit just observed was issued after them by the same thread,
            // and a commit tracks every earlier MMA of its thread.
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              uint32_t o[32];
              tmem_ld32(tO + c * 32, o);
              tmem_wait_ld(o);
#pragma unroll
              for (int e = 0; e < 32; ++e) o[e] = f2u(u2f(o[e]) * factor);
              tmem_st32(tO + c * 32, o);
            }
          }
        }

        // Publish P in two 64-key halves, each as soon as it sits in TMEM, so PV on keys
        // 0-63 overlaps the exps of keys 64-127.  The hand-off is a hardware named
        // barrier the MMA warp syncs on (about 40 cycles, against about 130 for an
        // mbarrier observed by a polling warp).
        tc_wait_st();
        tc_fence_before();
        __syncwarp();
        named_bar_arrive(kBarPHalf + 2 * i + 0, kPHalfThreads);
        exp_half(s[2], s[3], scale2, neg_m2, sum2, tP + 32);
        AVO_TRACE_HOOK(i, j, 3);
        tc_wait_st();
        tc_fence_before();
        __syncwarp();
        named_bar_arrive(kBarPHalf + 2 * i + 1, kPHalfThreads);
#pragma unroll
        for (int q = 1; q < kSumAcc; ++q) sum2[0] = f2_add(sum2[0], sum2[q]);
        float a0, a1;
        f2_unpack(sum2[0], a0, a1);
        l += a0 + a1;
        AVO_TRACE_HOOK(i, j, 4);
      }
      // After a watchdog abort (which can only happen before a tile's first arrival)
      // the MMA warp still runs its whole schedule, so this warp keeps its place in it:
      // one arrival per half for every remaining tile of every remaining item, and the
      // O release of every item.  These are blocking syncs, so an arrival can never run
      // ahead into the next generation of a barrier.
      for (; j < n_tiles; ++j) {
        __syncwarp();
        named_bar_sync(kBarPHalf + 2 * i + 0, kPHalfThreads);
        named_bar_sync(kBarPHalf + 2 * i + 1, kPHalfThreads);
      }


      // Epilogue.  A whole item: O / l -> bf16 -> this thread's output row, written
      // straight from registers as 8 whole 32-byte sectors (16-byte stores when o or its
      // head stride is not 32-byte aligned; rows past seq_q are not written).  The Q
      // buffer is not used for staging: the next unit's Q may already be loading into it.
      // A row that never saw a key keeps m = -inf (its l only holds the FMA-path exp2
      // floor of masked scores): it gets O = 0 and LSE = -inf.  Once a row sees a key, the
      // first rescale multiplies O and l by 2^(-inf) = 0, so no floor survives.
      // A continuation piece of a split item writes its unnormalised O, m and l to this
      // CTA's slot instead; the item's first piece merges those of CTAs cont_lo..cont_hi
      // (m = max over pieces, O and l rescaled by 2^(m_piece - m)) before normalising.
      sched::Unit u;
      u.bh = wst[4];
      u.q0 = wst[5];
      u.kind = wst[8];
      u.seg = wst[9];
      u.cont_lo = wst[10];
      u.cont_hi = wst[11];
      const int parity = u.seg & 1;
      // The slot flags are polled before the wait for O (both only wait; the flag polls
      // are L2 round trips that then overlap the last PV): a first piece needs every
      // continuation piece's slot full, a continuation piece needs its own slot free.
      if (u.kind == sched::kFirst) {
        ok = wait_flags(p.part_flag, u.cont_lo, u.cont_hi, parity, i, 1, watch) && ok;
      } else if (u.kind == sched::kCont) {
        ok = wait_flags(p.part_flag, blockIdx.x, blockIdx.x, parity, i, 0, watch) && ok;
      }
      if (ok && n_tiles > 0) {
        ok = __all_sync(0xffffffffu, wait_phase(bar(BAR_O_DONE + i), (ph >> 1) & 1u, watch));
        tc_fence_after();
      }
      const bool have = ok && n_tiles > 0;
      const int row = u.q0 + i * kBlockM + t;
      const bool write = row < p.seq_q && *abort_flag == 0;
      float m_fin = (have && l > 0.f) ? m : -CUDART_INF_F;
      float l_fin = m_fin == -CUDART_INF_F ? 0.f : l;
      float f_own = 1.f;
      if (u.kind == sched::kFirst && ok) {
        // (m, l) of all pieces merged online, two pieces' loads in flight at a time.
        for (int c = u.cont_lo; c <= u.cont_hi; c += 2) {
          const float* mla = p.part_ml + slot_index(c, parity, i) * kSlotMl;
          const float* mlb = p.part_ml + slot_index(c < u.cont_hi ? c + 1 : c, parity, i) * kSlotMl;
          const float ma = __ldcg(mla + t), la = __ldcg(mla + kBlockM + t);
          const float mb = __ldcg(mlb + t), lb = __ldcg(mlb + kBlockM + t);
          merge_ml(m_fin, l_fin, ma, la);
          if (c < u.cont_hi) merge_ml(m_fin, l_fin, mb, lb);
        }
        f_own = (!(have && l > 0.f) || m_fin == -CUDART_INF_F) ? 0.f : ex2_approx(m - m_fin);
      }
      const bool seen = (m_fin != -CUDART_INF_F) && (l_fin > 0.f);
      const float inv_l = seen ? 1.f / l_fin : 0.f;
      __nv_bfloat16* orow =
          static_cast<__nv_bfloat16*>(p.o) + (static_cast<long long>(u.bh) * p.o_head_stride +
                                              static_cast<long long>(row) * kHeadDim);
      // One 32-column chunk of the output row: O * inv_l -> bf16 -> 64 bytes of the row.
      auto store_row_chunk = [&](int c, const uint32_t (&o)[32]) {
        uint32_t w[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) w[e] = pack_bf16x2(u2f(o[2 * e]) * inv_l, u2f(o[2 * e + 1]) * inv_l);
        if (write && ok && p.o_sector_aligned) {
          st_global_v8(orow + c * 32, w[0], w[1], w[2], w[3], w[4], w[5], w[6], w[7]);
          st_global_v8(orow + c * 32 + 16, w[8], w[9], w[10], w[11], w[12], w[13], w[14], w[15]);
        } else if (write && ok) {
          uint4* o16 = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
          for (int q = 0; q < 4; ++q) o16[q] = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
        }
      };
      auto load_o_chunk = [&](int c, uint32_t (&o)[32]) {
        if (have) {
          tmem_ld32(tO + c * 32, o);
          tmem_wait_ld(o);
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = 0u;
        }
      };
      if (u.kind == sched::kWhole) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          load_o_chunk(c, o);
          store_row_chunk(c, o);
        }
      } else if (u.kind == sched::kCont) {
        float* const cont_o = p.part_o + slot_index(blockIdx.x, parity, i) * kSlotO;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          load_o_chunk(c, o);
          if (ok && *abort_flag == 0) {
#pragma unroll
            for (int q = 0; q < 4; ++q)
              st_global_v8(cont_o + ((c * 4 + q) * kBlockM + t) * 8, o[8 * q], o[8 * q + 1], o[8 * q + 2],
                           o[8 * q + 3], o[8 * q + 4], o[8 * q + 5], o[8 * q + 6], o[8 * q + 7]);
          }
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          load_o_chunk(c, o);
          if (ok) {
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = f2u(u2f(o[e]) * f_own);
            // Two pieces per round trip: each piece's row max and its 32 partial values
            // are loaded together, with no branch between them (a piece whose row saw no
            // key gets factor 0; its slot still holds finite values, zeros).  An odd last
            // piece loads only its own slot (zeros stand in for the second).
            for (int cc = u.cont_lo; cc <= u.cont_hi; cc += 2) {
              const bool two = cc < u.cont_hi;
              const long long sa = slot_index(cc, parity, i);
              const long long sb = slot_index(two ? cc + 1 : cc, parity, i);
              const float ma = __ldcg(p.part_ml + sa * kSlotMl + t);
              const float mb = __ldcg(p.part_ml + sb * kSlotMl + t);
              const float4* src_a = reinterpret_cast<const float4*>(p.part_o + sa * kSlotO);
              const float4* src_b = reinterpret_cast<const float4*>(p.part_o + sb * kSlotO);
              float4 va[8], vb[8];
#pragma unroll
              for (int q = 0; q < 8; ++q) {
                va[q] = __ldcg(src_a + ((c * 4 + (q >> 1)) * kBlockM + t) * 2 + (q & 1));
                vb[q] = two ? __ldcg(src_b + ((c * 4 + (q >> 1)) * kBlockM + t) * 2 + (q & 1))
                            : make_float4(0.f, 0.f, 0.f, 0.f);
              }
              const float fa = ma == -CUDART_INF_F ? 0.f : ex2_approx(ma - m_fin);
              const float fb = (!two || mb == -CUDART_INF_F) ? 0.f : ex2_approx(mb - m_fin);
#pragma unroll
              for (int q = 0; q < 8; ++q) {
                o[4 * q + 0] = f2u(fmaf(vb[q].x, fb, fmaf(va[q].x, fa, u2f(o[4 * q + 0]))));
                o[4 * q + 1] = f2u(fmaf(vb[q].y, fb, fmaf(va[q].y, fa, u2f(o[4 * q + 1]))));
                o[4 * q + 2] = f2u(fmaf(vb[q].z, fb, fmaf(va[q].z, fa, u2f(o[4 * q + 2]))));
                o[4 * q + 3] = f2u(fmaf(vb[q].w, fb, fmaf(va[q].w, fa, u2f(o[4 * q + 3]))));
              }
            }
          }
          store_row_chunk(c, o);
        }
      }
      if (n_tiles > 0) {
        // O_i may now be overwritten by the next unit's first PV.
        tc_fence_before();
        __syncwarp();
        if (ok) {
          named_bar_arrive(kBarOFree + i, kPHalfThreads);
        } else {
          named_bar_sync(kBarOFree + i, kPHalfThreads);
        }
      }
      if (u.kind == sched::kCont) {
        // Row max and sum, then publish the slot once all 128 rows are in it.
        float* ml = p.part_ml + slot_index(blockIdx.x, parity, i) * kSlotMl;
        if (ok && *abort_flag == 0) {
          ml[t] = m_fin;
          ml[kBlockM + t] = l_fin;
        }
        __threadfence();  // this thread's slot writes are visible GPU-wide before the flag
        named_bar_sync(kBarSlot + i, 128);
        if (t == 0 && ok && *abort_flag == 0) st_release_gpu(p.part_flag + slot_index(blockIdx.x, parity, i), 1);
      } else if (u.kind == sched::kFirst) {
        // Every row of this tile has read the continuation pieces: free their slots.
        named_bar_sync(kBarSlot + i, 128);
        if (t == 0 && ok) {
          __threadfence();
          for (int c = u.cont_lo; c <= u.cont_hi; ++c) st_release_gpu(p.part_flag + slot_index(c, parity, i), 0);
        }
      }
      if (p.lse != nullptr && write && ok && u.kind != sched::kCont) {
        const float lse = seen ? (m_fin + log2f(l_fin)) * 0.69314718055994531f : -CUDART_INF_F;
        p.lse[static_cast<long long>(u.bh) * p.lse_head_stride + row] = lse;
      }
      if (n_tiles > 0) ph ^= 2u | static_cast<uint32_t>(n_tiles & 1);
    }
  } else if (warp == kLoadWarp) {
    regs_decrease<kRegsOther>();
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const uint64_t pol_q = policy_evict_first();
      const uint64_t pol_kv = policy_evict_last();
      // Per slot, 2 bits: bit 0 = a copy was issued into it, bit 1 = phase parity of the
      // last one (all the abort drain needs; a register, not an indexed array).
      uint32_t last_copy = 0;
      int tt = 0;       // ring position (load order across items)
      int nq = 0;       // Q loads issued (items with work)
      bool stop = false;
      // No separate L2 prefetch of K/V: measured on B200 it cost 1-2 % here (the prefetch
      // operations share the TMA unit with the loads), the CTAs of a head reading the same
      // tiles close together in time already hit L2.
      sched::Walker walk(p.plan, static_cast<int>(blockIdx.x), table);
      sched::Unit u;
      while (!stop && walk.next(u)) {
        const int n_tiles = u.t1 - u.t0;
        if (n_tiles == 0) continue;
        if (nq > 0) {
          // The previous item's last S MMAs have read Q (committed to Q_EMPTY), and its
          // Q load has landed (as for the K/V slots below: always true unless aborted).
          if (!wait_phase(bar(BAR_Q_EMPTY), (nq - 1) & 1, watch)) break;
          if (!wait_phase(bar(BAR_Q), (nq - 1) & 1, watch)) break;
        }
        if (*abort_flag) break;
        mbar_arrive_expect_tx(bar(BAR_Q), kQTiles * kTileBytes);
        for (int i = 0; i < kQTiles; ++i)
          for (int h = 0; h < 2; ++h)
            tma_load_3d(sQ + i * kTileBytes + h * kHalfBytes, &tm_q, bar(BAR_Q), h * 64, u.q0 + i * kBlockM,
                        u.bh, pol_q);
        ++nq;
        for (int lt = 0; lt < 2 * n_tiles; ++lt, ++tt) {
          const int slot = tt % kStages;
          const int use = tt / kStages;
          if (use > 0) {
            if (!wait_phase(bar(BAR_KV_EMPTY + slot), (use - 1) & 1, watch)) { stop = true; break; }
            // The previous copy into this slot has landed.  Always true once the MMA
            // warp consumed it, except after an abort, when consumption no longer waits
            // for data: this keeps at most one copy per slot in flight, so the drain
            // below can name each slot's outstanding phase exactly.
            if (!wait_phase(bar(BAR_KV_FULL + slot), (use - 1) & 1, watch)) { stop = true; break; }
          }
          if (*abort_flag) { stop = true; break; }
          if (tt == p.test_skip_load) continue;  // test hook: this copy never arrives
          AVO_TRACE_HOOK(3, lt >> 1, lt & 1);
          mbar_arrive_expect_tx(bar(BAR_KV_FULL + slot), kTileBytes);
          const CUtensorMap* tm = (lt & 1) ? &tm_v : &tm_k;
          const int krow = (u.t0 + (lt >> 1)) * kBlockN;
          for (int h = 0; h < 2; ++h)
            tma_load_3d(sRing + slot * kTileBytes + h * kHalfBytes, tm, bar(BAR_KV_FULL + slot), h * 64, krow,
                        u.bh, pol_kv);
          last_copy = (last_copy & ~(3u << (2 * slot))) | ((1u | ((use & 1u) << 1)) << (2 * slot));
        }
      }
      if (*abort_flag) {
        // Copies already issued still land in shared memory: wait for them.  At most
        // one copy per slot is ever in flight (see above), so each slot's outstanding
        // phase is that of the last copy issued into it; likewise the last Q load.
        if (nq > 0) drain_phase(bar(BAR_Q), (nq - 1) & 1, watch);
#pragma unroll
        for (int s = 0; s < kStages; ++s)
          if ((last_copy >> (2 * s)) & 1u) drain_phase(bar(BAR_KV_FULL + s), (last_copy >> (2 * s + 1)) & 1u, watch);
      }
    }
    __syncwarp();
  } else if (warp == kMmaWarp) {
    regs_decrease<kRegsOther>();
    // ------------------------------------------------------------ MMA issuer
    // The whole warp runs the schedule and lane 0 issues.  It never reads shared
    // memory between MMA groups: on sm_100 any such read (an mbarrier wait included)
    // completes only after this thread's queued tcgen05.mma instructions have
    // drained, leaving the tensor pipe idle while it refills.  So it only ever waits
    // on hardware named barriers, which do not drain the queue: the softmax
    // warpgroups release it directly when a P half is in TMEM (and when an item's O
    // has been read out), and the waiter warp, which performs the Q and K/V mbarrier
    // waits, releases it when an operand tile is resident.  Every party takes a fixed
    // number of rounds (a function of the item sequence only), including after a
    // watchdog abort, so none can be left waiting.
    const bool leader = lane == 0;
    const uint32_t tS0 = tmem, tS1 = tmem + kBlockN;
    const uint32_t tP0 = tS0 + 64, tP1 = tS1 + 64;  // P_i: bf16 pairs in S_i's columns 64-127
    const uint32_t tO0 = tmem + 2 * kBlockN, tO1 = tO0 + kHeadDim;
    // Descriptor low words (smem_desc_lo): Q tiles, and ring slot 0 as a K (LBO 16 B) or
    // V (LBO one 64-column half) operand; slot s adds s * kTileBytes / 16.
    const uint32_t desc_hi = kDescHiSw128;
    const uint32_t q0_lo = smem_desc_lo(sQ, 16), q1_lo = smem_desc_lo(sQ + kTileBytes, 16);
    const uint32_t k_lo = smem_desc_lo(sRing, 16), v_lo = smem_desc_lo(sRing, kHalfBytes);
    constexpr uint32_t kSlotLo = kTileBytes >> 4;
    auto released = [&]() {
      __syncwarp();
      named_bar_sync(kBarMmaHandoff, 64);
      tc_fence_after();
    };
    auto p_ready = [&](int tile, int half) {
      __syncwarp();
      named_bar_sync(kBarPHalf + 2 * tile + half, kPHalfThreads);
      tc_fence_after();
    };
    auto o_free = [&](int tile) {
      __syncwarp();
      named_bar_sync(kBarOFree + tile, kPHalfThreads);
      tc_fence_after();
    };
    // Every item loads 2 * n_tiles operands into the 4-slot ring, so each item's first K
    // sits in slot 0 or 2: ring phase b.  Tile jj = j + b of an item then reads V from
    // slot (2 jj + 1) % 4 and the next K from (2 jj + 2) % 4, exactly as if the item
    // started the ring; the indices are a function of the loop counter alone, which
    // keeps the issue code between barrier and MMA minimal.
    int b = 0;
    bool any = false;  // a unit with work came before (its O must be released first)
    sched::Walker walk(p.plan, static_cast<int>(blockIdx.x), table);
    sched::Unit u;
    while (walk.next(u)) {
      const int n_tiles = u.t1 - u.t0;
      if (n_tiles == 0) continue;
      released();  // Q and K_0 of this item resident
      if (leader) {
        const uint32_t k0 = k_lo + 2 * b * kSlotLo;
        issue_qk(tS0, q0_lo, k0, desc_hi);
        mma_commit(bar(BAR_S_FULL + 0));
        issue_qk(tS1, q1_lo, k0, desc_hi);
        mma_commit(bar(BAR_S_FULL + 1));
        mma_commit(bar(BAR_KV_EMPTY + 2 * b));
        if (n_tiles == 1) mma_commit(bar(BAR_Q_EMPTY));
      }
      // Tile jj: PV for both Q tiles, and (kMore) the next tile's S as early as its P
      // half allows.  The first tile of an item (kFirst) overwrites O, so it first waits
      // until the previous item's epilogue has read O out.  First and last tiles are
      // peeled off the loop, so the steady-state body carries no test at all.
      auto tile = [&](int jj, auto first_tag, auto more_tag) {
        constexpr bool kFirst = decltype(first_tag)::value;
        constexpr bool kMore = decltype(more_tag)::value;
        const uint32_t vj = v_lo + ((2 * jj + 1) % kStages) * kSlotLo;
        const uint32_t kj = k_lo + ((2 * jj + 2) % kStages) * kSlotLo;
        released();  // V_j resident
        if (kFirst && any) o_free(0);
        p_ready(0, 0);
        if (leader) issue_pv_half(tO0, tP0, vj, desc_hi, 0, kFirst ? 0u : 1u);
        if (kMore) released();  // K_{j+1} resident (taken here, off the P0 -> S0 path)
        p_ready(0, 1);
        if (leader) {
          issue_pv_half(tO0, tP0, vj, desc_hi, 1, 1u);
          if (!kMore) mma_commit(bar(BAR_O_DONE + 0));  // the item's O_0 is complete
          if (kMore) {
            issue_qk(tS0, q0_lo, kj, desc_hi);
            mma_commit(bar(BAR_S_FULL + 0));
          }
        }
        if (kFirst && any) o_free(1);
        p_ready(1, 0);
        if (leader) issue_pv_half(tO1, tP1, vj, desc_hi, 0, kFirst ? 0u : 1u);
        p_ready(1, 1);
        if (leader) {
          issue_pv_half(tO1, tP1, vj, desc_hi, 1, 1u);
          if (!kMore) mma_commit(bar(BAR_O_DONE + 1));
          mma_commit(bar(BAR_KV_EMPTY + (2 * jj + 1) % kStages));
          if (kMore) {
            issue_qk(tS1, q1_lo, kj, desc_hi);
            mma_commit(bar(BAR_S_FULL + 1));
            mma_commit(bar(BAR_KV_EMPTY + (2 * jj + 2) % kStages));
          }
        }
      };
      using True = std::true_type;
      using False = std::false_type;
      if (n_tiles == 1) {
        tile(b, True{}, False{});
      } else {
        tile(b, True{}, True{});
        for (int jj = b + 1; jj < b + n_tiles - 1; ++jj) tile(jj, False{}, True{});
        // Every S of this item has been issued: Q may be reloaded once they complete.
        if (leader) mma_commit(bar(BAR_Q_EMPTY));
        tile(b + n_tiles - 1, False{}, False{});
      }
      b ^= n_tiles & 1;
      any = true;
    }
    if (any) {
      // The last item's O release (keeps the named barrier counts equal).
      o_free(0);
      o_free(1);
    }
    __syncwarp();
    if (leader && any) {
      // Every MMA issued above completes before TMEM and shared memory are released.
      mma_commit(bar(BAR_DRAIN));
      drain_phase(bar(BAR_DRAIN), 0, watch);
    }
    __syncwarp();
  } else if (warp == kWaitWarp) {
    regs_decrease<kRegsOther>();
    // ------------------------------------------------------------ waiter
    // Performs, in the MMA warp's consumption order, the Q and K/V mbarrier waits that
    // gate its MMA groups and releases it for each (see above): per item Q and K_0,
    // then per tile V_j and, if another tile follows, K_{j+1}.  After an abort its
    // waits return at once and it only keeps the round count.
    auto release = [&]() {
      __syncwarp();
      named_bar_sync(kBarMmaHandoff, 64);
    };
    int tt = 0;
    int nq = 0;
    sched::Walker walk(p.plan, static_cast<int>(blockIdx.x), table);
    sched::Unit u;
    while (walk.next(u)) {
      const int n_tiles = u.t1 - u.t0;
      if (n_tiles == 0) continue;
      if (lane == 0) {
        wait_phase(bar(BAR_Q), nq & 1, watch);
        wait_phase(bar(BAR_KV_FULL + tt % kStages), (tt / kStages) & 1, watch);
      }
      ++nq;
      ++tt;
      release();
      for (int j = 0; j < n_tiles; ++j) {
        if (lane == 0) wait_phase(bar(BAR_KV_FULL + tt % kStages), (tt / kStages) & 1, watch);
        ++tt;
        if (lane == 0) AVO_TRACE_HOOK(2, j, 5);
        release();
        if (j + 1 < n_tiles) {
          if (lane == 0) wait_phase(bar(BAR_KV_FULL + tt % kStages), (tt / kStages) & 1, watch);
          ++tt;
          if (lane == 0) AVO_TRACE_HOOK(2, j, 2);
          release();
        }
      }
    }
    __syncwarp();
  } else {
    regs_decrease<kRegsOther>();  // warp 11 completes the load/MMA/waiter warpgroup
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace avo_b200
