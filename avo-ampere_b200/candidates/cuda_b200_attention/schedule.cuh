// Work schedule of the persistent attention kernel: which (head, query block, key/value
// tile range) units each CTA processes, in which order.  Compiled for host and device,
// so the host can enumerate exactly what the kernel will do (tests check coverage and
// balance on the CPU) and every role of the kernel walks the same sequence.
//
// A work item is 256 query rows (two 128-row Q tiles) of one (batch, head) pair; it
// needs n KV tiles of 128 keys.  A unit is an item restricted to KV tiles [t0, t1).
// Three plans:
//
//   kWaves   every item whole, CTA c takes one item per wave of `grid` items, walking
//            the waves in alternating directions.  Causal items are ordered longest
//            first over all heads (balances the decreasing lengths).
//   kTail    non-causal: the first F full waves as above, then the remaining R < grid
//            items ("the tail") as one stream-K segment: their tiles, concatenated in
//            item order, are cut into `grid` equal runs, one per CTA.  Used when whole
//            items would leave a large share of the SMs idle in the last wave (few items
//            per SM, e.g. one head shard of a problem split over 8 GPUs).
//   kGroups  causal (same query and key positions): heads are taken in groups of
//            `group_pairs` (batch, head) pairs whose K/V fit comfortably in L2, and each
//            group is one stream-K segment, q blocks ascending within each pair.  Every
//            CTA gets the same number of tiles per group whatever the item lengths, and
//            the CTAs work on one group's K/V at a time.
//
// In a stream-K segment an item can be cut between consecutive CTAs.  CTA c's run may
// start inside an item (a continuation piece, written as an unnormalised partial to the
// CTA's scratch slot) and may end inside one (the item's first piece, whose CTA waits
// for the continuation pieces of CTAs c+1.. and merges them by log-sum-exp).  A
// continuation piece is always the first unit of its CTA's run and a first piece the
// last, so the merging CTA waits only for work its neighbours did at the start of their
// runs.
#pragma once

#include <cmath>

namespace avo_b200 {
namespace sched {

constexpr int kWaves = 0;
constexpr int kTail = 1;
constexpr int kGroups = 2;

constexpr int kWhole = 0;
constexpr int kFirst = 1;  // first piece of a split item: merges the continuation pieces
constexpr int kCont = 2;   // continuation piece: partial O, m, l to this CTA's slot

constexpr int kRowsPerItem = 256;
constexpr int kTileKeys = 128;

struct Plan {
  int mode;
  int grid;            // CTAs
  int num_bh;          // (batch, head) pairs
  int nq;              // query blocks per pair, ceil(seq_q / 256)
  int n_kv;            // KV tiles of the whole key range, ceil(seq_kv / 128)
  int causal;
  long long q_pos0;    // sequence positions (causal mask of the block entry point)
  long long kv_pos0;
  int seq_q;
  int wave_items;      // kTail: items [0, wave_items) go in whole-item waves
  int group_pairs;     // kGroups: pairs per group
  int pair_tiles;      // kGroups: KV tiles of one pair's items together
  int run_min;         // stream-K: shortest run per CTA (bounds the pieces of one item)
};

struct Unit {
  int bh, q0;
  int t0, t1;          // KV tiles [t0, t1) of the item
  int kind;            // kWhole, kFirst or kCont
  int seg;             // stream-K segment index (slot parity), -1 in a wave segment
  int cont_lo, cont_hi;  // kFirst: CTAs holding the continuation pieces
};

// KV tiles of item (pair, q block qb) in the plan's causal or non-causal geometry.
__host__ __device__ inline int item_tiles(const Plan& p, int q0) {
  if (!p.causal) return p.n_kv;
  const int q_end = q0 + kRowsPerItem < p.seq_q ? q0 + kRowsPerItem : p.seq_q;
  const long long lim = p.q_pos0 + q_end - 1 - p.kv_pos0;  // last local key any row may see
  if (lim < 0) return 0;
  const long long n = lim / kTileKeys + 1;
  return n < p.n_kv ? static_cast<int>(n) : p.n_kv;
}

// Item w of a wave segment (the order of the all-waves plan).
__host__ __device__ inline void wave_order_item(const Plan& p, int w, int& bh, int& q0) {
  int qb;
  if (p.causal) {
    qb = p.nq - 1 - w / p.num_bh;
    bh = w % p.num_bh;
  } else {
    bh = w / p.nq;
    qb = w % p.nq;
  }
  q0 = qb * kRowsPerItem;
}

// Item of CTA `cta` in wave r: alternating directions.
__host__ __device__ inline int wave_item(int r, int cta, int grid) {
  return r * grid + ((r & 1) ? grid - 1 - cta : cta);
}

// Tiles before q block qb of a pair in the kGroups geometry (standard causal: query and
// key positions equal, so block qb sees min(2 qb + 2, n_kv) tiles and only the last
// block can be clipped): qb (qb + 1).
__host__ __device__ inline long long group_prefix(int qb) { return static_cast<long long>(qb) * (qb + 1); }

// q block holding tile offset `rem` of a pair (kGroups).
__host__ __device__ inline int group_qb(const Plan& p, long long rem) {
  // largest qb with qb (qb + 1) <= rem, at most nq - 1
  int qb = static_cast<int>((sqrtf(4.0f * static_cast<float>(rem) + 1.0f) - 1.0f) * 0.5f);
  while (qb > 0 && group_prefix(qb) > rem) --qb;
  while (qb + 1 < p.nq && group_prefix(qb + 1) <= rem) ++qb;
  return qb < p.nq - 1 ? qb : p.nq - 1;
}

// Segment geometry.  Segment s of a plan: its first item index (kTail) or pair (kGroups),
// its total tiles, and the run length per CTA.
struct Segment {
  int kind;            // 0 waves, 1 stream-K
  int first;           // kTail: first item; kGroups: first pair
  int count;           // items (kTail) or pairs (kGroups)
  long long tiles;     // stream-K: total tiles
  long long run;       // stream-K: tiles per CTA run, ceil(tiles / grid)
};

__host__ __device__ inline int num_segments(const Plan& p) {
  if (p.mode == kWaves) return 1;
  if (p.mode == kTail) return 2;
  return (p.num_bh + p.group_pairs - 1) / p.group_pairs;
}

__host__ __device__ inline Segment segment(const Plan& p, int s) {
  Segment g{0, 0, 0, 0, 0};
  if (p.mode == kWaves) {
    g.kind = 0;
    g.count = p.num_bh * p.nq;
    return g;
  }
  if (p.mode == kTail) {
    if (s == 0) {
      g.kind = 0;
      g.count = p.wave_items;
      return g;
    }
    g.kind = 1;
    g.first = p.wave_items;
    g.count = p.num_bh * p.nq - p.wave_items;
    g.tiles = static_cast<long long>(g.count) * p.n_kv;
  } else {
    g.kind = 1;
    g.first = s * p.group_pairs;
    g.count = p.num_bh - g.first < p.group_pairs ? p.num_bh - g.first : p.group_pairs;
    g.tiles = static_cast<long long>(g.count) * p.pair_tiles;
  }
  g.run = (g.tiles + p.grid - 1) / p.grid;
  if (g.run < p.run_min) g.run = p.run_min;
  return g;
}

// Locates global tile `pos` of stream-K segment g: the item (bh, q0), the item's tile
// count n, and the tile index t within the item.
__host__ __device__ inline void locate(const Plan& p, const Segment& g, long long pos, int& bh, int& q0,
                                       int& n, int& t) {
  if (p.mode == kTail) {
    const int w = g.first + static_cast<int>(pos / p.n_kv);
    t = static_cast<int>(pos % p.n_kv);
    bh = w / p.nq;
    q0 = (w % p.nq) * kRowsPerItem;
    n = p.n_kv;
  } else {
    bh = g.first + static_cast<int>(pos / p.pair_tiles);
    const long long rem = pos % p.pair_tiles;
    const int qb = group_qb(p, rem);
    q0 = qb * kRowsPerItem;
    t = static_cast<int>(rem - group_prefix(qb));
    n = item_tiles(p, q0);
  }
}

// Chooses the plan of a launch.  `split_ok`: the caller provided scratch for split pieces
// and the launch can hold all CTAs resident at once (a cooperative launch); without it
// every item stays whole (kWaves).  `sms`: multiprocessors, one CTA each.
inline Plan make_plan(int num_bh, int seq_q, int seq_kv, int causal, long long q_pos0, long long kv_pos0, int sms,
                      bool split_ok, long long kv_group_budget_bytes = 48ll << 20) {
  Plan p{};
  p.mode = kWaves;
  p.num_bh = num_bh;
  p.nq = (seq_q + kRowsPerItem - 1) / kRowsPerItem;
  p.n_kv = (seq_kv + kTileKeys - 1) / kTileKeys;
  p.causal = causal ? 1 : 0;
  p.q_pos0 = q_pos0;
  p.kv_pos0 = kv_pos0;
  p.seq_q = seq_q;
  const long long items = static_cast<long long>(num_bh) * p.nq;
  p.grid = static_cast<int>(items < sms ? items : sms);
  p.run_min = 1;
  if (!split_ok || items == 0 || p.n_kv == 0 || sms <= 1) return p;
  const int run_min = (p.n_kv + 3) / 4 > 4 ? (p.n_kv + 3) / 4 : 4;
  if (!p.causal) {
    // Whole items: F full waves and a last wave of R items, (F + 1) * T tiles per CTA at
    // most.  Split: the R tail items' tiles spread evenly.  Take the split when it saves
    // at least 3 % (a split piece costs about two tiles of extra epilogue work).
    const long long T = p.n_kv;
    const long long F = items / sms, R = items - F * sms;
    if (R == 0) return p;
    long long run = (R * T + sms - 1) / sms;
    if (run < run_min) run = run_min;
    const long long whole = (F + 1) * T, split = F * T + run + 2;
    if ((whole - split) * 100 < 3 * whole) return p;
    p.mode = kTail;
    p.wave_items = static_cast<int>(F * sms);
    p.run_min = run_min;
    p.grid = F > 0 ? sms : static_cast<int>((R * T + run - 1) / run);
    return p;
  }
  if (q_pos0 != kv_pos0 || seq_q != seq_kv || items < 2ll * sms) return p;
  const long long pair_kv = static_cast<long long>(seq_kv) * 128 * 2 * 2;
  long long g = kv_group_budget_bytes / pair_kv;
  if (g < 1) g = 1;
  if (g > num_bh) g = num_bh;
  p.mode = kGroups;
  p.group_pairs = static_cast<int>(g);
  p.pair_tiles = (p.nq - 1) * p.nq + (2 * p.nq < p.n_kv ? 2 * p.nq : p.n_kv);
  p.run_min = run_min;
  p.grid = sms;
  return p;
}

// The unit sequence of one CTA.  Usage: Walker w(plan, cta); Unit u; while (w.next(u)) ...
// Units of zero tiles (causal blocks that see no key) are produced too (whole items with
// t1 == t0 == 0): the kernel writes their rows as empty.
class Walker {
 public:
  // `p` must outlive the walker (the kernel's parameter block).
  __host__ __device__ Walker(const Plan& p, int cta) : p_(p), cta_(cta), s_(0), r_(0), pos_(-1), end_(0) {}

  __host__ __device__ bool next(Unit& u) {
    const int nseg = num_segments(p_);
    while (s_ < nseg) {
      const Segment g = segment(p_, s_);
      if (g.kind == 0) {
        while (static_cast<long long>(r_) * p_.grid < g.count) {
          const int w = wave_item(r_, cta_, p_.grid);
          ++r_;
          if (w >= g.count) continue;
          wave_order_item(p_, w, u.bh, u.q0);
          u.t0 = 0;
          u.t1 = item_tiles(p_, u.q0);
          u.kind = kWhole;
          u.seg = -1;
          u.cont_lo = u.cont_hi = -1;
          return true;
        }
      } else {
        if (pos_ < 0) {
          pos_ = static_cast<long long>(cta_) * g.run;
          end_ = pos_ + g.run < g.tiles ? pos_ + g.run : g.tiles;
        }
        if (pos_ < end_) {
          int n, t;
          locate(p_, g, pos_, u.bh, u.q0, n, t);
          const long long item_start = pos_ - t;
          const long long item_end = item_start + n;
          const long long stop = end_ < item_end ? end_ : item_end;
          u.t0 = t;
          u.t1 = t + static_cast<int>(stop - pos_);
          u.seg = s_ - (p_.mode == kTail ? 1 : 0);
          u.cont_lo = u.cont_hi = -1;
          if (u.t0 > 0) {
            u.kind = kCont;
          } else if (u.t1 < n) {
            u.kind = kFirst;
            u.cont_lo = cta_ + 1;
            u.cont_hi = static_cast<int>((item_end - 1) / g.run);
          } else {
            u.kind = kWhole;
          }
          pos_ = stop;
          return true;
        }
      }
      ++s_;
      r_ = 0;
      pos_ = -1;
    }
    return false;
  }

 private:
  const Plan& p_;
  int cta_;
  int s_;
  int r_;
  long long pos_;
  long long end_;
};

}  // namespace sched
}  // namespace avo_b200
