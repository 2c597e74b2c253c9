// Work schedule of the persistent attention kernel: which (head, query block, key/value
// tile range) units each CTA processes, in which order.  Compiled for host and device,
// so the host can enumerate exactly what the kernel will do (tests check coverage and
// balance on the CPU) and every role of the kernel walks the same sequence.
//
// A work item is 256 query rows (two 128-row Q tiles) of one (batch, head) pair; it
// needs n KV tiles of 128 keys.  A unit is an item restricted to KV tiles [t0, t1).
// Two plans:
//
//   kWaves   every item whole, CTA c takes one item per wave of `grid` items, walking
//            the waves in alternating directions.  Causal items are ordered longest
//            first over all heads (balances the decreasing lengths within ~2 %).
//   kTail    non-causal: the first F full waves as above, then the remaining R < grid
//            items ("the tail") as one stream-K segment: their tiles, concatenated in
//            item order, are cut into equal runs, one per CTA.  Used when whole items
//            would leave a large share of the SMs idle in the last wave (few items per
//            SM, e.g. one head shard of a problem split over 8 GPUs).
//
// In a stream-K segment an item can be cut between consecutive CTAs.  CTA c's run may
// start inside an item (a continuation piece, written as an unnormalised partial to the
// CTA's scratch slot) and may end inside one (the item's first piece, whose CTA waits
// for the continuation pieces of CTAs c+1.. and merges them by log-sum-exp).  A
// continuation piece is always the first unit of its CTA's run and a first piece the
// last, so the merging CTA waits only for work its neighbours did at the start of their
// runs.
#pragma once


namespace avo_b200 {
namespace sched {

constexpr int kWaves = 0;
constexpr int kTail = 1;

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

// Segment geometry.  Segment s of a plan: its first item, its item count, its total tiles
// and the run length per CTA.
struct Segment {
  int kind;            // 0 waves, 1 stream-K
  int first;           // first item
  int count;           // items
  long long tiles;     // stream-K: total tiles
  long long run;       // stream-K: tiles per CTA run, ceil(tiles / grid)
};

__host__ __device__ inline int num_segments(const Plan& p) { return p.mode == kWaves ? 1 : 2; }

__host__ __device__ inline Segment segment(const Plan& p, int s) {
  Segment g{0, 0, 0, 0, 0};
  if (p.mode == kWaves) {
    g.kind = 0;
    g.count = p.num_bh * p.nq;
    return g;
  }
  if (s == 0) {
    g.kind = 0;
    g.count = p.wave_items;
    return g;
  }
  g.kind = 1;
  g.first = p.wave_items;
  g.count = p.num_bh * p.nq - p.wave_items;
  g.tiles = static_cast<long long>(g.count) * p.n_kv;
  g.run = (g.tiles + p.grid - 1) / p.grid;
  if (g.run < p.run_min) g.run = p.run_min;
  return g;
}

// Locates global tile `pos` of stream-K segment g: the item (bh, q0), the item's tile
// count n, and the tile index t within the item.
__host__ __device__ inline void locate(const Plan& p, const Segment& g, int pos, int& bh, int& q0, int& n,
                                       int& t) {
  const int w = g.first + pos / p.n_kv;
  t = pos % p.n_kv;
  bh = w / p.nq;
  q0 = (w % p.nq) * kRowsPerItem;
  n = p.n_kv;
}

// Chooses the plan of a launch.  `split_ok`: the caller provided scratch for split pieces
// and the launch can hold all CTAs resident at once (a cooperative launch); without it
// every item stays whole (kWaves).  `sms`: multiprocessors, one CTA each.
inline Plan make_plan(int num_bh, int seq_q, int seq_kv, int causal, long long q_pos0, long long kv_pos0, int sms,
                      bool split_ok) {
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
  if (!p.causal && static_cast<long long>(items) * p.n_kv <= 0x7fffffffll) {
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
  // Causal: whole items, longest first over all heads (balanced within ~2 % on the causal
  // workloads).  Head-grouped stream-K plans for causal work were measured on B200 and ran
  // 20-27 % slower: runs over a pair's first q blocks hold many 2-6 tile units, whose fixed
  // per-unit costs the tile balance does not see.
  return p;
}

// The unit sequence of one CTA.  Usage: Walker w(plan, cta); Unit u; while (w.next(u)) ...
// Units of zero tiles (causal blocks that see no key) are produced too (whole items with
// t1 == t0 == 0): the kernel writes their rows as empty.
class Walker {
 public:
  // `p` must outlive the walker (the kernel's parameter block).
  __host__ __device__ Walker(const Plan& p, int cta) : p_(p), cta_(cta), s_(0), r_(0), pos_(-1), end_(0) {}
  // Resumes from a state saved with save() (the softmax warps keep it in shared memory
  // across a unit's tile loop rather than in registers).
  __host__ __device__ Walker(const Plan& p, int cta, int s, int r, int pos, int end)
      : p_(p), cta_(cta), s_(s), r_(r), pos_(pos), end_(end) {}
  __host__ __device__ void save(int* out) const {
    out[0] = s_;
    out[1] = r_;
    out[2] = pos_;
    out[3] = end_;
  }

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
          const long long start = static_cast<long long>(cta_) * g.run;
          const long long stop = start + g.run < g.tiles ? start + g.run : g.tiles;
          pos_ = static_cast<int>(start < g.tiles ? start : g.tiles);
          end_ = static_cast<int>(stop);
        }
        if (pos_ < end_) {
          int n, t;
          locate(p_, g, pos_, u.bh, u.q0, n, t);
          const int item_start = pos_ - t;
          const int item_end = item_start + n;
          const int stop = end_ < item_end ? end_ : item_end;
          u.t0 = t;
          u.t1 = t + (stop - pos_);
          u.seg = s_ - 1;
          u.cont_lo = u.cont_hi = -1;
          if (u.t0 > 0) {
            u.kind = kCont;
          } else if (u.t1 < n) {
            u.kind = kFirst;
            u.cont_lo = cta_ + 1;
            u.cont_hi = static_cast<int>((item_end - 1) / g.run);  // run > 0 in a stream-K segment
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
  int pos_;   // tiles of a segment fit in int: the host refuses larger launches
  int end_;
};

}  // namespace sched
}  // namespace avo_b200
