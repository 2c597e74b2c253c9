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
//            first over all heads (balances the decreasing lengths within ~2 %).
//   kTail    non-causal: the first F full waves as above, then the remaining R < grid
//            items ("the tail") as one stream-K segment: their tiles, concatenated in
//            item order, are cut into equal runs, one per CTA.  Used when whole items
//            would leave a large share of the SMs idle in the last wave (few items per
//            SM, e.g. one head shard of a problem split over 8 GPUs).
//   kTable   causal, many items: whole items, greedy list scheduling (each item to the
//            CTA with the least work so far) over an order that takes the (batch, head)
//            pairs in groups whose K/V fit in L2 and, within a group, the longest query
//            blocks first.  The CTAs stay as balanced as with kWaves while the K/V read at
//            any moment belong to one or two groups instead of every pair.  The host
//            computes each CTA's item list; it travels in the kernel's parameter block.
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
constexpr int kTable = 2;

// kTable's item lists: CTA c takes items item[start[c] .. start[c + 1]) in order, each an
// index into the grouped order (decode_grouped).  25 KB, within the 32 KB a kernel
// parameter block may hold.
constexpr int kTableCtas = 160;
constexpr int kTableItems = 12288;
struct Table {
  unsigned short start[kTableCtas + 1];
  unsigned short item[kTableItems];
};

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
  int group_pairs;     // kTable: pairs per group of the grouped order
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

// Item k of kTable's grouped order: groups of group_pairs pairs (the last one may be
// smaller), within a group query blocks from the last down, pairs within a block.
__host__ __device__ inline void decode_grouped(const Plan& p, int k, int& bh, int& q0) {
  const int g = p.group_pairs;
  const int full = p.num_bh / g;
  const int per_group = g * p.nq;
  int first_pair, size, r;
  if (k < full * per_group) {
    first_pair = (k / per_group) * g;
    size = g;
    r = k % per_group;
  } else {
    first_pair = full * g;
    size = p.num_bh - first_pair;
    r = k - full * per_group;
  }
  bh = first_pair + r % size;
  q0 = (p.nq - 1 - r / size) * kRowsPerItem;
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

__host__ __device__ inline int num_segments(const Plan& p) { return p.mode == kTail ? 2 : 1; }

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
// kTable's lists for group size g: greedy list scheduling of the grouped order, each
// item's cost its tile count plus one tile of fixed per-item work.  Returns the largest
// CTA load; fills `t` if non-null.
inline long long build_table(const Plan& p, int g, Table* t) {
  Plan q = p;
  q.group_pairs = g;
  const int items = p.num_bh * p.nq;
  // Binary min-heap of (load, CTA), ties to the lower CTA index.
  long long hl[kTableCtas];
  int hc[kTableCtas];
  int count[kTableCtas];
  int n = p.grid;
  for (int c = 0; c < n; ++c) {
    hl[c] = 0;
    hc[c] = c;
    count[c] = 0;
  }
  auto less = [&](int a, int b) { return hl[a] < hl[b] || (hl[a] == hl[b] && hc[a] < hc[b]); };
  auto swap_at = [&](int a, int b) {
    const long long l = hl[a];
    hl[a] = hl[b];
    hl[b] = l;
    const int c = hc[a];
    hc[a] = hc[b];
    hc[b] = c;
  };
  static thread_local unsigned short owner[kTableItems];
  for (int k = 0; k < items; ++k) {
    int bh, q0;
    decode_grouped(q, k, bh, q0);
    const int cta = hc[0];
    owner[k] = static_cast<unsigned short>(cta);
    ++count[cta];
    hl[0] += item_tiles(q, q0) + 1;
    for (int i = 0;;) {  // sift down
      const int a = 2 * i + 1, b = a + 1;
      int m = i;
      if (a < n && less(a, m)) m = a;
      if (b < n && less(b, m)) m = b;
      if (m == i) break;
      swap_at(i, m);
      i = m;
    }
  }
  long long worst = 0;
  for (int c = 0; c < n; ++c) worst = hl[c] > worst ? hl[c] : worst;
  if (t != nullptr) {
    t->start[0] = 0;
    for (int c = 0; c < n; ++c) t->start[c + 1] = static_cast<unsigned short>(t->start[c] + count[c]);
    int fill[kTableCtas];
    for (int c = 0; c < n; ++c) fill[c] = t->start[c];
    for (int k = 0; k < items; ++k) t->item[fill[owner[k]]++] = static_cast<unsigned short>(k);
  }
  return worst;
}

inline Plan make_plan(int num_bh, int seq_q, int seq_kv, int causal, long long q_pos0, long long kv_pos0, int sms,
                      bool split_ok, Table* table = nullptr) {
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
  // Causal: whole items.  With a workspace (split_ok, checked above: launches without one
  // keep the longest-first waves), room for kTable's lists and at least two items per SM,
  // the grouped greedy plan: the smallest group whose pairs' K/V fit in 48 MB among those
  // within 2 % of the best makespan over all group sizes; otherwise longest first over all
  // heads in waves (within ~2 % of the mean tile count per CTA on the causal workloads).
  // Head-grouped stream-K plans for causal work were measured on B200 and ran 20-27 %
  // slower: runs over a pair's first q blocks hold many 2-6 tile units, whose fixed
  // per-unit costs the tile balance does not see.
  if (table == nullptr || items < 2ll * sms || items > kTableItems || sms > kTableCtas) return p;
  const long long pair_kv = static_cast<long long>(seq_kv) * 128 * 2 * 2;
  const int candidates[] = {num_bh, 32, 24, 16, 12, 8, 6, 4, 3, 2, 1};
  long long best = -1;
  long long span[11];
  for (int i = 0; i < 11; ++i) {
    span[i] = -1;
    if (candidates[i] > num_bh || (i > 0 && candidates[i] == num_bh)) continue;
    span[i] = build_table(p, candidates[i], nullptr);
    if (best < 0 || span[i] < best) best = span[i];
  }
  int chosen = num_bh;
  long long chosen_ws = -1;
  for (int i = 0; i < 11; ++i) {
    if (span[i] < 0 || span[i] * 100 > best * 102) continue;
    const long long ws = candidates[i] * pair_kv;
    const bool fits = ws <= (48ll << 20);
    const bool chosen_fits = chosen_ws >= 0 && chosen_ws <= (48ll << 20);
    if (chosen_ws < 0 || (fits && !chosen_fits) || (fits == chosen_fits && ws < chosen_ws)) {
      chosen = candidates[i];
      chosen_ws = ws;
    }
  }
  p.mode = kTable;
  p.group_pairs = chosen;
  build_table(p, chosen, table);
  return p;
}

// The unit sequence of one CTA.  Usage: Walker w(plan, cta); Unit u; while (w.next(u)) ...
// Units of zero tiles (causal blocks that see no key) are produced too (whole items with
// t1 == t0 == 0): the kernel writes their rows as empty.
class Walker {
 public:
  // `p` (and `t`, kTable's item lists, null for the other plans) must outlive the walker:
  // in the kernel both are in the parameter block.
  __host__ __device__ Walker(const Plan& p, int cta, const Table* t = nullptr)
      : p_(p), t_(t), cta_(cta), s_(0), r_(0), pos_(-1), end_(0) {}
  // Resumes from a state saved with save() (the softmax warps keep it in shared memory
  // across a unit's tile loop rather than in registers).
  __host__ __device__ Walker(const Plan& p, int cta, int s, int r, int pos, int end, const Table* t = nullptr)
      : p_(p), t_(t), cta_(cta), s_(s), r_(r), pos_(pos), end_(end) {}
  __host__ __device__ void save(int* out) const {
    out[0] = s_;
    out[1] = r_;
    out[2] = pos_;
    out[3] = end_;
  }

  __host__ __device__ bool next(Unit& u) {
    if (p_.mode == kTable) {
      if (pos_ < 0) {
        pos_ = t_->start[cta_];
        end_ = t_->start[cta_ + 1];
      }
      if (pos_ >= end_) return false;
      decode_grouped(p_, t_->item[pos_++], u.bh, u.q0);
      u.t0 = 0;
      u.t1 = item_tiles(p_, u.q0);
      u.kind = kWhole;
      u.seg = -1;
      u.cont_lo = u.cont_hi = -1;
      return true;
    }
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
  const Table* t_;
  int cta_;
  int s_;
  int r_;
  int pos_;   // tiles of a segment fit in int: the host refuses larger launches
  int end_;
};

}  // namespace sched
}  // namespace avo_b200
