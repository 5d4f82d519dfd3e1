// Host planner for the warm-prefill attention kernel.
//
// Builds the list of work units from the varlen metadata the nano-vllm model
// runner produces (nanovllm/engine/model_runner.py:194-320 prepare_prefill:
// cu_seqlens_q, cu_seqlens_k with bottom-right causal alignment) and bin-packs
// them onto a persistent grid of one CTA per SM (longest-processing-time first).
// A unit is a pair of query tiles of one (sequence, KV head) sharing one range
// of 128-key blocks (or a single tile).  Units whose key range is long (text
// after the image sees the whole image) are split into several units so the
// per-CTA work is balanced; the partial results are merged by a second small
// kernel.
//
// Pure host code (the only CUDA query is the SM count when num_sms == 0, which
// falls back to 148 without a device): usable without a GPU.
#include <algorithm>
#include <array>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <queue>
#include <vector>

#include "plan.h"
#include "vlcache_b200.h"

namespace {

constexpr int kBlockN = 128;  // keys per K/V tile in the kernel
constexpr int kTileRows = 128;
// Parts per split tile: the merge folds a row's parts with 4 lane groups, 5 parts
// each in flight at once, so up to 20 parts cost one round of loads.
constexpr int kMaxParts = 20;

struct Tile {
  int seq, kv_head, q_begin, q_count, kpos0, n_kb, kv_len, k_base;
  int self_row;  // cu_q[seq] when q_len == k_len, else -1
};

struct UnitRec {
  int32_t f[vlc::kUnitInts];
  double cost;
};

int validate(const int32_t* cu_q, const int32_t* cu_k, int num_seqs, int num_heads, int num_kv_heads,
             int head_dim) {
  if (!cu_q || !cu_k) return VLC_ERR_NULL;
  if (num_seqs < 0) return VLC_ERR_SHAPE;
  if (head_dim <= 64 || head_dim > 128 || head_dim % 16 != 0) return VLC_ERR_UNSUPPORTED;
  if (num_heads <= 0 || num_kv_heads <= 0 || num_heads % num_kv_heads != 0) return VLC_ERR_SHAPE;
  if (num_heads / num_kv_heads > kTileRows) return VLC_ERR_UNSUPPORTED;
  if (cu_q[0] != 0 || cu_k[0] != 0) return VLC_ERR_METADATA;
  for (int b = 0; b < num_seqs; ++b) {
    const int ql = cu_q[b + 1] - cu_q[b];
    const int kl = cu_k[b + 1] - cu_k[b];
    if (ql < 0 || kl < 0 || ql > kl) return VLC_ERR_METADATA;
  }
  return VLC_OK;
}

// Causal: row t0 + r of a sequence sees keys <= k_len - q_len + t0 + r (flash-attn's
// bottom-right alignment).  Non-causal: every row sees all k_len keys (kpos0 = k_len - 1,
// the kernel adds no per-row offset).
void build_tiles(const int32_t* cu_q, const int32_t* cu_k, int num_seqs, int num_kv_heads, int T, bool causal,
                 std::vector<Tile>& tiles) {
  size_t count = 0;
  for (int b = 0; b < num_seqs; ++b) count += (size_t)((cu_q[b + 1] - cu_q[b] + T - 1) / T) * num_kv_heads;
  tiles.reserve(count);
  for (int b = 0; b < num_seqs; ++b) {
    const int ql = cu_q[b + 1] - cu_q[b];
    const int kl = cu_k[b + 1] - cu_k[b];
    for (int g = 0; g < num_kv_heads; ++g) {
      for (int t0 = 0; t0 < ql; t0 += T) {
        Tile t;
        t.seq = b;
        t.kv_head = g;
        t.q_begin = cu_q[b] + t0;
        t.q_count = std::min(T, ql - t0);
        t.kpos0 = causal ? kl - ql + t0 : kl - 1;
        const int max_pos = causal ? t.kpos0 + t.q_count - 1 : kl - 1;
        t.n_kb = max_pos / kBlockN + 1;
        t.kv_len = kl;
        t.k_base = cu_k[b];
        t.self_row = ql == kl ? cu_q[b] : -1;
        tiles.push_back(t);
      }
    }
  }
}

// Non-causal self-attention whose sequences all fit a tile (the vision tower's windows):
// consecutive whole sequences are packed into tiles of at most T tokens.
bool packable(const int32_t* cu_q, const int32_t* cu_k, int num_seqs, int T, bool causal) {
  if (causal || num_seqs <= 0) return false;
  for (int b = 0; b <= num_seqs; ++b)
    if (cu_q[b] != cu_k[b]) return false;
  for (int b = 0; b < num_seqs; ++b)
    if (cu_q[b + 1] - cu_q[b] > T) return false;
  return true;
}

void build_packed_tiles(const int32_t* cu_q, int num_seqs, int num_kv_heads, int T, std::vector<Tile>& tiles) {
  for (int g = 0; g < num_kv_heads; ++g) {
    int b = 0;
    while (b < num_seqs) {
      if (cu_q[b + 1] == cu_q[b]) {
        ++b;
        continue;
      }
      const int q0 = cu_q[b];
      int e = b;
      while (e < num_seqs && cu_q[e + 1] - q0 <= T) ++e;
      Tile t;
      t.seq = -1;
      t.kv_head = g;
      t.q_begin = q0;
      t.q_count = cu_q[e] - q0;
      t.kpos0 = 0;  // unused: the packed kernel masks by the row's sequence
      t.n_kb = 1;
      t.kv_len = t.q_count;
      t.k_base = q0;
      t.self_row = -1;  // packed tiles read contiguous K/V only
      tiles.push_back(t);
      b = e;
    }
  }
}

// Unit kind of new plans: 0 / 1 pairs of tiles (prefill_attn_kernel), 2 quads of tiles
// on CTA pairs (prefill_attn_quad_kernel; packed plans always use pairs).
std::atomic<int> g_prefill_kernel{0};

}  // namespace

extern "C" int vlc_prefill_set_kernel(int mode) {
  if (mode < 0 || mode > 2) return VLC_ERR_SHAPE;
  g_prefill_kernel.store(mode);
  return VLC_OK;
}

extern "C" int64_t vlc_attention_plan_capacity(const int32_t* cu_q, const int32_t* cu_k, int num_seqs,
                                               int num_heads, int num_kv_heads, int causal, int num_sms) {
  if (validate(cu_q, cu_k, num_seqs, num_heads, num_kv_heads, 128) != VLC_OK) return -1;
  if (num_sms <= 0) num_sms = 148;
  const int G = num_heads / num_kv_heads;
  const int T = kTileRows / G;
  std::vector<Tile> tiles;
  const bool packed = packable(cu_q, cu_k, num_seqs, T, causal != 0);
  if (packed)
    build_packed_tiles(cu_q, num_seqs, num_kv_heads, T, tiles);
  else
    build_tiles(cu_q, cu_k, num_seqs, num_kv_heads, T, causal != 0, tiles);
  int64_t total_kb = 0;
  for (const Tile& t : tiles) total_kb += t.n_kb;
  const int64_t max_units = (int64_t)tiles.size() + total_kb;
  return vlc::kPlanHeaderInts + (num_sms + 1) + 2 * max_units * vlc::kUnitInts +
         (int64_t)tiles.size() * (vlc::kMergeInts + kTileRows) + (packed ? 2LL * cu_q[num_seqs] : 0);
}

extern "C" int64_t vlc_prefill_plan_capacity(const int32_t* cu_q, const int32_t* cu_k, int num_seqs,
                                             int num_heads, int num_kv_heads, int num_sms) {
  return vlc_attention_plan_capacity(cu_q, cu_k, num_seqs, num_heads, num_kv_heads, 1, num_sms);
}

extern "C" int vlc_attention_plan(const int32_t* cu_q, const int32_t* cu_k, int num_seqs, int num_heads,
                                  int num_kv_heads, int head_dim, int causal, int num_sms, int32_t* plan_out,
                                  int64_t plan_capacity, int64_t* plan_len) {
  using namespace vlc;
  const int v = validate(cu_q, cu_k, num_seqs, num_heads, num_kv_heads, head_dim);
  if (v != VLC_OK) return v;
  if (!plan_out || !plan_len) return VLC_ERR_NULL;
  if (num_sms <= 0) num_sms = vlc_num_sms();
  const int G = num_heads / num_kv_heads;
  const int T = kTileRows / G;
  std::vector<Tile> tiles;
  const bool packed = packable(cu_q, cu_k, num_seqs, T, causal != 0);
  if (packed)
    build_packed_tiles(cu_q, num_seqs, num_kv_heads, T, tiles);
  else
    build_tiles(cu_q, cu_k, num_seqs, num_kv_heads, T, causal != 0, tiles);

  // Pair the tiles of each (sequence, KV head) from the end: (last, second last),
  // ...; with an odd count the first (cheapest) tile stays alone.  The later tile
  // of a pair is tile A (it sees every key block tile B sees, and maybe one more).
  struct Pair {
    int a, b;  // tile indices, b = -1 for a single tile
  };
  // Quad mode: per (sequence, KV head), from the end, tiles (a0, a1, b0, b1) = (last, last - 1,
  // last - 2, last - 3); the even CTA of a pair takes a0 and b0, the odd one a1 and b1, and the
  // pair's MMAs run over a0's (and b0's) key blocks.  `pairs` then holds (a0, b0), `odd` (a1, b1).
  const bool quad = g_prefill_kernel.load() == 2 && !packed;
  const int bins = quad ? std::max(1, num_sms / 2) : num_sms;
  std::vector<Pair> pairs, odd;
  pairs.reserve(tiles.size());
  for (size_t i = 0; quad && i < tiles.size();) {
    size_t e = i;
    while (e < tiles.size() && tiles[e].seq == tiles[i].seq && tiles[e].kv_head == tiles[i].kv_head) ++e;
    for (int last = (int)e - 1; last >= (int)i; last -= 4) {
      auto at = [&](int k) { return last - k >= (int)i ? last - k : -1; };
      pairs.push_back(Pair{at(0), at(2)});
      odd.push_back(Pair{at(1), at(3)});
    }
    i = e;
  }
  for (size_t i = 0; !quad && i < tiles.size();) {
    size_t e = i;
    // (packed tiles, all of sequence -1, pair by KV head: each keeps its own key block)
    while (e < tiles.size() && tiles[e].seq == tiles[i].seq && tiles[e].kv_head == tiles[i].kv_head) ++e;
    if (e == i) e = i + 1;
    int last = (int)e - 1;
    while (last >= (int)i) {
      if (last - 1 >= (int)i) {
        pairs.push_back(Pair{last, last - 1});
        last -= 2;
      } else {
        pairs.push_back(Pair{last, -1});
        last -= 1;
      }
    }
    i = e;
  }

  // Time model, in single-tile key-block steps (measured on B200: a step of a
  // paired unit costs about 1.2 steps, each unit about 1.5 steps of start, drain and
  // epilogue; a split part adds a partial write and its share of the merge).
  const double kUnitOverhead = 1.5, kPartOverhead = 0.1;
  const double kPairStep = packed ? 1.0 : 0.2;  // packed pairs share no K/V block
  auto pair_cost = [&](const Pair& pr, int kb0, int kb1) {
    const int nb = pr.b >= 0 ? std::max(0, std::min(kb1, tiles[pr.b].n_kb) - kb0) : 0;
    return (kb1 - kb0) + kPairStep * nb + kUnitOverhead;
  };
  // Parts of a pair for a target unit cost M: the fewest equal parts whose cost
  // stays within M (a part of one block when M is below that).
  auto parts_for = [&](const Pair& pr, double M) {
    const int n = tiles[pr.a].n_kb;
    if (pair_cost(pr, 0, n) <= M) return 1;
    const double per_block = pr.b >= 0 ? 1.0 + kPairStep : 1.0;
    const double room = M - kUnitOverhead - kPartOverhead;
    const int np = room >= per_block ? (int)std::ceil(n * per_block / room) : n;
    return std::max(1, std::min(std::min(np, n), kMaxParts));
  };
  auto part_costs = [&](const Pair& pr, int np, std::vector<double>& out) {
    const int n = tiles[pr.a].n_kb;
    for (int i = 0; i < np; ++i) {
      const int kb0 = (int)((int64_t)n * i / np), kb1 = (int)((int64_t)n * (i + 1) / np);
      out.push_back(pair_cost(pr, kb0, kb1) + (np > 1 ? kPartOverhead : 0.0));
    }
  };
  // Longest-processing-time-first makespan of a set of unit costs on num_sms CTAs.
  auto lpt_makespan = [&](std::vector<double>& costs) {
    if ((int)costs.size() <= bins) return costs.empty() ? 0.0 : *std::max_element(costs.begin(), costs.end());
    std::sort(costs.begin(), costs.end(), std::greater<double>());
    std::priority_queue<double, std::vector<double>, std::greater<double>> heap;
    for (int c = 0; c < bins; ++c) heap.push(0.0);
    double mk = 0.0;
    for (double c : costs) {
      const double l = heap.top() + c;
      heap.pop();
      heap.push(l);
      mk = std::max(mk, l);
    }
    return mk;
  };
  // Choose the target M among candidates between the cheapest possible part and
  // the longest unsplit pair by the packed makespan; any split also costs the
  // merge launch (about two steps on the critical path).
  const double kMergeLaunch = 2.0;
  double max_pair = 0.0, total_unsplit = 0.0;
  for (const Pair& pr : pairs) {
    const double c = pair_cost(pr, 0, tiles[pr.a].n_kb);
    max_pair = std::max(max_pair, c);
    total_unsplit += c;
  }
  double best_M = max_pair;
  const double m_min = kUnitOverhead + kPartOverhead + 1.0 + kPairStep;  // a one-block part
  if (total_unsplit / std::max(1, bins) < max_pair) {
    // Mean CTA load after splitting every pair to M (decreasing in M).
    auto mean_load = [&](double M) {
      double tot = 0.0;
      for (const Pair& pr : pairs) {
        const int np = parts_for(pr, M);
        const int nb_full = pr.b >= 0 ? tiles[pr.b].n_kb : 0;
        tot += tiles[pr.a].n_kb + kPairStep * nb_full + np * kUnitOverhead + (np > 1 ? np * kPartOverhead : 0.0);
      }
      return tot / std::max(1, bins);
    };
    // M* where the largest unit meets the mean load, then the packed makespan
    // (LPT) of targets around it decides.
    double lo = m_min, hi = max_pair;
    for (int it = 0; it < 16; ++it) {
      const double mid = 0.5 * (lo + hi);
      if (mid < mean_load(mid))
        lo = mid;
      else
        hi = mid;
    }
    std::vector<double> costs;
    double best_score = 1e300;
    auto consider = [&](double M) {
      costs.clear();
      bool split = false;
      for (const Pair& pr : pairs) {
        const int np = parts_for(pr, M);
        split |= np > 1;
        part_costs(pr, np, costs);
      }
      const double sc = lpt_makespan(costs) + (split ? kMergeLaunch : 0.0);
      if (sc < best_score - 1e-9) {
        best_score = sc;
        best_M = M;
      }
    };
    consider(max_pair);
    static const double kScan[] = {0.8, 0.85, 0.9, 0.95, 1.0, 1.05, 1.1, 1.15, 1.2, 1.3, 1.4, 1.6, 2.0};
    for (double f : kScan) {
      const double M = hi * f;
      if (M >= m_min && M < max_pair) consider(M);
    }
  }
  std::vector<UnitRec> units;
  units.reserve(pairs.size() + 64);
  std::vector<std::array<int32_t, kMergeInts>> merges;
  int num_parts = 0;
  auto add_merge = [&](const Tile& t, int part0, int np) {
    std::array<int32_t, kMergeInts> m{};
    m[kMQBegin] = t.q_begin;
    m[kMQCount] = t.q_count;
    m[kMKvHead] = t.kv_head;
    m[kMPartBegin] = part0;
    m[kMNumParts] = np;
    // A warp is 4 groups of 8 lanes; few parts: one row per group, many parts:
    // the groups of a warp split one row's parts.
    m[kMRowsPerWarp] = np <= 4 ? 4 : np <= 8 ? 2 : 1;
    m[kMRows] = t.q_count * G;
    merges.push_back(m);
  };
  std::vector<UnitRec> units_odd;  // quad mode: the odd CTA's record of each unit
  for (size_t pi = 0; pi < pairs.size(); ++pi) {
    const Pair& pr = pairs[pi];
    const Tile& ta = tiles[pr.a];
    const int n = ta.n_kb;
    const int np = parts_for(pr, best_M);
    std::vector<int> cuts(np + 1);
    for (int i = 0; i <= np; ++i) cuts[i] = (int)((int64_t)n * i / np);
    // Parts of tile A: all np; parts of tile B: those that start before its end.
    const int nb_full = pr.b >= 0 ? tiles[pr.b].n_kb : 0;
    int np_b = 0;
    while (np_b < np && cuts[np_b] < nb_full) ++np_b;
    const int part_a = np > 1 ? num_parts : -1;
    if (np > 1) {
      add_merge(ta, part_a, np);
      num_parts += np;
    }
    const int part_b = np_b > 1 ? num_parts : -1;
    if (np_b > 1) {
      add_merge(tiles[pr.b], part_b, np_b);
      num_parts += np_b;
    }
    // The odd CTA's tiles (quad mode), each split like its even sibling; a missing one is
    // a ghost of the sibling (runs, writes nothing).
    const Pair po = quad ? odd[pi] : Pair{-1, -1};
    const int part_a1 = quad && po.a >= 0 && np > 1 ? num_parts : -1;
    if (part_a1 >= 0) {
      add_merge(tiles[po.a], part_a1, np);
      num_parts += np;
    }
    const int part_b1 = quad && po.b >= 0 && np_b > 1 ? num_parts : -1;
    if (part_b1 >= 0) {
      add_merge(tiles[po.b], part_b1, np_b);
      num_parts += np_b;
    }
    for (int i = 0; i < np; ++i) {
      UnitRec u{};
      for (int k = 0; k < kUnitInts; ++k) u.f[k] = 0;
      const int kb0 = cuts[i], kb1 = cuts[i + 1];
      u.f[kUSeq] = ta.seq;
      u.f[kUKvHead] = ta.kv_head;
      u.f[kUKbBegin] = kb0;
      u.f[kUKbEnd] = kb1;
      u.f[kUKvLen] = ta.kv_len;
      u.f[kUKBase] = ta.k_base;
      u.f[kUSelfRow] = ta.self_row;
      u.f[kUQBeginA] = ta.q_begin;
      u.f[kUQCountA] = ta.q_count;
      u.f[kUKpos0A] = ta.kpos0;
      u.f[kUPartA] = np > 1 ? part_a + i : -1;
      u.f[kUPartB] = -1;
      if (i < np_b) {
        const Tile& tb = tiles[pr.b];
        u.f[kUQBeginB] = tb.q_begin;
        u.f[kUQCountB] = tb.q_count;
        u.f[kUKpos0B] = tb.kpos0;
        u.f[kUPartB] = np_b > 1 ? part_b + i : -1;
        u.f[kUKbEndB] = std::min(kb1, nb_full);
      }
      u.cost = pair_cost(i < np_b ? pr : Pair{pr.a, -1}, kb0, kb1) + (np > 1 ? kPartOverhead : 0.0);
      u.f[kUCost] = (int32_t)(u.cost * 16);
      units.push_back(u);
      if (quad) {
        UnitRec w = u;  // same key range, sequence and KV head
        if (po.a >= 0) {
          const Tile& t1 = tiles[po.a];
          w.f[kUQBeginA] = t1.q_begin;
          w.f[kUQCountA] = t1.q_count;
          w.f[kUKpos0A] = t1.kpos0;
          w.f[kUPartA] = part_a1 >= 0 ? part_a1 + i : -1;
        } else {
          w.f[kUPartA] = kGhostPart;
        }
        if (i < np_b) {
          if (po.b >= 0) {
            const Tile& t1 = tiles[po.b];
            w.f[kUQBeginB] = t1.q_begin;
            w.f[kUQCountB] = t1.q_count;
            w.f[kUKpos0B] = t1.kpos0;
            w.f[kUPartB] = part_b1 >= 0 ? part_b1 + i : -1;
          } else {
            w.f[kUPartB] = kGhostPart;
          }
        }
        units_odd.push_back(w);
      }
    }
  }

  const int num_units = (int)units.size();
  const int grid = std::min(bins, num_units);  // CTAs, or CTA pairs in quad mode
  // Longest-processing-time-first bin packing onto `grid` persistent CTAs (ties in
  // unit order); each CTA runs its units longest first.
  std::vector<std::pair<double, int>> order(num_units);
  for (int i = 0; i < num_units; ++i) order[i] = std::make_pair(-units[i].cost, i);
  std::sort(order.begin(), order.end());
  std::vector<int> cta_of(num_units);
  {
    typedef std::pair<double, int> Load;
    std::vector<Load> heap_store;
    heap_store.reserve(grid);
    std::priority_queue<Load, std::vector<Load>, std::greater<Load>> heap(std::greater<Load>(),
                                                                         std::move(heap_store));
    for (int c = 0; c < grid; ++c) heap.push(Load(0.0, c));
    for (const auto& o : order) {
      Load l = heap.top();
      heap.pop();
      cta_of[o.second] = l.second;
      l.first -= o.first;
      heap.push(l);
    }
  }
  // Units grouped by CTA (counting sort, LPT order inside a CTA).  (Putting the
  // self-attention units first, so that with in-flight K/V they run while the scatter
  // finishes, measured slower: the LPT order's tail matters more.)
  std::vector<int> cta_begin(grid + 1, 0), by_cta(num_units);
  for (int i = 0; i < num_units; ++i) ++cta_begin[cta_of[i] + 1];
  for (int c = 0; c < grid; ++c) cta_begin[c + 1] += cta_begin[c];
  {
    std::vector<int> fill(cta_begin.begin(), cta_begin.end() - 1);
    for (const auto& o : order) by_cta[fill[cta_of[o.second]]++] = o.second;
  }

  const int recs = quad ? 2 : 1;  // records per unit (quad: the even and the odd CTA's)
  const int64_t off_cta = kPlanHeaderInts;
  const int64_t off_units = off_cta + grid + 1;
  const int64_t off_merges = off_units + (int64_t)num_units * recs * kUnitInts;
  // Merge launch: 8 warps per block, kMRowsPerWarp rows per warp.
  std::vector<int32_t> merge_blocks;
  for (size_t i = 0; i < merges.size(); ++i) {
    const int rpb = 8 * merges[i][kMRowsPerWarp];
    for (int r0 = 0; r0 < merges[i][kMRows]; r0 += rpb) merge_blocks.push_back((int32_t)((i << 8) | r0));
  }
  const int64_t off_mblocks = off_merges + (int64_t)merges.size() * kMergeInts;
  const int64_t off_segments = packed ? off_mblocks + (int64_t)merge_blocks.size() : 0;
  const int64_t total = off_mblocks + (int64_t)merge_blocks.size() + (packed ? 2LL * cu_q[num_seqs] : 0);
  if (total > plan_capacity) return VLC_ERR_PLAN;

  int32_t* h = plan_out;
  for (int i = 0; i < kPlanHeaderInts; ++i) h[i] = 0;
  h[kPMagic] = kPlanMagic;
  h[kPVersion] = kPlanVersion;
  h[kPGrid] = grid * recs;
  h[kPNumUnits] = num_units * recs;
  h[kPNumParts] = num_parts;
  h[kPNumMerges] = (int32_t)merges.size();
  h[kPRowsPerTile] = T * G;
  h[kPTokensPerTile] = T;
  h[kPGroup] = G;
  h[kPNumHeads] = num_heads;
  h[kPNumKvHeads] = num_kv_heads;
  h[kPTotalQ] = num_seqs > 0 ? cu_q[num_seqs] : 0;
  h[kPOffCta] = (int32_t)off_cta;
  h[kPOffUnits] = (int32_t)off_units;
  h[kPOffMerges] = (int32_t)off_merges;
  h[kPTotalLen] = (int32_t)total;
  h[kPMergeBlocks] = (int32_t)merge_blocks.size();
  h[kPOffMergeBlocks] = (int32_t)off_mblocks;
  h[kPCausal] = causal != 0 ? 1 : 0;
  h[kPHeadDim] = head_dim;
  h[kPOffSegments] = (int32_t)off_segments;
  h[kPQuad] = quad ? 1 : 0;
  if (packed) {
    int32_t* seg = h + off_segments;
    for (int b = 0; b < num_seqs; ++b)
      for (int t = cu_q[b]; t < cu_q[b + 1]; ++t) {
        seg[2 * (int64_t)t] = cu_q[b];
        seg[2 * (int64_t)t + 1] = cu_q[b + 1];
      }
  }
  int32_t* cta = h + off_cta;
  int32_t* up = h + off_units;
  for (int c = 0; c <= grid; ++c) cta[c] = cta_begin[c];
  for (int pos = 0; pos < num_units; ++pos) {
    const UnitRec& u = units[by_cta[pos]];
    for (int k = 0; k < kUnitInts; ++k) up[((int64_t)pos * recs) * kUnitInts + k] = u.f[k];
    if (quad) {
      const UnitRec& w = units_odd[by_cta[pos]];
      for (int k = 0; k < kUnitInts; ++k) up[((int64_t)pos * recs + 1) * kUnitInts + k] = w.f[k];
    }
  }
  int32_t* mp = h + off_merges;
  for (size_t i = 0; i < merges.size(); ++i)
    for (int k = 0; k < kMergeInts; ++k) mp[i * kMergeInts + k] = merges[i][k];
  for (size_t i = 0; i < merge_blocks.size(); ++i) h[off_mblocks + i] = merge_blocks[i];
  *plan_len = total;
  return VLC_OK;
}

extern "C" int vlc_prefill_plan(const int32_t* cu_q, const int32_t* cu_k, int num_seqs, int num_heads,
                                int num_kv_heads, int head_dim, int num_sms, int32_t* plan_out,
                                int64_t plan_capacity, int64_t* plan_len) {
  return vlc_attention_plan(cu_q, cu_k, num_seqs, num_heads, num_kv_heads, head_dim, 1, num_sms, plan_out,
                            plan_capacity, plan_len);
}
