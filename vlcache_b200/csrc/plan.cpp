// Host planner for the warm-prefill attention kernel.
//
// Builds the list of work units from the varlen metadata the nano-vllm model
// runner produces (nanovllm/engine/model_runner.py:194-320 prepare_prefill:
// cu_seqlens_q, cu_seqlens_k with bottom-right causal alignment) and bin-packs
// them onto a persistent grid of one CTA per SM (longest-processing-time first).
// A unit is one query tile over one range of 128-key blocks.  Tiles whose key
// range is long (text after the image sees the whole image) are split into
// several units so the per-CTA work is balanced; the partial results are merged
// by a second small kernel.
//
// Pure host code (the only CUDA query is the SM count when num_sms == 0, which
// falls back to 148 without a device): usable without a GPU.
#include <algorithm>
#include <array>
#include <cmath>
#include <cstdint>
#include <queue>
#include <vector>

#include "plan.h"
#include "vlcache_b200.h"

namespace {

constexpr int kBlockN = 128;  // keys per K/V tile in the kernel
constexpr int kTileRows = 128;

struct Tile {
  int seq, kv_head, q_begin, q_count, kpos0, n_kb, kv_len, k_base;
};

struct UnitRec {
  int32_t f[vlc::kUnitInts];
  double cost;
};

int validate(const int32_t* cu_q, const int32_t* cu_k, int num_seqs, int num_heads, int num_kv_heads,
             int head_dim) {
  if (!cu_q || !cu_k) return VLC_ERR_NULL;
  if (num_seqs < 0) return VLC_ERR_SHAPE;
  if (head_dim != 128) return VLC_ERR_UNSUPPORTED;
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

void build_tiles(const int32_t* cu_q, const int32_t* cu_k, int num_seqs, int num_kv_heads, int T,
                 std::vector<Tile>& tiles) {
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
        t.kpos0 = kl - ql + t0;
        const int max_pos = t.kpos0 + t.q_count - 1;
        t.n_kb = max_pos / kBlockN + 1;
        t.kv_len = kl;
        t.k_base = cu_k[b];
        tiles.push_back(t);
      }
    }
  }
}

}  // namespace

extern "C" int64_t vlc_prefill_plan_capacity(const int32_t* cu_q, const int32_t* cu_k, int num_seqs,
                                             int num_heads, int num_kv_heads, int num_sms) {
  if (validate(cu_q, cu_k, num_seqs, num_heads, num_kv_heads, 128) != VLC_OK) return -1;
  if (num_sms <= 0) num_sms = 148;
  const int G = num_heads / num_kv_heads;
  const int T = kTileRows / G;
  std::vector<Tile> tiles;
  build_tiles(cu_q, cu_k, num_seqs, num_kv_heads, T, tiles);
  int64_t total_kb = 0;
  for (const Tile& t : tiles) total_kb += t.n_kb;
  const int64_t max_units = (int64_t)tiles.size() + total_kb;
  return vlc::kPlanHeaderInts + (num_sms + 1) + max_units * vlc::kUnitInts +
         (int64_t)tiles.size() * vlc::kMergeInts;
}

extern "C" int vlc_prefill_plan(const int32_t* cu_q, const int32_t* cu_k, int num_seqs, int num_heads,
                                int num_kv_heads, int head_dim, int num_sms, int32_t* plan_out,
                                int64_t plan_capacity, int64_t* plan_len) {
  using namespace vlc;
  const int v = validate(cu_q, cu_k, num_seqs, num_heads, num_kv_heads, head_dim);
  if (v != VLC_OK) return v;
  if (!plan_out || !plan_len) return VLC_ERR_NULL;
  if (num_sms <= 0) num_sms = vlc_num_sms();
  const int G = num_heads / num_kv_heads;
  const int T = kTileRows / G;
  std::vector<Tile> tiles;
  build_tiles(cu_q, cu_k, num_seqs, num_kv_heads, T, tiles);

  // Time model (in key-block iterations of one tile): each unit pays a fixed
  // start/epilogue cost, each split part a partial write and its share of the merge.
  const double kUnitOverhead = 1.5, kPartOverhead = 0.5;
  double total_time = 0.0;
  for (const Tile& t : tiles) total_time += t.n_kb + kUnitOverhead;
  const double avg = total_time / std::max(1, num_sms);
  // Split only tiles well above the per-SM average, into parts of about the average.
  const double split_above = std::max(4.0, 1.5 * avg);
  const double target = std::max(3.0, avg);
  std::vector<UnitRec> units;
  std::vector<std::array<int32_t, kMergeInts>> merges;
  int num_parts = 0;
  auto add_merge = [&](const Tile& t, int part0, int np) {
    std::array<int32_t, kMergeInts> m{};
    m[kMQBegin] = t.q_begin;
    m[kMQCount] = t.q_count;
    m[kMKvHead] = t.kv_head;
    m[kMPartBegin] = part0;
    m[kMNumParts] = np;
    merges.push_back(m);
  };
  for (const Tile& ta : tiles) {
    int np = ta.n_kb + kUnitOverhead > split_above ? (int)std::ceil(ta.n_kb / target) : 1;
    np = std::max(1, std::min(np, ta.n_kb));
    const int part0 = np > 1 ? num_parts : -1;
    if (np > 1) {
      add_merge(ta, part0, np);
      num_parts += np;
    }
    for (int i = 0; i < np; ++i) {
      UnitRec u{};
      for (int k = 0; k < kUnitInts; ++k) u.f[k] = 0;
      const int kb0 = (int)((int64_t)ta.n_kb * i / np);
      const int kb1 = (int)((int64_t)ta.n_kb * (i + 1) / np);
      u.f[kUSeq] = ta.seq;
      u.f[kUKvHead] = ta.kv_head;
      u.f[kUKbBegin] = kb0;
      u.f[kUKbEnd] = kb1;
      u.f[kUKvLen] = ta.kv_len;
      u.f[kUKBase] = ta.k_base;
      u.f[kUQBeginA] = ta.q_begin;
      u.f[kUQCountA] = ta.q_count;
      u.f[kUKpos0A] = ta.kpos0;
      u.f[kUPartA] = np > 1 ? part0 + i : -1;
      u.f[kUQCountB] = 0;  // single-tile units (tile B fields unused)
      u.f[kUPartB] = -1;
      u.f[kUKbEndB] = kb0;
      u.cost = (kb1 - kb0) + kUnitOverhead + (np > 1 ? kPartOverhead : 0.0);
      u.f[kUCost] = (int32_t)(u.cost * 16);
      units.push_back(u);
    }
  }

  const int num_units = (int)units.size();
  const int grid = std::min(num_sms, num_units);
  // Longest-processing-time-first bin packing onto `grid` persistent CTAs.
  std::vector<int> order(num_units);
  for (int i = 0; i < num_units; ++i) order[i] = i;
  std::stable_sort(order.begin(), order.end(),
                   [&](int a, int b) { return units[a].cost > units[b].cost; });
  std::vector<std::vector<int>> per_cta(std::max(grid, 0));
  typedef std::pair<double, int> Load;
  std::priority_queue<Load, std::vector<Load>, std::greater<Load>> heap;
  for (int c = 0; c < grid; ++c) heap.push(Load(0.0, c));
  for (int idx : order) {
    Load l = heap.top();
    heap.pop();
    per_cta[l.second].push_back(idx);
    l.first += units[idx].cost;
    heap.push(l);
  }

  const int64_t off_cta = kPlanHeaderInts;
  const int64_t off_units = off_cta + grid + 1;
  const int64_t off_merges = off_units + (int64_t)num_units * kUnitInts;
  const int64_t total = off_merges + (int64_t)merges.size() * kMergeInts;
  if (total > plan_capacity) return VLC_ERR_PLAN;

  int32_t* h = plan_out;
  for (int i = 0; i < kPlanHeaderInts; ++i) h[i] = 0;
  h[kPMagic] = kPlanMagic;
  h[kPVersion] = kPlanVersion;
  h[kPGrid] = grid;
  h[kPNumUnits] = num_units;
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
  int32_t* cta = h + off_cta;
  int32_t* up = h + off_units;
  int pos = 0;
  for (int c = 0; c < grid; ++c) {
    cta[c] = pos;
    for (int idx : per_cta[c]) {
      for (int k = 0; k < kUnitInts; ++k) up[(int64_t)pos * kUnitInts + k] = units[idx].f[k];
      ++pos;
    }
  }
  cta[grid] = pos;
  int32_t* mp = h + off_merges;
  for (size_t i = 0; i < merges.size(); ++i)
    for (int k = 0; k < kMergeInts; ++k) mp[i * kMergeInts + k] = merges[i][k];
  *plan_len = total;
  return VLC_OK;
}
