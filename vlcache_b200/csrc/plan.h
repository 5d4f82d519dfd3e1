// Layout of the int32 warm-prefill plan shared by the host planner (plan.cpp)
// and the prefill kernels.  All offsets are in int32 elements from the start
// of the plan buffer.
#pragma once

#include <stdint.h>

namespace vlc {

constexpr int32_t kPlanMagic = 0x564C4350;  // 'VLCP'
constexpr int32_t kPlanVersion = 7;
constexpr int kPlanHeaderInts = 24;

// header fields
enum : int {
  kPMagic = 0,
  kPVersion = 1,
  kPGrid = 2,          // persistent CTAs
  kPNumUnits = 3,
  kPNumParts = 4,      // partial-result slots in the workspace
  kPNumMerges = 5,
  kPRowsPerTile = 6,   // T * G
  kPTokensPerTile = 7, // T
  kPGroup = 8,         // G
  kPNumHeads = 9,
  kPNumKvHeads = 10,
  kPTotalQ = 11,
  kPOffCta = 12,       // int32[grid + 1] unit ranges per CTA
  kPOffUnits = 13,     // int32[num_units][kUnitInts]
  kPOffMerges = 14,    // int32[num_merges][kMergeInts]
  kPTotalLen = 15,
  kPMergeBlocks = 16,     // blocks of the merge launch
  kPOffMergeBlocks = 17,  // int32[merge_blocks]: (merge index << 8) | first row of the block
  kPCausal = 18,          // 1: row i of a sequence sees keys <= k_len - q_len + i; 0: all k_len keys
  kPHeadDim = 19,         // head_dim the plan was made for (64 < d <= 128, d % 16 == 0)
  kPOffSegments = 20,     // 0, or int32[total_q][2]: {first, end} token of each query token's
                          // sequence, for packed tiles (several short sequences in one tile)
  kPQuad = 21,            // 1: quad units on CTA pairs (prefill_attn_quad_kernel): the CTA
                          // ranges index CTA pairs, and unit i is records 2i (even CTA), 2i + 1
};

// A unit is one or two query tiles of one (sequence, KV head) over one range of
// 128-key blocks; both tiles read the same K/V blocks.  Tile A holds the later
// tokens and covers blocks [kb_begin, kb_end) (at least one); tile B, when
// present (kUQCountB > 0), holds earlier tokens of the same sequence and covers
// [kb_begin, kb_end_b) with kb_begin < kb_end_b <= kb_end.
// Packed tile (kUSeq == -1, non-causal self-attention of short sequences, contiguous K/V
// only): tile A holds whole consecutive sequences, tokens [q_begin, q_begin + q_count); its one
// key block is the same tokens (k_base = q_begin, kv_len = q_count), and row t sees the keys of
// its own sequence, [segments[t][0], segments[t][1]).
constexpr int kUnitInts = 17;
enum : int {
  kUSeq = 0,       // row of block_tables (-1: packed tile)
  kUKvHead = 1,
  kUKbBegin = 2,   // first 128-key block (both tiles)
  kUKbEnd = 3,     // one past the last block of tile A
  kUKvLen = 4,     // keys of the sequence
  kUKBase = 5,     // first key row of the sequence when K/V are not paged
  kUCost = 6,      // planner cost estimate x16 (diagnostic)
  kUQBeginA = 7,   // tile A: first query token (absolute row of q)
  kUQCountA = 8,   //         valid tokens (1..T)
  kUKpos0A = 9,    //         logical position of its first token
  kUPartA = 10,    //         -1: write the normalised output; else partial slot
  kUQBeginB = 11,  // tile B (kUQCountB == 0: no tile B)
  kUQCountB = 12,
  kUKpos0B = 13,
  kUPartB = 14,
  kUKbEndB = 15,   // one past tile B's last block
  kUSelfRow = 16,  // q_len == k_len (the sequence attends over its own rows): the row of its
                   // first token in q, which is also its first key row in the in-flight K/V
                   // (the projection's output); -1 otherwise
};

// kUPartA / kUPartB of a ghost tile: a quad's stand-in for a missing tile (computed, not written)
constexpr int kGhostPart = -2;

// merge fields (one record per split query tile)
constexpr int kMergeInts = 8;
enum : int {
  kMQBegin = 0,
  kMQCount = 1,
  kMKvHead = 2,
  kMPartBegin = 3,
  kMNumParts = 4,
  kMRowsPerWarp = 5,  // rows one warp merges (4, 2 or 1: its 4 lane groups split a row's parts)
  kMRows = 6,         // rows to merge (valid tokens x G)
};

}  // namespace vlc
