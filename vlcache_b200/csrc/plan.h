// Layout of the int32 warm-prefill plan shared by the host planner (plan.cpp)
// and the prefill kernels.  All offsets are in int32 elements from the start
// of the plan buffer.
#pragma once

#include <stdint.h>

namespace vlc {

constexpr int32_t kPlanMagic = 0x564C4350;  // 'VLCP'
constexpr int32_t kPlanVersion = 1;
constexpr int kPlanHeaderInts = 16;

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
};

// unit fields
constexpr int kUnitInts = 12;
enum : int {
  kUSeq = 0,      // row of block_tables
  kUKvHead = 1,
  kUQBegin = 2,   // first query token (absolute row of q)
  kUQCount = 3,   // valid query tokens in the tile (<= T)
  kUKpos0 = 4,    // logical position of the first query token
  kUKbBegin = 5,  // first 128-key block
  kUKbEnd = 6,    // one past the last 128-key block
  kUKvLen = 7,    // keys of the sequence
  kUPart = 8,     // -1: write the normalised output; else partial slot
  kUCost = 9,     // planner cost estimate (diagnostic)
  kUKBase = 10,   // first key row of the sequence when K/V are not paged (cu_seqlens_k[seq])
};

// merge fields
constexpr int kMergeInts = 8;
enum : int {
  kMQBegin = 0,
  kMQCount = 1,
  kMKvHead = 2,
  kMPartBegin = 3,
  kMNumParts = 4,
};

}  // namespace vlc
