// Sparse-query paged prefill attention on sm_100a (tcgen05 + TMEM + TMA).
//
// Query rows are the recomputed rows of warm requests (text tokens and the
// first R vision tokens, flash-attn varlen layout).  Each query row attends,
// causally by logical position, over its sequence's paged K/V cache.
//
// Work decomposition (host planner, plan.cpp): a *tile* is T consecutive
// query tokens of one sequence x the G query heads of one KV head, packed into
// the 128 rows of a UMMA M=128 tile (row = token*G + head: GQA packing, so one
// K/V tile feeds G heads).  A *unit* is a pair of tiles of the same (sequence,
// KV head) -- A holds the later tokens, B the earlier ones -- over one range of
// 128-key blocks: every K/V block loaded feeds 256 query rows.  Long ranges are
// split into several units whose partial results are merged by
// prefill_merge_kernel.  Units are bin-packed onto a persistent grid of one CTA
// per SM.
//
// CTA roles (352 threads):
//   warps 0-3  softmax of tile A (thread i: row i = TMEM lane i, all 128 keys)
//   warps 4-7  softmax of tile B
//   warp  8    TMA producer of K/V blocks (2-stage ring)
//   warp  9    TMEM allocator + single-thread tcgen05.mma issuer
//   warp 10    TMA producer of Q tiles (2-slot ring: a tile's slot reloads for
//              the next unit once its last Q K^T has run)
// TMEM (512 columns): S_A | S_B | O_A | O_B, 128 fp32 columns each.  For each
// key block j the issuer runs, per tile X in (A, B):  O_X += P_X(j) V(j) as soon
// as the softmax of X has written P_X(j), then S_X = Q_X K(j+1)^T.  The two
// tiles interleave on the tensor pipe: while one tile's softmax works, the
// other tile's P*V and Q*K^T execute.  P (bf16 pairs) overwrites the first 64
// columns of S_X and is read from TMEM as the A operand of O += P V (V is an
// MN-major smem operand).  Online softmax in the log2 domain with lazy
// rescaling: the running max moves (and O is rescaled) only when it grows by
// more than 2^8.  The tensor pipe executes one thread's MMAs in issue order, so
// when S_X(j) is complete so is P_X(j-1) V(j-1): a softmax thread that has seen
// S_X(j) may rescale O_X without further waiting.
#include <algorithm>
#include <cmath>

#include "common.cuh"
#include "plan.h"
#include "runtime.h"

namespace vlc {
namespace prefill {

constexpr int BM = 128;    // tile rows (tokens * group)
constexpr int BN = 128;    // keys per K/V block
constexpr int HD = 128;    // head dim
constexpr int STAGES = 2;  // K/V ring depth
constexpr int QSLOTS = 2;  // Q ring depth (a unit holds up to two)
constexpr int NUM_THREADS = 352;
constexpr int HALF_BYTES = BM * 128;        // 128 rows x 128 B (64 bf16)
constexpr int TILE_BYTES = 2 * HALF_BYTES;  // 32 KB: full 128 x 128 bf16 tile

constexpr int OFF_Q = 0;
constexpr int OFF_K = OFF_Q + QSLOTS * TILE_BYTES;
constexpr int OFF_V = OFF_K + STAGES * TILE_BYTES;
constexpr int OFF_STG = OFF_V + STAGES * TILE_BYTES;  // epilogue staging, per tile two buffers of
constexpr int STG_BUF = BM * 64;                       // 32 output columns (128 rows x 64 B, 64-byte swizzle)
constexpr int STG_TILE = 2 * STG_BUF;
constexpr int OFF_BAR = OFF_STG + 2 * STG_TILE;
// barriers: q_full[3], q_empty[3], k_full[S], k_empty[S], v_full[S], v_empty[S],
//           s_full[2], p_lo[2], p_hi[2], o_done[2] (index = tile: 0 A, 1 B).  p_lo: P of
//           keys 0-63 written, p_hi: P of keys 64-127 written.
// Every parity wait below is on a barrier that is at most one phase behind the
// completion it waits for, and never ahead of it: each producer of a completion
// first waits for the consumer of the previous one.
constexpr int NUM_BARS = 2 * QSLOTS + 4 * STAGES + 8;
constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;  // + alignment slack
static_assert(SMEM_BYTES <= 232448, "shared memory budget");

constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t TMEM_S = 0;    // S of tile x at TMEM_S + 128 x
constexpr uint32_t TMEM_O = 256;  // O of tile x at TMEM_O + 128 x

constexpr uint32_t IDESC_QK = umma_idesc_bf16(128, 128, false, false);
constexpr uint32_t IDESC_PV = umma_idesc_bf16(128, 128, false, true);

constexpr int kTileThreads = 128;  // softmax threads per tile

struct Params {
  CUtensorMap tm_q;   // dims {d, num_heads, total_q}, box {64, G, T} (columns >= d fill with 0)
  CUtensorMap tm_k;   // dims {d, Hk, num_rows},    box {64, 1, BN}
  CUtensorMap tm_v;
  const int32_t* cta_offsets;  // [grid + 1]
  const int32_t* units;        // [num_units][kUnitInts]
  const int32_t* block_tables;
  int bt_stride;
  int block_size;
  int group;           // G = num_heads / num_kv_heads
  int rows;            // T * G (<= 128)
  float scale_log2;    // softmax_scale * log2(e)
  int64_t num_slots;
  CUtensorMap tm_o;   // out:    dims {d, num_heads, total_q}, box {32, G, T}
  CUtensorMap tm_p;   // part_o: dims {HD, num_parts * BM},   box {64, BM}
  // Same tensors, 128-byte swizzle, box {64, G, T} / {64, BM}: the last epilogue of a
  // tile stores straight from the tile's Q slot (same layout as the Q load).
  CUtensorMap tm_o128;
  CUtensorMap tm_p128;
  int tokens_per_tile;  // T
  int head_dim;         // d of q/k/v/out (64 < d <= 128); tiles are zero-padded to 128 columns
  int causal;           // 0: every row sees all of its sequence's keys
  const int32_t* segments;  // packed plans: {first, end} token of each query token's sequence
  __nv_bfloat16* out;
  int64_t out_token_stride;
  int out_store32;        // out rows are 32-byte aligned: 256-bit stores
  __nv_bfloat16* part_o;  // [num_parts][BM][HD] partial O / l (bf16)
  float* part_ml;         // [num_parts][BM][2]  (max in log2 domain, sum)
  // In-flight K/V (the projection's rows, dims {d, Hk, num_new_rows}, box {64, 1, BN}).
  // inflight == 1: units of self-attention sequences (kUSelfRow >= 0) load their keys from
  // here, and only the other units' K/V loads wait for the kernel launched just before.
  CUtensorMap tm_kn;
  CUtensorMap tm_vn;
  int inflight;
  // Quad kernel: the same K tensors with a box of 64 keys (a CTA's half of a block).
  CUtensorMap tm_k64;
  CUtensorMap tm_kn64;
};

struct Bars {
  uint64_t* q_full;   // [QSLOTS]
  uint64_t* q_empty;  // [QSLOTS]
  uint64_t* k_full;
  uint64_t* k_empty;
  uint64_t* v_full;
  uint64_t* v_empty;
  uint64_t* s_full;   // [2]
  uint64_t* p_lo;     // [2]
  uint64_t* p_hi;     // [2]
  uint64_t* o_done;   // [2]
};

__device__ __forceinline__ Bars make_bars(uint8_t* smem) {
  uint64_t* b = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  Bars r;
  r.q_full = b;
  r.q_empty = b + QSLOTS;
  r.k_full = b + 2 * QSLOTS;
  r.k_empty = r.k_full + STAGES;
  r.v_full = r.k_full + 2 * STAGES;
  r.v_empty = r.k_full + 3 * STAGES;
  r.s_full = r.k_full + 4 * STAGES;
  r.p_lo = r.s_full + 2;
  r.p_hi = r.s_full + 4;
  r.o_done = r.s_full + 6;
  return r;
}

__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, int code,
                                              volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (clock64() - t0 > VLC_WAIT_LIMIT_CYCLES) {
      record_error(code);
      *abort_flag = 1;
      return false;
    }
  }
}

// Unit fields the roles need.
struct UnitView {
  int n_a, n_b;  // key blocks of tile A (the unit's length) and of tile B (0: no tile B)
};

__device__ __forceinline__ UnitView unit_view(const int32_t* u) {
  UnitView v;
  v.n_a = u[kUKbEnd] - u[kUKbBegin];
  v.n_b = u[kUQCountB] > 0 ? u[kUKbEndB] - u[kUKbBegin] : 0;
  return v;
}

__device__ __forceinline__ bool unit_inflight(const Params& p, const int32_t* u) {
  return p.inflight && u[kUSelfRow] >= 0;
}

// Row (slot) of the first key of 128-key block `kb` of a unit.  In-flight unit: rows of
// the in-flight K/V from the sequence's first query row.  Paged mode (block_tables !=
// NULL, block_size % 128 == 0): through the block table.  Contiguous mode (block_tables
// == NULL): key rows of the sequence start at k_base.
__device__ __forceinline__ int key_block_slot(const Params& p, const int32_t* u, int kb) {
  const int key0 = kb * BN;
  int64_t slot;
  if (unit_inflight(p, u)) {
    slot = (int64_t)u[kUSelfRow] + key0;  // box may run past the end: zero fill, masked
  } else if (p.block_tables != nullptr) {
    const int page = __ldg(p.block_tables + (int64_t)u[kUSeq] * p.bt_stride + key0 / p.block_size);
    slot = (int64_t)page * p.block_size + (key0 % p.block_size);
    if (page < 0 || slot + BN > p.num_slots) {
      record_error(VLC_DEV_ERR_BLOCK_RANGE);
      slot = p.num_slots;  // fully out of range -> TMA zero fill
    }
  } else {
    slot = (int64_t)u[kUKBase] + key0;  // box may run past the end: zero fill, masked
  }
  return (int)slot;
}

// Descriptor low words: q_lo / k_lo / v_lo address the tile's first byte; the K
// steps of 16 add compile-time offsets (K-major: +32 B per step within a 64-column
// half, +16 KB to the second half; MN-major V: +2 KB per 16 keys).
constexpr uint32_t DESC_HI = umma_desc_sw128_hi(1024);

// kSteps: 16-column steps of the head dim that are multiplied (head dim 80: 5, the padding
// columns skipped; otherwise all 8).
template <int kSteps = HD / 16>
__device__ __forceinline__ void issue_qk(uint32_t d_tmem, uint32_t q_lo, uint32_t k_lo) {
#pragma unroll
  for (int k = 0; k < kSteps; ++k) {
    const uint32_t off = (uint32_t)(((k >> 2) * HALF_BYTES + (k & 3) * 32) >> 4);
    umma_ss_w(d_tmem, q_lo + off, DESC_HI, k_lo + off, DESC_HI, IDESC_QK, k > 0 ? 1u : 0u);
  }
}

// O += P V over keys [64 half, 64 half + 64) of the block; kIdesc sets N (the O columns
// computed: 80 for head dim 80, else 128).
template <uint32_t kIdesc = IDESC_PV>
__device__ __forceinline__ void issue_pv_half(uint32_t o_tmem, uint32_t p_tmem, uint32_t v_lo, int half,
                                              bool accumulate) {
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int kk = half * 4 + k;
    umma_ts_w(o_tmem, p_tmem + kk * 8, v_lo + (uint32_t)((kk * 2048) >> 4), DESC_HI, kIdesc,
              (accumulate || kk > 0) ? 1u : 0u);
  }
}

// kPacked: the plan packs several short sequences per tile (block-diagonal mask); a separate
// instantiation, so the causal path's code is not touched by it.  kDK: 16-column steps of
// the head dim in the MMAs (5 for head dim 80: Q K^T over its 80 columns and P V with N =
// 80, instead of the zero-padded 128; 8 otherwise).  O columns past 16 kDK are never
// written (nor stored: the epilogue writes the head dim's columns only).
template <bool kPacked, int kDK>
__global__ void __launch_bounds__(NUM_THREADS, 1) prefill_attn_kernel(const __grid_constant__ Params p) {
  constexpr uint32_t kIdescPV = umma_idesc_bf16(128, 16 * kDK, false, true);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const Bars bars = make_bars(smem);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + OFF_MISC + 4);

  const int warp = warp_id();
  const int lane = lane_id();
  const int u_begin = __ldg(p.cta_offsets + blockIdx.x);
  const int u_end = __ldg(p.cta_offsets + blockIdx.x + 1);

  if (warp == 9) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  if (threadIdx.x == 0) {
    *abort_flag = 0;
    for (int b = 0; b < QSLOTS; ++b) {
      mbar_init(bars.q_full + b, 1);
      mbar_init(bars.q_empty + b, 1);
    }
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bars.k_full + s, 1);
      mbar_init(bars.k_empty + s, 1);
      mbar_init(bars.v_full + s, 1);
      mbar_init(bars.v_empty + s, 1);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(bars.s_full + x, 1);
      mbar_init(bars.p_lo + x, kTileThreads);
      mbar_init(bars.p_hi + x, kTileThreads);
      mbar_init(bars.o_done + x, 1);
    }
    fence_mbar_init();
  }
  if (threadIdx.x == 0) pdl_launch_dependents();  // the merge may be scheduled as SMs free up
  if (warp == 8 && lane == 0) {
    tma_prefetch_desc(&p.tm_k);
    tma_prefetch_desc(&p.tm_v);
    if (p.inflight) {
      tma_prefetch_desc(&p.tm_kn);
      tma_prefetch_desc(&p.tm_vn);
    }
  }
  if (warp == 10 && lane == 0) {
    tma_prefetch_desc(&p.tm_q);
    tma_prefetch_desc(&p.tm_o128);
    tma_prefetch_desc(&p.tm_p128);
  }
  // Rows beyond T*G of the Q slots are never written by TMA: zero them once so
  // the unused accumulator rows stay finite.
  for (int i = threadIdx.x; i < QSLOTS * BM; i += NUM_THREADS) {
    const int r = i & 127;
    if (r >= p.rows) {
      const uint4 z = make_uint4(0, 0, 0, 0);
      uint8_t* q = smem + OFF_Q + (i >> 7) * TILE_BYTES;
      uint4* r0 = reinterpret_cast<uint4*>(q + r * 128);
      uint4* r1 = reinterpret_cast<uint4*>(q + HALF_BYTES + r * 128);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        r0[k] = z;
        r1[k] = z;
      }
    }
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 10) {
    // ------------------------------------------------------------ Q producer
    if (lane == 0) {
      // The plan is never written by the kernel launched just before (only q/k/v
      // are): the first unit's fields load while the wait runs.
      int g = 0, ntile = 0, q_a = 0, q_b = 0;
      auto fetch = [&](int ui) {
        const int32_t* u = p.units + (int64_t)ui * kUnitInts;
        g = u[kUKvHead];
        ntile = u[kUQCountB] > 0 ? 2 : 1;
        q_a = u[kUQBeginA];
        q_b = u[kUQBeginB];
      };
      if (u_begin < u_end) fetch(u_begin);
      if (!p.inflight) pdl_wait();  // Q may be written by the preceding kernel
      int load = 0;
      for (int ui = u_begin; ui < u_end; ++ui) {
        if (ui != u_begin) fetch(ui);
        bool ok = true;
        for (int x = 0; x < ntile; ++x, ++load) {
          const int slot = load % QSLOTS;
          if (load >= QSLOTS && !wait_or_abort(bars.q_empty + slot, (uint32_t)((load / QSLOTS) & 1) ^ 1u,
                                               VLC_DEV_ERR_TIMEOUT + 1, abort_flag)) {
            ok = false;
            break;
          }
          const int q_begin = x == 0 ? q_a : q_b;
          // At launch every CTA loads at once and HBM is the limit: the first tile's Q
          // (an operand of the first Q K^T) lands before the second tile's is requested.
          if (load == 1 && !wait_or_abort(bars.q_full + 0, 0u, VLC_DEV_ERR_TIMEOUT + 1, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* qdst = smem + OFF_Q + slot * TILE_BYTES;
          mbar_expect_tx(bars.q_full + slot, 2 * p.rows * 128);
          tma_load_3d(qdst, &p.tm_q, bars.q_full + slot, 0, g * p.group, q_begin);
          tma_load_3d(qdst + HALF_BYTES, &p.tm_q, bars.q_full + slot, 64, g * p.group, q_begin);
        }
        if (!ok) break;
      }
    }
  } else if (warp == 8) {
    // ------------------------------------------------------------ K/V producer
    if (lane == 0) {
      // Plan and block tables are never written by the kernel launched just before:
      // the first unit's fields and its first page are read while the wait runs.
      int g = 0, kb0 = 0, kb1 = 0, slot0 = 0;
      bool infl = false;
      const int32_t* u = nullptr;
      auto fetch = [&](int ui) {
        u = p.units + (int64_t)ui * kUnitInts;
        g = u[kUKvHead];
        kb0 = u[kUKbBegin];
        kb1 = u[kUKbEnd];
        infl = unit_inflight(p, u);
        slot0 = kb0 < kb1 ? key_block_slot(p, u, kb0) : 0;
      };
      if (u_begin < u_end) fetch(u_begin);
      bool waited = false;  // K/V rows (paged or contiguous) may be written by the preceding kernel
      int it = 0;
      for (int ui = u_begin; ui < u_end; ++ui) {
        if (ui != u_begin) fetch(ui);
        if (!infl && !waited) {
          pdl_wait();
          waited = true;
        }
        const CUtensorMap* tk = infl ? &p.tm_kn : &p.tm_k;
        const CUtensorMap* tv = infl ? &p.tm_vn : &p.tm_v;
        bool ok = true;
        // A packed unit's tile B has a key block of its own (its rows), next in the ring.
        const int kb_end = kPacked && u[kUQCountB] > 0 ? kb0 + 2 : kb1;
        for (int kb = kb0; kb < kb_end; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
          const int slot = kb == kb0 ? slot0 : kPacked ? u[kUQBeginB] : key_block_slot(p, u, kb);
          if (it >= STAGES && !wait_or_abort(bars.k_empty + s, ph ^ 1u, VLC_DEV_ERR_TIMEOUT + 2, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* kdst = smem + OFF_K + s * TILE_BYTES;
          mbar_expect_tx(bars.k_full + s, TILE_BYTES);
          tma_load_3d(kdst, tk, bars.k_full + s, 0, g, slot);
          tma_load_3d(kdst + HALF_BYTES, tk, bars.k_full + s, 64, g, slot);
          if (it >= STAGES && !wait_or_abort(bars.v_empty + s, ph ^ 1u, VLC_DEV_ERR_TIMEOUT + 3, abort_flag)) {
            ok = false;
            break;
          }
          // Likewise the first K block lands before V and the next blocks are requested.
          if (it == 0 && !wait_or_abort(bars.k_full + 0, 0u, VLC_DEV_ERR_TIMEOUT + 3, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* vdst = smem + OFF_V + s * TILE_BYTES;
          mbar_expect_tx(bars.v_full + s, TILE_BYTES);
          tma_load_3d(vdst, tv, bars.v_full + s, 0, g, slot);
          tma_load_3d(vdst + HALF_BYTES, tv, bars.v_full + s, 64, g, slot);
        }
        if (!ok) break;
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issuer
    // Step j of a unit (K/V block kv = it + j): for tile A then tile B (while it has
    // blocks): O += P(j) V(j), then S = Q K(j+1)^T.  At the unit's last step the
    // next Q K^T is the next unit's block 0 (same K/V ring, next Q slots), so the
    // softmax warps start the next unit while this one drains.
    if (lane == 0 && u_begin < u_end) {
      const uint32_t q_lo = umma_desc_sw128_lo(smem_u32(smem + OFF_Q), 16);
      const uint32_t k_lo = umma_desc_sw128_lo(smem_u32(smem + OFF_K), 16);
      const uint32_t v_lo = umma_desc_sw128_lo(smem_u32(smem + OFF_V), HALF_BYTES);
      constexpr uint32_t kTileLo = TILE_BYTES >> 4;  // one tile in descriptor address units
      int qload = 0;  // Q loads consumed (slot = load % QSLOTS, same order as the Q producer)
      struct Cur {
        UnitView v;
        int load_a, load_b;
      };
      auto next_unit = [&](int ui) {
        Cur c;
        c.v = unit_view(p.units + (int64_t)ui * kUnitInts);
        c.load_a = qload++;
        c.load_b = c.v.n_b > 0 ? qload++ : -1;
        return c;
      };
      auto wait_k = [&](int kv) {
        return wait_or_abort(bars.k_full + kv % STAGES, (uint32_t)(kv / STAGES) & 1u, VLC_DEV_ERR_TIMEOUT + 7,
                             abort_flag);
      };
      // S_x = Q(load) K(kv)^T; `first`: the tile's first block (wait for its Q),
      // `last`: its last block (release the Q slot once the MMA completes).
      auto qk = [&](int x, int load, int kv, bool first, bool last) {
        const int slot = load % QSLOTS;
        if (first && !wait_or_abort(bars.q_full + slot, (uint32_t)(load / QSLOTS) & 1u, VLC_DEV_ERR_TIMEOUT + 6,
                                    abort_flag))
          return false;
        tc_fence_after();
        issue_qk<kDK>(tmem_base + TMEM_S + x * 128, q_lo + slot * kTileLo, k_lo + (kv % STAGES) * kTileLo);
        umma_commit(bars.s_full + x);
        if (last) umma_commit(bars.q_empty + slot);
        return true;
      };
      if constexpr (kPacked) {
        // Packed units: tile A and tile B (when present) each have one key block of their
        // own, ring blocks r and r + 1.  Order: S_A, S_B of the first unit; then per unit
        // O_A += P_A V_A, the next unit's S_A, O_B += P_B V_B, the next unit's S_B.
        struct PU {
          bool has_b;
          int load_a, load_b, ra, rb;
        };
        int r = 0, pv_a = 0, pv_b = 0;
        auto fetch_pu = [&](int ui) {
          PU c;
          c.has_b = p.units[(int64_t)ui * kUnitInts + kUQCountB] > 0;
          c.load_a = qload++;
          c.load_b = c.has_b ? qload++ : -1;
          c.ra = r++;
          c.rb = c.has_b ? r++ : -1;
          return c;
        };
        auto qk1 = [&](int x, int load, int rb) {  // a tile's only block: first and last
          if (!wait_k(rb)) return false;
          if (!qk(x, load, rb, true, true)) return false;
          umma_commit(bars.k_empty + rb % STAGES);
          return true;
        };
        auto pv1 = [&](int x, int rb, int& pvc) {
          const int s = rb % STAGES;
          if (!wait_or_abort(bars.v_full + s, (uint32_t)(rb / STAGES) & 1u, VLC_DEV_ERR_TIMEOUT + 5, abort_flag) ||
              !wait_or_abort(bars.p_lo + x, (uint32_t)pvc & 1u, VLC_DEV_ERR_TIMEOUT + 4, abort_flag))
            return false;
          tc_fence_after();
          issue_pv_half<kIdescPV>(tmem_base + TMEM_O + x * 128, tmem_base + TMEM_S + x * 128, v_lo + s * kTileLo, 0, false);
          if (!wait_or_abort(bars.p_hi + x, (uint32_t)pvc & 1u, VLC_DEV_ERR_TIMEOUT + 4, abort_flag)) return false;
          tc_fence_after();
          issue_pv_half<kIdescPV>(tmem_base + TMEM_O + x * 128, tmem_base + TMEM_S + x * 128, v_lo + s * kTileLo, 1, true);
          ++pvc;
          umma_commit(bars.o_done + x);
          umma_commit(bars.v_empty + s);
          return true;
        };
        PU pc = fetch_pu(u_begin);
        bool pok = qk1(0, pc.load_a, pc.ra) && (!pc.has_b || qk1(1, pc.load_b, pc.rb));
        for (int ui = u_begin; pok && ui < u_end; ++ui) {
          const bool has_next = ui + 1 < u_end;
          PU pn{};
          if (has_next) pn = fetch_pu(ui + 1);
          pok = pv1(0, pc.ra, pv_a) && (!has_next || qk1(0, pn.load_a, pn.ra));
          if (pok && pc.has_b) pok = pv1(1, pc.rb, pv_b);
          if (pok && has_next && pn.has_b) pok = qk1(1, pn.load_b, pn.rb);
          pc = pn;
        }
      }
      Cur cur{};
      bool ok = !kPacked;
      if (!kPacked) {
        cur = next_unit(u_begin);
        ok = wait_k(0) && qk(0, cur.load_a, 0, true, cur.v.n_a == 1) &&
             (cur.v.n_b == 0 || qk(1, cur.load_b, 0, true, cur.v.n_b == 1));
      }
      if (ok) umma_commit(bars.k_empty + 0);
      int pv_a = 0, pv_b = 0;  // P*V issued per tile (p_lo / p_hi phases)
      int it = 0;              // K/V block index of the current unit's block 0
      for (int ui = u_begin; ok && ui < u_end; ++ui) {
        const bool has_next = ui + 1 < u_end;
        Cur nxt{};
        if (has_next) nxt = next_unit(ui + 1);
        for (int j = 0; j < cur.v.n_a; ++j) {
          const int kv = it + j, s = kv % STAGES;
          const bool last = j == cur.v.n_a - 1;
          const bool more = !last || has_next;  // a block kv + 1 follows
          // tile A
          if (!wait_or_abort(bars.p_lo + 0, (uint32_t)pv_a & 1u, VLC_DEV_ERR_TIMEOUT + 4, abort_flag) ||
              !wait_or_abort(bars.v_full + s, (uint32_t)(kv / STAGES) & 1u, VLC_DEV_ERR_TIMEOUT + 5, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_pv_half<kIdescPV>(tmem_base + TMEM_O, tmem_base + TMEM_S, v_lo + s * kTileLo, 0, j > 0);
          if (!wait_or_abort(bars.p_hi + 0, (uint32_t)pv_a & 1u, VLC_DEV_ERR_TIMEOUT + 4, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_pv_half<kIdescPV>(tmem_base + TMEM_O, tmem_base + TMEM_S, v_lo + s * kTileLo, 1, true);
          ++pv_a;
          if (last) umma_commit(bars.o_done + 0);
          if (more && !wait_k(kv + 1)) {
            ok = false;
            break;
          }
          if (!last)
            ok = qk(0, cur.load_a, kv + 1, false, j + 1 == cur.v.n_a - 1);
          else if (has_next)
            ok = qk(0, nxt.load_a, kv + 1, true, nxt.v.n_a == 1);
          if (!ok) break;
          // tile B
          if (j < cur.v.n_b) {
            if (!wait_or_abort(bars.p_lo + 1, (uint32_t)pv_b & 1u, VLC_DEV_ERR_TIMEOUT + 8, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_pv_half<kIdescPV>(tmem_base + TMEM_O + 128, tmem_base + TMEM_S + 128, v_lo + s * kTileLo, 0, j > 0);
            if (!wait_or_abort(bars.p_hi + 1, (uint32_t)pv_b & 1u, VLC_DEV_ERR_TIMEOUT + 8, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_pv_half<kIdescPV>(tmem_base + TMEM_O + 128, tmem_base + TMEM_S + 128, v_lo + s * kTileLo, 1, true);
            ++pv_b;
            if (j == cur.v.n_b - 1)
              umma_commit(bars.o_done + 1);
            else
              ok = qk(1, cur.load_b, kv + 1, false, j + 1 == cur.v.n_b - 1);
            if (!ok) break;
          }
          if (last && has_next && nxt.v.n_b > 0) {
            ok = qk(1, nxt.load_b, kv + 1, true, nxt.v.n_b == 1);
            if (!ok) break;
          }
          umma_commit(bars.v_empty + s);
          if (more) umma_commit(bars.k_empty + (kv + 1) % STAGES);
        }
        it += cur.v.n_a;
        cur = nxt;
      }
    }
  } else {
    // ------------------------------------------------------------ softmax (one warpgroup per tile)
    const int x = warp >> 2;            // 0: tile A, 1: tile B
    const int row = threadIdx.x & 127;  // == TMEM lane
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t s_addr = tmem_base + lane_off + TMEM_S + x * 128;
    const uint32_t o_addr = tmem_base + lane_off + TMEM_O + x * 128;
    int t = 0;      // blocks of this tile processed (s_full / p_lo / p_hi phases)
    int nunit = 0;  // units of this tile finished (o_done phases)
    int ring = 0;   // K/V ring blocks of the CTA's earlier units
    int qload = 0;  // Q loads of this CTA so far (the Q producer's order)
    for (int ui = u_begin; ui < u_end; ++ui) {
      const int32_t* u = p.units + (int64_t)ui * kUnitInts;
      const UnitView uv = unit_view(u);
      const int n = x == 0 ? uv.n_a : uv.n_b;
      const int my_load = qload + x;
      qload += u[kUQCountB] > 0 ? 2 : 1;
      // packed: tile B's keys are its own rows, in the ring block after tile A's
      const int ring0 = ring + (kPacked && x == 1 ? 1 : 0);
      ring += kPacked ? (u[kUQCountB] > 0 ? 2 : 1) : uv.n_a;
      if (n == 0) continue;
      // The tile's Q slot is free for the epilogue when fewer than QSLOTS loads follow
      // this tile's (no later Q lands in it).
      int after = qload - 1 - my_load;
      for (int uj = ui + 1; uj < u_end && after < QSLOTS; ++uj)
        after += p.units[(int64_t)uj * kUnitInts + kUQCountB] > 0 ? 2 : 1;
      const bool own_slot = after < QSLOTS;
      const int g = u[kUKvHead];
      const int kb0 = u[kUKbBegin];
      const int kv_len = kPacked && x == 1 ? u[kUQCountB] : u[kUKvLen];
      const int q_begin = u[x == 0 ? kUQBeginA : kUQBeginB];
      const int q_count = u[x == 0 ? kUQCountA : kUQCountB];
      const int kpos0 = u[x == 0 ? kUKpos0A : kUKpos0B];
      const int part = u[x == 0 ? kUPartA : kUPartB];
      const int tok = row / p.group;
      const bool row_valid = row < p.rows && tok < q_count;
      const int qpos = p.causal ? kpos0 + tok : kpos0;  // non-causal: kpos0 = k_len - 1

      float m_use = -INFINITY;
      float l_row = 0.f;
      bool ok = true;
      for (int j = 0; j < n; ++j, ++t) {
        if (!wait_or_abort(bars.s_full + x, (uint32_t)t & 1u, VLC_DEV_ERR_TIMEOUT + 9, abort_flag)) {
          ok = false;
          break;
        }
        __syncwarp();
        tc_fence_after();
        const int key0 = (kb0 + j) * BN;
        uint32_t sr[128];
#pragma unroll
        for (int q = 0; q < 4; ++q) tmem_ld32(s_addr + q * 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[q * 32]));
        tmem_wait_ld();
        if (kPacked) {
          // Packed tile (several short sequences, one key block = the same tokens): the row
          // sees keys [lo, hi) of the block, its own sequence's; rows past q_count none.
          int lo = 0, hi = 0;
          if (row_valid) {
            const int k_base = x == 1 ? u[kUQBeginB] : u[kUKBase];
            lo = __ldg(p.segments + 2 * (int64_t)(q_begin + tok)) - k_base;
            hi = __ldg(p.segments + 2 * (int64_t)(q_begin + tok) + 1) - k_base;
          }
#pragma unroll
          for (int c = 0; c < 128; ++c)
            if (c < lo || c >= hi) sr[c] = __float_as_uint(-INFINITY);
        } else if (key0 + BN - 1 > kpos0) {  // block touches the causal diagonal
          const int lim = qpos - key0;
#pragma unroll
          for (int c = 0; c < 128; ++c)
            if (c > lim) sr[c] = __float_as_uint(-INFINITY);
        }
        float mx[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) mx[k] = __uint_as_float(sr[k]);
#pragma unroll
        for (int c = 8; c < 128; c += 16)
#pragma unroll
          for (int k = 0; k < 8; ++k) mx[k] = fmax3(mx[k], __uint_as_float(sr[c + k]), __uint_as_float(sr[c + 8 + k]));
        const float m_tile = fmaxf(fmax3(mx[0], mx[1], mx[2]), fmax3(fmax3(mx[3], mx[4], mx[5]), mx[6], mx[7])) *
                             p.scale_log2;
        // Lazy rescaling: only move the reference max when it grows by > 2^8.
        const bool need = m_tile > m_use + 8.0f;
        const float m_new = need ? m_tile : m_use;
        const float f = (need && m_use != -INFINITY) ? fast_exp2(m_use - m_new) : 1.0f;
        m_use = m_new;
        const float mref = (m_use == -INFINITY) ? 0.f : m_use;
        // Keys past the sequence end: zero their V rows so 0 * garbage stays 0.  Tile A
        // has every block of the unit, and its P*V runs first.
        if ((kPacked || x == 0) && key0 + BN > kv_len) {
          const int rb = kPacked ? ring0 : t;  // ring index of this block (tile A's count = the ring's)
          const int st = rb % STAGES;
          if (!wait_or_abort(bars.v_full + st, (uint32_t)(rb / STAGES) & 1u, VLC_DEV_ERR_TIMEOUT + 11, abort_flag)) {
            ok = false;
            break;
          }
          if (key0 + row >= kv_len) {
            const uint4 z = make_uint4(0, 0, 0, 0);
            uint4* v0 = reinterpret_cast<uint4*>(smem + OFF_V + st * TILE_BYTES + row * 128);
            uint4* v1 = reinterpret_cast<uint4*>(smem + OFF_V + st * TILE_BYTES + HALF_BYTES + row * 128);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              v0[i] = z;
              v1[i] = z;
            }
          }
          fence_proxy_async_smem();
        }
        // P = exp2(s * scale_log2 - mref) as bf16 pairs: key pair (2c, 2c+1) goes to S
        // column c (its register is free: pair c reads registers 2c and 2c+1 >= c).  Each
        // half of the keys is released to the MMA as soon as it is in TMEM.
        const uint64_t scale2 = f2_pack(p.scale_log2, p.scale_log2);
        const uint64_t negm2 = f2_pack(-mref, -mref);
        uint64_t lsum = f2_pack(0.f, 0.f);
#pragma unroll
        for (int half = 0; half < 2; ++half) {
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            const int base = half * 64 + q * 32;
#pragma unroll
            for (int c = 0; c < 16; ++c) {
              const uint64_t x2 =
                  f2_fma(f2_pack(__uint_as_float(sr[base + 2 * c]), __uint_as_float(sr[base + 2 * c + 1])), scale2,
                         negm2);
              float x0, x1;
              f2_unpack(x2, x0, x1);
              const float e0 = fast_exp2(x0), e1 = fast_exp2(x1);
              lsum = f2_add(lsum, f2_pack(e0, e1));
              sr[base + c] = pack_bf16x2(e0, e1);
            }
            tmem_st16(s_addr + (base >> 1), *reinterpret_cast<uint32_t(*)[16]>(&sr[base]));
          }
          if (half == 0 && __any_sync(0xffffffffu, f != 1.0f)) {
            // O (stable: P(j-1) V(j-1) completed before S(j)) follows the moved max
            // before this block's P V starts.
#pragma unroll 1
            for (int cb = 0; cb < 8; ++cb) {
              uint32_t orr[16];
              tmem_ld16(o_addr + cb * 16, orr);
              tmem_wait_ld();
#pragma unroll
              for (int c = 0; c < 16; ++c) orr[c] = __float_as_uint(__uint_as_float(orr[c]) * f);
              tmem_st16(o_addr + cb * 16, orr);
            }
            l_row *= f;
          }
          tmem_wait_st();
          tc_fence_before();
          mbar_arrive(half == 0 ? bars.p_lo + x : bars.p_hi + x);
        }
        {
          float l0, l1;
          f2_unpack(lsum, l0, l1);
          l_row += l0 + l1;
        }
      }
      if (!ok) break;
      // ---------------------------------------------------------- epilogue
      if (!wait_or_abort(bars.o_done + x, (uint32_t)nunit & 1u, VLC_DEV_ERR_TIMEOUT + 12, abort_flag)) break;
      ++nunit;
      __syncwarp();
      tc_fence_after();
      const float inv = l_row > 0.f ? 1.0f / l_row : 0.f;
      __nv_bfloat16* dst;
      if (part < 0) {
        const int head = g * p.group + (row - tok * p.group);
        dst = p.out + (int64_t)(q_begin + tok) * p.out_token_stride + (int64_t)head * p.head_dim;
      } else {
        // Split partial: O / l as bf16 (the merge re-weights by l and the max).
        dst = p.part_o + ((int64_t)part * BM + row) * HD;
        reinterpret_cast<float2*>(p.part_ml)[(int64_t)part * BM + row] = make_float2(m_use, l_row);
      }
      const bool store = part < 0 ? row_valid : true;
      uint32_t orr[128];
#pragma unroll
      for (int q = 0; q < 4; ++q) tmem_ld32(o_addr + q * 32, *reinterpret_cast<uint32_t(*)[32]>(&orr[q * 32]));
      tmem_wait_ld();
#pragma unroll
      for (int c = 0; c < 64; ++c)
        orr[c] = pack_bf16x2(__uint_as_float(orr[2 * c]) * inv, __uint_as_float(orr[2 * c + 1]) * inv);
      if (own_slot && (part >= 0 || q_count == p.tokens_per_tile)) {
        // Full tile or split partial, Q slot free: the whole tile goes into the slot
        // in the Q load's layout (128-byte swizzle: 16-byte chunk c of row r of a
        // 64-column half at chunk c ^ (r % 8)) and leaves with two TMA stores.  The
        // slot's last reader, this tile's final Q K^T, completed before o_done.
        uint8_t* qs = smem + OFF_Q + (my_load % QSLOTS) * TILE_BYTES;
#pragma unroll
        for (int k = 0; k < 16; ++k)
          *reinterpret_cast<uint4*>(qs + (k >> 3) * HALF_BYTES + row * 128 + (((k & 7) ^ (row & 7)) << 4)) =
              make_uint4(orr[4 * k], orr[4 * k + 1], orr[4 * k + 2], orr[4 * k + 3]);
        fence_proxy_async_smem();
        named_bar_sync(1 + x, kTileThreads);
        if (row == 0) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            if (part < 0) {
              if (64 * h < p.head_dim)  // columns past head_dim are the zero padding
                tma_store_3d(&p.tm_o128, qs + h * HALF_BYTES, 64 * h, g * p.group, q_begin);
            } else {
              tma_store_2d(&p.tm_p128, qs + h * HALF_BYTES, 64 * h, part * BM);
            }
          }
          bulk_commit_group();
        }
      } else if (kPacked && (part >= 0 || q_count == p.tokens_per_tile) && (part >= 0 || p.out_store32)) {
        // Packed tiles (whose units are one block each, so an epilogue follows every block):
        // each thread writes its row with 32-byte stores (full sectors).  Measured faster than
        // the staged stores below for the vision windows (4K image 135 vs 148 us); for the
        // causal kernel they measured slower (cfg3 batch 207 vs 199 us), so it stages.
#pragma unroll
        for (int c = 0; c < 8; ++c)
          if (c * 16 < p.head_dim) st_global_v8(dst + c * 16, *reinterpret_cast<const uint32_t(*)[8]>(&orr[c * 8]));
      } else if (part >= 0 || q_count == p.tokens_per_tile) {
        // Full tile or split partial: stage 32 columns at a time in shared memory,
        // alternating two buffers (64-byte swizzle: 16-byte chunk c of row r at chunk
        // c ^ ((r / 2) % 4)), and let one thread write each with a TMA tensor store.
        uint8_t* stg = smem + OFF_STG + x * STG_TILE;
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          uint8_t* buf = stg + (r & 1) * STG_BUF;
          if (row == 0) bulk_wait_read_allbut1();  // the store that used this buffer has read it
          named_bar_sync(1 + x, kTileThreads);
#pragma unroll
          for (int c = 0; c < 4; ++c)
            *reinterpret_cast<uint4*>(buf + row * 64 + ((c ^ ((row >> 1) & 3)) << 4)) =
                make_uint4(orr[16 * r + 4 * c], orr[16 * r + 4 * c + 1], orr[16 * r + 4 * c + 2],
                           orr[16 * r + 4 * c + 3]);
          fence_proxy_async_smem();
          named_bar_sync(1 + x, kTileThreads);
          if (row == 0) {
            if (part < 0) {
              if (32 * r < p.head_dim) tma_store_3d(&p.tm_o, buf, 32 * r, g * p.group, q_begin);
            } else {
              tma_store_2d(&p.tm_p, buf, 32 * r, part * BM);
            }
            bulk_commit_group();
          }
        }
      } else if (store) {
        // Last, partial tile of a sequence: the tensor store would write the rows of
        // the following tokens, so each valid row is written directly.
        if (p.out_store32) {
#pragma unroll
          for (int c = 0; c < 8; ++c)
            if (c * 16 < p.head_dim)
              st_global_v8(dst + c * 16, *reinterpret_cast<const uint32_t(*)[8]>(&orr[c * 8]));
        } else {
#pragma unroll
          for (int c = 0; c < 16; ++c)
            if (c * 8 < p.head_dim)
              *reinterpret_cast<uint4*>(dst + c * 8) =
                  make_uint4(orr[4 * c], orr[4 * c + 1], orr[4 * c + 2], orr[4 * c + 3]);
        }
      }
      tc_fence_before();
    }
    if (row == 0) bulk_wait_all();  // this tile's output stores are complete
  }

  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}


namespace quad {
constexpr int KHALF_BYTES = 64 * 128;  // 64 keys x 64 dims (bf16): one dim-half of a CTA's K rows
// v_landed barriers after prefill_attn_kernel's barriers (the odd CTA's)
constexpr int QD_OFF_VL = OFF_BAR + NUM_BARS * 8;
constexpr int QD_OFF_MISC = QD_OFF_VL + STAGES * 8;
constexpr int QD_SMEM_BYTES = QD_OFF_MISC + 16 + 1024;
static_assert(QD_SMEM_BYTES <= 232448, "shared memory budget");
constexpr uint32_t IDESC_QK2 = umma_idesc_bf16(256, 128, false, false);
constexpr uint32_t IDESC_PV2 = umma_idesc_bf16(256, 128, false, true);
}  // namespace quad

// tcgen05 commit to the same barrier in both CTAs of the pair (one commit each).
__device__ __forceinline__ void commit_both(uint64_t* bar) { umma_commit_pair_both(bar); }

// S = Q K^T on the pair: A = this CTA's 128 Q rows (two 64-dim halves of 16 KB), B = this CTA's
// 64 K rows (two 64-dim halves of 8 KB); M = 256, N = 128.
__device__ __forceinline__ void issue_qk_quad(uint32_t d_tmem, uint32_t q_lo, uint32_t k_lo) {
#pragma unroll
  for (int k = 0; k < HD / 16; ++k) {
    const uint32_t qa = (uint32_t)(((k >> 2) * HALF_BYTES + (k & 3) * 32) >> 4);
    const uint32_t kb = (uint32_t)(((k >> 2) * quad::KHALF_BYTES + (k & 3) * 32) >> 4);
    umma_ss_pair(d_tmem, q_lo + qa, DESC_HI, k_lo + kb, DESC_HI, quad::IDESC_QK2, k > 0 ? 1u : 0u);
  }
}

// O += P V on the pair over keys [64 half, 64 half + 64): A = P from each CTA's TMEM, B = this
// CTA's 64 dims of the V block (MN-major, one 128-row half).
__device__ __forceinline__ void issue_pv_half_quad(uint32_t o_tmem, uint32_t p_tmem, uint32_t v_lo, int half,
                                                   bool accumulate) {
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int kk = half * 4 + k;
    umma_ts_pair(o_tmem, p_tmem + kk * 8, v_lo + (uint32_t)((kk * 2048) >> 4), DESC_HI, quad::IDESC_PV2,
                 (accumulate || kk > 0) ? 1u : 0u);
  }
}

// Quad units on CTA pairs (clusters of 2, tcgen05.mma.cta_group::2).  A quad is four query
// tiles of one (sequence, KV head) over one key range: tiles A0, B0 in the pair's even CTA
// (rank 0, the leader) and A1, B1 in the odd one, with the same roles, TMEM layout and
// softmax as prefill_attn_kernel.  The leader issues every MMA of the pair: S_X = Q_X K^T
// with M = 256 (each CTA's own 128 Q rows; each CTA holds half of the K block, keys
// [64 r, 64 r + 64)) and O_X += P_X V (P from each CTA's TMEM; each CTA holds half of the
// V block, dims [64 r, 64 r + 64)).  Per SM, K/V loads and Q K^T operand reads halve.
//   * both CTAs' TMA loads complete on the leader's q_full / k_full / v_full, armed by the
//     leader for both CTAs' bytes;
//   * both CTAs' softmax warps arrive on the leader's p_lo / p_hi (256 arrivals);
//   * the leader's MMAs signal s_full, o_done and the ring's empty barriers in both CTAs
//     (one commit per CTA), and the leader's issuer tells the odd CTA that a V block has
//     landed (v_landed: the odd CTA zeroes its rows past the sequence end);
//   * cluster barriers after set-up and before exit.
// A ghost tile (kUPart == kGhostPart) fills a quad short of four tiles: it runs like its
// sibling but writes nothing.
template <bool kPacked>
__global__ void __launch_bounds__(NUM_THREADS, 1) prefill_attn_quad_kernel(const __grid_constant__ Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const Bars bars = make_bars(smem);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + quad::QD_OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + quad::QD_OFF_MISC + 4);

  const int warp = warp_id();
  const int lane = lane_id();
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int u_begin = __ldg(p.cta_offsets + (blockIdx.x >> 1));
  const int u_end = __ldg(p.cta_offsets + (blockIdx.x >> 1) + 1);
  uint64_t* v_landed = reinterpret_cast<uint64_t*>(smem + quad::QD_OFF_VL);  // [STAGES], odd CTA
  auto unit_rec = [&](int ui) { return p.units + (2 * (int64_t)ui + rank) * kUnitInts; };

  if (warp == 9) {
    tmem_alloc_pair(tmem_slot, TMEM_COLS);
    tmem_relinquish_pair();
  }
  if (threadIdx.x == 0) {
    *abort_flag = 0;
    for (int b = 0; b < QSLOTS; ++b) {
      mbar_init(bars.q_full + b, 1);
      mbar_init(bars.q_empty + b, 1);
    }
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bars.k_full + s, 1);
      mbar_init(bars.k_empty + s, 1);
      mbar_init(bars.v_full + s, 1);
      mbar_init(bars.v_empty + s, 1);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(bars.s_full + x, 1);
      mbar_init(bars.p_lo + x, 2 * kTileThreads);  // both CTAs' rows (leader's barriers)
      mbar_init(bars.p_hi + x, 2 * kTileThreads);
      mbar_init(bars.o_done + x, 1);
    }
    for (int s = 0; s < STAGES; ++s) mbar_init(v_landed + s, 1);
    fence_mbar_init();
  }
  if (threadIdx.x == 0) pdl_launch_dependents();  // the merge may be scheduled as SMs free up
  if (warp == 8 && lane == 0) {
    tma_prefetch_desc(&p.tm_k);
    tma_prefetch_desc(&p.tm_v);
    if (p.inflight) {
      tma_prefetch_desc(&p.tm_kn);
      tma_prefetch_desc(&p.tm_vn);
    }
  }
  if (warp == 10 && lane == 0) {
    tma_prefetch_desc(&p.tm_q);
    tma_prefetch_desc(&p.tm_o128);
    tma_prefetch_desc(&p.tm_p128);
  }
  // Rows beyond T*G of the Q slots are never written by TMA: zero them once so
  // the unused accumulator rows stay finite.
  for (int i = threadIdx.x; i < QSLOTS * BM; i += NUM_THREADS) {
    const int r = i & 127;
    if (r >= p.rows) {
      const uint4 z = make_uint4(0, 0, 0, 0);
      uint8_t* q = smem + OFF_Q + (i >> 7) * TILE_BYTES;
      uint4* r0 = reinterpret_cast<uint4*>(q + r * 128);
      uint4* r1 = reinterpret_cast<uint4*>(q + HALF_BYTES + r * 128);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        r0[k] = z;
        r1[k] = z;
      }
    }
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers and TMEM exist before either uses the other's
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 10) {
    // ------------------------------------------------------------ Q producer
    if (lane == 0) {
      // The plan is never written by the kernel launched just before (only q/k/v
      // are): the first unit's fields load while the wait runs.
      int g = 0, ntile = 0, q_a = 0, q_b = 0;
      auto fetch = [&](int ui) {
        const int32_t* u = unit_rec(ui);
        g = u[kUKvHead];
        ntile = u[kUQCountB] > 0 ? 2 : 1;
        q_a = u[kUQBeginA];
        q_b = u[kUQBeginB];
      };
      if (u_begin < u_end) fetch(u_begin);
      if (!p.inflight) pdl_wait();  // Q may be written by the preceding kernel
      int load = 0;
      for (int ui = u_begin; ui < u_end; ++ui) {
        if (ui != u_begin) fetch(ui);
        bool ok = true;
        for (int x = 0; x < ntile; ++x, ++load) {
          const int slot = load % QSLOTS;
          if (load >= QSLOTS && !wait_or_abort(bars.q_empty + slot, (uint32_t)((load / QSLOTS) & 1) ^ 1u,
                                               VLC_DEV_ERR_TIMEOUT + 1, abort_flag)) {
            ok = false;
            break;
          }
          const int q_begin = x == 0 ? q_a : q_b;
          // At launch every CTA loads at once and HBM is the limit: the first tile's Q
          // (an operand of the first Q K^T) lands before the second tile's is requested.
          if (leader && load == 1 && !wait_or_abort(bars.q_full + 0, 0u, VLC_DEV_ERR_TIMEOUT + 1, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* qdst = smem + OFF_Q + slot * TILE_BYTES;
          if (leader) mbar_expect_tx(bars.q_full + slot, 2 * 2 * p.rows * 128);  // both CTAs' bytes
          const uint32_t qbar = mapa_shared(smem_u32(bars.q_full + slot), 0);
          tma_load_3d_pair(qdst, &p.tm_q, qbar, 0, g * p.group, q_begin);
          tma_load_3d_pair(qdst + HALF_BYTES, &p.tm_q, qbar, 64, g * p.group, q_begin);
        }
        if (!ok) break;
      }
    }
  } else if (warp == 8) {
    // ------------------------------------------------------------ K/V producer
    if (lane == 0) {
      // Plan and block tables are never written by the kernel launched just before:
      // the first unit's fields and its first page are read while the wait runs.
      int g = 0, kb0 = 0, kb1 = 0, slot0 = 0;
      bool infl = false;
      const int32_t* u = nullptr;
      auto fetch = [&](int ui) {
        u = unit_rec(ui);
        g = u[kUKvHead];
        kb0 = u[kUKbBegin];
        kb1 = u[kUKbEnd];
        infl = unit_inflight(p, u);
        slot0 = kb0 < kb1 ? key_block_slot(p, u, kb0) : 0;
      };
      if (u_begin < u_end) fetch(u_begin);
      bool waited = false;  // K/V rows (paged or contiguous) may be written by the preceding kernel
      int it = 0;
      for (int ui = u_begin; ui < u_end; ++ui) {
        if (ui != u_begin) fetch(ui);
        if (!infl && !waited) {
          pdl_wait();
          waited = true;
        }
        const CUtensorMap* tk = infl ? &p.tm_kn64 : &p.tm_k64;  // box of 64 keys
        const CUtensorMap* tv = infl ? &p.tm_vn : &p.tm_v;
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
          const int slot = kb == kb0 ? slot0 : key_block_slot(p, u, kb);
          if (it >= STAGES && !wait_or_abort(bars.k_empty + s, ph ^ 1u, VLC_DEV_ERR_TIMEOUT + 2, abort_flag)) {
            ok = false;
            break;
          }
          // this CTA's keys [64 rank, 64 rank + 64): two 64-dim halves of 64 rows
          uint8_t* kdst = smem + OFF_K + s * TILE_BYTES;
          if (leader) mbar_expect_tx(bars.k_full + s, TILE_BYTES);  // both CTAs' halves
          const uint32_t kbar = mapa_shared(smem_u32(bars.k_full + s), 0);
          tma_load_3d_pair(kdst, tk, kbar, 0, g, slot + 64 * (int)rank);
          tma_load_3d_pair(kdst + quad::KHALF_BYTES, tk, kbar, 64, g, slot + 64 * (int)rank);
          if (it >= STAGES && !wait_or_abort(bars.v_empty + s, ph ^ 1u, VLC_DEV_ERR_TIMEOUT + 3, abort_flag)) {
            ok = false;
            break;
          }
          // Likewise the first K block lands before V and the next blocks are requested.
          if (leader && it == 0 && !wait_or_abort(bars.k_full + 0, 0u, VLC_DEV_ERR_TIMEOUT + 3, abort_flag)) {
            ok = false;
            break;
          }
          // this CTA's dims [64 rank, 64 rank + 64) of all 128 keys
          uint8_t* vdst = smem + OFF_V + s * TILE_BYTES;
          if (leader) mbar_expect_tx(bars.v_full + s, TILE_BYTES);  // both CTAs' halves
          tma_load_3d_pair(vdst, tv, mapa_shared(smem_u32(bars.v_full + s), 0), 64 * (int)rank, g, slot);
        }
        if (!ok) break;
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issuer
    // Step j of a unit (K/V block kv = it + j): for tile A then tile B (while it has
    // blocks): O += P(j) V(j), then S = Q K(j+1)^T.  At the unit's last step the
    // next Q K^T is the next unit's block 0 (same K/V ring, next Q slots), so the
    // softmax warps start the next unit while this one drains.
    if (lane == 0 && leader && u_begin < u_end) {
      const uint32_t q_lo = umma_desc_sw128_lo(smem_u32(smem + OFF_Q), 16);
      const uint32_t k_lo = umma_desc_sw128_lo(smem_u32(smem + OFF_K), 16);
      const uint32_t v_lo = umma_desc_sw128_lo(smem_u32(smem + OFF_V), HALF_BYTES);
      constexpr uint32_t kTileLo = TILE_BYTES >> 4;  // one tile in descriptor address units
      int qload = 0;  // Q loads consumed (slot = load % QSLOTS, same order as the Q producer)
      struct Cur {
        UnitView v;
        int load_a, load_b;
      };
      auto next_unit = [&](int ui) {
        Cur c;
        c.v = unit_view(unit_rec(ui));
        c.load_a = qload++;
        c.load_b = c.v.n_b > 0 ? qload++ : -1;
        return c;
      };
      auto wait_k = [&](int kv) {
        return wait_or_abort(bars.k_full + kv % STAGES, (uint32_t)(kv / STAGES) & 1u, VLC_DEV_ERR_TIMEOUT + 7,
                             abort_flag);
      };
      // S_x = Q(load) K(kv)^T; `first`: the tile's first block (wait for its Q),
      // `last`: its last block (release the Q slot once the MMA completes).
      auto qk = [&](int x, int load, int kv, bool first, bool last) {
        const int slot = load % QSLOTS;
        if (first && !wait_or_abort(bars.q_full + slot, (uint32_t)(load / QSLOTS) & 1u, VLC_DEV_ERR_TIMEOUT + 6,
                                    abort_flag))
          return false;
        tc_fence_after();
        issue_qk_quad(tmem_base + TMEM_S + x * 128, q_lo + slot * kTileLo, k_lo + (kv % STAGES) * kTileLo);
        commit_both(bars.s_full + x);
        if (last) commit_both(bars.q_empty + slot);
        return true;
      };
      Cur cur = next_unit(u_begin);
      bool ok = wait_k(0) && qk(0, cur.load_a, 0, true, cur.v.n_a == 1) &&
                (cur.v.n_b == 0 || qk(1, cur.load_b, 0, true, cur.v.n_b == 1));
      if (ok) commit_both(bars.k_empty + 0);
      int pv_a = 0, pv_b = 0;  // P*V issued per tile (p_lo / p_hi phases)
      int it = 0;              // K/V block index of the current unit's block 0
      for (int ui = u_begin; ok && ui < u_end; ++ui) {
        const bool has_next = ui + 1 < u_end;
        Cur nxt{};
        if (has_next) nxt = next_unit(ui + 1);
        for (int j = 0; j < cur.v.n_a; ++j) {
          const int kv = it + j, s = kv % STAGES;
          const bool last = j == cur.v.n_a - 1;
          const bool more = !last || has_next;  // a block kv + 1 follows
          // tile A
          // V(kv) in both CTAs first: the odd CTA may zero rows of its half before its P
          if (!wait_or_abort(bars.v_full + s, (uint32_t)(kv / STAGES) & 1u, VLC_DEV_ERR_TIMEOUT + 5, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_cluster(mapa_shared(smem_u32(v_landed + s), 1));
          if (!wait_or_abort(bars.p_lo + 0, (uint32_t)pv_a & 1u, VLC_DEV_ERR_TIMEOUT + 4, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_pv_half_quad(tmem_base + TMEM_O, tmem_base + TMEM_S, v_lo + s * kTileLo, 0, j > 0);
          if (!wait_or_abort(bars.p_hi + 0, (uint32_t)pv_a & 1u, VLC_DEV_ERR_TIMEOUT + 4, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_pv_half_quad(tmem_base + TMEM_O, tmem_base + TMEM_S, v_lo + s * kTileLo, 1, true);
          ++pv_a;
          if (last) commit_both(bars.o_done + 0);
          if (more && !wait_k(kv + 1)) {
            ok = false;
            break;
          }
          if (!last)
            ok = qk(0, cur.load_a, kv + 1, false, j + 1 == cur.v.n_a - 1);
          else if (has_next)
            ok = qk(0, nxt.load_a, kv + 1, true, nxt.v.n_a == 1);
          if (!ok) break;
          // tile B
          if (j < cur.v.n_b) {
            if (!wait_or_abort(bars.p_lo + 1, (uint32_t)pv_b & 1u, VLC_DEV_ERR_TIMEOUT + 8, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_pv_half_quad(tmem_base + TMEM_O + 128, tmem_base + TMEM_S + 128, v_lo + s * kTileLo, 0, j > 0);
            if (!wait_or_abort(bars.p_hi + 1, (uint32_t)pv_b & 1u, VLC_DEV_ERR_TIMEOUT + 8, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_pv_half_quad(tmem_base + TMEM_O + 128, tmem_base + TMEM_S + 128, v_lo + s * kTileLo, 1, true);
            ++pv_b;
            if (j == cur.v.n_b - 1)
              commit_both(bars.o_done + 1);
            else
              ok = qk(1, cur.load_b, kv + 1, false, j + 1 == cur.v.n_b - 1);
            if (!ok) break;
          }
          if (last && has_next && nxt.v.n_b > 0) {
            ok = qk(1, nxt.load_b, kv + 1, true, nxt.v.n_b == 1);
            if (!ok) break;
          }
          commit_both(bars.v_empty + s);
          if (more) commit_both(bars.k_empty + (kv + 1) % STAGES);
        }
        it += cur.v.n_a;
        cur = nxt;
      }
    }
  } else {
    // ------------------------------------------------------------ softmax (one warpgroup per tile)
    const int x = warp >> 2;            // 0: tile A, 1: tile B
    const int row = threadIdx.x & 127;  // == TMEM lane
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t s_addr = tmem_base + lane_off + TMEM_S + x * 128;
    const uint32_t o_addr = tmem_base + lane_off + TMEM_O + x * 128;
    int t = 0;      // blocks of this tile processed (s_full / p_lo / p_hi phases)
    int nunit = 0;  // units of this tile finished (o_done phases)
    int qload = 0;  // Q loads of this CTA so far (the Q producer's order)
    for (int ui = u_begin; ui < u_end; ++ui) {
      const int32_t* u = unit_rec(ui);
      const UnitView uv = unit_view(u);
      const int n = x == 0 ? uv.n_a : uv.n_b;
      const int my_load = qload + x;
      qload += u[kUQCountB] > 0 ? 2 : 1;
      if (n == 0) continue;
      // The tile's Q slot is free for the epilogue when fewer than QSLOTS loads follow
      // this tile's (no later Q lands in it).
      int after = qload - 1 - my_load;
      for (int uj = ui + 1; uj < u_end && after < QSLOTS; ++uj)
        after += unit_rec(uj)[kUQCountB] > 0 ? 2 : 1;
      const bool own_slot = after < QSLOTS;
      const int g = u[kUKvHead];
      const int kb0 = u[kUKbBegin];
      const int kv_len = u[kUKvLen];
      const int q_begin = u[x == 0 ? kUQBeginA : kUQBeginB];
      const int q_count = u[x == 0 ? kUQCountA : kUQCountB];
      const int kpos0 = u[x == 0 ? kUKpos0A : kUKpos0B];
      const int part = u[x == 0 ? kUPartA : kUPartB];
      const int tok = row / p.group;
      const bool row_valid = row < p.rows && tok < q_count;
      const int qpos = p.causal ? kpos0 + tok : kpos0;  // non-causal: kpos0 = k_len - 1

      float m_use = -INFINITY;
      float l_row = 0.f;
      bool ok = true;
      for (int j = 0; j < n; ++j, ++t) {
        if (!wait_or_abort(bars.s_full + x, (uint32_t)t & 1u, VLC_DEV_ERR_TIMEOUT + 9, abort_flag)) {
          ok = false;
          break;
        }
        __syncwarp();
        tc_fence_after();
        const int key0 = (kb0 + j) * BN;
        uint32_t sr[128];
#pragma unroll
        for (int q = 0; q < 4; ++q) tmem_ld32(s_addr + q * 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[q * 32]));
        tmem_wait_ld();
        if (kPacked) {
          // Packed tile (several short sequences, one key block = the same tokens): the row
          // sees keys [lo, hi) of the block, its own sequence's; rows past q_count none.
          int lo = 0, hi = 0;
          if (row_valid) {
            const int k_base = unit_rec(ui)[kUKBase];
            lo = __ldg(p.segments + 2 * (int64_t)(q_begin + tok)) - k_base;
            hi = __ldg(p.segments + 2 * (int64_t)(q_begin + tok) + 1) - k_base;
          }
#pragma unroll
          for (int c = 0; c < 128; ++c)
            if (c < lo || c >= hi) sr[c] = __float_as_uint(-INFINITY);
        } else if (key0 + BN - 1 > kpos0) {  // block touches the causal diagonal
          const int lim = qpos - key0;
#pragma unroll
          for (int c = 0; c < 128; ++c)
            if (c > lim) sr[c] = __float_as_uint(-INFINITY);
        }
        float mx[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) mx[k] = __uint_as_float(sr[k]);
#pragma unroll
        for (int c = 8; c < 128; c += 16)
#pragma unroll
          for (int k = 0; k < 8; ++k) mx[k] = fmax3(mx[k], __uint_as_float(sr[c + k]), __uint_as_float(sr[c + 8 + k]));
        const float m_tile = fmaxf(fmax3(mx[0], mx[1], mx[2]), fmax3(fmax3(mx[3], mx[4], mx[5]), mx[6], mx[7])) *
                             p.scale_log2;
        // Lazy rescaling: only move the reference max when it grows by > 2^8.
        const bool need = m_tile > m_use + 8.0f;
        const float m_new = need ? m_tile : m_use;
        const float f = (need && m_use != -INFINITY) ? fast_exp2(m_use - m_new) : 1.0f;
        m_use = m_new;
        const float mref = (m_use == -INFINITY) ? 0.f : m_use;
        // Keys past the sequence end: zero their V rows so 0 * garbage stays 0.  Tile A
        // has every block of the unit, and its P*V runs first.
        if (x == 0 && key0 + BN > kv_len) {
          const int st = t % STAGES;
          if (!wait_or_abort(leader ? bars.v_full + st : v_landed + st, (uint32_t)(t / STAGES) & 1u,
                             VLC_DEV_ERR_TIMEOUT + 11, abort_flag)) {
            ok = false;
            break;
          }
          if (key0 + row >= kv_len) {
            const uint4 z = make_uint4(0, 0, 0, 0);
            uint4* v0 = reinterpret_cast<uint4*>(smem + OFF_V + st * TILE_BYTES + row * 128);
#pragma unroll
            for (int i = 0; i < 8; ++i) v0[i] = z;
          }
          fence_proxy_async_smem();
        }
        // P = exp2(s * scale_log2 - mref) as bf16 pairs: key pair (2c, 2c+1) goes to S
        // column c (its register is free: pair c reads registers 2c and 2c+1 >= c).  Each
        // half of the keys is released to the MMA as soon as it is in TMEM.
        const uint64_t scale2 = f2_pack(p.scale_log2, p.scale_log2);
        const uint64_t negm2 = f2_pack(-mref, -mref);
        uint64_t lsum = f2_pack(0.f, 0.f);
#pragma unroll
        for (int half = 0; half < 2; ++half) {
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            const int base = half * 64 + q * 32;
#pragma unroll
            for (int c = 0; c < 16; ++c) {
              const uint64_t x2 =
                  f2_fma(f2_pack(__uint_as_float(sr[base + 2 * c]), __uint_as_float(sr[base + 2 * c + 1])), scale2,
                         negm2);
              float x0, x1;
              f2_unpack(x2, x0, x1);
              const float e0 = fast_exp2(x0), e1 = fast_exp2(x1);
              lsum = f2_add(lsum, f2_pack(e0, e1));
              sr[base + c] = pack_bf16x2(e0, e1);
            }
            tmem_st16(s_addr + (base >> 1), *reinterpret_cast<uint32_t(*)[16]>(&sr[base]));
          }
          if (half == 0 && __any_sync(0xffffffffu, f != 1.0f)) {
            // O (stable: P(j-1) V(j-1) completed before S(j)) follows the moved max
            // before this block's P V starts.
#pragma unroll 1
            for (int cb = 0; cb < 8; ++cb) {
              uint32_t orr[16];
              tmem_ld16(o_addr + cb * 16, orr);
              tmem_wait_ld();
#pragma unroll
              for (int c = 0; c < 16; ++c) orr[c] = __float_as_uint(__uint_as_float(orr[c]) * f);
              tmem_st16(o_addr + cb * 16, orr);
            }
            l_row *= f;
          }
          tmem_wait_st();
          tc_fence_before();
          uint64_t* pb = half == 0 ? bars.p_lo + x : bars.p_hi + x;
          if (leader)
            mbar_arrive(pb);
          else
            mbar_arrive_cluster(mapa_shared(smem_u32(pb), 0));
        }
        {
          float l0, l1;
          f2_unpack(lsum, l0, l1);
          l_row += l0 + l1;
        }
      }
      if (!ok) break;
      // ---------------------------------------------------------- epilogue
      if (!wait_or_abort(bars.o_done + x, (uint32_t)nunit & 1u, VLC_DEV_ERR_TIMEOUT + 12, abort_flag)) break;
      ++nunit;
      __syncwarp();
      tc_fence_after();
      const float inv = l_row > 0.f ? 1.0f / l_row : 0.f;
      __nv_bfloat16* dst;
      if (part < 0) {
        const int head = g * p.group + (row - tok * p.group);
        dst = p.out + (int64_t)(q_begin + tok) * p.out_token_stride + (int64_t)head * p.head_dim;
      } else {
        // Split partial: O / l as bf16 (the merge re-weights by l and the max).
        dst = p.part_o + ((int64_t)part * BM + row) * HD;
        reinterpret_cast<float2*>(p.part_ml)[(int64_t)part * BM + row] = make_float2(m_use, l_row);
      }
      const bool ghost = part == kGhostPart;
      const bool store = ghost ? false : part < 0 ? row_valid : true;
      uint32_t orr[128];
#pragma unroll
      for (int q = 0; q < 4; ++q) tmem_ld32(o_addr + q * 32, *reinterpret_cast<uint32_t(*)[32]>(&orr[q * 32]));
      tmem_wait_ld();
#pragma unroll
      for (int c = 0; c < 64; ++c)
        orr[c] = pack_bf16x2(__uint_as_float(orr[2 * c]) * inv, __uint_as_float(orr[2 * c + 1]) * inv);
      if (!ghost && own_slot && (part >= 0 || q_count == p.tokens_per_tile)) {
        // Full tile or split partial, Q slot free: the whole tile goes into the slot
        // in the Q load's layout (128-byte swizzle: 16-byte chunk c of row r of a
        // 64-column half at chunk c ^ (r % 8)) and leaves with two TMA stores.  The
        // slot's last reader, this tile's final Q K^T, completed before o_done.
        uint8_t* qs = smem + OFF_Q + (my_load % QSLOTS) * TILE_BYTES;
#pragma unroll
        for (int k = 0; k < 16; ++k)
          *reinterpret_cast<uint4*>(qs + (k >> 3) * HALF_BYTES + row * 128 + (((k & 7) ^ (row & 7)) << 4)) =
              make_uint4(orr[4 * k], orr[4 * k + 1], orr[4 * k + 2], orr[4 * k + 3]);
        fence_proxy_async_smem();
        named_bar_sync(1 + x, kTileThreads);
        if (row == 0) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            if (part < 0) {
              if (64 * h < p.head_dim)  // columns past head_dim are the zero padding
                tma_store_3d(&p.tm_o128, qs + h * HALF_BYTES, 64 * h, g * p.group, q_begin);
            } else {
              tma_store_2d(&p.tm_p128, qs + h * HALF_BYTES, 64 * h, part * BM);
            }
          }
          bulk_commit_group();
        }
      } else if (!ghost && (part >= 0 || q_count == p.tokens_per_tile)) {
        // Full tile or split partial: stage 32 columns at a time in shared memory,
        // alternating two buffers (64-byte swizzle: 16-byte chunk c of row r at chunk
        // c ^ ((r / 2) % 4)), and let one thread write each with a TMA tensor store.
        uint8_t* stg = smem + OFF_STG + x * STG_TILE;
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          uint8_t* buf = stg + (r & 1) * STG_BUF;
          if (row == 0) bulk_wait_read_allbut1();  // the store that used this buffer has read it
          named_bar_sync(1 + x, kTileThreads);
#pragma unroll
          for (int c = 0; c < 4; ++c)
            *reinterpret_cast<uint4*>(buf + row * 64 + ((c ^ ((row >> 1) & 3)) << 4)) =
                make_uint4(orr[16 * r + 4 * c], orr[16 * r + 4 * c + 1], orr[16 * r + 4 * c + 2],
                           orr[16 * r + 4 * c + 3]);
          fence_proxy_async_smem();
          named_bar_sync(1 + x, kTileThreads);
          if (row == 0) {
            if (part < 0) {
              if (32 * r < p.head_dim) tma_store_3d(&p.tm_o, buf, 32 * r, g * p.group, q_begin);
            } else {
              tma_store_2d(&p.tm_p, buf, 32 * r, part * BM);
            }
            bulk_commit_group();
          }
        }
      } else if (store) {
        // Last, partial tile of a sequence: the tensor store would write the rows of
        // the following tokens, so each valid row is written directly.
        if (p.out_store32) {
#pragma unroll
          for (int c = 0; c < 8; ++c)
            if (c * 16 < p.head_dim)
              st_global_v8(dst + c * 16, *reinterpret_cast<const uint32_t(*)[8]>(&orr[c * 8]));
        } else {
#pragma unroll
          for (int c = 0; c < 16; ++c)
            if (c * 8 < p.head_dim)
              *reinterpret_cast<uint4*>(dst + c * 8) =
                  make_uint4(orr[4 * c], orr[4 * c + 1], orr[4 * c + 2], orr[4 * c + 3]);
        }
      }
      tc_fence_before();
    }
    if (row == 0) bulk_wait_all();  // this tile's output stores are complete
  }

  __syncthreads();
  cluster_sync();  // every remote arrival and every MMA into this CTA's TMEM is done
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}


// Merge split units.  Part p holds O_p / l_p (bf16), its max m_p and sum l_p:
//   O = sum_p w_p (O_p / l_p) / sum_p w_p,   w_p = 2^(m_p - M) l_p.
// 256-thread blocks listed by the planner as (merge, first row).  A warp is 4
// groups of 8 lanes; lane c of a group owns dims [16 c, 16 c + 16) (one 32-byte
// load per part).  With R rows per warp (4, 2 or 1) each row has K = 4 / R groups,
// group k folding parts k, k + K, ... with a running max, kMergeBatch parts per
// round with their loads in flight together; the K states of a row combine
// through shuffles.
constexpr int kMergeBatch = 5;
__global__ void __launch_bounds__(256, 3) prefill_merge_kernel(const int32_t* __restrict__ merges,
                                                               const int32_t* __restrict__ blocks,
                                                               const __nv_bfloat16* __restrict__ part_o,
                                                               const float* __restrict__ part_ml, int group,
                                                               __nv_bfloat16* __restrict__ out,
                                                               int64_t out_token_stride, int head_dim) {
  const int entry = __ldg(blocks + blockIdx.x);
  const int32_t* m = merges + (int64_t)(entry >> 8) * kMergeInts;
  const int q_begin = __ldg(m + kMQBegin), g = __ldg(m + kMKvHead);
  const int part0 = __ldg(m + kMPartBegin), nparts = __ldg(m + kMNumParts);
  const int R = __ldg(m + kMRowsPerWarp), nrows = __ldg(m + kMRows);
  // The next kernel may be scheduled now: every programmatic dependent here waits
  // (griddepcontrol.wait) for this grid to complete before it reads the output.
  pdl_launch_dependents();
  pdl_wait();  // the partials are written by the attention kernel launched just before
  const int K = 4 / R;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grp = lane >> 3, c = lane & 7;
  const int row = (entry & 255) + warp * R + grp / K;
  const int k0 = grp % K;
  const bool active = row < nrows;
  const float2* ml = reinterpret_cast<const float2*>(part_ml);
  float acc[16];
#pragma unroll
  for (int k = 0; k < 16; ++k) acc[k] = 0.f;
  float m_run = -INFINITY, L = 0.f;
  if (active) {
    // Batches of kMergeBatch parts: all loads of a batch are issued before any of
    // them is used, then the batch is folded with one rescale of the accumulator.
    for (int i0 = k0; i0 < nparts; i0 += kMergeBatch * K) {
      float2 v[kMergeBatch];
      uint4 r0[kMergeBatch], r1[kMergeBatch];
#pragma unroll
      for (int s = 0; s < kMergeBatch; ++s) {
        const int i = i0 + s * K;
        if (i < nparts) {
          const int64_t pr = (int64_t)(part0 + i) * BM + row;
          const uint4* src = reinterpret_cast<const uint4*>(part_o + pr * HD) + 2 * c;
          v[s] = __ldg(&ml[pr]);
          r0[s] = __ldg(src);
          r1[s] = __ldg(src + 1);
        } else {
          v[s] = make_float2(-INFINITY, 0.f);  // weight 0
          r0[s] = r1[s] = make_uint4(0, 0, 0, 0);
        }
      }
      float m_new = m_run;
#pragma unroll
      for (int s = 0; s < kMergeBatch; ++s) m_new = fmaxf(m_new, v[s].x);
      const float mr = m_new == -INFINITY ? 0.f : m_new;
      const float a = fast_exp2(m_run - mr);  // 0 while nothing is accumulated
      m_run = m_new;
      L *= a;
#pragma unroll
      for (int k = 0; k < 16; ++k) acc[k] *= a;
#pragma unroll
      for (int s = 0; s < kMergeBatch; ++s) {
        const float w = fast_exp2(v[s].x - mr) * v[s].y;  // weight of O_p / l_p (0 for an empty part)
        L += w;
        const uint32_t wds[8] = {r0[s].x, r0[s].y, r0[s].z, r0[s].w, r1[s].x, r1[s].y, r1[s].z, r1[s].w};
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float2 o = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&wds[k]));
          acc[2 * k] = fmaf(w, o.x, acc[2 * k]);
          acc[2 * k + 1] = fmaf(w, o.y, acc[2 * k + 1]);
        }
      }
    }
  }
  // Combine the K groups of a row (lanes 8 apart): xor 8 when K >= 2, then 16 when K == 4.
#pragma unroll
  for (int sh = 8; sh <= 16; sh <<= 1) {
    if (sh == 8 ? K < 2 : K < 4) break;
    const float m_oth = __shfl_xor_sync(0xffffffffu, m_run, sh);
    const float m_all = fmaxf(m_run, m_oth);
    const float mr = m_all == -INFINITY ? 0.f : m_all;
    const float a = fast_exp2(m_run - mr);
    L *= a;
    L += __shfl_xor_sync(0xffffffffu, L, sh);
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      acc[k] *= a;
      acc[k] += __shfl_xor_sync(0xffffffffu, acc[k], sh);
    }
    m_run = m_all;
  }
  if (!active || k0 != 0 || c * 16 >= head_dim) return;  // dims past head_dim: zero padding
  const float inv = L > 0.f ? 1.0f / L : 0.f;
  const int tok = row / group;
  const int head = g * group + (row - tok * group);
  __nv_bfloat16* dst = out + (int64_t)(q_begin + tok) * out_token_stride + (int64_t)head * head_dim + c * 16;
  uint4 p0, p1;
  p0.x = pack_bf16x2(acc[0] * inv, acc[1] * inv);
  p0.y = pack_bf16x2(acc[2] * inv, acc[3] * inv);
  p0.z = pack_bf16x2(acc[4] * inv, acc[5] * inv);
  p0.w = pack_bf16x2(acc[6] * inv, acc[7] * inv);
  p1.x = pack_bf16x2(acc[8] * inv, acc[9] * inv);
  p1.y = pack_bf16x2(acc[10] * inv, acc[11] * inv);
  p1.z = pack_bf16x2(acc[12] * inv, acc[13] * inv);
  p1.w = pack_bf16x2(acc[14] * inv, acc[15] * inv);
  reinterpret_cast<uint4*>(dst)[0] = p0;
  reinterpret_cast<uint4*>(dst)[1] = p1;
}

}  // namespace prefill
}  // namespace vlc

using namespace vlc;
using namespace vlc::prefill;

extern "C" int64_t vlc_prefill_workspace_size(const int32_t* plan_host) {
  if (!plan_host || plan_host[kPMagic] != kPlanMagic) return -1;
  const int64_t parts = plan_host[kPNumParts];
  return parts * (int64_t)BM * (HD * (int64_t)sizeof(__nv_bfloat16) + 2 * (int64_t)sizeof(float));
}

static int prefill_attn_impl(const void* q, int64_t q_token_stride, int total_q, int num_heads, const void* k_cache,
                             const void* v_cache, int64_t k_row_stride, int64_t v_row_stride, int64_t num_slots,
                             int num_kv_heads, int head_dim, const int32_t* block_tables, int block_table_stride,
                             int block_size, const int32_t* plan_dev, const int32_t* plan_host, float softmax_scale,
                             void* out, int64_t out_token_stride, void* workspace, int64_t workspace_bytes,
                             const void* k_new, const void* v_new, int64_t kn_row_stride, int64_t vn_row_stride,
                             int64_t num_new_rows, void* stream) {
  if (!q || !k_cache || !v_cache || !plan_dev || !plan_host || !out) return VLC_ERR_NULL;
  if (head_dim <= 64 || head_dim > HD || head_dim % 16 != 0) return VLC_ERR_UNSUPPORTED;
  if (num_heads <= 0 || num_kv_heads <= 0 || num_heads % num_kv_heads != 0) return VLC_ERR_SHAPE;
  if (block_tables && (block_size <= 0 || block_size % BN != 0)) return VLC_ERR_UNSUPPORTED;
  if (plan_host[kPMagic] != kPlanMagic || plan_host[kPVersion] != kPlanVersion) return VLC_ERR_PLAN;
  const int group = num_heads / num_kv_heads;
  if (plan_host[kPGroup] != group || plan_host[kPNumHeads] != num_heads ||
      plan_host[kPNumKvHeads] != num_kv_heads || plan_host[kPTotalQ] != total_q ||
      plan_host[kPHeadDim] != head_dim)
    return VLC_ERR_PLAN;
  const int grid = plan_host[kPGrid];
  if (grid == 0 || total_q == 0) return VLC_OK;
  if (q_token_stride % 8 != 0 || out_token_stride % 8 != 0 || k_row_stride % 8 != 0 || v_row_stride % 8 != 0)
    return VLC_ERR_STRIDE;
  if (q_token_stride < (int64_t)num_heads * head_dim || out_token_stride < (int64_t)num_heads * head_dim ||
      k_row_stride < (int64_t)num_kv_heads * head_dim || v_row_stride < (int64_t)num_kv_heads * head_dim)
    return VLC_ERR_STRIDE;
  if (!aligned16(q) || !aligned16(k_cache) || !aligned16(v_cache) || !aligned16(out)) return VLC_ERR_ALIGN;
  if ((k_new == nullptr) != (v_new == nullptr)) return VLC_ERR_NULL;
  if (k_new != nullptr) {
    // every self-attention sequence's keys are the in-flight rows of its queries
    if (num_new_rows < total_q || num_new_rows > 0x7fffff00) return VLC_ERR_SHAPE;
    if (kn_row_stride % 8 != 0 || vn_row_stride % 8 != 0 || kn_row_stride < (int64_t)num_kv_heads * head_dim ||
        vn_row_stride < (int64_t)num_kv_heads * head_dim)
      return VLC_ERR_STRIDE;
    if (!aligned16(k_new) || !aligned16(v_new)) return VLC_ERR_ALIGN;
  }
  const int64_t ws_need = vlc_prefill_workspace_size(plan_host);
  if (ws_need > 0 && (!workspace || workspace_bytes < ws_need)) return VLC_ERR_WORKSPACE;
  if (num_slots <= 0 || num_slots > 0x7fffff00) return VLC_ERR_SHAPE;

  Params prm;
  const int T = plan_host[kPTokensPerTile];
  const int rows = plan_host[kPRowsPerTile];
  {
    const uint64_t dims[3] = {(uint64_t)head_dim, (uint64_t)num_heads, (uint64_t)total_q};
    const uint64_t strides[2] = {(uint64_t)head_dim * 2, (uint64_t)q_token_stride * 2};
    const uint32_t box[3] = {64, (uint32_t)group, (uint32_t)T};
    if (encode_tmap_bf16(&prm.tm_q, q, 3, dims, strides, box, 128) != VLC_OK) return VLC_ERR_CUDA;
  }
  {
    const uint64_t dims[3] = {(uint64_t)head_dim, (uint64_t)num_kv_heads, (uint64_t)num_slots};
    const uint64_t ks[2] = {(uint64_t)head_dim * 2, (uint64_t)k_row_stride * 2};
    const uint64_t vs[2] = {(uint64_t)head_dim * 2, (uint64_t)v_row_stride * 2};
    const uint32_t box[3] = {64, 1, (uint32_t)BN};
    if (encode_tmap_bf16(&prm.tm_k, k_cache, 3, dims, ks, box, 128) != VLC_OK) return VLC_ERR_CUDA;
    if (encode_tmap_bf16(&prm.tm_v, v_cache, 3, dims, vs, box, 128) != VLC_OK) return VLC_ERR_CUDA;
  }
  prm.inflight = k_new != nullptr ? 1 : 0;
  if (prm.inflight) {
    const uint64_t dims[3] = {(uint64_t)head_dim, (uint64_t)num_kv_heads, (uint64_t)num_new_rows};
    const uint64_t ks[2] = {(uint64_t)head_dim * 2, (uint64_t)kn_row_stride * 2};
    const uint64_t vs[2] = {(uint64_t)head_dim * 2, (uint64_t)vn_row_stride * 2};
    const uint32_t box[3] = {64, 1, (uint32_t)BN};
    if (encode_tmap_bf16(&prm.tm_kn, k_new, 3, dims, ks, box, 128) != VLC_OK) return VLC_ERR_CUDA;
    if (encode_tmap_bf16(&prm.tm_vn, v_new, 3, dims, vs, box, 128) != VLC_OK) return VLC_ERR_CUDA;
  } else {
    prm.tm_kn = prm.tm_k;  // unused
    prm.tm_vn = prm.tm_v;
  }
  {
    const uint64_t dims[3] = {(uint64_t)head_dim, (uint64_t)num_heads, (uint64_t)total_q};
    const uint64_t strides[2] = {(uint64_t)head_dim * 2, (uint64_t)out_token_stride * 2};
    const uint32_t box[3] = {32, (uint32_t)group, (uint32_t)T};
    if (encode_tmap_bf16(&prm.tm_o, out, 3, dims, strides, box, 64) != VLC_OK) return VLC_ERR_CUDA;
    const uint32_t box128[3] = {64, (uint32_t)group, (uint32_t)T};
    if (encode_tmap_bf16(&prm.tm_o128, out, 3, dims, strides, box128, 128) != VLC_OK) return VLC_ERR_CUDA;
  }
  prm.cta_offsets = plan_dev + plan_host[kPOffCta];
  prm.units = plan_dev + plan_host[kPOffUnits];
  prm.block_tables = block_tables;
  prm.bt_stride = block_table_stride;
  prm.block_size = block_size;
  prm.group = group;
  prm.rows = rows;
  prm.scale_log2 = softmax_scale * 1.4426950408889634f;
  prm.num_slots = num_slots;
  prm.out = (__nv_bfloat16*)out;
  prm.out_token_stride = out_token_stride;
  prm.out_store32 = ((uintptr_t)out % 32 == 0) && (out_token_stride % 16 == 0);
  const int64_t parts = plan_host[kPNumParts];
  if (ws_need > 0 && (uintptr_t)workspace % 256 != 0) return VLC_ERR_ALIGN;
  prm.part_ml = (float*)workspace;  // [parts][BM][2] fp32 first (8-byte aligned), then bf16 O
  prm.part_o = workspace ? (__nv_bfloat16*)((float*)workspace + parts * BM * 2) : nullptr;
  if (parts > 0) {
    const uint64_t dims[2] = {(uint64_t)HD, (uint64_t)parts * BM};
    const uint64_t strides[1] = {(uint64_t)HD * 2};
    const uint32_t box[2] = {32, (uint32_t)BM};
    if (encode_tmap_bf16(&prm.tm_p, prm.part_o, 2, dims, strides, box, 64) != VLC_OK) return VLC_ERR_CUDA;
    const uint32_t box128[2] = {64, (uint32_t)BM};
    if (encode_tmap_bf16(&prm.tm_p128, prm.part_o, 2, dims, strides, box128, 128) != VLC_OK) return VLC_ERR_CUDA;
  } else {
    prm.tm_p = prm.tm_o;  // unused
    prm.tm_p128 = prm.tm_o128;
  }
  prm.tokens_per_tile = T;
  prm.head_dim = head_dim;
  prm.causal = plan_host[kPCausal];
  prm.segments = plan_host[kPOffSegments] > 0 ? plan_dev + plan_host[kPOffSegments] : nullptr;
  if (prm.segments != nullptr && block_tables != nullptr) return VLC_ERR_PLAN;  // packed tiles: contiguous K/V

  const bool packed = prm.segments != nullptr;
  const bool quad_units = plan_host[kPQuad] != 0;
  if (quad_units && (packed || grid % 2 != 0)) return VLC_ERR_PLAN;
  if (quad_units) {
    // the K tensors again with a box of 64 keys: each CTA of a pair loads half of a block
    const uint64_t dims[3] = {(uint64_t)head_dim, (uint64_t)num_kv_heads, (uint64_t)num_slots};
    const uint64_t ks[2] = {(uint64_t)head_dim * 2, (uint64_t)k_row_stride * 2};
    const uint32_t box[3] = {64, 1, 64};
    if (encode_tmap_bf16(&prm.tm_k64, k_cache, 3, dims, ks, box, 128) != VLC_OK) return VLC_ERR_CUDA;
    if (prm.inflight) {
      const uint64_t dn[3] = {(uint64_t)head_dim, (uint64_t)num_kv_heads, (uint64_t)num_new_rows};
      const uint64_t kns[2] = {(uint64_t)head_dim * 2, (uint64_t)kn_row_stride * 2};
      if (encode_tmap_bf16(&prm.tm_kn64, k_new, 3, dn, kns, box, 128) != VLC_OK) return VLC_ERR_CUDA;
    } else {
      prm.tm_kn64 = prm.tm_k64;  // unused
    }
  } else {
    prm.tm_k64 = prm.tm_k;  // unused
    prm.tm_kn64 = prm.tm_k;
  }
  // Head dim 80 (the vision tower's) multiplies its 80 columns only; other head dims run on
  // the zero-padded 128 columns.
  const bool d80 = head_dim == 80;
  const void* kfn = quad_units ? (const void*)prefill_attn_quad_kernel<false>
                    : packed   ? (d80 ? (const void*)prefill_attn_kernel<true, 5> : (const void*)prefill_attn_kernel<true, 8>)
                               : (d80 ? (const void*)prefill_attn_kernel<false, 5> : (const void*)prefill_attn_kernel<false, 8>);
  const int smem_bytes = quad_units ? quad::QD_SMEM_BYTES : SMEM_BYTES;
  static std::atomic<uint64_t> smem_set[5];
  const int kind = quad_units ? 4 : (packed ? 1 : 0) + (d80 ? 2 : 0);
  if (ensure_dynamic_smem(kfn, smem_bytes, smem_set[kind]) != VLC_OK) return VLC_ERR_CUDA;
  cudaStream_t st = (cudaStream_t)stream;
  // Both kernels are launched as programmatic dependents of their predecessor in the
  // stream (the attention: of the KV scatter; the merge: of the attention).  They wait
  // (griddepcontrol.wait) before reading the predecessor's outputs, so the launch and
  // prologue overlap its tail.
  cudaLaunchAttribute pdl;
  pdl.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  pdl.val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchAttribute attrs[2];
  attrs[0] = pdl;
  attrs[1].id = cudaLaunchAttributeClusterDimension;  // quad units: clusters of 2 (CTA pairs)
  attrs[1].val.clusterDim.x = 2;
  attrs[1].val.clusterDim.y = 1;
  attrs[1].val.clusterDim.z = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(NUM_THREADS);
  cfg.dynamicSmemBytes = smem_bytes;
  cfg.stream = st;
  cfg.attrs = attrs;
  cfg.numAttrs = quad_units ? 2 : 1;
  void* args[] = {&prm};
  const cudaError_t le = cudaLaunchKernelExC(&cfg, kfn, args);
  if (le != cudaSuccess) {
    (void)cudaGetLastError();
    return VLC_ERR_CUDA;
  }
  int rc = VLC_OK;
  const int mblocks = plan_host[kPMergeBlocks];
  if (mblocks > 0) {
    cudaLaunchConfig_t mcfg = {};
    mcfg.gridDim = dim3(mblocks);
    mcfg.blockDim = dim3(256);
    mcfg.stream = st;
    mcfg.attrs = &pdl;
    mcfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&mcfg, prefill_merge_kernel, (const int32_t*)(plan_dev + plan_host[kPOffMerges]),
                           (const int32_t*)(plan_dev + plan_host[kPOffMergeBlocks]), (const __nv_bfloat16*)prm.part_o,
                           (const float*)prm.part_ml, group, prm.out, out_token_stride, head_dim) != cudaSuccess) {
      (void)cudaGetLastError();
      rc = VLC_ERR_CUDA;
    }
  }
  return rc;
}

extern "C" int vlc_prefill_attn(const void* q, int64_t q_token_stride, int total_q, int num_heads,
                                const void* k_cache, const void* v_cache, int64_t k_row_stride,
                                int64_t v_row_stride, int64_t num_slots, int num_kv_heads, int head_dim,
                                const int32_t* block_tables, int block_table_stride, int block_size,
                                const int32_t* plan_dev, const int32_t* plan_host, float softmax_scale,
                                void* out, int64_t out_token_stride, void* workspace,
                                int64_t workspace_bytes, void* stream) {
  return prefill_attn_impl(q, q_token_stride, total_q, num_heads, k_cache, v_cache, k_row_stride, v_row_stride,
                           num_slots, num_kv_heads, head_dim, block_tables, block_table_stride, block_size, plan_dev,
                           plan_host, softmax_scale, out, out_token_stride, workspace, workspace_bytes, nullptr,
                           nullptr, 0, 0, 0, stream);
}

extern "C" int vlc_prefill_attn_inflight(const void* q, int64_t q_token_stride, int total_q, int num_heads,
                                         const void* k_cache, const void* v_cache, int64_t k_row_stride,
                                         int64_t v_row_stride, int64_t num_slots, int num_kv_heads, int head_dim,
                                         const int32_t* block_tables, int block_table_stride, int block_size,
                                         const int32_t* plan_dev, const int32_t* plan_host, float softmax_scale,
                                         void* out, int64_t out_token_stride, void* workspace,
                                         int64_t workspace_bytes, const void* k_new, const void* v_new,
                                         int64_t kn_row_stride, int64_t vn_row_stride, int64_t num_new_rows,
                                         void* stream) {
  if (!k_new || !v_new) return VLC_ERR_NULL;
  return prefill_attn_impl(q, q_token_stride, total_q, num_heads, k_cache, v_cache, k_row_stride, v_row_stride,
                           num_slots, num_kv_heads, head_dim, block_tables, block_table_stride, block_size, plan_dev,
                           plan_host, softmax_scale, out, out_token_stride, workspace, workspace_bytes, k_new, v_new,
                           kn_row_stride, vn_row_stride, num_new_rows, stream);
}
