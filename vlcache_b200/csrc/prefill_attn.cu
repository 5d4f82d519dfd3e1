// Sparse-query paged prefill attention on sm_100a (tcgen05 + TMEM + TMA).
//
// Query rows are the recomputed rows of warm requests (text tokens and the
// first R vision tokens, flash-attn varlen layout).  Each query row attends,
// causally by logical position, over its sequence's paged K/V cache.
//
// Work decomposition (host planner, plan.cpp): a *tile* is T consecutive
// query tokens of one sequence x the G query heads of one KV head, packed into
// the 128 rows of a UMMA M=128 tile (row = token*G + head: GQA packing, so one
// K/V tile feeds G heads).  A *unit* is a tile over a range of 128-key blocks;
// long ranges are split into several units whose partial results are merged by
// prefill_merge_kernel.  Units are bin-packed onto a persistent grid of one CTA
// per SM.
//
// CTA roles (320 threads):
//   warps 0-3  softmax, columns 0-63 of every S row   (thread i: row i = TMEM lane i)
//   warps 4-7  softmax, columns 64-127 of every S row
//   warp  8    TMA producer: Q tiles (double-buffered), K/V tiles (2-stage ring)
//   warp  9    TMEM allocator + single-thread tcgen05.mma issuer
// TMEM (512 columns): S0 | S1 | O (128 fp32 columns each).  S is double
// buffered: Q*K^T of key tile j+1 runs while the softmax works on tile j.  Each
// softmax thread handles half a row (64 values): the two halves exchange their
// maxima through shared memory once per tile, then write P (bf16 pairs) back
// over their half of the S buffer, where the next MMA reads it as the A operand
// of O += P V (V is an MN-major smem operand).  Online softmax in the log2
// domain with lazy rescaling: the running max moves (and O is rescaled) only
// when it grows by more than 2^8.
#include <algorithm>
#include <cmath>

#include "common.cuh"
#include "plan.h"
#include "runtime.h"

namespace vlc {
namespace prefill {

constexpr int BM = 128;   // tile rows (tokens * group)
constexpr int BN = 128;   // keys per K/V tile
constexpr int HD = 128;   // head dim
constexpr int STAGES = 2; // K/V ring depth
constexpr int NUM_THREADS = 320;
constexpr int HALF_BYTES = BM * 128;          // 128 rows x 128 B (64 bf16)
constexpr int TILE_BYTES = 2 * HALF_BYTES;    // 32 KB: full 128 x 128 bf16 tile

constexpr int OFF_Q = 0;                               // 2 buffers
constexpr int OFF_K = OFF_Q + 2 * TILE_BYTES;
constexpr int OFF_V = OFF_K + STAGES * TILE_BYTES;
constexpr int OFF_X = OFF_V + STAGES * TILE_BYTES;     // row-max exchange [2 parity][2 halves][128]
constexpr int OFF_L = OFF_X + 2 * 2 * BM * 4;          // row-sum exchange [2 halves][128]
constexpr int OFF_BAR = OFF_L + 2 * BM * 4;
// barriers: q_full[2], q_empty[2], k_full[S], k_empty[S], v_full[S], v_empty[S], s_full[2], p_full[2],
//           o_done[2] (P*V of tile t completes o_done[t % 2]), xchg[2] (half-row maxima, by tile
//           parity), xsum (row sums, per unit).
// A parity wait is only sound if the barrier is at most one phase behind the completion
// waited for.  For o_done that holds per buffer: S(t) is issued only after P(t-2)*V, so
// a thread that has seen S(t) knows P*V of tile t-2 is complete.  (A single o_done
// barrier could be two phases behind and accept an older completion.)
constexpr int NUM_BARS = 4 + 4 * STAGES + 6 + 3;
constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;  // + alignment slack

constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t TMEM_S = 0;     // S buffer b at TMEM_S + 128 b
constexpr uint32_t TMEM_O = 256;

constexpr uint32_t IDESC_QK = umma_idesc_bf16(128, 128, false, false);
constexpr uint32_t IDESC_PV = umma_idesc_bf16(128, 128, false, true);

constexpr int kSoftmaxThreads = 256;

struct Params {
  CUtensorMap tm_q;   // dims {HD, num_heads, total_q}, box {64, G, T}
  CUtensorMap tm_k;   // dims {HD, Hk, num_rows},    box {64, 1, BN}
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
  __nv_bfloat16* out;
  int64_t out_token_stride;
  __nv_bfloat16* part_o;  // [num_parts][BM][HD] partial O / l (bf16)
  float* part_ml;         // [num_parts][BM][2]  (max in log2 domain, sum)
};

struct Bars {
  uint64_t* q_full;   // [2]
  uint64_t* q_empty;  // [2]
  uint64_t* k_full;
  uint64_t* k_empty;
  uint64_t* v_full;
  uint64_t* v_empty;
  uint64_t* s_full;   // [2]
  uint64_t* p_full;   // [2]
  uint64_t* o_done;   // [2]
  uint64_t* xchg;     // [2]
  uint64_t* xsum;
};

__device__ __forceinline__ Bars make_bars(uint8_t* smem) {
  uint64_t* b = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  Bars r;
  r.q_full = b;
  r.q_empty = b + 2;
  r.k_full = b + 4;
  r.k_empty = b + 4 + STAGES;
  r.v_full = b + 4 + 2 * STAGES;
  r.v_empty = b + 4 + 3 * STAGES;
  r.s_full = b + 4 + 4 * STAGES;
  r.p_full = b + 6 + 4 * STAGES;
  r.o_done = b + 8 + 4 * STAGES;
  r.xchg = b + 10 + 4 * STAGES;
  r.xsum = b + 12 + 4 * STAGES;
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

// Row (slot) of the first key of 128-key block `kb` of a unit.  Paged mode
// (block_tables != NULL, block_size % 128 == 0): through the block table.
// Contiguous mode (block_tables == NULL): key rows of the sequence start at k_base.
__device__ __forceinline__ int key_block_slot(const Params& p, const int32_t* u, int kb) {
  const int key0 = kb * BN;
  int64_t slot;
  if (p.block_tables != nullptr) {
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

__device__ __forceinline__ void issue_qk(uint32_t d_tmem, uint32_t q_addr, uint32_t k_addr) {
#pragma unroll
  for (int k = 0; k < HD / 16; ++k) {
    const uint32_t off = (k >> 2) * HALF_BYTES + (k & 3) * 32;
    umma_ss(d_tmem, umma_desc_sw128(q_addr + off, 16, 1024), umma_desc_sw128(k_addr + off, 16, 1024), IDESC_QK,
            k > 0 ? 1u : 0u);
  }
}

__device__ __forceinline__ void issue_pv(uint32_t o_tmem, uint32_t p_tmem, uint32_t v_addr, bool accumulate) {
#pragma unroll
  for (int k = 0; k < BN / 16; ++k) {
    umma_ts(o_tmem, p_tmem + k * 8, umma_desc_sw128(v_addr + k * 2048, HALF_BYTES, 1024), IDESC_PV,
            (accumulate || k > 0) ? 1u : 0u);
  }
}

__global__ void __launch_bounds__(NUM_THREADS, 1) prefill_attn_kernel(const __grid_constant__ Params p) {
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
    for (int b = 0; b < 2; ++b) {
      mbar_init(bars.q_full + b, 1);
      mbar_init(bars.q_empty + b, 1);
      mbar_init(bars.s_full + b, 1);
      mbar_init(bars.p_full + b, kSoftmaxThreads);
    }
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bars.k_full + s, 1);
      mbar_init(bars.k_empty + s, 1);
      mbar_init(bars.v_full + s, 1);
      mbar_init(bars.v_empty + s, 1);
    }
    mbar_init(bars.o_done + 0, 1);
    mbar_init(bars.o_done + 1, 1);
    mbar_init(bars.xchg + 0, kSoftmaxThreads);
    mbar_init(bars.xchg + 1, kSoftmaxThreads);
    mbar_init(bars.xsum, kSoftmaxThreads);
    fence_mbar_init();
  }
  if (warp == 8 && lane == 0) {
    tma_prefetch_desc(&p.tm_q);
    tma_prefetch_desc(&p.tm_k);
    tma_prefetch_desc(&p.tm_v);
  }
  // Rows beyond T*G of the Q buffers are never written by TMA: zero them once so
  // the unused accumulator rows stay finite.
  if (threadIdx.x < 2 * BM && (threadIdx.x & 127) >= p.rows) {
    const uint4 z = make_uint4(0, 0, 0, 0);
    const int r = threadIdx.x & 127;
    uint8_t* q = smem + OFF_Q + (threadIdx.x >> 7) * TILE_BYTES;
    uint4* r0 = reinterpret_cast<uint4*>(q + r * 128);
    uint4* r1 = reinterpret_cast<uint4*>(q + HALF_BYTES + r * 128);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      r0[i] = z;
      r1[i] = z;
    }
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 8) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int it = 0;
      for (int ui = u_begin; ui < u_end; ++ui) {
        const int32_t* u = p.units + (int64_t)ui * kUnitInts;
        const int g = u[kUKvHead];
        const int kb0 = u[kUKbBegin], kb1 = u[kUKbEnd];
        const int lu = ui - u_begin;
        const int qb = lu & 1;
        if (lu >= 2 &&
            !wait_or_abort(bars.q_empty + qb, (uint32_t)((lu >> 1) - 1) & 1u, VLC_DEV_ERR_TIMEOUT + 1, abort_flag))
          break;
        uint8_t* qdst = smem + OFF_Q + qb * TILE_BYTES;
        mbar_expect_tx(bars.q_full + qb, 2 * p.rows * 128);
        tma_load_3d(qdst, &p.tm_q, bars.q_full + qb, 0, g * p.group, u[kUQBeginA]);
        tma_load_3d(qdst + HALF_BYTES, &p.tm_q, bars.q_full + qb, 64, g * p.group, u[kUQBeginA]);
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
          const int slot = key_block_slot(p, u, kb);
          if (it >= STAGES && !wait_or_abort(bars.k_empty + s, ph ^ 1u, VLC_DEV_ERR_TIMEOUT + 2, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* kdst = smem + OFF_K + s * TILE_BYTES;
          mbar_expect_tx(bars.k_full + s, TILE_BYTES);
          tma_load_3d(kdst, &p.tm_k, bars.k_full + s, 0, g, slot);
          tma_load_3d(kdst + HALF_BYTES, &p.tm_k, bars.k_full + s, 64, g, slot);
          if (it >= STAGES && !wait_or_abort(bars.v_empty + s, ph ^ 1u, VLC_DEV_ERR_TIMEOUT + 3, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* vdst = smem + OFF_V + s * TILE_BYTES;
          mbar_expect_tx(bars.v_full + s, TILE_BYTES);
          tma_load_3d(vdst, &p.tm_v, bars.v_full + s, 0, g, slot);
          tma_load_3d(vdst + HALF_BYTES, &p.tm_v, bars.v_full + s, 64, g, slot);
        }
        if (!ok) break;
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issuer
    // Global tile sequence t over this CTA's units.  For tile t it issues, in order:
    // S(t+1) = Q K(t+1)^T (lookahead, also across a unit boundary), then
    // O += P(t) V(t) once the softmax has written P(t).
    if (lane == 0 && u_begin < u_end) {
      const uint32_t q_addr = smem_u32(smem + OFF_Q);
      const uint32_t k_addr = smem_u32(smem + OFF_K);
      const uint32_t v_addr = smem_u32(smem + OFF_V);
      const uint32_t o_tmem = tmem_base + TMEM_O;
      // cursor of the lookahead tile
      int ui = u_begin, j = 0, na = 0;
      auto unit_na = [&](int uu) {
        const int32_t* u = p.units + (int64_t)uu * kUnitInts;
        return u[kUKbEnd] - u[kUKbBegin];
      };
      // Issue S(t) for the tile at cursor (ui, j); returns false on abort.
      auto issue_s = [&](int t, int uu, int jj, int nn) -> bool {
        const int lu = uu - u_begin;
        if (jj == 0) {
          if (!wait_or_abort(bars.q_full + (lu & 1), (uint32_t)(lu >> 1) & 1u, VLC_DEV_ERR_TIMEOUT + 6, abort_flag))
            return false;
        }
        const int s = t % STAGES;
        if (!wait_or_abort(bars.k_full + s, (uint32_t)(t / STAGES) & 1u, VLC_DEV_ERR_TIMEOUT + 7, abort_flag))
          return false;
        tc_fence_after();
        issue_qk(tmem_base + TMEM_S + (t & 1) * 128, q_addr + (lu & 1) * TILE_BYTES, k_addr + s * TILE_BYTES);
        umma_commit(bars.s_full + (t & 1));
        umma_commit(bars.k_empty + s);
        if (jj == nn - 1) umma_commit(bars.q_empty + (lu & 1));
        return true;
      };
      na = unit_na(ui);
      bool ok = issue_s(0, ui, 0, na);
      int t = 0;
      while (ok) {
        // cursor (ui, j) is tile t; find tile t+1
        int un = ui, jn = j + 1, nn = na;
        if (jn == na) {
          un = ui + 1;
          jn = 0;
          nn = un < u_end ? unit_na(un) : 0;
        }
        if (un < u_end) ok = issue_s(t + 1, un, jn, nn);
        if (!ok) break;
        // O += P(t) V(t)
        const int s = t % STAGES;
        if (!wait_or_abort(bars.p_full + (t & 1), (uint32_t)(t >> 1) & 1u, VLC_DEV_ERR_TIMEOUT + 4, abort_flag) ||
            !wait_or_abort(bars.v_full + s, (uint32_t)(t / STAGES) & 1u, VLC_DEV_ERR_TIMEOUT + 5, abort_flag))
          break;
        tc_fence_after();
        issue_pv(o_tmem, tmem_base + TMEM_S + (t & 1) * 128, v_addr + s * TILE_BYTES, j > 0);
        umma_commit(bars.v_empty + s);
        umma_commit(bars.o_done + (t & 1));
        ++t;
        ui = un;
        j = jn;
        na = nn;
        if (ui >= u_end) break;
      }
    }
  } else {
    // ------------------------------------------------------------ softmax (two column halves)
    const int h = warp >> 2;            // 0: columns 0-63, 1: columns 64-127
    const int row = threadIdx.x & 127;  // == TMEM lane
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t o_addr = tmem_base + lane_off + TMEM_O + h * 64;
    float* xmax = reinterpret_cast<float*>(smem + OFF_X);   // [parity][half][row]
    float* xsum = reinterpret_cast<float*>(smem + OFF_L);   // [half][row]
    int t = 0;  // global tile counter
    for (int ui = u_begin; ui < u_end; ++ui) {
      const int32_t* u = p.units + (int64_t)ui * kUnitInts;
      const int lu = ui - u_begin;
      const int g = u[kUKvHead];
      const int kb0 = u[kUKbBegin];
      const int n = u[kUKbEnd] - kb0;
      const int kv_len = u[kUKvLen];
      const int q_begin = u[kUQBeginA], q_count = u[kUQCountA];
      const int kpos0 = u[kUKpos0A];
      const int part = u[kUPartA];
      const int tok = row / p.group;
      const bool row_valid = row < p.rows && tok < q_count;
      const int qpos = kpos0 + tok;
      float m_use = -INFINITY;
      float l_part = 0.f;   // this half's share of the row sum
      bool ok = true;
      for (int j = 0; j < n; ++j, ++t) {
        const uint32_t s_addr = tmem_base + lane_off + TMEM_S + (t & 1) * 128;
        if (!wait_or_abort(bars.s_full + (t & 1), (uint32_t)(t >> 1) & 1u, VLC_DEV_ERR_TIMEOUT + 9, abort_flag)) {
          ok = false;
          break;
        }
        __syncwarp();
        tc_fence_after();
        const int key0 = (kb0 + j) * BN;
        uint32_t sr[64];
        tmem_ld32(s_addr + h * 64, *reinterpret_cast<uint32_t(*)[32]>(&sr[0]));
        tmem_ld32(s_addr + h * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[32]));
        tmem_wait_ld();
        if (key0 + BN - 1 > kpos0) {  // tile touches the causal diagonal
          const int lim = qpos - key0 - h * 64;
#pragma unroll
          for (int c = 0; c < 64; ++c)
            if (c > lim) sr[c] = __float_as_uint(-INFINITY);
        }
        float mx0 = __uint_as_float(sr[0]), mx1 = __uint_as_float(sr[1]);
        float mx2 = __uint_as_float(sr[2]), mx3 = __uint_as_float(sr[3]);
#pragma unroll
        for (int c = 4; c < 64; c += 4) {
          mx0 = fmaxf(mx0, __uint_as_float(sr[c]));
          mx1 = fmaxf(mx1, __uint_as_float(sr[c + 1]));
          mx2 = fmaxf(mx2, __uint_as_float(sr[c + 2]));
          mx3 = fmaxf(mx3, __uint_as_float(sr[c + 3]));
        }
        // Exchange the half-row maxima (double-buffered by tile parity).  The barrier
        // also orders this half's S loads before the other half overwrites S with P.
        float* xm = xmax + (t & 1) * 2 * BM;
        xm[h * BM + row] = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3));
        tc_fence_before();
        mbar_arrive(bars.xchg + (t & 1));
        if (!wait_or_abort(bars.xchg + (t & 1), (uint32_t)(t >> 1) & 1u, VLC_DEV_ERR_TIMEOUT + 13, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const float m_tile = fmaxf(xm[row], xm[BM + row]) * p.scale_log2;
        // Lazy rescaling: only move the reference max when it grows by > 2^8.
        const bool need = m_tile > m_use + 8.0f;
        if (__any_sync(0xffffffffu, need && j > 0)) {
          // O must be stable: wait for the previous tile's P*V.
          if (!wait_or_abort(bars.o_done + ((t - 1) & 1), (uint32_t)((t - 1) >> 1) & 1u, VLC_DEV_ERR_TIMEOUT + 10,
                             abort_flag)) {
            ok = false;
            break;
          }
          __syncwarp();
          tc_fence_after();
          const float m_new = need ? m_tile : m_use;
          const float f = (need && m_use != -INFINITY) ? fast_exp2(m_use - m_new) : 1.0f;
#pragma unroll 1
          for (int cb = 0; cb < 2; ++cb) {
            uint32_t orr[32];
            tmem_ld32(o_addr + cb * 32, orr);
            tmem_wait_ld();
#pragma unroll
            for (int c = 0; c < 32; ++c) orr[c] = __float_as_uint(__uint_as_float(orr[c]) * f);
            tmem_st32(o_addr + cb * 32, orr);
          }
          l_part *= f;
          m_use = m_new;
        } else if (need) {
          m_use = m_tile;  // first tile of the unit
        }
        const float mref = (m_use == -INFINITY) ? 0.f : m_use;
        // P = exp2(s * scale_log2 - mref) as bf16 pairs; pair c reuses register c.
        float l0 = 0.f, l1 = 0.f;
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const float e0 = fast_exp2(fmaf(__uint_as_float(sr[2 * c]), p.scale_log2, -mref));
          const float e1 = fast_exp2(fmaf(__uint_as_float(sr[2 * c + 1]), p.scale_log2, -mref));
          l0 += e0;
          l1 += e1;
          sr[c] = pack_bf16x2(e0, e1);
        }
        l_part += l0 + l1;
        tmem_st32(s_addr + h * 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[0]));
        // Keys past the sequence end: zero their V rows so 0 * garbage stays 0.
        if (h == 0 && key0 + BN > kv_len) {
          const int st = t % STAGES;
          if (!wait_or_abort(bars.v_full + st, (uint32_t)(t / STAGES) & 1u, VLC_DEV_ERR_TIMEOUT + 11, abort_flag)) {
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
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(bars.p_full + (t & 1));
      }
      if (!ok) break;
      // ---------------------------------------------------------- epilogue
      xsum[h * BM + row] = l_part;
      mbar_arrive(bars.xsum);
      if (!wait_or_abort(bars.xsum, (uint32_t)lu & 1u, VLC_DEV_ERR_TIMEOUT + 14, abort_flag)) break;
      const float l_sum = xsum[row] + xsum[BM + row];
      if (!wait_or_abort(bars.o_done + ((t - 1) & 1), (uint32_t)((t - 1) >> 1) & 1u, VLC_DEV_ERR_TIMEOUT + 12,
                         abort_flag))
        break;
      __syncwarp();
      tc_fence_after();
      const float inv = l_sum > 0.f ? 1.0f / l_sum : 0.f;
      __nv_bfloat16* dst;
      if (part < 0) {
        const int head = g * p.group + (row - tok * p.group);
        dst = p.out + (int64_t)(q_begin + tok) * p.out_token_stride + (int64_t)head * HD + h * 64;
      } else {
        // Split partial: O / l as bf16 (the merge re-weights by l and the max).
        dst = p.part_o + ((int64_t)part * BM + row) * HD + h * 64;
        if (h == 0) reinterpret_cast<float2*>(p.part_ml)[(int64_t)part * BM + row] = make_float2(m_use, l_sum);
      }
      const bool store = part < 0 ? row_valid : true;
#pragma unroll 1
      for (int cb = 0; cb < 2; ++cb) {
        uint32_t orr[32];
        tmem_ld32(o_addr + cb * 32, orr);
        tmem_wait_ld();
        if (store) {
#pragma unroll
          for (int c8 = 0; c8 < 4; ++c8) {
            uint4 pk;
            pk.x = pack_bf16x2(__uint_as_float(orr[c8 * 8 + 0]) * inv, __uint_as_float(orr[c8 * 8 + 1]) * inv);
            pk.y = pack_bf16x2(__uint_as_float(orr[c8 * 8 + 2]) * inv, __uint_as_float(orr[c8 * 8 + 3]) * inv);
            pk.z = pack_bf16x2(__uint_as_float(orr[c8 * 8 + 4]) * inv, __uint_as_float(orr[c8 * 8 + 5]) * inv);
            pk.w = pack_bf16x2(__uint_as_float(orr[c8 * 8 + 6]) * inv, __uint_as_float(orr[c8 * 8 + 7]) * inv);
            *reinterpret_cast<uint4*>(dst + cb * 32 + c8 * 8) = pk;
          }
        }
      }
      tc_fence_before();
    }
  }

  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// Merge split units.  Part p holds O_p / l_p (bf16), its max m_p and sum l_p:
//   O = sum_p w_p (O_p / l_p) / sum_p w_p,   w_p = 2^(m_p - M) l_p.
// One warp per tile row (8 rows per 256-thread block, every row of every merge in
// flight at once); lane p reads part p's (m, l) so the weights take one round of
// shuffles, and each lane accumulates 4 of the 128 dims over the parts with
// independent loads.
constexpr int kMergeRowsPerBlock = 8;

__global__ void __launch_bounds__(256) prefill_merge_kernel(const int32_t* __restrict__ merges,
                                                            const __nv_bfloat16* __restrict__ part_o,
                                                            const float* __restrict__ part_ml,
                                                            int group, int rows, int blocks_per_merge,
                                                            __nv_bfloat16* __restrict__ out,
                                                            int64_t out_token_stride) {
  const int mi = blockIdx.x / blocks_per_merge;
  const int row = (blockIdx.x - mi * blocks_per_merge) * kMergeRowsPerBlock + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int32_t* m = merges + (int64_t)mi * kMergeInts;
  const int q_begin = __ldg(m + kMQBegin), q_count = __ldg(m + kMQCount), g = __ldg(m + kMKvHead);
  const int part0 = __ldg(m + kMPartBegin), nparts = __ldg(m + kMNumParts);
  if (row >= rows) return;
  const int tok = row / group;
  if (tok >= q_count) return;
  const float2* ml = reinterpret_cast<const float2*>(part_ml);
  // Pass 1: global max over the parts (lanes stride over parts).
  float M = -INFINITY;
  for (int i = lane; i < nparts; i += 32) M = fmaxf(M, __ldg(&ml[(int64_t)(part0 + i) * BM + row].x));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
  const float mref = (M == -INFINITY) ? 0.f : M;
  float L = 0.f;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int base = 0; base < nparts; base += 32) {
    float w = 0.f;
    if (base + lane < nparts) {
      const float2 v = __ldg(&ml[(int64_t)(part0 + base + lane) * BM + row]);
      w = (v.x == -INFINITY) ? 0.f : exp2f(v.x - mref) * v.y;  // weight of O_p/l_p is 2^(m_p-M) l_p
      L += w;
    }
    const int n = min(32, nparts - base);
#pragma unroll 4
    for (int i = 0; i < n; ++i) {
      const float wi = __shfl_sync(0xffffffffu, w, i);
      if (wi == 0.f) continue;  // empty or fully masked part (its O may be unwritten)
      const uint2 raw = __ldg(reinterpret_cast<const uint2*>(part_o + ((int64_t)(part0 + base + i) * BM + row) * HD) + lane);
      const float2 o01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.x));
      const float2 o23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.y));
      acc.x += wi * o01.x;
      acc.y += wi * o01.y;
      acc.z += wi * o23.x;
      acc.w += wi * o23.y;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
  const float inv = L > 0.f ? 1.0f / L : 0.f;
  const int head = g * group + (row - tok * group);
  __nv_bfloat16* dst = out + (int64_t)(q_begin + tok) * out_token_stride + (int64_t)head * HD + lane * 4;
  uint2 pk;
  pk.x = pack_bf16x2(acc.x * inv, acc.y * inv);
  pk.y = pack_bf16x2(acc.z * inv, acc.w * inv);
  *reinterpret_cast<uint2*>(dst) = pk;
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

extern "C" int vlc_prefill_attn(const void* q, int64_t q_token_stride, int total_q, int num_heads,
                                const void* k_cache, const void* v_cache, int64_t k_row_stride,
                                int64_t v_row_stride, int64_t num_slots, int num_kv_heads, int head_dim,
                                const int32_t* block_tables, int block_table_stride, int block_size,
                                const int32_t* plan_dev, const int32_t* plan_host, float softmax_scale,
                                void* out, int64_t out_token_stride, void* workspace,
                                int64_t workspace_bytes, void* stream) {
  if (!q || !k_cache || !v_cache || !plan_dev || !plan_host || !out) return VLC_ERR_NULL;
  if (head_dim != HD) return VLC_ERR_UNSUPPORTED;
  if (num_heads <= 0 || num_kv_heads <= 0 || num_heads % num_kv_heads != 0) return VLC_ERR_SHAPE;
  if (block_tables && (block_size <= 0 || block_size % BN != 0)) return VLC_ERR_UNSUPPORTED;
  if (plan_host[kPMagic] != kPlanMagic || plan_host[kPVersion] != kPlanVersion) return VLC_ERR_PLAN;
  const int group = num_heads / num_kv_heads;
  if (plan_host[kPGroup] != group || plan_host[kPNumHeads] != num_heads ||
      plan_host[kPNumKvHeads] != num_kv_heads || plan_host[kPTotalQ] != total_q)
    return VLC_ERR_PLAN;
  const int grid = plan_host[kPGrid];
  if (grid == 0 || total_q == 0) return VLC_OK;
  if (q_token_stride % 8 != 0 || out_token_stride % 8 != 0 || k_row_stride % 8 != 0 || v_row_stride % 8 != 0)
    return VLC_ERR_STRIDE;
  if (q_token_stride < (int64_t)num_heads * HD || out_token_stride < (int64_t)num_heads * HD ||
      k_row_stride < (int64_t)num_kv_heads * HD || v_row_stride < (int64_t)num_kv_heads * HD)
    return VLC_ERR_STRIDE;
  if (!aligned16(q) || !aligned16(k_cache) || !aligned16(v_cache) || !aligned16(out)) return VLC_ERR_ALIGN;
  const int64_t ws_need = vlc_prefill_workspace_size(plan_host);
  if (ws_need > 0 && (!workspace || workspace_bytes < ws_need)) return VLC_ERR_WORKSPACE;
  if (num_slots <= 0 || num_slots > 0x7fffff00) return VLC_ERR_SHAPE;

  Params prm;
  const int T = plan_host[kPTokensPerTile];
  const int rows = plan_host[kPRowsPerTile];
  {
    const uint64_t dims[3] = {(uint64_t)HD, (uint64_t)num_heads, (uint64_t)total_q};
    const uint64_t strides[2] = {(uint64_t)HD * 2, (uint64_t)q_token_stride * 2};
    const uint32_t box[3] = {64, (uint32_t)group, (uint32_t)T};
    if (encode_tmap_bf16(&prm.tm_q, q, 3, dims, strides, box, true) != VLC_OK) return VLC_ERR_CUDA;
  }
  {
    const uint64_t dims[3] = {(uint64_t)HD, (uint64_t)num_kv_heads, (uint64_t)num_slots};
    const uint64_t ks[2] = {(uint64_t)HD * 2, (uint64_t)k_row_stride * 2};
    const uint64_t vs[2] = {(uint64_t)HD * 2, (uint64_t)v_row_stride * 2};
    const uint32_t box[3] = {64, 1, (uint32_t)BN};
    if (encode_tmap_bf16(&prm.tm_k, k_cache, 3, dims, ks, box, true) != VLC_OK) return VLC_ERR_CUDA;
    if (encode_tmap_bf16(&prm.tm_v, v_cache, 3, dims, vs, box, true) != VLC_OK) return VLC_ERR_CUDA;
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
  const int64_t parts = plan_host[kPNumParts];
  prm.part_ml = (float*)workspace;  // [parts][BM][2] fp32 first (8-byte aligned), then bf16 O
  prm.part_o = workspace ? (__nv_bfloat16*)((float*)workspace + parts * BM * 2) : nullptr;

  static bool attr_set = false;
  if (!attr_set) {
    if (cudaFuncSetAttribute(prefill_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) !=
        cudaSuccess)
      return VLC_ERR_CUDA;
    attr_set = true;
  }
  cudaStream_t st = (cudaStream_t)stream;
  prefill_attn_kernel<<<grid, NUM_THREADS, SMEM_BYTES, st>>>(prm);
  int rc = launch_status();
  if (rc != VLC_OK) return rc;
  const int nmerge = plan_host[kPNumMerges];
  if (nmerge > 0) {
    const int bpm = (rows + kMergeRowsPerBlock - 1) / kMergeRowsPerBlock;
    prefill_merge_kernel<<<nmerge * bpm, 32 * kMergeRowsPerBlock, 0, st>>>(
        plan_dev + plan_host[kPOffMerges], prm.part_o, prm.part_ml, group, rows, bpm, prm.out, out_token_stride);
    rc = launch_status();
  }
  return rc;
}
