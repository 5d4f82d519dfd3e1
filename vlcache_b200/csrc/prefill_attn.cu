// Sparse-query paged prefill attention on sm_100a (tcgen05 + TMEM + TMA).
//
// Query rows are the recomputed rows of warm requests (text tokens and the
// first R vision tokens, flash-attn varlen layout).  Each query row attends,
// causally by logical position, over its sequence's paged K/V cache.
//
// Work decomposition (host planner, plan.cpp): a *tile* is T consecutive
// query tokens of one sequence x the G query heads of one KV head, packed into
// the 128 rows of a UMMA M=128 tile (row = token*G + head: GQA packing, so one
// K/V tile feeds G heads).  A *unit* is a tile x a range of 128-key blocks;
// long rows are split into several units whose partial results are merged by
// vlc_prefill_merge_kernel.  Units are bin-packed onto a persistent grid.
//
// CTA roles (192 threads):
//   warps 0-3  softmax / correction / epilogue: thread i owns tile row i, which
//              is TMEM lane i (S and O accumulators live in TMEM)
//   warp  4    TMA producer: Q tile, K/V tiles (128 keys x 128 dims, SW128)
//   warp  5    TMEM allocator + single-thread tcgen05.mma issuer
// Pipelines: K/V smem ring (2 stages), two S buffers in TMEM (QK^T of tile
// j+1 runs while softmax of tile j executes), O accumulated in TMEM.
// P is written by the softmax threads into smem in the SW128 K-major layout
// and consumed as the A operand of O += P V (V is an MN-major B operand).
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
constexpr int NUM_THREADS = 192;
constexpr int HALF_BYTES = BM * 128;          // 128 rows x 128 B (64 bf16)
constexpr int TILE_BYTES = 2 * HALF_BYTES;    // 32 KB: full 128 x 128 bf16 tile

constexpr int OFF_Q = 0;
constexpr int OFF_K = OFF_Q + TILE_BYTES;
constexpr int OFF_V = OFF_K + STAGES * TILE_BYTES;
constexpr int OFF_P = OFF_V + STAGES * TILE_BYTES;
constexpr int OFF_BAR = OFF_P + TILE_BYTES;
// barriers: q_full, q_empty, k_full[S], k_empty[S], v_full[S], v_empty[S], s_full[2], p_full, o_done
constexpr int NUM_BARS = 2 + 4 * STAGES + 2 + 2;
constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;  // + alignment slack

constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t TMEM_S0 = 0, TMEM_S1 = 128, TMEM_O = 256;

constexpr uint32_t IDESC_QK = umma_idesc_bf16(128, 128, false, false);
constexpr uint32_t IDESC_PV = umma_idesc_bf16(128, 128, false, true);

struct Params {
  CUtensorMap tm_q;   // dims {HD, num_heads, total_q}, box {64, G, T}
  CUtensorMap tm_k;   // dims {HD, Hk, num_slots},   box {64, 1, BN}
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
  float* part_o;       // [num_parts][BM][HD] unnormalised
  float* part_ml;      // [num_parts][BM][2]  (max in log2 domain, sum)
};

struct Bars {
  uint64_t* q_full;
  uint64_t* q_empty;
  uint64_t* k_full;
  uint64_t* k_empty;
  uint64_t* v_full;
  uint64_t* v_empty;
  uint64_t* s_full;
  uint64_t* p_full;
  uint64_t* o_done;
};

__device__ __forceinline__ Bars make_bars(uint8_t* smem) {
  uint64_t* b = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  Bars r;
  r.q_full = b;
  r.q_empty = b + 1;
  r.k_full = b + 2;
  r.k_empty = b + 2 + STAGES;
  r.v_full = b + 2 + 2 * STAGES;
  r.v_empty = b + 2 + 3 * STAGES;
  r.s_full = b + 2 + 4 * STAGES;
  r.p_full = b + 4 + 4 * STAGES;
  r.o_done = b + 5 + 4 * STAGES;
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

  if (warp == 5) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  if (threadIdx.x == 0) {
    *abort_flag = 0;
    mbar_init(bars.q_full, 1);
    mbar_init(bars.q_empty, 1);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bars.k_full + s, 1);
      mbar_init(bars.k_empty + s, 1);
      mbar_init(bars.v_full + s, 1);
      mbar_init(bars.v_empty + s, 1);
    }
    mbar_init(bars.s_full + 0, 1);
    mbar_init(bars.s_full + 1, 1);
    mbar_init(bars.p_full, 128);
    mbar_init(bars.o_done, 1);
    fence_mbar_init();
  }
  if (warp == 4 && lane == 0) {
    tma_prefetch_desc(&p.tm_q);
    tma_prefetch_desc(&p.tm_k);
    tma_prefetch_desc(&p.tm_v);
  }
  // Rows beyond T*G of the Q tile are never written by TMA: zero them once so
  // the unused accumulator rows stay finite.
  if (threadIdx.x < BM && threadIdx.x >= p.rows) {
    uint4 z = make_uint4(0, 0, 0, 0);
    uint4* r0 = reinterpret_cast<uint4*>(smem + OFF_Q + threadIdx.x * 128);
    uint4* r1 = reinterpret_cast<uint4*>(smem + OFF_Q + HALF_BYTES + threadIdx.x * 128);
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

  if (warp == 4) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int it = 0;
      for (int ui = u_begin; ui < u_end; ++ui) {
        const int32_t* u = p.units + (int64_t)ui * kUnitInts;
        const int g = u[kUKvHead], q_begin = u[kUQBegin];
        const int kb0 = u[kUKbBegin], kb1 = u[kUKbEnd];
        const int lu = ui - u_begin;
        if (lu > 0 && !wait_or_abort(bars.q_empty, (lu - 1) & 1, VLC_DEV_ERR_TIMEOUT + 1, abort_flag))
          break;
        mbar_expect_tx(bars.q_full, 2 * p.rows * 128);
        tma_load_3d(smem + OFF_Q, &p.tm_q, bars.q_full, 0, g * p.group, q_begin);
        tma_load_3d(smem + OFF_Q + HALF_BYTES, &p.tm_q, bars.q_full, 64, g * p.group, q_begin);
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
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t q_addr = smem_u32(smem + OFF_Q);
      const uint32_t k_addr = smem_u32(smem + OFF_K);
      const uint32_t v_addr = smem_u32(smem + OFF_V);
      const uint32_t p_addr = smem_u32(smem + OFF_P);
      int it = 0;  // global K/V tile counter (== S buffer / P / O counters)
      bool ok = true;
      auto do_pv = [&](int t) -> bool {
        const int s = t % STAGES;
        if (!wait_or_abort(bars.p_full, (uint32_t)t & 1u, VLC_DEV_ERR_TIMEOUT + 4, abort_flag)) return false;
        if (!wait_or_abort(bars.v_full + s, (uint32_t)(t / STAGES) & 1u, VLC_DEV_ERR_TIMEOUT + 5, abort_flag))
          return false;
        tc_fence_after();
        return true;
      };
      for (int ui = u_begin; ui < u_end && ok; ++ui) {
        const int32_t* u = p.units + (int64_t)ui * kUnitInts;
        const int n = u[kUKbEnd] - u[kUKbBegin];
        const int lu = ui - u_begin;
        if (!wait_or_abort(bars.q_full, (uint32_t)lu & 1u, VLC_DEV_ERR_TIMEOUT + 6, abort_flag)) break;
        tc_fence_after();
        const int t_first = it;
        for (int i = 0; i < n; ++i, ++it) {
          const int s = it % STAGES;
          if (!wait_or_abort(bars.k_full + s, (uint32_t)(it / STAGES) & 1u, VLC_DEV_ERR_TIMEOUT + 7, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d_s = tmem_base + ((it & 1) ? TMEM_S1 : TMEM_S0);
          const uint32_t kb_addr = k_addr + s * TILE_BYTES;
#pragma unroll
          for (int k = 0; k < HD / 16; ++k) {
            const uint32_t off = (k >> 2) * HALF_BYTES + (k & 3) * 32;
            umma_ss(d_s, umma_desc_sw128(q_addr + off, 16, 1024), umma_desc_sw128(kb_addr + off, 16, 1024),
                    IDESC_QK, k > 0 ? 1u : 0u);
          }
          umma_commit(bars.s_full + (it & 1));
          umma_commit(bars.k_empty + s);
          if (i == n - 1) umma_commit(bars.q_empty);
          if (i > 0) {
            const int t = it - 1;
            if (!do_pv(t)) {
              ok = false;
              break;
            }
            const uint32_t vb = v_addr + (t % STAGES) * TILE_BYTES;
#pragma unroll
            for (int k = 0; k < BN / 16; ++k) {
              const uint32_t aoff = (k >> 2) * HALF_BYTES + (k & 3) * 32;
              umma_ss(tmem_base + TMEM_O, umma_desc_sw128(p_addr + aoff, 16, 1024),
                      umma_desc_sw128(vb + k * 2048, HALF_BYTES, 1024), IDESC_PV,
                      (t > t_first || k > 0) ? 1u : 0u);
            }
            umma_commit(bars.v_empty + (t % STAGES));
            umma_commit(bars.o_done);
          }
        }
        if (!ok) break;
        // PV of the unit's last tile.
        const int t = it - 1;
        if (!do_pv(t)) break;
        const uint32_t vb = v_addr + (t % STAGES) * TILE_BYTES;
#pragma unroll
        for (int k = 0; k < BN / 16; ++k) {
          const uint32_t aoff = (k >> 2) * HALF_BYTES + (k & 3) * 32;
          umma_ss(tmem_base + TMEM_O, umma_desc_sw128(p_addr + aoff, 16, 1024),
                  umma_desc_sw128(vb + k * 2048, HALF_BYTES, 1024), IDESC_PV,
                  (t > t_first || k > 0) ? 1u : 0u);
        }
        umma_commit(bars.v_empty + (t % STAGES));
        umma_commit(bars.o_done);
      }
    }
  } else {
    // ------------------------------------------------------------ softmax warpgroup
    const int row = threadIdx.x;  // 0..127 == TMEM lane
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    uint8_t* p_row0 = smem + OFF_P + row * 128;
    const int sw = row & 7;
    int it = 0;
    for (int ui = u_begin; ui < u_end; ++ui) {
      const int32_t* u = p.units + (int64_t)ui * kUnitInts;
      const int g = u[kUKvHead], q_begin = u[kUQBegin], q_count = u[kUQCount];
      const int kpos0 = u[kUKpos0], kb0 = u[kUKbBegin], kb1 = u[kUKbEnd];
      const int kv_len = u[kUKvLen], part = u[kUPart];
      const int tok = row / p.group;
      const bool row_valid = row < p.rows && tok < q_count;
      const int qpos = kpos0 + tok;
      float m_use = -INFINITY;
      float l_sum = 0.f;
      bool ok = true;
      for (int kb = kb0; kb < kb1; ++kb, ++it) {
        if (!wait_or_abort(bars.s_full + (it & 1), (uint32_t)(it >> 1) & 1u, VLC_DEV_ERR_TIMEOUT + 8, abort_flag)) {
          ok = false;
          break;
        }
        __syncwarp();
        tc_fence_after();
        const uint32_t s_addr = tmem_base + lane_off + ((it & 1) ? TMEM_S1 : TMEM_S0);
        uint32_t sr[4][32];
        tmem_ld32(s_addr + 0, sr[0]);
        tmem_ld32(s_addr + 32, sr[1]);
        tmem_ld32(s_addr + 64, sr[2]);
        tmem_ld32(s_addr + 96, sr[3]);
        tmem_wait_ld();
        float* s = reinterpret_cast<float*>(&sr[0][0]);
        const int key0 = kb * BN;
        if (key0 + BN - 1 > kpos0) {  // tile touches the causal diagonal
          const int lim = qpos - key0;
#pragma unroll
          for (int c = 0; c < BN; ++c)
            if (c > lim) s[c] = -INFINITY;
        }
        float mx = s[0];
#pragma unroll
        for (int c = 1; c < BN; ++c) mx = fmaxf(mx, s[c]);
        const float m_tile = mx * p.scale_log2;
        // P smem buffer and O are free once PV of the previous tile finished.
        if (kb > kb0) {
          if (!wait_or_abort(bars.o_done, (uint32_t)(it - 1) & 1u, VLC_DEV_ERR_TIMEOUT + 9, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
        }
        // Lazy rescaling: only move the reference max when it grows by > 2^8.
        const bool need = m_tile > m_use + 8.0f;
        if (__any_sync(0xffffffffu, need && kb > kb0)) {
          const float m_new = need ? m_tile : m_use;
          const float f = (need && m_use != -INFINITY) ? fast_exp2(m_use - m_new) : 1.0f;
          if (kb > kb0) {
            const uint32_t o_addr = tmem_base + lane_off + TMEM_O;
#pragma unroll
            for (int cb = 0; cb < 4; ++cb) {
              uint32_t orr[32];
              tmem_ld32(o_addr + cb * 32, orr);
              tmem_wait_ld();
#pragma unroll
              for (int c = 0; c < 32; ++c) orr[c] = __float_as_uint(__uint_as_float(orr[c]) * f);
              tmem_st32(o_addr + cb * 32, orr);
            }
            tmem_wait_st();
          }
          l_sum *= f;
          m_use = m_new;
        } else if (need) {
          m_use = m_tile;  // first tile of the unit
        }
        const float mref = (m_use == -INFINITY) ? 0.f : m_use;
        // P = exp2(s * scale_log2 - mref) -> bf16, SW128 K-major layout.
#pragma unroll
        for (int ch = 0; ch < 16; ++ch) {
          float e[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            e[j] = fast_exp2(fmaf(s[ch * 8 + j], p.scale_log2, -mref));
            l_sum += e[j];
          }
          uint4 pk;
          pk.x = pack_bf16x2(e[0], e[1]);
          pk.y = pack_bf16x2(e[2], e[3]);
          pk.z = pack_bf16x2(e[4], e[5]);
          pk.w = pack_bf16x2(e[6], e[7]);
          const int h = ch >> 3, cc = ch & 7;
          *reinterpret_cast<uint4*>(p_row0 + h * HALF_BYTES + ((cc ^ sw) << 4)) = pk;
        }
        // Keys past the sequence end: zero their V rows so 0 * garbage stays 0.
        if (key0 + BN > kv_len) {
          const int st = it % STAGES;
          if (!wait_or_abort(bars.v_full + st, (uint32_t)(it / STAGES) & 1u, VLC_DEV_ERR_TIMEOUT + 10, abort_flag)) {
            ok = false;
            break;
          }
          if (key0 + row >= kv_len) {
            uint4 z = make_uint4(0, 0, 0, 0);
            uint4* v0 = reinterpret_cast<uint4*>(smem + OFF_V + st * TILE_BYTES + row * 128);
            uint4* v1 = reinterpret_cast<uint4*>(smem + OFF_V + st * TILE_BYTES + HALF_BYTES + row * 128);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              v0[i] = z;
              v1[i] = z;
            }
          }
        }
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(bars.p_full);
      }
      if (!ok) break;
      // ---------------------------------------------------------- epilogue
      if (!wait_or_abort(bars.o_done, (uint32_t)(it - 1) & 1u, VLC_DEV_ERR_TIMEOUT + 11, abort_flag)) break;
      __syncwarp();
      tc_fence_after();
      const uint32_t o_addr = tmem_base + lane_off + TMEM_O;
      if (part < 0) {
        const float inv = l_sum > 0.f ? 1.0f / l_sum : 0.f;
        const int head = g * p.group + (row - tok * p.group);
        __nv_bfloat16* dst = p.out + (int64_t)(q_begin + tok) * p.out_token_stride + (int64_t)head * HD;
#pragma unroll
        for (int cb = 0; cb < 4; ++cb) {
          uint32_t orr[32];
          tmem_ld32(o_addr + cb * 32, orr);
          tmem_wait_ld();
          if (row_valid) {
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
      } else {
        float* po = p.part_o + ((int64_t)part * BM + row) * HD;
#pragma unroll
        for (int cb = 0; cb < 4; ++cb) {
          uint32_t orr[32];
          tmem_ld32(o_addr + cb * 32, orr);
          tmem_wait_ld();
#pragma unroll
          for (int c4 = 0; c4 < 8; ++c4) {
            *reinterpret_cast<uint4*>(po + cb * 32 + c4 * 4) =
                make_uint4(orr[c4 * 4 + 0], orr[c4 * 4 + 1], orr[c4 * 4 + 2], orr[c4 * 4 + 3]);
          }
        }
        float2* ml = reinterpret_cast<float2*>(p.part_ml) + (int64_t)part * BM + row;
        *ml = make_float2(m_use, l_sum);
      }
      tc_fence_before();
    }
  }

  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// Merge split units: O = sum_p 2^(m_p - M) O_p / sum_p 2^(m_p - M) l_p.
// One warp per tile row; lanes cover the 128 dims (4 each).
__global__ void __launch_bounds__(256) prefill_merge_kernel(const int32_t* __restrict__ merges,
                                                            const float* __restrict__ part_o,
                                                            const float* __restrict__ part_ml,
                                                            int group, int rows,
                                                            __nv_bfloat16* __restrict__ out,
                                                            int64_t out_token_stride) {
  const int32_t* m = merges + (int64_t)blockIdx.x * kMergeInts;
  const int q_begin = m[kMQBegin], q_count = m[kMQCount], g = m[kMKvHead];
  const int part0 = m[kMPartBegin], nparts = m[kMNumParts];
  const int lane = threadIdx.x & 31;
  for (int row = blockIdx.y * 8 + (threadIdx.x >> 5); row < rows; row += gridDim.y * 8) {
    const int tok = row / group;
    if (tok >= q_count) continue;
    float M = -INFINITY;
    for (int i = 0; i < nparts; ++i) M = fmaxf(M, part_ml[((int64_t)(part0 + i) * BM + row) * 2]);
    const float mref = (M == -INFINITY) ? 0.f : M;
    float L = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int i = 0; i < nparts; ++i) {
      const int64_t pr = (int64_t)(part0 + i) * BM + row;
      const float mi = part_ml[pr * 2], li = part_ml[pr * 2 + 1];
      const float w = (mi == -INFINITY) ? 0.f : exp2f(mi - mref);
      L += w * li;
      const float4 o = reinterpret_cast<const float4*>(part_o + pr * HD)[lane];
      acc.x += w * o.x;
      acc.y += w * o.y;
      acc.z += w * o.z;
      acc.w += w * o.w;
    }
    const float inv = L > 0.f ? 1.0f / L : 0.f;
    const int head = g * group + (row - tok * group);
    __nv_bfloat16* dst = out + (int64_t)(q_begin + tok) * out_token_stride + (int64_t)head * HD + lane * 4;
    uint2 pk;
    pk.x = pack_bf16x2(acc.x * inv, acc.y * inv);
    pk.y = pack_bf16x2(acc.z * inv, acc.w * inv);
    *reinterpret_cast<uint2*>(dst) = pk;
  }
}

}  // namespace prefill
}  // namespace vlc

using namespace vlc;
using namespace vlc::prefill;

extern "C" int64_t vlc_prefill_workspace_size(const int32_t* plan_host) {
  if (!plan_host || plan_host[kPMagic] != kPlanMagic) return -1;
  const int64_t parts = plan_host[kPNumParts];
  return parts * (int64_t)BM * (HD + 2) * (int64_t)sizeof(float);
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
  float* ws = (float*)workspace;
  const int64_t parts = plan_host[kPNumParts];
  prm.part_o = ws;
  prm.part_ml = ws ? ws + parts * BM * HD : nullptr;

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
    dim3 mg(nmerge, (rows + 7) / 8 < 4 ? (rows + 7) / 8 : 4);
    prefill_merge_kernel<<<mg, 256, 0, st>>>(plan_dev + plan_host[kPOffMerges], prm.part_o, prm.part_ml,
                                             group, rows, prm.out, out_token_stride);
    rc = launch_status();
  }
  return rc;
}
