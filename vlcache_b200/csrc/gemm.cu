// Linear layers of the recomputed rows on sm_100a: tcgen05 GEMM with TMA and TMEM.
//
// In a warm prefill only the recomputed rows (text + the first R vision rows) go
// through the decoder layers, so every projection is a GEMM with a short M (cfg2:
// 1,123 rows) and the model's weights as B:
//   C[M, N] = A[M, K] . W[N, K]^T      (nn.Linear / F.linear, both operands K-major)
// Replaces the reference's F.linear calls for the recomputed rows
// (nanovllm/layers/linear.py:73, :154 via QKVParallelLinear, MergedColumnParallelLinear
// and RowParallelLinear in nanovllm/models/qwen3.py:75-86, 112-116) with three epilogues:
//   kPlain   : C = acc (+ bias), bf16                          (o_proj, down_proj)
//   kSiluMul : out = silu(gate) * up over the gate and up halves of gate_up_proj's
//              output (nanovllm/layers/activation.py SiluAndMul), bf16
//   kQkvRope : qkv = acc + bias rounded to bf16 (the linear's output), then RoPE of the
//              q and k heads at the row's position (rotary_embedding.py:6-14, 37-48),
//              q to the attention input and k / v straight to their paged cache slot
//              (store_kvcache, attention.py:10-40): the QKV projection, the rotary
//              embedding and the KV scatter in one kernel.
//
// Structure: persistent CTAs (one per SM).  Output tiles are 128 x 256, numbered in
// M-fastest order (the ~9 M tiles of one weight tile run side by side and share it in
// L2), and the work is the sequence of (tile, 64-wide K block) pairs.  With a workspace
// (stream-K), CTA c takes the contiguous range [c T / G, (c + 1) T / G) of the T pairs,
// so every CTA does the same number of K blocks however few tiles there are (the short-M
// projections have fewer tiles than SMs).  A tile covered by several CTAs leaves an fp32
// partial from each; each CTA then takes a ticket on the tile's counter, and the one
// whose ticket completes the tile adds the others' partials (read from L2) to its own
// accumulator and runs the epilogue.  Nobody waits for another CTA.  Without a
// workspace every CTA takes whole tiles.
//   warp 0     TMA producer: A box {64, 128} and W box {64, 256} (or two {64, 128}
//              boxes, gate rows and up rows) per 64-wide K block into a 4-stage ring;
//   warp 1     allocates TMEM (2 x 256 columns) and issues tcgen05.mma from one thread:
//              4 MMAs of 128 x 256 x 16 per K block, the stage released by a commit;
//              the accumulator of a tile alternates between the two TMEM halves;
//   warps 2-5  epilogue: thread = TMEM lane = tile row; reads its row 32 columns at a
//              time, applies the epilogue, stores to global memory, then releases the
//              TMEM half so the issuer can start the tile after next in it.
// Every mbarrier wait is bounded; a timeout records a device error and the CTA unwinds.
#include <algorithm>
#include <cmath>

#include "common.cuh"
#include "runtime.h"

namespace vlc {
namespace gemm {

constexpr int BM = 128, BN = 256, BK = 64;
constexpr int A_BYTES = BM * BK * 2;            // 16 KB
constexpr int NUM_THREADS = 192;
constexpr uint32_t TMEM_COLS = 512;

// Single-SM kernel with output tiles of BM x TN (TN = 256, or 224 / 128 where narrower
// tiles fill the SMs of a short-M projection in one wave): as many stages of
// A (16 KB) + W (TN rows x 128 B) as fit (up to 6).
template <int TN>
struct Tile {
  static constexpr int B_BYTES = TN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (225 * 1024) / STAGE_BYTES < 6 ? (225 * 1024) / STAGE_BYTES : 6;
  static constexpr int OFF_BAR = STAGES * STAGE_BYTES;
  static constexpr int NUM_BARS = 2 * STAGES + 5;  // full[S], empty[S], acc_full[2], acc_empty[2], fix_full
  static constexpr int OFF_MISC = (OFF_BAR + NUM_BARS * 8 + 127) / 128 * 128;
  static constexpr int OFF_BIAS = OFF_MISC + 64;   // each epilogue warp's copy of the tile's bias
  static constexpr int SMEM_BYTES = OFF_BIAS + 4 * 256 * 2 + 1024;
  static constexpr uint32_t IDESC = umma_idesc_bf16(BM, TN, false, false);
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
  static_assert(OFF_BIAS % 16 == 0, "alignment of the bias copies");
  static_assert(TN % 32 == 0 && TN >= 128 && TN <= 256 && 2 * TN <= (int)TMEM_COLS, "tile width");
};
constexpr int HD = 128;  // head_dim of the QKV epilogue

enum Epi : int { kPlain = 0, kSiluMul = 1, kQkvRope = 2 };

struct Params {
  CUtensorMap tm_a;  // A [M, K]: dims {K, M}, box {64, 128}
  CUtensorMap tm_b;  // W [rows, K]: dims {K, rows}, box {64, 256} (kSiluMul: {64, 128})
  int m, n, k;       // n = output columns (kSiluMul: the intermediate size)
  int m_tiles, n_tiles, tiles, k_blocks;
  int up_row0;       // kSiluMul: first W row of the up half
  __nv_bfloat16* out;
  int64_t ldo;
  const __nv_bfloat16* bias;  // [n] or null (kPlain, kQkvRope)
  // kQkvRope
  // stream-K (partials == null: whole tiles, CTA c takes tiles c, c + G, ...)
  int64_t total_kb;     // tiles * k_blocks
  float* partials;      // [2 * SMs][BN / 4][BM] float4: a CTA's first and last partial tile
  int* counters;        // [tiles] tickets (after the partials); zero before the launch, left zero
  const int64_t* positions;
  const float* cos_sin;  // [max_position, 128]: 64 cos | 64 sin
  int64_t max_position;
  __nv_bfloat16* q_out;
  int64_t q_out_stride;
  __nv_bfloat16* k_cache;
  __nv_bfloat16* v_cache;
  const int32_t* slot_mapping;
  int64_t num_slots;
  int num_heads, num_kv_heads;
};

__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, int code, volatile int* abort_flag) {
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

__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// 32 bf16 values (16 packed words) to 64 bytes at dst (16-byte aligned).
__device__ __forceinline__ void store32(__nv_bfloat16* dst, const uint32_t (&w)[16]) {
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int i = 0; i < 4; ++i) d[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
}

// The tile's bias (tile columns [0, TN) = output columns n0 + [0, TN)) copied by one
// epilogue warp into its own shared-memory buffer, with zeros at columns >= n (n is a
// multiple of 8, so a group of 8 columns is wholly inside or outside).  Issued before the
// tile's accumulator is ready, so its global-memory round trip overlaps the main loop;
// each warp has its own copy, so only the warp itself synchronises on it.
template <int TN>
__device__ __forceinline__ void stage_bias(const __nv_bfloat16* bias, int n0, int n, __nv_bfloat16* bias_s) {
  const int lane = lane_id();
  __syncwarp();  // every lane is done with the previous tile's copy
  if (lane < TN / 8) {
    const int col = n0 + 8 * lane;
    const uint4 u = col < n ? __ldg(reinterpret_cast<const uint4*>(bias + col)) : make_uint4(0, 0, 0, 0);
    reinterpret_cast<uint4*>(bias_s)[lane] = u;
  }
  __syncwarp();
}

// 8 bias values of tile columns [c, c + 8) from the warp's copy (zeros without a bias).
__device__ __forceinline__ void bias8_smem(const __nv_bfloat16* bias_s, int c, float (&b)[8]) {
  if (bias_s == nullptr) {
#pragma unroll
    for (int i = 0; i < 8; ++i) b[i] = 0.f;
    return;
  }
  const uint4 u = *reinterpret_cast<const uint4*>(bias_s + c);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[j]));
    b[2 * j] = f.x;
    b[2 * j + 1] = f.y;
  }
}

// Loads as volatile asm: issued where they stand (before the accumulator wait, itself
// volatile asm), not moved by the compiler to their first use after it.
__device__ __forceinline__ float4 ld_nc_early(const float4* ptr) {
  float4 v;
  asm volatile("ld.global.nc.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(ptr));
  return v;
}
__device__ __forceinline__ int64_t ld_nc_early(const int64_t* ptr) {
  int64_t v;
  asm volatile("ld.global.nc.s64 %0, [%1];" : "=l"(v) : "l"(ptr));
  return v;
}
__device__ __forceinline__ int32_t ld_nc_early(const int32_t* ptr) {
  int32_t v;
  asm volatile("ld.global.nc.s32 %0, [%1];" : "=r"(v) : "l"(ptr));
  return v;
}

// Per-row inputs of the QKV epilogue, loaded before the tile's accumulator is ready so
// that no global-memory round trip is left between the last MMA and the stores: the
// row's position and cache slot, and its 64 cos and 64 sin values (one table row, shared
// by every q and k head of the row).
struct QkvRow {
  int64_t slot;
  bool row_ok, pos_ok, slot_ok;
  float4 cs[32];  // cos[0, 64) in cs[0, 16), sin[0, 64) in cs[16, 32)
};

template <int EPI>
__device__ __forceinline__ void qkv_prefetch(const Params& p, int row, QkvRow& q) {
  if (EPI != kQkvRope) return;
  q.row_ok = row < p.m;
  q.slot = -1;
  q.pos_ok = q.slot_ok = false;
  int64_t pos = 0;
  if (q.row_ok) {
    pos = ld_nc_early(p.positions + row);
    q.slot = ld_nc_early(p.slot_mapping + row);
    q.pos_ok = pos >= 0 && pos < p.max_position;
    q.slot_ok = q.slot >= -1 && q.slot < p.num_slots;
  }
  // an invalid position reads table row 0 (the values are then not used)
  const float4* cs = reinterpret_cast<const float4*>(p.cos_sin + (q.pos_ok ? pos : 0) * HD);
#pragma unroll
  for (int i = 0; i < 32; ++i) q.cs[i] = ld_nc_early(cs + i);
}

// A CTA's work as segments: (tile, first K block, end K block).  Stream-K: the CTA's
// range of the global (tile, K block) sequence cut at tile boundaries; otherwise whole
// tiles blockIdx.x, blockIdx.x + gridDim.x, ...
struct SegIter {
  int64_t g, g_end;  // stream-K position / end
  int tile, kb_lo, kb_hi;
  int index;         // segments before this one in the CTA
};

__device__ __forceinline__ int64_t sk_start(const Params& p, int c) { return (int64_t)c * p.total_kb / gridDim.x; }

__device__ __forceinline__ bool seg_first(const Params& p, SegIter& it) {
  it.index = 0;
  if (p.partials == nullptr) {
    it.tile = blockIdx.x;
    it.kb_lo = 0;
    it.kb_hi = p.k_blocks;
    return it.tile < p.tiles;
  }
  it.g = sk_start(p, blockIdx.x);
  it.g_end = sk_start(p, blockIdx.x + 1);
  if (it.g >= it.g_end) return false;
  it.tile = (int)(it.g / p.k_blocks);
  it.kb_lo = (int)(it.g - (int64_t)it.tile * p.k_blocks);
  it.kb_hi = (int)min((int64_t)p.k_blocks, it.kb_lo + (it.g_end - it.g));
  return true;
}

__device__ __forceinline__ bool seg_next(const Params& p, SegIter& it) {
  ++it.index;
  if (p.partials == nullptr) {
    it.tile += gridDim.x;
    return it.tile < p.tiles;
  }
  it.g += it.kb_hi - it.kb_lo;
  if (it.g >= it.g_end) return false;
  it.tile = (int)(it.g / p.k_blocks);
  it.kb_lo = 0;
  it.kb_hi = (int)min((int64_t)p.k_blocks, it.g_end - it.g);
  return true;
}

// First CTA whose stream-K range contains global K block g (ranges are [start(c), start(c+1))).
__device__ __forceinline__ int sk_owner(const Params& p, int64_t g) {
  int c = (int)(g * gridDim.x / p.total_kb);
  while (c + 1 < (int)gridDim.x && sk_start(p, c + 1) <= g) ++c;
  while (c > 0 && sk_start(p, c) > g) --c;
  return c;
}

// Partial slot of CTA c's segment of tile t: its first segment uses slot 2c, its last
// (when it has more than one) slot 2c + 1.
__device__ __forceinline__ int sk_slot(const Params& p, int c, int t) {
  return sk_start(p, c) >= (int64_t)t * p.k_blocks ? 2 * c : 2 * c + 1;
}

// 32 accumulator columns of this thread's row: the CTA's own TMEM accumulator, or, in a
// stream-K fix-up, the sum of the tile's parts in CTA order (this CTA's own from TMEM,
// the others' partials from L2), so the result does not depend on which CTA finished last.
struct Fixup {
  int c_lo, c_hi;  // CTAs covering the tile (none when c_lo > c_hi)
  int t;
  // The other CTAs' partials staged in this CTA's free operand ring, one 128-column half at a
  // time (stage_parts), or null: read from L2 (global memory).  Partial j (the j-th other CTA
  // in CTA order) at float4 j * 4096, in the workspace's own layout.
  const float4* stage;
  uint64_t* bar;  // completes once per staged half
  bool leader;    // issues the bulk copies
  volatile int* abort_flag;  // raised when a staged half does not arrive in time
};

// Stage column half h (chunks [4 h, 4 h + 4): 64 KB of each partial, contiguous in the
// workspace) of the tile's other partials into the ring.  Every epilogue thread calls it:
// the named barrier keeps the previous half's readers ahead of the copies that overwrite it.
__device__ __forceinline__ void stage_parts(const Params& p, const Fixup& fx, int h) {
  named_bar_sync(1, 128);
  if (fx.leader) {
    // the partials (global) and the previous half's shared-memory reads, before the copy
    // engine reads the one and overwrites the other
    asm volatile("fence.proxy.async;" ::: "memory");
    mbar_expect_tx(fx.bar, (uint32_t)(fx.c_hi - fx.c_lo) * 65536u);
    int j = 0;
    for (int c = fx.c_lo; c <= fx.c_hi; ++c) {
      if (c == (int)blockIdx.x) continue;
      const float4* src = reinterpret_cast<const float4*>(p.partials) + (int64_t)sk_slot(p, c, fx.t) * (BM * BN / 4) +
                          (int64_t)h * 32 * BM;
      bulk_load_1d(const_cast<float4*>(fx.stage) + j * 4096, src, 65536u, fx.bar);
      ++j;
    }
  }
  // a timeout records the error; the CTA then unwinds after this tile (its values are void)
  if (!mbar_wait_bounded(fx.bar, (uint32_t)h, VLC_DEV_ERR_TIMEOUT + 51, VLC_WAIT_LIMIT_CYCLES)) *fx.abort_flag = 1;
}

template <int TN>
__device__ __forceinline__ void load_acc32(const Params& p, uint32_t taddr, const Fixup& fx, int r_in, int col,
                                           float (&v)[32]) {
  uint32_t raw[32];
  tmem_ld32(taddr, raw);
  tmem_wait_ld();
  if (fx.c_lo > fx.c_hi) {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(raw[i]);
    return;
  }
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = 0.f;
  for (int c = fx.c_lo; c <= fx.c_hi; ++c) {
    if (c == (int)blockIdx.x) {
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] += __uint_as_float(raw[i]);
      continue;
    }
    const int j = c - fx.c_lo - (c > (int)blockIdx.x ? 1 : 0);  // among the other CTAs
    const float4* src = fx.stage != nullptr ? fx.stage + j * 4096 + ((col & 127) / 4) * BM + r_in
                                            : reinterpret_cast<const float4*>(p.partials) +
                                                  (int64_t)sk_slot(p, c, fx.t) * (BM * TN / 4) + (col / 4) * BM + r_in;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      // staged: a shared-memory load (ld.global.cg takes global addresses only)
      const float4 f = fx.stage != nullptr ? src[i * BM] : __ldcg(src + i * BM);
      v[4 * i] += f.x;
      v[4 * i + 1] += f.y;
      v[4 * i + 2] += f.z;
      v[4 * i + 3] += f.w;
    }
  }
}

// The epilogue of one accumulator tile: thread = row r_in of the tile (global row `row`),
// output columns of tile nt.  Values come from this CTA's TMEM (`tacc`), plus the other
// CTAs' partials in a stream-K fix-up (fx).  bias_s is the warp's copy of the tile's bias
// (stage_bias) or null; qr the row's prefetched QKV inputs (qkv_prefetch).
template <int EPI, int TN>
__device__ __forceinline__ void epilogue_tile(const Params& p, uint32_t tacc, const Fixup& fx, int r_in, int row,
                                              int nt, const __nv_bfloat16* bias_s, const QkvRow& qr) {
  const bool row_ok = row < p.m;
  if (EPI == kPlain) {
    const int n0 = nt * TN;
#pragma unroll 1
    for (int c = 0; c < TN / 32; ++c) {
      if (fx.stage != nullptr && fx.c_lo <= fx.c_hi && c % 4 == 0) stage_parts(p, fx, c / 4);
      float v[32];
      load_acc32<TN>(p, tacc + c * 32, fx, r_in, c * 32, v);
      const int col = n0 + c * 32;
      if (!row_ok || col >= p.n) continue;
      uint32_t w[16];
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        float b[8];
        bias8_smem(bias_s, c * 32 + 8 * g, b);
#pragma unroll
        for (int i = 0; i < 4; ++i) w[4 * g + i] = pack2(v[8 * g + 2 * i] + b[2 * i], v[8 * g + 2 * i + 1] + b[2 * i + 1]);
      }
      __nv_bfloat16* dst = p.out + (int64_t)row * p.ldo + col;
      if (col + 32 <= p.n) {
        store32(dst, w);
      } else {
        for (int g = 0; g < 4; ++g)
          if (col + 8 * g < p.n)
            reinterpret_cast<uint4*>(dst)[g] = make_uint4(w[4 * g], w[4 * g + 1], w[4 * g + 2], w[4 * g + 3]);
      }
    }
  } else if (EPI == kSiluMul) {
    // TMEM columns [0, 128): gate of output columns n0 + [0, 128); [128, 256): up.
    const int n0 = nt * (TN / 2);
#pragma unroll 1
    for (int c = 0; c < TN / 64; ++c) {
      float g[32], u[32];
      load_acc32<TN>(p, tacc + c * 32, fx, r_in, c * 32, g);
      load_acc32<TN>(p, tacc + TN / 2 + c * 32, fx, r_in, TN / 2 + c * 32, u);
      const int col = n0 + c * 32;
      if (!row_ok || col >= p.n) continue;
      uint32_t w[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        float o[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          // gate_up_proj's output is bf16; SiluAndMul evaluates silu(x) * y in fp32
          const float x = bf16_round(g[2 * i + e]);
          const float y = bf16_round(u[2 * i + e]);
          o[e] = x / (1.0f + __expf(-x)) * y;
        }
        w[i] = pack2(o[0], o[1]);
      }
      __nv_bfloat16* dst = p.out + (int64_t)row * p.ldo + col;
      if (col + 32 <= p.n) {
        store32(dst, w);
      } else {
        for (int q = 0; q < 4; ++q)
          if (col + 8 * q < p.n)
            reinterpret_cast<uint4*>(dst)[q] = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
      }
    }
  } else {
    // kQkvRope (whole tiles only: the accumulator is this CTA's): the tile's TN columns are
    // TN / 128 heads of the [q | k | v] layout.  Each head's 128 columns go in four steps
    // of (x1: 16 columns of the first half, x2: the matching 16 of the second half); step
    // j of every head uses the row's cos / sin values [16 j, 16 j + 16), prefetched in qr.
#pragma unroll 1
    for (int hh = 0; hh < TN / HD; ++hh) {
      const int head = nt * (TN / HD) + hh;
      const bool is_q = head < p.num_heads;
      const bool is_v = head >= p.num_heads + p.num_kv_heads;
      const int col0 = head * HD;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float x1[16], x2[16];
        {
          uint32_t a1[16], a2[16];
          tmem_ld16(tacc + hh * HD + 16 * j, a1);
          tmem_ld16(tacc + hh * HD + 64 + 16 * j, a2);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            x1[i] = __uint_as_float(a1[i]);
            x2[i] = __uint_as_float(a2[i]);
          }
        }
        // (tcgen05.ld is warp-collective: rows past m load too, and write nothing)
        if (!qr.row_ok || col0 >= p.n) continue;
        // As vlc_rope_store_kvcache: a k or v row needs a valid slot, a q or k row a valid
        // position; a row that has neither is recorded and not stored (q does not use the slot).
        const bool bad_slot = !is_q && !qr.slot_ok, bad_pos = !is_v && !qr.pos_ok;
        if (bad_slot || bad_pos) {
          if (j == 0) record_error(bad_slot ? VLC_DEV_ERR_SLOT_RANGE : VLC_DEV_ERR_POSITION);
          continue;
        }
        __nv_bfloat16* dst;
        if (is_q) {
          dst = p.q_out + (int64_t)row * p.q_out_stride + (int64_t)head * HD;
        } else {
          if (qr.slot < 0) continue;
          const int kvh = is_v ? head - p.num_heads - p.num_kv_heads : head - p.num_heads;
          dst = (is_v ? p.v_cache : p.k_cache) + qr.slot * ((int64_t)p.num_kv_heads * HD) + (int64_t)kvh * HD;
        }
        // the linear's bf16 output: acc + bias, rounded (bias 8 columns at a time)
#pragma unroll
        for (int g = 0; g < 2; ++g) {
          float bx[8], by[8];
          bias8_smem(bias_s, hh * HD + 16 * j + 8 * g, bx);
          bias8_smem(bias_s, hh * HD + 64 + 16 * j + 8 * g, by);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            x1[8 * g + e] = bf16_round(x1[8 * g + e] + bx[e]);
            x2[8 * g + e] = bf16_round(x2[8 * g + e] + by[e]);
          }
        }
        if (!is_v) {
          // apply_rotary_emb in fp32, each product and sum rounded on its own
#pragma unroll
          for (int i4 = 0; i4 < 4; ++i4) {
            const float4 c4 = qr.cs[4 * j + i4];
            const float4 s4 = qr.cs[16 + 4 * j + i4];
            const float cv[4] = {c4.x, c4.y, c4.z, c4.w}, sv[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int i = 4 * i4 + e;
              const float y1 = __fsub_rn(__fmul_rn(x1[i], cv[e]), __fmul_rn(x2[i], sv[e]));
              const float y2 = __fadd_rn(__fmul_rn(x2[i], cv[e]), __fmul_rn(x1[i], sv[e]));
              x1[i] = y1;
              x2[i] = y2;
            }
          }
        }
        uint32_t w1[8], w2[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          w1[i] = pack2(x1[2 * i], x1[2 * i + 1]);
          w2[i] = pack2(x2[2 * i], x2[2 * i + 1]);
        }
        uint4* o1 = reinterpret_cast<uint4*>(dst + 16 * j);
        uint4* o2 = reinterpret_cast<uint4*>(dst + 64 + 16 * j);
        o1[0] = make_uint4(w1[0], w1[1], w1[2], w1[3]);
        o1[1] = make_uint4(w1[4], w1[5], w1[6], w1[7]);
        o2[0] = make_uint4(w2[0], w2[1], w2[2], w2[3]);
        o2[1] = make_uint4(w2[4], w2[5], w2[6], w2[7]);
      }
    }
  }
}

template <int EPI, int TN>
__global__ void __launch_bounds__(NUM_THREADS, 1) gemm_kernel(const __grid_constant__ Params p) {
  using TL = Tile<TN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + TL::OFF_BAR);
  uint64_t* empty = full + TL::STAGES;
  uint64_t* acc_full = full + 2 * TL::STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* fix_full = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + TL::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + TL::OFF_MISC + 4);
  volatile int* ticket_last = reinterpret_cast<volatile int*>(smem + TL::OFF_MISC + 8);
  const int warp = warp_id(), lane = lane_id();

  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  if (threadIdx.x == 0) {
    *abort_flag = 0;
    for (int s = 0; s < TL::STAGES; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(acc_full + b, 1);
      mbar_init(acc_empty + b, 128);
    }
    mbar_init(fix_full, 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&p.tm_a);
    tma_prefetch_desc(&p.tm_b);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      pdl_wait();  // A may be written by the kernel launched just before
      int it = 0;
      bool ok = true;
      SegIter sg;
      for (bool more = seg_first(p, sg); ok && more; more = seg_next(p, sg)) {
        const int mt = sg.tile % p.m_tiles, nt = sg.tile / p.m_tiles;
        for (int kb = sg.kb_lo; kb < sg.kb_hi; ++kb, ++it) {
          const int s = it % TL::STAGES;
          if (it >= TL::STAGES &&
              !wait_bar(empty + s, (uint32_t)((it / TL::STAGES) & 1) ^ 1u, VLC_DEV_ERR_TIMEOUT + 40, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* a_dst = smem + s * TL::STAGE_BYTES;
          uint8_t* b_dst = a_dst + A_BYTES;
          mbar_expect_tx(full + s, TL::STAGE_BYTES);
          tma_load_2d(a_dst, &p.tm_a, full + s, kb * BK, mt * BM);
          if (EPI == kSiluMul) {
            tma_load_2d(b_dst, &p.tm_b, full + s, kb * BK, nt * (TN / 2));
            tma_load_2d(b_dst + TL::B_BYTES / 2, &p.tm_b, full + s, kb * BK, p.up_row0 + nt * (TN / 2));
          } else {
            tma_load_2d(b_dst, &p.tm_b, full + s, kb * BK, nt * TN);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t base_lo = umma_desc_sw128_lo(smem_u32(smem), 16);
      constexpr uint32_t hi = umma_desc_sw128_hi(1024);
      int it = 0, local = 0;
      bool ok = true;
      SegIter sg;
      for (bool more = seg_first(p, sg); ok && more; more = seg_next(p, sg), ++local) {
        const int buf = local & 1;
        if (local >= 2 &&
            !wait_bar(acc_empty + buf, (uint32_t)((local >> 1) & 1) ^ 1u, VLC_DEV_ERR_TIMEOUT + 41, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)buf * TN;
        for (int kb = sg.kb_lo; kb < sg.kb_hi; ++kb, ++it) {
          const int s = it % TL::STAGES;
          if (!wait_bar(full + s, (uint32_t)(it / TL::STAGES) & 1u, VLC_DEV_ERR_TIMEOUT + 42, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_lo = base_lo + (uint32_t)((s * TL::STAGE_BYTES) >> 4);
          const uint32_t b_lo = a_lo + (uint32_t)(A_BYTES >> 4);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_ss_w(d, a_lo + (uint32_t)(k * 2), hi, b_lo + (uint32_t)(k * 2), hi, TL::IDESC,
                      (kb > sg.kb_lo || k > 0) ? 1u : 0u);
          umma_commit(empty + s);
        }
        if (!ok) break;
        umma_commit(acc_full + buf);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2-5)
    pdl_wait();  // positions, slots and bias may be written by the kernel launched just before
    const int quarter = warp & 3;             // TMEM lanes [32 quarter, 32 quarter + 32)
    const int r_in = quarter * 32 + lane;     // tile row
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const bool leader = warp == 2 && lane == 0;
    __nv_bfloat16* bias_s =
        p.bias != nullptr ? reinterpret_cast<__nv_bfloat16*>(smem + TL::OFF_BIAS) + (warp - 2) * 256 : nullptr;
    QkvRow qr;
    int local = 0;
    SegIter sg;
    for (bool more = seg_first(p, sg); more; more = seg_next(p, sg), ++local) {
      const int t = sg.tile;
      const int mt = t % p.m_tiles, nt = t / p.m_tiles;
      const int buf = local & 1;
      const int row = mt * BM + r_in;
      // inputs of the epilogue that do not depend on the accumulator: loaded while the MMAs run
      if (bias_s != nullptr) stage_bias<TN>(p.bias, nt * TN, p.n, bias_s);
      qkv_prefetch<EPI>(p, row, qr);
      if (!wait_bar(acc_full + buf, (uint32_t)(local >> 1) & 1u, VLC_DEV_ERR_TIMEOUT + 43, abort_flag)) break;
      __syncwarp();
      tc_fence_after();
      const uint32_t tacc = tmem_base + lane_off + (uint32_t)buf * TN;
      Fixup fx;
      fx.t = t;
      fx.c_lo = 1;
      fx.c_hi = 0;  // no partials to add
      fx.stage = nullptr;
      fx.bar = fix_full;
      fx.leader = leader;
      fx.abort_flag = abort_flag;
      if (EPI != kQkvRope && (sg.kb_lo != 0 || sg.kb_hi != p.k_blocks)) {
        // Stream-K: this CTA covers part of the tile.  Leave the partial, take a ticket.
        // Partial layout: 16-byte piece q (columns 4q .. 4q + 3) of row r at float4 index
        // q * 128 + r, so one warp instruction stores (or loads) 512 contiguous bytes.
        float4* dst = reinterpret_cast<float4*>(p.partials) +
                      (int64_t)(sg.index == 0 ? 2 * blockIdx.x : 2 * blockIdx.x + 1) * (BM * TN / 4) + r_in;
#pragma unroll 1
        for (int c = 0; c < TN / 32; ++c) {
          uint32_t v[32];
          tmem_ld32(tacc + c * 32, v);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 8; ++i)
            dst[(c * 8 + i) * BM] = make_float4(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1]),
                                                __uint_as_float(v[4 * i + 2]), __uint_as_float(v[4 * i + 3]));
        }
        named_bar_sync(1, 128);  // every row of the partial is written
        const int c_lo = sk_owner(p, (int64_t)t * p.k_blocks);
        const int c_hi = sk_owner(p, (int64_t)(t + 1) * p.k_blocks - 1);
        if (leader) {
          __threadfence();  // the partial is visible before the ticket
          const int ticket = atomicAdd(p.counters + t, 1);
          const bool last = ticket == c_hi - c_lo;
          if (last) {
            __threadfence();  // the other partials are visible to this CTA
            p.counters[t] = 0;  // ready for the next launch
          }
          *ticket_last = last ? 1 : 0;
        }
        named_bar_sync(1, 128);
        if (!*ticket_last) {
          tc_fence_before();
          mbar_arrive(acc_empty + buf);
          if (*abort_flag) break;
          continue;
        }
        fx.c_lo = c_lo;
        fx.c_hi = c_hi;
        // At the CTA's last segment every MMA has completed and no load is in flight: the
        // ring (4 x 48 KB) holds up to 3 other partials' halves (3 x 64 KB).  A CTA stages at
        // most once (its last segment), so fix_full completes phases 0 and 1.
        SegIter nx = sg;
        if (EPI == kPlain && TN == BN && c_hi - c_lo <= 3 && !seg_next(p, nx))
          fx.stage = reinterpret_cast<const float4*>(smem);
      }
      epilogue_tile<EPI, TN>(p, tacc, fx, r_in, row, nt, bias_s, qr);
      tc_fence_before();
      mbar_arrive(acc_empty + buf);
      if (*abort_flag) break;
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------------------
// The same GEMM on CTA pairs (clusters of 2, tcgen05.mma.cta_group::2): an output tile is
// 256 x 256; CTA rank r of the pair holds rows [128 r, 128 r + 128) of x's tile and rows
// [128 r, 128 r + 128) of W's tile (kSiluMul: rank 0 the gate rows, rank 1 the up rows),
// 32 KB a stage in a 6-stage ring.  Per 64-wide K block one SM reads 8 KB of operands per
// 128 x 256 x 16 of MMA work, against 12 KB in the single-SM kernel.
//   * both CTAs' TMA loads complete on the leader's (rank 0) full barrier, which the leader's
//     producer arms for both CTAs' bytes;
//   * the leader issues 4 MMAs of 256 x 256 x 16 per K block and commits to the stage's empty
//     barrier, and after a tile's last block to acc_full, in both CTAs (a commit to each);
//   * each CTA's epilogue reads its own 128 accumulator rows and arrives on the leader's
//     acc_empty (256 arrivals) so the leader can reuse the TMEM half;
//   * a cluster barrier after set-up (barriers initialised, TMEM allocated) and before
//     exit (no remote arrival lands on a CTA that has left).
// Whole tiles only: pair p takes tiles p, p + #pairs, ... (M-fastest).
constexpr int PAIR_STAGES = 6;
constexpr int PA_BYTES = 128 * BK * 2;            // 16 KB: this CTA's rows of x
constexpr int PB_BYTES = 128 * BK * 2;            // 16 KB: this CTA's rows of W
constexpr int PSTAGE = PA_BYTES + PB_BYTES;       // 32 KB
constexpr int P_OFF_BAR = PAIR_STAGES * PSTAGE;
constexpr int P_NUM_BARS = 2 * PAIR_STAGES + 4;
constexpr int P_OFF_MISC = (P_OFF_BAR + P_NUM_BARS * 8 + 127) / 128 * 128;
constexpr int P_OFF_BIAS = P_OFF_MISC + 64;
constexpr int P_SMEM_BYTES = P_OFF_BIAS + 4 * 256 * 2 + 1024;
static_assert(P_SMEM_BYTES <= 232448, "shared memory budget");
static_assert(P_OFF_BIAS % 16 == 0, "alignment of the bias copies");
constexpr uint32_t IDESC_PAIR = umma_idesc_bf16(2 * BM, BN, false, false);
constexpr int PM = 2 * BM;  // output rows of a pair tile

template <int EPI>
__global__ void __launch_bounds__(NUM_THREADS, 1) gemm_pair_kernel(const __grid_constant__ Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + P_OFF_BAR);
  uint64_t* empty = full + PAIR_STAGES;
  uint64_t* acc_full = full + 2 * PAIR_STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + P_OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + P_OFF_MISC + 4);
  const int warp = warp_id(), lane = lane_id();
  const uint32_t rank = cluster_ctarank();
  const int pair = (int)(blockIdx.x >> 1), npairs = (int)(gridDim.x >> 1);

  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, TMEM_COLS);
    tmem_relinquish_pair();
  }
  if (threadIdx.x == 0) {
    *abort_flag = 0;
    for (int s = 0; s < PAIR_STAGES; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(acc_full + b, 1);
      mbar_init(acc_empty + b, 2 * 128);
    }
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&p.tm_a);
    tma_prefetch_desc(&p.tm_b);
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers and TMEM exist before either uses the other's
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      pdl_wait();  // x may be written by the kernel launched just before
      int it = 0;
      bool ok = true;
      for (int t = pair; ok && t < p.tiles; t += npairs) {
        const int mt = t % p.m_tiles, nt = t / p.m_tiles;
        const int b_row = EPI == kSiluMul ? (rank == 0 ? nt * (BN / 2) : p.up_row0 + nt * (BN / 2))
                                          : nt * BN + (int)rank * (BN / 2);
        for (int kb = 0; kb < p.k_blocks; ++kb, ++it) {
          const int s = it % PAIR_STAGES;
          if (it >= PAIR_STAGES &&
              !wait_bar(empty + s, (uint32_t)((it / PAIR_STAGES) & 1) ^ 1u, VLC_DEV_ERR_TIMEOUT + 44, abort_flag)) {
            ok = false;
            break;
          }
          if (rank == 0) mbar_expect_tx(full + s, 2 * PSTAGE);  // both CTAs' bytes
          const uint32_t bar = mapa_shared(smem_u32(full + s), 0);
          uint8_t* a_dst = smem + s * PSTAGE;
          tma_load_2d_pair(a_dst, &p.tm_a, bar, kb * BK, mt * PM + (int)rank * BM);
          tma_load_2d_pair(a_dst + PA_BYTES, &p.tm_b, bar, kb * BK, b_row);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader only)
    if (lane == 0 && rank == 0) {
      const uint32_t base_lo = umma_desc_sw128_lo(smem_u32(smem), 16);
      constexpr uint32_t hi = umma_desc_sw128_hi(1024);
      int it = 0, local = 0;
      bool ok = true;
      for (int t = pair; ok && t < p.tiles; t += npairs, ++local) {
        const int buf = local & 1;
        if (local >= 2 &&
            !wait_bar(acc_empty + buf, (uint32_t)((local >> 1) & 1) ^ 1u, VLC_DEV_ERR_TIMEOUT + 45, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)buf * BN;
        for (int kb = 0; kb < p.k_blocks; ++kb, ++it) {
          const int s = it % PAIR_STAGES;
          if (!wait_bar(full + s, (uint32_t)(it / PAIR_STAGES) & 1u, VLC_DEV_ERR_TIMEOUT + 46, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_lo = base_lo + (uint32_t)((s * PSTAGE) >> 4);
          const uint32_t b_lo = a_lo + (uint32_t)(PA_BYTES >> 4);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_ss_pair(d, a_lo + (uint32_t)(k * 2), hi, b_lo + (uint32_t)(k * 2), hi, IDESC_PAIR,
                         (kb > 0 || k > 0) ? 1u : 0u);
          umma_commit_pair_both(empty + s);
        }
        if (!ok) break;
        umma_commit_pair_both(acc_full + buf);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2-5, both CTAs)
    pdl_wait();
    const int quarter = warp & 3;
    const int r_in = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    Fixup fx;  // whole tiles only: no partials to add, nothing to stage
    fx.t = 0;
    fx.c_lo = 1;
    fx.c_hi = 0;
    fx.stage = nullptr;
    fx.bar = nullptr;
    fx.leader = false;
    fx.abort_flag = abort_flag;
    __nv_bfloat16* bias_s =
        p.bias != nullptr ? reinterpret_cast<__nv_bfloat16*>(smem + P_OFF_BIAS) + (warp - 2) * 256 : nullptr;
    QkvRow qr;
    int local = 0;
    for (int t = pair; t < p.tiles; t += npairs, ++local) {
      const int mt = t % p.m_tiles, nt = t / p.m_tiles;
      const int buf = local & 1;
      const int row = mt * PM + (int)rank * BM + r_in;
      if (bias_s != nullptr) stage_bias<BN>(p.bias, nt * BN, p.n, bias_s);
      qkv_prefetch<EPI>(p, row, qr);
      if (!wait_bar(acc_full + buf, (uint32_t)(local >> 1) & 1u, VLC_DEV_ERR_TIMEOUT + 47, abort_flag)) break;
      __syncwarp();
      tc_fence_after();
      const uint32_t tacc = tmem_base + lane_off + (uint32_t)buf * BN;
      epilogue_tile<EPI, BN>(p, tacc, fx, r_in, row, nt, bias_s, qr);
      tc_fence_before();
      if (rank == 0)
        mbar_arrive(acc_empty + buf);
      else
        mbar_arrive_cluster(mapa_shared(smem_u32(acc_empty + buf), 0));
      if (*abort_flag) break;
    }
  }

  __syncthreads();
  cluster_sync();  // every remote arrival and every MMA into this CTA's TMEM is done
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

// Tiles of an output of m x n with tiles TN wide (kSiluMul: n = intermediate size, TN / 2
// output columns a tile).
inline void tile_counts(int kind, int m, int n, int k, int& m_tiles, int& n_tiles, int& k_blocks, int tn = BN) {
  m_tiles = (m + BM - 1) / BM;
  n_tiles = kind == kSiluMul ? (n + tn / 2 - 1) / (tn / 2) : (n + tn - 1) / tn;
  k_blocks = (k + BK - 1) / BK;
}

// Stream-K grid: one CTA per SM, each with at least 4 K blocks.
inline int streamk_grid(int64_t total_kb, int sms) {
  return (int)std::max<int64_t>(1, std::min<int64_t>(sms, total_kb / 4));
}

// Workspace layout: [partials: 2 slots per SM][tickets: one int per tile].  The partial
// region's size depends only on the SM count, so every launch on a device finds its
// tickets at the same offset and no launch's partials overlap another's tickets.
inline int64_t partials_bytes(int sms) { return 2LL * sms * BM * BN * (int64_t)sizeof(float); }

int64_t workspace_bytes(int kind, int m, int n, int k) {
  if (m <= 0 || n <= 0 || k <= 0) return 0;
  int mt, nt, kb;
  tile_counts(kind, m, n, k, mt, nt, kb);
  const int64_t tiles = (int64_t)mt * nt;
  return partials_bytes(std::max(1, vlc_num_sms())) + (tiles * 4 + 255) / 256 * 256;
}

template <int EPI, int TN>
int launch(Params& prm, const void* a, int64_t lda, const void* w, int64_t ldw, int64_t w_rows, void* workspace,
           int64_t ws_bytes, void* stream) {
  using TL = Tile<TN>;
  {
    const uint64_t dims[2] = {(uint64_t)prm.k, (uint64_t)prm.m};
    const uint64_t strides[1] = {(uint64_t)lda * 2};
    const uint32_t box[2] = {BK, BM};
    if (encode_tmap_bf16(&prm.tm_a, a, 2, dims, strides, box, 128) != VLC_OK) return VLC_ERR_CUDA;
  }
  {
    const uint64_t dims[2] = {(uint64_t)prm.k, (uint64_t)w_rows};
    const uint64_t strides[1] = {(uint64_t)ldw * 2};
    const uint32_t box[2] = {BK, (uint32_t)(EPI == kSiluMul ? TN / 2 : TN)};
    if (encode_tmap_bf16(&prm.tm_b, w, 2, dims, strides, box, 128) != VLC_OK) return VLC_ERR_CUDA;
  }
  tile_counts(EPI, prm.m, prm.n, prm.k, prm.m_tiles, prm.n_tiles, prm.k_blocks, TN);
  prm.tiles = prm.m_tiles * prm.n_tiles;
  prm.total_kb = (int64_t)prm.tiles * prm.k_blocks;
  const int sms = std::max(1, vlc_num_sms());
  // The stream-K split pays where whole tiles would leave SMs idle and each tile is long
  // enough (>= 64 K blocks) to amortise the partial write and the fix-up (measured on
  // B200: down_proj of 1,123 rows, K = 11,008, 72 tiles: 59.8 vs 67.8 us; qkv_proj, K =
  // 2,048, 90 tiles: 30.8 vs 17.8 us); elsewhere the workspace is left unused.
  // The QKV epilogue takes whole tiles only.
  const bool split = EPI != kQkvRope && prm.tiles * 4 < sms * 3 && prm.k_blocks >= 64;
  int grid;
  if (workspace != nullptr && split) {
    // Stream-K needs the whole workspace (tickets zeroed by the caller once; every launch
    // leaves them zero).
    if (ws_bytes < workspace_bytes(EPI, prm.m, prm.n, prm.k)) return VLC_ERR_WORKSPACE;
    if ((uintptr_t)workspace % 256 != 0) return VLC_ERR_ALIGN;
    grid = streamk_grid(prm.total_kb, sms);
    prm.partials = (float*)workspace;
    prm.counters = (int*)((uint8_t*)workspace + partials_bytes(sms));
  } else {
    grid = std::min(prm.tiles, sms);
    prm.counters = nullptr;
    prm.partials = nullptr;
  }
  static std::atomic<uint64_t> smem_set{0};
  if (ensure_dynamic_smem((const void*)gemm_kernel<EPI, TN>, TL::SMEM_BYTES, smem_set) != VLC_OK)
    return VLC_ERR_CUDA;
  cudaLaunchAttribute pdl;
  pdl.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  pdl.val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(NUM_THREADS);
  cfg.dynamicSmemBytes = TL::SMEM_BYTES;
  cfg.stream = (cudaStream_t)stream;
  cfg.attrs = &pdl;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, gemm_kernel<EPI, TN>, prm) != cudaSuccess) {
    (void)cudaGetLastError();
    return VLC_ERR_CUDA;
  }
  return VLC_OK;
}

// Kernel selection: 0 = automatic, 1 = single-SM 128 x 256 tiles (stream-K where it pays),
// 2 = CTA pairs (256 x 256), 3 = single-SM 128 x 128, 4 = single-SM 128 x 224 (plain only).
static std::atomic<int> g_kernel_mode{0};

template <int EPI>
int launch_pair(Params& prm, const void* a, int64_t lda, const void* w, int64_t ldw, int64_t w_rows, void* stream) {
  {
    const uint64_t dims[2] = {(uint64_t)prm.k, (uint64_t)prm.m};
    const uint64_t strides[1] = {(uint64_t)lda * 2};
    const uint32_t box[2] = {BK, BM};
    if (encode_tmap_bf16(&prm.tm_a, a, 2, dims, strides, box, 128) != VLC_OK) return VLC_ERR_CUDA;
  }
  {
    const uint64_t dims[2] = {(uint64_t)prm.k, (uint64_t)w_rows};
    const uint64_t strides[1] = {(uint64_t)ldw * 2};
    const uint32_t box[2] = {BK, (uint32_t)(BN / 2)};
    if (encode_tmap_bf16(&prm.tm_b, w, 2, dims, strides, box, 128) != VLC_OK) return VLC_ERR_CUDA;
  }
  prm.m_tiles = (prm.m + PM - 1) / PM;
  prm.n_tiles = EPI == kSiluMul ? (prm.n + BN / 2 - 1) / (BN / 2) : (prm.n + BN - 1) / BN;
  prm.tiles = prm.m_tiles * prm.n_tiles;
  prm.k_blocks = (prm.k + BK - 1) / BK;
  prm.total_kb = 0;
  prm.partials = nullptr;
  prm.counters = nullptr;
  static std::atomic<uint64_t> smem_set{0};
  if (ensure_dynamic_smem((const void*)gemm_pair_kernel<EPI>, P_SMEM_BYTES, smem_set) != VLC_OK) return VLC_ERR_CUDA;
  cudaLaunchAttribute attrs[2];
  attrs[0].id = cudaLaunchAttributeClusterDimension;
  attrs[0].val.clusterDim.x = 2;
  attrs[0].val.clusterDim.y = 1;
  attrs[0].val.clusterDim.z = 1;
  attrs[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[1].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(NUM_THREADS);
  cfg.dynamicSmemBytes = P_SMEM_BYTES;
  cfg.stream = (cudaStream_t)stream;
  cfg.attrs = attrs;
  cfg.numAttrs = 2;
  // Pairs resident at once (clusters of two SMs), queried once per device.
  static std::atomic<int> max_pairs_dev[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return VLC_ERR_CUDA;
  int max_pairs = max_pairs_dev[dev].load();
  if (max_pairs <= 0) {
    cfg.gridDim = dim3(2 * std::max(1, vlc_num_sms() / 2));
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, (const void*)gemm_pair_kernel<EPI>, &cfg) != cudaSuccess || n <= 0) {
      (void)cudaGetLastError();
      n = std::max(1, vlc_num_sms() / 2);
    }
    max_pairs = n;
    max_pairs_dev[dev].store(n);
  }
  cfg.gridDim = dim3(2 * std::min(prm.tiles, max_pairs));
  if (cudaLaunchKernelEx(&cfg, gemm_pair_kernel<EPI>, prm) != cudaSuccess) {
    (void)cudaGetLastError();
    return VLC_ERR_CUDA;
  }
  return VLC_OK;
}

// Automatic configuration: the one whose launch is estimated to end first.  Model (cycles,
// fitted to B200 timings of the 1,123-row projections of Qwen2.5-VL-3B / 7B, 32-296 K
// blocks, all four configurations): the tiles run in waves of one tile per SM (or SM
// pair); a wave with `act` SMs busy costs k_blocks * (f + s * act) -- the operands of
// every busy SM come through the shared L2, so a K block gets slower the more SMs load at
// once -- and the first wave adds the fill / drain / epilogue cost of a tile (later waves
// a fifth of it: the next tile's MMAs overlap the previous epilogue).
struct Cfg {
  int mode, tm, tn;  // vlc_linear_set_kernel mode, tile rows, tile columns (output)
  int per_unit;      // SMs per unit of work (2: CTA pairs)
  double tile, f, s;
};
constexpr Cfg kCfgs[] = {
    {2, 2 * BM, BN, 2, 9400.0, 483.0, 1.87},  // CTA pairs, 256 x 256
    {1, BM, 256, 1, 8300.0, 762.0, 0.0},      // single SM, 128 x 256
    {4, BM, 224, 1, 8500.0, 583.0, 0.67},     // single SM, 128 x 224 (plain epilogue)
    {3, BM, 128, 1, 9600.0, 400.0, 1.03},     // single SM, 128 x 128 (plain, QKV)
};

inline double estimate_cycles(const Cfg& c, int kind, int m, int n, int k_blocks, int sms) {
  const int units = std::max(1, sms / c.per_unit);
  const int cols = kind == kSiluMul ? c.tn / 2 : c.tn;
  int64_t left = (int64_t)((m + c.tm - 1) / c.tm) * ((n + cols - 1) / cols);
  double t = 0.0;
  for (int wave = 0; left > 0; ++wave, left -= units) {
    const double act = (double)std::min<int64_t>(left, units) * c.per_unit;
    t += (wave == 0 ? c.tile : 0.2 * c.tile) + k_blocks * (c.f + c.s * act);
  }
  return t;
}

inline int auto_mode(int kind, int m, int n, int k) {
  const int sms = std::max(2, vlc_num_sms());
  const int k_blocks = (k + BK - 1) / BK;
  double best = 1e300;
  int best_mode = 2;
  for (const Cfg& c : kCfgs) {
    if (kind == kSiluMul && c.mode >= 3) continue;  // gate and up halves of 128 columns
    if (kind == kQkvRope && c.mode == 4) continue;  // head-aligned tiles only
    const double t = estimate_cycles(c, kind, m, n, k_blocks, sms);
    if (t < best) {
      best = t;
      best_mode = c.mode;
    }
  }
  return best_mode;
}

// Which kernel runs a launch: the configuration asked for (vlc_linear_set_kernel), or the
// automatic one.
template <int EPI>
int dispatch(Params& prm, const void* a, int64_t lda, const void* w, int64_t ldw, int64_t w_rows, void* workspace,
             int64_t ws_bytes, void* stream) {
  int mode = g_kernel_mode.load();
  // 128-wide tiles have no room for SiLU's gate and up halves, 224-wide ones split heads:
  // those epilogues take the automatic choice instead.
  if (mode == 0 || (mode == 3 && EPI == kSiluMul) || (mode == 4 && EPI != kPlain))
    mode = auto_mode(EPI, prm.m, prm.n, prm.k);
  if (mode == 1) return launch<EPI, 256>(prm, a, lda, w, ldw, w_rows, workspace, ws_bytes, stream);
  if (mode == 3)
    return launch<EPI, EPI == kSiluMul ? 256 : 128>(prm, a, lda, w, ldw, w_rows, workspace, ws_bytes, stream);
  if (mode == 4)
    return launch<EPI, EPI == kPlain ? 224 : 256>(prm, a, lda, w, ldw, w_rows, workspace, ws_bytes, stream);
  return launch_pair<EPI>(prm, a, lda, w, ldw, w_rows, stream);
}

int check_common(const void* a, int64_t lda, const void* w, int64_t ldw, int m, int k) {
  if (!a || !w) return VLC_ERR_NULL;
  if (m < 0 || k <= 0) return VLC_ERR_SHAPE;
  if (lda < k || ldw < k) return VLC_ERR_STRIDE;
  if (lda % 8 != 0 || ldw % 8 != 0 || k % 8 != 0) return VLC_ERR_STRIDE;
  if (!aligned16(a) || !aligned16(w)) return VLC_ERR_ALIGN;
  return VLC_OK;
}

}  // namespace gemm
}  // namespace vlc

using namespace vlc;
using namespace vlc::gemm;

extern "C" int64_t vlc_linear_workspace_size(int kind, int m, int n, int k) {
  if (kind < kPlain || kind > kQkvRope) return -1;
  return workspace_bytes(kind, m, n, k);
}

extern "C" int vlc_linear(const void* x, int64_t ldx, const void* weight, int64_t ldw, const void* bias, void* out,
                          int64_t ldo, int m, int n, int k, void* workspace, int64_t workspace_bytes,
                          void* stream) {
  int rc = check_common(x, ldx, weight, ldw, m, k);
  if (rc != VLC_OK) return rc;
  if (!out) return VLC_ERR_NULL;
  if (n <= 0 || n % 8 != 0) return VLC_ERR_SHAPE;
  if (ldo < n || ldo % 8 != 0) return VLC_ERR_STRIDE;
  if (!aligned16(out) || (bias && !aligned16(bias))) return VLC_ERR_ALIGN;
  if (m == 0) return VLC_OK;
  Params prm = {};
  prm.m = m;
  prm.n = n;
  prm.k = k;
  prm.out = (__nv_bfloat16*)out;
  prm.ldo = ldo;
  prm.bias = (const __nv_bfloat16*)bias;
  return dispatch<kPlain>(prm, x, ldx, weight, ldw, n, workspace, workspace_bytes, stream);
}

extern "C" int vlc_linear_silu_mul(const void* x, int64_t ldx, const void* gate_up_weight, int64_t ldw, void* out,
                                   int64_t ldo, int m, int intermediate, int k, void* workspace,
                                   int64_t workspace_bytes, void* stream) {
  int rc = check_common(x, ldx, gate_up_weight, ldw, m, k);
  if (rc != VLC_OK) return rc;
  if (!out) return VLC_ERR_NULL;
  if (intermediate <= 0 || intermediate % 8 != 0) return VLC_ERR_SHAPE;
  if (ldo < intermediate || ldo % 8 != 0) return VLC_ERR_STRIDE;
  if (!aligned16(out)) return VLC_ERR_ALIGN;
  if (m == 0) return VLC_OK;
  Params prm = {};
  prm.m = m;
  prm.n = intermediate;
  prm.k = k;
  prm.out = (__nv_bfloat16*)out;
  prm.ldo = ldo;
  prm.up_row0 = intermediate;
  return dispatch<kSiluMul>(prm, x, ldx, gate_up_weight, ldw, 2LL * intermediate, workspace, workspace_bytes,
                          stream);
}

extern "C" int vlc_qkv_rope_store_kvcache(const void* x, int64_t ldx, const void* qkv_weight, int64_t ldw,
                                          const void* qkv_bias, const int64_t* positions,
                                          const float* cos_sin_cache, int64_t max_position, void* q_out,
                                          int64_t q_out_stride, void* k_cache, void* v_cache,
                                          const int32_t* slot_mapping, int64_t num_slots, int m, int hidden,
                                          int num_heads, int num_kv_heads, int head_dim, void* workspace,
                                          int64_t workspace_bytes, void* stream) {
  int rc = check_common(x, ldx, qkv_weight, ldw, m, hidden);
  if (rc != VLC_OK) return rc;
  if (!q_out || !k_cache || !v_cache || !slot_mapping || !positions || !cos_sin_cache) return VLC_ERR_NULL;
  if (head_dim != HD) return VLC_ERR_UNSUPPORTED;
  if (num_heads <= 0 || num_kv_heads <= 0 || num_heads % num_kv_heads != 0) return VLC_ERR_SHAPE;
  if (max_position <= 0 || num_slots <= 0) return VLC_ERR_SHAPE;
  if (q_out_stride < (int64_t)num_heads * HD || q_out_stride % 8 != 0) return VLC_ERR_STRIDE;
  if (!aligned16(q_out) || !aligned16(k_cache) || !aligned16(v_cache) || !aligned16(cos_sin_cache) ||
      (qkv_bias && !aligned16(qkv_bias)))
    return VLC_ERR_ALIGN;
  if (m == 0) return VLC_OK;
  const int n = (num_heads + 2 * num_kv_heads) * HD;
  Params prm = {};
  prm.m = m;
  prm.n = n;
  prm.k = hidden;
  prm.bias = (const __nv_bfloat16*)qkv_bias;
  prm.positions = positions;
  prm.cos_sin = cos_sin_cache;
  prm.max_position = max_position;
  prm.q_out = (__nv_bfloat16*)q_out;
  prm.q_out_stride = q_out_stride;
  prm.k_cache = (__nv_bfloat16*)k_cache;
  prm.v_cache = (__nv_bfloat16*)v_cache;
  prm.slot_mapping = slot_mapping;
  prm.num_slots = num_slots;
  prm.num_heads = num_heads;
  prm.num_kv_heads = num_kv_heads;
  return dispatch<kQkvRope>(prm, x, ldx, qkv_weight, ldw, n, workspace, workspace_bytes, stream);
}

extern "C" int vlc_linear_set_kernel(int mode) {
  if (mode < 0 || mode > 4) return VLC_ERR_UNSUPPORTED;
  g_kernel_mode.store(mode);
  return VLC_OK;
}
