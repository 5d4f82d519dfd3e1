// KV-cache row kernels: the paged scatter (store_kvcache) and the M-RoPE
// position shift of reused vision K.  Both are HBM-bound row copies done with
// 128-bit vector loads/stores, one warp-slice per row.
#include <cmath>

#include "common.cuh"
#include "runtime.h"

namespace vlc {

// ---------------------------------------------------------------------------
// store_kvcache: k_cache.view(-1, D)[slot[i]] = key[i]  (and V), slot -1 skipped.
// Semantics of nanovllm/layers/attention.py:10-30 (Triton store_kvcache_kernel).
// One warp per token; each lane moves 16-byte chunks of the K and V rows.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) store_kvcache_kernel(
    const uint4* __restrict__ key, int64_t key_stride16, const uint4* __restrict__ value,
    int64_t value_stride16, uint4* __restrict__ k_cache, uint4* __restrict__ v_cache,
    const int32_t* __restrict__ slot_mapping, int num_tokens, int chunks_per_row,
    int64_t num_slots) {
  pdl_launch_dependents();  // the attention that follows may start its prologue
  const int token = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (token >= num_tokens) return;
  const int lane = threadIdx.x & 31;
  const int slot = __ldg(slot_mapping + token);
  if (slot == -1) return;
  if (slot < -1 || (int64_t)slot >= num_slots) {
    if (lane == 0) record_error(VLC_DEV_ERR_SLOT_RANGE);
    return;
  }
  const uint4* ks = key + (int64_t)token * key_stride16;
  const uint4* vs = value + (int64_t)token * value_stride16;
  uint4* kd = k_cache + (int64_t)slot * chunks_per_row;
  uint4* vd = v_cache + (int64_t)slot * chunks_per_row;
  for (int c = lane; c < chunks_per_row; c += 32) {
    const uint4 kv = __ldg(ks + c);
    const uint4 vv = __ldg(vs + c);
    kd[c] = kv;
    vd[c] = vv;
  }
}

// ---------------------------------------------------------------------------
// M-RoPE shift.  Rotate-half pairs (j, j+half): a K row stored rotated at
// position p is re-rotated by the per-section delta d_sec(j):
//   y1 = x1*cos(a_j) - x2*sin(a_j),  y2 = x2*cos(a_j) + x1*sin(a_j),
//   a_j = inv_freq[j] * d_sec(j)
// which equals the rotation at p + d because R(a+b) = R(b) R(a) per pair.
// Thread = one head x 8 consecutive pairs (two 16-byte loads); V rows are
// copied with the same threads when moving rows to new slots.
// ---------------------------------------------------------------------------
constexpr int kMaxHalf = 128;
struct RopeTable {
  float c[kMaxHalf];
  float s[kMaxHalf];
};

__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint4 u;
  u.x = pack_bf16x2(f[0], f[1]);
  u.y = pack_bf16x2(f[2], f[3]);
  u.z = pack_bf16x2(f[4], f[5]);
  u.w = pack_bf16x2(f[6], f[7]);
  return u;
}

constexpr int kShiftRowsPerThread = 2;

// 4 blocks per SM (64 registers, no spill) instead of the 3 that 72 registers allow.
__global__ void __launch_bounds__(256, 4) mrope_shift_kernel(
    __nv_bfloat16* __restrict__ k_cache, __nv_bfloat16* __restrict__ v_cache,
    int64_t layer_stride, int64_t num_slots, int num_kv_heads, int head_dim,
    const int32_t* __restrict__ src_slots, const int32_t* __restrict__ dst_slots, int num_rows,
    const __grid_constant__ RopeTable tab) {
  const int half = head_dim >> 1;
  const int chunks_per_head = half >> 3;  // 8 pairs per thread
  const int threads_per_row = num_kv_heads * chunks_per_head;
  const int rows_per_block = blockDim.x / threads_per_row;
  const int r_local = threadIdx.x / threads_per_row;
  const int t = threadIdx.x - r_local * threads_per_row;
  // The cos/sin table in shared memory: threads of a warp index it by their pair chunk,
  // which the constant bank would serialise.
  __shared__ float4 s_cs[2][kMaxHalf / 4];
  for (int i = threadIdx.x; i < half / 4; i += blockDim.x) {
    s_cs[0][i] = make_float4(tab.c[4 * i], tab.c[4 * i + 1], tab.c[4 * i + 2], tab.c[4 * i + 3]);
    s_cs[1][i] = make_float4(tab.s[4 * i], tab.s[4 * i + 1], tab.s[4 * i + 2], tab.s[4 * i + 3]);
  }
  __syncthreads();
  if (r_local >= rows_per_block) return;
  const int layer = blockIdx.y;
  const int head = t / chunks_per_head;
  const int c = t - head * chunks_per_head;
  const int64_t row_elems = (int64_t)num_kv_heads * head_dim;
  const int64_t lbase = (int64_t)layer * layer_stride + (int64_t)head * head_dim + c * 8;
  const bool move_v = v_cache != nullptr && dst_slots != nullptr;
  // kShiftRowsPerThread rows per thread, every K and V load issued before any math.
  int64_t so[kShiftRowsPerThread], dof[kShiftRowsPerThread];
  bool live[kShiftRowsPerThread];
  uint4 u1[kShiftRowsPerThread], u2[kShiftRowsPerThread], w1[kShiftRowsPerThread], w2[kShiftRowsPerThread];
#pragma unroll
  for (int k = 0; k < kShiftRowsPerThread; ++k) {
    const int row = (blockIdx.x * kShiftRowsPerThread + k) * rows_per_block + r_local;
    live[k] = row < num_rows;
    if (!live[k]) continue;
    const int src = __ldg(src_slots + row);
    const int dst = dst_slots ? __ldg(dst_slots + row) : src;
    if (src < 0 || dst < 0 || (int64_t)src >= num_slots || (int64_t)dst >= num_slots) {
      if (t == 0 && layer == 0) record_error(VLC_DEV_ERR_SLOT_RANGE);
      live[k] = false;
      continue;
    }
    so[k] = lbase + (int64_t)src * row_elems;
    dof[k] = lbase + (int64_t)dst * row_elems;
    u1[k] = *reinterpret_cast<const uint4*>(k_cache + so[k]);
    u2[k] = *reinterpret_cast<const uint4*>(k_cache + so[k] + half);
    if (move_v) {
      // the same thread moves the two matching 16-byte chunks of the V row
      w1[k] = *reinterpret_cast<const uint4*>(v_cache + so[k]);
      w2[k] = *reinterpret_cast<const uint4*>(v_cache + so[k] + half);
    }
  }
  float csv[8], snv[8];
  *reinterpret_cast<float4*>(&csv[0]) = s_cs[0][2 * c];
  *reinterpret_cast<float4*>(&csv[4]) = s_cs[0][2 * c + 1];
  *reinterpret_cast<float4*>(&snv[0]) = s_cs[1][2 * c];
  *reinterpret_cast<float4*>(&snv[4]) = s_cs[1][2 * c + 1];
#pragma unroll
  for (int k = 0; k < kShiftRowsPerThread; ++k) {
    if (!live[k]) continue;
    float x1[8], x2[8], y1[8], y2[8];
    unpack8(u1[k], x1);
    unpack8(u2[k], x2);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float t1 = __fmul_rn(x2[i], snv[i]);
      const float t2 = __fmul_rn(x1[i], snv[i]);
      y1[i] = __fmaf_rn(x1[i], csv[i], -t1);
      y2[i] = __fmaf_rn(x2[i], csv[i], t2);
    }
    *reinterpret_cast<uint4*>(k_cache + dof[k]) = pack8(y1);
    *reinterpret_cast<uint4*>(k_cache + dof[k] + half) = pack8(y2);
    if (move_v) {
      *reinterpret_cast<uint4*>(v_cache + dof[k]) = w1[k];
      *reinterpret_cast<uint4*>(v_cache + dof[k] + half) = w2[k];
    }
  }
}

// ---------------------------------------------------------------------------
// Rotary embedding of new rows fused with the paged KV scatter.
// Semantics of nanovllm/layers/rotary_embedding.py:6-14 + 37-48 (apply_rotary_emb on
// query and key, cos/sin gathered from cos_sin_cache[positions]) followed by
// store_kvcache (nanovllm/layers/attention.py:10-40):
//   q_out[i] = rope(q[i], positions[i]);  the K row roped and the V row copied to
//   k_cache / v_cache row slot_mapping[i] (slot -1: neither stored).
// Without slot_mapping the roped K rows go to k_out instead (RotaryEmbedding.forward).
// cos_sin_cache rows are the caller's [max_position, 128] fp32 (64 cos | 64 sin).  Each
// fp32 product, sum and difference is rounded on its own (no FMA contraction), as the
// reference function evaluates them op by op, and the result is rounded to bf16 to
// nearest even.  Thread = 8 rotate-half pairs (j, j + 64) of one head in kRopeTokens
// consecutive tokens: two 16-byte loads and stores per token, all loads issued before
// any math; a token group's threads cover its query heads, then its key heads, then
// its value heads (copied).
// ---------------------------------------------------------------------------
constexpr int kRopeDim = 128;                 // head_dim == rotary_dim
constexpr int kRopeThreads = kRopeDim / 16;   // threads per head (8 pairs each)
constexpr int kRopeTokens = 2;                // tokens per thread: all their loads issued first

// 5 blocks per SM (48 registers, no spill): 40 warps keep more rows in flight than the 4 blocks
// (64 registers) the unconstrained build allows.
__global__ void __launch_bounds__(256, 5) rope_store_kvcache_kernel(
    const int64_t* __restrict__ positions, const __nv_bfloat16* q, int64_t q_stride, __nv_bfloat16* q_out,
    int64_t q_out_stride, const __nv_bfloat16* key, int64_t key_stride, const __nv_bfloat16* __restrict__ value,
    int64_t value_stride, const float* __restrict__ cos_sin, int64_t max_position,
    __nv_bfloat16* __restrict__ k_cache, __nv_bfloat16* __restrict__ v_cache,
    const int32_t* __restrict__ slot_mapping, int64_t num_slots, __nv_bfloat16* k_out, int64_t k_out_stride,
    int num_tokens, int num_heads, int num_kv_heads) {
  pdl_launch_dependents();  // the attention that follows may start its prologue
  const int per_group = (num_heads + 2 * num_kv_heads) * kRopeThreads;
  const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t groups = ((int64_t)num_tokens + kRopeTokens - 1) / kRopeTokens;
  if (gid >= groups * per_group) return;
  const int64_t grp = gid / per_group;
  const int u = (int)(gid - grp * per_group);
  const int head = u / kRopeThreads;  // query heads, key heads, value heads
  const int c = u - head * kRopeThreads;
  const bool is_q = head < num_heads;
  const bool is_v = head >= num_heads + num_kv_heads;
  const int kh = head - num_heads;                 // key head (is_q false, is_v false)
  const int vh = head - num_heads - num_kv_heads;  // value head (is_v)
  const int64_t row_elems = (int64_t)num_kv_heads * kRopeDim;
  constexpr int half = kRopeDim / 2;
  __nv_bfloat16* const dst_base = is_v ? v_cache : is_q ? q_out : slot_mapping != nullptr ? k_cache : k_out;
  // First every load that depends on nothing: the row chunks, slots and positions of all
  // the thread's tokens go out together (one memory latency), then the checks.
  uint4 a[kRopeTokens], b[kRopeTokens];
  int64_t slot[kRopeTokens], pos[kRopeTokens], dst_off[kRopeTokens];
#pragma unroll
  for (int t = 0; t < kRopeTokens; ++t) {
    const int token = (int)(grp * kRopeTokens + t);
    slot[t] = -1;
    pos[t] = 0;
    if (token >= num_tokens || (is_v && slot_mapping == nullptr)) continue;  // no value rows to copy
    const __nv_bfloat16* src = is_v ? value + (int64_t)token * value_stride + vh * kRopeDim
                               : is_q ? q + (int64_t)token * q_stride + head * kRopeDim
                                      : key + (int64_t)token * key_stride + kh * kRopeDim;
    a[t] = *reinterpret_cast<const uint4*>(src + 8 * c);
    b[t] = *reinterpret_cast<const uint4*>(src + half + 8 * c);
    if (!is_q && slot_mapping != nullptr) slot[t] = __ldg(slot_mapping + token);
    if (!is_v) pos[t] = __ldg(positions + token);
  }
#pragma unroll
  for (int t = 0; t < kRopeTokens; ++t) {
    const int token = (int)(grp * kRopeTokens + t);
    dst_off[t] = -1;  // nothing to store
    if (token >= num_tokens || (is_v && slot_mapping == nullptr)) continue;
    if (slot[t] < -1 || slot[t] >= num_slots) {
      if (c == 0) record_error(VLC_DEV_ERR_SLOT_RANGE);
      continue;
    }
    if (!is_v && (pos[t] < 0 || pos[t] >= max_position)) {
      if (c == 0) record_error(VLC_DEV_ERR_POSITION);
      continue;
    }
    if (is_q)
      dst_off[t] = (int64_t)token * q_out_stride + head * kRopeDim;
    else if (slot_mapping == nullptr)
      dst_off[t] = is_v ? -1 : (int64_t)token * k_out_stride + kh * kRopeDim;
    else if (slot[t] >= 0)
      dst_off[t] = slot[t] * row_elems + (is_v ? vh : kh) * kRopeDim;
  }
#pragma unroll
  for (int t = 0; t < kRopeTokens; ++t) {
    if (dst_off[t] < 0) continue;
    __nv_bfloat16* dst = dst_base + dst_off[t];
    if (!is_v) {
      const float4* cs = reinterpret_cast<const float4*>(cos_sin + pos[t] * kRopeDim);
      const float4 c0 = __ldg(cs + 2 * c), c1 = __ldg(cs + 2 * c + 1);
      const float4 s0 = __ldg(cs + half / 4 + 2 * c), s1 = __ldg(cs + half / 4 + 2 * c + 1);
      const float cv[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
      const float sv[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
      float x1[8], x2[8];
      unpack8(a[t], x1);
      unpack8(b[t], x2);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float y1 = __fsub_rn(__fmul_rn(x1[i], cv[i]), __fmul_rn(x2[i], sv[i]));
        const float y2 = __fadd_rn(__fmul_rn(x2[i], cv[i]), __fmul_rn(x1[i], sv[i]));
        x1[i] = y1;
        x2[i] = y2;
      }
      a[t] = pack8(x1);
      b[t] = pack8(x2);
    }
    *reinterpret_cast<uint4*>(dst + 8 * c) = a[t];
    *reinterpret_cast<uint4*>(dst + half + 8 * c) = b[t];
  }
}

// inv_freq[j] in fp32 exactly as the RoPE reference builds it:
//   1 / (theta ** (float(2j) / float(dim)))
static float inv_freq_f32(float theta, int j, int head_dim) {
  const float e = (float)(2 * j) / (float)head_dim;
  const float p = powf(theta, e);
  return 1.0f / p;
}

}  // namespace vlc

using namespace vlc;

extern "C" int vlc_store_kvcache(const void* key, int64_t key_stride, const void* value,
                                 int64_t value_stride, void* k_cache, void* v_cache,
                                 const int32_t* slot_mapping, int num_tokens, int row_elems,
                                 int64_t num_slots, void* stream) {
  if (num_tokens < 0 || row_elems <= 0) return VLC_ERR_SHAPE;
  if (num_tokens == 0) return VLC_OK;
  if (!key || !value || !k_cache || !v_cache || !slot_mapping) return VLC_ERR_NULL;
  if (row_elems % 8 != 0 || key_stride % 8 != 0 || value_stride % 8 != 0) return VLC_ERR_STRIDE;
  if (key_stride < row_elems || value_stride < row_elems) return VLC_ERR_STRIDE;
  if (!aligned16(key) || !aligned16(value) || !aligned16(k_cache) || !aligned16(v_cache))
    return VLC_ERR_ALIGN;
  const int warps = 8;
  dim3 grid((num_tokens + warps - 1) / warps);
  store_kvcache_kernel<<<grid, warps * 32, 0, (cudaStream_t)stream>>>(
      (const uint4*)key, key_stride / 8, (const uint4*)value, value_stride / 8, (uint4*)k_cache,
      (uint4*)v_cache, slot_mapping, num_tokens, row_elems / 8, num_slots);
  return launch_status();
}

extern "C" int vlc_rope_store_kvcache(const int64_t* positions, const void* q, int64_t q_stride, void* q_out,
                                      int64_t q_out_stride, const void* key, int64_t key_stride,
                                      const void* value, int64_t value_stride, const float* cos_sin_cache,
                                      int64_t max_position, int rotary_dim, void* k_cache, void* v_cache,
                                      const int32_t* slot_mapping, int64_t num_slots, void* k_out,
                                      int64_t k_out_stride, int num_tokens, int num_heads, int num_kv_heads,
                                      int head_dim, void* stream) {
  if (num_tokens < 0 || num_heads <= 0 || num_kv_heads <= 0 || max_position <= 0) return VLC_ERR_SHAPE;
  if (head_dim != kRopeDim || rotary_dim != head_dim) return VLC_ERR_UNSUPPORTED;
  if (num_tokens == 0) return VLC_OK;
  if (!positions || !q || !q_out || !key || !cos_sin_cache) return VLC_ERR_NULL;
  const bool fused = slot_mapping != nullptr;
  if (fused ? (!value || !k_cache || !v_cache) : !k_out) return VLC_ERR_NULL;
  if (fused && num_slots <= 0) return VLC_ERR_SHAPE;
  if (q_stride % 8 || q_out_stride % 8 || key_stride % 8 || (fused && value_stride % 8) ||
      (!fused && k_out_stride % 8))
    return VLC_ERR_STRIDE;
  if (q_stride < (int64_t)num_heads * head_dim || q_out_stride < (int64_t)num_heads * head_dim ||
      key_stride < (int64_t)num_kv_heads * head_dim || (fused && value_stride < (int64_t)num_kv_heads * head_dim) ||
      (!fused && k_out_stride < (int64_t)num_kv_heads * head_dim))
    return VLC_ERR_STRIDE;
  if (!aligned16(q) || !aligned16(q_out) || !aligned16(key) || !aligned16(cos_sin_cache) ||
      (fused && (!aligned16(value) || !aligned16(k_cache) || !aligned16(v_cache))) || (!fused && !aligned16(k_out)))
    return VLC_ERR_ALIGN;
  const int64_t threads =
      ((int64_t)num_tokens + kRopeTokens - 1) / kRopeTokens * (num_heads + 2 * num_kv_heads) * kRopeThreads;
  const int block = 256;
  const int64_t grid = (threads + block - 1) / block;
  if (grid > 0x7fffffff) return VLC_ERR_SHAPE;
  rope_store_kvcache_kernel<<<(unsigned)grid, block, 0, (cudaStream_t)stream>>>(
      positions, (const __nv_bfloat16*)q, q_stride, (__nv_bfloat16*)q_out, q_out_stride,
      (const __nv_bfloat16*)key, key_stride, (const __nv_bfloat16*)value, value_stride, cos_sin_cache,
      max_position, (__nv_bfloat16*)k_cache, (__nv_bfloat16*)v_cache, slot_mapping, num_slots,
      (__nv_bfloat16*)k_out, k_out_stride, num_tokens, num_heads, num_kv_heads);
  return launch_status();
}

extern "C" int vlc_mrope_shift(void* k_cache, void* v_cache, int64_t layer_stride, int num_layers,
                               int64_t num_slots, int num_kv_heads, int head_dim,
                               const int32_t* src_slots, const int32_t* dst_slots, int num_rows,
                               const int32_t* delta_thw, const int32_t* mrope_section,
                               float rope_theta, void* stream) {
  if (num_rows < 0 || num_layers < 0) return VLC_ERR_SHAPE;
  if (num_rows == 0 || num_layers == 0) return VLC_OK;
  if (!k_cache || !src_slots || !delta_thw || !mrope_section) return VLC_ERR_NULL;
  if (head_dim % 16 != 0 || head_dim / 2 > kMaxHalf || num_kv_heads <= 0) return VLC_ERR_UNSUPPORTED;
  const int half = head_dim / 2;
  if (mrope_section[0] < 0 || mrope_section[1] < 0 || mrope_section[2] < 0 ||
      mrope_section[0] + mrope_section[1] + mrope_section[2] != half)
    return VLC_ERR_SHAPE;
  const int threads_per_row = num_kv_heads * (half / 8);
  if (threads_per_row > 256) return VLC_ERR_UNSUPPORTED;
  if (!aligned16(k_cache) || (v_cache && !aligned16(v_cache))) return VLC_ERR_ALIGN;
  if (num_layers > 1 && (layer_stride % 8 != 0 || layer_stride < num_slots * num_kv_heads * head_dim))
    return VLC_ERR_STRIDE;
  RopeTable tab;
  for (int j = 0; j < half; ++j) {
    const int sec = j < mrope_section[0] ? 0 : (j < mrope_section[0] + mrope_section[1] ? 1 : 2);
    const double a = (double)inv_freq_f32(rope_theta, j, head_dim) * (double)delta_thw[sec];
    tab.c[j] = (float)cos(a);
    tab.s[j] = (float)sin(a);
  }
  const int rows_per_block = 256 / threads_per_row;
  const int rows_per_grid_x = rows_per_block * kShiftRowsPerThread;
  dim3 grid((num_rows + rows_per_grid_x - 1) / rows_per_grid_x, num_layers);
  mrope_shift_kernel<<<grid, rows_per_block * threads_per_row, 0, (cudaStream_t)stream>>>(
      (__nv_bfloat16*)k_cache, (__nv_bfloat16*)v_cache, layer_stride, num_slots, num_kv_heads,
      head_dim, src_slots, dst_slots, num_rows, tab);
  return launch_status();
}
