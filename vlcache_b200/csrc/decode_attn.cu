// Split-K paged flash-decode (one query token per sequence), sm_100a.
//
// Decode is HBM-bound (every K/V byte is read once per step), so the design
// goal is bytes in flight, not tensor throughput:
//   * grid = (key split, KV head, sequence); each CTA streams one split of one
//     KV head's pages through a 3-stage TMA ring (64 keys x 128 dims of K and V
//     per stage, 128-byte swizzled), two CTAs per SM;
//   * GQA packing: the G query heads of the KV head form the M rows of
//     m16n8k16 bf16 MMAs, so each K/V byte is read from smem exactly once;
//   * 4 consumer warps each take 16 keys of every stage and keep their own
//     online-softmax state; a dedicated producer warp issues the TMA loads;
//   * splits are merged with their log-sum-exp by decode_combine_kernel.
// The grid depends only on (num_seqs, max_context_len), never on device data,
// so the launch is CUDA-graph capturable; per-sequence lengths are read on the
// device and CTAs past a sequence's last split exit immediately.
#include <algorithm>
#include <cmath>
#include <mutex>

#include "common.cuh"
#include "runtime.h"

namespace vlc {
namespace decode {

constexpr int HD = 128;
constexpr int CHUNK = 64;                  // keys per stage
constexpr int STAGES = 3;
constexpr int NCW = 4;                     // consumer warps
constexpr int NUM_THREADS = (NCW + 1) * 32;
constexpr int HALF = CHUNK * 128;          // 64 keys x 64 dims bf16 = 8 KB
constexpr int KV_TILE = 2 * HALF;          // 16 KB
constexpr int STAGE_BYTES = 2 * KV_TILE;   // K + V
constexpr int OFF_BAR = STAGES * STAGE_BYTES;
constexpr int SMEM_BYTES = OFF_BAR + 2 * STAGES * 8 + 16 + 1024;
constexpr int MAX_GROUP = 16;

struct Params {
  CUtensorMap tm_k;  // dims {HD, Hk, num_slots}, box {64, 1, CHUNK}
  CUtensorMap tm_v;
  const __nv_bfloat16* q;
  int64_t q_seq_stride;
  const int32_t* block_tables;
  int bt_stride;
  int block_size;
  const int32_t* context_lens;
  int split_keys;
  int max_splits;
  int group;
  int num_heads;
  float scale_log2;
  int64_t num_slots;
  __nv_bfloat16* out;
  int64_t out_seq_stride;
  float* part_o;   // [num_seqs][max_splits][num_heads][HD]
  float* part_ml;  // [num_seqs][max_splits][num_heads][2]
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void named_bar_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

__global__ void __launch_bounds__(NUM_THREADS, 2) decode_attn_kernel(const __grid_constant__ Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* empty = full + STAGES;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + OFF_BAR + 2 * STAGES * 8);

  const int split = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
  int len = __ldg(p.context_lens + b);
  // The grid (and the partials' workspace) covers max_splits * split_keys keys, the
  // host's max_context_len rounded up: a longer device length is recorded and clamped,
  // so no split index reaches past the partials of this sequence.
  const int cap = p.max_splits * p.split_keys;
  if (len > cap) {
    if (split == 0 && g == 0 && threadIdx.x == 0) record_error(VLC_DEV_ERR_LENGTH);
    len = cap;
  }
  const int nsplit = len > 0 ? (len + p.split_keys - 1) / p.split_keys : 0;
  const int G = p.group;
  const int warp = warp_id(), lane = lane_id();
  if (split >= nsplit) {
    // Empty sequence: define the output as zeros (written once, by split 0).
    if (len <= 0 && split == 0) {
      for (int i = threadIdx.x; i < G * HD; i += blockDim.x) {
        const int h = g * G + i / HD;
        p.out[(int64_t)b * p.out_seq_stride + (int64_t)h * HD + (i % HD)] = __float2bfloat16(0.f);
      }
    }
    return;
  }
  const int k_begin = split * p.split_keys;
  const int k_end = min(len, k_begin + p.split_keys);
  const int nchunks = (k_end - k_begin + CHUNK - 1) / CHUNK;

  if (threadIdx.x == 0) {
    *abort_flag = 0;
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, NCW);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == NCW) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&p.tm_k);
      tma_prefetch_desc(&p.tm_v);
      const int32_t* bt = p.block_tables + (int64_t)b * p.bt_stride;
      for (int c = 0; c < nchunks; ++c) {
        const int s = c % STAGES;
        if (c >= STAGES) {
          const uint32_t par = (uint32_t)((c / STAGES) - 1) & 1u;
          if (!mbar_try_wait(empty + s, par)) {
            const long long t0 = clock64();
            bool ok = false;
            while (!*abort_flag) {
              if (mbar_try_wait(empty + s, par)) { ok = true; break; }
              if (clock64() - t0 > VLC_WAIT_LIMIT_CYCLES) {
                record_error(VLC_DEV_ERR_TIMEOUT + 20);
                *abort_flag = 1;
                break;
              }
            }
            if (!ok) break;
          }
        }
        const int key0 = k_begin + c * CHUNK;
        const int pidx = key0 / p.block_size;
        const int page = pidx < p.bt_stride ? __ldg(bt + pidx) : -1;  // past the row: recorded below
        int64_t slot = (int64_t)page * p.block_size + key0 % p.block_size;
        if (page < 0 || slot + CHUNK > p.num_slots) {
          record_error(VLC_DEV_ERR_BLOCK_RANGE);
          slot = p.num_slots;  // fully out of range: TMA fills zeros
        }
        uint8_t* st = smem + s * STAGE_BYTES;
        mbar_expect_tx(full + s, STAGE_BYTES);
        tma_load_3d(st, &p.tm_k, full + s, 0, g, (int)slot);
        tma_load_3d(st + HALF, &p.tm_k, full + s, 64, g, (int)slot);
        tma_load_3d(st + KV_TILE, &p.tm_v, full + s, 0, g, (int)slot);
        tma_load_3d(st + KV_TILE + HALF, &p.tm_v, full + s, 64, g, (int)slot);
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  const int r = lane >> 2, t = lane & 3;
  // Q fragments (rows = the G query heads of KV head g; rows >= G are zero).
  uint32_t qa[8][4];
  {
    const __nv_bfloat16* q0 = p.q + (int64_t)b * p.q_seq_stride + (int64_t)(g * G) * HD;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const int c0 = kk * 16 + 2 * t;
      qa[kk][0] = r < G ? *reinterpret_cast<const uint32_t*>(q0 + r * HD + c0) : 0u;
      qa[kk][1] = r + 8 < G ? *reinterpret_cast<const uint32_t*>(q0 + (r + 8) * HD + c0) : 0u;
      qa[kk][2] = r < G ? *reinterpret_cast<const uint32_t*>(q0 + r * HD + c0 + 8) : 0u;
      qa[kk][3] = r + 8 < G ? *reinterpret_cast<const uint32_t*>(q0 + (r + 8) * HD + c0 + 8) : 0u;
    }
  }
  float o[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  const uint32_t smem_base = smem_u32(smem);
  const int mi = lane >> 3, ri = lane & 7;
  bool ok = true;

  for (int c = 0; c < nchunks; ++c) {
    const int s = c % STAGES;
    const uint32_t par = (uint32_t)(c / STAGES) & 1u;
    if (!mbar_try_wait(full + s, par)) {
      const long long t0 = clock64();
      while (true) {
        if (mbar_try_wait(full + s, par)) break;
        if (*abort_flag || clock64() - t0 > VLC_WAIT_LIMIT_CYCLES) {
          if (!*abort_flag) record_error(VLC_DEV_ERR_TIMEOUT + 21);
          *abort_flag = 1;
          ok = false;
          break;
        }
      }
      if (!ok) break;
    }
    __syncwarp();
    const uint32_t kbase = smem_base + s * STAGE_BYTES;
    const uint32_t vbase = kbase + KV_TILE;
    const int key0 = k_begin + c * CHUNK;
    // ---- S = Q K^T for this warp's 16 keys (two n8 tiles)
    float sacc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const int key = warp * 16 + (mi >> 1) * 8 + ri;
      const int ch = 2 * kk + (mi & 1);
      const uint32_t addr = kbase + (ch >> 3) * HALF + key * 128 + (((ch & 7) ^ (key & 7)) << 4);
      uint32_t b0, b1, b2, b3;
      ldsm_x4(addr, b0, b1, b2, b3);
      mma16816(sacc[0], qa[kk], b0, b1);
      mma16816(sacc[1], qa[kk], b2, b3);
    }
    // ---- mask keys past the split end, online softmax (log2 domain)
    const bool tail = key0 + CHUNK > k_end;
    if (tail) {
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int key = key0 + warp * 16 + j * 8 + 2 * t + (e & 1);
          if (key >= k_end) sacc[j][e] = -INFINITY;
        }
    }
    float mx0 = fmaxf(fmaxf(sacc[0][0], sacc[0][1]), fmaxf(sacc[1][0], sacc[1][1]));
    float mx1 = fmaxf(fmaxf(sacc[0][2], sacc[0][3]), fmaxf(sacc[1][2], sacc[1][3]));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(m0, mx0 * p.scale_log2);
    const float mn1 = fmaxf(m1, mx1 * p.scale_log2);
    const float f0 = (m0 == -INFINITY) ? 0.f : fast_exp2(m0 - mn0);
    const float f1 = (m1 == -INFINITY) ? 0.f : fast_exp2(m1 - mn1);
    m0 = mn0;
    m1 = mn1;
    const float r0 = (mn0 == -INFINITY) ? 0.f : mn0;
    const float r1 = (mn1 == -INFINITY) ? 0.f : mn1;
    float pv[2][4];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      pv[j][0] = fast_exp2(fmaf(sacc[j][0], p.scale_log2, -r0));
      pv[j][1] = fast_exp2(fmaf(sacc[j][1], p.scale_log2, -r0));
      pv[j][2] = fast_exp2(fmaf(sacc[j][2], p.scale_log2, -r1));
      pv[j][3] = fast_exp2(fmaf(sacc[j][3], p.scale_log2, -r1));
    }
    l0 = l0 * f0 + (pv[0][0] + pv[0][1] + pv[1][0] + pv[1][1]);
    l1 = l1 * f1 + (pv[0][2] + pv[0][3] + pv[1][2] + pv[1][3]);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      o[j][0] *= f0;
      o[j][1] *= f0;
      o[j][2] *= f1;
      o[j][3] *= f1;
    }
    uint32_t pa[4];
    pa[0] = pack_bf16x2(pv[0][0], pv[0][1]);
    pa[1] = pack_bf16x2(pv[0][2], pv[0][3]);
    pa[2] = pack_bf16x2(pv[1][0], pv[1][1]);
    pa[3] = pack_bf16x2(pv[1][2], pv[1][3]);
    // Zero V rows of keys past the split end (their P is 0, but the rows may hold NaN bits).
    if (tail) {
      if (lane < 16) {
        const int krow = warp * 16 + lane;
        if (key0 + krow >= k_end) {
          uint4* v0 = reinterpret_cast<uint4*>(smem + s * STAGE_BYTES + KV_TILE + krow * 128);
          uint4* v1 = reinterpret_cast<uint4*>(smem + s * STAGE_BYTES + KV_TILE + HALF + krow * 128);
          const uint4 z = make_uint4(0, 0, 0, 0);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            v0[i] = z;
            v1[i] = z;
          }
        }
      }
      __syncwarp();
    }
    // ---- O += P V  (16 n8 tiles over the head dim)
#pragma unroll
    for (int jp = 0; jp < 8; ++jp) {
      const int key = warp * 16 + (mi & 1) * 8 + ri;
      const int ch = 2 * jp + (mi >> 1);
      const uint32_t addr = vbase + (ch >> 3) * HALF + key * 128 + (((ch & 7) ^ (key & 7)) << 4);
      uint32_t b0, b1, b2, b3;
      ldsm_x4_t(addr, b0, b1, b2, b3);
      mma16816(o[2 * jp], pa, b0, b1);
      mma16816(o[2 * jp + 1], pa, b2, b3);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(empty + s);
  }

  // -------------------------------------------------------------- merge warps
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  // All consumer warps are done with the ring and every TMA load completed
  // (each was waited on), so the stage memory is reused for the merge.
  named_bar_sync(1, NCW * 32);
  if (!ok || *abort_flag) return;
  float* sm_o = reinterpret_cast<float*>(smem);                 // [NCW][16][HD]
  float* sm_ml = reinterpret_cast<float*>(smem + NCW * 16 * HD * 4);  // [NCW][16][2]
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int d = j * 8 + 2 * t;
    *reinterpret_cast<float2*>(sm_o + (warp * 16 + r) * HD + d) = make_float2(o[j][0], o[j][1]);
    *reinterpret_cast<float2*>(sm_o + (warp * 16 + r + 8) * HD + d) = make_float2(o[j][2], o[j][3]);
  }
  if (t == 0) {
    sm_ml[(warp * 16 + r) * 2] = m0;
    sm_ml[(warp * 16 + r) * 2 + 1] = l0;
    sm_ml[(warp * 16 + r + 8) * 2] = m1;
    sm_ml[(warp * 16 + r + 8) * 2 + 1] = l1;
  }
  named_bar_sync(1, NCW * 32);
  // 128 threads: row = tid / 8 (16 rows), 16 dims each.
  const int tid = threadIdx.x;
  const int row = tid >> 3;
  const int d0 = (tid & 7) * 16;
  if (row >= G) return;
  float M = -INFINITY;
#pragma unroll
  for (int w = 0; w < NCW; ++w) M = fmaxf(M, sm_ml[(w * 16 + row) * 2]);
  const float mref = (M == -INFINITY) ? 0.f : M;
  float wgt[NCW];
  float L = 0.f;
#pragma unroll
  for (int w = 0; w < NCW; ++w) {
    const float mw = sm_ml[(w * 16 + row) * 2];
    wgt[w] = (mw == -INFINITY) ? 0.f : fast_exp2(mw - mref);
    L += wgt[w] * sm_ml[(w * 16 + row) * 2 + 1];
  }
  float acc[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    float a = 0.f;
#pragma unroll
    for (int w = 0; w < NCW; ++w) a += wgt[w] * sm_o[(w * 16 + row) * HD + d0 + i];
    acc[i] = a;
  }
  const int h = g * G + row;
  if (nsplit == 1) {
    const float inv = L > 0.f ? 1.0f / L : 0.f;
    __nv_bfloat16* dst = p.out + (int64_t)b * p.out_seq_stride + (int64_t)h * HD + d0;
    uint4 v0, v1;
    v0.x = pack_bf16x2(acc[0] * inv, acc[1] * inv);
    v0.y = pack_bf16x2(acc[2] * inv, acc[3] * inv);
    v0.z = pack_bf16x2(acc[4] * inv, acc[5] * inv);
    v0.w = pack_bf16x2(acc[6] * inv, acc[7] * inv);
    v1.x = pack_bf16x2(acc[8] * inv, acc[9] * inv);
    v1.y = pack_bf16x2(acc[10] * inv, acc[11] * inv);
    v1.z = pack_bf16x2(acc[12] * inv, acc[13] * inv);
    v1.w = pack_bf16x2(acc[14] * inv, acc[15] * inv);
    reinterpret_cast<uint4*>(dst)[0] = v0;
    reinterpret_cast<uint4*>(dst)[1] = v1;
  } else {
    const int64_t pi = ((int64_t)b * p.max_splits + split) * p.num_heads + h;
    float4* dst = reinterpret_cast<float4*>(p.part_o + pi * HD + d0);
#pragma unroll
    for (int i = 0; i < 4; ++i) dst[i] = make_float4(acc[4 * i], acc[4 * i + 1], acc[4 * i + 2], acc[4 * i + 3]);
    if ((tid & 7) == 0) reinterpret_cast<float2*>(p.part_ml)[pi] = make_float2(M, L);
  }
}

// Merge the splits of each (sequence, head): one warp per head, 4 dims per lane.
__global__ void __launch_bounds__(128) decode_combine_kernel(const float* __restrict__ part_o,
                                                             const float* __restrict__ part_ml,
                                                             const int32_t* __restrict__ context_lens,
                                                             int split_keys, int max_splits, int num_heads,
                                                             __nv_bfloat16* __restrict__ out,
                                                             int64_t out_seq_stride) {
  const int b = blockIdx.x;
  const int h = blockIdx.y * 4 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (h >= num_heads) return;
  const int len = min(__ldg(context_lens + b), max_splits * split_keys);  // as clamped by the decode kernel
  const int nsplit = len > 0 ? (len + split_keys - 1) / split_keys : 0;
  if (nsplit <= 1) return;  // written directly by the decode kernel
  float M = -INFINITY;
  for (int s = 0; s < nsplit; ++s)
    M = fmaxf(M, part_ml[(((int64_t)b * max_splits + s) * num_heads + h) * 2]);
  const float mref = (M == -INFINITY) ? 0.f : M;
  float L = 0.f;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int s = 0; s < nsplit; ++s) {
    const int64_t pi = ((int64_t)b * max_splits + s) * num_heads + h;
    const float ms = part_ml[pi * 2], ls = part_ml[pi * 2 + 1];
    const float w = (ms == -INFINITY) ? 0.f : exp2f(ms - mref);
    L += w * ls;
    const float4 v = reinterpret_cast<const float4*>(part_o + pi * HD)[lane];
    acc.x += w * v.x;
    acc.y += w * v.y;
    acc.z += w * v.z;
    acc.w += w * v.w;
  }
  const float inv = L > 0.f ? 1.0f / L : 0.f;
  uint2 pk;
  pk.x = pack_bf16x2(acc.x * inv, acc.y * inv);
  pk.y = pack_bf16x2(acc.z * inv, acc.w * inv);
  *reinterpret_cast<uint2*>(out + (int64_t)b * out_seq_stride + (int64_t)h * HD + lane * 4) = pk;
}

// Key-split length: small enough to give every SM several CTAs, large enough
// (>= 512 keys) to amortise the per-CTA prologue/merge.  Depends only on host
// values so the grid is fixed for graph capture.
static int choose_split_keys(int num_seqs, int num_kv_heads, int max_context_len, int num_sms) {
  const int64_t pairs = (int64_t)num_seqs * num_kv_heads;
  const int64_t target_ctas = 8LL * num_sms;
  int64_t splits = (target_ctas + pairs - 1) / std::max<int64_t>(1, pairs);
  splits = std::max<int64_t>(1, splits);
  int64_t sk = (max_context_len + splits - 1) / splits;
  sk = ((sk + 255) / 256) * 256;
  sk = std::max<int64_t>(512, std::min<int64_t>(sk, 2048));
  return (int)sk;
}

}  // namespace decode
}  // namespace vlc

using namespace vlc;
using namespace vlc::decode;

extern "C" int64_t vlc_decode_workspace_size(int num_seqs, int num_heads, int num_kv_heads,
                                             int max_context_len) {
  if (num_seqs <= 0 || num_heads <= 0 || num_kv_heads <= 0 || max_context_len <= 0) return 0;
  const int sk = choose_split_keys(num_seqs, num_kv_heads, max_context_len, vlc_num_sms());
  const int64_t max_splits = (max_context_len + sk - 1) / sk;
  if (max_splits <= 1) return 0;
  return (int64_t)num_seqs * max_splits * num_heads * (HD + 2) * (int64_t)sizeof(float);
}

extern "C" int vlc_decode_attn(const void* q, int64_t q_seq_stride, int num_seqs, int num_heads,
                               const void* k_cache, const void* v_cache, int64_t num_slots, int num_kv_heads,
                               int head_dim, const int32_t* block_tables, int block_table_stride,
                               int block_size, const int32_t* context_lens, int max_context_len,
                               float softmax_scale, void* out, int64_t out_seq_stride, void* workspace,
                               int64_t workspace_bytes, void* stream) {
  if (num_seqs < 0 || max_context_len < 0) return VLC_ERR_SHAPE;
  if (num_seqs == 0) return VLC_OK;
  if (!q || !k_cache || !v_cache || !block_tables || !context_lens || !out) return VLC_ERR_NULL;
  if (head_dim != HD) return VLC_ERR_UNSUPPORTED;
  if (num_heads <= 0 || num_kv_heads <= 0 || num_heads % num_kv_heads != 0) return VLC_ERR_SHAPE;
  const int G = num_heads / num_kv_heads;
  if (G > MAX_GROUP) return VLC_ERR_UNSUPPORTED;
  if (block_size <= 0 || block_size % CHUNK != 0) return VLC_ERR_UNSUPPORTED;
  if (q_seq_stride % 8 != 0 || out_seq_stride % 8 != 0) return VLC_ERR_STRIDE;
  if (!aligned16(q) || !aligned16(k_cache) || !aligned16(v_cache) || !aligned16(out)) return VLC_ERR_ALIGN;
  if (num_slots <= 0 || num_slots > 0x7fffff00) return VLC_ERR_SHAPE;
  if (max_context_len == 0) max_context_len = 1;
  if (num_kv_heads > 65535 || num_seqs > 65535) return VLC_ERR_SHAPE;

  const int sk = choose_split_keys(num_seqs, num_kv_heads, max_context_len, vlc_num_sms());
  const int max_splits = (max_context_len + sk - 1) / sk;
  const int64_t ws_need = vlc_decode_workspace_size(num_seqs, num_heads, num_kv_heads, max_context_len);
  if (ws_need > 0 && (!workspace || workspace_bytes < ws_need)) return VLC_ERR_WORKSPACE;

  Params prm;
  {
    const uint64_t dims[3] = {(uint64_t)HD, (uint64_t)num_kv_heads, (uint64_t)num_slots};
    const uint64_t strides[2] = {(uint64_t)HD * 2, (uint64_t)num_kv_heads * HD * 2};
    const uint32_t box[3] = {64, 1, (uint32_t)CHUNK};
    if (encode_tmap_bf16(&prm.tm_k, k_cache, 3, dims, strides, box, 128) != VLC_OK) return VLC_ERR_CUDA;
    if (encode_tmap_bf16(&prm.tm_v, v_cache, 3, dims, strides, box, 128) != VLC_OK) return VLC_ERR_CUDA;
  }
  prm.q = (const __nv_bfloat16*)q;
  prm.q_seq_stride = q_seq_stride;
  prm.block_tables = block_tables;
  prm.bt_stride = block_table_stride;
  prm.block_size = block_size;
  prm.context_lens = context_lens;
  prm.split_keys = sk;
  prm.max_splits = max_splits;
  prm.group = G;
  prm.num_heads = num_heads;
  prm.scale_log2 = softmax_scale * 1.4426950408889634f;
  prm.num_slots = num_slots;
  prm.out = (__nv_bfloat16*)out;
  prm.out_seq_stride = out_seq_stride;
  float* ws = (float*)workspace;
  prm.part_o = ws;
  prm.part_ml = ws ? ws + (int64_t)num_seqs * max_splits * num_heads * HD : nullptr;

  static std::atomic<uint64_t> smem_set{0};
  if (ensure_dynamic_smem((const void*)decode_attn_kernel, SMEM_BYTES, smem_set) != VLC_OK) return VLC_ERR_CUDA;
  cudaStream_t st = (cudaStream_t)stream;
  dim3 grid(max_splits, num_kv_heads, num_seqs);
  decode_attn_kernel<<<grid, NUM_THREADS, SMEM_BYTES, st>>>(prm);
  int rc = launch_status();
  if (rc != VLC_OK || max_splits <= 1) return rc;
  dim3 cg(num_seqs, (num_heads + 3) / 4);
  decode_combine_kernel<<<cg, 128, 0, st>>>(prm.part_o, prm.part_ml, context_lens, sk, max_splits, num_heads,
                                           prm.out, out_seq_stride);
  return launch_status();
}

// ---------------------------------------------------------------------------
// Decode without any device allocation.
//
// Some callers cannot allocate device memory at all: a runtime that hands this
// library a fixed memory budget up front, a host process that is not allowed to
// call cudaMalloc after start-up, or code running where an allocation could block
// or fail at a bad time.  For them the split-K partial results live in one
// file-scope device array that is part of the library image, so every GPU that
// loads the library holds it until the process exits.
//
//   * Limit: kNoAllocScratchBytes (8 MiB).  A request whose split partials need more
//     (vlc_decode_workspace_size() > 8 MiB) is rejected with VLC_ERR_WORKSPACE before
//     anything is launched.
//   * Nothing in the array has to start at zero: every split that the combine step
//     reads is written by the same call first.  The array keeps the last call's
//     contents.
//   * All calls on a device share the one array: two calls whose kernels overlap on
//     the GPU (different streams, or different host threads) race on it.  Serialise
//     them, e.g. on one stream.
//   * Host code cannot use the array's name as a device address; its address is
//     fetched once per device with cudaGetSymbolAddress by the first call made while
//     that device is current.  Make that first call before any stream capture.
// ---------------------------------------------------------------------------
namespace vlc {
namespace decode {

constexpr int64_t kNoAllocScratchBytes = 8ll << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
static void* g_noalloc_ptr[kMaxDevices] = {nullptr};
static std::mutex g_noalloc_mutex;

static int noalloc_scratch(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return VLC_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) {
      cudaGetLastError();
      return VLC_ERR_CUDA;
    }
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return VLC_OK;
}

}  // namespace decode
}  // namespace vlc

extern "C" int64_t vlc_decode_noalloc_scratch_bytes(void) { return vlc::decode::kNoAllocScratchBytes; }

extern "C" int vlc_decode_attn_noalloc(const void* q, int64_t q_seq_stride, int num_seqs, int num_heads,
                                       const void* k_cache, const void* v_cache, int64_t num_slots,
                                       int num_kv_heads, int head_dim, const int32_t* block_tables,
                                       int block_table_stride, int block_size, const int32_t* context_lens,
                                       int max_context_len, float softmax_scale, void* out,
                                       int64_t out_seq_stride, void* stream) {
  const int64_t need = vlc_decode_workspace_size(num_seqs, num_heads, num_kv_heads, max_context_len);
  if (need > vlc::decode::kNoAllocScratchBytes) return VLC_ERR_WORKSPACE;
  void* scratch = nullptr;
  if (need > 0) {
    const int rc = vlc::decode::noalloc_scratch(&scratch);
    if (rc != VLC_OK) return rc;
  }
  return vlc_decode_attn(q, q_seq_stride, num_seqs, num_heads, k_cache, v_cache, num_slots, num_kv_heads,
                         head_dim, block_tables, block_table_stride, block_size, context_lens, max_context_len,
                         softmax_scale, out, out_seq_stride, scratch,
                         need > 0 ? vlc::decode::kNoAllocScratchBytes : 0, stream);
}
