// Content hash of encoder-cache inputs (pixel tensors), on the GPU or on the host.
//
// The reference keys its encoder cache (and the reuse of an image's KV) by XXH64 over
// the image's grid_thw bytes followed by its pixel bytes, computed on the host after a
// device-to-host copy (nanovllm/engine/encoder_cache_manager.py:24-29, called per image
// at nanovllm/engine/llm_engine.py:52): about 198 MB for a 4K image.  One XXH64 stream
// is a sequential chain, so this library defines a tree of XXH64 (xxHash's published
// round, merge and avalanche steps, restated here) whose leaves hash in parallel:
//
//   level 1: d1[i] = XXH64(data[i*1024, (i+1)*1024), seed 1)        (last chunk shorter)
//   level 2: d2[j] = XXH64(le64(d1)[j*512, (j+1)*512), seed 2)       (64 digests a chunk)
//   level 3: d3[k] = XXH64(le64(d2)[k*1024, (k+1)*1024), seed 3)     (128 digests a chunk)
//   digest  = XXH64(le64 words: header_len, header zero-padded to 8 bytes, nbytes, n1,
//                   d3[0 .. n3), seed 4)
//
// (n1 = number of level-1 chunks, 0 for empty data; header = the caller's bytes, e.g.
// grid_thw, at most 256.)  The keys are used only inside one engine process, so any
// strong 64-bit content hash keeps the reference's behaviour: same bytes, same key.
// The GPU path is two launches: a block of 256 threads stages 64 chunks in shared memory
// with TMA loads, hashes each chunk with four threads (level 1) and then its 64 digests (its
// level-2 digest: a level-2 chunk is exactly one block's digests, so level 1 never goes
// to global memory); one block then hashes the level-2 digests (level 3) and the short
// final stream.  The host path splits level 1 over threads.  Both give the same digest for
// the same bytes.
#include <algorithm>
#include <cstring>
#include <thread>
#include <vector>

#include "common.cuh"
#include "runtime.h"

namespace vlc {
namespace chash {

constexpr int64_t kChunk = 1024;
constexpr int kMaxHeader = 256;
constexpr uint64_t P1 = 0x9E3779B185EBCA87ull;
constexpr uint64_t P2 = 0xC2B2AE3D27D4EB4Full;
constexpr uint64_t P3 = 0x165667B19E3779F9ull;
constexpr uint64_t P4 = 0x85EBCA77C2B2AE63ull;
constexpr uint64_t P5 = 0x27D4EB2F165667C5ull;

__host__ __device__ __forceinline__ uint64_t rotl64(uint64_t x, int r) { return (x << r) | (x >> (64 - r)); }
__host__ __device__ __forceinline__ uint64_t xround(uint64_t acc, uint64_t in) {
  acc += in * P2;
  acc = rotl64(acc, 31);
  return acc * P1;
}
__host__ __device__ __forceinline__ uint64_t xmerge(uint64_t acc, uint64_t v) {
  acc ^= xround(0, v);
  return acc * P1 + P4;
}
__host__ __device__ __forceinline__ uint64_t avalanche(uint64_t h) {
  h ^= h >> 33;
  h *= P2;
  h ^= h >> 29;
  h *= P3;
  h ^= h >> 32;
  return h;
}
__host__ __device__ __forceinline__ uint64_t rd64(const uint8_t* p) {
  uint64_t v;
  memcpy(&v, p, 8);
  return v;  // little-endian hosts and GPUs
}
__host__ __device__ __forceinline__ uint32_t rd32(const uint8_t* p) {
  uint32_t v;
  memcpy(&v, p, 4);
  return v;
}

// XXH64 tail and final mix: h already holds the stripe result (or seed + P5) plus len.
__host__ __device__ inline uint64_t xfinish(uint64_t h, const uint8_t* p, int64_t rem) {
  while (rem >= 8) {
    h ^= xround(0, rd64(p));
    h = rotl64(h, 27) * P1 + P4;
    p += 8;
    rem -= 8;
  }
  if (rem >= 4) {
    h ^= (uint64_t)rd32(p) * P1;
    h = rotl64(h, 23) * P2 + P3;
    p += 4;
    rem -= 4;
  }
  while (rem > 0) {
    h ^= (uint64_t)(*p) * P5;
    h = rotl64(h, 11) * P1;
    ++p;
    --rem;
  }
  return avalanche(h);
}

__host__ __device__ inline uint64_t xstripes_done(uint64_t v1, uint64_t v2, uint64_t v3, uint64_t v4) {
  uint64_t h = rotl64(v1, 1) + rotl64(v2, 7) + rotl64(v3, 12) + rotl64(v4, 18);
  h = xmerge(h, v1);
  h = xmerge(h, v2);
  h = xmerge(h, v3);
  return xmerge(h, v4);
}

// XXH64 of n 64-bit words (8n bytes, little-endian): the aligned final stream.
__host__ __device__ inline uint64_t xxh64_words(const uint64_t* w, int64_t n, uint64_t seed) {
  uint64_t h;
  int64_t i = 0;
  if (n >= 4) {
    uint64_t v1 = seed + P1 + P2, v2 = seed + P2, v3 = seed, v4 = seed - P1;
    for (; i + 4 <= n; i += 4) {
      v1 = xround(v1, w[i]);
      v2 = xround(v2, w[i + 1]);
      v3 = xround(v3, w[i + 2]);
      v4 = xround(v4, w[i + 3]);
    }
    h = xstripes_done(v1, v2, v3, v4);
  } else {
    h = seed + P5;
  }
  h += (uint64_t)(8 * n);
  for (; i < n; ++i) {
    h ^= xround(0, w[i]);
    h = rotl64(h, 27) * P1 + P4;
  }
  return avalanche(h);
}

// XXH64 of a contiguous buffer (host, or device memory read by one thread).
__host__ __device__ inline uint64_t xxh64(const uint8_t* p, int64_t len, uint64_t seed) {
  const uint8_t* const end = p + len;
  uint64_t h;
  if (len >= 32) {
    uint64_t v1 = seed + P1 + P2, v2 = seed + P2, v3 = seed, v4 = seed - P1;
    const uint8_t* const limit = end - 32;
    do {
      v1 = xround(v1, rd64(p));
      v2 = xround(v2, rd64(p + 8));
      v3 = xround(v3, rd64(p + 16));
      v4 = xround(v4, rd64(p + 24));
      p += 32;
    } while (p <= limit);
    h = xstripes_done(v1, v2, v3, v4);
  } else {
    h = seed + P5;
  }
  h += (uint64_t)len;
  return xfinish(h, p, end - p);
}

// One XXH64 of `len` bytes (at most one chunk) hashed by four consecutive threads of a warp,
// thread `ln` running accumulator lane ln over the 64-bit words 4 s + ln of the full 32-byte
// stripes (the four lanes of XXH64 are independent chains: split over four threads, each
// chain has its own warp slot to hide its multiply latency).  word(i) returns the i-th
// little-endian 64-bit word, byte(i) the i-th byte.  Every thread of the warp calls this
// (the lanes meet through shuffles); the digest is returned in lane 0 of each group of four.
__device__ __forceinline__ uint64_t lane_init(uint64_t seed, int ln) {
  return ln == 0 ? seed + P1 + P2 : ln == 1 ? seed + P2 : ln == 2 ? seed : seed - P1;
}

// The end of xxh64_4lanes: every thread of the warp passes its lane's accumulator v (after
// the len / 32 full stripes); lane 0 of each group of four merges the four, hashes the
// tail and returns the digest (the others return 0).
template <typename Word, typename Byte>
__device__ __forceinline__ uint64_t xxh64_4lanes_finish(uint64_t v, int64_t len, uint64_t seed, int ln, bool active,
                                                        Word word, Byte byte) {
  const unsigned full = 0xffffffffu;
  const uint64_t v2 = __shfl_down_sync(full, v, 1), v3 = __shfl_down_sync(full, v, 2),
                 v4 = __shfl_down_sync(full, v, 3);
  if (!active || ln != 0) return 0;
  const int64_t nstripes = len / 32;
  uint64_t h = (len >= 32 ? xstripes_done(v, v2, v3, v4) : seed + P5) + (uint64_t)len;
  // the tail (fewer than 32 bytes) and the final mix, as xfinish does
  int64_t i = nstripes * 32;
  for (; i + 8 <= len; i += 8) {
    h ^= xround(0, word(i / 8));
    h = rotl64(h, 27) * P1 + P4;
  }
  if (i + 4 <= len) {
    const uint32_t w4 = (uint32_t)byte(i) | ((uint32_t)byte(i + 1) << 8) | ((uint32_t)byte(i + 2) << 16) |
                        ((uint32_t)byte(i + 3) << 24);
    h ^= (uint64_t)w4 * P1;
    h = rotl64(h, 23) * P2 + P3;
    i += 4;
  }
  for (; i < len; ++i) {
    h ^= (uint64_t)byte(i) * P5;
    h = rotl64(h, 11) * P1;
  }
  return avalanche(h);
}

template <typename Word, typename Byte>
__device__ __forceinline__ uint64_t xxh64_4lanes(int64_t len, uint64_t seed, int ln, bool active, Word word,
                                                 Byte byte) {
  const int64_t nstripes = active ? len / 32 : 0;
  uint64_t v = lane_init(seed, ln);
#pragma unroll 8
  for (int64_t s = 0; s < nstripes; ++s) v = xround(v, word(4 * s + ln));
  return xxh64_4lanes_finish(v, len, seed, ln, active, word, byte);
}

// Levels 1 and 2 on the GPU: block b hashes chunks [64 b, 64 b + 64), four threads a chunk
// (xxh64_4lanes), and then their 64 digests, d2[b].  kStaged (16-byte aligned data): the
// block's full chunks come into shared memory by 8 TMA tensor loads over the chunks viewed
// as a 2-D tensor [chunks][1,024 bytes]: load b is the 128-byte column slab b of all 64
// chunks (8 KB, 128-byte swizzle: 16-byte unit u of chunk c at unit u ^ (c & 7)), so a
// warp's 8-byte reads (8 chunks x 4 lanes) hit every bank evenly; the shorter last chunk
// (past the tensor's rows, which the loads fill with zeros) is copied by the block's
// threads into a buffer of its own.  Unaligned data is read from global memory.  The wait
// is bounded (a timeout records a device error and the block returns, leaving its digest
// unwritten).
constexpr int kStageChunks = 64;              // level-1 chunks per block = digests per level-2 chunk
constexpr int kLevel1Threads = 4 * kStageChunks;
constexpr int kL3Group = 128;                 // level-2 digests per level-3 chunk
constexpr int kSlabBytes = kStageChunks * 128;  // one 128-byte column of every chunk: 8 KB
constexpr int kSlabs = kChunk / 128;
constexpr int kOffTail = kSlabs * kSlabBytes;   // the shorter last chunk
constexpr int kOffDig = kOffTail + kChunk;      // the block's level-1 digests
constexpr int kOffBar = kOffDig + kStageChunks * 8;
constexpr int kStageSmem = kOffBar + 64 + 1024;  // + alignment of the swizzled slabs to 1,024 bytes
constexpr int kPlainSmem = kStageChunks * 8 + 64;
template <bool kStaged>
__global__ void __launch_bounds__(kLevel1Threads, 3) hash_level12_kernel(const __grid_constant__ CUtensorMap tm,
                                                                         const uint8_t* __restrict__ data,
                                                                         int64_t nbytes,
                                                                         uint64_t* __restrict__ d2) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  uint8_t* sm = kStaged ? reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023))
                        : smem_raw;
  uint64_t* dig = reinterpret_cast<uint64_t*>(sm + (kStaged ? kOffDig : 0));
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + (kStaged ? kOffBar : kStageChunks * 8));
  const int64_t n1 = (nbytes + kChunk - 1) / kChunk, full = nbytes / kChunk;
  const int64_t c0 = (int64_t)blockIdx.x * kStageChunks;
  const int nb = (int)min((int64_t)kStageChunks, n1 - c0);                    // chunks of this block
  const int t = threadIdx.x, ci = t >> 2, ln = t & 3;
  int nfull = 0;
  if (kStaged) {
    nfull = (int)max((int64_t)0, min((int64_t)nb, full - c0));
    if (t == 0) {
      mbar_init(bar, 1);
      fence_mbar_init();
    }
    __syncthreads();
    if (t == 0 && nfull > 0) {
      mbar_expect_tx(bar, (uint32_t)(kSlabs * kSlabBytes));  // whole boxes (rows past the tensor: zeros)
      for (int sb = 0; sb < kSlabs; ++sb) tma_load_2d(sm + sb * kSlabBytes, &tm, bar, sb * 64, (int)c0);
    }
    if (nb > nfull && t < kChunk / 16) {
      // the shorter last chunk (only the last block has one): 16 bytes a thread, the bytes
      // past nbytes one at a time
      const int64_t off = (c0 + nfull) * kChunk;
      const int rem = (int)(nbytes - off), b0 = 16 * t;
      uint8_t* tail = sm + kOffTail;
      if (b0 + 16 <= rem)
        *reinterpret_cast<uint4*>(tail + b0) = *reinterpret_cast<const uint4*>(data + off + b0);
      else
        for (int bb = b0; bb < rem; ++bb) tail[bb] = data[off + bb];
    }
    // Warp 0 polls the loads' barrier (sleeping between polls, so that the hashing warps of
    // the SM's other blocks keep its issue slots); the other warps wait at the block barrier,
    // which also carries warp 0's observation of the loaded bytes to them.
    bool ok = true;
    if (t < 32 && nfull > 0) {
      const long long t0 = clock64();
      while (!mbar_try_wait(bar, 0)) {
        if (clock64() - t0 > VLC_WAIT_LIMIT_CYCLES) {
          if (t == 0) record_error(VLC_DEV_ERR_TIMEOUT + 50);
          ok = false;
          break;
        }
        __nanosleep(64);
      }
    }
    if (!__syncthreads_and(ok)) return;  // every thread leaves together (and the last chunk is in place)
  }
  const int64_t off = (c0 + ci) * kChunk;
  const int64_t len = ci < nb ? min(kChunk, nbytes - off) : 0;
  uint64_t h;
  if (kStaged) {
    // A full chunk in the slabs: lane ln's words 4 s + ln are bytes 32 s + 8 ln, i.e. slab
    // s / 4, 16-byte unit 2 (s % 4) + ln / 2 (swizzled by the chunk's row), half ln % 2: four
    // offsets per thread, one add per word.  The shorter last chunk: from its own buffer.
    const uint8_t* tail = sm + kOffTail;
    uint64_t v = lane_init(1, ln);
    if (ci < nfull) {
      const uint8_t* row = sm + ci * 128 + 8 * (ln & 1);
      const int sw = ci & 7;
      int offj[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) offj[j] = ((2 * j + (ln >> 1)) ^ sw) * 16;
#pragma unroll
      for (int g = 0; g < kSlabs; ++g)
#pragma unroll
        for (int j = 0; j < 4; ++j) v = xround(v, *reinterpret_cast<const uint64_t*>(row + g * kSlabBytes + offj[j]));
    } else if (ci < nb) {
      const uint64_t* tw = reinterpret_cast<const uint64_t*>(tail);
      for (int64_t s2 = 0; s2 < len / 32; ++s2) v = xround(v, tw[4 * s2 + ln]);
    }
    h = xxh64_4lanes_finish(
        v, len, 1, ln, ci < nb, [&](int64_t i) { return reinterpret_cast<const uint64_t*>(tail)[i]; },
        [&](int64_t i) { return tail[i]; });  // the tail bytes: only the shorter chunk has them
  } else {
    const uint8_t* src = data + off;
    h = xxh64_4lanes(
        len, 1, ln, ci < nb, [&](int64_t i) { return rd64(src + 8 * i); }, [&](int64_t i) { return src[i]; });
  }
  if (ln == 0 && ci < nb) dig[ci] = h;
  __syncthreads();
  if (t == 0) d2[blockIdx.x] = xxh64_words(dig, nb, 2);
}

struct Header {
  uint8_t bytes[kMaxHeader];
  int len;
};

// Level 3 and the digest, one block: the level-2 digests come into shared memory in
// windows of kFinalWindow words (coalesced, eight loads in flight per thread), four threads
// hash each level-3 chunk of the window (128 level-2 digests, fewer in the last) into the
// final word stream, also in shared memory, and thread 0 hashes that stream.
constexpr int kFinalThreads = 256;
constexpr int kFinalWindow = kFinalThreads / 4 * kL3Group;  // words: 64 KB, one level-3 chunk per 4 threads
constexpr int kFinalSmemMax = 200 * 1024;
__global__ void __launch_bounds__(kFinalThreads) hash_final_kernel(const uint64_t* __restrict__ d2, int64_t n2,
                                                                   int64_t n1, int64_t nbytes,
                                                                   const __grid_constant__ Header hdr, uint64_t* out) {
  extern __shared__ uint64_t smem_words[];  // [window][1 + header words + 2 + n3]
  uint64_t* win = smem_words;
  uint64_t* words = smem_words + kFinalWindow;
  const int hw = (hdr.len + 7) / 8;
  const int t = threadIdx.x, ck = t >> 2, ln = t & 3;
  for (int64_t w0 = 0; w0 < n2; w0 += kFinalWindow) {
    const int64_t cnt = min((int64_t)kFinalWindow, n2 - w0);
    __syncthreads();  // the previous window is hashed
    for (int64_t j0 = 0; j0 < cnt; j0 += 8 * kFinalThreads) {
      uint64_t v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int64_t j = j0 + u * kFinalThreads + t;
        v[u] = j < cnt ? d2[w0 + j] : 0;
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int64_t j = j0 + u * kFinalThreads + t;
        if (j < cnt) win[j] = v[u];
      }
    }
    __syncthreads();
    const int64_t k = (int64_t)ck;  // level-3 chunk of this window
    const int64_t nw = max((int64_t)0, min((int64_t)kL3Group, cnt - k * kL3Group));
    const uint64_t* cw = win + k * kL3Group;
    const uint64_t h = xxh64_4lanes(
        8 * nw, 3, ln, nw > 0, [&](int64_t i) { return cw[i]; },
        [&](int64_t i) { return (uint8_t)(cw[i >> 3] >> (8 * (i & 7))); });
    if (ln == 0 && nw > 0) words[3 + hw + w0 / kL3Group + k] = h;
  }
  if (t == 0) {
    words[0] = (uint64_t)hdr.len;
    for (int k = 0; k < hw; ++k) {
      uint64_t v = 0;
      for (int b = 0; b < 8 && 8 * k + b < hdr.len; ++b) v |= (uint64_t)hdr.bytes[8 * k + b] << (8 * b);
      words[1 + k] = v;
    }
    words[1 + hw] = (uint64_t)nbytes;
    words[2 + hw] = (uint64_t)n1;
  }
  __syncthreads();
  if (threadIdx.x == 0) *out = xxh64_words(words, 3 + hw + (n2 + kL3Group - 1) / kL3Group, 4);
}

inline int64_t level1_chunks(int64_t nbytes) { return (nbytes + kChunk - 1) / kChunk; }
inline int64_t level2_chunks(int64_t n1) { return (n1 + kStageChunks - 1) / kStageChunks; }
inline int64_t level3_chunks(int64_t n2) { return (n2 + kL3Group - 1) / kL3Group; }

// Host digest from the level-1 digests (the same steps as the device kernels).
uint64_t host_final(const std::vector<uint64_t>& d1, int64_t nbytes, const uint8_t* header, int header_len) {
  const int64_t n1 = (int64_t)d1.size();
  const int64_t n2 = level2_chunks(n1), n3 = level3_chunks(n2);
  std::vector<uint64_t> d2((size_t)n2);
  for (int64_t j = 0; j < n2; ++j)
    d2[(size_t)j] = xxh64_words(d1.data() + j * kStageChunks, std::min<int64_t>(kStageChunks, n1 - j * kStageChunks), 2);
  const int hw = (header_len + 7) / 8;
  std::vector<uint64_t> w((size_t)(3 + hw + n3), 0);
  w[0] = (uint64_t)header_len;
  for (int b = 0; b < header_len; ++b) w[1 + b / 8] |= (uint64_t)header[b] << (8 * (b % 8));
  w[1 + hw] = (uint64_t)nbytes;
  w[2 + hw] = (uint64_t)n1;
  for (int64_t k = 0; k < n3; ++k)
    w[(size_t)(3 + hw + k)] = xxh64_words(d2.data() + k * kL3Group, std::min<int64_t>(kL3Group, n2 - k * kL3Group), 3);
  return xxh64_words(w.data(), (int64_t)w.size(), 4);
}

}  // namespace chash
}  // namespace vlc

using namespace vlc;
using namespace vlc::chash;

extern "C" int64_t vlc_content_hash_workspace_size(int64_t nbytes) {
  if (nbytes < 0) return -1;
  return std::max<int64_t>(1, level2_chunks(level1_chunks(nbytes))) * 8;  // the level-2 digests
}

extern "C" int vlc_content_hash_device(const void* data, int64_t nbytes, const void* header, int header_bytes,
                                       void* workspace, int64_t workspace_bytes, uint64_t* digest, void* stream) {
  if (nbytes < 0 || header_bytes < 0) return VLC_ERR_SHAPE;
  if (header_bytes > kMaxHeader) return VLC_ERR_UNSUPPORTED;
  if ((nbytes > 0 && !data) || (header_bytes > 0 && !header) || !digest || !workspace) return VLC_ERR_NULL;
  if (workspace_bytes < vlc_content_hash_workspace_size(nbytes)) return VLC_ERR_WORKSPACE;
  if ((uintptr_t)workspace % 16 != 0 || (uintptr_t)digest % 8 != 0) return VLC_ERR_ALIGN;
  const int64_t n1 = level1_chunks(nbytes);
  const int64_t n2 = level2_chunks(n1);
  const int64_t final_smem = (kFinalWindow + 3 + (header_bytes + 7) / 8 + level3_chunks(n2)) * 8;
  if (final_smem > kFinalSmemMax || n2 > 0x7fffffff) return VLC_ERR_UNSUPPORTED;  // inputs above about 100 GB
  uint64_t* d2 = (uint64_t*)workspace;
  cudaStream_t st = (cudaStream_t)stream;
  if (n1 > 0) {
    const int64_t full = nbytes / kChunk;
    CUtensorMap tm;
    memset(&tm, 0, sizeof(tm));
    if (aligned16(data) && full > 0) {
      // the full chunks as a 2-D tensor [full][512 two-byte elements], boxes {64, 64}
      const uint64_t dims[2] = {(uint64_t)(kChunk / 2), (uint64_t)full};
      const uint64_t strides[1] = {(uint64_t)kChunk};
      const uint32_t box[2] = {64, (uint32_t)kStageChunks};
      if (encode_tmap_bf16(&tm, data, 2, dims, strides, box, 128) != VLC_OK) return VLC_ERR_CUDA;
      static std::atomic<uint64_t> staged_set{0};
      if (ensure_dynamic_smem((const void*)hash_level12_kernel<true>, kStageSmem, staged_set) != VLC_OK)
        return VLC_ERR_CUDA;
      hash_level12_kernel<true><<<(unsigned)n2, kLevel1Threads, kStageSmem, st>>>(tm, (const uint8_t*)data, nbytes,
                                                                                  d2);
    } else {
      hash_level12_kernel<false><<<(unsigned)n2, kLevel1Threads, kPlainSmem, st>>>(tm, (const uint8_t*)data, nbytes,
                                                                                   d2);
    }
    const int rc = launch_status();
    if (rc != VLC_OK) return rc;
  }
  Header h;
  memset(&h, 0, sizeof(h));
  if (header_bytes) memcpy(h.bytes, header, (size_t)header_bytes);
  h.len = header_bytes;
  static std::atomic<uint64_t> smem_set{0};
  if (ensure_dynamic_smem((const void*)hash_final_kernel, kFinalSmemMax, smem_set) != VLC_OK) return VLC_ERR_CUDA;
  hash_final_kernel<<<1, kFinalThreads, (size_t)final_smem, st>>>(d2, n2, n1, nbytes, h, digest);
  return launch_status();
}

extern "C" int vlc_content_hash_host(const void* data, int64_t nbytes, const void* header, int header_bytes,
                                     int num_threads, uint64_t* digest) {
  if (nbytes < 0 || header_bytes < 0) return VLC_ERR_SHAPE;
  if (header_bytes > kMaxHeader) return VLC_ERR_UNSUPPORTED;
  if ((nbytes > 0 && !data) || (header_bytes > 0 && !header) || !digest) return VLC_ERR_NULL;
  const int64_t n1 = level1_chunks(nbytes);
  std::vector<uint64_t> d1((size_t)n1);
  const uint8_t* p = (const uint8_t*)data;
  if (num_threads <= 0) num_threads = (int)std::max(1u, std::thread::hardware_concurrency());
  const int nt = (int)std::max<int64_t>(1, std::min<int64_t>(num_threads, n1 / 256 + 1));
  auto work = [&](int t) {
    for (int64_t i = n1 * t / nt; i < n1 * (t + 1) / nt; ++i)
      d1[(size_t)i] = xxh64(p + i * kChunk, std::min(kChunk, nbytes - i * kChunk), 1);
  };
  std::vector<std::thread> pool;
  for (int t = 1; t < nt; ++t) pool.emplace_back(work, t);
  work(0);
  for (auto& th : pool) th.join();
  *digest = host_final(d1, nbytes, (const uint8_t*)header, header_bytes);
  return VLC_OK;
}

// Plain XXH64 of a host buffer (the primitive the tree is built from; exposed so tests
// can check it against the xxHash package's digests).
extern "C" uint64_t vlc_xxh64(const void* data, int64_t nbytes, uint64_t seed) {
  if (nbytes < 0 || (nbytes > 0 && !data)) return 0;
  return xxh64((const uint8_t*)data, nbytes, seed);
}
