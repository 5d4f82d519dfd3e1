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
//   level 2: d2[j] = XXH64(le64(d1)[j*1024, (j+1)*1024), seed 2)
//   digest  = XXH64(le64 words: header_len, header zero-padded to 8 bytes, nbytes, n1,
//                   d2[0 .. n2), seed 3)
//
// (n1 = number of level-1 chunks, 0 for empty data; header = the caller's bytes, e.g.
// grid_thw, at most 256.)  The keys are used only inside one engine process, so any
// strong 64-bit content hash keeps the reference's behaviour: same bytes, same key.
// The GPU path: level 1 stages each block's chunks in shared memory with bulk copies and
// hashes one chunk per thread; level 2 and the digest follow.  The host path splits level 1
// over threads.  Both give the same digest for the same bytes.
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

// Level 1 on the GPU: thread i hashes chunk i.  Full chunks stream 16-byte loads (the
// four of two 32-byte stripes in flight before their rounds); the last, shorter chunk
// (and every chunk of a buffer that is not 16-byte aligned) takes the byte-wise path.
__global__ void __launch_bounds__(256) hash_chunks_kernel(const uint8_t* __restrict__ data, int64_t nbytes,
                                                          uint64_t* __restrict__ out, int64_t nchunks, uint64_t seed,
                                                          int aligned) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nchunks) return;
  const int64_t off = i * kChunk;
  const int64_t len = min(kChunk, nbytes - off);
  const uint8_t* p = data + off;
  if (len < kChunk || !aligned) {
    out[i] = xxh64(p, len, seed);
    return;
  }
  uint64_t v1 = seed + P1 + P2, v2 = seed + P2, v3 = seed, v4 = seed - P1;
  const uint4* q = reinterpret_cast<const uint4*>(p);
#pragma unroll 4
  for (int s = 0; s < kChunk / 64; ++s) {
    const uint4 a = __ldg(q + 4 * s), b = __ldg(q + 4 * s + 1), c = __ldg(q + 4 * s + 2), d = __ldg(q + 4 * s + 3);
    v1 = xround(v1, ((uint64_t)a.y << 32) | a.x);
    v2 = xround(v2, ((uint64_t)a.w << 32) | a.z);
    v3 = xround(v3, ((uint64_t)b.y << 32) | b.x);
    v4 = xround(v4, ((uint64_t)b.w << 32) | b.z);
    v1 = xround(v1, ((uint64_t)c.y << 32) | c.x);
    v2 = xround(v2, ((uint64_t)c.w << 32) | c.z);
    v3 = xround(v3, ((uint64_t)d.y << 32) | d.x);
    v4 = xround(v4, ((uint64_t)d.w << 32) | d.z);
  }
  const uint64_t h = xstripes_done(v1, v2, v3, v4) + (uint64_t)kChunk;
  out[i] = avalanche(h);  // a full chunk leaves no tail
}

// Level 1, staged: a block's 64 full chunks come into shared memory with one 1 KB bulk copy
// each (the copy engine streams whole chunks; a lane-per-chunk global read would touch 32
// lines per warp access), rows padded to 1,040 bytes so that the 8 lanes of a 16-byte
// shared-memory access hit distinct banks; then thread i hashes chunk i from shared memory.
// The waits are bounded (a timeout records a device error and the block returns).
constexpr int kStageChunks = 64;
constexpr int kStageRow = kChunk + 16;
constexpr int kStageSmem = kStageChunks * kStageRow + 64;
__global__ void __launch_bounds__(kStageChunks) hash_chunks_staged_kernel(const uint8_t* __restrict__ data,
                                                                          uint64_t* __restrict__ out,
                                                                          int64_t full_chunks, uint64_t seed) {
  extern __shared__ __align__(128) uint8_t stage[];
  uint64_t* bar = reinterpret_cast<uint64_t*>(stage + kStageChunks * kStageRow);
  const int64_t c0 = (int64_t)blockIdx.x * kStageChunks;
  const int n = (int)min((int64_t)kStageChunks, full_chunks - c0);
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    mbar_expect_tx(bar, (uint32_t)(n * kChunk));
    for (int i = 0; i < n; ++i) bulk_load_1d(stage + i * kStageRow, data + (c0 + i) * kChunk, kChunk, bar);
  }
  if (!mbar_wait_bounded(bar, 0, VLC_DEV_ERR_TIMEOUT + 50, VLC_WAIT_LIMIT_CYCLES)) return;
  const int i = threadIdx.x;
  if (i >= n) return;
  uint64_t v1 = seed + P1 + P2, v2 = seed + P2, v3 = seed, v4 = seed - P1;
  const ulonglong2* q = reinterpret_cast<const ulonglong2*>(stage + i * kStageRow);
#pragma unroll 8
  for (int s = 0; s < kChunk / 32; ++s) {
    const ulonglong2 a = q[2 * s], b = q[2 * s + 1];
    v1 = xround(v1, a.x);
    v2 = xround(v2, a.y);
    v3 = xround(v3, b.x);
    v4 = xround(v4, b.y);
  }
  out[c0 + i] = avalanche(xstripes_done(v1, v2, v3, v4) + (uint64_t)kChunk);
}

struct Header {
  uint8_t bytes[kMaxHeader];
  int len;
};

// Level 2: thread j hashes level-2 chunk j, i.e. 128 level-1 digests (fewer in the
// last), as 64-bit words with 16-byte loads: XXH64 of 8k bytes is xxh64_words of k words.
__global__ void __launch_bounds__(256) hash_level2_kernel(const uint64_t* __restrict__ d1, int64_t n1,
                                                          uint64_t* __restrict__ d2, int64_t n2) {
  const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= n2) return;
  const int64_t w0 = j * (kChunk / 8);
  const int64_t cnt = min((int64_t)(kChunk / 8), n1 - w0);
  if (cnt < kChunk / 8) {
    d2[j] = xxh64_words(d1 + w0, cnt, 2);
    return;
  }
  uint64_t v1 = 2 + P1 + P2, v2 = 2 + P2, v3 = 2, v4 = 2 - P1;
  const ulonglong2* q = reinterpret_cast<const ulonglong2*>(d1 + w0);
#pragma unroll 4
  for (int s = 0; s < kChunk / 32; ++s) {
    const ulonglong2 a = q[2 * s], b = q[2 * s + 1];
    v1 = xround(v1, a.x);
    v2 = xround(v2, a.y);
    v3 = xround(v3, b.x);
    v4 = xround(v4, b.y);
  }
  d2[j] = avalanche(xstripes_done(v1, v2, v3, v4) + (uint64_t)kChunk);
}

// The digest, one block: the final word stream is gathered in shared memory (the level-2
// digests copied by all threads), then thread 0 hashes it.
constexpr int kFinalThreads = 256;
constexpr int kFinalSmemMax = 200 * 1024;
__global__ void __launch_bounds__(kFinalThreads) hash_final_kernel(const uint64_t* __restrict__ d2, int64_t n2,
                                                                   int64_t n1, int64_t nbytes,
                                                                   const __grid_constant__ Header hdr, uint64_t* out) {
  extern __shared__ uint64_t words[];  // [1 + header words + 2 + n2]
  const int hw = (hdr.len + 7) / 8;
  for (int64_t j = threadIdx.x; j < n2; j += blockDim.x) words[3 + hw + j] = d2[j];
  if (threadIdx.x == 0) {
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
  if (threadIdx.x == 0) *out = xxh64_words(words, 3 + hw + n2, 3);
}

inline int64_t level1_chunks(int64_t nbytes) { return (nbytes + kChunk - 1) / kChunk; }
inline int64_t level2_chunks(int64_t n1) { return (n1 * 8 + kChunk - 1) / kChunk; }

// Host digest from the level-1 digests (the same steps as hash_final_kernel).
uint64_t host_final(const std::vector<uint64_t>& d1, int64_t nbytes, const uint8_t* header, int header_len) {
  const int64_t n1 = (int64_t)d1.size();
  const int64_t bytes1 = n1 * 8;
  const int64_t n2 = level2_chunks(n1);
  const int hw = (header_len + 7) / 8;
  std::vector<uint64_t> w((size_t)(3 + hw + n2), 0);
  w[0] = (uint64_t)header_len;
  for (int b = 0; b < header_len; ++b) w[1 + b / 8] |= (uint64_t)header[b] << (8 * (b % 8));
  w[1 + hw] = (uint64_t)nbytes;
  w[2 + hw] = (uint64_t)n1;
  const uint8_t* b1 = reinterpret_cast<const uint8_t*>(d1.data());
  for (int64_t j = 0; j < n2; ++j)
    w[(size_t)(3 + hw + j)] = xxh64(b1 + j * kChunk, std::min(kChunk, bytes1 - j * kChunk), 2);
  return xxh64_words(w.data(), (int64_t)w.size(), 3);
}

}  // namespace chash
}  // namespace vlc

using namespace vlc;
using namespace vlc::chash;

extern "C" int64_t vlc_content_hash_workspace_size(int64_t nbytes) {
  if (nbytes < 0) return -1;
  const int64_t n1 = level1_chunks(nbytes);
  return std::max<int64_t>(1, n1 + level2_chunks(n1)) * 8;  // the level-1 and level-2 digests
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
  const int64_t final_smem = (3 + (header_bytes + 7) / 8 + n2) * 8;
  if (final_smem > kFinalSmemMax) return VLC_ERR_UNSUPPORTED;  // inputs above about 3 TB
  uint64_t* d1 = (uint64_t*)workspace;
  uint64_t* d2 = d1 + n1;  // 16-byte aligned chunks of d1 (1,024 bytes each)
  cudaStream_t st = (cudaStream_t)stream;
  if (n1 > 0) {
    const int64_t blocks = (n1 + 255) / 256;
    if (blocks > 0x7fffffff) return VLC_ERR_SHAPE;
    int rc;
    const int64_t full = nbytes / kChunk;
    if (aligned16(data) && full > 0) {
      // full chunks staged through shared memory; the shorter last chunk on its own
      static std::atomic<uint64_t> staged_set{0};
      if (ensure_dynamic_smem((const void*)hash_chunks_staged_kernel, kStageSmem, staged_set) != VLC_OK)
        return VLC_ERR_CUDA;
      hash_chunks_staged_kernel<<<(unsigned)((full + kStageChunks - 1) / kStageChunks), kStageChunks, kStageSmem,
                                  st>>>((const uint8_t*)data, d1, full, 1);
      rc = launch_status();
      if (rc != VLC_OK) return rc;
      if (full < n1) {
        hash_chunks_kernel<<<1, 32, 0, st>>>((const uint8_t*)data + full * kChunk, nbytes - full * kChunk,
                                             d1 + full, 1, 1, 0);
        rc = launch_status();
        if (rc != VLC_OK) return rc;
      }
    } else {
      hash_chunks_kernel<<<(unsigned)blocks, 256, 0, st>>>((const uint8_t*)data, nbytes, d1, n1, 1,
                                                           aligned16(data) ? 1 : 0);
      rc = launch_status();
      if (rc != VLC_OK) return rc;
    }
    hash_level2_kernel<<<(unsigned)((n2 + 255) / 256), 256, 0, st>>>(d1, n1, d2, n2);
    rc = launch_status();
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
