// Host-side helpers shared by the C-ABI translation units.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

#include "vlcache_b200.h"

namespace vlc {

// Encode a bf16 tiled TMA descriptor.  dims/box are innermost-first; strides_bytes
// has rank-1 entries (stride of dims[1..rank-1]); swizzle_bytes is 0, 64 or 128.
// Returns a VLC status.
int encode_tmap_bf16(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                     const uint64_t* strides_bytes, const uint32_t* box, int swizzle_bytes);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Raise a kernel's dynamic shared-memory limit on the current device, once per device
// (the attribute is per device; `done` holds one bit per device ordinal < 64).
inline int ensure_dynamic_smem(const void* func, int bytes, std::atomic<uint64_t>& done) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return VLC_ERR_CUDA;
  const uint64_t bit = dev < 64 ? (uint64_t)1 << dev : 0;
  if (bit && (done.load(std::memory_order_acquire) & bit)) return VLC_OK;
  if (cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess) {
    (void)cudaGetLastError();
    return VLC_ERR_CUDA;
  }
  done.fetch_or(bit, std::memory_order_acq_rel);
  return VLC_OK;
}

inline int launch_status() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? VLC_OK : VLC_ERR_CUDA;
}

}  // namespace vlc
