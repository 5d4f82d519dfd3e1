// Host-side helpers shared by the C-ABI translation units.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "vlcache_b200.h"

namespace vlc {

// Encode a bf16 tiled TMA descriptor.  dims/box are innermost-first; strides_bytes
// has rank-1 entries (stride of dims[1..rank-1]); swizzle_bytes is 0, 64 or 128.
// Returns a VLC status.
int encode_tmap_bf16(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                     const uint64_t* strides_bytes, const uint32_t* box, int swizzle_bytes);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline int launch_status() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? VLC_OK : VLC_ERR_CUDA;
}

}  // namespace vlc
