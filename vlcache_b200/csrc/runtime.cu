// Host-side runtime pieces of the C ABI: status strings, the device error word,
// SM count query and TMA tensor-map encoding through the driver entry point
// (so the library does not link libcuda directly).
#include <cstdio>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "runtime.h"

namespace vlc {
__device__ int g_device_error = 0;
}

extern "C" int vlc_version(void) { return 100; }

extern "C" const char* vlc_status_string(int status) {
  switch (status) {
    case VLC_OK: return "ok";
    case VLC_ERR_NULL: return "required pointer is NULL";
    case VLC_ERR_SHAPE: return "unsupported or inconsistent sizes";
    case VLC_ERR_STRIDE: return "stride/contiguity requirement violated";
    case VLC_ERR_ALIGN: return "pointer or stride not 16-byte aligned";
    case VLC_ERR_UNSUPPORTED: return "unsupported configuration";
    case VLC_ERR_WORKSPACE: return "workspace missing or too small";
    case VLC_ERR_CUDA: return "CUDA call failed";
    case VLC_ERR_PLAN: return "plan malformed or too small";
    case VLC_ERR_METADATA: return "sequence metadata inconsistent";
    default: return "unknown status";
  }
}

extern "C" int vlc_get_device_error(int reset) {
  if (cudaDeviceSynchronize() != cudaSuccess) return -1;
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, vlc::g_device_error, sizeof(int)) != cudaSuccess) return -1;
  if (reset && v != 0) {
    int z = 0;
    if (cudaMemcpyToSymbol(vlc::g_device_error, &z, sizeof(int)) != cudaSuccess) return -1;
  }
  return v;
}

// Self-test of the bounded mbarrier wait every kernel uses: one warp waits on a
// barrier that is (arrive != 0) or is not (arrive == 0) completed.  Without the
// arrival the wait gives up after limit_cycles and records
// VLC_DEV_ERR_TIMEOUT + VLC_SELFTEST_ROLE; the kernel then returns normally.
namespace vlc {
__global__ void bounded_wait_selftest_kernel(long long limit_cycles, int arrive) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncwarp();
  if (arrive && threadIdx.x == 0) mbar_arrive(&bar);
  mbar_wait_bounded(&bar, 0, VLC_DEV_ERR_TIMEOUT + VLC_SELFTEST_ROLE, limit_cycles);
}
}  // namespace vlc

extern "C" int vlc_selftest_bounded_wait(long long limit_cycles, int arrive, void* stream) {
  if (limit_cycles <= 0 || limit_cycles > VLC_WAIT_LIMIT_CYCLES) return VLC_ERR_SHAPE;
  vlc::bounded_wait_selftest_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(limit_cycles, arrive);
  return vlc::launch_status();
}

extern "C" int vlc_num_sms(void) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return 148;
  }
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    return 148;
  }
  return n;
}

namespace vlc {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, []() {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<EncodeTiledFn>(p);
    } else {
      cudaGetLastError();
    }
  });
  return fn;
}

int encode_tmap_bf16(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                     const uint64_t* strides_bytes, const uint32_t* box, int swizzle_bytes) {
  EncodeTiledFn fn = get_encode_fn();
  if (!fn) return VLC_ERR_CUDA;
  cuuint64_t d[5];
  cuuint64_t s[4];
  cuuint32_t b[5];
  cuuint32_t e[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
  }
  for (int i = 0; i < rank - 1; ++i) s[i] = strides_bytes[i];
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (cuuint32_t)rank, const_cast<void*>(base),
                  d, s, b, e, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle_bytes == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                  : swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                        : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? VLC_OK : VLC_ERR_CUDA;
}

}  // namespace vlc
