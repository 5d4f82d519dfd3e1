// Warm-prefill metadata on the device.
//
// The host side of nano-vllm's warm prefill builds, per step, O(tokens) integer
// arrays in Python loops: positions and slot_mapping of every query row
// (nanovllm/engine/model_runner.py:160-168 `_compute_slots`, :232-276 the warm
// branch of `prepare_prefill`), the padded block tables of the virtual
// sub-sequences (:182-192), and the old/new slots of every reused image row
// (nanovllm/engine/llm_engine.py:75-89 `_do_image_kv_copy`).  Here the host only
// lists O(requests) descriptors and one launch writes all of those arrays.
//
// Virtual sequence v (a cold request, or one of the two sub-sequences of a warm
// request: [0, img_start + R) and [img_end, seqlen)):
//   positions[q_begin + i] = pos0 + i,
//   slot_mapping[slot_begin + i] = bt[p / bs] * bs + p % bs   with p = pos0 + i,
//   block_tables[bt_row] = the request's block table, padded with -1 to the row width
// (requests without a block table have no slot rows and no block-table row, as in
// the reference).
// Reuse item w (a warm request): rows p in [new_pos0, new_pos0 + count) of the new
// request and the same rows p - new_pos0 + old_pos0 of the cached image entry:
//   dst_slots[out0 + i] = new_bt[p / bs] * bs + p % bs,
//   src_slots[out0 + i] = old_bt[p' / bs] * bs + p' % bs.
// A page index past a block table's length is recorded as device error 102 and its
// slot written as -1 (the scatter skips -1).
#include "common.cuh"
#include "runtime.h"

namespace vlc {
namespace meta {

// virtual-sequence descriptor fields (int32 x 7)
enum : int {
  kVQBegin = 0,    // first row of positions
  kVQLen = 1,
  kVPos0 = 2,      // position of the first row
  kVBtOff = 3,     // block table: offset in the flat table array, length
  kVBtLen = 4,
  kVSlotBegin = 5, // first row of slot_mapping (-1: the request has no block table)
  kVBtRow = 6,     // row of the output block tables (-1: none)
  kVInts = 7
};
// reuse descriptor fields (int32 x 8)
enum : int {
  kROut0 = 0,
  kRCount = 1,
  kRNewPos0 = 2,
  kRNewBtOff = 3,
  kRNewBtLen = 4,
  kROldPos0 = 5,
  kROldBtOff = 6,
  kROldBtLen = 7,
  kRInts = 8
};

__device__ __forceinline__ int32_t slot_of(const int32_t* __restrict__ bt, int bt_len, int p, int bs) {
  const int page = p / bs;
  if (page >= bt_len) {
    record_error(VLC_DEV_ERR_BLOCK_RANGE);
    return -1;
  }
  return __ldg(bt + page) * bs + (p - page * bs);
}

// Blocks [0, num_vseqs): one virtual sequence each; blocks [num_vseqs, +num_reuse):
// one reuse item each.  Threads stride over the rows.
__global__ void __launch_bounds__(256) warm_metadata_kernel(
    const int32_t* __restrict__ vdesc, int num_vseqs, const int32_t* __restrict__ rdesc, int num_reuse,
    const int32_t* __restrict__ bt_flat, int block_size, int64_t* __restrict__ positions,
    int32_t* __restrict__ slot_mapping, int32_t* __restrict__ block_tables, int bt_width,
    int32_t* __restrict__ src_slots, int32_t* __restrict__ dst_slots) {
  const int b = blockIdx.x;
  if (b < num_vseqs) {
    const int32_t* d = vdesc + (int64_t)b * kVInts;
    const int q0 = __ldg(d + kVQBegin), n = __ldg(d + kVQLen), pos0 = __ldg(d + kVPos0);
    const int bt_off = __ldg(d + kVBtOff), bt_len = __ldg(d + kVBtLen);
    const int s0 = __ldg(d + kVSlotBegin), row = __ldg(d + kVBtRow);
    const int32_t* bt = bt_flat + bt_off;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const int p = pos0 + i;
      if (positions) positions[q0 + i] = p;
      if (slot_mapping && s0 >= 0) slot_mapping[s0 + i] = slot_of(bt, bt_len, p, block_size);
    }
    if (block_tables && row >= 0) {
      for (int i = threadIdx.x; i < bt_width; i += blockDim.x)
        block_tables[(int64_t)row * bt_width + i] = i < bt_len ? __ldg(bt + i) : -1;
    }
  } else if (b < num_vseqs + num_reuse) {
    const int32_t* d = rdesc + (int64_t)(b - num_vseqs) * kRInts;
    const int out0 = __ldg(d + kROut0), n = __ldg(d + kRCount);
    const int np0 = __ldg(d + kRNewPos0), op0 = __ldg(d + kROldPos0);
    const int32_t* nbt = bt_flat + __ldg(d + kRNewBtOff);
    const int32_t* obt = bt_flat + __ldg(d + kROldBtOff);
    const int nlen = __ldg(d + kRNewBtLen), olen = __ldg(d + kROldBtLen);
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      dst_slots[out0 + i] = slot_of(nbt, nlen, np0 + i, block_size);
      src_slots[out0 + i] = slot_of(obt, olen, op0 + i, block_size);
    }
  }
}

}  // namespace meta
}  // namespace vlc

using namespace vlc;
using namespace vlc::meta;

extern "C" int vlc_warm_metadata(const int32_t* vseq_desc, int num_vseqs, const int32_t* reuse_desc,
                                 int num_reuse, const int32_t* block_tables_flat, int block_size,
                                 int64_t* positions, int32_t* slot_mapping, int32_t* block_tables,
                                 int block_table_width, int32_t* src_slots, int32_t* dst_slots, void* stream) {
  if (num_vseqs < 0 || num_reuse < 0 || block_table_width < 0) return VLC_ERR_SHAPE;
  if (num_vseqs + num_reuse == 0) return VLC_OK;
  if (block_size <= 0) return VLC_ERR_SHAPE;
  if (num_vseqs > 0 && !vseq_desc) return VLC_ERR_NULL;
  if (num_reuse > 0 && (!reuse_desc || !src_slots || !dst_slots)) return VLC_ERR_NULL;
  if (!block_tables_flat) return VLC_ERR_NULL;
  if (block_tables && block_table_width == 0) return VLC_ERR_SHAPE;
  warm_metadata_kernel<<<num_vseqs + num_reuse, 256, 0, (cudaStream_t)stream>>>(
      vseq_desc, num_vseqs, reuse_desc, num_reuse, block_tables_flat, block_size, positions, slot_mapping,
      block_tables, block_table_width, src_slots, dst_slots);
  return launch_status();
}
