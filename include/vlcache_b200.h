/*
 * vlcache_b200 — C ABI of the B200-native (sm_100a) warm-prefill attention path
 * for Qwen2.5-VL in VLCache / nano-vllm.
 *
 * Every entry point takes plain device pointers, element strides, int32
 * metadata and a CUDA stream (passed as `void*`, NULL = legacy default stream),
 * and returns an int status (VLC_OK = 0).  No entry point allocates device
 * memory: callers own the KV cache, metadata, outputs and workspaces.
 * Argument errors are reported before any launch; data-dependent errors found
 * on the device (e.g. an out-of-range slot) are recorded in a device error
 * word that vlc_get_device_error() reads.
 *
 * Layout conventions (all bf16 unless stated):
 *   q        [num_tokens, num_heads, head_dim]      token stride given, head stride = head_dim
 *   key/value[num_tokens, num_kv_heads, head_dim]   token stride given (views of the QKV split)
 *   k_cache/v_cache per layer [num_slots, num_kv_heads, head_dim] contiguous,
 *            num_slots = num_blocks * block_size  (nano-vllm: [num_blocks, 256, Hk, D])
 *   block_tables [num_seqs, block_table_stride] int32, padded with -1
 *   slot_mapping [num_tokens] int32, -1 = skip
 */
#ifndef VLCACHE_B200_H
#define VLCACHE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes (host side) ---- */
#define VLC_OK 0
#define VLC_ERR_NULL 1        /* required pointer is NULL */
#define VLC_ERR_SHAPE 2       /* unsupported or inconsistent sizes */
#define VLC_ERR_STRIDE 3      /* stride/contiguity requirement violated */
#define VLC_ERR_ALIGN 4       /* pointer/stride not 16-byte aligned */
#define VLC_ERR_UNSUPPORTED 5 /* e.g. head_dim != 128 */
#define VLC_ERR_WORKSPACE 6   /* workspace missing or too small */
#define VLC_ERR_CUDA 7        /* a CUDA runtime/driver call failed */
#define VLC_ERR_PLAN 8        /* plan buffer malformed or too small */
#define VLC_ERR_METADATA 9    /* cu_seqlens / lengths inconsistent */

/* ---- device error codes (recorded by kernels, read by vlc_get_device_error) ---- */
#define VLC_DEV_ERR_SLOT_RANGE 101   /* slot >= num_slots or < -1 */
#define VLC_DEV_ERR_BLOCK_RANGE 102  /* block table entry out of range where a key is needed */
#define VLC_DEV_ERR_POSITION 103     /* rotary position outside the cos/sin cache */
#define VLC_DEV_ERR_LENGTH 104       /* a device length exceeds the host-side bound the grid was sized for */
#define VLC_DEV_ERR_TIMEOUT 110      /* an mbarrier wait hit its bound (base; +role id) */

/* Library version (major*10000 + minor*100 + patch). */
int vlc_version(void);

/* Human-readable text for a status code. */
const char* vlc_status_string(int status);

/* Synchronises the current device and returns its device error word (0 = none).
 * reset != 0 clears the word afterwards. */
int vlc_get_device_error(int reset);

/* Number of SMs of the current device (used by the planners). */
int vlc_num_sms(void);

/* Self-test of the bounded waits every kernel uses (no fault, no hang): one warp
 * waits on a shared-memory barrier that is completed (arrive != 0) or never
 * completed (arrive == 0).  In the second case the wait gives up after
 * limit_cycles (1 .. about 4e9) and records VLC_DEV_ERR_TIMEOUT + VLC_SELFTEST_ROLE
 * in the device error word; the kernel returns and the context stays usable. */
#define VLC_SELFTEST_ROLE 31
int vlc_selftest_bounded_wait(long long limit_cycles, int arrive, void* stream);

/* --------------------------------------------------------------------------
 * KV scatter.
 * Replaces nanovllm/layers/attention.py:10-40 (store_kvcache_kernel + store_kvcache):
 *   k_cache.view(-1, D)[slot_mapping[i]] = key[i];  v_cache likewise;  slot -1 skipped.
 * key/value rows are row_elems = num_kv_heads*head_dim contiguous bf16 elements;
 * key_stride/value_stride are token strides in elements.  Bit-exact copy.
 * ------------------------------------------------------------------------ */
int vlc_store_kvcache(const void* key, int64_t key_stride, const void* value, int64_t value_stride,
                      void* k_cache, void* v_cache, const int32_t* slot_mapping, int num_tokens,
                      int row_elems, int64_t num_slots, void* stream);

/* --------------------------------------------------------------------------
 * Rotary embedding fused with the KV scatter.
 * Replaces RotaryEmbedding.forward (nanovllm/layers/rotary_embedding.py:37-48,
 * rotate-half apply_rotary_emb :6-14) followed by store_kvcache (attention.py:10-40):
 *   q_out[i] = rope(q[i], positions[i])        (q_out may be q: in place)
 *   slot_mapping != NULL: rope(key[i]) and value[i] to k_cache / v_cache row
 *                         slot_mapping[i] (-1 skipped; rows of num_kv_heads*head_dim)
 *   slot_mapping == NULL: rope(key[i]) to k_out[i] (value, caches unused)
 * positions: int64 [num_tokens]; cos_sin_cache: fp32 [max_position, head_dim]
 * (first half cos, second half sin, as the reference's buffer); head_dim ==
 * rotary_dim == 128.  Strides are token strides in elements.  fp32 math with each
 * product and sum rounded separately, bf16 round-to-nearest-even output.
 * ------------------------------------------------------------------------ */
int vlc_rope_store_kvcache(const int64_t* positions, const void* q, int64_t q_stride, void* q_out,
                           int64_t q_out_stride, const void* key, int64_t key_stride, const void* value,
                           int64_t value_stride, const float* cos_sin_cache, int64_t max_position,
                           int rotary_dim, void* k_cache, void* v_cache, const int32_t* slot_mapping,
                           int64_t num_slots, void* k_out, int64_t k_out_stride, int num_tokens,
                           int num_heads, int num_kv_heads, int head_dim, void* stream);

/* --------------------------------------------------------------------------
 * M-RoPE position shift of reused vision K (new capability; replaces the
 * verbatim row copy of nanovllm/engine/model_runner.py:170-180 copy_image_kv,
 * driven by nanovllm/engine/llm_engine.py:58-89).
 * For each of num_layers layers (layer l at k_cache + l*layer_stride elements)
 * and each row i: K row at src_slots[i] is rotated by the per-section position
 * delta (delta_thw[0..2] for the t/h/w sections of mrope_section[0..2] pairs)
 * and written to dst_slots[i] (dst_slots == NULL: in place).  When v_cache is
 * non-NULL and dst_slots is non-NULL, the V row is copied verbatim too.
 * RoPE convention: rotate-half pairs (j, j + head_dim/2), inv_freq[j] =
 * theta^(-2j/head_dim) (HF transformers modeling_qwen2_5_vl.py:627-665).
 * Math in fp32 with a host-built cos/sin table; bf16 storage.
 * src/dst rows must be disjoint sets (or dst == src in place).
 * ------------------------------------------------------------------------ */
int vlc_mrope_shift(void* k_cache, void* v_cache, int64_t layer_stride, int num_layers,
                    int64_t num_slots, int num_kv_heads, int head_dim, const int32_t* src_slots,
                    const int32_t* dst_slots, int num_rows, const int32_t* delta_thw,
                    const int32_t* mrope_section, float rope_theta, void* stream);

/* --------------------------------------------------------------------------
 * Warm-prefill attention plan (host-only, no CUDA calls).
 * Replaces the work decomposition flash-attn derives inside
 * flash_attn_varlen_func (called at nanovllm/layers/attention.py:64-70).
 * Inputs are HOST copies of cu_seqlens_q / cu_seqlens_k ([num_seqs+1]).
 * Query row i of sequence b has logical position
 *   k_len_b - q_len_b + i   (causal, bottom-right aligned, as flash-attn).
 * Writes an int32 plan into plan_out (capacity plan_capacity ints) and returns
 * VLC_OK; *plan_len receives the number of ints used.  num_sms = 0 queries the
 * current device (falls back to 148 without a device).
 * ------------------------------------------------------------------------ */
int vlc_prefill_plan(const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_k, int num_seqs,
                     int num_heads, int num_kv_heads, int head_dim, int num_sms,
                     int32_t* plan_out, int64_t plan_capacity, int64_t* plan_len);

/* Upper bound (ints) of the plan for these sequences. */
int64_t vlc_prefill_plan_capacity(const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_k,
                                  int num_seqs, int num_heads, int num_kv_heads, int num_sms);

/* The same plan for the general varlen attention: causal != 0 is vlc_prefill_plan;
 * causal == 0 lets every query row of a sequence see all k_len keys of it, as
 * flash_attn_varlen_func(..., causal=False) in the vision tower's window and full
 * attention (nanovllm/models/qwen2_5_vl.py:202-211).  head_dim: 64 < d <= 128,
 * a multiple of 16 (Qwen2.5-VL's vision heads: 80).  vlc_prefill_plan(...) equals
 * vlc_attention_plan(..., causal = 1, ...). */
int vlc_attention_plan(const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_k, int num_seqs, int num_heads,
                       int num_kv_heads, int head_dim, int causal, int num_sms, int32_t* plan_out,
                       int64_t plan_capacity, int64_t* plan_len);
int64_t vlc_attention_plan_capacity(const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_k, int num_seqs,
                                    int num_heads, int num_kv_heads, int causal, int num_sms);

/* Unit kind of the prefill plans built from now on (process-wide): 1 = pairs of query
 * tiles sharing each K/V block on one SM; 2 = quads of tiles on CTA pairs (clusters of 2,
 * tcgen05.mma.cta_group::2; each SM loads half of every K/V block); 0 = the default (1).
 * Packed plans always use pairs.  A plan records its kind; vlc_prefill_attn follows it. */
int vlc_prefill_set_kernel(int mode);

/* Workspace bytes vlc_prefill_attn needs for a given (host) plan. */
int64_t vlc_prefill_workspace_size(const int32_t* plan_host);

/* --------------------------------------------------------------------------
 * Sparse-query paged prefill attention (tcgen05 / TMEM / TMA, sm_100a).
 * Replaces flash_attn_varlen_func(q, k, v, cu_seqlens_q, cu_seqlens_k,
 * max_seqlen_q, max_seqlen_k, softmax_scale, causal=True, block_table=...)
 * at nanovllm/layers/attention.py:64-70, both of its branches:
 *   paged      (block_tables != NULL): k/v are one layer's caches, key j of
 *              sequence b lives at row block_tables[b][j / block_size] *
 *              block_size + j % block_size (block_size a multiple of 128);
 *   contiguous (block_tables == NULL): key j of sequence b is row
 *              cu_seqlens_k[b] + j of k/v (the in-flight K/V of a cold prefill).
 *   o[i, h, :] = softmax(scale * q[i,h,:] . K[j, h/G, :]^T, j <= pos(i)) V
 * with GQA group G = num_heads / num_kv_heads.  k_row_stride / v_row_stride
 * are the element strides between consecutive key rows (num_kv_heads*head_dim
 * for a cache); num_kv_rows is the number of rows addressable through k/v.
 * plan_dev is the plan from vlc_prefill_plan copied to device memory;
 * plan_host is the same plan on the host (only its header is read).
 * out: [total_q, num_heads, head_dim] bf16 with token stride out_token_stride.
 * head_dim: 64 < d <= 128, a multiple of 16, equal to the plan's (q/k/v tiles are
 * zero-padded to 128 columns on load; outputs are written for the d real ones).
 * The plan's causal flag selects the mask (vlc_attention_plan).
 * Launch order: the attention is a programmatic dependent launch of the kernel
 * enqueued just before it on `stream` (its setup overlaps that kernel's tail).
 * That kernel may write q, k and v; plan_dev and block_tables must have been
 * written by a copy or by an earlier kernel.
 * ------------------------------------------------------------------------ */
int vlc_prefill_attn(const void* q, int64_t q_token_stride, int total_q, int num_heads,
                     const void* k, const void* v, int64_t k_row_stride, int64_t v_row_stride,
                     int64_t num_kv_rows, int num_kv_heads, int head_dim,
                     const int32_t* block_tables, int block_table_stride, int block_size,
                     const int32_t* plan_dev, const int32_t* plan_host, float softmax_scale,
                     void* out, int64_t out_token_stride, void* workspace,
                     int64_t workspace_bytes, void* stream);

/* Same as vlc_prefill_attn, plus the step's in-flight K/V: k_new / v_new hold the
 * rows the projection produced for the queries ([num_new_rows >= total_q, num_kv_heads,
 * head_dim], row strides kn_row_stride / vn_row_stride; row i is the key / value of query
 * row i, before store_kvcache copies it into the cache).  A sequence whose q_len equals
 * its k_len attends over exactly its own rows (a warm request's first sub-sequence:
 * model_runner.py:237-242 builds Q = K = tokens [0, img_start + R)), so its keys are read
 * from these rows instead of the cache and its work does not wait for the kernel
 * launched just before; the other sequences' K/V loads do.  That kernel may only write
 * the paged cache (the KV scatter), and must be an ordinary stream-ordered launch: q,
 * k_new, v_new complete and out / workspace free when it starts. */
int vlc_prefill_attn_inflight(const void* q, int64_t q_token_stride, int total_q, int num_heads,
                              const void* k, const void* v, int64_t k_row_stride, int64_t v_row_stride,
                              int64_t num_kv_rows, int num_kv_heads, int head_dim,
                              const int32_t* block_tables, int block_table_stride, int block_size,
                              const int32_t* plan_dev, const int32_t* plan_host, float softmax_scale,
                              void* out, int64_t out_token_stride, void* workspace,
                              int64_t workspace_bytes, const void* k_new, const void* v_new,
                              int64_t kn_row_stride, int64_t vn_row_stride, int64_t num_new_rows,
                              void* stream);

/* --------------------------------------------------------------------------
 * Split-K paged flash-decode.
 * Replaces flash_attn_with_kvcache(q.unsqueeze(1), k_cache, v_cache,
 * cache_seqlens=context_lens, block_table=block_tables, softmax_scale, causal=True)
 * at nanovllm/layers/attention.py:71-74 (one query token per sequence).
 * q: [num_seqs, num_heads, head_dim] (token stride q_seq_stride); out likewise.
 * context_lens [num_seqs] int32 on device; max_context_len is a host-side upper
 * bound used only to size the grid (graph-capture safe: no host reads).  A
 * context length above the keys that grid covers is recorded as
 * VLC_DEV_ERR_LENGTH and only the covered keys are attended (no access outside
 * the workspace).
 * ------------------------------------------------------------------------ */
int vlc_decode_attn(const void* q, int64_t q_seq_stride, int num_seqs, int num_heads,
                    const void* k_cache, const void* v_cache, int64_t num_slots, int num_kv_heads,
                    int head_dim, const int32_t* block_tables, int block_table_stride,
                    int block_size, const int32_t* context_lens, int max_context_len,
                    float softmax_scale, void* out, int64_t out_seq_stride, void* workspace,
                    int64_t workspace_bytes, void* stream);

/* Workspace bytes vlc_decode_attn needs. */
int64_t vlc_decode_workspace_size(int num_seqs, int num_heads, int num_kv_heads,
                                  int max_context_len);

/* --------------------------------------------------------------------------
 * Decode that allocates nothing.  No counterpart in the reference: it exists for
 * callers that cannot allocate device memory (a runtime with a fixed memory budget,
 * a process that may not call cudaMalloc after start-up).  Same arguments and
 * result as vlc_decode_attn minus the workspace: the split partials go to a
 * library-owned device array of vlc_decode_noalloc_scratch_bytes() (8 MiB) that
 * every GPU loading the library holds until exit.  Requests needing more
 * (vlc_decode_workspace_size() larger than that) return VLC_ERR_WORKSPACE without
 * launching.  Calls on one device share the array: calls that overlap on the GPU
 * race.  The first call on each device looks up the array's device address; make
 * it before any stream capture.
 * ------------------------------------------------------------------------ */
int vlc_decode_attn_noalloc(const void* q, int64_t q_seq_stride, int num_seqs, int num_heads,
                            const void* k_cache, const void* v_cache, int64_t num_slots,
                            int num_kv_heads, int head_dim, const int32_t* block_tables,
                            int block_table_stride, int block_size, const int32_t* context_lens,
                            int max_context_len, float softmax_scale, void* out,
                            int64_t out_seq_stride, void* stream);

/* Size in bytes of the built-in scratch array used by vlc_decode_attn_noalloc. */
int64_t vlc_decode_noalloc_scratch_bytes(void);

/* --------------------------------------------------------------------------
 * Warm-prefill metadata on the device.  Replaces the O(tokens) host loops of
 * nanovllm/engine/model_runner.py:160-168 (_compute_slots), :182-192 (padded block
 * tables), :232-276 (warm branch of prepare_prefill: positions, slot_mapping) and
 * nanovllm/engine/llm_engine.py:75-89 (_do_image_kv_copy: old/new slots of the
 * reused image rows).  The host lists O(requests) descriptors (device int32):
 *   vseq_desc[num_vseqs][7]  = {q_begin, q_len, first position, block-table offset
 *                               into block_tables_flat, block-table length, first
 *                               slot_mapping row (-1: none), output block-table row
 *                               (-1: none)}; a warm request is two virtual sequences,
 *                               [0, img_start + R) and [img_end, seqlen);
 *   reuse_desc[num_reuse][8] = {output offset, rows, first new position, new table
 *                               offset, new table length, first old position, old
 *                               table offset, old table length}.
 * Outputs (device; positions / slot_mapping / block_tables may be NULL):
 *   positions[q] (int64), slot_mapping[q] (int32), block_tables[num_vseqs][width]
 *   (int32, -1 padded), src_slots / dst_slots[rows] (int32).
 * slot(p) = table[p / block_size] * block_size + p % block_size; a page index past
 * the table's length writes -1 and records VLC_DEV_ERR_BLOCK_RANGE.  One launch. */
int vlc_warm_metadata(const int32_t* vseq_desc, int num_vseqs, const int32_t* reuse_desc, int num_reuse,
                      const int32_t* block_tables_flat, int block_size, int64_t* positions,
                      int32_t* slot_mapping, int32_t* block_tables, int block_table_width,
                      int32_t* src_slots, int32_t* dst_slots, void* stream);

/* --------------------------------------------------------------------------
 * Linear layers of the recomputed rows (tcgen05 GEMM, sm_100a).  All take
 * x [m, k] bf16 (row stride ldx) and a weight [rows, k] bf16 (row stride ldw,
 * nn.Linear layout), compute in fp32 and write bf16.  k, strides and output
 * columns must be multiples of 8; pointers 16-byte aligned.
 *
 * Workspace (optional, all three): with workspace != NULL the K-block work may
 * be split evenly over one CTA per SM (stream-K), which keeps every SM busy when
 * the output has fewer 128 x 256 tiles than the GPU has SMs and each tile is
 * long (>= 64 K blocks: down_proj of the recomputed rows); the library uses the
 * split only there and otherwise leaves the workspace untouched.  Size: vlc_linear_workspace_size(kind,
 * m, n, k) bytes, 256-byte aligned, ZEROED before its first use; each launch
 * leaves it reusable (its tickets back at zero).  Launches sharing one
 * workspace must not overlap on the GPU.  After a recorded device error, zero
 * it again.  workspace == NULL: whole output tiles per CTA.
 * kind: 0 vlc_linear, 1 vlc_linear_silu_mul (n = intermediate), 2 vlc_qkv_*
 * (n = (num_heads + 2 num_kv_heads) * head_dim).
 *
 * vlc_linear: out[m, n] = x . weight^T (+ bias[n]).
 *   Replaces F.linear in RowParallelLinear / ColumnParallelLinear
 *   (nanovllm/layers/linear.py:73, :154; o_proj and down_proj of
 *   nanovllm/models/qwen3.py:86, :116).
 * ------------------------------------------------------------------------ */
int64_t vlc_linear_workspace_size(int kind, int m, int n, int k);

/* Which GEMM kernel the linear entry points use, process-wide: 0 automatic (default: a
 * cost model fitted on B200 picks per shape), 1 single-SM 128 x 256 tiles (with the
 * stream-K split where it pays), 2 CTA pairs (clusters of 2, tcgen05.mma.cta_group::2,
 * 256 x 256 tiles), 3 single-SM 128 x 128 tiles, 4 single-SM 128 x 224 tiles (vlc_linear
 * only; the fused epilogues use the automatic choice).  A tuning and test switch; results
 * agree within the GEMM tolerance. */
int vlc_linear_set_kernel(int mode);

int vlc_linear(const void* x, int64_t ldx, const void* weight, int64_t ldw, const void* bias, void* out,
               int64_t ldo, int m, int n, int k, void* workspace, int64_t workspace_bytes, void* stream);

/* vlc_linear_silu_mul: gate_up_weight is [2 * intermediate, k] (gate rows, then up
 * rows, MergedColumnParallelLinear's layout); out[m, intermediate] =
 * silu(g) * u with g, u the bf16-rounded gate / up outputs, evaluated in fp32.
 *   Replaces gate_up_proj + SiluAndMul (nanovllm/models/qwen3.py:112-114,
 *   nanovllm/layers/activation.py:8-14). */
int vlc_linear_silu_mul(const void* x, int64_t ldx, const void* gate_up_weight, int64_t ldw, void* out,
                        int64_t ldo, int m, int intermediate, int k, void* workspace, int64_t workspace_bytes,
                        void* stream);

/* vlc_qkv_rope_store_kvcache: the QKV projection of the recomputed rows with its
 * bias, the rotary embedding and the KV scatter in one kernel.  qkv_weight is
 * [(num_heads + 2 num_kv_heads) * head_dim, hidden] (q rows, k rows, v rows,
 * QKVParallelLinear's layout).  Row i: qkv = bf16(x[i] . W^T + bias); q and k
 * heads rotated at positions[i] as vlc_rope_store_kvcache does (cos_sin_cache
 * [max_position, 128] fp32); q to q_out[i] ([m, num_heads, 128], row stride
 * q_out_stride); k and v rows to k_cache / v_cache row slot_mapping[i] (-1:
 * not stored; rows of num_kv_heads * 128).  head_dim must be 128.
 *   Replaces qkv_proj -> rotary_emb -> store_kvcache
 *   (nanovllm/models/qwen3.py:75-84, rotary_embedding.py:37-48, attention.py:10-40).
 * Out-of-range slots / positions are recorded as VLC_DEV_ERR_SLOT_RANGE /
 * VLC_DEV_ERR_POSITION and the row's stores skipped.  Whole output tiles only:
 * the workspace arguments are accepted and left untouched. */
int vlc_qkv_rope_store_kvcache(const void* x, int64_t ldx, const void* qkv_weight, int64_t ldw,
                               const void* qkv_bias, const int64_t* positions, const float* cos_sin_cache,
                               int64_t max_position, void* q_out, int64_t q_out_stride, void* k_cache,
                               void* v_cache, const int32_t* slot_mapping, int64_t num_slots, int m, int hidden,
                               int num_heads, int num_kv_heads, int head_dim, void* workspace,
                               int64_t workspace_bytes, void* stream);

/* --------------------------------------------------------------------------
 * Content hash of encoder-cache inputs.  Replaces EncoderCacheManager.compute_hash
 * (nanovllm/engine/encoder_cache_manager.py:24-29: XXH64 of grid_thw bytes then
 * pixel bytes, on the host, called per image at nanovllm/engine/llm_engine.py:52)
 * with a tree of XXH64 whose leaves hash in parallel (same bytes -> same key):
 *   d1[i] = XXH64(data[1024 i, 1024 (i+1)), seed 1)      (last chunk shorter)
 *   d2[j] = XXH64(d1 as little-endian bytes [512 j, 512 (j+1)), seed 2)
 *   d3[k] = XXH64(d2 as little-endian bytes [1024 k, 1024 (k+1)), seed 3)
 *   digest = XXH64(little-endian uint64 words {header_len, header zero-padded to a
 *            multiple of 8 bytes, nbytes, n1 = #d1, d3...}, seed 4)
 * header: the caller's bytes (e.g. grid_thw as int64 x 3), at most 256.
 *
 * vlc_content_hash_device: data in device memory; digest (one uint64) written to
 *   device memory `digest` on `stream` (two launches); workspace of
 *   vlc_content_hash_workspace_size(nbytes) bytes, 16-byte aligned.
 * vlc_content_hash_host: data in host memory, level 1 split over num_threads
 *   threads (<= 0: all hardware threads); digest written to *digest.
 * vlc_xxh64: plain XXH64 of a host buffer (the tree's primitive). */
int64_t vlc_content_hash_workspace_size(int64_t nbytes);
int vlc_content_hash_device(const void* data, int64_t nbytes, const void* header, int header_bytes, void* workspace,
                            int64_t workspace_bytes, uint64_t* digest, void* stream);
int vlc_content_hash_host(const void* data, int64_t nbytes, const void* header, int header_bytes, int num_threads,
                          uint64_t* digest);
uint64_t vlc_xxh64(const void* data, int64_t nbytes, uint64_t seed);

#ifdef __cplusplus
}
#endif

#endif /* VLCACHE_B200_H */
