/* C ABI of libmsattn.so: MiniServe's per-step attention path on B200 (sm_100a).
 *
 * Every entry point is extern "C", takes plain pointers and sizes, returns 0 on success or a
 * positive MS_ERR_* code (ms_last_error() then describes it), never allocates device memory and
 * never synchronises the stream it is given (except ms_device_status, whose job is to).
 * Device pointers are raw CUDA addresses; `stream` is a cudaStream_t passed as void*.
 *
 * Geometry: head_dim 128, 16-token KV blocks, two query heads per KV head (Qwen3-0.6B:
 * 16 query heads, 8 KV heads).  Activations are bf16; the cos/sin tables are fp32.
 *
 * KV pool layout (one layer): [num_blocks][num_kv_heads][2: K,V][2: d/64][16 tokens][64] bf16, so
 * K and V of one (block, head) are 8 KiB contiguous.  The layer's "k_cache" pointer is the start
 * of that region and "v_cache" must be k_cache + 4096 bytes; slot = block * 16 + token.
 */
#ifndef MSATTN_H_
#define MSATTN_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MS_ABI_VERSION 1

#if defined(__GNUC__)
#define MS_API __attribute__((visibility("default")))
#else
#define MS_API
#endif

enum {
  MS_OK = 0,
  MS_ERR_ARG = 1,     /* a size, shape, stride or pointer argument is invalid */
  MS_ERR_LAYOUT = 2,  /* the KV pool views are not in the layout described above */
  MS_ERR_PLAN = 3,    /* the batch description cannot be planned (table too short, ...) */
  MS_ERR_CUDA = 4,    /* a CUDA runtime/driver call failed */
  MS_ERR_CAPACITY = 5 /* an output buffer given to the planner is too small */
};

/* Device status bits reported by ms_device_status. */
#define MS_DEV_BAD_SLOT 1u     /* slot_mapping entry outside the pool: that row was not written */
#define MS_DEV_BAD_BLOCK 2u    /* block table entry outside the pool: read as zeros */
#define MS_DEV_TIMEOUT 4u      /* a bounded pipeline wait gave up */
#define MS_DEV_BAD_POSITION 8u /* RoPE position outside the cos/sin table: row 0 used */

/* Library version (MS_ABI_VERSION * 100 + minor). */
MS_API int ms_version(void);

/* Description of the last error raised on the calling thread ("" if none). */
MS_API const char* ms_last_error(void);

/* Synchronises `stream`, then reads (and if `clear` != 0 resets) the current device's status
 * word into *flags.  Call it at points where the caller already synchronises. */
MS_API int ms_device_status(void* stream, uint32_t* flags, int clear);

/* ---- Per-step plan (host only) ---------------------------------------------------------------
 * Replaces build_attention_metadata (src/miniserve/attention/backends.py:80-142) and the int64
 * index/mask tensors it builds.  The batch is described the way SeqChunk does
 * (backends.py:36-47): for sequence i, its new tokens are rows flat_start[i] .. +num_new[i] of
 * the flat batch and num_cached[i] tokens are already in the pool; its block table is
 * tables[table_offsets[i] .. table_offsets[i+1]).  The plan is a packed int32 buffer, uploaded
 * once per step and read by every layer.
 */
typedef struct MsPlanInfo {
  int32_t num_seqs;
  int32_t num_tokens;
  int32_t n_decode_items;  /* work items of <= 8 query tokens (decode / speculative verify) */
  int32_t n_tile_items;    /* work items of 9..64-token chunks (mma.sync tile kernel) */
  int32_t n_combine;       /* split tiles (and cascade rows) whose partials must be merged */
  int32_t off_seqs;        /* int32 offsets of each section inside the packed buffer */
  int32_t off_tables;
  int32_t off_decode;
  int32_t off_tile;
  int32_t off_combine;
  int32_t total_ints;      /* length of the packed buffer actually written */
  int32_t pages_per_split; /* split size chosen (pages of 16 tokens) */
  int64_t part_rows;       /* rows of fp32 partial output held in the workspace */
  int64_t workspace_bytes_per_kv_head; /* scratch per KV head the attention call needs:
                                          ms_paged_attention wants this x num_kv_heads bytes
                                          (0 when no tile is split) */
  int64_t total_pages;     /* sum over work tiles of KV pages read (per KV head) */
  int32_t n_tc_items;      /* work items of 64 query tokens of chunks longer than 64 tokens,
                              run on the tcgen05 tensor-core kernel */
  int32_t off_tc;
  int32_t n_cascade;       /* shared-prefix groups: runs of >= 16 consecutive decode / verify
                              rows whose tables share >= 16 cached blocks attend that prefix
                              once (tensor-core items over the group's tokens) and merge it with
                              their own pages; sequence records num_seqs .. num_seqs+n_cascade-1
                              describe the groups */
  int32_t decode_pages;    /* pages (per KV head) the decode / verify items read, in total */
  int32_t combine_tokens_max; /* most query tokens of one combine record (sizes its grid) */
  int32_t reserved[3];
} MsPlanInfo;

/* Upper bound on the packed buffer length (int32 elements) for a batch of this size. */
MS_API int64_t ms_plan_capacity(int32_t num_seqs, int32_t num_tokens, int64_t total_table_entries);

/* Builds the plan.  block_size must be 16.  num_sms sizes the split-KV work; pages_per_split
 * forces a split size (0 = automatic).  Replaces backends.py:80-142 (grouping, padding, masks). */
MS_API int ms_plan_build(int32_t num_seqs, const int32_t* flat_start, const int32_t* num_new,
                  const int32_t* num_cached, const int64_t* table_offsets, const int32_t* tables,
                  int32_t num_tokens, int32_t block_size, int32_t num_sms,
                  int32_t pages_per_split, int32_t* out, int64_t out_capacity, MsPlanInfo* info);

/* Runner step preparation (host only).  Replaces the attention inputs of ModelRunner.prepare
 * (src/miniserve/runner/model_runner.py:162-205), which walks every scheduled token in Python:
 * sequence i schedules num_new[i] tokens after num_cached[i] computed ones, with block table
 * tables[table_offsets[i] .. table_offsets[i+1]).  Writes flat_start[i] (its first row in the
 * flat batch), and for its tokens, in flat-batch order, positions[t] = num_cached[i] + k and
 * slot_mapping[t] = table[p / block_size] * block_size + p % block_size (the reference's slot
 * formula, model_runner.py:188), and *num_tokens.  The outputs feed ms_plan_build and
 * ms_qk_norm_rope_scatter directly.  Errors: MS_ERR_ARG (bad sizes), MS_ERR_PLAN (a table
 * shorter than its context), MS_ERR_CAPACITY (more tokens than capacity_tokens). */
MS_API int ms_prepare_step(int32_t num_seqs, const int32_t* num_new, const int32_t* num_cached,
                    const int64_t* table_offsets, const int32_t* tables, int32_t block_size,
                    int32_t* flat_start, int64_t* positions, int64_t* slot_mapping,
                    int64_t capacity_tokens, int32_t* num_tokens);

/* ---- Kernel A: q/k RMSNorm + RoPE + K/V scatter ----------------------------------------------
 * Replaces, for one layer, qwen3.py:94-98 (split, q_norm, k_norm, apply_rope) and the K/V
 * index_copy_ at backends.py:159-160.  qkv is the fused projection output [T, (H+2*KVH)*128];
 * q_out receives the normalised, rotated queries [T, H, 128]; the normalised, rotated keys and
 * the raw values go to slot_mapping[t] of the pool.  cos/sin are either per-token rows [T, 128]
 * (positions == NULL, what Qwen3ForCausalLM.forward gathers at qwen3.py:149) or the whole
 * [max_positions, 128] table indexed by positions[t]. */
MS_API int ms_qk_norm_rope_scatter(const void* qkv, int64_t qkv_row_stride, int32_t num_tokens,
                            int32_t num_heads, int32_t num_kv_heads, const void* q_weight,
                            const void* k_weight, float eps, const float* cos, const float* sin,
                            int64_t cs_row_stride, const int64_t* positions,
                            int64_t max_positions, const int64_t* slot_mapping, void* q_out,
                            int64_t q_out_row_stride, void* k_cache, void* v_cache,
                            int32_t num_blocks, void* stream);

/* ---- Kernel E: qkv projection with kernel A as its epilogue -----------------------------------
 * Replaces, for one layer, `self.qkv_proj(x)` and the split/q_norm/k_norm/apply_rope after it
 * (qwen3.py:94-98, the projection built at qwen3.py:75-77 as nn.Linear(hidden, (H+2*KVH)*128,
 * bias=False)) plus the K/V index_copy_ at backends.py:159-160, in one tensor-core launch: the
 * projection output never reaches memory.  x is [T, hidden] bf16 (hidden a multiple of 64), w_qkv
 * the projection weight [(H+2*KVH)*128, hidden] bf16 as nn.Linear stores it; every other argument
 * means what it means for ms_qk_norm_rope_scatter, with x, w_qkv, q_out and the two norm weights
 * 16-byte aligned (row strides multiples of 8 elements).  The result equals
 * ms_qk_norm_rope_scatter applied to bf16(x @ w_qkv^T) except where the GEMM's fp32 accumulation
 * order moves a projection output by one bf16 ulp. */
MS_API int ms_qkv_proj_norm_rope_scatter(const void* x, int64_t x_row_stride, int32_t num_tokens,
                                  int32_t hidden, const void* w_qkv, int64_t w_row_stride,
                                  int32_t num_heads, int32_t num_kv_heads, const void* q_weight,
                                  const void* k_weight, float eps, const float* cos,
                                  const float* sin, int64_t cs_row_stride,
                                  const int64_t* positions, int64_t max_positions,
                                  const int64_t* slot_mapping, void* q_out,
                                  int64_t q_out_row_stride, void* k_cache, void* v_cache,
                                  int32_t num_blocks, void* stream);

/* Scatter only (backends.py:159-160): k, v [T, KVH, 128] with the given row strides. */
MS_API int ms_kv_scatter(const void* k, int64_t k_row_stride, const void* v, int64_t v_row_stride,
                  int32_t num_tokens, int32_t num_kv_heads, const int64_t* slot_mapping,
                  void* k_cache, void* v_cache, int32_t num_blocks, void* stream);

/* ---- Kernels B + C: attention through the pool ------------------------------------------------
 * Replaces backends.py:161-197 (gather, GQA fold, masked SDPA, output scatter).  q, out:
 * [T, H, 128] bf16 with the given row strides; plan_dev is the uploaded packed plan and `plan`
 * its host-side info; workspace holds plan->workspace_bytes_per_kv_head * num_kv_heads bytes of
 * scratch (may be NULL when that is 0).  Only rows covered by the plan's sequences are written. */
MS_API int ms_paged_attention(const void* q, int64_t q_row_stride, void* out, int64_t out_row_stride,
                       int32_t num_heads, int32_t num_kv_heads, const void* k_cache,
                       const void* v_cache, int32_t num_blocks, const int32_t* plan_dev,
                       const MsPlanInfo* plan, void* workspace, int64_t workspace_bytes,
                       float scale, void* stream);

/* ---- Attention for callers that cannot allocate device memory -------------------------------
 * No counterpart in the reference (MiniServe allocates everything through PyTorch).
 *
 * Same work and arguments as ms_paged_attention, minus the workspace: the split-KV partials go
 * to a fixed scratch array compiled into the library, MS_NOALLOC_SCRATCH_BYTES on every GPU that
 * loads it, held until the process exits.  It is meant for hosts that never let a plugin call
 * cudaMalloc (an engine that gives all GPU memory to its own arena, a custom-op interface with
 * no allocator hook, a loop that cannot take cudaMalloc's implicit synchronisation).  The call
 * itself allocates nothing.
 *
 *  - A plan needing more than MS_NOALLOC_SCRATCH_BYTES of partials
 *    (plan->workspace_bytes_per_kv_head * num_kv_heads) is rejected with MS_ERR_CAPACITY; plan
 *    with a larger pages_per_split or use ms_paged_attention.
 *  - Every call looks up the current context's address of the array (with that device current),
 *    so a context recreated after cudaDeviceReset gets the new address.  The first call in a
 *    process may load the library's device code; make that first call before any stream capture.
 *  - All calls share the array: calls that overlap on the GPU race on it; calls ordered on one
 *    stream are safe.  No state carries over between calls. */
#define MS_NOALLOC_SCRATCH_BYTES (16u * 1024u * 1024u)

MS_API int ms_paged_attention_noalloc(const void* q, int64_t q_row_stride, void* out,
                                      int64_t out_row_stride, int32_t num_heads,
                                      int32_t num_kv_heads, const void* k_cache,
                                      const void* v_cache, int32_t num_blocks,
                                      const int32_t* plan_dev, const MsPlanInfo* plan,
                                      float scale, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MSATTN_H_ */
