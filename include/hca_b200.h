/*
 * hca_b200.h -- C ABI of libhca_b200.so, the B200 (sm_100a) kernels of the
 * ERNIE 5.5 Heavily Compressed Attention (HCA) layer path.
 *
 * Conventions (all entry points):
 *   - device pointers and plain integer sizes/strides only; strides are in
 *     elements of the pointed-to type unless the name ends in "_bytes";
 *   - every call is asynchronous on `stream` (a cudaStream_t, NULL = legacy
 *     default stream) and allocates no memory;
 *   - return HCA_OK (0) or a negative HCA_E_* status; nothing is thrown
 *     across the ABI.  hca_status_string() names a status;
 *   - slot / index value -1 means "skip" exactly as in the reference.
 *
 * Cached KV row layout ("fp8_ds_mla", generalised to head_dim D = N + R with
 * N % 64 == 0): a page of P rows holds P data rows of N float8_e4m3 bytes
 * followed by R bf16 values (N + 2R bytes), then P scale rows of N/64 UE8M0
 * bytes plus one zero pad byte.  Page stride is given in bytes.  At D = 512
 * this is the reference's 584-byte row.
 *
 * Citations: E/ = src/vllm_ernie/models/ernie5_5/ of baidu/vLLM-ERNIE;
 * V/ = the vllm package the plugin inherits (vLLM 0.22.0 sources here).
 */
#ifndef HCA_B200_H_
#define HCA_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HCA_OK 0
#define HCA_E_INVALID (-1)     /* bad pointer, size, stride or alignment */
#define HCA_E_UNSUPPORTED (-2) /* shape not instantiated in this build */
#define HCA_E_CUDA (-3)        /* CUDA launch error */
#define HCA_E_WORKSPACE (-4)   /* workspace too small */
#define HCA_E_TOO_LARGE (-5)   /* needs more than HCA_NOALLOC_WORKSPACE_BYTES of split-K scratch */

/* Size of the static split-K scratch of hca_sparse_decode_noalloc (16 MiB). */
#define HCA_NOALLOC_WORKSPACE_BYTES (16ll * 1024 * 1024)

const char* hca_status_string(int status);

/* The CUDA error string behind this thread's last HCA_E_CUDA status (a
 * library diagnostic with no counterpart in the reference). */
const char* hca_last_cuda_error(void);

/* Library ABI version (major * 100 + minor). */
int hca_version(void);
/* Device error word of the current device (synchronous read): non-zero if a
 * kernel gave up on a bounded wait (bit 0 loader, 1 dequant, 2 MMA, 3
 * softmax of hca_sparse_decode; bit 4 the streamed many-token path of
 * hca_qnorm_rope_kv_insert, bit 5 that of hca_vha_inv_rope_fp8_quant).
 * clear != 0 resets it to zero. */
int hca_device_error(int32_t* value, int32_t clear);

/* ---------------------------------------------------------------------- */
/* Metadata builders (integer, bit-exact with the reference)               */
/* ---------------------------------------------------------------------- */

/* token -> request index; replaces the host repeat_interleave of
 * V/v1/attention/backends/mla/sparse_swa.py:286-294 and
 * V/models/deepseek_v4/compressor.py:107-112. */
int hca_token_to_req(int32_t* out, const int32_t* query_start_loc, int32_t num_reqs,
                     int32_t num_tokens, void* stream);

/* Per-token slot bt[p / bs] * bs + p % bs (SWA and compressor-state caches),
 * the model runner's slot mapping for these caches. */
int hca_slot_mapping(int64_t* out, const int32_t* query_start_loc, const int32_t* seq_lens,
                     const int32_t* block_table, int64_t bt_stride, int32_t num_reqs,
                     int32_t block_size, void* stream);

/* Replaces get_compressed_slot_mapping
 * (V/v1/attention/backends/mla/compressor_utils.py:8-86).  Writes -1 to all
 * out_len entries, then the slot of the compressed entry each completing
 * token writes. */
int hca_compressed_slot_mapping(int64_t* out, int32_t out_len, const int32_t* query_start_loc,
                                const int32_t* seq_lens, const int32_t* block_table,
                                int64_t bt_stride, int32_t num_reqs, int32_t block_size,
                                int32_t compress_ratio, void* stream);

/* Replaces _compute_swa_indices_and_lens_kernel and the lens zeroing of
 * DeepseekSparseSWAMetadataBuilder.build
 * (V/v1/attention/backends/mla/sparse_swa.py:296-314,449-503). */
int hca_swa_indices_and_lens(int32_t* indices, int64_t indices_stride, int32_t* lens,
                             int32_t lens_len, int32_t num_decode_tokens, int32_t window,
                             const int32_t* query_start_loc, const int32_t* seq_lens,
                             const int32_t* token_to_req, const uint8_t* is_valid_token,
                             const int32_t* block_table, int64_t bt_stride, int32_t block_size,
                             void* stream);

/* Replaces build_c128a_topk_metadata
 * (V/v1/attention/backends/mla/flashmla_sparse.py:1032-1149). */
int hca_c128a_topk_metadata(int32_t* global_decode, int64_t global_decode_stride,
                            int32_t* decode_lens, int32_t* prefill_local,
                            int64_t prefill_local_stride, const int64_t* positions,
                            int32_t num_tokens, int32_t compress_ratio,
                            int32_t max_compressed_tokens, int32_t num_decode_tokens,
                            const int32_t* token_to_req, const int32_t* block_table,
                            int64_t bt_stride, int32_t block_size, const int64_t* slot_mapping,
                            void* stream);

/* Replaces _compute_prefill_metadata_kernel
 * (V/v1/attention/backends/mla/sparse_swa.py:422-446). */
int hca_prefill_gather_lens(int32_t* gather_lens, const int32_t* seq_lens,
                            const int32_t* query_start_loc, int32_t num_prefills,
                            int32_t num_decodes, int32_t window, void* stream);

/* Replaces combine_topk_swa_indices
 * (V/models/deepseek_v4/common/ops/cache_utils.py:476-594).  Rows of
 * `combined` (width `combined_width`) are written in full, -1 padded. */
int hca_combine_topk_swa_indices(int32_t* combined, int64_t combined_stride,
                                 int32_t combined_width, int32_t* combined_lens,
                                 const int32_t* topk_indices, int64_t topk_stride,
                                 const int32_t* query_start_loc, const int32_t* seq_lens,
                                 const int32_t* gather_lens, int32_t num_reqs,
                                 int32_t num_tokens, int32_t window, int32_t compress_ratio,
                                 int32_t top_k, int32_t M, int32_t N, void* stream);

/* ---------------------------------------------------------------------- */
/* Norms, KV-cache write, compressor                                       */
/* ---------------------------------------------------------------------- */

/* Replaces fused_q_kv_rmsnorm
 * (V/models/deepseek_v4/common/ops/fused_qk_rmsnorm.py:57-96); bf16 in/out,
 * fp32 math. */
int hca_qk_rmsnorm(void* q_out, int64_t q_out_stride, const void* q_in, int64_t q_in_stride,
                   const void* q_weight, int32_t q_size, void* kv_out, int64_t kv_out_stride,
                   const void* kv_in, int64_t kv_in_stride, const void* kv_weight,
                   int32_t kv_size, int32_t num_tokens, float eps, void* stream);

/* Replaces torch.ops._C.fused_deepseek_v4_qnorm_rope_kv_rope_quant_insert
 * (V/models/deepseek_v4/attention.py:497-542): q [T, H, D] bf16 ->
 * weightless per-head RMSNorm + GPT-J RoPE of the last R dims -> q_out
 * [T, padded_heads, D] bf16 (extra heads zero); kv [T, D] bf16 -> RoPE ->
 * UE8M0 FP8 NoPE / bf16 RoPE row written to the SWA cache at slot_mapping
 * (-1 skipped).  cos_sin: fp32 [max_pos, R] (cos | sin). */
int hca_qnorm_rope_kv_insert(void* q_out, int64_t q_out_stride_tok, int64_t q_out_stride_head,
                             int32_t padded_heads, const void* q, int64_t q_stride_tok,
                             int64_t q_stride_head, int32_t num_heads, const void* kv,
                             int64_t kv_stride, uint8_t* swa_cache, int32_t page_size,
                             int64_t page_stride_bytes, const int64_t* slot_mapping,
                             const int64_t* positions, const float* cos_sin,
                             int64_t cos_sin_stride, int32_t num_tokens, int32_t head_dim,
                             int32_t rope_dim, float eps, void* stream);

/* Replaces quantize_and_insert_k_cache
 * (V/models/deepseek_v4/common/ops/cache_utils.py:23-194): k [T, D] bf16
 * (already rotated) quantised and written at slot_mapping. */
int hca_quantize_insert_k(uint8_t* cache, int32_t page_size, int64_t page_stride_bytes,
                          const void* k, int64_t k_stride, const int64_t* slot_mapping,
                          int32_t num_tokens, int32_t head_dim, int32_t rope_dim, void* stream);

/* Replaces dequantize_and_gather_k_cache
 * (V/models/deepseek_v4/common/ops/cache_utils.py:197-380): out[req,
 * offset + i] = row of position seq_len - gather_len + i (bf16).
 * gather_lens may be NULL (gather whole sequence). */
int hca_dequantize_gather_k(void* out, int64_t out_stride_req, int64_t out_stride_tok,
                            const uint8_t* cache, int32_t page_size, int64_t page_stride_bytes,
                            const int32_t* seq_lens, const int32_t* gather_lens,
                            const int32_t* block_table, int64_t bt_stride, int32_t num_reqs,
                            int32_t offset, int32_t head_dim, int32_t rope_dim, void* stream);

/* Replaces save_partial_states
 * (V/models/deepseek_v4/common/ops/save_partial_states.py:9-101):
 * state[slot] = [kv, score + ape[pos % ratio]] (fp32). */
int hca_save_partial_states(float* state, int64_t state_stride_block, int64_t state_stride_tok,
                            const float* kv, int64_t kv_stride, const float* score,
                            int64_t score_stride, const float* ape, int64_t ape_stride,
                            const int64_t* positions, const int64_t* slot_mapping,
                            int32_t num_tokens, int32_t block_size, int32_t head_size,
                            int32_t state_width, int32_t compress_ratio, void* stream);

/* Replaces compress_norm_rope_store_{triton,cutedsl}
 * (V/models/deepseek_v4/common/ops/fused_compress_quant_cache.py:34-296;
 * dispatch V/models/deepseek_v4/compressor.py:338-380) for ratio 128: at each
 * token with (p + 1) % ratio == 0, softmax-pool the last `ratio` states,
 * RMSNorm, quantise, RoPE at the block start and store into the compressed
 * cache at kv_slot_mapping. */
int hca_compress_norm_rope_store(const float* state, int64_t state_stride_block,
                                 int64_t state_stride_tok, int32_t state_width,
                                 const int32_t* token_to_req, const int64_t* positions,
                                 const int64_t* state_slot_mapping, const int32_t* block_table,
                                 int64_t bt_stride, int32_t block_size, const float* norm_weight,
                                 float eps, const float* cos_sin, int64_t cos_sin_stride,
                                 uint8_t* kv_cache, const int64_t* kv_slot_mapping,
                                 int32_t kv_page_size, int64_t kv_page_stride_bytes,
                                 int32_t num_tokens, int32_t head_dim, int32_t rope_dim,
                                 int32_t compress_ratio, void* stream);

/* One launch for a decode step's per-layer cache work: the three calls above
 * (hca_qnorm_rope_kv_insert, hca_save_partial_states,
 * hca_compress_norm_rope_store, in that order) fused, with the same output
 * bytes.  It has no single reference counterpart: it replaces the decode-time
 * sequence of the `_C` fused q-norm / RoPE / KV insert
 * (V/models/deepseek_v4/attention.py:497-542), save_partial_states
 * (V/models/deepseek_v4/common/ops/save_partial_states.py:48-101) and the
 * block compressor (.../fused_compress_quant_cache.py:112-296).  The batch
 * must be decode-shaped: tokens [query_start_loc[r], query_start_loc[r + 1])
 * of request r, query_start_loc[num_reqs] == num_tokens; a request's blocks
 * are pooled by the CTA that saved its tokens' states.  state_kv / state_score
 * are the two halves of the compressor's fp32 kv_score. */
int hca_decode_prep(void* q_out, int64_t q_out_stride_tok, int64_t q_out_stride_head, int32_t padded_heads,
                    const void* q, int64_t q_stride_tok, int64_t q_stride_head, int32_t num_heads,
                    const void* kv, int64_t kv_stride, uint8_t* swa_cache, int32_t swa_page_size,
                    int64_t swa_page_stride_bytes, const int64_t* swa_slot_mapping, const int64_t* positions,
                    const float* cos_sin, int64_t cos_sin_stride, const float* state_kv, int64_t state_kv_stride,
                    const float* state_score, int64_t state_score_stride, const float* ape, int64_t ape_stride,
                    float* state, int64_t state_stride_block, int64_t state_stride_tok, int32_t state_width,
                    int32_t state_block_size, const int64_t* state_slot_mapping, const int32_t* state_block_table,
                    int64_t state_bt_stride, const float* norm_weight, uint8_t* comp_cache,
                    const int64_t* comp_slot_mapping, int32_t comp_page_size, int64_t comp_page_stride_bytes,
                    const int32_t* query_start_loc, const int32_t* token_to_req, int32_t num_reqs,
                    int32_t num_tokens, int32_t head_dim, int32_t rope_dim, int32_t compress_ratio, float eps,
                    void* stream);

/* ---------------------------------------------------------------------- */
/* Sparse attention over [window || compressed] rows                        */
/* ---------------------------------------------------------------------- */

/* Workspace bytes hca_sparse_decode needs for these sizes (0 if
 * num_splits == 1): split-K partials (bf16 rows at head_dim 128, fp32 at
 * 512, each with an fp32 running max and sum), written by the attention
 * kernel and merged by a second launch on the same stream.  Calls that share one
 * workspace must be ordered on one stream. */
int64_t hca_sparse_decode_workspace_bytes(int32_t num_groups, int32_t max_group_tokens,
                                          int32_t num_heads, int32_t head_dim,
                                          int32_t num_splits);

/* Replaces flash_mla_with_kvcache with indices / extra_indices over the
 * fp8 SWA and compressed caches
 * (V/models/deepseek_v4/nvidia/flashmla.py:210-302;
 * V/third_party/flashmla/flash_mla_interface.py:54-92).
 * q [T, H, D] bf16 -> out [T, H, D] bf16; lse (optional, [T, H] fp32,
 * natural log, without the sink).  group_starts (optional, [num_groups + 1])
 * groups the consecutive-position query tokens of one request (decode with
 * MTP drafts) so they share one pass over their rows; NULL = one token per
 * group.  A group must be all-valid tokens or all padding. */
int hca_sparse_decode(void* out, int64_t out_stride_tok, int64_t out_stride_head, float* lse,
                      const void* q, int64_t q_stride_tok, int64_t q_stride_head,
                      int32_t num_tokens, int32_t num_heads, int32_t head_dim,
                      int32_t rope_dim, const uint8_t* swa_cache, int32_t swa_page_size,
                      int64_t swa_page_stride_bytes, const int32_t* swa_indices,
                      int64_t swa_indices_stride, const int32_t* swa_lens,
                      const uint8_t* comp_cache, int32_t comp_page_size,
                      int64_t comp_page_stride_bytes, const int32_t* comp_indices,
                      int64_t comp_indices_stride, const int32_t* comp_lens,
                      const int32_t* group_starts, int32_t num_groups, int32_t max_group_tokens,
                      float softmax_scale, const float* attn_sink, int32_t num_splits,
                      void* workspace, int64_t workspace_bytes, void* stream);

/* Decode work list, built once per step on the device (replaces FlashMLA's
 * get_mla_metadata -> tile_scheduler_metadata / num_splits, called at
 * V/models/deepseek_v4/nvidia/flashmla.py:210-302 and
 * V/v1/attention/backends/mla/flashmla_sparse.py:565-687).  Group g's union
 * rows (window of its first token + tail of its last token + the last
 * token's compressed rows) make c_g chunks of 64; the smallest per-CTA chunk
 * budget whose CTA count fits max_items (at most 16 CTAs per group, at least
 * one) is chosen, so the longest CTA of one wave is as short as possible.
 * schedule: int32[hca_decode_schedule_ints(num_groups, max_items)], 16-byte
 * aligned; max_items >= num_groups (one wave = the SM count).  group_starts
 * as for hca_sparse_decode (NULL: one token per group, num_groups = tokens);
 * comp_lens NULL = no compressed rows.  Valid for every layer of the step. */
int64_t hca_decode_schedule_ints(int32_t num_groups, int32_t max_items);
int hca_decode_schedule(int32_t* schedule, int32_t max_items, const int32_t* group_starts,
                        int32_t num_groups, int32_t num_tokens, const int32_t* swa_lens,
                        const int32_t* comp_lens, void* stream);

/* Limit, in ns, of every mbarrier wait of the head_dim-128 attention kernel
 * for launches made from now on in this process (default 2e9; < 0 restores
 * it).  Diagnostic, with no counterpart in the reference: with 0 a wait that
 * is not already satisfied fails at once, so a launch ends early with its
 * device error bits set -- the path a stalled pipeline takes. */
int hca_set_attention_wait_limit_ns(int64_t limit_ns);

/* hca_sparse_decode over a work list from hca_decode_schedule (same
 * max_items) instead of uniform splits.  Workspace:
 * hca_sparse_decode_workspace_bytes(1, max_group_tokens, num_heads, head_dim,
 * max_items) bytes (one partial slot per work item). */
int hca_sparse_decode_scheduled(void* out, int64_t out_stride_tok, int64_t out_stride_head,
                                float* lse, const void* q, int64_t q_stride_tok,
                                int64_t q_stride_head, int32_t num_tokens, int32_t num_heads,
                                int32_t head_dim, int32_t rope_dim, const uint8_t* swa_cache,
                                int32_t swa_page_size, int64_t swa_page_stride_bytes,
                                const int32_t* swa_indices, int64_t swa_indices_stride,
                                const int32_t* swa_lens, const uint8_t* comp_cache,
                                int32_t comp_page_size, int64_t comp_page_stride_bytes,
                                const int32_t* comp_indices, int64_t comp_indices_stride,
                                const int32_t* comp_lens, const int32_t* group_starts,
                                int32_t num_groups, int32_t max_group_tokens, float softmax_scale,
                                const float* attn_sink, const int32_t* schedule, int32_t max_items,
                                void* workspace, int64_t workspace_bytes, void* stream);

/* Decode attention fused with the output stage: the scheduled
 * hca_sparse_decode, whose split partials are merged per token by a second
 * launch that also applies the VHA head mix, the inverse RoPE and the FP8
 * quant of wo_a's input (hca_vha_inv_rope_fp8_quant's outputs and layout),
 * so O never round-trips through memory in bf16.  Replaces the
 * flash_mla_with_kvcache decode call followed by the plugin's fused
 * VHA + inverse RoPE + FP8 quant (V/models/deepseek_v4/nvidia/flashmla.py:210-302;
 * E/nvidia/attention.py:166-285, 471-539).  O is rounded to bf16 before the
 * mix, as in the unfused path.  D = 128, H % 16 == 0, H <= 64.  Workspace:
 * hca_sparse_decode_vha_workspace_bytes(max_items, max_group_tokens,
 * num_heads, head_dim) bytes. */
int64_t hca_sparse_decode_vha_workspace_bytes(int32_t max_items, int32_t max_group_tokens,
                                              int32_t num_heads, int32_t head_dim);
int hca_sparse_decode_vha_fp8_quant(
    uint8_t* out, int32_t* scale, const void* q, int64_t q_stride_tok, int64_t q_stride_head,
    int32_t num_tokens, int32_t num_heads, int32_t head_dim, int32_t rope_dim,
    const uint8_t* swa_cache, int32_t swa_page_size, int64_t swa_page_stride_bytes,
    const int32_t* swa_indices, int64_t swa_indices_stride, const int32_t* swa_lens,
    const uint8_t* comp_cache, int32_t comp_page_size, int64_t comp_page_stride_bytes,
    const int32_t* comp_indices, int64_t comp_indices_stride, const int32_t* comp_lens,
    const int32_t* group_starts, int32_t num_groups, int32_t max_group_tokens,
    float softmax_scale, const float* attn_sink, const int32_t* schedule, int32_t max_items,
    const void* mix, const int64_t* positions, const float* cos_sin, int64_t cos_sin_stride,
    int32_t n_groups, void* workspace, int64_t workspace_bytes, void* stream);

/* hca_sparse_decode for callers that cannot allocate device memory: a
 * runtime that owns every allocation itself (its caching allocator must not
 * be bypassed, or its memory budget is fixed before serving starts) or that
 * calls from a context where cudaMalloc is not allowed, and so cannot supply
 * `workspace`.  No counterpart in the reference (FlashMLA's decode takes its
 * split buffers from the caller).  Same arguments and results as
 * hca_sparse_decode without workspace / workspace_bytes; the split-K partials
 * go to a static device array of HCA_NOALLOC_WORKSPACE_BYTES that every GPU
 * loading this library holds until exit, and a call whose
 * hca_sparse_decode_workspace_bytes exceeds it returns HCA_E_TOO_LARGE.  No
 * memory is allocated.  The first call on a device looks up the array's
 * device address with that device current and keeps it for the life of the
 * process; make that first call before any stream capture, and do not call
 * this entry point again after cudaDeviceReset.  Argument and shape errors
 * (num_splits outside 1..16, head_dim other than 128 / 512) are reported as
 * HCA_E_INVALID / HCA_E_UNSUPPORTED before the size check.  All calls on a GPU share the array: calls whose kernels
 * overlap on the GPU race, so order them on one stream.  Nothing in the array
 * needs clearing between calls (each call writes every partial it merges). */
int hca_sparse_decode_noalloc(void* out, int64_t out_stride_tok, int64_t out_stride_head, float* lse,
                              const void* q, int64_t q_stride_tok, int64_t q_stride_head,
                              int32_t num_tokens, int32_t num_heads, int32_t head_dim,
                              int32_t rope_dim, const uint8_t* swa_cache, int32_t swa_page_size,
                              int64_t swa_page_stride_bytes, const int32_t* swa_indices,
                              int64_t swa_indices_stride, const int32_t* swa_lens,
                              const uint8_t* comp_cache, int32_t comp_page_size,
                              int64_t comp_page_stride_bytes, const int32_t* comp_indices,
                              int64_t comp_indices_stride, const int32_t* comp_lens,
                              const int32_t* group_starts, int32_t num_groups,
                              int32_t max_group_tokens, float softmax_scale,
                              const float* attn_sink, int32_t num_splits, void* stream);

/* Replaces the chunked gather + flash_mla_sparse_fwd of
 * DeepseekV4FlashMLASparseImpl._forward_prefill
 * (V/models/deepseek_v4/nvidia/flashmla.py:304-424): every prefill token at
 * position p of request r attends compressed entries 0 .. (p+1)/ratio - 1 and
 * window positions max(p - W + 1, 0) .. p, read straight from the fp8 caches
 * through the block tables (no bf16 workspace). */
int hca_sparse_prefill(void* out, int64_t out_stride_tok, int64_t out_stride_head,
                       const void* q, int64_t q_stride_tok, int64_t q_stride_head,
                       int32_t num_heads, int32_t head_dim, int32_t rope_dim,
                       const int32_t* query_start_loc, const int32_t* seq_lens, int32_t num_reqs,
                       int32_t num_tokens, const uint8_t* swa_cache, int32_t swa_page_size,
                       int64_t swa_page_stride_bytes, const int32_t* swa_block_table,
                       int64_t swa_bt_stride, const uint8_t* comp_cache, int32_t comp_page_size,
                       int64_t comp_page_stride_bytes, const int32_t* comp_block_table,
                       int64_t comp_bt_stride, int32_t window, int32_t compress_ratio,
                       float softmax_scale, const float* attn_sink, void* stream);

/* ---------------------------------------------------------------------- */
/* Output path                                                              */
/* ---------------------------------------------------------------------- */

/* Replaces the plugin's vha_inv_rope_fp8_quant (E/nvidia/attention.py:166-285):
 * y = mix @ o over heads (bf16 operands, fp32 accumulation), inverse GPT-J
 * RoPE at the token position, UE8M0 1x128 FP8.  out: [G, T, (H/G) * D] e4m3;
 * scale: int32 [G, H/G, aligned_T] (aligned_T = round_up(T, 4)), byte c of
 * each int32 = exponent byte of 128-chunk c (zero bytes past D/128 chunks;
 * padding rows zero). */
int hca_vha_inv_rope_fp8_quant(uint8_t* out, int32_t* scale, const void* o, int64_t o_stride_tok,
                               int64_t o_stride_head, const void* mix, const int64_t* positions,
                               const float* cos_sin, int64_t cos_sin_stride, int32_t num_tokens,
                               int32_t num_heads, int32_t n_groups, int32_t head_dim,
                               int32_t rope_dim, void* stream);

/* Unfused bf16-wo_a output path (E/nvidia/attention.py:121-157,525 then the
 * inverse RoPE of V/v1/attention/ops/rocm_aiter_mla_sparse.py:894-927):
 * out [T, H, D] bf16 = inverse-RoPE(mix @ o).  mix may be NULL (identity). */
int hca_vha_inv_rope(void* out, int64_t out_stride_tok, int64_t out_stride_head, const void* o,
                     int64_t o_stride_tok, int64_t o_stride_head, const void* mix,
                     const int64_t* positions, const float* cos_sin, int64_t cos_sin_stride,
                     int32_t num_tokens, int32_t num_heads, int32_t head_dim, int32_t rope_dim,
                     void* stream);

/* Replaces fused_inv_rope_fp8_quant with tma_aligned_scales=True
 * (V/models/deepseek_v4/common/ops/fused_inv_rope_fp8_quant.py:17-212):
 * out [G, T, (H/G) * D] e4m3; scale int32 [G, packs, aligned_T] with packs =
 * ceil((H/G) * D / 512), byte c of pack k = exponent of 128-chunk 4k + c. */
int hca_inv_rope_fp8_quant(uint8_t* out, int32_t* scale, const void* o, int64_t o_stride_tok,
                           int64_t o_stride_head, const int64_t* positions, const float* cos_sin,
                           int64_t cos_sin_stride, int32_t num_tokens, int32_t num_heads,
                           int32_t n_groups, int32_t head_dim, int32_t rope_dim, void* stream);

/* Replaces sigmoid_mul_quant_fp8 (E/nvidia/attention.py:288-361):
 * x * sigmoid(gate) with the unfused bf16 roundings, 1x128 UE8M0 FP8.
 * out [rows, hidden] e4m3; scale int32 with strides (1, aligned_rows),
 * aligned_rows = round_up(rows, 4), shape [rows, hidden / 512]. */
int hca_sigmoid_mul_quant_fp8(uint8_t* out, int32_t* scale, const void* x, int64_t x_stride,
                              const void* gate, int64_t gate_stride, int32_t rows,
                              int32_t hidden, void* stream);

/* Replaces the block-scaled FP8 GEMMs of the output path: the grouped wo_a
 * einsum (DeepGEMM fp8_einsum "bhr,hdr->bhd", V/models/deepseek_v4/
 * attention.py:317-347) and the gated wo_b linear (GatedDeepGemmLinear,
 * E/nvidia/attention.py:364-395, apply_block_scaled_mm).
 *   out[t, g, n] = sum_k x[t, g, k] * sx[t, g, k / 128] * w[g, n, k] * sw[g, n / 128, k / 128]
 * x e4m3 rows of K bytes at x + g * x_stride_group + t * x_stride_tok (16-byte
 * aligned); sx UE8M0 bytes, byte (b % xs_per_int) of the int32 at
 * x_scale[t * xs_stride_tok + g * xs_stride_group + (b / xs_per_int) *
 * xs_stride_pack] for K block b (xs_per_int 1 or 4: the layouts written by
 * hca_vha_inv_rope_fp8_quant, hca_sparse_decode_vha_fp8_quant and
 * hca_sigmoid_mul_quant_fp8); w e4m3 [G, N, K] contiguous with fp32 block
 * scales w_scale [G, ceil(N / 128), K / 128]; out bf16 with element strides
 * (out_stride_tok, out_stride_group), 16-byte aligned rows.  N a multiple of
 * 64, K of 128; otherwise HCA_E_UNSUPPORTED.  fp32 accumulation: each
 * 128-wide K block's partial product is scaled once and summed in fp32.
 * Small token counts split K over a thread-block cluster of 2-8 CTAs whose
 * fp32 partial tiles go through `workspace` (16-byte aligned, at least
 * hca_fp8_grouped_gemm_workspace_bytes(...) bytes; NULL when that is 0;
 * HCA_E_WORKSPACE if smaller).  Calls sharing a workspace must be ordered on
 * one stream. */
int64_t hca_fp8_grouped_gemm_workspace_bytes(int32_t num_tokens, int32_t num_groups, int32_t n,
                                             int32_t k);
int hca_fp8_grouped_gemm(void* out, int64_t out_stride_tok, int64_t out_stride_group,
                         const uint8_t* x, int64_t x_stride_tok, int64_t x_stride_group,
                         const int32_t* x_scale, int64_t xs_stride_tok, int64_t xs_stride_group,
                         int64_t xs_stride_pack, int32_t xs_per_int, const uint8_t* w,
                         const float* w_scale, int32_t num_tokens, int32_t num_groups, int32_t n,
                         int32_t k, void* workspace, int64_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* HCA_B200_H_ */
