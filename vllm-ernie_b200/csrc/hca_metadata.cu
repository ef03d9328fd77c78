// Integer metadata builders of the HCA path: slot mappings, window indices,
// compressed-entry indices and the prefill index combine.  All are tiny,
// latency-bound launches (a few KB of int traffic per step); the layout of
// their outputs is the reference's, bit for bit.
#include "hca_common.cuh"

namespace hca {
namespace {

// One block per request; threads stride over its query tokens.
__global__ void token_to_req_kernel(int32_t* out, const int32_t* qsl) {
  const int r = blockIdx.x;
  const int qs = qsl[r], qe = qsl[r + 1];
  for (int t = qs + threadIdx.x; t < qe; t += blockDim.x) out[t] = r;
}

__global__ void slot_mapping_kernel(int64_t* out, const int32_t* qsl, const int32_t* seq_lens,
                                    const int32_t* bt, int64_t bt_stride, int block_size) {
  const int r = blockIdx.x;
  const int qs = qsl[r], qe = qsl[r + 1];
  const int64_t start = static_cast<int64_t>(seq_lens[r]) - (qe - qs);
  for (int i = threadIdx.x; i < qe - qs; i += blockDim.x) {
    const int64_t p = start + i;
    const int64_t blk = bt[r * bt_stride + p / block_size];
    out[qs + i] = blk * block_size + p % block_size;
  }
}

__global__ void fill_i64_kernel(int64_t* out, int n, int64_t v) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) out[i] = v;
}

// V/v1/attention/backends/mla/compressor_utils.py:8-50
__global__ void compressed_slot_mapping_kernel(int64_t* out, const int32_t* qsl,
                                               const int32_t* seq_lens, const int32_t* bt,
                                               int64_t bt_stride, int block_size, int ratio) {
  const int r = blockIdx.x;
  const int qs = qsl[r], qe = qsl[r + 1];
  const int64_t start = static_cast<int64_t>(seq_lens[r]) - (qe - qs);
  for (int i = threadIdx.x; i < qe - qs; i += blockDim.x) {
    const int64_t p = start + i;
    int64_t slot = -1;
    if ((p + 1) % ratio == 0) {
      const int64_t c = p / ratio;
      slot = static_cast<int64_t>(bt[r * bt_stride + c / block_size]) * block_size + c % block_size;
    }
    out[qs + i] = slot;
  }
}

// V/v1/attention/backends/mla/sparse_swa.py:449-503 (one block per token).
__global__ void swa_indices_kernel(int32_t* idx, int64_t idx_stride, int32_t* lens,
                                   int num_decode_tokens, int lens_len, int window,
                                   const int32_t* qsl, const int32_t* seq_lens,
                                   const int32_t* t2r, const uint8_t* is_valid,
                                   const int32_t* bt, int64_t bt_stride, int block_size) {
  const int t = blockIdx.x;
  if (t >= num_decode_tokens) {
    // the extra last block zeroes lens past the decode tokens (sparse_swa.py:296)
    for (int i = num_decode_tokens + threadIdx.x; i < lens_len; i += blockDim.x) lens[i] = 0;
    return;
  }
  if (!is_valid[t]) {
    if (threadIdx.x == 0) lens[t] = 0;
    return;
  }
  const int r = t2r[t];
  const int qs = qsl[r], qe = qsl[r + 1];
  const int64_t pos = static_cast<int64_t>(seq_lens[r]) - (qe - qs) + (t - qs);
  const int64_t start = pos - window + 1 > 0 ? pos - window + 1 : 0;
  const int n = static_cast<int>(pos + 1 - start);
  if (threadIdx.x == 0) lens[t] = n;
  for (int i = threadIdx.x; i < window; i += blockDim.x) {
    int32_t v = -1;
    if (i < n) {
      const int64_t p = start + i;
      v = static_cast<int32_t>(static_cast<int64_t>(bt[r * bt_stride + p / block_size]) * block_size +
                               p % block_size);
    }
    idx[t * idx_stride + i] = v;
  }
}

// V/v1/attention/backends/mla/flashmla_sparse.py:1083-1149 (one block per token).
__global__ void c128a_kernel(int32_t* gdec, int64_t gdec_stride, int32_t* dlens, int32_t* plocal,
                             int64_t plocal_stride, const int64_t* positions, int ratio, int maxc,
                             int num_decode_tokens, const int32_t* t2r, const int32_t* bt,
                             int64_t bt_stride, int block_size, const int64_t* slot_mapping) {
  const int t = blockIdx.x;
  const int64_t p = positions[t];
  int64_t nc = (p + 1) / ratio;
  if (nc > maxc) nc = maxc;
  const int n = static_cast<int>(nc);
  if (t < num_decode_tokens) {
    const int r = t2r[t];
    for (int i = threadIdx.x; i < maxc; i += blockDim.x) {
      int32_t v = -1;
      if (i < n)
        v = static_cast<int32_t>(static_cast<int64_t>(bt[r * bt_stride + i / block_size]) * block_size +
                                 i % block_size);
      gdec[t * gdec_stride + i] = v;
    }
    if (threadIdx.x == 0) dlens[t] = slot_mapping[t] >= 0 ? n : 0;
  } else {
    const int pt = t - num_decode_tokens;
    for (int i = threadIdx.x; i < maxc; i += blockDim.x)
      plocal[pt * plocal_stride + i] = i < n ? i : -1;
  }
}

// V/v1/attention/backends/mla/sparse_swa.py:422-446
__global__ void prefill_gather_lens_kernel(int32_t* out, const int32_t* seq_lens,
                                           const int32_t* qsl, int num_prefills, int num_decodes,
                                           int window) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < num_prefills; i += gridDim.x * blockDim.x) {
    const int r = num_decodes + i;
    const int ql = qsl[r + 1] - qsl[r];
    const int prefix = seq_lens[r] - ql;
    out[i] = ql + (prefix < window - 1 ? prefix : window - 1);
  }
}

// V/models/deepseek_v4/common/ops/cache_utils.py:510-594 (one block per token).
__global__ void combine_kernel(int32_t* comb, int64_t comb_stride, int width, int32_t* comb_lens,
                               const int32_t* topk, int64_t topk_stride, const int32_t* qsl,
                               const int32_t* seq_lens, const int32_t* gather_lens, int num_reqs,
                               int window, int ratio, int top_k, int M, int N) {
  const int t_local = blockIdx.x;
  const int base = qsl[0];
  // request of this token: qsl is sorted
  int lo = 0, hi = num_reqs - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (qsl[mid] - base <= t_local) lo = mid; else hi = mid - 1;
  }
  const int b = lo;
  const int qs = qsl[b] - base, qe = qsl[b + 1] - base;
  const int sl = seq_lens[b];
  const int gstart = sl - gather_lens[b];
  const int pos = sl - (qe - qs) + (t_local - qs);
  int tk = (pos + 1) / ratio;
  if (tk > top_k) tk = top_k;
  const int sw = pos + 1 < window ? pos + 1 : window;
  for (int i = threadIdx.x; i < width; i += blockDim.x) {
    int32_t v = -1;
    if (i < tk) v = topk[t_local * topk_stride + i] + M * b;
    else if (i < tk + sw) v = M * b + N + (i - tk) + pos - sw + 1 - gstart;
    comb[t_local * comb_stride + i] = v;
  }
  if (threadIdx.x == 0) comb_lens[t_local] = tk + sw;
}

}  // namespace
}  // namespace hca

using namespace hca;

extern "C" int hca_token_to_req(int32_t* out, const int32_t* query_start_loc, int32_t num_reqs,
                                int32_t num_tokens, void* stream) {
  HCA_CHECK_ARG(num_reqs >= 0 && num_tokens >= 0);
  if (num_reqs == 0 || num_tokens == 0) return HCA_OK;
  HCA_CHECK_ARG(out && query_start_loc);
  token_to_req_kernel<<<num_reqs, 128, 0, as_stream(stream)>>>(out, query_start_loc);
  return HCA_LAUNCH_STATUS();
}

extern "C" int hca_slot_mapping(int64_t* out, const int32_t* query_start_loc,
                                const int32_t* seq_lens, const int32_t* block_table,
                                int64_t bt_stride, int32_t num_reqs, int32_t block_size,
                                void* stream) {
  HCA_CHECK_ARG(num_reqs >= 0 && block_size > 0);
  if (num_reqs == 0) return HCA_OK;
  HCA_CHECK_ARG(out && query_start_loc && seq_lens && block_table);
  slot_mapping_kernel<<<num_reqs, 128, 0, as_stream(stream)>>>(out, query_start_loc, seq_lens,
                                                               block_table, bt_stride, block_size);
  return HCA_LAUNCH_STATUS();
}

extern "C" int hca_compressed_slot_mapping(int64_t* out, int32_t out_len,
                                           const int32_t* query_start_loc,
                                           const int32_t* seq_lens, const int32_t* block_table,
                                           int64_t bt_stride, int32_t num_reqs,
                                           int32_t block_size, int32_t compress_ratio,
                                           void* stream) {
  HCA_CHECK_ARG(out_len >= 0 && num_reqs >= 0 && block_size > 0 && compress_ratio > 0);
  if (out_len > 0) {
    HCA_CHECK_ARG(out);
    fill_i64_kernel<<<cdiv(out_len, 256) < 1024 ? cdiv(out_len, 256) : 1024, 256, 0,
                      as_stream(stream)>>>(out, out_len, -1);
  }
  if (num_reqs > 0) {
    HCA_CHECK_ARG(query_start_loc && seq_lens && block_table);
    compressed_slot_mapping_kernel<<<num_reqs, 128, 0, as_stream(stream)>>>(
        out, query_start_loc, seq_lens, block_table, bt_stride, block_size, compress_ratio);
  }
  return HCA_LAUNCH_STATUS();
}

extern "C" int hca_swa_indices_and_lens(int32_t* indices, int64_t indices_stride, int32_t* lens,
                                        int32_t lens_len, int32_t num_decode_tokens,
                                        int32_t window, const int32_t* query_start_loc,
                                        const int32_t* seq_lens, const int32_t* token_to_req,
                                        const uint8_t* is_valid_token,
                                        const int32_t* block_table, int64_t bt_stride,
                                        int32_t block_size, void* stream) {
  HCA_CHECK_ARG(num_decode_tokens >= 0 && lens_len >= num_decode_tokens && window > 0 &&
                block_size > 0 && indices_stride >= window);
  // Blocks past num_decode_tokens zero the tail of `lens`.
  const int tail = lens_len - num_decode_tokens;
  const int grid = num_decode_tokens + (tail > 0 ? 1 : 0);
  if (grid == 0) return HCA_OK;
  HCA_CHECK_ARG(lens);
  if (num_decode_tokens > 0)
    HCA_CHECK_ARG(indices && query_start_loc && seq_lens && token_to_req && is_valid_token &&
                  block_table);
  swa_indices_kernel<<<grid, 128, 0, as_stream(stream)>>>(
      indices, indices_stride, lens, num_decode_tokens, lens_len, window, query_start_loc,
      seq_lens, token_to_req, is_valid_token, block_table, bt_stride, block_size);
  return HCA_LAUNCH_STATUS();
}

extern "C" int hca_c128a_topk_metadata(int32_t* global_decode, int64_t global_decode_stride,
                                       int32_t* decode_lens, int32_t* prefill_local,
                                       int64_t prefill_local_stride, const int64_t* positions,
                                       int32_t num_tokens, int32_t compress_ratio,
                                       int32_t max_compressed_tokens, int32_t num_decode_tokens,
                                       const int32_t* token_to_req, const int32_t* block_table,
                                       int64_t bt_stride, int32_t block_size,
                                       const int64_t* slot_mapping, void* stream) {
  HCA_CHECK_ARG(num_tokens >= 0 && num_decode_tokens >= 0 && num_decode_tokens <= num_tokens &&
                compress_ratio > 0 && max_compressed_tokens > 0 && block_size > 0);
  if (num_tokens == 0) return HCA_OK;
  HCA_CHECK_ARG(positions);
  if (num_decode_tokens > 0)
    HCA_CHECK_ARG(global_decode && decode_lens && token_to_req && block_table && slot_mapping &&
                  global_decode_stride >= max_compressed_tokens);
  if (num_tokens > num_decode_tokens)
    HCA_CHECK_ARG(prefill_local && prefill_local_stride >= max_compressed_tokens);
  c128a_kernel<<<num_tokens, 256, 0, as_stream(stream)>>>(
      global_decode, global_decode_stride, decode_lens, prefill_local, prefill_local_stride,
      positions, compress_ratio, max_compressed_tokens, num_decode_tokens, token_to_req,
      block_table, bt_stride, block_size, slot_mapping);
  return HCA_LAUNCH_STATUS();
}

extern "C" int hca_prefill_gather_lens(int32_t* gather_lens, const int32_t* seq_lens,
                                       const int32_t* query_start_loc, int32_t num_prefills,
                                       int32_t num_decodes, int32_t window, void* stream) {
  HCA_CHECK_ARG(num_prefills >= 0 && num_decodes >= 0 && window > 0);
  if (num_prefills == 0) return HCA_OK;
  HCA_CHECK_ARG(gather_lens && seq_lens && query_start_loc);
  prefill_gather_lens_kernel<<<cdiv(num_prefills, 128), 128, 0, as_stream(stream)>>>(
      gather_lens, seq_lens, query_start_loc, num_prefills, num_decodes, window);
  return HCA_LAUNCH_STATUS();
}

extern "C" int hca_combine_topk_swa_indices(int32_t* combined, int64_t combined_stride,
                                              int32_t combined_width, int32_t* combined_lens,
                                              const int32_t* topk_indices, int64_t topk_stride,
                                              const int32_t* query_start_loc,
                                              const int32_t* seq_lens, const int32_t* gather_lens,
                                            int32_t num_reqs, int32_t num_tokens,
                                            int32_t window, int32_t compress_ratio,
                                            int32_t top_k, int32_t M, int32_t N, void* stream) {
  HCA_CHECK_ARG(num_reqs >= 0 && num_tokens >= 0 && window > 0 && compress_ratio > 0 &&
                top_k >= 0 && combined_width >= top_k + window &&
                combined_stride >= combined_width);
  if (num_reqs == 0 || num_tokens == 0) return HCA_OK;
  HCA_CHECK_ARG(combined && combined_lens && query_start_loc && seq_lens && gather_lens);
  HCA_CHECK_ARG(top_k == 0 || topk_indices);
  combine_kernel<<<num_tokens, 128, 0, as_stream(stream)>>>(
      combined, combined_stride, combined_width, combined_lens, topk_indices, topk_stride,
      query_start_loc, seq_lens, gather_lens, num_reqs, window, compress_ratio, top_k, M, N);
  return HCA_LAUNCH_STATUS();
}
