// hca_sparse_decode_noalloc: the split-K decode attention for callers that
// cannot allocate device memory.
//
// Who needs it: a host runtime that owns every device allocation itself (a
// caching allocator that must not be bypassed, a process whose memory budget
// is fixed before serving starts) or that calls in from a context where
// cudaMalloc is not allowed, and so cannot hand hca_sparse_decode a workspace.
// The split-K partials then live in one file-scope device array of fixed size,
// HCA_NOALLOC_WORKSPACE_BYTES, which every GPU that loads this library holds
// until the process exits.
//
// What the array holds between calls: the previous call's partials.  Nothing
// in it needs to start at zero: each call writes the running max and sum of
// every valid query row of every split before the merge reads them, and the
// merge reads a split's output partial only where that split's sum is
// positive, i.e. where this call wrote it.  All calls on one GPU share the
// array, so two calls whose kernels overlap on that GPU (different streams
// without ordering between them, or different host threads) race on it;
// order them on one stream.
#include <mutex>

#include "hca_common.cuh"

namespace {

constexpr int64_t kNoallocBytes = HCA_NOALLOC_WORKSPACE_BYTES;
constexpr int kMaxDevices = 64;

// The split-K scratch.  In host code this name is only a stand-in for the
// symbol, never a device address: host code passes the address that
// cudaGetSymbolAddress returns for the current device.
static __device__ __align__(256) unsigned char g_noalloc_workspace[kNoallocBytes];

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevices] = {};

// Device address of the scratch on the current device, looked up once per
// device (with that device current) and cached for the life of the process:
// after cudaDeviceReset (or any teardown of the device's primary context)
// the cached address is stale, so this entry point must not be used again
// in that process.
int noalloc_workspace(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return HCA_E_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return HCA_E_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_workspace) != cudaSuccess || !p) return HCA_E_CUDA;
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return HCA_OK;
}

}  // namespace

extern "C" int hca_sparse_decode_noalloc(void* out, int64_t out_stride_tok, int64_t out_stride_head, float* lse,
                                         const void* q, int64_t q_stride_tok, int64_t q_stride_head,
                                         int32_t num_tokens, int32_t num_heads, int32_t head_dim,
                                         int32_t rope_dim, const uint8_t* swa_cache, int32_t swa_page_size,
                                         int64_t swa_page_stride_bytes, const int32_t* swa_indices,
                                         int64_t swa_indices_stride, const int32_t* swa_lens,
                                         const uint8_t* comp_cache, int32_t comp_page_size,
                                         int64_t comp_page_stride_bytes, const int32_t* comp_indices,
                                         int64_t comp_indices_stride, const int32_t* comp_lens,
                                         const int32_t* group_starts, int32_t num_groups,
                                         int32_t max_group_tokens, float softmax_scale, const float* attn_sink,
                                         int32_t num_splits, void* stream) {
  // the same grouping rule as hca_sparse_decode: no group table = one token per group
  const int32_t groups = group_starts ? num_groups : num_tokens;
  const int32_t group_tokens = group_starts ? max_group_tokens : 1;
  // argument and shape errors are reported as such before the size check
  if (num_splits < 1 || num_splits > 16 || num_tokens < 0 || groups < 0 || num_heads < 1 || group_tokens < 1)
    return HCA_E_INVALID;
  if ((head_dim != 128 && head_dim != 512) || rope_dim != 64) return HCA_E_UNSUPPORTED;
  void* ws = nullptr;
  int64_t need = 0;
  if (num_splits > 1 && groups > 0 && num_tokens > 0) {
    need = hca_sparse_decode_workspace_bytes(groups, group_tokens, num_heads, head_dim, num_splits);
    if (need > kNoallocBytes) return HCA_E_TOO_LARGE;
    if (need > 0) {
      const int rc = noalloc_workspace(&ws);
      if (rc != HCA_OK) return rc;
    }
  }
  return hca_sparse_decode(out, out_stride_tok, out_stride_head, lse, q, q_stride_tok, q_stride_head, num_tokens,
                           num_heads, head_dim, rope_dim, swa_cache, swa_page_size, swa_page_stride_bytes,
                           swa_indices, swa_indices_stride, swa_lens, comp_cache, comp_page_size,
                           comp_page_stride_bytes, comp_indices, comp_indices_stride, comp_lens, group_starts,
                           num_groups, max_group_tokens, softmax_scale, attn_sink, num_splits, ws,
                           need > 0 ? kNoallocBytes : 0, stream);
}
