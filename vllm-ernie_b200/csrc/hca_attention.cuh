// Shared description of a sparse HCA attention launch: the parameter block
// every attention kernel takes, the per-group row resolution (window rows then
// compressed rows, per-token masks) and small conversions.  Used by the
// head_dim-128 kernels and by the head_dim-512 CTA-pair kernel.
#pragma once

#include "hca_common.cuh"

namespace hca {

constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Where the rows of a group come from.
struct AttnParams {
  // q / out
  const __nv_bfloat16* q;
  int64_t q_st, q_sh;
  __nv_bfloat16* out;
  int64_t o_st, o_sh;
  float* lse;
  int num_heads, rope_dim;
  // caches
  const uint8_t* swa_cache;
  int swa_page;
  int64_t swa_pstride;
  const uint8_t* comp_cache;
  int comp_page;
  int64_t comp_pstride;
  // decode: index tables
  const int32_t* swa_idx;
  int64_t swa_idx_st;
  const int32_t* swa_lens;
  const int32_t* comp_idx;
  int64_t comp_idx_st;
  const int32_t* comp_lens;
  const int32_t* group_starts;  // nullptr: one token per group
  // prefill: block tables
  const int32_t* qsl;
  const int32_t* seq_lens;
  int num_reqs;
  const int32_t* swa_bt;
  int64_t swa_bt_st;
  const int32_t* comp_bt;
  int64_t comp_bt_st;
  int window, ratio;
  int group_tokens;  // prefill tile size in tokens
  // softmax
  float scale_log2;
  const float* sink;
  // split-K
  int num_splits;
  float* ws_o;      // [groups][splits][rows][D], or [items][rows][D] with a schedule
  float* ws_ml;     // [groups][splits][rows][2], or [items][rows][2] with a schedule
  int max_rows;     // query rows per group slot in the workspace
  // decode work list (nullptr: num_splits uniform splits per group):
  // sched[4 * i .. 4 * i + 3] = {group, split, chunk begin, chunk end} of CTA
  // i (group -1: idle), then per group {first item, items}
  const int32_t* sched;
  int sched_items;
  // every CTA writes its partial, even a group's only CTA (the merge happens
  // in the fused combine + VHA kernel)
  int force_partials;
  // the partial O rows are bf16 (the fused merge + VHA path): half the bytes,
  // every split of a token in flight at once in the merge
  int bf16_partials;
  // limit of every mbarrier wait of the head_dim-128 kernel (0: probe once)
  uint64_t wait_ns;
};

// Resolved description of one group.
struct Group {
  int t0, ntok;        // first token, tokens
  int n_win, n_comp;   // union rows: window then compressed
  // decode (index tables)
  int len0, len_last, first_tok, last_tok;
  // prefill (block tables)
  int req;
  int64_t p0;          // position of token t0
  int64_t win_start;   // position of union window row 0
};

// Decode: the consecutive query tokens [t0, t1) of one request.
__device__ __forceinline__ void resolve_tokens(const AttnParams& P, int t0, int t1, Group& G) {
  G.t0 = t0;
  G.ntok = t1 - t0;
  G.first_tok = t0;
  G.last_tok = t1 - 1;
  G.len0 = P.swa_lens[t0];
  G.len_last = P.swa_lens[t1 - 1];
  if (G.len0 <= 0) {  // padding group
    G.n_win = 0;
    G.n_comp = 0;
    return;
  }
  int extra = G.ntok - 1;
  if (extra > G.len_last) extra = G.len_last;
  G.n_win = G.len0 + extra;
  G.n_comp = P.comp_cache ? P.comp_lens[t1 - 1] : 0;
  if (G.n_comp < 0) G.n_comp = 0;
}

// Decode: the group's tokens (gidx-th of group_starts, or token gidx).
__device__ __forceinline__ void group_tokens(const AttnParams& P, int gidx, int& t0, int& t1) {
  if (P.group_starts) {
    t0 = P.group_starts[gidx];
    t1 = P.group_starts[gidx + 1];
  } else {
    t0 = gidx;
    t1 = gidx + 1;
  }
}

template <bool kPrefill>
__device__ __forceinline__ bool resolve_group(const AttnParams& P, int gidx, Group& G) {
  if (!kPrefill) {
    int t0, t1;
    group_tokens(P, gidx, t0, t1);
    resolve_tokens(P, t0, t1, G);
    return true;
  }
  // prefill: tile gidx -> (request, first token) by walking the requests
  int tile = gidx;
  for (int r = 0; r < P.num_reqs; ++r) {
    const int qs = P.qsl[r], qe = P.qsl[r + 1];
    const int ntiles = (qe - qs + P.group_tokens - 1) / P.group_tokens;
    if (tile < ntiles) {
      G.req = r;
      G.t0 = qs + tile * P.group_tokens;
      G.ntok = min(P.group_tokens, qe - G.t0);
      G.p0 = static_cast<int64_t>(P.seq_lens[r]) - (qe - qs) + (G.t0 - qs);
      const int64_t plast = G.p0 + G.ntok - 1;
      G.win_start = G.p0 - P.window + 1 > 0 ? G.p0 - P.window + 1 : 0;
      G.n_win = static_cast<int>(plast + 1 - G.win_start);
      G.n_comp = P.comp_cache ? static_cast<int>((plast + 1) / P.ratio) : 0;
      return true;
    }
    tile -= ntiles;
  }
  return false;
}

// Source slot of union row u and the bitmask of group tokens that attend it.
template <bool kPrefill>
__device__ __forceinline__ void row_source(const AttnParams& P, const Group& G, int u,
                                           bool& is_comp, int64_t& slot, uint32_t& mask) {
  mask = 0;
  slot = -1;
  is_comp = u >= G.n_win;
  if (!kPrefill) {
    if (!is_comp) {
      slot = u < G.len0 ? P.swa_idx[G.first_tok * P.swa_idx_st + u]
                        : P.swa_idx[G.last_tok * P.swa_idx_st + (G.len_last - (G.n_win - u))];
      for (int k = 0; k < G.ntok; ++k) {
        const int lk = P.swa_lens[G.t0 + k];
        if (lk > 0 && u >= k + G.len0 - lk && u <= k + G.len0 - 1) mask |= 1u << k;
      }
    } else {
      const int i = u - G.n_win;
      slot = P.comp_idx[G.last_tok * P.comp_idx_st + i];
      for (int k = 0; k < G.ntok; ++k)
        if (i < P.comp_lens[G.t0 + k]) mask |= 1u << k;
    }
    if (slot < 0) mask = 0;
    return;
  }
  if (!is_comp) {
    const int64_t pos = G.win_start + u;
    slot = static_cast<int64_t>(P.swa_bt[G.req * P.swa_bt_st + pos / P.swa_page]) * P.swa_page +
           pos % P.swa_page;
    for (int k = 0; k < G.ntok; ++k) {
      const int64_t pk = G.p0 + k;
      if (pos <= pk && pos > pk - P.window) mask |= 1u << k;
    }
  } else {
    const int i = u - G.n_win;
    slot = static_cast<int64_t>(P.comp_bt[G.req * P.comp_bt_st + i / P.comp_page]) * P.comp_page +
           i % P.comp_page;
    for (int k = 0; k < G.ntok; ++k)
      if (i < (G.p0 + k + 1) / P.ratio) mask |= 1u << k;
  }
}

// Launch the head_dim-512 CTA-pair kernel (decode: grid of splits x group
// tiles; prefill: one pair per tile of tokens).  Defined in
// hca_attention_wide.cu.
int launch_wide_attention(const AttnParams& P, bool prefill, int num_groups, int max_group_tokens, int* err,
                          cudaStream_t s);

// Query tokens one pair handles at head count H (one M=128 tile of rows, at
// most 31 tokens: a row's token mask keeps bit 31 for its "loaded" flag).
inline int wide_tile_tokens(int num_heads) { return num_heads > 0 ? (128 / num_heads < 31 ? 128 / num_heads : 31) : 0; }

}  // namespace hca
