// Sparse HCA attention over [window || compressed] rows of the fp8 caches,
// with the per-head attention sink.  One kernel serves decode (rows named by
// the FlashMLA-style index tables) and chunked prefill (rows derived from the
// block tables and positions).
//
// Work unit: a "group" of up to 192 / H query tokens of one request at
// consecutive positions (MTP drafts in decode, neighbouring tokens in
// prefill).  Because K = V is one KV head shared by all H heads, the group's
// G*H query rows are multiplied against the union of the group's rows, each
// K row fetched and dequantised once per CTA; per-token masks select the
// rows each token attends.
//
// Per CTA: one warp per 16 query rows (<= 12 warps); KV rows stream in
// chunks of 64: the raw e4m3 / bf16 bytes of chunk c+1 are loaded into
// registers while chunk c is multiplied, then dequantised into a bf16 smem
// tile.  S = Q K^T and O += P V run on the tensor cores (m16n8k16 bf16, fp32
// accumulate), softmax online in base 2.  Decode splits a group's rows
// across CTAs (split-K) and the last CTA to finish combines the partials.
#include "hca_common.cuh"

namespace hca {
namespace {

constexpr int kChunk = 64;     // KV rows per pipeline step
constexpr int kMaxWarps = 12;  // 192 query rows per CTA
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ void mma16816(float* c, const uint32_t* a, const uint32_t* b) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t* r, const void* smem) {
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(a));
}

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t* r, const void* smem) {
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(a));
}

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
  float* ws_o;      // [groups][splits][rows][D]
  float* ws_ml;     // [groups][splits][rows][2]
  int max_rows;     // query rows per group slot in the workspace
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

template <bool kPrefill>
__device__ __forceinline__ bool resolve_group(const AttnParams& P, int gidx, Group& G) {
  if (!kPrefill) {
    int t0, t1;
    if (P.group_starts) {
      t0 = P.group_starts[gidx];
      t1 = P.group_starts[gidx + 1];
    } else {
      t0 = gidx;
      t1 = gidx + 1;
    }
    G.t0 = t0;
    G.ntok = t1 - t0;
    G.first_tok = t0;
    G.last_tok = t1 - 1;
    G.len0 = P.swa_lens[t0];
    G.len_last = P.swa_lens[t1 - 1];
    if (G.len0 <= 0) {  // padding group
      G.n_win = 0;
      G.n_comp = 0;
      return true;
    }
    int extra = G.ntok - 1;
    if (extra > G.len_last) extra = G.len_last;
    G.n_win = G.len0 + extra;
    G.n_comp = P.comp_cache ? P.comp_lens[t1 - 1] : 0;
    if (G.n_comp < 0) G.n_comp = 0;
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

template <int D, int NOPE, int NW, bool kPrefill>
__global__ void __launch_bounds__(NW * 32, 1) hca_attention_kernel(const AttnParams P) {
  constexpr int kStride = D + 8;  // bf16 elements per smem row (conflict-free ldmatrix)
  constexpr int kNT_S = kChunk / 8;  // n-tiles of S per chunk
  constexpr int kKS_Q = D / 16;      // k-steps of Q K^T
  constexpr int kNT_O = D / 8;       // n-tiles of O
  constexpr int kSegs = D / 8;
  constexpr int kNopeSegs = NOPE / 8;
  constexpr RowGeom kG = {NOPE, NOPE + 2 * (D - NOPE), NOPE / kQuantBlock + 1};

  __shared__ __align__(16) __nv_bfloat16 ktile[2][kChunk * kStride];
  // row metadata ring (chunk c uses entry c % 3): slot, and token mask with
  // bit 31 = row comes from the compressed cache
  __shared__ int64_t rslot[3][kChunk];
  __shared__ uint32_t rmask[3][kChunk];

  const int gidx = blockIdx.y;
  const int split = blockIdx.x;
  Group G;
  if (!resolve_group<kPrefill>(P, gidx, G)) return;
  const int H = P.num_heads;
  const int rows_q = G.ntok * H;
  // a group larger than this launch (or its workspace slot) is never touched
  if (rows_q > NW * 16 || rows_q > P.max_rows) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int nthreads = NW * 32;
  const bool warp_active = warp * 16 < rows_q;
  const int my_tok = warp_active ? (warp * 16) / H : 0;

  const int n_u = G.n_win + G.n_comp;
  const int nchunks = (n_u + kChunk - 1) / kChunk;
  const int c_begin = static_cast<int>((static_cast<int64_t>(split) * nchunks) / P.num_splits);
  const int c_end = static_cast<int>((static_cast<int64_t>(split + 1) * nchunks) / P.num_splits);

  // Q fragments (A operand) straight from global: 16 rows x D per warp.
  uint32_t qf[kKS_Q][4];
  {
    const int g = lane >> 2, c = lane & 3;
#pragma unroll
    for (int kk = 0; kk < kKS_Q; ++kk) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int r = warp * 16 + g + ((j & 1) ? 8 : 0);
        const int d = kk * 16 + 2 * c + ((j & 2) ? 8 : 0);
        uint32_t v = 0;
        if (warp_active && r < rows_q) {
          const int tok = G.t0 + r / H, h = r % H;
          v = *reinterpret_cast<const uint32_t*>(P.q + tok * P.q_st + h * P.q_sh + d);
        }
        qf[kk][j] = v;
      }
    }
  }

  float oacc[kNT_O][4];
#pragma unroll
  for (int j = 0; j < kNT_O; ++j) oacc[j][0] = oacc[j][1] = oacc[j][2] = oacc[j][3] = 0.0f;
  float m_run[2] = {-INFINITY, -INFINITY};
  float l_run[2] = {0.0f, 0.0f};

  // ---- chunk pipeline ----
  constexpr int kItems = kChunk * kSegs;         // (row, 8-element segment) items
  constexpr int kPer = (kItems + nthreads - 1) / nthreads;
  uint4 raw[kPer];
  float scl[kPer];
  constexpr uint32_t kCompBit = 1u << 31;
  // resolve the rows of chunk c into ring entry e (one thread per row)
  auto resolve_chunk = [&](int c, int e) {
    for (int i = threadIdx.x; i < kChunk; i += nthreads) {
      const int u = c * kChunk + i;
      uint32_t mask = 0;
      int64_t slot = -1;
      if (u < n_u) {
        bool is_comp;
        row_source<kPrefill>(P, G, u, is_comp, slot, mask);
        if (slot < 0) mask = 0;
        if (is_comp) mask |= kCompBit;
      }
      rslot[e][i] = slot;
      rmask[e][i] = mask;
    }
  };
  // issue the raw loads of the chunk whose metadata is in ring entry e
  auto load_chunk = [&](int e) {
#pragma unroll
    for (int it = 0; it < kPer; ++it) {
      const int item = threadIdx.x + it * nthreads;
      raw[it] = make_uint4(0, 0, 0, 0);
      scl[it] = 0.0f;
      if (item < kItems) {
        const int row = item / kSegs, seg = item % kSegs;
        const int64_t slot = rslot[e][row];
        if (slot >= 0) {
          const bool is_comp = (rmask[e][row] & kCompBit) != 0;
          const RowPtr p = is_comp ? row_ptr(const_cast<uint8_t*>(P.comp_cache), slot, P.comp_page, P.comp_pstride, kG)
                                   : row_ptr(const_cast<uint8_t*>(P.swa_cache), slot, P.swa_page, P.swa_pstride, kG);
          if (seg < kNopeSegs) {
            const uint2 v = *reinterpret_cast<const uint2*>(p.data + seg * 8);
            raw[it] = make_uint4(v.x, v.y, 0, 0);
            scl[it] = exp2i(static_cast<int>(p.scale[(seg * 8) / kQuantBlock]) - 127);
          } else {
            raw[it] = *reinterpret_cast<const uint4*>(p.data + NOPE + (seg - kNopeSegs) * 16);
          }
        }
      }
    }
  };
  auto store_chunk = [&](int buf) {
#pragma unroll
    for (int it = 0; it < kPer; ++it) {
      const int item = threadIdx.x + it * nthreads;
      if (item < kItems) {
        const int row = item / kSegs, seg = item % kSegs;
        uint4 outv;
        if (seg < kNopeSegs) {
          const float s = scl[it];
          const float2 f0 = e4m3x2_to_float2(static_cast<uint16_t>(raw[it].x & 0xffff));
          const float2 f1 = e4m3x2_to_float2(static_cast<uint16_t>(raw[it].x >> 16));
          const float2 f2 = e4m3x2_to_float2(static_cast<uint16_t>(raw[it].y & 0xffff));
          const float2 f3 = e4m3x2_to_float2(static_cast<uint16_t>(raw[it].y >> 16));
          outv.x = pack_bf16(f0.x * s, f0.y * s);
          outv.y = pack_bf16(f1.x * s, f1.y * s);
          outv.z = pack_bf16(f2.x * s, f2.y * s);
          outv.w = pack_bf16(f3.x * s, f3.y * s);
        } else {
          outv = raw[it];
        }
        *reinterpret_cast<uint4*>(&ktile[buf][row * kStride + seg * 8]) = outv;
      }
    }
  };

  if (c_begin < c_end) {
    resolve_chunk(c_begin, 0);
    __syncthreads();
    load_chunk(0);
    store_chunk(0);
    if (c_begin + 1 < c_end) resolve_chunk(c_begin + 1, 1);
  }
  __syncthreads();
  const int g = lane >> 2, cq = lane & 3;
  for (int c = c_begin; c < c_end; ++c) {
    const int i = c - c_begin;
    const int buf = i & 1, ring = i % 3;
    const bool has_next = c + 1 < c_end;
    if (has_next) load_chunk((i + 1) % 3);
    if (warp_active) {
      // ---- S = Q K^T (16 x 64 per warp) ----
      float s[kNT_S][4];
#pragma unroll
      for (int j = 0; j < kNT_S; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.0f;
      const __nv_bfloat16* kt = ktile[buf];
#pragma unroll
      for (int j = 0; j < kNT_S; ++j) {
#pragma unroll
        for (int kk = 0; kk < kKS_Q; kk += 2) {
          uint32_t b[4];
          ldmatrix_x4(b, kt + (j * 8 + (lane & 7)) * kStride + kk * 16 + (lane >> 3) * 8);
          mma16816(s[j], qf[kk], b);
          mma16816(s[j], qf[kk + 1], b + 2);
        }
      }
      // ---- mask + online softmax (base 2) ----
      float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
      for (int j = 0; j < kNT_S; ++j) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int col = j * 8 + 2 * cq + (e & 1);
          const bool ok = (rmask[ring][col] >> my_tok) & 1u;
          const float v = ok ? s[j][e] * P.scale_log2 : -INFINITY;
          s[j][e] = v;
          mx[e >> 1] = fmaxf(mx[e >> 1], v);
        }
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
        mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
      }
      float alpha[2], base[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float mn = fmaxf(m_run[h], mx[h]);
        base[h] = mn == -INFINITY ? 0.0f : mn;
        alpha[h] = exp2f(m_run[h] - base[h]);
        m_run[h] = mn;
      }
      float rs[2] = {0.0f, 0.0f};
#pragma unroll
      for (int j = 0; j < kNT_S; ++j) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float p = exp2f(s[j][e] - base[e >> 1]);
          s[j][e] = p;
          rs[e >> 1] += p;
        }
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) l_run[h] = l_run[h] * alpha[h] + rs[h];
#pragma unroll
      for (int j = 0; j < kNT_O; ++j) {
        oacc[j][0] *= alpha[0];
        oacc[j][1] *= alpha[0];
        oacc[j][2] *= alpha[1];
        oacc[j][3] *= alpha[1];
      }
      // ---- O += P V ----
#pragma unroll
      for (int kk = 0; kk < kChunk / 16; ++kk) {
        uint32_t a[4];
        a[0] = pack_bf16(s[2 * kk][0], s[2 * kk][1]);
        a[1] = pack_bf16(s[2 * kk][2], s[2 * kk][3]);
        a[2] = pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]);
        a[3] = pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
        for (int j = 0; j < kNT_O; j += 2) {
          uint32_t b[4];
          const int row = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
          const int col = j * 8 + (lane >> 4) * 8;
          ldmatrix_x4_trans(b, kt + row * kStride + col);
          mma16816(oacc[j], a, b);
          mma16816(oacc[j + 1], a, b + 2);
        }
      }
    }
    if (has_next) store_chunk(buf ^ 1);
    if (c + 2 < c_end) resolve_chunk(c + 2, (i + 2) % 3);
    __syncthreads();
  }
  // row sums: reduce across the quad
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], 1);
    l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], 2);
  }

  const float kLn2 = 0.6931471805599453f;
  if (P.num_splits == 1) {
    if (!warp_active) return;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = warp * 16 + g + h * 8;
      if (r >= rows_q) continue;
      const int tok = G.t0 + r / H, head = r % H;
      const float sink2 = P.sink ? P.sink[head] * kLog2e : -INFINITY;
      float inv = 0.0f;
      if (l_run[h] > 0.0f) inv = 1.0f / (l_run[h] + exp2f(sink2 - m_run[h]));
      __nv_bfloat16* orow = P.out + tok * P.o_st + head * P.o_sh;
#pragma unroll
      for (int j = 0; j < kNT_O; ++j) {
        const int d = j * 8 + 2 * cq;
        *reinterpret_cast<uint32_t*>(orow + d) = pack_bf16(oacc[j][2 * h] * inv, oacc[j][2 * h + 1] * inv);
      }
      if (P.lse && cq == 0)
        P.lse[tok * H + head] = l_run[h] > 0.0f ? (m_run[h] + log2f(l_run[h])) * kLn2 : -INFINITY;
    }
    return;
  }

  // ---- split-K: write this split's partial (O unnormalised, m, l) ----
  const int S = P.num_splits;
  const int64_t slot_base = (static_cast<int64_t>(gidx) * S + split) * P.max_rows;
  if (warp_active) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = warp * 16 + g + h * 8;
      if (r >= rows_q) continue;
      float* orow = P.ws_o + (slot_base + r) * D;
#pragma unroll
      for (int j = 0; j < kNT_O; ++j)
        *reinterpret_cast<float2*>(orow + j * 8 + 2 * cq) = make_float2(oacc[j][2 * h], oacc[j][2 * h + 1]);
      if (cq == 0) {
        P.ws_ml[(slot_base + r) * 2] = m_run[h];
        P.ws_ml[(slot_base + r) * 2 + 1] = l_run[h];
      }
    }
  }
}

// Split-K combine: grid (groups, ceil(max_rows / 16)), 256 threads; a CTA
// merges 16 query rows of one group: thread (row, 8-dim segment) sums the
// S partials weighted by 2^(m_s - m), then applies the sink and writes bf16.
template <int D, bool kPrefill>
__global__ void __launch_bounds__(256) hca_attention_combine_kernel(const AttnParams P) {
  constexpr int kSegs = D / 8;
  static_assert(16 * kSegs <= 256 * 4, "one pass per CTA");
  __shared__ float w_s[16][16 + 1];
  __shared__ float inv_s[16];
  const int gidx = blockIdx.x;
  Group G;
  if (!resolve_group<kPrefill>(P, gidx, G)) return;
  const int H = P.num_heads;
  const int rows_q = G.ntok * H;
  if (rows_q > P.max_rows) return;
  const int S = P.num_splits;
  const int r0 = blockIdx.y * 16;
  if (r0 >= rows_q) return;
  const int64_t gbase = static_cast<int64_t>(gidx) * S * P.max_rows;
  // weights per (row, split): one warp per 2 rows
  if (threadIdx.x < 16 * 16) {
    const int rr = threadIdx.x >> 4, sp = threadIdx.x & 15;
    const int r = r0 + rr;
    float m = -INFINITY, l = 0.0f;
    if (sp < S && r < rows_q) {
      const int64_t i = (gbase + static_cast<int64_t>(sp) * P.max_rows + r) * 2;
      m = __ldcg(P.ws_ml + i);
      l = __ldcg(P.ws_ml + i + 1);
      if (!(l > 0.0f)) m = -INFINITY;
    }
    float mx = m;
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const float base = mx == -INFINITY ? 0.0f : mx;
    const float w = (l > 0.0f) ? exp2f(m - base) : 0.0f;
    float lw = l * w;
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) lw += __shfl_xor_sync(0xffffffffu, lw, o);
    if (sp < 16) w_s[rr][sp] = w;
    if (sp == 0 && r < rows_q) {
      const int head = r % H;
      const float sink2 = P.sink ? P.sink[head] * kLog2e : -INFINITY;
      inv_s[rr] = lw > 0.0f ? 1.0f / (lw + exp2f(sink2 - base)) : 0.0f;
      if (P.lse) P.lse[(G.t0 + r / H) * H + head] = lw > 0.0f ? (base + log2f(lw)) * 0.6931471805599453f : -INFINITY;
    }
  }
  __syncthreads();
  for (int item = threadIdx.x; item < 16 * kSegs; item += blockDim.x) {
    const int rr = item / kSegs, seg = item % kSegs;
    const int r = r0 + rr;
    if (r >= rows_q) continue;
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll 4
    for (int sp = 0; sp < S; ++sp) {
      const float w = w_s[rr][sp];
      const float4* src = reinterpret_cast<const float4*>(
          P.ws_o + (gbase + static_cast<int64_t>(sp) * P.max_rows + r) * D + seg * 8);
      const float4 a = __ldcg(src), b = __ldcg(src + 1);
      if (w != 0.0f) {
        acc[0] += w * a.x; acc[1] += w * a.y; acc[2] += w * a.z; acc[3] += w * a.w;
        acc[4] += w * b.x; acc[5] += w * b.y; acc[6] += w * b.z; acc[7] += w * b.w;
      }
    }
    const float inv = inv_s[rr];
    const int tok = G.t0 + r / H, head = r % H;
    uint4 v;
    v.x = pack_bf16(acc[0] * inv, acc[1] * inv);
    v.y = pack_bf16(acc[2] * inv, acc[3] * inv);
    v.z = pack_bf16(acc[4] * inv, acc[5] * inv);
    v.w = pack_bf16(acc[6] * inv, acc[7] * inv);
    *reinterpret_cast<uint4*>(P.out + tok * P.o_st + head * P.o_sh + seg * 8) = v;
  }
}

int64_t align_up(int64_t v, int64_t a) { return (v + a - 1) / a * a; }

}  // namespace
}  // namespace hca

using namespace hca;

extern "C" int64_t hca_sparse_decode_workspace_bytes(int32_t num_groups, int32_t max_group_tokens,
                                                     int32_t num_heads, int32_t head_dim,
                                                     int32_t num_splits) {
  if (num_splits <= 1 || num_groups <= 0) return 0;
  const int64_t rows = static_cast<int64_t>(max_group_tokens) * num_heads;
  const int64_t o = align_up(static_cast<int64_t>(num_groups) * num_splits * rows * head_dim * 4, 256);
  const int64_t ml = align_up(static_cast<int64_t>(num_groups) * num_splits * rows * 2 * 4, 256);
  return o + ml;
}

static bool attn_shape_ok(int num_heads, int head_dim, int rope_dim, int group_tokens) {
  return head_dim == 128 && rope_dim == 64 && num_heads > 0 && num_heads % 16 == 0 &&
         group_tokens >= 1 && group_tokens <= 32 && group_tokens * num_heads <= kMaxWarps * 16;
}

// One warp per 16 query rows, rounded up to 4, 8 or 12 warps.
template <bool kPrefill>
static int launch_attention(const AttnParams& P, int num_groups, int group_tokens,
                            cudaStream_t s) {
  const int warps = (group_tokens * P.num_heads + 15) / 16;
  dim3 grid(P.num_splits, num_groups);
  if (warps <= 4)
    hca_attention_kernel<128, 64, 4, kPrefill><<<grid, 128, 0, s>>>(P);
  else if (warps <= 8)
    hca_attention_kernel<128, 64, 8, kPrefill><<<grid, 256, 0, s>>>(P);
  else
    hca_attention_kernel<128, 64, 12, kPrefill><<<grid, 384, 0, s>>>(P);
  if (P.num_splits > 1)
    hca_attention_combine_kernel<128, kPrefill><<<dim3(num_groups, (P.max_rows + 15) / 16), 256, 0, s>>>(P);
  return HCA_LAUNCH_STATUS();
}

extern "C" int hca_sparse_decode(void* out, int64_t out_stride_tok, int64_t out_stride_head,
                                 float* lse, const void* q, int64_t q_stride_tok,
                                 int64_t q_stride_head, int32_t num_tokens, int32_t num_heads,
                                 int32_t head_dim, int32_t rope_dim, const uint8_t* swa_cache,
                                 int32_t swa_page_size, int64_t swa_page_stride_bytes,
                                 const int32_t* swa_indices, int64_t swa_indices_stride,
                                 const int32_t* swa_lens, const uint8_t* comp_cache,
                                 int32_t comp_page_size, int64_t comp_page_stride_bytes,
                                 const int32_t* comp_indices, int64_t comp_indices_stride,
                                 const int32_t* comp_lens, const int32_t* group_starts,
                                 int32_t num_groups, int32_t max_group_tokens,
                                 float softmax_scale, const float* attn_sink, int32_t num_splits,
                                 void* workspace, int64_t workspace_bytes, void* stream) {
  if (!group_starts) {
    num_groups = num_tokens;
    max_group_tokens = 1;
  }
  HCA_CHECK_ARG(num_tokens >= 0 && num_groups >= 0 && num_splits >= 1 && num_splits <= 16 &&
                swa_page_size > 0);
  if (!attn_shape_ok(num_heads, head_dim, rope_dim, max_group_tokens)) return HCA_E_UNSUPPORTED;
  if (num_tokens == 0 || num_groups == 0) return HCA_OK;
  HCA_CHECK_ARG(out && q && swa_cache && swa_indices && swa_lens);
  HCA_CHECK_ARG(!comp_cache || (comp_indices && comp_lens && comp_page_size > 0));
  HCA_CHECK_ARG(swa_page_stride_bytes % 16 == 0 && (!comp_cache || comp_page_stride_bytes % 16 == 0));
  HCA_CHECK_ARG(q_stride_head % 2 == 0 && q_stride_tok % 2 == 0);
  // the split-K combine stores 16-byte vectors
  HCA_CHECK_ARG(out_stride_head % 8 == 0 && out_stride_tok % 8 == 0 &&
                reinterpret_cast<uintptr_t>(out) % 16 == 0);
  AttnParams P{};
  P.q = static_cast<const __nv_bfloat16*>(q);
  P.q_st = q_stride_tok;
  P.q_sh = q_stride_head;
  P.out = static_cast<__nv_bfloat16*>(out);
  P.o_st = out_stride_tok;
  P.o_sh = out_stride_head;
  P.lse = lse;
  P.num_heads = num_heads;
  P.rope_dim = rope_dim;
  P.swa_cache = swa_cache;
  P.swa_page = swa_page_size;
  P.swa_pstride = swa_page_stride_bytes;
  P.comp_cache = comp_cache;
  P.comp_page = comp_page_size > 0 ? comp_page_size : 1;
  P.comp_pstride = comp_page_stride_bytes;
  P.swa_idx = swa_indices;
  P.swa_idx_st = swa_indices_stride;
  P.swa_lens = swa_lens;
  P.comp_idx = comp_indices;
  P.comp_idx_st = comp_indices_stride;
  P.comp_lens = comp_lens;
  P.group_starts = group_starts;
  P.scale_log2 = softmax_scale * kLog2e;
  P.sink = attn_sink;
  P.num_splits = num_splits;
  P.max_rows = max_group_tokens * num_heads;
  if (num_splits > 1) {
    const int64_t need = hca_sparse_decode_workspace_bytes(num_groups, max_group_tokens, num_heads,
                                                           head_dim, num_splits);
    if (!workspace || workspace_bytes < need) return HCA_E_WORKSPACE;
    const int64_t rows = static_cast<int64_t>(max_group_tokens) * num_heads;
    const int64_t o = align_up(static_cast<int64_t>(num_groups) * num_splits * rows * head_dim * 4, 256);
    const int64_t ml = align_up(static_cast<int64_t>(num_groups) * num_splits * rows * 2 * 4, 256);
    (void)ml;
    char* w = static_cast<char*>(workspace);
    P.ws_o = reinterpret_cast<float*>(w);
    P.ws_ml = reinterpret_cast<float*>(w + o);
  }
  return launch_attention<false>(P, num_groups, max_group_tokens, as_stream(stream));
}

extern "C" int hca_sparse_prefill(void* out, int64_t out_stride_tok, int64_t out_stride_head,
                                  const void* q, int64_t q_stride_tok, int64_t q_stride_head,
                                  int32_t num_heads, int32_t head_dim, int32_t rope_dim,
                                  const int32_t* query_start_loc, const int32_t* seq_lens,
                                  int32_t num_reqs, int32_t num_tokens, const uint8_t* swa_cache,
                                  int32_t swa_page_size, int64_t swa_page_stride_bytes,
                                  const int32_t* swa_block_table, int64_t swa_bt_stride,
                                  const uint8_t* comp_cache, int32_t comp_page_size,
                                  int64_t comp_page_stride_bytes,
                                  const int32_t* comp_block_table, int64_t comp_bt_stride,
                                  int32_t window, int32_t compress_ratio, float softmax_scale,
                                  const float* attn_sink, void* stream) {
  HCA_CHECK_ARG(num_reqs >= 0 && num_tokens >= 0 && swa_page_size > 0 && window > 0 &&
                compress_ratio > 0);
  const int group_tokens = num_heads > 0 ? (kMaxWarps * 16) / num_heads : 0;
  if (group_tokens < 1 || !attn_shape_ok(num_heads, head_dim, rope_dim, group_tokens))
    return HCA_E_UNSUPPORTED;
  if (num_reqs == 0 || num_tokens == 0) return HCA_OK;
  HCA_CHECK_ARG(out && q && query_start_loc && seq_lens && swa_cache && swa_block_table);
  HCA_CHECK_ARG(!comp_cache || (comp_block_table && comp_page_size > 0));
  HCA_CHECK_ARG(swa_page_stride_bytes % 16 == 0 && (!comp_cache || comp_page_stride_bytes % 16 == 0));
  AttnParams P{};
  P.q = static_cast<const __nv_bfloat16*>(q);
  P.q_st = q_stride_tok;
  P.q_sh = q_stride_head;
  P.out = static_cast<__nv_bfloat16*>(out);
  P.o_st = out_stride_tok;
  P.o_sh = out_stride_head;
  P.num_heads = num_heads;
  P.rope_dim = rope_dim;
  P.swa_cache = swa_cache;
  P.swa_page = swa_page_size;
  P.swa_pstride = swa_page_stride_bytes;
  P.comp_cache = comp_cache;
  P.comp_page = comp_page_size > 0 ? comp_page_size : 1;
  P.comp_pstride = comp_page_stride_bytes;
  P.qsl = query_start_loc;
  P.seq_lens = seq_lens;
  P.num_reqs = num_reqs;
  P.swa_bt = swa_block_table;
  P.swa_bt_st = swa_bt_stride;
  P.comp_bt = comp_block_table;
  P.comp_bt_st = comp_bt_stride;
  P.window = window;
  P.ratio = compress_ratio;
  P.group_tokens = group_tokens;
  P.max_rows = group_tokens * num_heads;
  P.scale_log2 = softmax_scale * kLog2e;
  P.sink = attn_sink;
  P.num_splits = 1;
  // tiles never straddle requests: at most tokens / G + requests of them
  const int num_tiles = num_tokens / group_tokens + num_reqs;
  return launch_attention<true>(P, num_tiles, group_tokens, as_stream(stream));
}
