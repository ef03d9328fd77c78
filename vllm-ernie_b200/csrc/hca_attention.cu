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
#include <atomic>

#include "hca_attention.cuh"
#include "hca_common.cuh"
#include "hca_tc.cuh"

namespace hca {
namespace {

constexpr int kChunk = 64;     // KV rows per pipeline step
constexpr int kMaxWarps = 12;  // 192 query rows per CTA

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
  pdl_wait_and_release();
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
  // the group's partials: S consecutive workspace slots from gbase
  int S = P.num_splits;
  int64_t first = static_cast<int64_t>(gidx) * S;
  if (!kPrefill && P.sched) {
    first = P.sched[4 * P.sched_items + 2 * gidx];
    S = P.sched[4 * P.sched_items + 2 * gidx + 1];
    if (S <= 1) return;  // its only CTA wrote the output itself
  }
  const int r0 = blockIdx.y * 16;
  if (r0 >= rows_q) return;
  const int64_t gbase = first * P.max_rows;
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
      const int64_t e0 = (gbase + static_cast<int64_t>(sp) * P.max_rows + r) * D + seg * 8;
      float4 a, b;
      if (P.bf16_partials) {
        // bf16 partial rows: the 8 dims in one 16-byte load
        const uint4 u = __ldcg(reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(P.ws_o) + e0));
        a = make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u), __uint_as_float(u.y << 16),
                        __uint_as_float(u.y & 0xffff0000u));
        b = make_float4(__uint_as_float(u.z << 16), __uint_as_float(u.z & 0xffff0000u), __uint_as_float(u.w << 16),
                        __uint_as_float(u.w & 0xffff0000u));
      } else {
        const float4* src = reinterpret_cast<const float4*>(P.ws_o + e0);
        a = __ldcg(src);
        b = __ldcg(src + 1);
      }
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

// ============================================================================
// Output path of a decode layer at head_dim 128: split-K merge, VHA mix
// (I + V U^T over heads, mma.sync), inverse GPT-J RoPE at the query position
// and the FP8 / UE8M0 quant of wo_a's input, one token per CTA
// (hca_combine_vha_quant_kernel).
// ============================================================================
struct VhaOut {
  uint8_t* out;          // [n_groups][tokens][hpg * D] e4m3
  int32_t* scale;        // [n_groups * hpg][aligned tokens] UE8M0 exponent bytes
  const __nv_bfloat16* mix;  // [H][H] bf16, I + V U^T
  const int64_t* positions;
  const float* cos_sin;
  int64_t cs_stride;
  int num_tokens, aligned_t, n_groups, num_groups;
};

namespace vt {
constexpr int D = 128, kMaxH = 64, kMixStride = kMaxH + 8, kOStride = D + 8, kMaxSplits = 16;
struct Smem {
  __nv_bfloat16 mix[kMaxH * kMixStride];
  __nv_bfloat16 o[kMaxH * kOStride];  // one token's merged rows, bf16
  float cs[64];                       // the token's cos | sin
  float amax[2][kMaxH];
  float w[kMaxH][kMaxSplits];         // split weights 2^(m_split - m)
  float inv[kMaxH];                   // 1 / (sum l + sink)
};
}  // namespace vt

// The mix into shared memory (all threads; a barrier follows before use).
__device__ __forceinline__ void vha_load_mix(const VhaOut& V, int H, vt::Smem& sm) {
  for (int i = threadIdx.x; i < H * (H / 8); i += blockDim.x) {
    const int r = i / (H / 8), c8 = i % (H / 8);
    *reinterpret_cast<uint4*>(&sm.mix[r * vt::kMixStride + c8 * 8]) =
        *reinterpret_cast<const uint4*>(V.mix + static_cast<int64_t>(r) * H + c8 * 8);
  }
}

// Merge token t's S split partials (workspace slots first .. first + S - 1 of
// the group whose first token is t0) into normalised bf16 rows in sm.o.
// Whole block; ends with a barrier.  Items (head, 16-dim segment) are spread
// over the threads; per item the splits are added two at a time, the first
// pair requested before the split weights are formed.
__device__ __forceinline__ void vha_merge_token(const AttnParams& P, int t, int t0, int first, int S, vt::Smem& sm) {
  using namespace vt;
  const int H = P.num_heads;
  const int lane = threadIdx.x & 31;
  (void)lane;
  const int64_t row0 = static_cast<int64_t>(first) * P.max_rows + static_cast<int64_t>(t - t0) * H;
  const int nitems = H * 8;
  // the partials are bf16 (the fused path's attention launch writes them
  // so): four splits' 16 dims (2 x 16 bytes each) in flight per round
  const __nv_bfloat16* ob = reinterpret_cast<const __nv_bfloat16*>(P.ws_o);
  const int64_t b_step = static_cast<int64_t>(P.max_rows) * D / 8;  // uint4s between splits
  uint4 vb[4][2];
  auto load_round = [&](int it, int sp) {
    const int h = it >> 3, seg = it & 7;
    const uint4* bp = reinterpret_cast<const uint4*>(ob + (row0 + h) * D + seg * 16);
#pragma unroll
    for (int k = 0; k < 4; ++k)
#pragma unroll
      for (int q = 0; q < 2; ++q)
        vb[k][q] = (it < nitems && sp + k < S) ? __ldcg(bp + (sp + k) * b_step + q) : make_uint4(0, 0, 0, 0);
  };
  // the first round of splits of this thread's first item
  load_round(threadIdx.x, 0);
  // split weights: thread (head, split) pairs, two per thread in flight;
  // H * kMaxSplits is a multiple of 256, so validity is uniform per warp
  for (int base = 0; base < H * kMaxSplits; base += 2 * blockDim.x) {
    float2 mlv[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int i = base + k * blockDim.x + threadIdx.x;
      const int hh = i / kMaxSplits, sp = i % kMaxSplits;
      mlv[k] = (i < H * kMaxSplits && sp < S)
                   ? __ldcg(reinterpret_cast<const float2*>(P.ws_ml + (row0 + static_cast<int64_t>(sp) * P.max_rows + hh) * 2))
                   : make_float2(-INFINITY, 0.0f);
    }
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int i = base + k * blockDim.x + threadIdx.x;
      if (i >= H * kMaxSplits) break;
      const int hh = i / kMaxSplits, sp = i % kMaxSplits;
      const float m = mlv[k].x, l = mlv[k].y;
      float mx = l > 0.0f ? m : -INFINITY;
#pragma unroll
      for (int o = kMaxSplits / 2; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float bse = mx == -INFINITY ? 0.0f : mx;
      // an empty split's row was never written: weight 0
      const float wt = l > 0.0f ? exp2f(m - bse) : 0.0f;
      float lw = l > 0.0f ? l * wt : 0.0f;
#pragma unroll
      for (int o = kMaxSplits / 2; o > 0; o >>= 1) lw += __shfl_xor_sync(0xffffffffu, lw, o);
      sm.w[hh][sp] = wt;
      if (sp == 0) {
        const float sink2 = P.sink ? P.sink[hh] * kLog2e : -INFINITY;
        sm.inv[hh] = lw > 0.0f ? 1.0f / (lw + exp2f(sink2 - bse)) : 0.0f;
      }
    }
  }
  __syncthreads();
  for (int it = threadIdx.x; it < nitems; it += blockDim.x) {
    const int h = it >> 3, seg = it & 7;
    float acc[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) acc[e] = 0.0f;
    for (int sp = 0; sp < S; sp += 4) {
      if (sp > 0 || it != threadIdx.x) load_round(it, sp);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float wt = sp + k < S ? sm.w[h][sp + k] : 0.0f;
        if (wt == 0.0f) continue;  // an empty split's row was never written
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const uint32_t w4[4] = {vb[k][q].x, vb[k][q].y, vb[k][q].z, vb[k][q].w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            acc[8 * q + 2 * e] += wt * __uint_as_float(w4[e] << 16);
            acc[8 * q + 2 * e + 1] += wt * __uint_as_float(w4[e] & 0xffff0000u);
          }
        }
      }
    }
    const float inv = sm.inv[h];
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      uint4 pk;
      pk.x = pack_bf16(acc[8 * q] * inv, acc[8 * q + 1] * inv);
      pk.y = pack_bf16(acc[8 * q + 2] * inv, acc[8 * q + 3] * inv);
      pk.z = pack_bf16(acc[8 * q + 4] * inv, acc[8 * q + 5] * inv);
      pk.w = pack_bf16(acc[8 * q + 6] * inv, acc[8 * q + 7] * inv);
      *reinterpret_cast<uint4*>(&sm.o[h * kOStride + seg * 16 + q * 8]) = pk;
    }
  }
  __syncthreads();
}

// Mix, inverse RoPE and quantise token t's rows (sm.o, sm.mix and sm.cs
// ready) and store the e4m3 row and UE8M0 scales.  Warps 0-7 compute (warp
// = 16 heads x 64 dims); every thread of the block calls it (one barrier).
__device__ __forceinline__ void vha_mix_quant_token(const AttnParams& P, const VhaOut& V, int t, vt::Smem& sm) {
  using namespace vt;
  const int H = P.num_heads;
  const int hpg = H / V.n_groups;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int ht = warp & 3, dh = (warp >> 2) & 1;
  const int gq = lane >> 2, cq = lane & 3;
  const int h0 = ht * 16 + gq, h1 = h0 + 8;
  const bool active = warp < 8 && ht * 16 < H;
  float acc[8][4];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.0f;
  if (active) {
    for (int kk = 0; kk < H / 16; ++kk) {
      uint32_t a[4];
      ldmatrix_x4(a, &sm.mix[(ht * 16 + (lane & 15)) * kMixStride + kk * 16 + (lane >> 4) * 8]);
#pragma unroll
      for (int j = 0; j < 8; j += 2) {
        uint32_t b[4];
        ldmatrix_x4_trans(b, &sm.o[(kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8) * kOStride + dh * 64 + j * 8 +
                                   (lane >> 4) * 8]);
        mma16816(acc[j], a, b);
        mma16816(acc[j + 1], a, b + 2);
      }
    }
    // inverse GPT-J RoPE on the dims >= nope
    const int nope = D - P.rope_dim;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int d = dh * 64 + j * 8 + 2 * cq;
      if (d >= nope) {
        const int pr = (d - nope) >> 1;
        const float c = sm.cs[pr], sn = sm.cs[P.rope_dim / 2 + pr];
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const float e = acc[j][2 * hh], od = acc[j][2 * hh + 1];
          acc[j][2 * hh] = e * c + od * sn;
          acc[j][2 * hh + 1] = od * c - e * sn;
        }
      }
    }
    float am0 = 0.0f, am1 = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      am0 = fmaxf(am0, fmaxf(fabsf(acc[j][0]), fabsf(acc[j][1])));
      am1 = fmaxf(am1, fmaxf(fabsf(acc[j][2]), fabsf(acc[j][3])));
    }
#pragma unroll
    for (int off = 1; off < 4; off <<= 1) {
      am0 = fmaxf(am0, __shfl_xor_sync(0xffffffffu, am0, off));
      am1 = fmaxf(am1, __shfl_xor_sync(0xffffffffu, am1, off));
    }
    if (cq == 0) {
      sm.amax[dh][h0] = am0;
      sm.amax[dh][h1] = am1;
    }
  }
  __syncthreads();
  if (!active) return;
  // ---- quantise: one UE8M0 scale per (head, 128 dims) ----
  const float a0 = fmaxf(sm.amax[0][h0], sm.amax[1][h0]), a1 = fmaxf(sm.amax[0][h1], sm.amax[1][h1]);
  const int e0 = ue8m0_exponent(a0, 1e-10f, false), e1 = ue8m0_exponent(a1, 1e-10f, false);
  const float i0 = exp2i(-e0), i1 = exp2i(-e1);
  uint8_t* r0 = V.out + (static_cast<int64_t>(h0 / hpg) * V.num_tokens + t) * (hpg * D) + (h0 % hpg) * D;
  uint8_t* r1 = V.out + (static_cast<int64_t>(h1 / hpg) * V.num_tokens + t) * (hpg * D) + (h1 % hpg) * D;
  uint32_t p0[8], p1[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    p0[j] = to_e4m3(acc[j][0] * i0) | (to_e4m3(acc[j][1] * i0) << 8);
    p1[j] = to_e4m3(acc[j][2] * i1) | (to_e4m3(acc[j][3] * i1) << 8);
  }
  // 16 contiguous bytes per lane: one full-sector store instead of eight 2-byte ones
  *reinterpret_cast<uint4*>(r0 + dh * 64 + 16 * cq) = quad_gather_fp8(p0, cq);
  *reinterpret_cast<uint4*>(r1 + dh * 64 + 16 * cq) = quad_gather_fp8(p1, cq);
  if (dh == 0 && cq == 0) {
    V.scale[static_cast<int64_t>(h0) * V.aligned_t + t] = static_cast<int32_t>(encode_ue8m0(e0));
    V.scale[static_cast<int64_t>(h1) * V.aligned_t + t] = static_cast<int32_t>(encode_ue8m0(e1));
  }
}

// ============================================================================
// tcgen05 decode kernel (head_dim 128 = 64 e4m3 NoPE + 64 bf16 RoPE)
//
// One CTA per (group, split); up to 256 query rows = two M=128 tiles.
//   warps 0-7  softmax: tile t = warp / 4, TMEM lane quadrant = warp % 4,
//              one thread per query row (S row read from TMEM, P written back)
//   warp  8    MMA issuer (lane 0) + TMEM owner
//   warps 9-12 producers: each owns 16 of the 64 KV rows of every chunk.  It
//              resolves their slots from the index tables, gathers the rows
//              with 16-byte cp.async into its slice of a kStages-deep raw ring
//              (kStages - 1 chunks in flight, completion by cp.async groups),
//              then dequantises them (e4m3 x UE8M0 -> bf16, RoPE half copied)
//              into the 128B-swizzled K tile.  A random-row gather is bound by
//              the requests one SM keeps in flight, so four warps issue them.
// S = Q K^T: M=128, N=64, K=128 (8 x K16), Q and K tile K-major in smem.
// O += P V: M=128, N=128, K=64 (4 x K16), P from TMEM, V = the same K tile
// read MN-major.  TMEM: O tiles at columns 0 / 128, S/P double-buffered at
// 256 + (tile * 2 + buf) * 64.  Softmax runs in base 2 with the row max
// raised lazily (O is rescaled only when the max grows by more than 2^8).
// Every mbarrier wait is bounded; a timeout sets the device error word.
// ============================================================================
namespace tcd {
constexpr int kD = 128;
constexpr int kNope = 64;
constexpr int kRowBytes = 192;  // kNope e4m3 + 64 bf16
constexpr int kCh = 64;         // KV rows per step
// raw gather ring: one chunk in flight while the previous one is dequantised.
// Deeper rings start every CTA with a larger burst of gathers (all CTAs
// reach their first chunk at once), which delays the first chunk more than
// the extra prefetch helps: a chunk's MMAs and softmax outlast its gather.
constexpr int kStages = 2;
constexpr int kSoftmaxWarps = 8;
constexpr int kMmaWarp = 8;
constexpr int kProdWarp0 = 9;
constexpr int kProdWarps = 4;
constexpr int kProdRows = kCh / kProdWarps;  // 16 rows of each chunk per producer warp
constexpr int kThreads = (kProdWarp0 + kProdWarps) * 32;
constexpr int kMaxRows = 256;
constexpr int kQTile = 2 * 128 * 128;          // two 64-column regions of 128 rows x 128 B
constexpr int kQRegion = 128 * 128;
constexpr int kQOff = 0;
constexpr int kKBufs = 4;                      // bf16 K-tile ring: dequant runs ahead of the MMAs
constexpr int kKOff = kQOff + 2 * kQTile;      // 65536
constexpr int kKRegion = kCh * 128;            // 8192
constexpr int kKBuf = 2 * kKRegion;            // 16384
constexpr int kRawOff = kKOff + kKBufs * kKBuf;
// raw stage: e4m3 NoPE [64][64] | bf16 RoPE [64][128] | 16-byte scale blocks [64][16]
constexpr int kRawNope = 0;
constexpr int kRawRope = kCh * kNope;
constexpr int kRawSblk = kRawRope + kCh * 128;
constexpr int kRawStage = kRawSblk + kCh * 16;  // 13312
constexpr int kScaleOff = kRawOff + kStages * kRawStage;  // [stage][row] byte index of the scale in its block
constexpr int kMaskOff = kScaleOff + kStages * kCh;       // [stage][row] token mask | kOkBit
constexpr int kKMaskOff = kMaskOff + kStages * kCh * 4;   // [kbuf][token][4] 16-bit column masks
constexpr int kBarOff = kKMaskOff + kKBufs * kCh * 4;
// k_full[kKBufs] k_empty[kKBufs] s_full[2] p_full[2] pv_done[2] q_full
constexpr int kNumBars = 2 * kKBufs + 7;
constexpr int kMiscOff = kBarOff + kNumBars * 8;
constexpr int kTokOff = kMiscOff + 64;  // [32] + [32] ints
constexpr int kSmemBytes = kTokOff + 256 + 1024;  // + 1024 alignment slack
constexpr int kQWarps = 9;  // softmax warps + MMA warp load Q
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kOkBit = 1u << 31;

__device__ __forceinline__ uint32_t s_col(int tile, int buf) { return 256u + (tile * 2 + buf) * 64u; }

// Query row held by TMEM lane / smem row `rit` of M-tile `tile`, or -1: a
// tile with R valid rows puts q = ceil(R / 4) of them at the start of each
// 32-lane quadrant.
__device__ __forceinline__ int tile_row_to_query(int tile, int rit, int rows_q) {
  const int R = min(128, rows_q - tile * 128);
  if (R <= 0) return -1;
  const int q = (R + 3) >> 2;
  const int quad = rit >> 5, ln = rit & 31;
  const int local = quad * q + ln;
  return (ln < q && local < R) ? tile * 128 + local : -1;
}

// Lane quadrants (softmax warps) of M-tile `tile` that hold query rows.
__device__ __forceinline__ int active_quads(int tile, int rows_q) {
  const int R = min(128, rows_q - tile * 128);
  if (R <= 0) return 0;
  const int q = (R + 3) >> 2;
  return (R + q - 1) / q;
}

__device__ __forceinline__ void report(int* err, uint32_t* s_err, int code) {
  *s_err = 1;
  if (err) atomicOr(err, code);
}
}  // namespace tcd

template <bool kPrefill>
__global__ void __launch_bounds__(tcd::kThreads, 1) hca_tc_attention_kernel(const AttnParams P, int* err) {
  // Everything up to pdl_wait() reads only per-step metadata (schedule,
  // group starts, lengths, index and block tables), written before any layer
  // kernel ran, so it overlaps the kernel before this one; Q and the cache
  // rows, which that kernel may still be writing, are read after the wait.
  // CTAs that exit early wait first, so this launch completes only after its
  // predecessor.
  pdl_release();
  using namespace tcd;
  using namespace tc;
  extern __shared__ uint8_t smem_dyn[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
  const uint64_t wait_ns = P.wait_ns;

  // this CTA's work: a (group, chunk range) from the schedule, or split
  // blockIdx.x of group blockIdx.y; `item` numbers its partial in the workspace.
  // Prefill: tile blockIdx.x of the requests' tokens, all of its rows.
  int gidx, c_begin = 0, c_end = 1 << 30;
  int64_t item;
  bool single;  // the group has no other CTA: write the final output directly
  if (kPrefill) {
    gidx = blockIdx.x;
    item = gidx;
    single = true;
  } else if (P.sched) {
    const int4 it = reinterpret_cast<const int4*>(P.sched)[blockIdx.x];
    if (it.x < 0) {
      pdl_wait();
      return;
    }
    gidx = it.x;
    c_begin = it.z;
    c_end = it.w;
    item = blockIdx.x;
    single = P.sched[4 * P.sched_items + 2 * gidx + 1] == 1;
  } else {
    gidx = blockIdx.y;
    item = static_cast<int64_t>(gidx) * P.num_splits + blockIdx.x;
    single = P.num_splits == 1;
  }
  if (P.force_partials) single = false;
  Group G;
  if (!resolve_group<kPrefill>(P, gidx, G) || G.ntok * P.num_heads > kMaxRows ||
      G.ntok * P.num_heads > P.max_rows || G.ntok > 31) {  // 31 token mask bits (bit 31: loaded)
    pdl_wait();
    return;
  }
  const int H = P.num_heads;
  const int rows_q = G.ntok * H;
  const int ntiles = (rows_q + 127) / 128;
  // softmax warps with rows: quadrants 0 .. act0 - 1 of tile 0, 0 .. act1 - 1 of tile 1
  const int act0 = active_quads(0, rows_q), act1 = active_quads(1, rows_q);
  const int nact = act0 + act1;
  const int n_u = G.n_win + G.n_comp;
  const int nchunks = (n_u + kCh - 1) / kCh;
  if (!kPrefill && !P.sched) {
    const int split = blockIdx.x;
    c_begin = static_cast<int>((static_cast<int64_t>(split) * nchunks) / P.num_splits);
    c_end = static_cast<int>((static_cast<int64_t>(split + 1) * nchunks) / P.num_splits);
  }
  if (c_end > nchunks) c_end = nchunks;
  if (c_begin > c_end) c_begin = c_end;
  const int n = c_end - c_begin;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kBarOff);
  uint64_t* k_full = bars;
  uint64_t* k_empty = k_full + kKBufs;
  uint64_t* s_full = k_empty + kKBufs;
  uint64_t* p_full = s_full + 2;
  uint64_t* pv_done = p_full + 2;
  uint64_t* q_full = pv_done + 2;
  uint32_t* misc = reinterpret_cast<uint32_t*>(smem + kMiscOff);  // [0] tmem, [1] err
  uint8_t* scale_s = smem + kScaleOff;
  uint32_t* mask_s = reinterpret_cast<uint32_t*>(smem + kMaskOff);
  uint32_t* kmask = reinterpret_cast<uint32_t*>(smem + kKMaskOff);

  int* tok_len = reinterpret_cast<int*>(smem + kTokOff);  // [32] window length per token
  int* tok_clen = tok_len + 32;                             // [32] compressed length per token

  if (warp == kMmaWarp) {
    tmem_alloc(misc, kTmemCols);
    tmem_relinquish();
    tc_fence_before();
  }
  if (threadIdx.x == 0) {
    for (int b = 0; b < kKBufs; ++b) {
      mbar_init(k_full + b, kProdWarps);
      mbar_init(k_empty + b, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(s_full + b, 1);
      mbar_init(p_full + b, nact);  // one arrival per softmax warp with rows
      mbar_init(pv_done + b, 1);
    }
    mbar_init(q_full, kQWarps * 32 + kQWarps);  // per-thread cp.async completions + one arrival per warp
    misc[1] = 0;
    mbar_fence_init();
  }
  if (!kPrefill && threadIdx.x < G.ntok) {
    tok_len[threadIdx.x] = P.swa_lens[G.t0 + threadIdx.x];
    tok_clen[threadIdx.x] = P.comp_cache ? P.comp_lens[G.t0 + threadIdx.x] : 0;
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = misc[0];

  if (warp < kSoftmaxWarps || warp == kMmaWarp) {
    pdl_wait();  // Q was written by an earlier kernel of this layer
    // Q rows -> two K-major 128B-swizzled M=128 tiles (rows past rows_q zero),
    // loaded by the softmax and MMA warps while the loader already streams KV.
    // A tile with R < 128 query rows spreads them evenly over the four TMEM
    // lane quadrants (q = ceil(R / 4) rows each) so every SM sub-partition
    // runs the same softmax load.
    // Valid rows arrive by cp.async (all copies in flight at once, completion
    // counted on q_full); padding rows are zeroed with plain stores.
    const int qt = warp < kSoftmaxWarps ? threadIdx.x : kSoftmaxWarps * 32 + lane;
    for (int item = qt; item < ntiles * 128 * (kD / 8); item += kQWarps * 32) {
      const int row = item >> 4, ch = item & 15;
      const int tile = row >> 7, rit = row & 127, region = ch >> 3, c8 = ch & 7;
      const int r = tile_row_to_query(tile, rit, rows_q);
      uint8_t* dst = smem + kQOff + tile * kQTile + region * kQRegion + rit * 128 + ((c8 ^ (rit & 7)) << 4);
      if (r >= 0) {
        const int tok = G.t0 + r / H, h = r % H;
        cp_async16(dst, P.q + tok * P.q_st + h * P.q_sh + ch * 8);
      } else {
        *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
      }
    }
    cp_async_arrive_noinc(q_full);
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(q_full);
  }

  if (warp >= kProdWarp0) {
    // -------------------------------------------------------------- producer
    const int row0 = (warp - kProdWarp0) * kProdRows;  // this warp's rows of every chunk
    // Slot, token mask and cache of row row0 + lane (lanes < kProdRows) of
    // chunk c, from the index tables; the per-token lengths deciding the mask
    // are in shared memory.
    struct Resolved {
      int64_t slot;
      uint32_t mask;
      bool comp;
    };
    auto resolve = [&](int c, Resolved& R) {
      const int u = c * kCh + row0 + lane;
      R.slot = -1;
      R.mask = 0;
      R.comp = false;
      if (kPrefill) {
        // positions: window row u is position win_start + u, compressed row
        // u - n_win is entry u - n_win; slots through the block tables
        if (lane < kProdRows && u < n_u) {
          bool comp;
          int64_t slot;
          uint32_t m;
          row_source<true>(P, G, u, comp, slot, m);
          R.slot = slot;
          R.comp = comp;
          R.mask = m;
        }
      } else if (lane < kProdRows && u < n_u) {
        uint32_t m = 0;
        if (u < G.n_win) {
          R.slot = u < G.len0 ? P.swa_idx[G.first_tok * P.swa_idx_st + u]
                              : P.swa_idx[G.last_tok * P.swa_idx_st + (G.len_last - (G.n_win - u))];
          for (int k = 0; k < G.ntok; ++k) {
            const int lk = tok_len[k];
            if (lk > 0 && u >= k + G.len0 - lk && u <= k + G.len0 - 1) m |= 1u << k;
          }
        } else {
          const int ci = u - G.n_win;
          R.slot = P.comp_idx[G.last_tok * P.comp_idx_st + ci];
          R.comp = true;
          for (int k = 0; k < G.ntok; ++k)
            if (ci < tok_clen[k]) m |= 1u << k;
        }
        R.mask = m;
      }
    };
    // Gather this warp's rows of local chunk i into raw stage i % kStages and
    // close one cp.async group (an empty group past the last chunk keeps the
    // group count uniform).
    auto issue = [&](int i, const Resolved& R) {
      if (i < n) {
        const int s = i % kStages;
        uint8_t* const stage = smem + kRawOff + s * kRawStage;
        const int row = row0 + lane;
        // Row addresses in 32-bit slot arithmetic: a slot is below 2^31 in
        // any cache that fits in device memory (every row takes > 64 bytes).
        const bool ok = R.slot >= 0;
        uint64_t rbase = 0;
        if (ok) {
          const uint32_t sl = static_cast<uint32_t>(R.slot);
          const uint32_t psz = R.comp ? static_cast<uint32_t>(P.comp_page) : static_cast<uint32_t>(P.swa_page);
          const uint32_t page = sl / psz, off = sl - page * psz;
          const uint8_t* base =
              (R.comp ? P.comp_cache : P.swa_cache) + static_cast<int64_t>(page) * (R.comp ? P.comp_pstride : P.swa_pstride);
          rbase = reinterpret_cast<uint64_t>(base + off * kRowBytes);
          const uintptr_t sa = reinterpret_cast<uintptr_t>(base + psz * kRowBytes + off * (kNope / kQuantBlock + 1));
          cp_async16(stage + kRawSblk + row * 16, reinterpret_cast<const void*>(sa & ~uintptr_t(15)));
          scale_s[s * kCh + row] = static_cast<uint8_t>(sa & 15);
        }
        if (lane < kProdRows) mask_s[s * kCh + row] = ok ? (R.mask | kOkBit) : 0u;
        // 12 pieces of 16 bytes per row, consecutive lanes on consecutive
        // pieces (a cp.async instruction touches ~3 rows); pieces 0-3 are the
        // e4m3 NoPE bytes, 4-11 the bf16 RoPE half.
#pragma unroll
        for (int k = 0; k < kProdRows * (kRowBytes / 16) / 32; ++k) {
          const int piece = k * 32 + lane;
          const int r = piece / (kRowBytes / 16), j = piece - r * (kRowBytes / 16);
          const uint64_t src = __shfl_sync(0xffffffffu, rbase, r);
          uint8_t* dst = j < 4 ? stage + kRawNope + (row0 + r) * kNope + j * 16
                               : stage + kRawRope + (row0 + r) * 128 + (j - 4) * 16;
          if (src) cp_async16(dst, reinterpret_cast<const void*>(src + j * 16));
        }
      }
      cp_async_commit();
    };
    // prologue: the first kStages - 1 chunks (index loads first, all in flight)
    Resolved rq[kStages - 1];
#pragma unroll
    for (int i = 0; i < kStages - 1; ++i) {
      rq[i].slot = -1;
      if (i < n) resolve(c_begin + i, rq[i]);
    }
    pdl_wait();  // the cache rows: the kernel before may still be inserting
#pragma unroll
    for (int i = 0; i < kStages - 1; ++i) issue(i, rq[i]);
    Resolved rn;  // slots of the next chunk to issue
    rn.slot = -1;
    if (kStages - 1 < n) resolve(c_begin + kStages - 1, rn);
    for (int i = 0; i < n; ++i) {
      const int s = i % kStages, b = i % kKBufs;
      if (kPrefill && i == 0) {
        // prefill: chunk 0 lands before the next gathers go out (a tile's
        // CTA requests its Q tile and first rows at once, and the first S
        // needs only those: 3.50 -> 3.44 ms a config-3 layer).  Decode keeps
        // chunk 1 in flight: in the decode chain the delay cost more (33.7
        // -> 34.1 us a layer) than the smaller start-up burst saved.
        cp_async_wait_group<0>();
        issue(kStages - 1, rn);
        if (kStages < n) resolve(c_begin + kStages, rn);
      } else {
        issue(i + kStages - 1, rn);
        if (i + kStages < n) resolve(c_begin + i + kStages, rn);
        cp_async_wait_group<kStages - 1>();  // chunk i's group has landed
      }
      __syncwarp();
      if (i >= kKBufs && !mbar_wait(k_empty + b, ((i / kKBufs) - 1) & 1, wait_ns)) {
        report(err, misc + 1, 2);
        break;
      }
      const uint8_t* stage = smem + kRawOff + s * kRawStage;
      uint8_t* kt = smem + kKOff + b * kKBuf;
      // NoPE: lane -> row row0 + lane / 2, 32 e4m3 values (half lane & 1)
      {
        const int r = row0 + (lane >> 1), h = lane & 1;
        const uint32_t mask = mask_s[s * kCh + r];
        const bool ok = (mask & kOkBit) != 0;
        // rows that are not loaded must come out exactly zero: their smem
        // bytes are stale (a stale scale of 255 would be inf, 0 * inf = NaN)
        const float sc = ok ? exp2i(static_cast<int>(stage[kRawSblk + r * 16 + scale_s[s * kCh + r]]) - 127) : 0.0f;
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const uint4 in = ok ? *reinterpret_cast<const uint4*>(stage + kRawNope + r * kNope + h * 32 + q * 16)
                              : make_uint4(0, 0, 0, 0);
#pragma unroll
          for (int w2 = 0; w2 < 2; ++w2) {
            const uint32_t w0 = w2 ? in.z : in.x, w1 = w2 ? in.w : in.y;
            const float2 f0 = e4m3x2_to_float2(static_cast<uint16_t>(w0 & 0xffff));
            const float2 f1 = e4m3x2_to_float2(static_cast<uint16_t>(w0 >> 16));
            const float2 f2 = e4m3x2_to_float2(static_cast<uint16_t>(w1 & 0xffff));
            const float2 f3 = e4m3x2_to_float2(static_cast<uint16_t>(w1 >> 16));
            uint4 o;
            o.x = pack_bf16(f0.x * sc, f0.y * sc);
            o.y = pack_bf16(f1.x * sc, f1.y * sc);
            o.z = pack_bf16(f2.x * sc, f2.y * sc);
            o.w = pack_bf16(f3.x * sc, f3.y * sc);
            const int c8 = h * 4 + q * 2 + w2;  // 16-byte chunk of the 128-byte NoPE row
            *reinterpret_cast<uint4*>(kt + r * 128 + ((c8 ^ (r & 7)) << 4)) = o;
          }
        }
      }
      // RoPE half: 16 rows x 8 pieces, copied into K-tile region 1
#pragma unroll
      for (int k = 0; k < kProdRows * 8 / 32; ++k) {
        const int piece = k * 32 + lane;
        const int r = row0 + (piece >> 3), c8 = piece & 7;
        const bool ok = (mask_s[s * kCh + r] & kOkBit) != 0;
        const uint4 v = ok ? *reinterpret_cast<const uint4*>(stage + kRawRope + r * 128 + c8 * 16) : make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(kt + kKRegion + r * 128 + ((c8 ^ (r & 7)) << 4)) = v;
      }
      // per-token 16-bit column masks of these rows: halfword (k * 4 + warp
      // slice) of buffer b, so word k * 2 + hi covers KV rows hi * 32 .. + 31
      {
        const uint32_t mask = lane < kProdRows ? mask_s[s * kCh + row0 + lane] : 0u;
        uint16_t* km16 = reinterpret_cast<uint16_t*>(kmask + b * kCh);
        for (int k = 0; k < G.ntok; ++k) {
          const uint32_t bits = __ballot_sync(0xffffffffu, (mask >> k) & 1u);
          if (lane == 0) km16[k * 4 + (row0 / kProdRows)] = static_cast<uint16_t>(bits & 0xffffu);
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(k_full + b);
    }
    cp_async_wait_group<0>();  // no copy may still target shared memory at exit
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------------- MMA
    if (lane == 0) {
      const uint32_t idesc_s = umma_idesc_bf16(128, kCh, false, false);
      const uint32_t idesc_o = umma_idesc_bf16(128, kD, false, true);
      // shared-memory descriptors built once; a K step or buffer moves the
      // start-address field (bits 0-13, address / 16) by offset / 16
      const uint64_t dq = umma_desc_sw128(smem_u32(smem + kQOff), 16, 1024);
      const uint64_t dk = umma_desc_sw128(smem_u32(smem + kKOff), 16, 1024);
      const uint64_t dv = umma_desc_sw128(smem_u32(smem + kKOff), kKRegion, 1024);
      bool ok = mbar_wait(q_full, 0, wait_ns);
      // Q arrived through cp.async (generic proxy); the MMAs read it through
      // the async proxy
      fence_proxy_async_smem();
      auto issue_s = [&](int i) {
        const int kb = i % kKBufs, sb = i & 1;
        tc_fence_after();
        for (int t = 0; t < ntiles; ++t) {
#pragma unroll
          for (int kk = 0; kk < kD / 16; ++kk) {
            const uint32_t qo = (t * kQTile + (kk >> 2) * kQRegion + (kk & 3) * 32) >> 4;
            const uint32_t ko = (kb * kKBuf + (kk >> 2) * kKRegion + (kk & 3) * 32) >> 4;
            umma_ss(tmem + s_col(t, sb), dq + qo, dk + ko, idesc_s, kk > 0 ? 1u : 0u);
          }
        }
        umma_commit(s_full + sb);
      };
      auto issue_pv = [&](int i) {
        const int kb = i % kKBufs, sb = i & 1;
        tc_fence_after();
        for (int t = 0; t < ntiles; ++t) {
#pragma unroll
          for (int kk = 0; kk < kCh / 16; ++kk)
            umma_ts(tmem + t * 128, tmem + s_col(t, sb) + kk * 8, dv + ((kb * kKBuf + kk * 2048) >> 4), idesc_o,
                    (i > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(k_empty + kb);
        umma_commit(pv_done + sb);
      };
      // Issue order S(0), then per chunk S(i + 1) -- as soon as its K tile is
      // ready, so softmax finds the next S waiting -- and P.V(i) once softmax
      // has written P(i).  S(i + 1) reuses the TMEM buffer of chunk i - 1,
      // whose P.V is already issued.  The waits suspend the thread (no
      // polling that would take issue slots from the softmax warps) and are
      // bounded: an error after kWaitLimitNs.
      if (ok && n > 0) {
        ok = mbar_wait(k_full, 0, wait_ns);
        if (ok) issue_s(0);
      }
      for (int i = 0; ok && i < n; ++i) {
        if (i + 1 < n) {
          ok = mbar_wait(k_full + (i + 1) % kKBufs, ((i + 1) / kKBufs) & 1, wait_ns);
          if (!ok) break;
          issue_s(i + 1);
        }
        ok = mbar_wait(p_full + (i & 1), (i >> 1) & 1, wait_ns);
        if (!ok) break;
        issue_pv(i);
      }
      if (!ok) report(err, misc + 1, 4);
    }
    __syncwarp();
  } else {
    // --------------------------------------------------------------- softmax
    // one thread per query row: its S row lives in TMEM lane `rit` of tile t
    const int t = warp >> 2, quad = warp & 3;
    const int rit = quad * 32 + lane;
    const int r = tile_row_to_query(t, rit, rows_q);
    const bool row_valid = r >= 0;
    const bool warp_active = __any_sync(0xffffffffu, row_valid);
    const int tok = row_valid ? r / H : 0;
    const int head = row_valid ? r % H : 0;
    const uint32_t lane_addr = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t o_col = static_cast<uint32_t>(t) * 128u;
    const float scale = P.scale_log2;
    float m_used = -INFINITY, l = 0.0f;
    bool ok = true;
    if (warp_active) {
      for (int i = 0; i < n; ++i) {
        const int b = i & 1, kb = i % kKBufs;
        if (!mbar_wait(s_full + b, (i >> 1) & 1, wait_ns) || !mbar_wait(k_full + kb, (i / kKBufs) & 1, wait_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // valid columns of this row's token: bit j of lo / hi = KV row j / 32 + j
        const uint32_t lo = row_valid ? kmask[kb * kCh + tok * 2] : 0u;
        const uint32_t hi = row_valid ? kmask[kb * kCh + tok * 2 + 1] : 0u;
        const bool full = (lo & hi) == 0xffffffffu;
        const uint32_t s_addr = tmem + lane_addr + s_col(t, b);
        uint32_t sr[kCh];
        tmem_ld32(s_addr, sr);
        tmem_ld32(s_addr + 32, sr + 32);
        tmem_wait_ld();
        // masked columns become -inf: they drop out of the max and 2^-inf = 0
        if (!full) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            sr[j] = ((lo >> j) & 1u) ? sr[j] : 0xff800000u;
            sr[32 + j] = ((hi >> j) & 1u) ? sr[32 + j] : 0xff800000u;
          }
        }
        // row max as a tree of 3-input maxima (short dependency chains)
        float m8[8];
#pragma unroll
        for (int k = 0; k < 8; ++k)
          m8[k] = fmax3(__uint_as_float(sr[k]), __uint_as_float(sr[k + 8]), __uint_as_float(sr[k + 16]));
#pragma unroll
        for (int k = 0; k < 8; ++k) m8[k] = fmax3(m8[k], __uint_as_float(sr[k + 24]), __uint_as_float(sr[k + 32]));
#pragma unroll
        for (int k = 0; k < 8; ++k) m8[k] = fmax3(m8[k], __uint_as_float(sr[k + 40]), __uint_as_float(sr[k + 48]));
#pragma unroll
        for (int k = 0; k < 8; ++k) m8[k] = fmaxf(m8[k], __uint_as_float(sr[k + 56]));
        float mx = fmax3(fmax3(m8[0], m8[1], m8[2]), fmax3(m8[3], m8[4], m8[5]), fmaxf(m8[6], m8[7]));
        mx *= scale;  // scale > 0 commutes with the max
        // raise the running max lazily: only when it grows by more than 2^8
        const bool need = mx > m_used + 8.0f;
        const bool rescale = __any_sync(0xffffffffu, need);
        float f = 1.0f;
        if (rescale) {
          const float new_m = fmaxf(m_used, mx);
          f = m_used == -INFINITY ? 0.0f : exp2f(m_used - new_m);
          l *= f;
          m_used = new_m;
        }
        // P = 2^(s * scale - m) as bf16 pairs; exponents by packed FMAs,
        // row sum in four packed accumulators
        const float nb = m_used == -INFINITY ? 0.0f : -m_used;
        const float2 sc2 = make_float2(scale, scale), nb2 = make_float2(nb, nb);
        float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          uint32_t pk[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float2 x = fma2(make_float2(__uint_as_float(sr[hh * 32 + 2 * j]), __uint_as_float(sr[hh * 32 + 2 * j + 1])),
                                  sc2, nb2);
            const float2 p2 = make_float2(ex2_approx(x.x), ex2_approx(x.y));
            acc[j & 3] = add2(acc[j & 3], p2);
            pk[j] = pack_bf16(p2.x, p2.y);
          }
          tmem_st16(s_addr + hh * 16, pk);
        }
        const float2 a01 = add2(add2(acc[0], acc[1]), add2(acc[2], acc[3]));
        const float rs = a01.x + a01.y;
        l += rs;
        if (rescale && i > 0) {
          // O holds chunks < i at the old max: wait for PV(i-1), then scale it
          if (!mbar_wait(pv_done + ((i - 1) & 1), ((i - 1) >> 1) & 1, wait_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll 1
          for (int q4 = 0; q4 < kD / 32; ++q4) {
            uint32_t o[32];
            tmem_ld32(tmem + lane_addr + o_col + q4 * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * f);
            tmem_st32(tmem + lane_addr + o_col + q4 * 32, o);
          }
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(p_full + b);
      }
      if (ok && n > 0) {
        if (!mbar_wait(pv_done + ((n - 1) & 1), ((n - 1) >> 1) & 1, wait_ns)) ok = false;
        tc_fence_after();
      }
      if (!ok) report(err, misc + 1, 8);
      // ---- epilogue: normalise (single split) or write the partial ----
      const bool have_o = ok && n > 0 && l > 0.0f;
      if (single) {
        const float sink2 = (P.sink && row_valid) ? P.sink[head] * kLog2e : -INFINITY;
        const float inv = have_o ? 1.0f / (l + exp2f(sink2 - m_used)) : 0.0f;
        __nv_bfloat16* orow = P.out + (G.t0 + tok) * P.o_st + head * P.o_sh;
#pragma unroll 1
        for (int q4 = 0; q4 < kD / 32; ++q4) {
          uint32_t o[32];
          if (ok && n > 0) {
            tmem_ld32(tmem + lane_addr + o_col + q4 * 32, o);
            tmem_wait_ld();
          }
          if (row_valid) {
            uint32_t pkd[16];
#pragma unroll
            for (int e = 0; e < 16; ++e)
              pkd[e] = have_o ? pack_bf16(__uint_as_float(o[2 * e]) * inv, __uint_as_float(o[2 * e + 1]) * inv) : 0u;
#pragma unroll
            for (int e = 0; e < 4; ++e)
              reinterpret_cast<uint4*>(orow + q4 * 32)[e] = make_uint4(pkd[4 * e], pkd[4 * e + 1], pkd[4 * e + 2], pkd[4 * e + 3]);
          }
        }
        if (P.lse && row_valid)
          P.lse[(G.t0 + tok) * H + head] = have_o ? (m_used + log2f(l)) * 0.6931471805599453f : -INFINITY;
      } else {
        // The fp32 partial rows are staged in shared memory (the Q and K
        // tiles are free once the last MMA has completed) as query-ordered
        // 512-byte rows whose 16-byte chunks are XOR-swizzled by row, so both
        // the per-thread row writes and the per-warp row reads below are
        // bank-conflict free; each warp then stores whole rows, one
        // coalesced 512-byte line group per instruction.
        const int64_t rr = item * P.max_rows + (row_valid ? r : 0);
        float* stage = reinterpret_cast<float*>(smem + kQOff);  // [rows][128] fp32
        const bool any_o = ok && n > 0;
#pragma unroll 1
        for (int q4 = 0; q4 < kD / 32; ++q4) {
          uint32_t o[32];
          if (any_o) {
            tmem_ld32(tmem + lane_addr + o_col + q4 * 32, o);
            tmem_wait_ld();
          }
          if (row_valid && have_o) {
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const int j = q4 * 8 + e;  // 16-byte chunk of the row
              *reinterpret_cast<float4*>(stage + r * kD + ((j ^ (r & 7)) << 2)) =
                  make_float4(__uint_as_float(o[4 * e]), __uint_as_float(o[4 * e + 1]),
                              __uint_as_float(o[4 * e + 2]), __uint_as_float(o[4 * e + 3]));
            }
          }
        }
        if (row_valid) {
          P.ws_ml[rr * 2] = have_o ? m_used : -INFINITY;
          P.ws_ml[rr * 2 + 1] = have_o ? l : 0.0f;
        }
        if (n > 0) {
          // the softmax warps with rows meet here -- the condition is
          // uniform across the CTA, even when a wait timed out; rows whose sum
          // is zero carry whatever the stage holds: the merge never reads them
          asm volatile("bar.sync 2, %0;\n" ::"r"(nact * 32) : "memory");
          const int aidx = (warp >> 2) == 0 ? (warp & 3) : act0 + (warp & 3);  // index among active warps
          for (int row = aidx; row < rows_q; row += nact) {
            const float4 v = *reinterpret_cast<const float4*>(stage + row * kD + ((lane ^ (row & 7)) << 2));
            if (P.bf16_partials) {
              // bf16 rows, 256 bytes: lane's 4 dims as 8 bytes
              reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(P.ws_o) + (item * P.max_rows + row) * kD)[lane] =
                  make_uint2(pack_bf16(v.x, v.y), pack_bf16(v.z, v.w));
            } else {
              reinterpret_cast<float4*>(P.ws_o + (item * P.max_rows + row) * kD)[lane] = v;
            }
          }
        }
      }
    }
  }

  // ---- teardown: free TMEM ----
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ============================================================================
// Decode work list (one CTA, kSchedThreads threads).  Group g has c_g chunks
// of 64 union rows (the decode kernel's own count).  The smallest per-CTA
// chunk budget t with sum_g max(1, ceil(c_g / t)) <= max_items and at most
// kSchedMaxSplits CTAs per group is found by bisection; group g then gets
// s_g = max(1, ceil(c_g / t)) CTAs over even chunk ranges, numbered group by
// group.  With max_items = one wave of CTAs this minimises the longest CTA.
// ============================================================================
constexpr int kSchedThreads = 1024;
constexpr int kSchedMaxGroups = 8192;
constexpr int kSchedMaxSplits = 16;

__device__ __forceinline__ int sched_chunks(const int32_t* group_starts, const int32_t* swa_lens,
                                            const int32_t* comp_lens, int g) {
  const int t0 = group_starts ? group_starts[g] : g;
  const int t1 = group_starts ? group_starts[g + 1] : g + 1;
  const int len0 = swa_lens[t0];
  if (len0 <= 0) return 0;  // padding group: one CTA writes its zeros
  const int len_last = swa_lens[t1 - 1];
  const int extra = min(t1 - t0 - 1, len_last);
  const int n_comp = comp_lens ? max(comp_lens[t1 - 1], 0) : 0;
  return (len0 + extra + n_comp + tcd::kCh - 1) / tcd::kCh;
}

__device__ __forceinline__ int block_sum(int v, int* red) {
  __syncthreads();
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  int s = 0;
  for (int w = 0; w < kSchedThreads / 32; ++w) s += red[w];
  return s;
}

__global__ void __launch_bounds__(kSchedThreads) hca_decode_schedule_kernel(
    int32_t* sched, int max_items, const int32_t* group_starts, int num_groups, const int32_t* swa_lens,
    const int32_t* comp_lens) {
  __shared__ int c_s[kSchedMaxGroups];
  __shared__ int red[kSchedThreads / 32];
  int maxc = 1;
  for (int g = threadIdx.x; g < num_groups; g += kSchedThreads) {
    c_s[g] = sched_chunks(group_starts, swa_lens, comp_lens, g);
    maxc = max(maxc, c_s[g]);
  }
  for (int o = 16; o > 0; o >>= 1) maxc = max(maxc, __shfl_xor_sync(0xffffffffu, maxc, o));
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = maxc;
  __syncthreads();
  for (int w = 0; w < kSchedThreads / 32; ++w) maxc = max(maxc, red[w]);
  // bisection on the budget t in [lo, hi]; t = hi = maxc always fits
  // (num_groups <= max_items is checked on the host)
  int lo = max(1, (maxc + kSchedMaxSplits - 1) / kSchedMaxSplits), hi = max(lo, maxc);
  while (lo < hi) {
    const int t = (lo + hi) >> 1;
    int cnt = 0;
    for (int g = threadIdx.x; g < num_groups; g += kSchedThreads) cnt += max(1, (c_s[g] + t - 1) / t);
    if (block_sum(cnt, red) <= max_items)
      hi = t;
    else
      lo = t + 1;
  }
  const int t = lo;
  // exclusive prefix sum of s_g: each thread owns a contiguous run of groups
  const int per = (num_groups + kSchedThreads - 1) / kSchedThreads;
  const int g0 = threadIdx.x * per, g1 = min(num_groups, g0 + per);
  int local = 0;
  for (int g = g0; g < g1; ++g) local += max(1, (c_s[g] + t - 1) / t);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = local;  // inclusive scan within the warp, then over warp totals
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  __syncthreads();
  if (lane == 31) red[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int w = red[lane];
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    red[lane] = w;
  }
  __syncthreads();
  int first = incl - local + (warp > 0 ? red[warp - 1] : 0);
  const int total = red[kSchedThreads / 32 - 1];
  int32_t* groups = sched + 4 * static_cast<int64_t>(max_items);
  for (int g = g0; g < g1; ++g) {
    const int c = c_s[g];
    const int sg = max(1, (c + t - 1) / t);
    for (int k = 0; k < sg; ++k) {
      int4 it;
      it.x = g;
      it.y = k;
      it.z = static_cast<int>((static_cast<int64_t>(k) * c) / sg);
      it.w = static_cast<int>((static_cast<int64_t>(k + 1) * c) / sg);
      reinterpret_cast<int4*>(sched)[first + k] = it;
    }
    groups[2 * g] = first;
    groups[2 * g + 1] = sg;
    first += sg;
  }
  // idle slots past the last item
  for (int i = total + threadIdx.x; i < max_items; i += kSchedThreads)
    reinterpret_cast<int4*>(sched)[i] = make_int4(-1, 0, 0, 0);
}

// ============================================================================
// Fused split-K merge + VHA head mix + inverse RoPE + FP8 quant (decode).
// One CTA (512 threads) per token, padded to a multiple of 4 tokens.
//   merge: thread (head h = tid / 8, 16-dim segment tid % 8) sums the
//          group's bf16 partials (all of up to four splits' loads in flight
//          at once) weighted by 2^(m_s - m), applies the sink and
//          rounds O to bf16 in shared memory (the combine kernel's math);
//   mix:   warp w < 8: heads 16 (w % 4) .. +15, dims 64 (w / 4) .. +63 of
//          y = mix @ O (mma.sync m16n8k16 bf16, fp32 accumulate);
//   out:   inverse GPT-J RoPE on the RoPE dims, per-head amax over the two
//          dim halves, UE8M0 scale, e4m3 bytes in wo_a's input layout.
// ============================================================================
// Token t's group: its first token t0, first work-list item and item count
// (S = 0: no group holds it).  Each warp finds it on its own (ballot over
// groups whose start, end and schedule entry are loaded together), so no
// block barrier waits on it.
__device__ __forceinline__ void vha_token_group(const AttnParams& P, const VhaOut& V, int t, int& t0, int& first,
                                                int& S) {
  const int lane = threadIdx.x & 31;
  first = 0;
  S = 0;
  t0 = t;
  const int32_t* gt = P.sched ? P.sched + 4 * P.sched_items : nullptr;
  if (!P.group_starts) {
    first = gt ? gt[2 * t] : t * P.num_splits;
    S = gt ? gt[2 * t + 1] : P.num_splits;
    return;
  }
  for (int base = 0; base < V.num_groups; base += 128) {
    int a[4], f[4], sc[4];
    bool hit[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int g = base + k * 32 + lane;
      hit[k] = false;
      a[k] = f[k] = sc[k] = 0;
      if (g < V.num_groups) {
        a[k] = P.group_starts[g];
        const int b = P.group_starts[g + 1];
        f[k] = gt ? gt[2 * g] : g * P.num_splits;
        sc[k] = gt ? gt[2 * g + 1] : P.num_splits;
        hit[k] = a[k] <= t && t < b;
      }
    }
    bool found = false;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const unsigned m = __ballot_sync(0xffffffffu, hit[k]);
      if (m && !found) {
        const int src = __ffs(m) - 1;
        first = __shfl_sync(0xffffffffu, f[k], src);
        S = __shfl_sync(0xffffffffu, sc[k], src);
        t0 = __shfl_sync(0xffffffffu, a[k], src);
        found = true;
      }
    }
    if (found) break;
  }
}

// Split-K merge + VHA + inverse RoPE + FP8 quant, one 512-thread CTA per
// token (two per SM).  Up to the dependency wait this kernel reads only
// weights (the mix), the RoPE table and per-step metadata (positions, groups,
// work list), none of which a layer kernel writes, so it overlaps the
// attention still running on other SMs; the partials (and every store) come
// after the wait.
__global__ void __launch_bounds__(512, 2) hca_combine_vha_quant_kernel(const AttnParams P, const VhaOut V) {
  pdl_release();
  __shared__ __align__(16) vt::Smem sm;
  const int H = P.num_heads;
  const int t = blockIdx.x;
  if (t >= V.num_tokens) {
    pdl_wait();
    for (int h = threadIdx.x; h < H; h += blockDim.x) V.scale[static_cast<int64_t>(h) * V.aligned_t + t] = 0;
    return;
  }
  vha_load_mix(V, H, sm);
  if (threadIdx.x < P.rope_dim) sm.cs[threadIdx.x] = V.cos_sin[V.positions[t] * V.cs_stride + threadIdx.x];
  int t0, first, S;
  vha_token_group(P, V, t, t0, first, S);
  // a group larger than the workspace rows was skipped by the attention launch
  if ((t - t0 + 1) * H > P.max_rows || S > vt::kMaxSplits) S = 0;
  pdl_wait();  // the attention launch has written the partials
  vha_merge_token(P, t, t0, first, S, sm);
  vha_mix_quant_token(P, V, t, sm);
}

int64_t align_up(int64_t v, int64_t a) { return (v + a - 1) / a * a; }

}  // namespace
}  // namespace hca

using namespace hca;

// Device error word: bit 0 loader, bit 1 dequant, bit 2 MMA, bit 3 softmax
// of the attention kernels, bit 4 the streamed Q prep, bit 5 the streamed
// VHA output kernel timed out on an mbarrier.  Zero in normal operation.
__device__ int g_hca_device_error;

int* hca::device_error_word() {
  int* p = nullptr;
  return cudaGetSymbolAddress(reinterpret_cast<void**>(&p), g_hca_device_error) == cudaSuccess ? p : nullptr;
}

extern "C" int hca_device_error(int32_t* value, int32_t clear) {
  if (!value) return HCA_E_INVALID;
  if (cudaMemcpyFromSymbol(value, g_hca_device_error, sizeof(int)) != cudaSuccess) return HCA_E_CUDA;
  if (clear) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(g_hca_device_error, &zero, sizeof(int)) != cudaSuccess) return HCA_E_CUDA;
  }
  return HCA_OK;
}

extern "C" int64_t hca_sparse_decode_workspace_bytes(int32_t num_groups, int32_t max_group_tokens,
                                                     int32_t num_heads, int32_t head_dim,
                                                     int32_t num_splits) {
  if (num_splits <= 1 || num_groups <= 0) return 0;
  const int64_t rows = static_cast<int64_t>(max_group_tokens) * num_heads;
  const int64_t o = align_up(static_cast<int64_t>(num_groups) * num_splits * rows * head_dim * 4, 256);
  const int64_t ml = align_up(static_cast<int64_t>(num_groups) * num_splits * rows * 2 * 4, 256);
  return o + ml;
}

// Limit of every mbarrier wait of the head_dim-128 attention kernel for
// launches made from now on; < 0 restores the default.  A diagnostic: with
// 0 a wait that is not already satisfied fails at once, so the launch ends
// early with its device error bits set (used to test the bounded waits).
static std::atomic<int64_t> g_attn_wait_ns{-1};

static uint64_t attention_wait_ns() {
  const int64_t v = g_attn_wait_ns.load();
  return v < 0 ? tc::kWaitLimitNs : static_cast<uint64_t>(v);
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

static int sparse_decode_impl(void* out, int64_t out_stride_tok, int64_t out_stride_head,
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
                                 const int32_t* schedule, int32_t max_items, int fused,
                                 void* workspace, int64_t workspace_bytes, void* stream,
                                 AttnParams* fused_params = nullptr) {
  if (!group_starts) {
    num_groups = num_tokens;
    max_group_tokens = 1;
  }
  HCA_CHECK_ARG(num_tokens >= 0 && num_groups >= 0 && swa_page_size > 0);
  if (schedule) {
    HCA_CHECK_ARG(max_items >= num_groups && max_items >= 1 && num_groups <= kSchedMaxGroups &&
                  reinterpret_cast<uintptr_t>(schedule) % 16 == 0);
    num_splits = 1;
  } else {
    HCA_CHECK_ARG(num_splits >= 1 && num_splits <= 16);
  }
  // head_dim 512 runs on CTA pairs (uniform splits, unfused output)
  const bool wide = head_dim == 512;
  if (wide) {
    // with the work list, every group fits one pair's tile
    if (rope_dim != 64 || fused || num_heads < 1 || num_heads > 128 || max_group_tokens < 1 ||
        max_group_tokens > 30 || (schedule && max_group_tokens > wide_tile_tokens(num_heads)))
      return HCA_E_UNSUPPORTED;
  } else if (head_dim != 128 || rope_dim != 64 || num_heads < 1 || max_group_tokens < 1 || max_group_tokens > 30 ||
             max_group_tokens * num_heads > tcd::kMaxRows) {
    return HCA_E_UNSUPPORTED;
  }
  if (num_tokens == 0 || num_groups == 0) return HCA_OK;
  HCA_CHECK_ARG(out && q && swa_cache && swa_indices && swa_lens);
  HCA_CHECK_ARG(!comp_cache || (comp_indices && comp_lens && comp_page_size > 0));
  HCA_CHECK_ARG(swa_page_stride_bytes % 16 == 0 && (!comp_cache || comp_page_stride_bytes % 16 == 0));
  HCA_CHECK_ARG(reinterpret_cast<uintptr_t>(swa_cache) % 16 == 0 && reinterpret_cast<uintptr_t>(comp_cache) % 16 == 0 &&
                reinterpret_cast<uintptr_t>(q) % 16 == 0 && q_stride_tok % 8 == 0 && q_stride_head % 8 == 0);
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
  P.sched = schedule;
  P.sched_items = schedule ? max_items : 0;
  P.force_partials = fused;
  // D=128 split partials are bf16 rows (half the bytes through L2 for the
  // attention's epilogue and the merge); the D=512 pair kernel writes fp32
  P.bf16_partials = !wide;
  P.wait_ns = attention_wait_ns();
  // partial slots: groups x splits, or one per work-list item
  const int32_t slot_groups = schedule ? 1 : num_groups;
  const int32_t slot_splits = schedule ? max_items : num_splits;
  if (slot_splits > 1 || fused) {
    const int64_t rows = static_cast<int64_t>(max_group_tokens) * num_heads;
    const int64_t slots = static_cast<int64_t>(slot_groups) * slot_splits;
    const int64_t o = align_up(slots * rows * head_dim * 4, 256);
    const int64_t need = o + align_up(slots * rows * 2 * 4, 256);
    if (!workspace || workspace_bytes < need) return HCA_E_WORKSPACE;
    const int64_t ml = align_up(static_cast<int64_t>(num_groups) * num_splits * rows * 2 * 4, 256);
    (void)ml;
    char* w = static_cast<char*>(workspace);
    P.ws_o = reinterpret_cast<float*>(w);
    P.ws_ml = reinterpret_cast<float*>(w + o);
  }
  cudaStream_t s = as_stream(stream);
  int* err = nullptr;
  if (cudaGetSymbolAddress(reinterpret_cast<void**>(&err), g_hca_device_error) != cudaSuccess) return HCA_E_CUDA;
  if (wide) {
    P.group_tokens = wide_tile_tokens(num_heads);
    const int wrc = launch_wide_attention(P, false, num_groups, max_group_tokens, err, s);
    if (wrc != HCA_OK || slot_splits == 1) return wrc;
    return launch_pdl(hca_attention_combine_kernel<512, false>, dim3(num_groups, (P.max_rows + 15) / 16), dim3(256),
                      0, s, P);
  }
  static bool smem_set[kMaxDevices] = {};
  if (set_func_attr_once(hca_tc_attention_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, tcd::kSmemBytes,
                         smem_set) != HCA_OK)
    return HCA_E_CUDA;
  const int lrc = launch_pdl(hca_tc_attention_kernel<false>, schedule ? dim3(max_items, 1) : dim3(num_splits, num_groups),
                             dim3(tcd::kThreads), tcd::kSmemBytes, s, P, err);
  if (lrc != HCA_OK) return lrc;
  if (fused) {
    *fused_params = P;
    return HCA_OK;
  }
  if (slot_splits > 1)
    return launch_pdl(hca_attention_combine_kernel<128, false>, dim3(num_groups, (P.max_rows + 15) / 16), dim3(256),
                      0, s, P);
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
  return sparse_decode_impl(out, out_stride_tok, out_stride_head, lse, q, q_stride_tok, q_stride_head, num_tokens,
                            num_heads, head_dim, rope_dim, swa_cache, swa_page_size, swa_page_stride_bytes,
                            swa_indices, swa_indices_stride, swa_lens, comp_cache, comp_page_size,
                            comp_page_stride_bytes, comp_indices, comp_indices_stride, comp_lens, group_starts,
                            num_groups, max_group_tokens, softmax_scale, attn_sink, num_splits, nullptr, 0, 0,
                            workspace, workspace_bytes, stream);
}

extern "C" int64_t hca_decode_schedule_ints(int32_t num_groups, int32_t max_items) {
  if (num_groups < 0 || max_items < num_groups || max_items < 1 || num_groups > kSchedMaxGroups) return -1;
  return 4 * static_cast<int64_t>(max_items) + 2 * static_cast<int64_t>(num_groups);
}

extern "C" int hca_decode_schedule(int32_t* schedule, int32_t max_items, const int32_t* group_starts,
                                   int32_t num_groups, int32_t num_tokens, const int32_t* swa_lens,
                                   const int32_t* comp_lens, void* stream) {
  HCA_CHECK_ARG(hca_decode_schedule_ints(num_groups, max_items) > 0);
  HCA_CHECK_ARG(num_tokens >= 0 && (group_starts || num_groups == num_tokens));
  HCA_CHECK_ARG(schedule && reinterpret_cast<uintptr_t>(schedule) % 16 == 0);
  if (num_groups == 0) {
    // every CTA idle
    hca_decode_schedule_kernel<<<1, kSchedThreads, 0, as_stream(stream)>>>(schedule, max_items, group_starts, 0,
                                                                           swa_lens, comp_lens);
    return HCA_LAUNCH_STATUS();
  }
  HCA_CHECK_ARG(swa_lens);
  hca_decode_schedule_kernel<<<1, kSchedThreads, 0, as_stream(stream)>>>(schedule, max_items, group_starts,
                                                                         num_groups, swa_lens, comp_lens);
  return HCA_LAUNCH_STATUS();
}

extern "C" int64_t hca_sparse_decode_vha_workspace_bytes(int32_t max_items, int32_t max_group_tokens,
                                                         int32_t num_heads, int32_t head_dim) {
  if (max_items < 1 || max_group_tokens < 1 || num_heads < 1 || head_dim < 1) return 0;
  const int64_t slots = max_items, rows = static_cast<int64_t>(max_group_tokens) * num_heads;
  return align_up(slots * rows * head_dim * 4, 256) + align_up(slots * rows * 2 * 4, 256);
}

extern "C" int hca_sparse_decode_vha_fp8_quant(
    uint8_t* out, int32_t* scale, const void* q, int64_t q_stride_tok, int64_t q_stride_head, int32_t num_tokens,
    int32_t num_heads, int32_t head_dim, int32_t rope_dim, const uint8_t* swa_cache, int32_t swa_page_size,
    int64_t swa_page_stride_bytes, const int32_t* swa_indices, int64_t swa_indices_stride, const int32_t* swa_lens,
    const uint8_t* comp_cache, int32_t comp_page_size, int64_t comp_page_stride_bytes, const int32_t* comp_indices,
    int64_t comp_indices_stride, const int32_t* comp_lens, const int32_t* group_starts, int32_t num_groups,
    int32_t max_group_tokens, float softmax_scale, const float* attn_sink, const int32_t* schedule,
    int32_t max_items, const void* mix, const int64_t* positions, const float* cos_sin, int64_t cos_sin_stride,
    int32_t n_groups, void* workspace, int64_t workspace_bytes, void* stream) {
  HCA_CHECK_ARG(num_tokens >= 0 && n_groups > 0 && num_heads > 0 && num_heads % n_groups == 0);
  if (head_dim != 128 || rope_dim != 64 || num_heads % 16 || num_heads > 64) return HCA_E_UNSUPPORTED;
  if (num_tokens == 0) return HCA_OK;
  HCA_CHECK_ARG(out && scale && schedule && mix && positions && cos_sin && workspace);
  HCA_CHECK_ARG(reinterpret_cast<uintptr_t>(mix) % 16 == 0 && reinterpret_cast<uintptr_t>(workspace) % 16 == 0 &&
                reinterpret_cast<uintptr_t>(out) % 16 == 0);
  // the attention launch writes only split partials here; `out` of the
  // attention stage is unused, so the (aligned) workspace stands in for it
  AttnParams P{};
  const int rc = sparse_decode_impl(workspace, 8, 8, nullptr, q, q_stride_tok, q_stride_head, num_tokens, num_heads,
                                    head_dim, rope_dim, swa_cache, swa_page_size, swa_page_stride_bytes, swa_indices,
                                    swa_indices_stride, swa_lens, comp_cache, comp_page_size, comp_page_stride_bytes,
                                    comp_indices, comp_indices_stride, comp_lens, group_starts, num_groups,
                                    max_group_tokens, softmax_scale, attn_sink, 1, schedule, max_items, 1, workspace,
                                    workspace_bytes, stream, &P);
  if (rc != HCA_OK) return rc;
  VhaOut V;
  V.out = out;
  V.scale = scale;
  V.mix = static_cast<const __nv_bfloat16*>(mix);
  V.positions = positions;
  V.cos_sin = cos_sin;
  V.cs_stride = cos_sin_stride;
  V.num_tokens = num_tokens;
  V.aligned_t = (num_tokens + 3) / 4 * 4;
  V.n_groups = n_groups;
  V.num_groups = group_starts ? num_groups : num_tokens;
  static bool carveout_set[kMaxDevices] = {};  // two CTAs per SM: prefer shared memory over L1
  if (set_func_attr_once(hca_combine_vha_quant_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                         cudaSharedmemCarveoutMaxShared, carveout_set) != HCA_OK)
    return HCA_E_CUDA;
  return launch_pdl(hca_combine_vha_quant_kernel, dim3(V.aligned_t), dim3(512), 0, as_stream(stream), P, V);
}

extern "C" int hca_set_attention_wait_limit_ns(int64_t limit_ns) {
  g_attn_wait_ns.store(limit_ns);
  return HCA_OK;
}

extern "C" int hca_sparse_decode_scheduled(void* out, int64_t out_stride_tok, int64_t out_stride_head,
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
                                           float softmax_scale, const float* attn_sink,
                                           const int32_t* schedule, int32_t max_items,
                                           void* workspace, int64_t workspace_bytes, void* stream) {
  if (!schedule) return HCA_E_INVALID;
  return sparse_decode_impl(out, out_stride_tok, out_stride_head, lse, q, q_stride_tok, q_stride_head, num_tokens,
                            num_heads, head_dim, rope_dim, swa_cache, swa_page_size, swa_page_stride_bytes,
                            swa_indices, swa_indices_stride, swa_lens, comp_cache, comp_page_size,
                            comp_page_stride_bytes, comp_indices, comp_indices_stride, comp_lens, group_starts,
                            num_groups, max_group_tokens, softmax_scale, attn_sink, 1, schedule, max_items, 0,
                            workspace, workspace_bytes, stream);
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
  const bool wide = head_dim == 512;
  // head_dim 128 with up to 256 heads runs on the tcgen05 kernel (any head
  // count); the mma.sync kernel is the fallback for the other shapes
  const bool tc = head_dim == 128 && rope_dim == 64 && num_heads >= 1 && num_heads <= tcd::kMaxRows;
  const int group_tokens = num_heads > 0 ? (wide ? wide_tile_tokens(num_heads) : (kMaxWarps * 16) / num_heads) : 0;
  if (wide) {
    if (rope_dim != 64 || num_heads < 1 || num_heads > 128) return HCA_E_UNSUPPORTED;
  } else if (!tc && (group_tokens < 1 || !attn_shape_ok(num_heads, head_dim, rope_dim, group_tokens))) {
    return HCA_E_UNSUPPORTED;
  }
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
  P.wait_ns = attention_wait_ns();
  if (wide) {
    // CTA pairs over tiles of 128 / H tokens, all of a tile's rows
    HCA_CHECK_ARG(reinterpret_cast<uintptr_t>(swa_cache) % 16 == 0 && reinterpret_cast<uintptr_t>(comp_cache) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(q) % 16 == 0 && q_stride_tok % 8 == 0 && q_stride_head % 8 == 0);
    HCA_CHECK_ARG(out_stride_head % 8 == 0 && out_stride_tok % 8 == 0 && reinterpret_cast<uintptr_t>(out) % 16 == 0);
    int* err = nullptr;
    if (cudaGetSymbolAddress(reinterpret_cast<void**>(&err), g_hca_device_error) != cudaSuccess) return HCA_E_CUDA;
    const int num_tiles = num_tokens / group_tokens + num_reqs;
    return launch_wide_attention(P, true, num_tiles, 0, err, as_stream(stream));
  }
  if (tc) {
    // tcgen05 path: tiles of up to 256 query rows, at most 31 tokens (one
    // mask bit each; bit 31 of a row's mask is its "loaded" flag), all of a
    // tile's rows in one CTA
    const int tc_tokens = min(31, tcd::kMaxRows / num_heads);
    P.group_tokens = tc_tokens;
    P.max_rows = tc_tokens * num_heads;
    HCA_CHECK_ARG(reinterpret_cast<uintptr_t>(swa_cache) % 16 == 0 && reinterpret_cast<uintptr_t>(comp_cache) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(q) % 16 == 0 && q_stride_tok % 8 == 0 && q_stride_head % 8 == 0);
    HCA_CHECK_ARG(out_stride_head % 8 == 0 && out_stride_tok % 8 == 0 && reinterpret_cast<uintptr_t>(out) % 16 == 0);
    static bool smem_set[kMaxDevices] = {};
    if (set_func_attr_once(hca_tc_attention_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           tcd::kSmemBytes, smem_set) != HCA_OK)
      return HCA_E_CUDA;
    int* err = nullptr;
    if (cudaGetSymbolAddress(reinterpret_cast<void**>(&err), g_hca_device_error) != cudaSuccess) return HCA_E_CUDA;
    // tiles never straddle requests: at most tokens / G + requests of them
    const int num_tiles = num_tokens / tc_tokens + num_reqs;
    return launch_pdl(hca_tc_attention_kernel<true>, dim3(num_tiles), dim3(tcd::kThreads), tcd::kSmemBytes,
                      as_stream(stream), P, err);
  }
  // tiles never straddle requests: at most tokens / G + requests of them
  const int num_tiles = num_tokens / group_tokens + num_reqs;
  return launch_attention<true>(P, num_tiles, group_tokens, as_stream(stream));
}
