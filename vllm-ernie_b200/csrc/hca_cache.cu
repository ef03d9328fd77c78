// KV-cache side of the HCA path: QK RMSNorm, query head-norm + RoPE with the
// fused fp8 SWA-cache insert, plain quantised insert, dequant gather, the
// compressor state save and the per-128-token block compressor.
//
// All of these are HBM-bound, byte-moving kernels: one warp (or one CTA)
// per row, 16-byte vector accesses where the row layout allows, no tensor
// cores.  Row geometry is templated on the head dim (128 or 512).
#include <algorithm>

#include "hca_common.cuh"
#include "hca_tc.cuh"

namespace hca {
namespace {

// ----------------------------------------------------------------------------
// QK RMSNorm: grid (T, 2), y = x * rsqrt(mean(x^2) + eps) * w, fp32 math.
// ----------------------------------------------------------------------------
__global__ void qk_rmsnorm_kernel(__nv_bfloat16* q_out, int64_t q_out_stride,
                                  const __nv_bfloat16* q_in, int64_t q_in_stride,
                                  const __nv_bfloat16* q_w, int q_size, __nv_bfloat16* kv_out,
                                  int64_t kv_out_stride, const __nv_bfloat16* kv_in,
                                  int64_t kv_in_stride, const __nv_bfloat16* kv_w, int kv_size,
                                  float eps) {
  __shared__ float red[32];
  const int64_t t = blockIdx.x;
  const bool is_q = blockIdx.y == 0;
  const int n = is_q ? q_size : kv_size;
  const __nv_bfloat16* x = is_q ? q_in + t * q_in_stride : kv_in + t * kv_in_stride;
  const __nv_bfloat16* w = is_q ? q_w : kv_w;
  __nv_bfloat16* y = is_q ? q_out + t * q_out_stride : kv_out + t * kv_out_stride;
  float ss = 0.0f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = __bfloat162float(x[i]);
    ss += v * v;
  }
  ss = block_sum(ss, red);
  const float rrms = rsqrtf(ss / static_cast<float>(n) + eps);
  for (int i = threadIdx.x; i < n; i += blockDim.x)
    y[i] = __float2bfloat16_rn(__bfloat162float(x[i]) * rrms * __bfloat162float(w[i]));
}

// ----------------------------------------------------------------------------
// One cached row held by one warp: lane l owns elements [l*E, (l+1)*E).
// ----------------------------------------------------------------------------
template <int D>
struct WarpRow {
  static constexpr int E = D / 32;  // elements per lane
  static_assert(E % 4 == 0, "head_dim must be a multiple of 128");
  float v[E];

  __device__ __forceinline__ void load_bf16(const __nv_bfloat16* row, int lane) {
    const uint16_t* p = reinterpret_cast<const uint16_t*>(row) + lane * E;
    if ((reinterpret_cast<uintptr_t>(p) & 7) == 0) {
      // E % 4 == 0 here: 8-byte vector loads
#pragma unroll
      for (int i = 0; i < E; i += 4) {
        const uint2 w = *reinterpret_cast<const uint2*>(p + i);
        v[i] = bf16_bits_to_float(static_cast<uint16_t>(w.x & 0xffff));
        v[i + 1] = bf16_bits_to_float(static_cast<uint16_t>(w.x >> 16));
        v[i + 2] = bf16_bits_to_float(static_cast<uint16_t>(w.y & 0xffff));
        v[i + 3] = bf16_bits_to_float(static_cast<uint16_t>(w.y >> 16));
      }
    } else {
#pragma unroll
      for (int i = 0; i < E; ++i) v[i] = bf16_bits_to_float(p[i]);
    }
  }

  // Rows known to be 8-byte aligned (shared-memory stages): no alignment test.
  __device__ __forceinline__ void load_bf16_aligned(const __nv_bfloat16* row, int lane) {
    const uint2* p = reinterpret_cast<const uint2*>(row + lane * E);
#pragma unroll
    for (int i = 0; i < E; i += 4) {
      const uint2 w = p[i / 4];
      v[i] = __uint_as_float(w.x << 16);
      v[i + 1] = __uint_as_float(w.x & 0xffff0000u);
      v[i + 2] = __uint_as_float(w.y << 16);
      v[i + 3] = __uint_as_float(w.y & 0xffff0000u);
    }
  }

  // Two round-to-nearest-even bf16 conversions in one instruction.
  static __device__ __forceinline__ uint32_t pack2(float lo, float hi) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
  }

  __device__ __forceinline__ void store_bf16_aligned(__nv_bfloat16* row, int lane) const {
    uint2* o = reinterpret_cast<uint2*>(row + lane * E);
#pragma unroll
    for (int i = 0; i < E; i += 4) o[i / 4] = make_uint2(pack2(v[i], v[i + 1]), pack2(v[i + 2], v[i + 3]));
  }

  // bf16 of every element, 8-byte vector stores when aligned
  __device__ __forceinline__ void store_bf16(__nv_bfloat16* row, int lane) const {
    uint16_t* o = reinterpret_cast<uint16_t*>(row) + lane * E;
    if ((reinterpret_cast<uintptr_t>(o) & 7) == 0) {
#pragma unroll
      for (int i = 0; i < E; i += 4) *reinterpret_cast<uint2*>(o + i) = make_uint2(pack2(v[i], v[i + 1]), pack2(v[i + 2], v[i + 3]));
    } else {
#pragma unroll
      for (int i = 0; i < E; ++i) o[i] = float_to_bf16_bits(v[i]);
    }
  }

  // GPT-J rotation of the pairs that fall in the last R dims.
  __device__ __forceinline__ void rope(const float* cs, int rope_dim, int lane, bool inverse) {
    const int nope = D - rope_dim;
    const int half = rope_dim / 2;
#pragma unroll
    for (int i = 0; i < E; i += 2) {
      const int d = lane * E + i;
      if (d >= nope) {
        const int pr = (d - nope) >> 1;
        const float c = cs[pr];
        const float s = inverse ? -cs[half + pr] : cs[half + pr];
        rope_pair(v[i], v[i + 1], c, s);
      }
    }
  }

  // Quantise the NoPE part (from `v`, already bf16 valued) and store the row:
  // fp8 NoPE bytes, RoPE as bf16 of `rope_src`, UE8M0 scale bytes + pad 0.
  __device__ __forceinline__ void store_cache_row(RowPtr dst, int rope_dim, int lane, bool divide,
                                                  const float* rope_src) {
    const int nope = D - rope_dim;
    const int d0 = lane * E;
    constexpr int kLanesPerBlock = kQuantBlock / E;  // lanes sharing one scale
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < E; ++i) amax = fmaxf(amax, fabsf(v[i]));
#pragma unroll
    for (int o = 1; o < kLanesPerBlock; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (d0 < nope) {
      const int e = ue8m0_exponent(amax, 1e-4f, divide);
      const float inv = exp2i(-e);
      uint8_t q[E];
#pragma unroll
      for (int i = 0; i < E; ++i) q[i] = to_e4m3(v[i] * inv);
#pragma unroll
      for (int i = 0; i < E; ++i) dst.data[d0 + i] = q[i];
      if ((d0 % kQuantBlock) == 0) dst.scale[d0 / kQuantBlock] = encode_ue8m0(e);
    } else {
      uint16_t* r = reinterpret_cast<uint16_t*>(dst.data + nope) + (d0 - nope);
#pragma unroll
      for (int i = 0; i < E; ++i) r[i] = float_to_bf16_bits(rope_src[i]);
    }
    if (lane == 0) dst.scale[nope / kQuantBlock] = 0;
  }
};

// grid (T, ceil((padded_heads + 1) / 4)), 128 threads: warp w of block y
// handles head y*4 + w; head index == padded_heads is the KV row.
template <int D>
__global__ void qnorm_rope_kv_insert_kernel(__nv_bfloat16* q_out, int64_t qo_st, int64_t qo_sh,
                                            int padded_heads, const __nv_bfloat16* q,
                                            int64_t q_st, int64_t q_sh, int num_heads,
                                            const __nv_bfloat16* kv, int64_t kv_stride,
                                            uint8_t* cache, int page_size, int64_t page_stride,
                                            const int64_t* slot_mapping,
                                            const int64_t* positions, const float* cos_sin,
                                            int64_t cs_stride, int rope_dim, float eps) {
  pdl_wait_and_release();
  constexpr int E = WarpRow<D>::E;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const int64_t t = blockIdx.x;
  const float* cs = cos_sin + positions[t] * cs_stride;
  // this lane's RoPE pairs (dims lane * E + 2i, + 1): cos / sin once per warp
  const int nope = D - rope_dim;
  float pc[E / 2], ps[E / 2];
#pragma unroll
  for (int i = 0; i < E / 2; ++i) {
    const int d = lane * E + 2 * i;
    pc[i] = 1.0f;
    ps[i] = 0.0f;
    if (d >= nope) {
      pc[i] = cs[(d - nope) >> 1];
      ps[i] = cs[rope_dim / 2 + ((d - nope) >> 1)];
    }
  }
  auto rope = [&](WarpRow<D>& r) {
#pragma unroll
    for (int i = 0; i < E / 2; ++i) rope_pair(r.v[2 * i], r.v[2 * i + 1], pc[i], ps[i]);
  };
  // CTA (t, y) owns rows [y * rpc, (y + 1) * rpc) of token t: the query heads,
  // the zero padding heads, and row padded_heads = the KV row.  Warp w takes
  // rows w, w + nwarps, ...; they are loaded kBatch at a time before any is
  // used (more bytes in flight).
  const int nrows = padded_heads + 1;
  const int rpc = (nrows + gridDim.y - 1) / gridDim.y;
  const int row_lo = blockIdx.y * rpc, row_hi = min(nrows, row_lo + rpc);
  constexpr int kBatch = D == 128 ? 8 : 4;  // rows loaded per warp before any is used
  for (int hb = row_lo + warp; hb < row_hi; hb += nwarps * kBatch) {
    WarpRow<D> rows[kBatch];
#pragma unroll
    for (int b = 0; b < kBatch; ++b) {
      const int h = hb + b * nwarps;
      if (h < row_hi && h < num_heads) rows[b].load_bf16(q + t * q_st + h * q_sh, lane);
      else if (h < row_hi && h == padded_heads) rows[b].load_bf16(kv + t * kv_stride, lane);
    }
#pragma unroll
    for (int b = 0; b < kBatch; ++b) {
      const int h = hb + b * nwarps;
      if (h >= row_hi) continue;
      if (h < num_heads) {
        WarpRow<D>& row = rows[b];
        float ss = 0.0f;
#pragma unroll
        for (int i = 0; i < E; ++i) ss += row.v[i] * row.v[i];
        ss = warp_sum(ss);
        const float rrms = rsqrtf(ss / static_cast<float>(D) + eps);
#pragma unroll
        for (int i = 0; i < E; ++i) row.v[i] *= rrms;
        rope(row);
        row.store_bf16(q_out + t * qo_st + h * qo_sh, lane);
      } else if (h < padded_heads) {
        uint16_t* o = reinterpret_cast<uint16_t*>(q_out + t * qo_st + h * qo_sh) + lane * E;
#pragma unroll
        for (int i = 0; i < E; ++i) o[i] = 0;
      } else {
        // the KV row: RoPE, fp8 NoPE quant, insert
        const int64_t slot = slot_mapping[t];
        if (slot < 0) continue;
        WarpRow<D> r2 = rows[b];
        rope(r2);
        const RowGeom g = row_geom(D, rope_dim);
        rows[b].store_cache_row(row_ptr(cache, slot, page_size, page_stride, g), rope_dim, lane, true, r2.v);
      }
    }
  }
}

// ----------------------------------------------------------------------------
// Streamed Q prep for many tokens (prefill).  Persistent CTAs walk tokens
// t = blockIdx.x, + gridDim.x, ...  Warp 8 (the producer) copies each
// token's contiguous Q block (num_heads x D bf16), its KV row and its cos /
// sin row into the next stage of a shared-memory ring with one bulk async
// copy each (completion counted in bytes on the stage's `full` mbarrier).
// Warps 0-7 (the consumers) take rows h = warp, warp + 8, ... of the token
// out of shared memory, kStreamBatch at a time, store them and release the
// stage on its `empty` mbarrier.  The arithmetic of every row is the one of
// qnorm_rope_kv_insert_kernel (same lane layout, same order of operations),
// so both kernels write identical bytes; this one keeps stages x 16 KB per CTA
// in flight instead of a few rows per warp.
// ----------------------------------------------------------------------------
struct QPrepStream {
  __nv_bfloat16* q_out;
  int64_t qo_st;  // heads of a token are contiguous (stride D)
  const __nv_bfloat16* q;
  int64_t q_st;  // heads of a token are contiguous (stride D)
  const __nv_bfloat16* kv;
  int64_t kv_stride;
  uint8_t* cache;
  int64_t page_stride;
  const int64_t* slot_mapping;
  const int64_t* positions;
  const float* cos_sin;
  int64_t cs_stride;
  int* err;  // bit 4 on a wait that gave up
  int page_size, padded_heads, num_heads, rope_dim, num_tokens, stages;
  uint32_t q_bytes, kv_off, cs_off, stage_bytes;
  float eps;
};

constexpr int kStreamConsumers = 8;     // consumer warps; warp 8 is the producer
constexpr int kStreamMaxStages = 8;
constexpr int kStreamBatch = 4;         // rows a consumer warp reads before it uses any
constexpr int kStreamErrBit = 1 << 4;

template <int D>
__global__ void __launch_bounds__(32 * (kStreamConsumers + 1), D == 128 ? 4 : 1) qprep_stream_kernel(const QPrepStream P) {
  extern __shared__ __align__(128) uint8_t qs_ring[];
  __shared__ __align__(8) uint64_t full[kStreamMaxStages], empty[kStreamMaxStages];
  __shared__ int64_t slot_s[kStreamMaxStages];
  constexpr int E = WarpRow<D>::E;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int S = P.stages;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], kStreamConsumers);
    }
    tc::mbar_fence_init();
  }
  __syncthreads();
  pdl_wait_and_release();
  const int T = P.num_tokens;
  if (warp == kStreamConsumers) {
    // producer: positions and slots of the next 32 tokens of this CTA are
    // loaded one per lane, so the cos / sin address is known without a
    // dependent load per token
    int64_t pos_l = 0, slot_l = -1;
    for (int k = 0;; ++k) {
      const int64_t t = blockIdx.x + static_cast<int64_t>(k) * gridDim.x;
      if (t >= T) break;
      if ((k & 31) == 0) {
        const int64_t tl = t + static_cast<int64_t>(lane) * gridDim.x;
        pos_l = tl < T ? P.positions[tl] : 0;
        slot_l = tl < T ? P.slot_mapping[tl] : -1;
      }
      const int64_t pos = __shfl_sync(0xffffffffu, pos_l, k & 31);
      const int64_t slot = __shfl_sync(0xffffffffu, slot_l, k & 31);
      const int s = k % S, n = k / S;
      int ok = 1;
      if (lane == 0) {
        if (n > 0 && !tc::mbar_wait(&empty[s], (n - 1) & 1)) ok = 0;
        if (ok) {
          uint8_t* st = qs_ring + static_cast<size_t>(s) * P.stage_bytes;
          slot_s[s] = slot;
          tc::mbar_arrive_expect_tx(&full[s], P.q_bytes + D * 2 + P.rope_dim * 4);
          tc::bulk_copy_g2s(st, P.q + t * P.q_st, P.q_bytes, &full[s]);
          tc::bulk_copy_g2s(st + P.kv_off, P.kv + t * P.kv_stride, D * 2, &full[s]);
          tc::bulk_copy_g2s(st + P.cs_off, P.cos_sin + pos * P.cs_stride, P.rope_dim * 4, &full[s]);
        }
      }
      if (!__shfl_sync(0xffffffffu, ok, 0)) {
        if (lane == 0) atomicOr(P.err, kStreamErrBit);
        break;
      }
    }
    return;
  }
  // consumers
  const int nope = D - P.rope_dim;
  const int nrows = P.padded_heads + 1;
  for (int k = 0;; ++k) {
    const int64_t t = blockIdx.x + static_cast<int64_t>(k) * gridDim.x;
    if (t >= T) break;
    const int s = k % S;
    if (!tc::mbar_wait(&full[s], (k / S) & 1)) {
      if (lane == 0) atomicOr(P.err, kStreamErrBit);
      break;
    }
    const uint8_t* st = qs_ring + static_cast<size_t>(s) * P.stage_bytes;
    const __nv_bfloat16* qs = reinterpret_cast<const __nv_bfloat16*>(st);
    const float* cs = reinterpret_cast<const float*>(st + P.cs_off);
    float pc[E / 2], ps[E / 2];
#pragma unroll
    for (int i = 0; i < E / 2; ++i) {
      const int d = lane * E + 2 * i;
      pc[i] = 1.0f;
      ps[i] = 0.0f;
      if (d >= nope) {
        pc[i] = cs[(d - nope) >> 1];
        ps[i] = cs[P.rope_dim / 2 + ((d - nope) >> 1)];
      }
    }
    auto rope = [&](WarpRow<D>& r) {
#pragma unroll
      for (int i = 0; i < E / 2; ++i) rope_pair(r.v[2 * i], r.v[2 * i + 1], pc[i], ps[i]);
    };
    __nv_bfloat16* qo = P.q_out + t * P.qo_st;
    for (int hb = warp; hb < nrows; hb += kStreamConsumers * kStreamBatch) {
      WarpRow<D> rows[kStreamBatch];
#pragma unroll
      for (int b = 0; b < kStreamBatch; ++b) {
        const int h = hb + b * kStreamConsumers;
        if (h < P.num_heads) rows[b].load_bf16_aligned(qs + h * D, lane);
        else if (h == P.padded_heads)
          rows[b].load_bf16_aligned(reinterpret_cast<const __nv_bfloat16*>(st + P.kv_off), lane);
      }
#pragma unroll
      for (int b = 0; b < kStreamBatch; ++b) {
        const int h = hb + b * kStreamConsumers;
        if (h >= nrows) continue;
        if (h < P.num_heads) {
          WarpRow<D>& row = rows[b];
          float ss = 0.0f;
#pragma unroll
          for (int i = 0; i < E; ++i) ss += row.v[i] * row.v[i];
          ss = warp_sum(ss);
          // ss * (1 / D) == ss / D exactly: D is a power of two
          const float rrms = rsqrtf(ss * (1.0f / static_cast<float>(D)) + P.eps);
#pragma unroll
          for (int i = 0; i < E; ++i) row.v[i] *= rrms;
          rope(row);
          row.store_bf16_aligned(qo + h * D, lane);
        } else if (h < P.padded_heads) {
          uint16_t* o = reinterpret_cast<uint16_t*>(qo + h * D) + lane * E;
#pragma unroll
          for (int i = 0; i < E; ++i) o[i] = 0;
        } else {
          // the KV row: RoPE, fp8 NoPE quant, insert
          const int64_t slot = slot_s[s];
          if (slot < 0) continue;
          WarpRow<D> r2 = rows[b];
          rope(r2);
          const RowGeom g = row_geom(D, P.rope_dim);
          rows[b].store_cache_row(row_ptr(P.cache, slot, P.page_size, P.page_stride, g), P.rope_dim, lane, true,
                                  r2.v);
        }
      }
    }
    __syncwarp();
    if (lane == 0) tc::mbar_arrive(&empty[s]);
  }
}

// Quantise already-rotated rows and insert (one warp per token).
template <int D>
__global__ void quantize_insert_kernel(uint8_t* cache, int page_size, int64_t page_stride,
                                       const __nv_bfloat16* k, int64_t k_stride,
                                       const int64_t* slot_mapping, int num_tokens, int rope_dim) {
  const int lane = threadIdx.x & 31;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= num_tokens) return;
  const int64_t slot = slot_mapping[t];
  if (slot < 0) return;
  WarpRow<D> row;
  row.load_bf16(k + t * k_stride, lane);
  const RowGeom g = row_geom(D, rope_dim);
  row.store_cache_row(row_ptr(cache, slot, page_size, page_stride, g), rope_dim, lane, true, row.v);
}

// Dequantise one cached row into bf16 (one warp per row).
template <int D>
__device__ __forceinline__ void dequant_row_to_bf16(const uint8_t* cache, int64_t slot,
                                                    int page_size, int64_t page_stride,
                                                    int rope_dim, __nv_bfloat16* out, int lane) {
  constexpr int E = D / 32;
  const RowGeom g = row_geom(D, rope_dim);
  const RowPtr p = row_ptr(const_cast<uint8_t*>(cache), slot, page_size, page_stride, g);
  const int d0 = lane * E;
  uint16_t* o = reinterpret_cast<uint16_t*>(out) + d0;
  if (d0 < g.nope) {
    const float sc = exp2i(static_cast<int>(p.scale[d0 / kQuantBlock]) - 127);
#pragma unroll
    for (int i = 0; i < E; ++i) o[i] = float_to_bf16_bits(e4m3_to_float(p.data[d0 + i]) * sc);
  } else {
    const uint16_t* r = reinterpret_cast<const uint16_t*>(p.data + g.nope) + (d0 - g.nope);
#pragma unroll
    for (int i = 0; i < E; ++i) o[i] = r[i];
  }
}

// grid (num_reqs, 32), 4 warps per block; warps stride over gather rows.
template <int D>
__global__ void dequant_gather_kernel(__nv_bfloat16* out, int64_t out_sr, int64_t out_st,
                                      const uint8_t* cache, int page_size, int64_t page_stride,
                                      const int32_t* seq_lens, const int32_t* gather_lens,
                                      const int32_t* bt, int64_t bt_stride, int offset,
                                      int rope_dim) {
  const int b = blockIdx.x;
  const int lane = threadIdx.x & 31;
  const int worker = blockIdx.y * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int nworkers = gridDim.y * (blockDim.x >> 5);
  const int sl = seq_lens[b];
  const int gl = gather_lens ? gather_lens[b] : sl;
  const int start = sl - gl;
  for (int i = worker; i < gl; i += nworkers) {
    const int pos = start + i;
    const int64_t slot =
        static_cast<int64_t>(bt[b * bt_stride + pos / page_size]) * page_size + pos % page_size;
    dequant_row_to_bf16<D>(cache, slot, page_size, page_stride, rope_dim,
                           out + b * out_sr + static_cast<int64_t>(offset + i) * out_st, lane);
  }
}

// ----------------------------------------------------------------------------
// Compressor state save: state[slot] = [kv, score + ape[pos % ratio]].
// ----------------------------------------------------------------------------
__global__ void save_partial_states_kernel(float* state, int64_t s_blk, int64_t s_tok,
                                           const float* kv, int64_t kv_stride,
                                           const float* score, int64_t score_stride,
                                           const float* ape, int64_t ape_stride,
                                           const int64_t* positions, const int64_t* slot_mapping,
                                           int block_size, int head_size, int state_width,
                                           int ratio) {
  pdl_wait_and_release();
  const int64_t t = blockIdx.x;
  const int64_t slot = slot_mapping[t];
  if (slot < 0) return;
  const int64_t blk = slot / block_size;
  float* base = state + blk * s_blk + (slot - blk * block_size) * s_tok;
  const float* a = ape + (positions[t] % ratio) * ape_stride;
  const float* k = kv + t * kv_stride;
  const float* s = score + t * score_stride;
  for (int i = threadIdx.x; i < head_size; i += blockDim.x) {
    base[i] = k[i];
    base[state_width + i] = s[i] + a[i];
  }
}

// ----------------------------------------------------------------------------
// Block compressor: a 512-thread CTA per 32 tokens pools each of them that
// completes a block.  Thread (g, c) owns channel c of token group g (512 / D
// groups split the `ratio` pooled tokens); each thread pools its tokens in
// batches of kPoolBatch with independent loads (online softmax per channel,
// one rescale per batch), the groups merge in shared memory, then the
// D threads of group 0 apply RMSNorm, the NoPE quant of the bf16 rounding,
// and RoPE of the fp32 normed value at the block start position, and store
// the row into the compressed cache.
// ----------------------------------------------------------------------------
constexpr int kCompressThreads = 512;

// Per-thread values of a block's compression that depend only on step
// metadata and weights (position, destination slot, norm weight, RoPE).
struct CompressCtx {
  int64_t p, slot;
  float nw, co, si;
};

// First part of the compression of the block completed by token t: the
// metadata loads, and the state-row offsets of the `ratio` pooled positions
// into row_off (shared memory; the caller synchronises the CTA before
// compress_pool reads them).  Reads no state and no layer activation.
template <int D>
__device__ __forceinline__ CompressCtx compress_begin(int64_t t, int64_t s_blk, int64_t s_tok, const int32_t* t2r,
                                                      const int64_t* positions, const int64_t* kv_slot,
                                                      const int32_t* bt, int64_t bt_stride, int block_size,
                                                      const float* norm_w, const float* cos_sin, int64_t cs_stride,
                                                      int rope_dim, int ratio, int64_t* row_off) {
  CompressCtx x;
  x.p = positions[t];
  x.slot = kv_slot[t];
  const int req = t2r[t];
  const int c = threadIdx.x % D;
  // loads of the epilogue, issued now so they land during the pooling
  x.nw = norm_w[c];
  const int nope = D - rope_dim;
  x.co = 1.0f;
  x.si = 0.0f;
  if (c >= nope) {
    const float* cs = cos_sin + (x.p / ratio) * ratio * cs_stride;
    const int pr = (c - nope) >> 1;
    x.co = cs[pr];
    x.si = cs[rope_dim / 2 + pr];
  }
  // Row offsets of the `ratio` states (all positions are >= 0 at a boundary).
  for (int i = threadIdx.x; i < ratio; i += kCompressThreads) {
    const int64_t pos = x.p - ratio + 1 + i;
    const int64_t blk = bt[req * bt_stride + pos / block_size];
    row_off[i] = blk * s_blk + (pos % block_size) * s_tok;
  }
  return x;
}

constexpr int kPoolBatch = 16;  // pooled states per batch of independent loads

// Running online-softmax state of one (group, channel) thread of the pooling.
struct PoolAcc {
  float m, den, acc;
};

// One batch of kPoolBatch pooled positions (score sc, kv value kv; unused
// members -inf / 0) folded into the running state.
__device__ __forceinline__ void pool_batch(PoolAcc& a, const float* sc, const float* kv) {
  float mb = a.m;
#pragma unroll
  for (int j = 0; j < kPoolBatch; ++j) mb = fmaxf(mb, sc[j]);
  const float f = a.m == -INFINITY ? 0.0f : expf(a.m - mb);
  a.den *= f;
  a.acc *= f;
#pragma unroll
  for (int j = 0; j < kPoolBatch; ++j) {
    const float w = sc[j] == -INFINITY ? 0.0f : expf(sc[j] - mb);
    a.den += w;
    a.acc += w * kv[j];
  }
  a.m = mb;
}

// Start of the last batch of the last token group: the pooled positions from
// here on are the only ones a fast-path compression leaves for after the wait.
template <int D>
__host__ __device__ constexpr int last_pool_batch(int ratio) {
  return (kCompressThreads / D - 1) * ((ratio + kCompressThreads / D - 1) / (kCompressThreads / D)) +
         ((ratio - 1 - (kCompressThreads / D - 1) * ((ratio + kCompressThreads / D - 1) / (kCompressThreads / D))) /
          kPoolBatch) * kPoolBatch;
}

// pool_batch on a batch staged in this thread's column of `pre`
// (pre[j * kCompressThreads] score, pre[(kPoolBatch + j) * kCompressThreads]
// kv): the same operations in the same order, with few registers live.
__device__ __forceinline__ void pool_batch_smem(PoolAcc& a, const float* pre) {
  float mb = a.m;
#pragma unroll
  for (int j = 0; j < kPoolBatch; ++j) mb = fmaxf(mb, pre[j * kCompressThreads]);
  const float f = a.m == -INFINITY ? 0.0f : expf(a.m - mb);
  a.den *= f;
  a.acc *= f;
#pragma unroll
  for (int j = 0; j < kPoolBatch; ++j) {
    const float sc = pre[j * kCompressThreads];
    const float w = sc == -INFINITY ? 0.0f : expf(sc - mb);
    a.den += w;
    a.acc += w * pre[(kPoolBatch + j) * kCompressThreads];
  }
  a.m = mb;
}

// Before the dependency wait: pool this thread's states of earlier steps
// (block positions below n_old) in the batches compress_pool would use, each
// staged through this thread's column of `pre` (pre[j * kCompressThreads +
// tid] score, pre[(kPoolBatch + j) * kCompressThreads + tid] kv).  The batch
// holding position n_old (the last of the last group) is not pooled: it stays
// staged, without its members from this launch, which the state save writes
// into the same slots before compress_pool pools the batch.  row_off must be
// visible to the CTA.
template <int D>
__device__ __forceinline__ void compress_prepool(const float* state, int state_width, int ratio, const int64_t* row_off,
                                                 int n_old, float* pre, PoolAcc& a) {
  constexpr int kGroups = kCompressThreads / D;
  const int c = threadIdx.x % D, grp = threadIdx.x / D;
  const int per = (ratio + kGroups - 1) / kGroups;
  const int i0 = grp * per, i1 = min(ratio, i0 + per);
  float* col = pre + threadIdx.x;
  a.m = -INFINITY;
  a.den = 0.0f;
  a.acc = 0.0f;
  constexpr int kHalf = kPoolBatch / 2;
  for (int b0 = i0; b0 < i1; b0 += kPoolBatch) {
    // half a batch of loads in flight before any is stored (the whole batch
    // at once would not fit the registers of two CTAs per SM)
#pragma unroll
    for (int h = 0; h < kPoolBatch; h += kHalf) {
      float sc[kHalf], kv[kHalf];
#pragma unroll
      for (int j = 0; j < kHalf; ++j) {
        const int i = b0 + h + j;
        const bool ld = i < i1 && i < n_old;
        sc[j] = ld ? __ldcg(state + row_off[i] + state_width + c) : -INFINITY;
        kv[j] = ld ? __ldcg(state + row_off[i] + c) : 0.0f;
      }
#pragma unroll
      for (int j = 0; j < kHalf; ++j) {
        const int i = b0 + h + j;
        if (i < n_old || i >= i1) {  // slots of this launch's states are the save's
          col[(h + j) * kCompressThreads] = sc[j];
          col[(kPoolBatch + h + j) * kCompressThreads] = kv[j];
        }
      }
    }
    if (min(b0 + kPoolBatch, i1) > n_old) break;  // the pending batch
    pool_batch_smem(a, col);
  }
}

// Second part: pool the states, normalise, quantise and store the row (the
// whole CTA; returns with every thread past its last barrier).  pre_pooled:
// nullptr (load and pool every batch here), or this thread's state after
// compress_prepool with the pending batch complete in `pre`.
template <int D>
__device__ __forceinline__ void compress_pool(const CompressCtx& x, const PoolAcc* pre_pooled, const float* pre,
                                              const float* state,
                                              int state_width, float eps, uint8_t* kv_cache, int kv_page_size,
                                              int64_t kv_page_stride, int rope_dim, int ratio, float* red,
                                              const int64_t* row_off, float* part_flat) {
  constexpr int kGroups = kCompressThreads / D;
  constexpr int kSub = kPoolBatch;
  float(*part)[kGroups][D] = reinterpret_cast<float(*)[kGroups][D]>(part_flat);
  const int c = threadIdx.x % D, grp = threadIdx.x / D;
  const RowGeom g = row_geom(D, rope_dim);
  const int nope = g.nope;
  const float nw = x.nw, co = x.co, si = x.si;
  const int64_t slot = x.slot;
  const int per = (ratio + kGroups - 1) / kGroups;
  const int i0 = grp * per, i1 = min(ratio, i0 + per);
  PoolAcc pa;
  if (pre_pooled) {
    // the earlier-step batches were pooled before the wait; the last batch of
    // the last group is staged in pre, this launch's states included
    pa = *pre_pooled;
    const int pend = last_pool_batch<D>(ratio);
    if (pend >= i0 && pend < i1) {
      float sc[kSub], kv[kSub];
#pragma unroll
      for (int j = 0; j < kSub; ++j) {
        sc[j] = pre[j * kCompressThreads + threadIdx.x];
        kv[j] = pre[(kSub + j) * kCompressThreads + threadIdx.x];
      }
      pool_batch(pa, sc, kv);
    }
  } else {
    pa.m = -INFINITY;
    pa.den = 0.0f;
    pa.acc = 0.0f;
    for (int b0 = i0; b0 < i1; b0 += kSub) {
      float sc[kSub], kv[kSub];
#pragma unroll
      for (int j = 0; j < kSub; ++j) {
        const int i = b0 + j;
        // coherent (L2) loads: the fused decode prep pools states that its
        // own CTA saved earlier in the same launch
        sc[j] = i < i1 ? __ldcg(state + row_off[i] + state_width + c) : -INFINITY;
        kv[j] = i < i1 ? __ldcg(state + row_off[i] + c) : 0.0f;
      }
      pool_batch(pa, sc, kv);
    }
  }
  part[0][grp][c] = pa.m;
  part[1][grp][c] = pa.den;
  part[2][grp][c] = pa.acc;
  __syncthreads();
  float comp = 0.0f;
  if (grp == 0) {
    float mm = -INFINITY;
#pragma unroll
    for (int g2 = 0; g2 < kGroups; ++g2) mm = fmaxf(mm, part[0][g2][c]);
    float dd = 0.0f, aa = 0.0f;
#pragma unroll
    for (int g2 = 0; g2 < kGroups; ++g2) {
      const float mg = part[0][g2][c];
      const float w = mg == -INFINITY ? 0.0f : expf(mg - mm);
      dd += part[1][g2][c] * w;
      aa += part[2][g2][c] * w;
    }
    comp = aa / dd;
  }
  const float ss = block_sum(comp * comp, red);
  if (grp != 0) return;  // no barrier below involves the other groups
  const float normed = comp * rsqrtf(ss / static_cast<float>(D) + eps) * nw;
  if (slot < 0) return;  // uniform across the CTA
  const RowPtr dst = row_ptr(kv_cache, slot, kv_page_size, kv_page_stride, g);
  // NoPE: UE8M0 quant of the bf16 rounding; 64-channel blocks = 2 warps.
  const float qv = bf16_round(normed);
  float amax = warp_max(c < nope ? fabsf(qv) : 0.0f);
  // only the D threads of group 0 are left: sync them with a named barrier
  asm volatile("bar.sync 1, %0;\n" ::"r"(D) : "memory");
  if ((c & 31) == 0) red[c >> 5] = amax;
  asm volatile("bar.sync 1, %0;\n" ::"r"(D) : "memory");
  amax = fmaxf(red[(c >> 6) * 2], red[(c >> 6) * 2 + 1]);
  // RoPE partner (adjacent channel) in fp32.
  const float partner = __shfl_xor_sync(0xffffffffu, normed, 1);
  if (c < nope) {
    const int e = ue8m0_exponent(amax, 1e-4f, false);
    dst.data[c] = to_e4m3(qv * exp2i(-e));
    if ((c % kQuantBlock) == 0) dst.scale[c / kQuantBlock] = encode_ue8m0(e);
  } else {
    const bool even = ((c - nope) & 1) == 0;
    const float r = even ? normed * co - partner * si : normed * co + partner * si;
    reinterpret_cast<uint16_t*>(dst.data + nope)[c - nope] = float_to_bf16_bits(r);
  }
  if (c == 0) dst.scale[nope / kQuantBlock] = 0;
}


// The whole compression of the block completed by token t.
template <int D>
__device__ __forceinline__ void compress_token(
    int64_t t, const float* state, int64_t s_blk, int64_t s_tok, int state_width, const int32_t* t2r,
    const int64_t* positions, const int64_t* kv_slot, const int32_t* bt, int64_t bt_stride, int block_size,
    const float* norm_w, float eps, const float* cos_sin, int64_t cs_stride, uint8_t* kv_cache, int kv_page_size,
    int64_t kv_page_stride, int rope_dim, int ratio, float* red, int64_t* row_off, float* part_flat) {
  const CompressCtx x = compress_begin<D>(t, s_blk, s_tok, t2r, positions, kv_slot, bt, bt_stride, block_size, norm_w,
                                          cos_sin, cs_stride, rope_dim, ratio, row_off);
  __syncthreads();
  compress_pool<D>(x, nullptr, nullptr, state, state_width, eps, kv_cache, kv_page_size, kv_page_stride, rope_dim, ratio, red,
                   row_off, part_flat);
}

template <int D>
__global__ void __launch_bounds__(kCompressThreads) compress_kernel(
    const float* state, int64_t s_blk, int64_t s_tok, int state_width, const int32_t* t2r,
    const int64_t* positions, const int64_t* state_slot, const int32_t* bt, int64_t bt_stride,
    int block_size, const float* norm_w, float eps, const float* cos_sin, int64_t cs_stride,
    uint8_t* kv_cache, const int64_t* kv_slot, int kv_page_size, int64_t kv_page_stride,
    int rope_dim, int ratio, int64_t num_tokens) {
  pdl_wait_and_release();
  constexpr int kGroups = kCompressThreads / D;
  __shared__ float red[32];
  __shared__ int64_t row_off[512];
  __shared__ float part[3][kGroups][D];
  __shared__ unsigned boundary_bits;
  // This CTA scans tokens 32 * blockIdx.x .. + 31 (one coalesced load of
  // their positions and state slots) and pools every one that completes a
  // block; a 32-token run holds at most one boundary per request.
  const int64_t tbase = static_cast<int64_t>(blockIdx.x) * 32;
  if (threadIdx.x < 32) {
    const int64_t tt = tbase + threadIdx.x;
    bool b = false;
    if (tt < num_tokens) {
      const int64_t ss = state_slot[tt], pp = positions[tt];
      b = ss >= 0 && (pp + 1) % ratio == 0;
    }
    const unsigned bits = __ballot_sync(0xffffffffu, b);
    if (threadIdx.x == 0) boundary_bits = bits;
  }
  __syncthreads();
  unsigned todo = boundary_bits;
  while (todo) {
    const int64_t t = tbase + (__ffs(todo) - 1);
    todo &= todo - 1;
    compress_token<D>(t, state, s_blk, s_tok, state_width, t2r, positions, kv_slot, bt, bt_stride, block_size,
                      norm_w, eps, cos_sin, cs_stride, kv_cache, kv_page_size, kv_page_stride, rope_dim, ratio, red,
                      row_off, &part[0][0][0]);
    __syncthreads();  // the shared buffers are reused by the next boundary
  }
}

// ----------------------------------------------------------------------------
// Decode prep: the per-layer cache work of a decode step in one launch.
//   CTAs [0, num_reqs): request r.  Its tokens' KV rows (RoPE, fp8 NoPE
//     quant, SWA insert) and compressor states are written, then -- after a
//     block barrier, so the pooling reads the states just saved -- every block
//     one of its tokens completes is pooled into the compressed cache
//     (compress_token, the same code as compress_kernel).  A request's
//     tokens are consecutive positions of that request only, so no other CTA
//     writes the states it pools.
//   CTAs [num_reqs, ...): prep_rows<D>() query rows each (head RMSNorm +
//     RoPE; padding heads written as zeros), 16 / (D / 32) consecutive rows
//     per warp with all their loads issued first.  Two CTAs per SM: the
//     rows are spread over the SMs (the traffic of one SM, not the DRAM,
//     bounds a CTA that streams many rows).
// The arithmetic of every row is the one of qnorm_rope_kv_insert_kernel,
// save_partial_states_kernel and compress_kernel, so the outputs are the
// same bytes as those three launches.
// ----------------------------------------------------------------------------
constexpr int kPrepDynSmem = 2 * kPoolBatch * kCompressThreads * 4;  // 64 KB

template <int D>
constexpr int prep_rows_per_warp() { return 16 / (D / 32); }  // 4 at D=128, 1 at D=512
template <int D>
constexpr int prep_rows() { return (kCompressThreads / 32) * prep_rows_per_warp<D>(); }

struct DecodePrepParams {
  // queries
  __nv_bfloat16* q_out;
  int64_t qo_st, qo_sh;
  int padded_heads;
  const __nv_bfloat16* q;
  int64_t q_st, q_sh;
  int num_heads;
  // KV rows -> SWA cache
  const __nv_bfloat16* kv;
  int64_t kv_stride;
  uint8_t* swa_cache;
  int swa_page;
  int64_t swa_pstride;
  const int64_t* swa_slot;
  // RoPE
  const int64_t* positions;
  const float* cos_sin;
  int64_t cs_stride;
  int rope_dim;
  float eps;
  // compressor states
  const float* st_kv;
  int64_t st_kv_stride;
  const float* st_score;
  int64_t st_score_stride;
  const float* ape;
  int64_t ape_stride;
  float* state;
  int64_t s_blk, s_tok;
  int state_width, state_page;
  const int64_t* state_slot;
  const int32_t* state_bt;
  int64_t state_bt_stride;
  // compressed cache
  const float* norm_w;
  uint8_t* comp_cache;
  const int64_t* comp_slot;
  int comp_page;
  int64_t comp_pstride;
  int ratio;
  // batch
  const int32_t* qsl;
  const int32_t* t2r;
  int num_reqs;
  int64_t num_tokens;
};

template <int D>
__global__ void __launch_bounds__(kCompressThreads, 2) decode_prep_kernel(const DecodePrepParams p) {
  // Reads before pdl_wait() touch only step metadata (positions, slot maps,
  // block tables), weights and the RoPE table; q, kv and the compressor
  // inputs (outputs of the layer's projections) and every store come after.
  pdl_release();
  constexpr int E = WarpRow<D>::E;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  constexpr int kWarps = kCompressThreads / 32;
  const int nope = D - p.rope_dim;
  // this lane's RoPE pairs (dims lane * E + 2i, + 1) at position `pos`
  auto load_cs = [&](int64_t pos, float* pc, float* ps) {
    const float* cs = p.cos_sin + pos * p.cs_stride;
#pragma unroll
    for (int i = 0; i < E / 2; ++i) {
      const int d = lane * E + 2 * i;
      pc[i] = 1.0f;
      ps[i] = 0.0f;
      if (d >= nope) {
        pc[i] = cs[(d - nope) >> 1];
        ps[i] = cs[p.rope_dim / 2 + ((d - nope) >> 1)];
      }
    }
  };
  if (blockIdx.x >= p.num_reqs) {
    // ---------------------------------------------------------- query rows
    constexpr int kRpw = prep_rows_per_warp<D>();
    // 32-bit row arithmetic (the host checks num_tokens * padded_heads < 2^31);
    // one division per warp, then (token, head) stepped row by row
    const int base = (static_cast<int>(blockIdx.x) - p.num_reqs) * prep_rows<D>() + warp * kRpw;
    const int nrows = static_cast<int>(p.num_tokens) * p.padded_heads;
    if (base >= nrows) {
      pdl_wait();
      return;
    }
    WarpRow<D> rows[kRpw];
    int tok[kRpw], head[kRpw];
    {
      int t = base / p.padded_heads, h = base - t * p.padded_heads;
#pragma unroll
      for (int b = 0; b < kRpw; ++b) {
        tok[b] = t;
        head[b] = h;
        if (++h == p.padded_heads) {
          h = 0;
          ++t;
        }
      }
    }
    // cos / sin of the first and last token of these rows, loaded before any
    // store (a store may alias them, so later loads could not be hoisted);
    // with padded_heads >= kRpw no other token occurs
    const int tok_a = tok[0], tok_b = (base + kRpw - 1 < nrows ? base + kRpw - 1 : nrows - 1) / p.padded_heads;
    float ca[E / 2], sa[E / 2], cb[E / 2], sb[E / 2];
    load_cs(p.positions[tok_a], ca, sa);
    load_cs(p.positions[tok_b], cb, sb);
    pdl_wait();  // q is an output of the layer's projection
#pragma unroll
    for (int b = 0; b < kRpw; ++b)
      if (base + b < nrows && head[b] < p.num_heads)
        rows[b].load_bf16(p.q + tok[b] * p.q_st + head[b] * p.q_sh, lane);
#pragma unroll
    for (int b = 0; b < kRpw; ++b) {
      if (base + b >= nrows) continue;
      if (head[b] < p.num_heads) {
        float pc[E / 2], ps[E / 2];
        if (tok[b] == tok_a || tok[b] == tok_b) {
          const bool first = tok[b] == tok_a;
#pragma unroll
          for (int i = 0; i < E / 2; ++i) {
            pc[i] = first ? ca[i] : cb[i];
            ps[i] = first ? sa[i] : sb[i];
          }
        } else {
          load_cs(p.positions[tok[b]], pc, ps);
        }
        WarpRow<D>& row = rows[b];
        float ss = 0.0f;
#pragma unroll
        for (int i = 0; i < E; ++i) ss += row.v[i] * row.v[i];
        ss = warp_sum(ss);
        const float rrms = rsqrtf(ss / static_cast<float>(D) + p.eps);
#pragma unroll
        for (int i = 0; i < E; ++i) row.v[i] *= rrms;
#pragma unroll
        for (int i = 0; i < E / 2; ++i) rope_pair(row.v[2 * i], row.v[2 * i + 1], pc[i], ps[i]);
        row.store_bf16(p.q_out + tok[b] * p.qo_st + head[b] * p.qo_sh, lane);
      } else {
        uint16_t* o = reinterpret_cast<uint16_t*>(p.q_out + tok[b] * p.qo_st + head[b] * p.qo_sh) + lane * E;
#pragma unroll
        for (int i = 0; i < E; ++i) o[i] = 0;
      }
    }
    return;
  }
  // ------------------------------------------------------------ request r
  __shared__ float red[32];
  __shared__ int64_t row_off[512];
  __shared__ float part[3][kCompressThreads / D][D];
  extern __shared__ float pre_s[];  // one pooling batch per thread column: kPrepDynSmem bytes
  const int r = blockIdx.x;
  const int t0 = p.qsl[r], t1 = p.qsl[r + 1];
  const RowGeom g = row_geom(D, p.rope_dim);
  // The first token that completes a block: its metadata loads and state-row
  // offsets are done before the wait (the request's CTA is resident early).
  int jb = -1;
  for (int j = 0; j < t1 - t0; ++j)
    if (p.state_slot[t0 + j] >= 0 && (p.positions[t0 + j] + 1) % p.ratio == 0) {
      jb = j;
      break;
    }
  CompressCtx cx{};
  // Fast path (uniform across the CTA): the block's positions from this
  // launch -- the request's tokens up to the block end, consecutive, all with
  // a state slot -- are at most one pooling batch, the last of the last
  // group.  The earlier-step states (no kernel of this step writes them) are
  // then pooled before the wait, and the pending batch takes this launch's
  // states from shared memory, written where they are saved.
  bool fast = false;
  int64_t blk_start = 0;
  PoolAcc pa{-INFINITY, 0.0f, 0.0f};
  if (jb >= 0) {
    cx = compress_begin<D>(t0 + jb, p.s_blk, p.s_tok, p.t2r, p.positions, p.comp_slot, p.state_bt, p.state_bt_stride,
                           p.state_page, p.norm_w, p.cos_sin, p.cs_stride, p.rope_dim, p.ratio, row_off);
    const int64_t p0 = p.positions[t0], pend = p.positions[t0 + jb];
    const int nnew = static_cast<int>(pend - p0 + 1);
    blk_start = pend - p.ratio + 1;
    fast = nnew >= 1 && nnew <= kPoolBatch && nnew <= p.ratio - last_pool_batch<D>(p.ratio);
    for (int k = 0; fast && k <= jb; ++k)
      fast = p.state_slot[t0 + k] >= 0 && p.positions[t0 + k] == p0 + k;
    __syncthreads();
    if (fast) compress_prepool<D>(p.state, p.state_width, p.ratio, row_off, p.ratio - nnew, pre_s, pa);
  }
  pdl_wait();  // kv and the compressor inputs are outputs of the layer's projections
  // KV rows: one warp per token
  for (int j = warp; j < t1 - t0; j += kWarps) {
    const int64_t t = t0 + j;
    const int64_t slot = p.swa_slot[t];
    if (slot < 0) continue;
    WarpRow<D> row;
    row.load_bf16(p.kv + t * p.kv_stride, lane);
    float pc[E / 2], ps[E / 2];
    load_cs(p.positions[t], pc, ps);
    WarpRow<D> r2 = row;
#pragma unroll
    for (int i = 0; i < E / 2; ++i) rope_pair(r2.v[2 * i], r2.v[2 * i + 1], pc[i], ps[i]);
    row.store_cache_row(row_ptr(p.swa_cache, slot, p.swa_page, p.swa_pstride, g), p.rope_dim, lane, true, r2.v);
  }
  // compressor states: state[slot] = [kv, score + ape[pos % ratio]]
  for (int i = threadIdx.x; i < (t1 - t0) * D; i += kCompressThreads) {
    const int t = t0 + i / D;
    const int c = i % D;
    const int64_t slot64 = p.state_slot[t];
    if (slot64 < 0) continue;
    // 32-bit: a state row is >= 1 KB, so any state cache that fits in device
    // memory has fewer than 2^31 slots; positions are below the model length
    const int slot = static_cast<int>(slot64);
    const int blk = slot / p.state_page;
    float* sb = p.state + blk * p.s_blk + (slot - blk * p.state_page) * p.s_tok;
    const int64_t pos = p.positions[t];
    const int pm = static_cast<int>(pos) % p.ratio;
    const float kvv = p.st_kv[t * p.st_kv_stride + c];
    const float scv = p.st_score[t * p.st_score_stride + c] + p.ape[pm * p.ape_stride + c];
    sb[c] = kvv;
    sb[p.state_width + c] = scv;
    if (fast && pos >= blk_start && pos < blk_start + p.ratio) {
      // this launch's member of the pending batch: the slot of its pooling
      // thread (last group, channel c)
      constexpr int kGroups = kCompressThreads / D;
      const int bi = static_cast<int>(pos - blk_start);
      const int owner = (bi / ((p.ratio + kGroups - 1) / kGroups)) * D + c;
      const int jj = bi - last_pool_batch<D>(p.ratio);
      pre_s[jj * kCompressThreads + owner] = scv;
      pre_s[(kPoolBatch + jj) * kCompressThreads + owner] = kvv;
    }
  }
  __syncthreads();  // the states (and row_off) are visible to the whole CTA
  if (jb >= 0) {
    compress_pool<D>(cx, fast ? &pa : nullptr, pre_s, p.state, p.state_width, p.eps, p.comp_cache, p.comp_page,
                     p.comp_pstride, p.rope_dim, p.ratio, red, row_off, &part[0][0][0]);
    __syncthreads();
  }
  // any further block end among the request's tokens (more than `ratio`
  // tokens per request): metadata and pooling in sequence
  for (int j = jb + 1; jb >= 0 && j < t1 - t0; ++j) {
    const int64_t t = t0 + j;
    if (p.state_slot[t] < 0 || (p.positions[t] + 1) % p.ratio != 0) continue;  // uniform
    compress_token<D>(t, p.state, p.s_blk, p.s_tok, p.state_width, p.t2r, p.positions, p.comp_slot, p.state_bt,
                      p.state_bt_stride, p.state_page, p.norm_w, p.eps, p.cos_sin, p.cs_stride, p.comp_cache,
                      p.comp_page, p.comp_pstride, p.rope_dim, p.ratio, red, row_off, &part[0][0][0]);
    __syncthreads();
  }
}

}  // namespace
}  // namespace hca

using namespace hca;

// Instantiated row widths: the BASELINE head dim 128 and the model's 512.
static bool geom_ok(int head_dim, int rope_dim) {
  return (head_dim == 128 || head_dim == 512) && valid_geom(head_dim, rope_dim);
}

extern "C" int hca_qk_rmsnorm(void* q_out, int64_t q_out_stride, const void* q_in,
                              int64_t q_in_stride, const void* q_weight, int32_t q_size,
                              void* kv_out, int64_t kv_out_stride, const void* kv_in,
                              int64_t kv_in_stride, const void* kv_weight, int32_t kv_size,
                              int32_t num_tokens, float eps, void* stream) {
  HCA_CHECK_ARG(num_tokens >= 0 && q_size > 0 && kv_size > 0);
  if (num_tokens == 0) return HCA_OK;
  HCA_CHECK_ARG(q_out && q_in && q_weight && kv_out && kv_in && kv_weight);
  qk_rmsnorm_kernel<<<dim3(num_tokens, 2), 256, 0, as_stream(stream)>>>(
      static_cast<__nv_bfloat16*>(q_out), q_out_stride, static_cast<const __nv_bfloat16*>(q_in),
      q_in_stride, static_cast<const __nv_bfloat16*>(q_weight), q_size,
      static_cast<__nv_bfloat16*>(kv_out), kv_out_stride,
      static_cast<const __nv_bfloat16*>(kv_in), kv_in_stride,
      static_cast<const __nv_bfloat16*>(kv_weight), kv_size, eps);
  return HCA_LAUNCH_STATUS();
}

extern "C" int hca_qnorm_rope_kv_insert(void* q_out, int64_t q_out_stride_tok,
                                        int64_t q_out_stride_head, int32_t padded_heads,
                                        const void* q, int64_t q_stride_tok,
                                        int64_t q_stride_head, int32_t num_heads, const void* kv,
                                        int64_t kv_stride, uint8_t* swa_cache, int32_t page_size,
                                        int64_t page_stride_bytes, const int64_t* slot_mapping,
                                        const int64_t* positions, const float* cos_sin,
                                        int64_t cos_sin_stride, int32_t num_tokens,
                                        int32_t head_dim, int32_t rope_dim, float eps,
                                        void* stream) {
  HCA_CHECK_ARG(num_tokens >= 0 && num_heads > 0 && padded_heads >= num_heads && page_size > 0);
  if (!geom_ok(head_dim, rope_dim)) return HCA_E_UNSUPPORTED;
  if (num_tokens == 0) return HCA_OK;
  HCA_CHECK_ARG(q_out && q && kv && swa_cache && slot_mapping && positions && cos_sin);
  auto* qo = static_cast<__nv_bfloat16*>(q_out);
  auto* qi = static_cast<const __nv_bfloat16*>(q);
  auto* ki = static_cast<const __nv_bfloat16*>(kv);
  const bool few = num_tokens < 4096;
  // many tokens (prefill) with contiguous heads and 16-byte aligned rows:
  // the streamed kernel (persistent CTAs, bulk copies into a shared-memory ring)
  const auto a16 = [](const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; };
  const int64_t q_bytes = static_cast<int64_t>(num_heads) * head_dim * 2;
  const auto up16 = [](int64_t v) { return (v + 15) / 16 * 16; };
  const int64_t stage_bytes = up16(q_bytes) + head_dim * 2 + up16(rope_dim * 4);
  if (!few && q_stride_head == head_dim && q_out_stride_head == head_dim && a16(q) && a16(q_out) && a16(kv) &&
      a16(cos_sin) && (q_stride_tok * 2) % 16 == 0 && (q_out_stride_tok * 2) % 16 == 0 && (kv_stride * 2) % 16 == 0 &&
      (cos_sin_stride * 4) % 16 == 0 && (rope_dim * 4) % 16 == 0 && 2 * stage_bytes <= 200 * 1024) {
    QPrepStream P;
    P.q_out = qo;
    P.qo_st = q_out_stride_tok;
    P.q = qi;
    P.q_st = q_stride_tok;
    P.kv = ki;
    P.kv_stride = kv_stride;
    P.cache = swa_cache;
    P.page_stride = page_stride_bytes;
    P.slot_mapping = slot_mapping;
    P.positions = positions;
    P.cos_sin = cos_sin;
    P.cs_stride = cos_sin_stride;
    P.err = device_error_word();
    if (!P.err) return HCA_E_CUDA;
    P.page_size = page_size;
    P.padded_heads = padded_heads;
    P.num_heads = num_heads;
    P.rope_dim = rope_dim;
    P.num_tokens = num_tokens;
    P.q_bytes = static_cast<uint32_t>(q_bytes);
    P.kv_off = static_cast<uint32_t>(up16(q_bytes));
    P.cs_off = P.kv_off + head_dim * 2;
    P.stage_bytes = static_cast<uint32_t>(stage_bytes);
    P.eps = eps;
    // ~50 KB of stages per CTA and up to 4 CTAs (~200 KB) per SM: 3 stages
    // x 4 CTAs per SM at 64 heads x 128 dims
    P.stages = static_cast<int>(std::max<int64_t>(2, std::min<int64_t>(kStreamMaxStages, 52000 / stage_bytes)));
    const int64_t smem = P.stages * stage_bytes;
    auto* kfn = head_dim == 128 ? qprep_stream_kernel<128> : qprep_stream_kernel<512>;
    const int threads = 32 * (kStreamConsumers + 1);
    if (cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) != cudaSuccess)
      return HCA_E_CUDA;
    // resident CTAs per SM (registers and shared memory), at most 4
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kfn, threads, static_cast<size_t>(smem)) != cudaSuccess)
      return HCA_E_CUDA;
    per_sm = std::max(1, std::min(4, per_sm));
    const int grid = static_cast<int>(std::min<int64_t>(num_tokens, static_cast<int64_t>(per_sm) * device_sm_count()));
    return launch_pdl(kfn, dim3(grid), dim3(threads), static_cast<size_t>(smem), as_stream(stream), P);
  }
  // few tokens (decode): CTAs of 4 warps over 4 rows each (many small CTAs
  // spread over the SMs); many tokens otherwise: one CTA per token, its
  // padded_heads + 1 rows over 9 warps of 8 rows in flight each (D=128) or 16
  // warps of 4 (D=512)
  const int ysplit = few ? (padded_heads + 1 + 3) / 4 : 1;
  const int threads = few ? 128 : (head_dim == 128 ? 32 * ((padded_heads + 1 + 7) / 8) : 512);
  if (threads > 1024) return HCA_E_UNSUPPORTED;
  return launch_pdl(head_dim == 128 ? qnorm_rope_kv_insert_kernel<128> : qnorm_rope_kv_insert_kernel<512>,
                    dim3(num_tokens, ysplit), dim3(threads), 0, as_stream(stream), qo, q_out_stride_tok, q_out_stride_head, padded_heads, qi,
                    q_stride_tok, q_stride_head, num_heads, ki, kv_stride, swa_cache, page_size,
                    page_stride_bytes, slot_mapping, positions, cos_sin, cos_sin_stride, rope_dim, eps);
}

extern "C" int hca_quantize_insert_k(uint8_t* cache, int32_t page_size, int64_t page_stride_bytes,
                                     const void* k, int64_t k_stride,
                                     const int64_t* slot_mapping, int32_t num_tokens,
                                     int32_t head_dim, int32_t rope_dim, void* stream) {
  HCA_CHECK_ARG(num_tokens >= 0 && page_size > 0);
  if (!geom_ok(head_dim, rope_dim)) return HCA_E_UNSUPPORTED;
  if (num_tokens == 0) return HCA_OK;
  HCA_CHECK_ARG(cache && k && slot_mapping);
  const int grid = cdiv(num_tokens, 4);
  auto* kp = static_cast<const __nv_bfloat16*>(k);
  if (head_dim == 128)
    quantize_insert_kernel<128><<<grid, 128, 0, as_stream(stream)>>>(
        cache, page_size, page_stride_bytes, kp, k_stride, slot_mapping, num_tokens, rope_dim);
  else
    quantize_insert_kernel<512><<<grid, 128, 0, as_stream(stream)>>>(
        cache, page_size, page_stride_bytes, kp, k_stride, slot_mapping, num_tokens, rope_dim);
  return HCA_LAUNCH_STATUS();
}

extern "C" int hca_dequantize_gather_k(void* out, int64_t out_stride_req, int64_t out_stride_tok,
                                       const uint8_t* cache, int32_t page_size,
                                       int64_t page_stride_bytes, const int32_t* seq_lens,
                                       const int32_t* gather_lens, const int32_t* block_table,
                                       int64_t bt_stride, int32_t num_reqs, int32_t offset,
                                       int32_t head_dim, int32_t rope_dim, void* stream) {
  HCA_CHECK_ARG(num_reqs >= 0 && page_size > 0 && offset >= 0);
  if (!geom_ok(head_dim, rope_dim)) return HCA_E_UNSUPPORTED;
  if (num_reqs == 0) return HCA_OK;
  HCA_CHECK_ARG(out && cache && seq_lens && block_table);
  dim3 grid(num_reqs, 32);
  auto* o = static_cast<__nv_bfloat16*>(out);
  if (head_dim == 128)
    dequant_gather_kernel<128><<<grid, 128, 0, as_stream(stream)>>>(
        o, out_stride_req, out_stride_tok, cache, page_size, page_stride_bytes, seq_lens,
        gather_lens, block_table, bt_stride, offset, rope_dim);
  else
    dequant_gather_kernel<512><<<grid, 128, 0, as_stream(stream)>>>(
        o, out_stride_req, out_stride_tok, cache, page_size, page_stride_bytes, seq_lens,
        gather_lens, block_table, bt_stride, offset, rope_dim);
  return HCA_LAUNCH_STATUS();
}

extern "C" int hca_save_partial_states(float* state, int64_t state_stride_block,
                                       int64_t state_stride_tok, const float* kv,
                                       int64_t kv_stride, const float* score,
                                       int64_t score_stride, const float* ape, int64_t ape_stride,
                                       const int64_t* positions, const int64_t* slot_mapping,
                                       int32_t num_tokens, int32_t block_size,
                                       int32_t head_size, int32_t state_width,
                                       int32_t compress_ratio, void* stream) {
  HCA_CHECK_ARG(num_tokens >= 0 && block_size > 0 && head_size > 0 &&
                state_width >= head_size && compress_ratio > 0);
  if (num_tokens == 0) return HCA_OK;
  HCA_CHECK_ARG(state && kv && score && ape && positions && slot_mapping);
  return launch_pdl(save_partial_states_kernel, dim3(num_tokens), dim3(128), 0, as_stream(stream), state,
                    state_stride_block, state_stride_tok, kv, kv_stride, score, score_stride, ape, ape_stride,
                    positions, slot_mapping, block_size, head_size, state_width, compress_ratio);
}

extern "C" int hca_compress_norm_rope_store(
    const float* state, int64_t state_stride_block, int64_t state_stride_tok, int32_t state_width,
    const int32_t* token_to_req, const int64_t* positions, const int64_t* state_slot_mapping,
    const int32_t* block_table, int64_t bt_stride, int32_t block_size, const float* norm_weight,
    float eps, const float* cos_sin, int64_t cos_sin_stride, uint8_t* kv_cache,
    const int64_t* kv_slot_mapping, int32_t kv_page_size, int64_t kv_page_stride_bytes,
    int32_t num_tokens, int32_t head_dim, int32_t rope_dim, int32_t compress_ratio,
    void* stream) {
  HCA_CHECK_ARG(num_tokens >= 0 && block_size > 0 && kv_page_size > 0 &&
                state_width >= head_dim && compress_ratio > 0 && compress_ratio <= 512);
  if (!geom_ok(head_dim, rope_dim)) return HCA_E_UNSUPPORTED;
  if (num_tokens == 0) return HCA_OK;
  HCA_CHECK_ARG(state && token_to_req && positions && state_slot_mapping && block_table &&
                norm_weight && cos_sin && kv_cache && kv_slot_mapping);
  return launch_pdl(head_dim == 128 ? compress_kernel<128> : compress_kernel<512>, dim3((num_tokens + 31) / 32),
                    dim3(kCompressThreads), 0, as_stream(stream), state, state_stride_block, state_stride_tok,
                    state_width, token_to_req, positions, state_slot_mapping, block_table, bt_stride, block_size,
                    norm_weight, eps, cos_sin, cos_sin_stride, kv_cache, kv_slot_mapping, kv_page_size,
                    kv_page_stride_bytes, rope_dim, compress_ratio, static_cast<int64_t>(num_tokens));
}

extern "C" int hca_decode_prep(
    void* q_out, int64_t q_out_stride_tok, int64_t q_out_stride_head, int32_t padded_heads, const void* q,
    int64_t q_stride_tok, int64_t q_stride_head, int32_t num_heads, const void* kv, int64_t kv_stride,
    uint8_t* swa_cache, int32_t swa_page_size, int64_t swa_page_stride_bytes, const int64_t* swa_slot_mapping,
    const int64_t* positions, const float* cos_sin, int64_t cos_sin_stride, const float* state_kv,
    int64_t state_kv_stride, const float* state_score, int64_t state_score_stride, const float* ape,
    int64_t ape_stride, float* state, int64_t state_stride_block, int64_t state_stride_tok, int32_t state_width,
    int32_t state_block_size, const int64_t* state_slot_mapping, const int32_t* state_block_table,
    int64_t state_bt_stride, const float* norm_weight, uint8_t* comp_cache, const int64_t* comp_slot_mapping,
    int32_t comp_page_size, int64_t comp_page_stride_bytes, const int32_t* query_start_loc,
    const int32_t* token_to_req, int32_t num_reqs, int32_t num_tokens, int32_t head_dim, int32_t rope_dim,
    int32_t compress_ratio, float eps, void* stream) {
  HCA_CHECK_ARG(num_tokens >= 0 && num_reqs >= 0 && num_heads > 0 && padded_heads >= num_heads &&
                swa_page_size > 0 && state_block_size > 0 && comp_page_size > 0 && state_width >= head_dim &&
                compress_ratio > 0 && compress_ratio <= 512);
  if (!geom_ok(head_dim, rope_dim)) return HCA_E_UNSUPPORTED;
  if (num_tokens == 0) return HCA_OK;
  HCA_CHECK_ARG(static_cast<int64_t>(num_tokens) * padded_heads < (int64_t(1) << 31));
  HCA_CHECK_ARG(q_out && q && kv && swa_cache && swa_slot_mapping && positions && cos_sin && state_kv &&
                state_score && ape && state && state_slot_mapping && state_block_table && norm_weight && comp_cache &&
                comp_slot_mapping && query_start_loc && token_to_req && num_reqs > 0);
  DecodePrepParams p{};
  p.q_out = static_cast<__nv_bfloat16*>(q_out);
  p.qo_st = q_out_stride_tok;
  p.qo_sh = q_out_stride_head;
  p.padded_heads = padded_heads;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.q_st = q_stride_tok;
  p.q_sh = q_stride_head;
  p.num_heads = num_heads;
  p.kv = static_cast<const __nv_bfloat16*>(kv);
  p.kv_stride = kv_stride;
  p.swa_cache = swa_cache;
  p.swa_page = swa_page_size;
  p.swa_pstride = swa_page_stride_bytes;
  p.swa_slot = swa_slot_mapping;
  p.positions = positions;
  p.cos_sin = cos_sin;
  p.cs_stride = cos_sin_stride;
  p.rope_dim = rope_dim;
  p.eps = eps;
  p.st_kv = state_kv;
  p.st_kv_stride = state_kv_stride;
  p.st_score = state_score;
  p.st_score_stride = state_score_stride;
  p.ape = ape;
  p.ape_stride = ape_stride;
  p.state = state;
  p.s_blk = state_stride_block;
  p.s_tok = state_stride_tok;
  p.state_width = state_width;
  p.state_page = state_block_size;
  p.state_slot = state_slot_mapping;
  p.state_bt = state_block_table;
  p.state_bt_stride = state_bt_stride;
  p.norm_w = norm_weight;
  p.comp_cache = comp_cache;
  p.comp_slot = comp_slot_mapping;
  p.comp_page = comp_page_size;
  p.comp_pstride = comp_page_stride_bytes;
  p.ratio = compress_ratio;
  p.qsl = query_start_loc;
  p.t2r = token_to_req;
  p.num_reqs = num_reqs;
  p.num_tokens = num_tokens;
  const int rows_per_cta = head_dim == 128 ? prep_rows<128>() : prep_rows<512>();
  const int64_t q_ctas = (static_cast<int64_t>(num_tokens) * padded_heads + rows_per_cta - 1) / rows_per_cta;
  auto kernel = head_dim == 128 ? decode_prep_kernel<128> : decode_prep_kernel<512>;
  static bool smem_set[2][kMaxDevices] = {};  // per kernel and device
  if (set_func_attr_once(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kPrepDynSmem, smem_set[head_dim == 512]) !=
      HCA_OK)
    return HCA_E_CUDA;
  return launch_pdl(kernel, dim3(static_cast<unsigned>(num_reqs + q_ctas)), dim3(kCompressThreads), kPrepDynSmem,
                    as_stream(stream), p);
}
