// Output side of the HCA path: VHA head post-mix fused with inverse RoPE and
// the 1x128 UE8M0 FP8 quant that feeds the grouped wo_a einsum, the plain
// inverse-RoPE quant, the bf16 (unquantised) variant, and the sigmoid gate
// fused into wo_b's input quant.
//
// These kernels read the attention output once (T * H * D bf16) and write
// it once as e4m3 -- HBM-bound.  The head mix is a [H x H] x [H x D] product
// per token (H = 64: 0.5 MFLOP/token), done on CUDA cores from L1.
#include "hca_common.cuh"
#include "hca_tc.cuh"

namespace hca {
namespace {

// One CTA per token (padded to aligned_T rows), 8 warps; warp w handles
// heads w, w + 8, ...; lane l owns dims [l*E, (l+1)*E).
//   mode 0: VHA + inverse RoPE + FP8, per-head int32 scale (plugin layout)
//   mode 1: inverse RoPE + FP8, packed int32 scale (vLLM layout), no mix
//   mode 2: VHA + inverse RoPE, bf16 output
template <int D, int MODE>
__global__ void __launch_bounds__(256) vha_out_kernel(
    uint8_t* out_fp8, int32_t* scale, __nv_bfloat16* out_bf16, int64_t ob_st, int64_t ob_sh,
    const __nv_bfloat16* o, int64_t o_st, int64_t o_sh, const __nv_bfloat16* mix,
    const int64_t* positions, const float* cos_sin, int64_t cs_stride, int num_tokens,
    int aligned_t, int num_heads, int n_groups, int rope_dim) {
  constexpr int E = D / 32;
  constexpr int kChunks = D / 128;  // quant chunks per head
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t t = blockIdx.x;
  const int hpg = num_heads / n_groups;
  if (t >= num_tokens) {
    // TMA-aligned padding rows of the scale buffer are zero.
    if (MODE == 0) {
      for (int h = threadIdx.x; h < num_heads; h += blockDim.x) {
        const int g = h / hpg, hh = h % hpg;
        scale[(static_cast<int64_t>(g) * hpg + hh) * aligned_t + t] = 0;
      }
    } else if (MODE == 1) {
      const int packs = (hpg * kChunks + 3) / 4;
      for (int i = threadIdx.x; i < n_groups * packs; i += blockDim.x)
        scale[static_cast<int64_t>(i) * aligned_t + t] = 0;
    }
    return;
  }
  const float* cs = cos_sin + positions[t] * cs_stride;
  const int nope = D - rope_dim;
  const __nv_bfloat16* ot = o + t * o_st;
  for (int h = warp; h < num_heads; h += 8) {
    float y[E];
    if (MODE == 1 || mix == nullptr) {
      const uint16_t* src = reinterpret_cast<const uint16_t*>(ot + h * o_sh) + lane * E;
#pragma unroll
      for (int i = 0; i < E; ++i) y[i] = bf16_bits_to_float(src[i]);
    } else {
#pragma unroll
      for (int i = 0; i < E; ++i) y[i] = 0.0f;
      const __nv_bfloat16* mrow = mix + static_cast<int64_t>(h) * num_heads;
      for (int gh = 0; gh < num_heads; ++gh) {
        const float m = __bfloat162float(mrow[gh]);
        const uint16_t* src = reinterpret_cast<const uint16_t*>(ot + gh * o_sh) + lane * E;
#pragma unroll
        for (int i = 0; i < E; ++i) y[i] = fmaf(m, bf16_bits_to_float(src[i]), y[i]);
      }
    }
    // inverse GPT-J RoPE of the last R dims (pairs never straddle lanes)
#pragma unroll
    for (int i = 0; i < E; i += 2) {
      const int d = lane * E + i;
      if (d >= nope) {
        const int pr = (d - nope) >> 1;
        const float c = cs[pr], s = cs[rope_dim / 2 + pr];
        const float e = y[i], od = y[i + 1];
        y[i] = e * c + od * s;
        y[i + 1] = od * c - e * s;
      }
    }
    if (MODE == 2) {
      uint16_t* dst = reinterpret_cast<uint16_t*>(out_bf16 + t * ob_st + h * ob_sh) + lane * E;
#pragma unroll
      for (int i = 0; i < E; ++i) dst[i] = float_to_bf16_bits(y[i]);
      continue;
    }
    // per-128 amax: 128 / E lanes share a chunk
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < E; ++i) amax = fmaxf(amax, fabsf(y[i]));
#pragma unroll
    for (int off = 1; off < 128 / E; off <<= 1)
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    const int e = ue8m0_exponent(amax, 1e-10f, false);
    const float inv = exp2i(-e);
    const int g = h / hpg, hh = h % hpg;
    uint8_t* dst = out_fp8 + (static_cast<int64_t>(g) * num_tokens + t) * (hpg * D) + hh * D + lane * E;
#pragma unroll
    for (int i = 0; i < E; ++i) dst[i] = to_e4m3(y[i] * inv);
    // exponent byte of chunk k lives in lane k * (128 / E)
    uint32_t packed = 0;
#pragma unroll
    for (int k = 0; k < kChunks; ++k) {
      const int ek = __shfl_sync(0xffffffffu, e, k * (128 / E));
      packed |= static_cast<uint32_t>(encode_ue8m0(ek)) << (8 * k);
    }
    if (lane == 0) {
      if (MODE == 0) {
        scale[(static_cast<int64_t>(g) * hpg + hh) * aligned_t + t] = static_cast<int32_t>(packed);
      } else {
        // chunk index within the group = hh * kChunks + k; pack = idx / 4
        if (kChunks == 4) {
          scale[(static_cast<int64_t>(g) * ((hpg * kChunks + 3) / 4) + hh) * aligned_t + t] =
              static_cast<int32_t>(packed);
        } else {
          const int idx = hh * kChunks;
          unsigned char* b = reinterpret_cast<unsigned char*>(
              scale + (static_cast<int64_t>(g) * ((hpg * kChunks + 3) / 4) + idx / 4) * aligned_t + t);
          b[idx % 4] = static_cast<unsigned char>(packed & 0xff);
        }
      }
    }
  }
}

// ----------------------------------------------------------------------------
// VHA head mix on the tensor cores: one CTA per token row (padded to
// aligned_T), H / 16 warps; warp w computes heads 16w .. 16w+15 of
// y = mix @ o[t] (m16n8k16 bf16 -> fp32) 128 dims at a time, applies the
// inverse RoPE in registers (pairs never straddle a thread) and either
// quantises per (head, 128-chunk) to e4m3 (MODE 0) or stores bf16 (MODE 2).
// ----------------------------------------------------------------------------
__device__ __forceinline__ void mma16816_o(float* c, const uint32_t* a, const uint32_t* b) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

__device__ __forceinline__ void ldsm_x4(uint32_t* r, const void* p, bool trans) {
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p));
  if (trans)
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(a));
  else
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(a));
}

template <int D, int MODE>
__global__ void __launch_bounds__(256) vha_mma_kernel(uint8_t* out_fp8, int32_t* scale, __nv_bfloat16* out_bf16,
                                                      int64_t ob_st, int64_t ob_sh, const __nv_bfloat16* o,
                                                      int64_t o_st, int64_t o_sh, const __nv_bfloat16* mix,
                                                      const int64_t* positions, const float* cos_sin,
                                                      int64_t cs_stride, int num_tokens, int aligned_t,
                                                      int num_heads, int n_groups, int rope_dim) {
  pdl_wait_and_release();
  constexpr int kCk = 128;             // dims per pass
  constexpr int kMaxH = 64;            // heads of one (TP-local) layer
  constexpr int kMixStride = kMaxH + 8;  // padded rows: conflict-free ldmatrix
  constexpr int kOStride = kCk + 8;
  constexpr int kChunks = D / kCk;
  __shared__ __align__(16) __nv_bfloat16 mix_s[kMaxH * kMixStride];
  __shared__ __align__(16) __nv_bfloat16 o_s[kMaxH * kOStride];
  const int H = num_heads;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t t = blockIdx.x;
  const int hpg = H / n_groups;
  if (t >= num_tokens) {
    if (MODE == 0)
      for (int h = threadIdx.x; h < H; h += blockDim.x)
        scale[(static_cast<int64_t>(h / hpg) * hpg + h % hpg) * aligned_t + t] = 0;
    return;
  }
  for (int i = threadIdx.x; i < H * (H / 8); i += blockDim.x) {
    const int r = i / (H / 8), c8 = i % (H / 8);
    *reinterpret_cast<uint4*>(&mix_s[r * kMixStride + c8 * 8]) =
        *reinterpret_cast<const uint4*>(mix + static_cast<int64_t>(r) * H + c8 * 8);
  }
  const float* cs = cos_sin + positions[t] * cs_stride;
  const int nope = D - rope_dim;
  const int g = lane >> 2, cq = lane & 3;
  const int h0 = warp * 16 + g, h1 = h0 + 8;
  uint32_t packed0 = 0, packed1 = 0;  // exponent bytes of heads h0 / h1
  for (int ck = 0; ck < kChunks; ++ck) {
    __syncthreads();
    for (int i = threadIdx.x; i < H * (kCk / 8); i += blockDim.x) {
      const int r = i / (kCk / 8), c8 = i % (kCk / 8);
      *reinterpret_cast<uint4*>(&o_s[r * kOStride + c8 * 8]) =
          *reinterpret_cast<const uint4*>(o + t * o_st + r * o_sh + ck * kCk + c8 * 8);
    }
    __syncthreads();
    if (warp * 16 >= H) continue;
    float acc[kCk / 8][4];
#pragma unroll
    for (int j = 0; j < kCk / 8; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.0f;
    for (int kk = 0; kk < H / 16; ++kk) {
      uint32_t a[4];
      ldsm_x4(a, &mix_s[(warp * 16 + (lane & 15)) * kMixStride + kk * 16 + (lane >> 4) * 8], false);
#pragma unroll
      for (int j = 0; j < kCk / 8; j += 2) {
        uint32_t b[4];
        ldsm_x4(b, &o_s[(kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8) * kOStride + j * 8 + (lane >> 4) * 8], true);
        mma16816_o(acc[j], a, b);
        mma16816_o(acc[j + 1], a, b + 2);
      }
    }
    // inverse GPT-J RoPE on the dims >= nope
#pragma unroll
    for (int j = 0; j < kCk / 8; ++j) {
      const int d = ck * kCk + j * 8 + 2 * cq;
      if (d >= nope) {
        const int pr = (d - nope) >> 1;
        const float c = cs[pr], s = cs[rope_dim / 2 + pr];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const float e = acc[j][2 * h], od = acc[j][2 * h + 1];
          acc[j][2 * h] = e * c + od * s;
          acc[j][2 * h + 1] = od * c - e * s;
        }
      }
    }
    if (MODE == 2) {
#pragma unroll
      for (int j = 0; j < kCk / 8; ++j) {
        const int d = ck * kCk + j * 8 + 2 * cq;
        __nv_bfloat162 v0 = __floats2bfloat162_rn(acc[j][0], acc[j][1]);
        __nv_bfloat162 v1 = __floats2bfloat162_rn(acc[j][2], acc[j][3]);
        *reinterpret_cast<__nv_bfloat162*>(out_bf16 + t * ob_st + h0 * ob_sh + d) = v0;
        *reinterpret_cast<__nv_bfloat162*>(out_bf16 + t * ob_st + h1 * ob_sh + d) = v1;
      }
      continue;
    }
    float am0 = 0.0f, am1 = 0.0f;
#pragma unroll
    for (int j = 0; j < kCk / 8; ++j) {
      am0 = fmaxf(am0, fmaxf(fabsf(acc[j][0]), fabsf(acc[j][1])));
      am1 = fmaxf(am1, fmaxf(fabsf(acc[j][2]), fabsf(acc[j][3])));
    }
#pragma unroll
    for (int off = 1; off < 4; off <<= 1) {
      am0 = fmaxf(am0, __shfl_xor_sync(0xffffffffu, am0, off));
      am1 = fmaxf(am1, __shfl_xor_sync(0xffffffffu, am1, off));
    }
    const int e0 = ue8m0_exponent(am0, 1e-10f, false), e1 = ue8m0_exponent(am1, 1e-10f, false);
    const float i0 = exp2i(-e0), i1 = exp2i(-e1);
    packed0 |= static_cast<uint32_t>(encode_ue8m0(e0)) << (8 * ck);
    packed1 |= static_cast<uint32_t>(encode_ue8m0(e1)) << (8 * ck);
    uint8_t* r0 = out_fp8 + (static_cast<int64_t>(h0 / hpg) * num_tokens + t) * (hpg * D) + (h0 % hpg) * D;
    uint8_t* r1 = out_fp8 + (static_cast<int64_t>(h1 / hpg) * num_tokens + t) * (hpg * D) + (h1 % hpg) * D;
#pragma unroll
    for (int j = 0; j < kCk / 8; ++j) {
      const int d = ck * kCk + j * 8 + 2 * cq;
      *reinterpret_cast<uint16_t*>(r0 + d) =
          static_cast<uint16_t>(to_e4m3(acc[j][0] * i0) | (to_e4m3(acc[j][1] * i0) << 8));
      *reinterpret_cast<uint16_t*>(r1 + d) =
          static_cast<uint16_t>(to_e4m3(acc[j][2] * i1) | (to_e4m3(acc[j][3] * i1) << 8));
    }
  }
  if (MODE == 0 && cq == 0 && warp * 16 < H) {
    scale[(static_cast<int64_t>(h0 / hpg) * hpg + h0 % hpg) * aligned_t + t] = static_cast<int32_t>(packed0);
    scale[(static_cast<int64_t>(h1 / hpg) * hpg + h1 % hpg) * aligned_t + t] = static_cast<int32_t>(packed1);
  }
}

// ----------------------------------------------------------------------------
// Multi-token VHA mix: a CTA of 8 warps handles `tpc` consecutive tokens with
// the mix loaded once.  Warp w: heads 16 (w % 4) .. +15, dims 64 (w / 4) ..
// +63 of each 128-dim chunk.  The O chunk and the cos / sin row of the next
// (token, chunk) stream in by cp.async (double buffer) while the current one
// is mixed, rotated back, and quantised per (head, 128 dims) -- the amax of
// the two dim halves meets in shared memory -- (MODE 0) or stored bf16 (MODE 2).
// ----------------------------------------------------------------------------
__device__ __forceinline__ void cp16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
               "l"(src)
               : "memory");
}

constexpr int kVhaStages = 3;
constexpr int kVhaDynSmem = kVhaStages * 64 * (128 + 8) * 2;

template <int D, int MODE>
__global__ void __launch_bounds__(256, 3) vha_tok_kernel(uint8_t* out_fp8, int32_t* scale, __nv_bfloat16* out_bf16,
                                                         int64_t ob_st, int64_t ob_sh, const __nv_bfloat16* o,
                                                         int64_t o_st, int64_t o_sh, const __nv_bfloat16* mix,
                                                         const int64_t* positions, const float* cos_sin,
                                                         int64_t cs_stride, int num_tokens, int aligned_t,
                                                         int num_heads, int n_groups, int rope_dim, int tpc) {
  pdl_wait_and_release();
  constexpr int kCk = 128, kMaxH = 64, kMixStride = kMaxH + 8, kOStride = kCk + 8, kChunks = D / kCk;
  __shared__ __align__(16) __nv_bfloat16 mix_s[kMaxH * kMixStride];
  constexpr int kStages = kVhaStages;  // O chunks in flight: the next two stream in while one is mixed
  extern __shared__ __align__(16) uint8_t vha_dyn[];
  auto o_s = reinterpret_cast<__nv_bfloat16(*)[kMaxH * kOStride]>(vha_dyn);  // [kStages][...]
  __shared__ __align__(16) float cs_s[kStages][64];
  __shared__ float amax_s[2][kMaxH];
  const int H = num_heads, hpg = H / n_groups, nope = D - rope_dim;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int ht = warp & 3, dh = warp >> 2, gq = lane >> 2, cq = lane & 3;
  const int h0 = ht * 16 + gq, h1 = h0 + 8;
  const bool active = ht * 16 < H;
  const int t_begin = blockIdx.x * tpc;
  const int t_end = min(t_begin + tpc, num_tokens);
  if (MODE == 0)
    for (int t = max(t_begin, num_tokens); t < min(t_begin + tpc, aligned_t); ++t)
      for (int h = threadIdx.x; h < H; h += blockDim.x) scale[static_cast<int64_t>(h) * aligned_t + t] = 0;
  const int items = max(0, t_end - t_begin) * kChunks;
  if (items == 0) return;
  for (int i = threadIdx.x; i < H * (H / 8); i += blockDim.x) {
    const int r = i / (H / 8), c8 = i % (H / 8);
    cp16(&mix_s[r * kMixStride + c8 * 8], mix + static_cast<int64_t>(r) * H + c8 * 8);
  }
  // O chunk + cos / sin row of item k into buffer k % kStages
  auto prefetch = [&](int k) {
    const int t = t_begin + k / kChunks, ck = k % kChunks;
    const int b = k % kStages;
    for (int i = threadIdx.x; i < H * (kCk / 8); i += blockDim.x) {
      const int r = i / (kCk / 8), c8 = i % (kCk / 8);
      cp16(&o_s[b][r * kOStride + c8 * 8], o + static_cast<int64_t>(t) * o_st + static_cast<int64_t>(r) * o_sh + ck * kCk + c8 * 8);
    }
    // cos / sin rows rotate by token (a token's chunks all read its row;
    // at most kStages - 1 items, so fewer tokens, are ahead of the current one)
    if (ck == 0 && threadIdx.x < rope_dim / 4)
      cp16(&cs_s[(t - t_begin) % kStages][threadIdx.x * 4], cos_sin + positions[t] * cs_stride + threadIdx.x * 4);
  };
#pragma unroll
  for (int k = 0; k < kStages - 1; ++k) {
    if (k < items) prefetch(k);
    asm volatile("cp.async.commit_group;\n" ::: "memory");
  }
  uint32_t packed0 = 0, packed1 = 0;
  for (int k = 0; k < items; ++k) {
    const int t = t_begin + k / kChunks, ck = k % kChunks, b = k % kStages;
    if (k + kStages - 1 < items) prefetch(k + kStages - 1);
    asm volatile("cp.async.commit_group;\n" ::: "memory");
    asm volatile("cp.async.wait_group %0;\n" ::"n"(kStages - 1) : "memory");
    __syncthreads();
    float acc[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.0f;
    if (active) {
      for (int kk = 0; kk < H / 16; ++kk) {
        uint32_t a[4];
        ldsm_x4(a, &mix_s[(ht * 16 + (lane & 15)) * kMixStride + kk * 16 + (lane >> 4) * 8], false);
#pragma unroll
        for (int j = 0; j < 8; j += 2) {
          uint32_t bq[4];
          ldsm_x4(bq, &o_s[b][(kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8) * kOStride + dh * 64 + j * 8 + (lane >> 4) * 8],
                  true);
          mma16816_o(acc[j], a, bq);
          mma16816_o(acc[j + 1], a, bq + 2);
        }
      }
      const float* cs = cs_s[(t - t_begin) % kStages];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int d = ck * kCk + dh * 64 + j * 8 + 2 * cq;
        if (d >= nope) {
          const int pr = (d - nope) >> 1;
          const float c = cs[pr], sn = cs[rope_dim / 2 + pr];
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const float e = acc[j][2 * hh], od = acc[j][2 * hh + 1];
            acc[j][2 * hh] = e * c + od * sn;
            acc[j][2 * hh + 1] = od * c - e * sn;
          }
        }
      }
    }
    if (MODE == 2) {
      if (active) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int d = ck * kCk + dh * 64 + j * 8 + 2 * cq;
          *reinterpret_cast<__nv_bfloat162*>(out_bf16 + t * ob_st + h0 * ob_sh + d) = __floats2bfloat162_rn(acc[j][0], acc[j][1]);
          *reinterpret_cast<__nv_bfloat162*>(out_bf16 + t * ob_st + h1 * ob_sh + d) = __floats2bfloat162_rn(acc[j][2], acc[j][3]);
        }
      }
      __syncthreads();  // buffer b is refilled kStages items on
      continue;
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
    if (active && cq == 0) {
      amax_s[dh][h0] = am0;
      amax_s[dh][h1] = am1;
    }
    __syncthreads();
    if (active) {
      const float a0 = fmaxf(amax_s[0][h0], amax_s[1][h0]), a1 = fmaxf(amax_s[0][h1], amax_s[1][h1]);
      const int e0 = ue8m0_exponent(a0, 1e-10f, false), e1 = ue8m0_exponent(a1, 1e-10f, false);
      const float i0 = exp2i(-e0), i1 = exp2i(-e1);
      uint8_t* r0 = out_fp8 + (static_cast<int64_t>(h0 / hpg) * num_tokens + t) * (hpg * D) + (h0 % hpg) * D;
      uint8_t* r1 = out_fp8 + (static_cast<int64_t>(h1 / hpg) * num_tokens + t) * (hpg * D) + (h1 % hpg) * D;
      uint32_t p0[8], p1[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        p0[j] = to_e4m3(acc[j][0] * i0) | (to_e4m3(acc[j][1] * i0) << 8);
        p1[j] = to_e4m3(acc[j][2] * i1) | (to_e4m3(acc[j][3] * i1) << 8);
      }
      // 16 contiguous bytes per lane: one full-sector store instead of eight 2-byte ones
      const int dseg = ck * kCk + dh * 64 + 16 * cq;
      *reinterpret_cast<uint4*>(r0 + dseg) = quad_gather_fp8(p0, cq);
      *reinterpret_cast<uint4*>(r1 + dseg) = quad_gather_fp8(p1, cq);
      if (ck == 0) packed0 = packed1 = 0;
      packed0 |= static_cast<uint32_t>(encode_ue8m0(e0)) << (8 * ck);
      packed1 |= static_cast<uint32_t>(encode_ue8m0(e1)) << (8 * ck);
      if (ck == kChunks - 1 && dh == 0 && cq == 0) {
        scale[(static_cast<int64_t>(h0 / hpg) * hpg + h0 % hpg) * aligned_t + t] = static_cast<int32_t>(packed0);
        scale[(static_cast<int64_t>(h1 / hpg) * hpg + h1 % hpg) * aligned_t + t] = static_cast<int32_t>(packed1);
      }
    }
    __syncthreads();  // amax_s and buffer b are reused
  }
}

// ----------------------------------------------------------------------------
// Streamed VHA + inverse RoPE + FP8 quant for many tokens (prefill, D=128,
// plugin scale layout).  Persistent CTAs walk tokens t = blockIdx.x,
// + gridDim.x, ...  Warp 4 (the producer) copies each token's H rows of O
// (256 bytes each, one bulk async copy per row into rows padded to 272 bytes,
// so the transposed ldmatrix reads are free of bank conflicts) and its cos /
// sin row into the next stage of a shared-memory ring.  The H / 16 consumer
// warps of a group each own 16 output heads x all 128 dims: their mix rows
// stay in registers for the whole kernel, the head amax is a quad shuffle,
// and the stage is released right after the MMAs and the RoPE, before the
// quant and stores.  With H < 64 several groups work on alternate tokens.
// Per element the arithmetic is the one of vha_tok_kernel<128, 0> (same MMA
// order over the heads), so both write identical bytes.
// ----------------------------------------------------------------------------
constexpr int kVsConsumers = 4;         // consumer warps; warp 4 is the producer
constexpr int kVsStages = 4;
constexpr int kVsRowBytes = 272;        // 256 bytes of O + 16 of padding
constexpr int kVsStageBytes = 64 * kVsRowBytes + 256;  // H <= 64 rows + cos / sin (R <= 64)
constexpr int kVsDynSmem = kVsStages * kVsStageBytes;
constexpr int kVsErrBit = 1 << 5;

struct VhaStream {
  uint8_t* out_fp8;
  int32_t* scale;
  const __nv_bfloat16* o;
  int64_t o_st, o_sh;
  const __nv_bfloat16* mix;
  const int64_t* positions;
  const float* cos_sin;
  int64_t cs_stride;
  int* err;
  int num_tokens, aligned_t, num_heads, n_groups, rope_dim;
};

// m16n8k16 with a zero accumulator input (the first k block of a tile).
__device__ __forceinline__ void mma16816_z(float* c, const uint32_t* a, const uint32_t* b) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%10,%10,%10,%10};\n"
      : "=f"(c[0]), "=f"(c[1]), "=f"(c[2]), "=f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]), "f"(0.0f));
}

// (x * s, y * s) with one packed instruction (each product rounded as fmul.rn).
__device__ __forceinline__ float2 mul2(float x, float y, float s) {
  uint64_t d;
  const float2 a = make_float2(x, y), b = make_float2(s, s);
  asm("mul.rn.f32x2 %0, %1, %2;\n"
      : "=l"(d)
      : "l"(*reinterpret_cast<const uint64_t*>(&a)), "l"(*reinterpret_cast<const uint64_t*>(&b)));
  return *reinterpret_cast<float2*>(&d);
}

// Two e4m3 conversions (clamp to +-448, round to nearest even) in one
// instruction: lo in bits 0-7, hi in bits 8-15.
__device__ __forceinline__ uint32_t e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;\n" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

template <int kH>
__global__ void __launch_bounds__(32 * (kVsConsumers + 1), 3) vha_stream_kernel(const VhaStream P) {
  extern __shared__ __align__(128) uint8_t vs_ring[];
  __shared__ __align__(8) uint64_t full[kVsStages], empty[kVsStages];
  constexpr int D = 128, kRope = 64, kNope = D - kRope, kMixStride = 64 + 8;
  constexpr int kWpg = kH / 16;             // consumer warps per token
  constexpr int kG = kVsConsumers / kWpg;   // token groups
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int hpg = kH / P.n_groups;
  const int grp = warp / kWpg, mem = warp % kWpg;
  // the mix (a weight, not written by the previous kernel) is staged in the
  // ring before the dependency wait; each consumer warp keeps its 16 rows as
  // MMA A fragments
  __nv_bfloat16* mix_s = reinterpret_cast<__nv_bfloat16*>(vs_ring);
  for (int i = threadIdx.x; i < kH * (kH / 8); i += blockDim.x) {
    const int r = i / (kH / 8), c8 = i % (kH / 8);
    cp16(&mix_s[r * kMixStride + c8 * 8], P.mix + static_cast<int64_t>(r) * kH + c8 * 8);
  }
  asm volatile("cp.async.commit_group;\n" ::: "memory");
  if (threadIdx.x == 0) {
    for (int s = 0; s < kVsStages; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], kWpg);
    }
    tc::mbar_fence_init();
  }
  asm volatile("cp.async.wait_group 0;\n" ::: "memory");
  __syncthreads();
  uint32_t a[kH / 16][4];
  if (warp < kVsConsumers) {
#pragma unroll
    for (int kk = 0; kk < kH / 16; ++kk)
      ldsm_x4(a[kk], &mix_s[(mem * 16 + (lane & 15)) * kMixStride + kk * 16 + (lane >> 4) * 8], false);
  }
  __syncthreads();  // the ring is overwritten from here on
  pdl_wait_and_release();
  const int T = P.num_tokens;
  if (blockIdx.x == 0)
    for (int i = threadIdx.x; i < (P.aligned_t - T) * kH; i += blockDim.x)
      P.scale[static_cast<int64_t>(i % kH) * P.aligned_t + T + i / kH] = 0;
  if (warp == kVsConsumers) {
    // producer: positions of the next 32 tokens of this CTA, one per lane
    int64_t pos_l = 0;
    for (int k = 0;; ++k) {
      const int64_t t = blockIdx.x + static_cast<int64_t>(k) * gridDim.x;
      if (t >= T) break;
      if ((k & 31) == 0) {
        const int64_t tl = t + static_cast<int64_t>(lane) * gridDim.x;
        pos_l = tl < T ? P.positions[tl] : 0;
      }
      const int64_t pos = __shfl_sync(0xffffffffu, pos_l, k & 31);
      const int s = k % kVsStages, n = k / kVsStages;
      int ok = 1;
      if (lane == 0) {
        if (n > 0 && !tc::mbar_wait(&empty[s], (n - 1) & 1)) ok = 0;
        if (ok) tc::mbar_arrive_expect_tx(&full[s], kH * 256 + kRope * 4);
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) {
        if (lane == 0) atomicOr(P.err, kVsErrBit);
        break;
      }
      uint8_t* st = vs_ring + s * kVsStageBytes;
#pragma unroll
      for (int r = lane; r < kH; r += 32)
        tc::bulk_copy_g2s(st + r * kVsRowBytes, P.o + t * P.o_st + r * P.o_sh, 256, &full[s]);
      if (lane == 0) tc::bulk_copy_g2s(st + 64 * kVsRowBytes, P.cos_sin + pos * P.cs_stride, kRope * 4, &full[s]);
    }
    return;
  }
  const int gq = lane >> 2, cq = lane & 3;
  const int h0 = mem * 16 + gq, h1 = h0 + 8;
  uint8_t* r0b = P.out_fp8 + (static_cast<int64_t>(h0 / hpg) * T) * (hpg * D) + (h0 % hpg) * D + 16 * cq;
  uint8_t* r1b = P.out_fp8 + (static_cast<int64_t>(h1 / hpg) * T) * (hpg * D) + (h1 % hpg) * D + 16 * cq;
  // this lane's ldmatrix row within a 16-row k block, and its column
  const uint32_t ring_u32 = tc::smem_u32(vs_ring);
  const uint32_t ld_off = ((lane & 7) + ((lane >> 3) & 1) * 8) * kVsRowBytes + (lane >> 4) * 16;
  for (int k = grp;; k += kG) {
    const int64_t t = blockIdx.x + static_cast<int64_t>(k) * gridDim.x;
    if (t >= T) break;
    const int s = k % kVsStages;
    if (!tc::mbar_wait(&full[s], (k / kVsStages) & 1)) {
      if (lane == 0) atomicOr(P.err, kVsErrBit);
      break;
    }
    const uint32_t st = ring_u32 + s * kVsStageBytes;
    const float* cs = reinterpret_cast<const float*>(vs_ring + s * kVsStageBytes + 64 * kVsRowBytes);
    float acc[16][4];
#pragma unroll
    for (int kk = 0; kk < kH / 16; ++kk) {
#pragma unroll
      for (int j = 0; j < 16; j += 2) {
        uint32_t bq[4];
        asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                     : "=r"(bq[0]), "=r"(bq[1]), "=r"(bq[2]), "=r"(bq[3])
                     : "r"(st + ld_off + kk * 16 * kVsRowBytes + j * 16));
        if (kk == 0) {
          mma16816_z(acc[j], a[kk], bq);
          mma16816_z(acc[j + 1], a[kk], bq + 2);
        } else {
          mma16816_o(acc[j], a[kk], bq);
          mma16816_o(acc[j + 1], a[kk], bq + 2);
        }
      }
    }
    // inverse GPT-J RoPE: columns 8 j + 2 cq, + 1 are RoPE dims for j >= 8
#pragma unroll
    for (int j = kNope / 8; j < 16; ++j) {
      const int pr = (j * 8 + 2 * cq - kNope) >> 1;
      const float c = cs[pr], sn = cs[kRope / 2 + pr];
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const float e = acc[j][2 * hh], od = acc[j][2 * hh + 1];
        acc[j][2 * hh] = e * c + od * sn;
        acc[j][2 * hh + 1] = od * c - e * sn;
      }
    }
    __syncwarp();
    if (lane == 0) tc::mbar_arrive(&empty[s]);
    // head amax (max is exact in any order: a tree, then over the quad)
    float m0[8], m1[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      m0[j] = fmaxf(fmaxf(fabsf(acc[j][0]), fabsf(acc[j][1])), fmaxf(fabsf(acc[j + 8][0]), fabsf(acc[j + 8][1])));
      m1[j] = fmaxf(fmaxf(fabsf(acc[j][2]), fabsf(acc[j][3])), fmaxf(fabsf(acc[j + 8][2]), fabsf(acc[j + 8][3])));
    }
#pragma unroll
    for (int w = 4; w > 0; w >>= 1)
#pragma unroll
      for (int j = 0; j < w; ++j) {
        m0[j] = fmaxf(m0[j], m0[j + w]);
        m1[j] = fmaxf(m1[j], m1[j + w]);
      }
    float am0 = m0[0], am1 = m1[0];
#pragma unroll
    for (int off = 1; off < 4; off <<= 1) {
      am0 = fmaxf(am0, __shfl_xor_sync(0xffffffffu, am0, off));
      am1 = fmaxf(am1, __shfl_xor_sync(0xffffffffu, am1, off));
    }
    const int e0 = ue8m0_exponent(am0, 1e-10f, false), e1 = ue8m0_exponent(am1, 1e-10f, false);
    const float i0 = exp2i(-e0), i1 = exp2i(-e1);
    uint8_t* r0 = r0b + t * (hpg * D);
    uint8_t* r1 = r1b + t * (hpg * D);
#pragma unroll
    for (int seg = 0; seg < 2; ++seg) {
      uint32_t p0[8], p1[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float2 y0 = mul2(acc[seg * 8 + j][0], acc[seg * 8 + j][1], i0);
        const float2 y1 = mul2(acc[seg * 8 + j][2], acc[seg * 8 + j][3], i1);
        p0[j] = e4m3x2(y0.x, y0.y);
        p1[j] = e4m3x2(y1.x, y1.y);
      }
      *reinterpret_cast<uint4*>(r0 + seg * 64) = quad_gather_fp8(p0, cq);
      *reinterpret_cast<uint4*>(r1 + seg * 64) = quad_gather_fp8(p1, cq);
    }
    if (cq == 0) {
      P.scale[static_cast<int64_t>(h0) * P.aligned_t + t] = static_cast<int32_t>(encode_ue8m0(e0));
      P.scale[static_cast<int64_t>(h1) * P.aligned_t + t] = static_cast<int32_t>(encode_ue8m0(e1));
    }
  }
}

// x * sigmoid(gate) -> 1x128 FP8; one CTA of 128 threads per (512-col pack, row).
__global__ void __launch_bounds__(128) sigmoid_mul_quant_kernel(
    uint8_t* out, int32_t* scale, const __nv_bfloat16* x, int64_t x_stride,
    const __nv_bfloat16* gate, int64_t g_stride, int rows, int hidden, int aligned_rows) {
  __shared__ int exps[4];
  const int pack = blockIdx.x;
  const int64_t r = blockIdx.y;
  const int col = pack * 512 + threadIdx.x * 4;
  float y[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float gv = __bfloat162float(gate[r * g_stride + col + i]);
    const float s = bf16_round(1.0f / (1.0f + expf(-gv)));
    y[i] = bf16_round(__bfloat162float(x[r * x_stride + col + i]) * s);
  }
  float amax = fmaxf(fmaxf(fabsf(y[0]), fabsf(y[1])), fmaxf(fabsf(y[2]), fabsf(y[3])));
  amax = warp_max(amax);
  const int e = ue8m0_exponent(amax, 1e-10f, false);
  const float inv = exp2i(-e);
  uint32_t q = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) q |= static_cast<uint32_t>(to_e4m3(y[i] * inv)) << (8 * i);
  *reinterpret_cast<uint32_t*>(out + r * hidden + col) = q;
  if ((threadIdx.x & 31) == 0) exps[threadIdx.x >> 5] = e;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t packed = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) packed |= static_cast<uint32_t>(exps[k] + 127) << (8 * k);
    scale[static_cast<int64_t>(pack) * aligned_rows + r] = static_cast<int32_t>(packed);
  }
}

template <int MODE>
int launch_vha(uint8_t* out_fp8, int32_t* scale, __nv_bfloat16* out_bf16, int64_t ob_st,
               int64_t ob_sh, const void* o, int64_t o_st, int64_t o_sh, const void* mix,
               const int64_t* positions, const float* cos_sin, int64_t cs_stride, int num_tokens,
               int num_heads, int n_groups, int head_dim, int rope_dim, cudaStream_t s) {
  const int aligned = MODE == 2 ? num_tokens : (num_tokens + 3) / 4 * 4;
  if (aligned == 0) return HCA_OK;
  auto* op = static_cast<const __nv_bfloat16*>(o);
  auto* mp = static_cast<const __nv_bfloat16*>(mix);
  if (MODE != 1 && mp != nullptr) {
    // head mix on the tensor cores: H % 16 == 0, H <= 64, 16-byte aligned rows
    if (num_heads % 16 || num_heads > 64 || o_sh % 8 || o_st % 8 || reinterpret_cast<uintptr_t>(o) % 16 ||
        reinterpret_cast<uintptr_t>(mix) % 16 || reinterpret_cast<uintptr_t>(cos_sin) % 16 || cs_stride % 4 ||
        rope_dim > 64 || reinterpret_cast<uintptr_t>(out_fp8) % 16)
      return HCA_E_UNSUPPORTED;
    if (MODE == 0 && head_dim == 128 && num_tokens >= 1024 && rope_dim == 64 &&
        (num_heads == 16 || num_heads == 32 || num_heads == 64)) {
      // many tokens: the streamed kernel (persistent CTAs, one bulk copy per O row)
      auto* kfn = num_heads == 64 ? vha_stream_kernel<64> : num_heads == 32 ? vha_stream_kernel<32> : vha_stream_kernel<16>;
      static bool vs_smem_set[3][kMaxDevices] = {};  // per kernel and device
      const int ki = num_heads == 64 ? 0 : num_heads == 32 ? 1 : 2;
      if (set_func_attr_once(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, kVsDynSmem, vs_smem_set[ki]) != HCA_OK)
        return HCA_E_CUDA;
      VhaStream V;
      V.out_fp8 = out_fp8;
      V.scale = scale;
      V.o = op;
      V.o_st = o_st;
      V.o_sh = o_sh;
      V.mix = mp;
      V.positions = positions;
      V.cos_sin = cos_sin;
      V.cs_stride = cs_stride;
      V.err = device_error_word();
      if (!V.err) return HCA_E_CUDA;
      V.num_tokens = num_tokens;
      V.aligned_t = aligned;
      V.num_heads = num_heads;
      V.n_groups = n_groups;
      V.rope_dim = rope_dim;
      const int grid = min(num_tokens, 3 * device_sm_count());
      return launch_pdl(kfn, dim3(grid), dim3(32 * (kVsConsumers + 1)), kVsDynSmem, s, V);
    }
    // tokens per CTA: the mix is loaded once per CTA; keep >= 2 CTAs per SM busy
    const int tpc = max(1, min(16, aligned / (2 * 148 * 2)));
    const int ctas = (aligned + tpc - 1) / tpc;
    auto* kfn = head_dim == 128 ? vha_tok_kernel<128, MODE> : vha_tok_kernel<512, MODE>;
    static bool smem_set[2][kMaxDevices] = {};  // per head dim and device
    if (set_func_attr_once(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, kVhaDynSmem, smem_set[head_dim == 128]) !=
        HCA_OK)
      return HCA_E_CUDA;
    return launch_pdl(kfn, dim3(ctas), dim3(256), kVhaDynSmem, s, out_fp8, scale, out_bf16, ob_st, ob_sh, op, o_st, o_sh, mp, positions,
                      cos_sin, cs_stride, num_tokens, aligned, num_heads, n_groups, rope_dim, tpc);
  }
  if (head_dim == 128)
    vha_out_kernel<128, MODE><<<aligned, 256, 0, s>>>(out_fp8, scale, out_bf16, ob_st, ob_sh, op,
                                                      o_st, o_sh, mp, positions, cos_sin,
                                                      cs_stride, num_tokens, aligned, num_heads,
                                                      n_groups, rope_dim);
  else
    vha_out_kernel<512, MODE><<<aligned, 256, 0, s>>>(out_fp8, scale, out_bf16, ob_st, ob_sh, op,
                                                      o_st, o_sh, mp, positions, cos_sin,
                                                      cs_stride, num_tokens, aligned, num_heads,
                                                      n_groups, rope_dim);
  return HCA_LAUNCH_STATUS();
}

bool out_geom_ok(int head_dim, int rope_dim) {
  return (head_dim == 128 || head_dim == 512) && valid_geom(head_dim, rope_dim) &&
         // the RoPE tail must sit inside the last 128-chunk (fused_inv_rope_fp8_quant.py:170)
         rope_dim <= 128;
}

}  // namespace
}  // namespace hca

using namespace hca;

extern "C" int hca_vha_inv_rope_fp8_quant(uint8_t* out, int32_t* scale, const void* o,
                                          int64_t o_stride_tok, int64_t o_stride_head,
                                          const void* mix, const int64_t* positions,
                                          const float* cos_sin, int64_t cos_sin_stride,
                                          int32_t num_tokens, int32_t num_heads,
                                          int32_t n_groups, int32_t head_dim, int32_t rope_dim,
                                          void* stream) {
  HCA_CHECK_ARG(num_tokens >= 0 && num_heads > 0 && n_groups > 0 && num_heads % n_groups == 0);
  if (!out_geom_ok(head_dim, rope_dim)) return HCA_E_UNSUPPORTED;
  if (num_tokens == 0) return HCA_OK;
  HCA_CHECK_ARG(out && scale && o && mix && positions && cos_sin);
  return launch_vha<0>(out, scale, nullptr, 0, 0, o, o_stride_tok, o_stride_head, mix, positions,
                       cos_sin, cos_sin_stride, num_tokens, num_heads, n_groups, head_dim,
                       rope_dim, as_stream(stream));
}

extern "C" int hca_inv_rope_fp8_quant(uint8_t* out, int32_t* scale, const void* o,
                                      int64_t o_stride_tok, int64_t o_stride_head,
                                      const int64_t* positions, const float* cos_sin,
                                      int64_t cos_sin_stride, int32_t num_tokens,
                                      int32_t num_heads, int32_t n_groups, int32_t head_dim,
                                      int32_t rope_dim, void* stream) {
  HCA_CHECK_ARG(num_tokens >= 0 && num_heads > 0 && n_groups > 0 && num_heads % n_groups == 0);
  if (!out_geom_ok(head_dim, rope_dim)) return HCA_E_UNSUPPORTED;
  if (num_tokens == 0) return HCA_OK;
  HCA_CHECK_ARG(out && scale && o && positions && cos_sin);
  if (head_dim == 128) {
    // bytes of a pack are written by different warps: clear the packs first
    const int hpg = num_heads / n_groups;
    const int packs = (hpg + 3) / 4;
    const int aligned = (num_tokens + 3) / 4 * 4;
    if (cudaMemsetAsync(scale, 0, sizeof(int32_t) * static_cast<size_t>(n_groups) * packs * aligned,
                        as_stream(stream)) != cudaSuccess)
      return HCA_E_CUDA;
  }
  return launch_vha<1>(out, scale, nullptr, 0, 0, o, o_stride_tok, o_stride_head, nullptr,
                       positions, cos_sin, cos_sin_stride, num_tokens, num_heads, n_groups,
                       head_dim, rope_dim, as_stream(stream));
}

extern "C" int hca_vha_inv_rope(void* out, int64_t out_stride_tok, int64_t out_stride_head,
                                const void* o, int64_t o_stride_tok, int64_t o_stride_head,
                                const void* mix, const int64_t* positions, const float* cos_sin,
                                int64_t cos_sin_stride, int32_t num_tokens, int32_t num_heads,
                                int32_t head_dim, int32_t rope_dim, void* stream) {
  HCA_CHECK_ARG(num_tokens >= 0 && num_heads > 0);
  if (!out_geom_ok(head_dim, rope_dim)) return HCA_E_UNSUPPORTED;
  if (num_tokens == 0) return HCA_OK;
  HCA_CHECK_ARG(out && o && positions && cos_sin);
  return launch_vha<2>(nullptr, nullptr, static_cast<__nv_bfloat16*>(out), out_stride_tok,
                       out_stride_head, o, o_stride_tok, o_stride_head, mix, positions, cos_sin,
                       cos_sin_stride, num_tokens, num_heads, 1, head_dim, rope_dim,
                       as_stream(stream));
}

extern "C" int hca_sigmoid_mul_quant_fp8(uint8_t* out, int32_t* scale, const void* x,
                                         int64_t x_stride, const void* gate, int64_t gate_stride,
                                         int32_t rows, int32_t hidden, void* stream) {
  HCA_CHECK_ARG(rows >= 0 && hidden > 0 && hidden % 512 == 0);
  if (rows == 0) return HCA_OK;
  HCA_CHECK_ARG(out && scale && x && gate);
  const int aligned = (rows + 3) / 4 * 4;
  sigmoid_mul_quant_kernel<<<dim3(hidden / 512, rows), 128, 0, as_stream(stream)>>>(
      out, scale, static_cast<const __nv_bfloat16*>(x), x_stride,
      static_cast<const __nv_bfloat16*>(gate), gate_stride, rows, hidden, aligned);
  return HCA_LAUNCH_STATUS();
}
