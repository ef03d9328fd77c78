// FP8 projection GEMMs of the HCA output path on tcgen05:
//   grouped wo_a   z[t, g, :] = W_a[g] . x[t, g, :]   (x: e4m3, one UE8M0 scale
//                  per 128 elements; W_a: e4m3 with one fp32 scale per 128 x 128
//                  block), the role of DeepGEMM's fp8_einsum
//                  (V/models/deepseek_v4/attention.py:317-347);
//   gated wo_b     y = W_b . q(z * g), the same GEMM with G = 1 on the output of
//                  the fused sigmoid gate quant (E/nvidia/attention.py:364-395).
//
// Swap-AB: the weight is the MMA's M = 128 operand and the token tile (TT <=
// 192 tokens) its N, so at decode sizes (a few hundred tokens) one CTA reads
// each weight byte once for all tokens.  CTA (split rank r, 128-row weight
// tile, group x token tile), a cluster of `split` CTAs along K.  10 warps:
//   warp 0     TMA producer (lane 0): per 128-wide K block, the 128 x 128-byte
//              weight box and the TT x 128-byte token box, 128B-swizzled,
//              into a kStages-deep ring (tokens past T read as zero)
//   warp 1     TMEM owner and MMA issuer (lane 0): tcgen05.mma.kind::f8f6f4,
//              M128 x N=TT x K32, e4m3 x e4m3 -> fp32; K block i of this CTA
//              accumulates into TMEM buffer i % 2, so the block scales (one
//              per weight block, one per token) are applied once per block
//   warps 2-9  epilogue: weight row = TMEM lane (quadrant warp % 4), half of
//              the token columns each; per K block, acc * sw[kb] * sx[t, kb]
//              added to fp32 registers (the promotion step of DeepGEMM's
//              block-scaled GEMM), the buffer handed back to the MMA warp
// The CTA's partial [TT x 128] fp32 tile goes to the caller's workspace (L2);
// after one cluster barrier CTA r sums rank r's token slice over the
// cluster's partial tiles, rounds to bf16 and stores coalesced rows.
// Every mbarrier wait is bounded; a timeout sets the device error word, and
// the producer and MMA threads wait (bounded) for their copies and MMAs in
// flight before the CTA frees its TMEM; the cluster barriers are taken by
// every thread on every path.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>

#include "hca_common.cuh"
#include "hca_tc.cuh"

namespace hca {
namespace {

constexpr int kStages = 4;
constexpr int kAccBufs = 2;
constexpr int kEpiWarps = 8;
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kWBox = 128 * 128;  // one 128-row x 128-byte weight box
constexpr int kPStride = 128 + 4;  // floats per token row of the partial tile (bank spread)
constexpr int kMaxSplit = 8;
constexpr int kMaxKBlocks = 64;  // K blocks of one CTA (its scale table)

template <int TT>
struct GemmSmem {
  static constexpr int kXBox = TT * 128;
  static constexpr int kStage = kWBox + kXBox;
  static constexpr int kPipe = kStages * kStage;
  static constexpr int kPart = TT * kPStride * 4;  // reuses the ring after the K loop
  static constexpr int kBody = kPipe > kPart ? kPipe : kPart;
  static constexpr int kScale = kBody;  // [kMaxKBlocks][TT] floats: sx * sw of each K block and token
  static constexpr int kBar = kScale + kMaxKBlocks * TT * 4 + kMaxKBlocks * 4;
  // full[kStages] empty[kStages] acc_full[2] acc_empty[2] drain
  static constexpr int kMisc = kBar + (2 * kStages + 2 * kAccBufs + 1) * 8;
  static constexpr int kBytes = kMisc + 64 + 1024;  // + 1024 alignment slack
  static constexpr int kTmemCols = TT * kAccBufs <= 256 ? 256 : 512;
  static_assert(kBytes <= 227 * 1024, "shared memory");
  static_assert(TT % 64 == 0 && TT <= 192, "token tile");
};

struct GemmArgs {
  __nv_bfloat16* out;
  int64_t out_st, out_sg;  // elements
  const int32_t* xs;       // activation scales: byte (kb % per_int) of xs[t * xs_t + g * xs_g + (kb / per_int) * xs_k]
  int64_t xs_t, xs_g, xs_k;
  int per_int;
  const float* ws;         // weight scales [G][ceil(N / 128)][K / 128]
  int T, G, N, K;
  int n_blocks;            // ceil(N / 128)
  int split;               // CTAs per cluster along K
  float* ws_part;          // split > 1: [tiles][split][TT][128] fp32 partial tiles
  uint64_t wait_ns;
};

// kind::f8f6f4 instruction descriptor: e4m3 A and B (format 0), fp32 D,
// both K-major.
__host__ __device__ constexpr uint32_t umma_idesc_e4m3(int M, int N) {
  return (1u << 4)                               // D format F32
         | (0u << 7)                             // A format E4M3
         | (0u << 10)                            // B format E4M3
         | (static_cast<uint32_t>(N >> 3) << 17)  // N
         | (static_cast<uint32_t>(M >> 4) << 24);  // M
}

__device__ __forceinline__ void umma_f8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0));
}

__device__ __forceinline__ uint32_t pack_bf16_rn(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// 10 warps: at most 168 registers a thread (three warps share one SM
// sub-partition's 16K registers); the epilogue holds up to 96 fp32 partial
// sums per lane
template <int TT>
__global__ void __launch_bounds__(kThreads, 1)
    hca_fp8_gemm_kernel(const GemmArgs A, int* err, const __grid_constant__ CUtensorMap xmap,
                        const __grid_constant__ CUtensorMap wmap) {
  using namespace tc;
  using L = GemmSmem<TT>;
  extern __shared__ uint8_t smem_dyn[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
  // TMEM is allocated after the wait (the kernel before may hold columns on
  // this SM) and dependents are released after it (a dependent that takes
  // columns before its own wait cannot starve this CTA)
  pdl_wait();  // x and its scales were written by the kernel before this one
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int split = A.split;
  const int rank = static_cast<int>(blockIdx.x);  // rank in the cluster (cluster = the grid's x extent)
  const int n0 = blockIdx.y * 128;
  const int g = static_cast<int>(blockIdx.z) % A.G;
  const int t0 = (static_cast<int>(blockIdx.z) / A.G) * TT;
  const int nkb = A.K / 128;
  const int kb0 = rank * nkb / split, nk = (rank + 1) * nkb / split - kb0;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBar);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;
  uint64_t* acc_empty = acc_full + kAccBufs;
  uint64_t* drain = acc_empty + kAccBufs;
  uint32_t* misc = reinterpret_cast<uint32_t*>(smem + L::kMisc);  // [0] tmem
  if (warp == 1) {
    tmem_alloc(misc, L::kTmemCols);
    tmem_relinquish();
    tc_fence_before();
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int b = 0; b < kAccBufs; ++b) {
      mbar_init(acc_full + b, 1);
      mbar_init(acc_empty + b, kEpiWarps);  // lane 0 of each epilogue warp
    }
    mbar_init(drain, 1);
    mbar_fence_init();
  }
  __syncthreads();
  tc_fence_after();
  pdl_release();
  const uint32_t tmem = misc[0];
  float o[TT / 2];  // epilogue: this lane's weight row over this warp's token half
  bool ok = true;
  if (warp == 0) {
    // ---------------------------------------------------------------- TMA
    if (lane == 0) {
      int issued = 0;
      for (int i = 0; i < nk; ++i) {
        const int s = i % kStages;
        if (i >= kStages && !mbar_wait(empty + s, ((i / kStages) - 1) & 1, A.wait_ns)) {
          ok = false;
          break;
        }
        uint8_t* st = smem + s * L::kStage;
        mbar_arrive_expect_tx(full + s, L::kStage);
        tma_load_3d(st, &wmap, (kb0 + i) * 128, n0, g, full + s);
        tma_load_3d(st + kWBox, &xmap, (kb0 + i) * 128, t0, g, full + s);
        issued = i + 1;
      }
      // the copies still in flight land before the ring is reused
      for (int i = issued > kStages ? issued - kStages : 0; i < issued; ++i)
        ok &= mbar_wait(full + i % kStages, (i / kStages) & 1, A.wait_ns);
      if (!ok && err) atomicOr(err, 1 << 7);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_e4m3(128, TT);
      const uint64_t d0 = umma_desc_sw128(smem_u32(smem), 16, 1024);
      for (int i = 0; i < nk; ++i) {
        const int s = i % kStages, b = i % kAccBufs;
        if (!mbar_wait(full + s, (i / kStages) & 1, A.wait_ns) ||
            (i >= kAccBufs && !mbar_wait(acc_empty + b, ((i / kAccBufs) - 1) & 1, A.wait_ns))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t so = static_cast<uint32_t>(s * L::kStage);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)  // 32 e4m3 (32 bytes) of K per MMA
          umma_f8(tmem + b * TT, d0 + ((so + kk * 32) >> 4), d0 + ((so + kWBox + kk * 32) >> 4), idesc,
                  kk > 0 ? 1u : 0u);
        umma_commit(empty + s);
        umma_commit(acc_full + b);
      }
      // every MMA issued completes before the ring and the TMEM are reused
      umma_commit(drain);
      ok &= mbar_wait(drain, 0, A.wait_ns);
      if (!ok && err) atomicOr(err, 1 << 7);
    }
  } else {
    // ----------------------------------------------------------- epilogue
    constexpr int kCols = TT / 2;     // token columns of this warp
    constexpr int kHalf = kCols / 2;  // columns per TMEM round trip
    const int e = warp - 2;
    const int quad = warp & 3, c0 = (e >> 2) * kCols;
    const uint32_t lane_addr = static_cast<uint32_t>(quad * 32) << 16;
    // the scale of every (K block, token) of this CTA, weight scale folded
    // in, loaded once while the ring fills (tokens past T: 0)
    float* tab = reinterpret_cast<float*>(smem + L::kScale);
    {
      // each packed scale int of the CTA's (K block, token) range loaded once
      // (up to kU per thread, all in flight together), with this CTA's weight
      // block scales staged in shared memory first
      constexpr int kU = 8, kStep = 32 * kEpiWarps;
      float* wtab = tab + kMaxKBlocks * TT;  // [kMaxKBlocks]
      const int tid = threadIdx.x - 64;
      const int p0 = kb0 / A.per_int, npk = (kb0 + nk - 1) / A.per_int - p0 + 1;
      const int total = npk * TT;
      const float wv = tid < nk ? A.ws[(static_cast<int64_t>(g) * A.n_blocks + n0 / 128) * nkb + kb0 + tid] : 0.0f;
      int32_t xv[kU];
      auto load = [&](int base) {
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const int idx = base + u * kStep;
          const int pk = idx / TT, t = t0 + idx - pk * TT;
          xv[u] = 0;
          if (idx < total && t < A.T) xv[u] = A.xs[t * A.xs_t + g * A.xs_g + (p0 + pk) * A.xs_k];
        }
      };
      auto expand = [&](int base) {
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const int idx = base + u * kStep;
          if (idx < total) {
            const int pk = idx / TT, tl = idx - pk * TT;
            const bool live = t0 + tl < A.T;
            for (int c = 0; c < A.per_int; ++c) {
              const int kq = (p0 + pk) * A.per_int + c - kb0;
              if (kq >= 0 && kq < nk) {
                const int ex = static_cast<int>((static_cast<uint32_t>(xv[u]) >> (8 * c)) & 0xffu);
                tab[kq * TT + tl] = live ? exp2i(ex - 127) * wtab[kq] : 0.0f;
              }
            }
          }
        }
      };
      load(tid);  // every epilogue thread, in-range or not, reaches the barrier below
      if (tid < nk) wtab[tid] = wv;
      asm volatile("bar.sync 1, %0;\n" ::"n"(32 * kEpiWarps) : "memory");
      expand(tid);
      for (int base = tid + kU * kStep; base < total; base += kU * kStep) {
        load(base);
        expand(base);
      }
      asm volatile("bar.sync 1, %0;\n" ::"n"(32 * kEpiWarps) : "memory");  // the epilogue warps
    }
#pragma unroll
    for (int j = 0; j < kCols; ++j) o[j] = 0.0f;
    for (int i = 0; i < nk; ++i) {
      const int b = i % kAccBufs;
      if (!mbar_wait(acc_full + b, (i / kAccBufs) & 1, A.wait_ns)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const float* sc = tab + i * TT + c0;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t v[kHalf];
#pragma unroll
        for (int c = 0; c < kHalf / 16; ++c) tmem_ld16(tmem + lane_addr + b * TT + c0 + h * kHalf + c * 16, v + c * 16);
        tmem_wait_ld();
#pragma unroll
        for (int q = 0; q < kHalf / 4; ++q) {
          const float4 s4 = *reinterpret_cast<const float4*>(sc + h * kHalf + q * 4);
          float* oo = o + h * kHalf + q * 4;
          oo[0] = fmaf(__uint_as_float(v[q * 4 + 0]), s4.x, oo[0]);
          oo[1] = fmaf(__uint_as_float(v[q * 4 + 1]), s4.y, oo[1]);
          oo[2] = fmaf(__uint_as_float(v[q * 4 + 2]), s4.z, oo[2]);
          oo[3] = fmaf(__uint_as_float(v[q * 4 + 3]), s4.w, oo[3]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_empty + b);
    }
    if (!ok && lane == 0 && err) atomicOr(err, 1 << 7);
  }
  // Split-K: CTA r owns tokens [r S, (r + 1) S) of the tile (S = TT /
  // split).  Every CTA writes its partial tile [TT tokens][128 rows] fp32 to
  // its slot of the workspace (coalesced, L2-resident), one cluster barrier
  // (release / acquire at cluster scope) makes the cluster's slots visible,
  // and each CTA sums the split rows of its tokens from L2 and stores bf16.
  // Without a split the partial tile goes through the CTA's own (idle) ring.
  __syncthreads();
  const int slice = TT / split;
  constexpr int kCols = TT / 2;
  float* part;
  int64_t pstride;  // floats per token row
  if (split > 1) {
    part = A.ws_part + (static_cast<int64_t>(blockIdx.z) * gridDim.y + blockIdx.y) * split * TT * 128;
    pstride = 128;
  } else {
    part = reinterpret_cast<float*>(smem);
    pstride = kPStride;
  }
  if (warp >= 2) {
    const int row = (warp & 3) * 32 + lane, c0 = ((warp - 2) >> 2) * kCols;
    float* dst = part + static_cast<int64_t>(rank * TT + c0) * pstride + row;
    if (split > 1) {
#pragma unroll
      for (int j = 0; j < kCols; ++j) __stcg(dst + j * pstride, o[j]);
    } else {
#pragma unroll
      for (int j = 0; j < kCols; ++j) dst[j * pstride] = o[j];
    }
  }
  if (split > 1) {
    cluster_sync();
  } else {
    __syncthreads();
  }
  {
    const int items = slice * 16;  // 8 weight rows (16 output bytes) per item
    for (int it = threadIdx.x; it < items; it += kThreads) {
      const int tl = rank * slice + it / 16, r8 = (it % 16) * 8;
      const int t = t0 + tl, n = n0 + r8;
      // every split's 8 values requested before any is summed
      float4 xq[2 * kMaxSplit];
#pragma unroll
      for (int q = 0; q < kMaxSplit; ++q) {
        if (q < split) {
          const float4* src = reinterpret_cast<const float4*>(part + static_cast<int64_t>(q * TT + tl) * pstride + r8);
          xq[2 * q] = split > 1 ? __ldcg(src) : src[0];
          xq[2 * q + 1] = split > 1 ? __ldcg(src + 1) : src[1];
        }
      }
      float acc[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) acc[k] = 0.0f;
#pragma unroll
      for (int q = 0; q < kMaxSplit; ++q) {
        if (q < split) {
          acc[0] += xq[2 * q].x;
          acc[1] += xq[2 * q].y;
          acc[2] += xq[2 * q].z;
          acc[3] += xq[2 * q].w;
          acc[4] += xq[2 * q + 1].x;
          acc[5] += xq[2 * q + 1].y;
          acc[6] += xq[2 * q + 1].z;
          acc[7] += xq[2 * q + 1].w;
        }
      }
      if (ok && t < A.T && n < A.N) {
        uint4 w;
        w.x = pack_bf16_rn(acc[0], acc[1]);
        w.y = pack_bf16_rn(acc[2], acc[3]);
        w.z = pack_bf16_rn(acc[4], acc[5]);
        w.w = pack_bf16_rn(acc[6], acc[7]);
        *reinterpret_cast<uint4*>(A.out + static_cast<int64_t>(t) * A.out_st + static_cast<int64_t>(g) * A.out_sg +
                                  n) = w;
      }
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, L::kTmemCols);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encoder() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult qr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &qr) == cudaSuccess &&
        qr == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 3-D byte tensor [d2][d1][d0] (strides s1, s2 bytes) in 128 x rows boxes
// with the 128-byte swizzle.
bool encode_u8_3d(CUtensorMap* m, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s1, uint64_t s2,
                  uint32_t box_rows) {
  std::memset(m, 0, sizeof(*m));
  auto enc = encoder();
  if (!enc) return false;
  const cuuint64_t dims[3] = {d0, d1, d2};
  const cuuint64_t strides[2] = {s1, s2};
  const cuuint32_t box[3] = {128, box_rows, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int TT>
int launch_gemm(const GemmArgs& A, int t_tiles, int* err, const CUtensorMap& xm, const CUtensorMap& wm,
                cudaStream_t s) {
  static bool attr_set[kMaxDevices] = {};
  if (set_func_attr_once(hca_fp8_gemm_kernel<TT>, cudaFuncAttributeMaxDynamicSharedMemorySize, GemmSmem<TT>::kBytes,
                         attr_set) != HCA_OK)
    return HCA_E_CUDA;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = static_cast<unsigned>(A.split);
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(A.split), static_cast<unsigned>(A.n_blocks),
                     static_cast<unsigned>(A.G * t_tiles));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = GemmSmem<TT>::kBytes;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cuda_status(cudaLaunchKernelEx(&cfg, hca_fp8_gemm_kernel<TT>, A, err, xm, wm));
}

}  // namespace
}  // namespace hca

using namespace hca;

namespace hca {
namespace {

// Token tile, token tiles and split-K factor of one call.
struct GemmPlan {
  int tt, t_tiles, n_blocks, split;
  int64_t ws_bytes;  // split-K workspace (0 without a split)
};

GemmPlan plan_gemm(int num_tokens, int num_groups, int n, int k) {
  GemmPlan P{};
  // token tile: all tokens up to 192 (a multiple of 64), else 192-token tiles
  P.tt = num_tokens >= 192 ? 192 : ((num_tokens + 63) / 64) * 64;
  P.t_tiles = (num_tokens + P.tt - 1) / P.tt;
  P.n_blocks = (n + 127) / 128;
  const int sms = device_sm_count();
  // split K over a cluster while the CTAs fit one wave and each keeps at
  // least two K blocks; at most kMaxKBlocks K blocks per CTA (its scale table)
  const int64_t base = static_cast<int64_t>(P.n_blocks) * num_groups * P.t_tiles;
  const int nkb = k / 128;
  P.split = 1;
  while (P.split < kMaxSplit && base * P.split * 2 <= sms && nkb >= P.split * 4) P.split *= 2;
  while (P.split < kMaxSplit && nkb > P.split * kMaxKBlocks) P.split *= 2;
  P.ws_bytes = P.split > 1 ? base * P.split * P.tt * 128 * static_cast<int64_t>(sizeof(float)) : 0;
  return P;
}

}  // namespace
}  // namespace hca

extern "C" int64_t hca_fp8_grouped_gemm_workspace_bytes(int32_t num_tokens, int32_t num_groups, int32_t n,
                                                        int32_t k) {
  if (num_tokens <= 0 || num_groups < 1 || n < 64 || k < 128 || k % 128 || n % 64) return 0;
  return hca::plan_gemm(num_tokens, num_groups, n, k).ws_bytes;
}

extern "C" int hca_fp8_grouped_gemm(void* out, int64_t out_stride_tok, int64_t out_stride_group, const uint8_t* x,
                                    int64_t x_stride_tok, int64_t x_stride_group, const int32_t* x_scale,
                                    int64_t xs_stride_tok, int64_t xs_stride_group, int64_t xs_stride_pack,
                                    int32_t xs_per_int, const uint8_t* w, const float* w_scale, int32_t num_tokens,
                                    int32_t num_groups, int32_t n, int32_t k, void* workspace,
                                    int64_t workspace_bytes, void* stream) {
  HCA_CHECK_ARG(num_tokens >= 0 && num_groups >= 1 && n >= 1 && k >= 128);
  HCA_CHECK_ARG(xs_per_int == 1 || xs_per_int == 4);
  // N a multiple of 64 and K of 128 (the 128 x 128 weight blocks; N = 64
  // covers a rank-64 group)
  if (k % 128 || n % 64) return HCA_E_UNSUPPORTED;
  if (num_tokens == 0) return HCA_OK;
  HCA_CHECK_ARG(out && x && x_scale && w && w_scale);
  HCA_CHECK_ARG(reinterpret_cast<uintptr_t>(x) % 16 == 0 && reinterpret_cast<uintptr_t>(w) % 16 == 0 &&
                x_stride_tok % 16 == 0 && x_stride_group % 16 == 0 && x_stride_tok >= k);
  HCA_CHECK_ARG(reinterpret_cast<uintptr_t>(out) % 16 == 0 && out_stride_tok % 8 == 0 && out_stride_group % 8 == 0);
  const GemmPlan P = plan_gemm(num_tokens, num_groups, n, k);
  HCA_CHECK_ARG(static_cast<int64_t>(P.t_tiles) * num_groups <= 65535);
  if (k / 128 > P.split * kMaxKBlocks) return HCA_E_UNSUPPORTED;
  if (P.ws_bytes > 0) {
    if (!workspace || reinterpret_cast<uintptr_t>(workspace) % 16 != 0) return HCA_E_INVALID;
    if (workspace_bytes < P.ws_bytes) return HCA_E_WORKSPACE;
  }
  GemmArgs A{};
  A.out = static_cast<__nv_bfloat16*>(out);
  A.out_st = out_stride_tok;
  A.out_sg = out_stride_group;
  A.xs = x_scale;
  A.xs_t = xs_stride_tok;
  A.xs_g = xs_stride_group;
  A.xs_k = xs_stride_pack;
  A.per_int = xs_per_int;
  A.ws = w_scale;
  A.T = num_tokens;
  A.G = num_groups;
  A.N = n;
  A.K = k;
  A.n_blocks = P.n_blocks;
  A.split = P.split;
  A.ws_part = static_cast<float*>(workspace);
  A.wait_ns = tc::kWaitLimitNs;
  CUtensorMap xm, wm;
  // x [G][T][K] bytes (token stride x_stride_tok, group stride
  // x_stride_group); w [G][N][K] contiguous
  const uint64_t gstride = num_groups > 1 ? static_cast<uint64_t>(x_stride_group)
                                          : static_cast<uint64_t>(x_stride_tok) * num_tokens;
  if (!encode_u8_3d(&xm, x, k, num_tokens, num_groups, x_stride_tok, gstride, static_cast<uint32_t>(P.tt)) ||
      !encode_u8_3d(&wm, w, k, n, num_groups, k, static_cast<uint64_t>(n) * k, 128))
    return HCA_E_UNSUPPORTED;
  int* err = device_error_word();
  cudaStream_t s = as_stream(stream);
  switch (P.tt) {
    case 64: return launch_gemm<64>(A, P.t_tiles, err, xm, wm, s);
    case 128: return launch_gemm<128>(A, P.t_tiles, err, xm, wm, s);
    default: return launch_gemm<192>(A, P.t_tiles, err, xm, wm, s);
  }
}
