// FP8 projection GEMMs of the HCA output path on tcgen05:
//   grouped wo_a   z[t, g, :] = W_a[g] . x[t, g, :]   (x: e4m3, one UE8M0 scale
//                  per 128 elements; W_a: e4m3 with one fp32 scale per 128 x 128
//                  block), the role of DeepGEMM's fp8_einsum
//                  (V/models/deepseek_v4/attention.py:317-347);
//   gated wo_b     y = W_b . q(z * g), the same GEMM with G = 1 on the output of
//                  the fused sigmoid gate quant (E/nvidia/attention.py:364-395).
//
// One CTA per (128-token tile, N tile, group); 6 warps:
//   warp 0     TMA producer (lane 0): per 128-wide K block, the 128 x 128-byte
//              x box and the N_TILE x 128-byte weight box, 128B-swizzled, into
//              a kStages-deep ring (rows past the token count read as zero)
//   warp 1     TMEM owner and MMA issuer (lane 0): tcgen05.mma.kind::f8f6f4,
//              M128 x N_TILE x K32, e4m3 x e4m3 -> fp32; K block kb
//              accumulates into TMEM buffer kb % kAccBufs, so the block scales
//              (per token and per weight block) are applied once per block
//   warps 2-5  epilogue: one token row per lane (TMEM lane quadrant =
//              warp % 4); per K block, acc_kb * sx[t, kb] * sw[kb] added to
//              fp32 registers (the promotion of DeepGEMM's block-scaled GEMM),
//              the buffer handed back to the MMA warp, the sum rounded to bf16
// Every mbarrier wait is bounded; a timeout sets the device error word, and
// the producer and MMA threads wait (bounded) for their copies and MMAs in
// flight before the CTA frees its TMEM and exits.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>

#include "hca_common.cuh"
#include "hca_tc.cuh"

namespace hca {
namespace {

constexpr int kStages = 4;
constexpr int kAccBufs = 4;
constexpr int kThreads = 192;
constexpr int kBoxBytes = 128 * 128;  // one 128 x 128-byte swizzled box

template <int N_TILE>
struct GemmSmem {
  static constexpr int kA = 0;
  static constexpr int kB = kStages * kBoxBytes;
  static constexpr int kBBytes = N_TILE * 128;
  // full[kStages] empty[kStages] acc_full[kAccBufs] acc_empty[kAccBufs] drain
  static constexpr int kBar = kB + kStages * kBBytes;
  static constexpr int kMisc = kBar + (2 * kStages + 2 * kAccBufs + 1) * 8;
  static constexpr int kBytes = kMisc + 64 + 1024;  // + 1024 alignment slack
  static constexpr int kTmemCols = N_TILE * kAccBufs;
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

template <int N_TILE>
__global__ void __launch_bounds__(kThreads, 1)
    hca_fp8_gemm_kernel(const GemmArgs A, int* err, const __grid_constant__ CUtensorMap xmap,
                        const __grid_constant__ CUtensorMap wmap) {
  using namespace tc;
  using L = GemmSmem<N_TILE>;
  extern __shared__ uint8_t smem_dyn[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
  // TMEM is allocated after the wait (the kernel before may hold columns on
  // this SM) and dependents are released after it (a dependent that takes
  // columns before its own wait cannot starve this CTA)
  pdl_wait();  // x and its scales were written by the kernel before this one
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * 128, n0 = blockIdx.y * N_TILE, g = blockIdx.z;
  const int nkb = A.K / 128;
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
      mbar_init(acc_empty + b, 4);  // lane 0 of each epilogue warp
    }
    mbar_init(drain, 1);
    mbar_fence_init();
  }
  __syncthreads();
  tc_fence_after();
  pdl_release();
  const uint32_t tmem = misc[0];
  if (warp == 0 && lane == 0) {
    // ---------------------------------------------------------------- TMA
    bool ok = true;
    int issued = 0;
    for (int kb = 0; kb < nkb; ++kb) {
      const int s = kb % kStages;
      if (kb >= kStages && !mbar_wait(empty + s, ((kb / kStages) - 1) & 1, A.wait_ns)) {
        ok = false;
        break;
      }
      mbar_arrive_expect_tx(full + s, kBoxBytes + L::kBBytes);
      tma_load_3d(smem + L::kA + s * kBoxBytes, &xmap, kb * 128, m0, g, full + s);
      tma_load_3d(smem + L::kB + s * L::kBBytes, &wmap, kb * 128, n0, g, full + s);
      issued = kb + 1;
    }
    // the copies still in flight land before the CTA exits
    for (int kb = issued > kStages ? issued - kStages : 0; kb < issued; ++kb)
      ok &= mbar_wait(full + kb % kStages, (kb / kStages) & 1, A.wait_ns);
    if (!ok && err) atomicOr(err, 1 << 7);
  } else if (warp == 1 && lane == 0) {
    // ---------------------------------------------------------------- MMA
    bool ok = true;
    const uint32_t idesc = umma_idesc_e4m3(128, N_TILE);
    const uint64_t da = umma_desc_sw128(smem_u32(smem + L::kA), 16, 1024);
    const uint64_t dw = umma_desc_sw128(smem_u32(smem + L::kB), 16, 1024);
    for (int kb = 0; kb < nkb; ++kb) {
      const int s = kb % kStages, b = kb % kAccBufs;
      if (!mbar_wait(full + s, (kb / kStages) & 1, A.wait_ns) ||
          (kb >= kAccBufs && !mbar_wait(acc_empty + b, ((kb / kAccBufs) - 1) & 1, A.wait_ns))) {
        ok = false;
        break;
      }
      tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)  // 32 e4m3 (32 bytes) of K per MMA
        umma_f8(tmem + b * N_TILE, da + ((s * kBoxBytes + kk * 32) >> 4), dw + ((s * L::kBBytes + kk * 32) >> 4),
                idesc, kk > 0 ? 1u : 0u);
      umma_commit(empty + s);
      umma_commit(acc_full + b);
    }
    // every MMA issued completes before the TMEM is freed
    umma_commit(drain);
    ok &= mbar_wait(drain, 0, A.wait_ns);
    if (!ok && err) atomicOr(err, 1 << 7);
  } else if (warp >= 2) {
    // ----------------------------------------------------------- epilogue
    const int quad = warp & 3;
    const int t = m0 + quad * 32 + lane;
    const int64_t wbase = (static_cast<int64_t>(g) * A.n_blocks + n0 / 128) * nkb;
    auto block_scale = [&](int kb) -> float {
      float sx = 0.0f;
      if (t < A.T) {
        const int32_t v = A.xs[t * A.xs_t + g * A.xs_g + (kb / A.per_int) * A.xs_k];
        sx = exp2i(static_cast<int>((static_cast<uint32_t>(v) >> (8 * (kb % A.per_int))) & 0xffu) - 127);
      }
      return sx * A.ws[wbase + kb];
    };
    const uint32_t lane_addr = static_cast<uint32_t>(quad * 32) << 16;
    float o[N_TILE];
#pragma unroll
    for (int e = 0; e < N_TILE; ++e) o[e] = 0.0f;
    bool ok = true;
    float sc_next = block_scale(0);
    for (int kb = 0; kb < nkb; ++kb) {
      const float sc = sc_next;
      if (kb + 1 < nkb) sc_next = block_scale(kb + 1);  // in flight during the wait
      const int b = kb % kAccBufs;
      if (!mbar_wait(acc_full + b, (kb / kAccBufs) & 1, A.wait_ns)) {
        ok = false;
        break;
      }
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < N_TILE / 32; ++c) {
        uint32_t v[32];
        tmem_ld32(tmem + lane_addr + b * N_TILE + c * 32, v);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e) o[c * 32 + e] = fmaf(__uint_as_float(v[e]), sc, o[c * 32 + e]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_empty + b);
    }
    if (!ok && lane == 0 && err) atomicOr(err, 1 << 7);
    if (ok && t < A.T) {
      uint4* dst = reinterpret_cast<uint4*>(A.out + static_cast<int64_t>(t) * A.out_st +
                                            static_cast<int64_t>(g) * A.out_sg + n0);
#pragma unroll
      for (int q = 0; q < N_TILE / 8; ++q) {
        uint4 w;
        w.x = pack_bf16_rn(o[8 * q + 0], o[8 * q + 1]);
        w.y = pack_bf16_rn(o[8 * q + 2], o[8 * q + 3]);
        w.z = pack_bf16_rn(o[8 * q + 4], o[8 * q + 5]);
        w.w = pack_bf16_rn(o[8 * q + 6], o[8 * q + 7]);
        dst[q] = w;
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

template <int N_TILE>
int launch_gemm(const GemmArgs& A, int* err, const CUtensorMap& xm, const CUtensorMap& wm, cudaStream_t s) {
  static bool attr_set[kMaxDevices] = {};
  if (set_func_attr_once(hca_fp8_gemm_kernel<N_TILE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         GemmSmem<N_TILE>::kBytes, attr_set) != HCA_OK)
    return HCA_E_CUDA;
  dim3 grid((A.T + 127) / 128, A.N / N_TILE, A.G);
  return launch_pdl(hca_fp8_gemm_kernel<N_TILE>, grid, dim3(kThreads), GemmSmem<N_TILE>::kBytes, s, A, err, xm, wm);
}

}  // namespace
}  // namespace hca

using namespace hca;

extern "C" int hca_fp8_grouped_gemm(void* out, int64_t out_stride_tok, int64_t out_stride_group, const uint8_t* x,
                                    int64_t x_stride_tok, int64_t x_stride_group, const int32_t* x_scale,
                                    int64_t xs_stride_tok, int64_t xs_stride_group, int64_t xs_stride_pack,
                                    int32_t xs_per_int, const uint8_t* w, const float* w_scale, int32_t num_tokens,
                                    int32_t num_groups, int32_t n, int32_t k, void* stream) {
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
  // 128-column N tiles while they fill the SMs, else 64
  const int64_t m_tiles = (num_tokens + 127) / 128;
  int sms = 148;
  {
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  }
  const int n_tile = (n % 128 == 0 && m_tiles * (n / 128) * num_groups >= sms) ? 128 : 64;
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
  A.n_blocks = (n + 127) / 128;
  A.wait_ns = tc::kWaitLimitNs;
  CUtensorMap xm, wm;
  // x [G][T][K] bytes (token stride x_stride_tok, group stride
  // x_stride_group); w [G][N][K] contiguous
  const uint64_t gstride = num_groups > 1 ? static_cast<uint64_t>(x_stride_group)
                                          : static_cast<uint64_t>(x_stride_tok) * num_tokens;
  if (!encode_u8_3d(&xm, x, k, num_tokens, num_groups, x_stride_tok, gstride, 128) ||
      !encode_u8_3d(&wm, w, k, n, num_groups, k, static_cast<uint64_t>(n) * k, n_tile))
    return HCA_E_UNSUPPORTED;
  int* err = device_error_word();
  cudaStream_t s = as_stream(stream);
  return n_tile == 128 ? launch_gemm<128>(A, err, xm, wm, s) : launch_gemm<64>(A, err, xm, wm, s);
}
