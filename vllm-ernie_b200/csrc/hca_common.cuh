// Shared device helpers of libhca_b200: status plumbing, bf16 / e4m3 /
// UE8M0 conversions, GPT-J RoPE and the cached-row geometry.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "hca_b200.h"

#define HCA_CHECK_ARG(cond)            \
  do {                                 \
    if (!(cond)) return HCA_E_INVALID; \
  } while (0)

#define HCA_LAUNCH_STATUS() (::hca::cuda_status(cudaGetLastError()))

namespace hca {

constexpr float kFp8Max = 448.0f;
constexpr int kQuantBlock = 64;  // NoPE quantisation block of the cached rows

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Quad transpose of e4m3 byte pairs from an m16n8 accumulator row: lane cq
// (0..3) of a 4-lane quad holds the pair for columns 8 j + 2 cq, + 1 of
// j = 0..7 (pair[j], low 16 bits).  Returns this lane's 16 contiguous bytes,
// columns 16 cq .. 16 cq + 15 of the quad's 64-column segment, so the row
// is written with one 16-byte store per lane instead of eight 2-byte ones.
__device__ __forceinline__ uint4 quad_gather_fp8(const uint32_t pair[8], int cq) {
  // m[x]: this lane's pairs 2x, 2x + 1; lane cq needs word cq of every quad
  // lane s (a 4 x 4 word transpose over the quad), done as two butterfly
  // exchanges: over lane bit 0 (words 0 <-> 1, 2 <-> 3), then over lane
  // bit 1 (words 0 <-> 2, 1 <-> 3).  After both, m[s] = word cq of lane s.
  uint32_t m[4];
#pragma unroll
  for (int x = 0; x < 4; ++x) m[x] = __byte_perm(pair[2 * x], pair[2 * x + 1], 0x5410);
  const bool b0 = cq & 1, b1 = cq & 2;
#pragma unroll
  for (int x = 0; x < 4; x += 2) {
    const uint32_t r = __shfl_xor_sync(0xffffffffu, b0 ? m[x] : m[x + 1], 1);
    if (b0) m[x] = r; else m[x + 1] = r;
  }
#pragma unroll
  for (int x = 0; x < 2; ++x) {
    const uint32_t r = __shfl_xor_sync(0xffffffffu, b1 ? m[x] : m[x + 2], 2);
    if (b1) m[x] = r; else m[x + 2] = r;
  }
  uint4 o;
  o.x = __byte_perm(m[0], m[1], 0x5410);
  o.y = __byte_perm(m[2], m[3], 0x5410);
  o.z = __byte_perm(m[0], m[1], 0x7632);
  o.w = __byte_perm(m[2], m[3], 0x7632);
  return o;
}

// Programmatic dependent launch for the per-layer chain of kernels.  A kernel
// launched with launch_pdl may be scheduled while the kernel before it on the
// stream is still running; it first waits (griddepcontrol.wait) until that
// kernel has completed and its writes are visible -- before any global read
// and before any early return, so completion stays transitive along the
// chain -- and then lets its own successor launch (launch_dependents).  The
// successor only launches once every CTA of this kernel has started, so its
// waiting CTAs never hold resources this kernel still needs.  Without a
// programmatic predecessor the wait returns at once.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void pdl_release() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }
__device__ __forceinline__ void pdl_wait_and_release() {
  pdl_wait();
  pdl_release();
}

// The CUDA error behind the last HCA_E_CUDA status of this thread
// (hca_last_cuda_error).
const char*& last_cuda_error();

// HCA_OK, or HCA_E_CUDA with the error recorded for hca_last_cuda_error.
inline int cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return HCA_OK;
  last_cuda_error() = cudaGetErrorString(e);
  return HCA_E_CUDA;
}

template <typename... KArgs, typename... Args>
inline int launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...));
}

inline int cdiv(int64_t a, int64_t b) { return static_cast<int>((a + b - 1) / b); }

// Device address of the library's error word (hca_device_error), or nullptr.
int* device_error_word();

constexpr int kMaxDevices = 64;

// cudaFuncSetAttribute once per (kernel, device): an attribute set while one
// device is current does not carry to another device's context.  `done` holds
// one kernel's flags for one attribute (devices past kMaxDevices set it on
// every call).
template <typename K>
inline int set_func_attr_once(K kernel, cudaFuncAttribute attr, int value, bool (&done)[kMaxDevices]) {
  int dev = 0;
  if (cuda_status(cudaGetDevice(&dev)) != HCA_OK) return HCA_E_CUDA;
  const bool tracked = dev >= 0 && dev < kMaxDevices;
  if (tracked && done[dev]) return HCA_OK;
  if (cuda_status(cudaFuncSetAttribute(kernel, attr, value)) != HCA_OK) return HCA_E_CUDA;
  if (tracked) done[dev] = true;
  return HCA_OK;
}

// Streaming multiprocessors of the current device (queried once per device;
// 148, a B200's count, if the query fails).
inline int device_sm_count() {
  static int n[kMaxDevices] = {};
  int dev = 0, v = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  const bool tracked = dev >= 0 && dev < kMaxDevices;
  if (tracked && n[dev] > 0) return n[dev];
  if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
  if (tracked) n[dev] = v;
  return v;
}

// Geometry of one cached row: N fp8 bytes + R bf16, then N/64 + 1 scale bytes.
struct RowGeom {
  int nope, data_bytes, scale_bytes;
};

__host__ __device__ inline RowGeom row_geom(int head_dim, int rope_dim) {
  RowGeom g;
  g.nope = head_dim - rope_dim;
  g.data_bytes = g.nope + 2 * rope_dim;
  g.scale_bytes = g.nope / kQuantBlock + 1;
  return g;
}

inline bool valid_geom(int head_dim, int rope_dim) {
  return head_dim > rope_dim && rope_dim > 0 && rope_dim % 16 == 0 &&
         (head_dim - rope_dim) % kQuantBlock == 0;
}

// Address of the data row and of the scale bytes of `slot` in a paged cache.
struct RowPtr {
  uint8_t* data;
  uint8_t* scale;
};

__device__ __forceinline__ RowPtr row_ptr(uint8_t* cache, int64_t slot, int page_size,
                                          int64_t page_stride, RowGeom g) {
  const int64_t page = slot / page_size;
  const int off = static_cast<int>(slot - page * page_size);
  uint8_t* base = cache + page * page_stride;
  RowPtr p;
  p.data = base + static_cast<int64_t>(off) * g.data_bytes;
  p.scale = base + static_cast<int64_t>(page_size) * g.data_bytes +
            static_cast<int64_t>(off) * g.scale_bytes;
  return p;
}

// ceil(log2(x)) of a positive finite float, exactly (from its bits).
__device__ __forceinline__ int ceil_log2(float x) {
  const uint32_t b = __float_as_uint(x);
  const int e = static_cast<int>((b >> 23) & 0xff);
  const uint32_t m = b & 0x7fffff;
  if (e == 0) {  // subnormal: x = m * 2^-149
    return (32 - __clz(static_cast<int>(m - 1))) - 149;
  }
  return (e - 127) + (m != 0 ? 1 : 0);
}

// UE8M0 exponent of a block with abs-max `amax`.  `divide` selects
// amax / 448 (KV insert) vs amax * (1/448) (every other quantiser).
__device__ __forceinline__ int ue8m0_exponent(float amax, float floor_v, bool divide) {
  const float a = fmaxf(amax, floor_v);
  const float raw = divide ? __fdiv_rn(a, kFp8Max) : __fmul_rn(a, 1.0f / kFp8Max);
  return ceil_log2(raw);
}

__device__ __forceinline__ uint8_t encode_ue8m0(int e) {
  int v = e + 127;
  v = v < 0 ? 0 : (v > 255 ? 255 : v);
  return static_cast<uint8_t>(v);
}

// 2^e as float for e in the normal range.
__device__ __forceinline__ float exp2i(int e) {
  return __uint_as_float(static_cast<uint32_t>(e + 127) << 23);
}

// clamp(x, +-448) then round-to-nearest-even to e4m3.
__device__ __forceinline__ uint8_t to_e4m3(float x) {
  return static_cast<uint8_t>(__nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3));
}

__device__ __forceinline__ float e4m3_to_float(uint8_t v) {
  __half_raw h = __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(v), __NV_E4M3);
  return __half2float(__half(h));
}

// Two e4m3 bytes (little endian in `v`) to float2.
__device__ __forceinline__ float2 e4m3x2_to_float2(uint16_t v) {
  __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(v), __NV_E4M3);
  return __half22float2(__half2(h));
}

__device__ __forceinline__ float bf16_bits_to_float(uint16_t b) {
  return __uint_as_float(static_cast<uint32_t>(b) << 16);
}

__device__ __forceinline__ uint16_t float_to_bf16_bits(float x) {
  __nv_bfloat16 h = __float2bfloat16_rn(x);
  return *reinterpret_cast<uint16_t*>(&h);
}

__device__ __forceinline__ float bf16_round(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum for blockDim.x <= 1024; `red` holds >= 32 floats.
__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  const int nw = (blockDim.x + 31) >> 5;
  float t = lane < nw ? red[lane] : 0.0f;
  t = warp_sum(t);
  return t;
}

__device__ __forceinline__ float block_max(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  const int nw = (blockDim.x + 31) >> 5;
  float t = lane < nw ? red[lane] : -INFINITY;
  t = warp_max(t);
  return t;
}

// GPT-J rotation of one (even, odd) pair: forward uses +sin, inverse -sin.
__device__ __forceinline__ void rope_pair(float& e, float& o, float c, float s) {
  const float ne = e * c - o * s;
  const float no = o * c + e * s;
  e = ne;
  o = no;
}

}  // namespace hca
