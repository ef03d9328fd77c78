// Sparse HCA attention at the model's own head_dim 512 (448 e4m3 NoPE bytes +
// 64 bf16 RoPE values per cached row, 584-byte rows with their scales).
//
// An M=128 tile of query rows with a 512-wide fp32 O accumulator would fill
// all 512 TMEM columns and leave none for S; its Q tile alone is 128 KB.  So
// each tile is handled by a PAIR of CTAs (a 2-CTA cluster on two SMs), CTA h
// owning head dims [256 h, 256 h + 256):
//   - it holds Q[:, half] (64 KB), gathers and dequantises only its half of
//     every cached row (256 or 320 raw bytes instead of 584), and keeps its
//     half of O in TMEM columns 0-255;
//   - S = Q K^T = Q_0 K_0^T + Q_1 K_1^T: each CTA computes its partial S (an
//     M128 N64 tcgen05.mma chain over 256 dims), writes it into the peer's
//     shared memory (distributed shared memory, 32 KB per 64-row chunk) and
//     adds the peer's partial to its own.  fp32 addition commutes, so both
//     CTAs hold the identical S, run the identical softmax and produce the
//     identical P, m and l;
//   - O_h += P V_h runs on each CTA's own half (V = K, M128 N256).
// Warp roles per CTA: warps 0-3 softmax (one thread per query row), warp 4
// MMA issuer + TMEM owner, warps 5-8 gather + dequant producers, 16 rows of
// every 64-row chunk each.  Exchanges are paced by two mbarriers per CTA:
// x_full counts the bytes of the peer's partial landing here (the peer writes
// it with st.async, complete_tx on this barrier; warp 0 arms each phase with
// the expected byte count), x_empty takes one remote arrival per peer softmax
// warp once it has read the partial this CTA wrote there.  Every wait is
// bounded (device error word); both CTAs meet at a cluster barrier before
// exit, so neither leaves while the other may still write its shared memory.
//
// Work: decode -- split s of tile k of group g, a tile being up to 128 / H
// consecutive tokens of the group (their union of rows, per-token masks);
// the split partials go to the group's workspace rows (tile k at row
// k * tokens_per_tile * H) for the head_dim-512 split merge.  With the
// balanced work list, groups hold at most one tile and pair i runs item i.
// Prefill -- one pair per tile of tokens, rows from the block tables, output
// written directly.
#include "hca_attention.cuh"
#include "hca_common.cuh"
#include "hca_tc.cuh"

namespace hca {
namespace {
namespace tcw {
constexpr int kHalf = 256;          // head dims per CTA of the pair
constexpr int kRowBytes = 576;      // 448 e4m3 + 64 bf16
constexpr int kScaleBytes = 8;      // 7 UE8M0 bytes + pad
constexpr int kCh = 64;             // KV rows per chunk
constexpr int kStages = 2;          // raw ring: one chunk in flight
constexpr int kKBufs = 2;           // bf16 K-tile ring
constexpr int kSoftmaxWarps = 4;
constexpr int kMmaWarp = 4;
constexpr int kProdWarp0 = 5;
constexpr int kProdWarps = 4;
constexpr int kProdRows = kCh / kProdWarps;  // 16
constexpr int kThreads = (kProdWarp0 + kProdWarps) * 32;
constexpr int kQWarps = 5;                   // softmax + MMA warps load Q
constexpr int kRegions = kHalf / 64;         // 64-dim 128B-swizzle regions
constexpr int kQRegion = 128 * 128;          // 128 rows x 128 B
constexpr int kQOff = 0;
constexpr int kKRegion = kCh * 128;          // 64 rows x 128 B
constexpr int kKBuf = kRegions * kKRegion;   // 32768
constexpr int kKOff = kQOff + kRegions * kQRegion;
constexpr int kRawData = 320;                // raw bytes per row and CTA (half 0 uses 256)
constexpr int kRawScale = kCh * kRawData;    // the rows' 8 scale bytes follow the data
constexpr int kRawStage = kRawScale + kCh * kScaleBytes;
constexpr int kRawOff = kKOff + kKBufs * kKBuf;
constexpr int kXOff = kRawOff + kStages * kRawStage;  // the peer's partial S: [16][128] float4
constexpr int kXBytes = 128 * kCh * 4;
constexpr int kMaskOff = kXOff + kXBytes;             // [stage][row] token mask | kOkBit
constexpr int kKMaskOff = kMaskOff + kStages * kCh * 4;  // [kbuf][token][2] 32-bit column masks
constexpr int kBarOff = kKMaskOff + kKBufs * kCh * 4;
// k_full[2] k_empty[2] s_full[2] p_full[2] pv_done[2] q_full x_full x_empty
constexpr int kNumBars = 2 * kKBufs + 9;
constexpr int kMiscOff = kBarOff + kNumBars * 8;
constexpr int kTokOff = kMiscOff + 64;  // [32] + [32] ints
constexpr int kSmemBytes = kTokOff + 256 + 1024;  // + 1024 alignment slack
static_assert(kSmemBytes <= 232448, "one CTA per SM");
static_assert(kXOff % 16 == 0 && kKOff % 1024 == 0 && kBarOff % 8 == 0, "alignment");
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kOkBit = 1u << 31;

__device__ __forceinline__ uint32_t s_col(int buf) { return 256u + buf * 64u; }

// Query row of TMEM lane / smem row `rit`, or -1: R < 128 rows are spread
// evenly over the four lane quadrants (ceil(R / 4) at the start of each).
__device__ __forceinline__ int row_to_query(int rit, int rows_q) {
  const int R = min(128, rows_q);
  if (R <= 0) return -1;
  const int q = (R + 3) >> 2;
  const int quad = rit >> 5, ln = rit & 31;
  const int local = quad * q + ln;
  return (ln < q && local < R) ? local : -1;
}

// Lane quadrants (softmax warps) that hold query rows.
__device__ __forceinline__ int active_quads(int rows_q) {
  const int R = min(128, rows_q);
  if (R <= 0) return 0;
  const int q = (R + 3) >> 2;
  return (R + q - 1) / q;
}

__device__ __forceinline__ void report(int* err, uint32_t* s_err, int code) {
  *s_err = 1;
  if (err) atomicOr(err, code);
}
}  // namespace tcw

template <bool kPrefill>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(tcw::kThreads, 1)
    hca_wide_attention_kernel(const AttnParams P, int tiles_per_group, int* err) {
  using namespace tcw;
  using namespace tc;
  extern __shared__ uint8_t smem_dyn[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
  const uint32_t half = cluster_ctarank();
  const uint32_t peer = half ^ 1u;
  const int H = P.num_heads;

  // ---- this pair's work (both CTAs read the same inputs and agree) ----
  const int work = blockIdx.x >> 1;
  int c_begin = 0, c_end = 1 << 30;
  int64_t item = 0;  // workspace slot (decode)
  int row_off = 0;   // first workspace row of this tile in its group
  bool single = true;
  Group G;
  if (kPrefill) {
    if (!resolve_group<true>(P, work, G)) return;
  } else if (P.sched) {
    // balanced work list over groups of at most one tile of tokens
    const int4 it = reinterpret_cast<const int4*>(P.sched)[work];
    if (it.x < 0) return;
    int t0, t1;
    group_tokens(P, it.x, t0, t1);
    if (t1 - t0 > P.group_tokens || (t1 - t0) * H > P.max_rows) return;
    resolve_tokens(P, t0, t1, G);
    item = work;
    single = P.sched[4 * P.sched_items + 2 * it.x + 1] == 1;
    c_begin = it.z;
    c_end = it.w;
  } else {
    const int split = work % P.num_splits;
    const int gt = work / P.num_splits;
    const int gidx = gt / tiles_per_group, tile = gt % tiles_per_group;
    int t0, t1;
    group_tokens(P, gidx, t0, t1);
    const int a = t0 + tile * P.group_tokens;
    const int b = min(t1, a + P.group_tokens);
    if (a >= b || (t1 - t0) * H > P.max_rows) return;
    resolve_tokens(P, a, b, G);
    row_off = tile * P.group_tokens * H;
    item = static_cast<int64_t>(gidx) * P.num_splits + split;
    single = P.num_splits == 1;
    const int nch = (G.n_win + G.n_comp + kCh - 1) / kCh;
    c_begin = static_cast<int>((static_cast<int64_t>(split) * nch) / P.num_splits);
    c_end = static_cast<int>((static_cast<int64_t>(split + 1) * nch) / P.num_splits);
  }
  const int rows_q = G.ntok * H;  // <= 128: tiles hold at most 128 / H tokens
  if (rows_q > 128 || G.ntok > 31) return;  // 31 mask bits per row (bit 31: loaded)
  const int nact = active_quads(rows_q);
  const int n_u = G.n_win + G.n_comp;
  const int nchunks = (n_u + kCh - 1) / kCh;
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
  uint64_t* x_full = q_full + 1;
  uint64_t* x_empty = x_full + 1;
  uint32_t* misc = reinterpret_cast<uint32_t*>(smem + kMiscOff);  // [0] tmem, [1] err
  uint32_t* mask_s = reinterpret_cast<uint32_t*>(smem + kMaskOff);
  uint32_t* kmask = reinterpret_cast<uint32_t*>(smem + kKMaskOff);
  int* tok_len = reinterpret_cast<int*>(smem + kTokOff);
  int* tok_clen = tok_len + 32;

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
      mbar_init(p_full + b, nact);
      mbar_init(pv_done + b, 1);
    }
    mbar_init(q_full, kQWarps * 32 + kQWarps);
    mbar_init(x_full, 1);      // this CTA's arming arrival; the peer's bytes as tx
    mbar_init(x_empty, nact);  // one arrival per peer softmax warp with rows
    misc[1] = 0;
    mbar_fence_init();
  }
  if (!kPrefill && threadIdx.x < G.ntok) {
    tok_len[threadIdx.x] = P.swa_lens[G.t0 + threadIdx.x];
    tok_clen[threadIdx.x] = P.comp_cache ? P.comp_lens[G.t0 + threadIdx.x] : 0;
  }
  __syncthreads();
  // the peer's barriers are initialised before anyone arrives on them
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = misc[0];

  if (warp < kSoftmaxWarps || warp == kMmaWarp) {
    // Q[:, this half] -> one K-major 128B-swizzled M=128 tile (4 regions of
    // 64 dims); padding rows zero
    const int qt = warp < kSoftmaxWarps ? threadIdx.x : kSoftmaxWarps * 32 + lane;
    for (int it = qt; it < 128 * (kHalf / 8); it += kQWarps * 32) {
      const int rit = it >> 5, ch = it & 31;
      const int region = ch >> 3, c8 = ch & 7;
      const int r = row_to_query(rit, rows_q);
      uint8_t* dst = smem + kQOff + region * kQRegion + rit * 128 + ((c8 ^ (rit & 7)) << 4);
      if (r >= 0) {
        const int tok = G.t0 + r / H, h = r % H;
        cp_async16(dst, P.q + tok * P.q_st + h * P.q_sh + half * kHalf + ch * 8);
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
    const int row0 = (warp - kProdWarp0) * kProdRows;
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
      if (lane >= kProdRows || u >= n_u) return;
      if (kPrefill) {
        bool comp;
        int64_t slot;
        uint32_t m;
        row_source<true>(P, G, u, comp, slot, m);
        R.slot = slot;
        R.comp = comp;
        R.mask = m;
      } else {
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
    // this CTA's part of a row: half 0 = e4m3 bytes 0-255 (scale blocks
    // 0-3); half 1 = e4m3 bytes 256-447 (blocks 4-6) + the 128 RoPE bytes
    const int pieces = half ? 20 : 16;
    auto issue = [&](int i, const Resolved& R) {
      if (i < n) {
        const int s = i % kStages;
        uint8_t* const stage = smem + kRawOff + s * kRawStage;
        const int row = row0 + lane;
        const bool ok = R.slot >= 0;
        uint64_t rbase = 0;
        if (ok) {
          const int64_t psz = R.comp ? P.comp_page : P.swa_page;
          const int64_t page = R.slot / psz, off = R.slot - page * psz;
          const uint8_t* base = (R.comp ? P.comp_cache : P.swa_cache) + page * (R.comp ? P.comp_pstride : P.swa_pstride);
          rbase = reinterpret_cast<uint64_t>(base + off * kRowBytes + half * kHalf);
          cp_async8(stage + kRawScale + row * kScaleBytes, base + psz * kRowBytes + off * kScaleBytes);
        }
        if (lane < kProdRows) mask_s[s * kCh + row] = ok ? (R.mask | kOkBit) : 0u;
#pragma unroll
        for (int k = 0; k < kProdRows * 20 / 32; ++k) {
          const int piece = k * 32 + lane;
          const int r = piece / pieces, j = piece - r * pieces;
          const uint64_t src = __shfl_sync(0xffffffffu, rbase, r);
          if (r < kProdRows && src)
            cp_async16(stage + (row0 + r) * kRawData + j * 16, reinterpret_cast<const void*>(src + j * 16));
        }
      }
      cp_async_commit();
    };
    Resolved rq[kStages - 1];
#pragma unroll
    for (int i = 0; i < kStages - 1; ++i) {
      rq[i].slot = -1;
      if (i < n) resolve(c_begin + i, rq[i]);
    }
#pragma unroll
    for (int i = 0; i < kStages - 1; ++i) issue(i, rq[i]);
    Resolved rn;
    rn.slot = -1;
    if (kStages - 1 < n) resolve(c_begin + kStages - 1, rn);
    for (int i = 0; i < n; ++i) {
      const int s = i % kStages, b = i % kKBufs;
      issue(i + kStages - 1, rn);
      if (i + kStages < n) resolve(c_begin + i + kStages, rn);
      cp_async_wait_group<kStages - 1>();
      __syncwarp();
      if (i >= kKBufs && !mbar_wait(k_empty + b, ((i / kKBufs) - 1) & 1)) {
        report(err, misc + 1, 2);
        break;
      }
      const uint8_t* stage = smem + kRawOff + s * kRawStage;
      uint8_t* kt = smem + kKOff + b * kKBuf;
      // e4m3 regions: lane -> row row0 + lane / 2, 32 values (half lane & 1)
      {
        const int r = row0 + (lane >> 1), hh = lane & 1;
        const bool ok = (mask_s[s * kCh + r] & kOkBit) != 0;
        const int nreg = half ? 3 : 4;
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          if (g < nreg) {
            // rows that are not loaded come out exactly zero (stale bytes)
            const float sc = ok ? exp2i(static_cast<int>(stage[kRawScale + r * kScaleBytes + half * 4 + g]) - 127) : 0.0f;
#pragma unroll
            for (int q = 0; q < 2; ++q) {
              const uint4 in = ok ? *reinterpret_cast<const uint4*>(stage + r * kRawData + g * 64 + hh * 32 + q * 16)
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
                const int c8 = hh * 4 + q * 2 + w2;
                *reinterpret_cast<uint4*>(kt + g * kKRegion + r * 128 + ((c8 ^ (r & 7)) << 4)) = o;
              }
            }
          }
        }
      }
      if (half) {
        // RoPE dims 448-511 (raw bytes 192-319): 16 rows x 8 pieces -> region 3
#pragma unroll
        for (int k = 0; k < kProdRows * 8 / 32; ++k) {
          const int piece = k * 32 + lane;
          const int r = row0 + (piece >> 3), c8 = piece & 7;
          const bool ok = (mask_s[s * kCh + r] & kOkBit) != 0;
          const uint4 v = ok ? *reinterpret_cast<const uint4*>(stage + r * kRawData + 192 + c8 * 16) : make_uint4(0, 0, 0, 0);
          *reinterpret_cast<uint4*>(kt + 3 * kKRegion + r * 128 + ((c8 ^ (r & 7)) << 4)) = v;
        }
      }
      // per-token 16-bit column masks: halfword (k * 4 + warp slice) of buffer b
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
    cp_async_wait_group<0>();
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------------- MMA
    if (lane == 0) {
      const uint32_t idesc_s = umma_idesc_bf16(128, kCh, false, false);   // S: M128 N64, K-major
      const uint32_t idesc_o = umma_idesc_bf16(128, kHalf, false, true);  // O: M128 N256, V MN-major
      // descriptors built once; offsets move the start-address field (/ 16)
      const uint64_t dq = umma_desc_sw128(smem_u32(smem + kQOff), 16, 1024);
      const uint64_t dk = umma_desc_sw128(smem_u32(smem + kKOff), 16, 1024);
      const uint64_t dv = umma_desc_sw128(smem_u32(smem + kKOff), kKRegion, 1024);
      bool ok = mbar_wait(q_full, 0);
      fence_proxy_async_smem();
      auto issue_s = [&](int i) {
        const int kb = i % kKBufs, sb = i & 1;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kHalf / 16; ++kk) {
          const uint32_t qo = ((kk >> 2) * kQRegion + (kk & 3) * 32) >> 4;
          const uint32_t ko = (kb * kKBuf + (kk >> 2) * kKRegion + (kk & 3) * 32) >> 4;
          umma_ss(tmem + s_col(sb), dq + qo, dk + ko, idesc_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(s_full + sb);
      };
      auto issue_pv = [&](int i) {
        const int kb = i % kKBufs, sb = i & 1;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kCh / 16; ++kk)
          umma_ts(tmem, tmem + s_col(sb) + kk * 8, dv + ((kb * kKBuf + kk * 2048) >> 4), idesc_o,
                  (i > 0 || kk > 0) ? 1u : 0u);
        umma_commit(k_empty + kb);
        umma_commit(pv_done + sb);
      };
      // S(0), then per chunk S(i + 1) and P.V(i); suspending, bounded waits
      if (ok && n > 0) {
        ok = mbar_wait(k_full, 0);
        if (ok) issue_s(0);
      }
      for (int i = 0; ok && i < n; ++i) {
        if (i + 1 < n) {
          ok = mbar_wait(k_full + (i + 1) % kKBufs, ((i + 1) / kKBufs) & 1);
          if (!ok) break;
          issue_s(i + 1);
        }
        ok = mbar_wait(p_full + (i & 1), (i >> 1) & 1);
        if (!ok) break;
        issue_pv(i);
      }
      if (!ok) report(err, misc + 1, 4);
    }
    __syncwarp();
  } else if (warp < nact) {
    // --------------------------------------------------------------- softmax
    const int rit = warp * 32 + lane;
    const int r = row_to_query(rit, rows_q);
    const bool row_valid = r >= 0;
    const int tok = row_valid ? r / H : 0;
    const int head = row_valid ? r % H : 0;
    const uint32_t lane_addr = static_cast<uint32_t>(warp * 32) << 16;
    const float scale = P.scale_log2;
    // where this thread's row of partial S goes in the peer, and comes from here
    const uint32_t x_local = smem_u32(smem + kXOff) + rit * 16;
    const uint32_t x_remote = mapa_shared(x_local, peer);
    const uint32_t x_full_remote = mapa_shared(smem_u32(x_full), peer);
    const uint32_t x_empty_remote = mapa_shared(smem_u32(x_empty), peer);
    float m_used = -INFINITY, l = 0.0f;
    bool ok = true;
    for (int i = 0; i < n; ++i) {
      const int b = i & 1, kb = i % kKBufs;
      if (!mbar_wait(s_full + b, (i >> 1) & 1) || !mbar_wait(k_full + kb, (i / kKBufs) & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t lo = row_valid ? kmask[kb * kCh + tok * 2] : 0u;
      const uint32_t hi = row_valid ? kmask[kb * kCh + tok * 2 + 1] : 0u;
      const bool full = (lo & hi) == 0xffffffffu;
      const uint32_t s_addr = tmem + lane_addr + s_col(b);
      uint32_t sr[kCh];
      tmem_ld32(s_addr, sr);
      tmem_ld32(s_addr + 32, sr + 32);
      tmem_wait_ld();
      // ---- exchange the partial S with the peer and add its partial ----
      // Arm this chunk's phase of x_full with the bytes the peer's softmax
      // threads will store.  Phase i - 1 completed before (this thread waited
      // on it), and phase i cannot complete before every warp here has read
      // chunk i - 1: the peer sends chunk i only after all of them arrived
      // on its x_empty.
      if (warp == 0 && lane == 0) mbar_arrive_expect_tx(x_full, static_cast<uint32_t>(nact * 32 * kCh * 4));
      if (i > 0 && !mbar_wait_cluster(x_empty, (i - 1) & 1)) {
        ok = false;
        break;
      }
#pragma unroll
      for (int c4 = 0; c4 < kCh / 4; ++c4)
        st_async_v4(x_remote + c4 * 128 * 16, sr[4 * c4], sr[4 * c4 + 1], sr[4 * c4 + 2], sr[4 * c4 + 3],
                    x_full_remote);
      if (!mbar_wait_cluster(x_full, i & 1)) {
        ok = false;
        break;
      }
#pragma unroll
      for (int c4 = 0; c4 < kCh / 4; ++c4) {
        const float4 v = *reinterpret_cast<const float4*>(smem + kXOff + (c4 * 128 + rit) * 16);
        sr[4 * c4] = __float_as_uint(__uint_as_float(sr[4 * c4]) + v.x);
        sr[4 * c4 + 1] = __float_as_uint(__uint_as_float(sr[4 * c4 + 1]) + v.y);
        sr[4 * c4 + 2] = __float_as_uint(__uint_as_float(sr[4 * c4 + 2]) + v.z);
        sr[4 * c4 + 3] = __float_as_uint(__uint_as_float(sr[4 * c4 + 3]) + v.w);
      }
      // the warp's reads of the buffer are done: one release arrival frees it
      // for the peer's next chunk
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(x_empty_remote);
      // ---- softmax (base 2, lazily raised max) ----
      if (!full) {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          sr[j] = ((lo >> j) & 1u) ? sr[j] : 0xff800000u;
          sr[32 + j] = ((hi >> j) & 1u) ? sr[32 + j] : 0xff800000u;
        }
      }
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
      mx *= scale;
      const bool need = mx > m_used + 8.0f;
      const bool rescale = __any_sync(0xffffffffu, need);
      float f = 1.0f;
      if (rescale) {
        const float new_m = fmaxf(m_used, mx);
        f = m_used == -INFINITY ? 0.0f : exp2f(m_used - new_m);
        l *= f;
        m_used = new_m;
      }
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
      l += a01.x + a01.y;
      if (rescale && i > 0) {
        // O holds chunks < i at the old max: wait for PV(i-1), then scale it
        if (!mbar_wait(pv_done + ((i - 1) & 1), ((i - 1) >> 1) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll 1
        for (int q4 = 0; q4 < kHalf / 32; ++q4) {
          uint32_t o[32];
          tmem_ld32(tmem + lane_addr + q4 * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * f);
          tmem_st32(tmem + lane_addr + q4 * 32, o);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full + b);
    }
    if (ok && n > 0) {
      if (!mbar_wait(pv_done + ((n - 1) & 1), ((n - 1) >> 1) & 1)) ok = false;
      tc_fence_after();
    }
    if (!ok) report(err, misc + 1, 8);
    // ---- epilogue: this CTA's 256 dims of every row ----
    const bool have_o = ok && n > 0 && l > 0.0f;
    const bool any_o = ok && n > 0;
    if (single) {
      const float sink2 = (P.sink && row_valid) ? P.sink[head] * kLog2e : -INFINITY;
      const float inv = have_o ? 1.0f / (l + exp2f(sink2 - m_used)) : 0.0f;
      __nv_bfloat16* orow = P.out + (G.t0 + tok) * P.o_st + head * P.o_sh + half * kHalf;
#pragma unroll 1
      for (int q4 = 0; q4 < kHalf / 32; ++q4) {
        uint32_t o[32];
        if (any_o) {
          tmem_ld32(tmem + lane_addr + q4 * 32, o);
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
      if (P.lse && row_valid && half == 0)
        P.lse[(G.t0 + tok) * H + head] = have_o ? (m_used + log2f(l)) * 0.6931471805599453f : -INFINITY;
    } else {
      // fp32 partial rows staged in the freed Q / K tiles (128 rows x 1 KB,
      // 16-byte chunks XOR-swizzled by row), then stored as whole rows
      float* stage = reinterpret_cast<float*>(smem + kQOff);
#pragma unroll 1
      for (int q4 = 0; q4 < kHalf / 32; ++q4) {
        uint32_t o[32];
        if (any_o) {
          tmem_ld32(tmem + lane_addr + q4 * 32, o);
          tmem_wait_ld();
        }
        if (row_valid && have_o) {
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int j = q4 * 8 + e;
            *reinterpret_cast<float4*>(stage + r * kHalf + ((j ^ (r & 7)) << 2)) =
                make_float4(__uint_as_float(o[4 * e]), __uint_as_float(o[4 * e + 1]), __uint_as_float(o[4 * e + 2]),
                            __uint_as_float(o[4 * e + 3]));
          }
        }
      }
      const int64_t wrow = item * P.max_rows + row_off;
      if (row_valid && half == 0) {
        P.ws_ml[(wrow + r) * 2] = have_o ? m_used : -INFINITY;
        P.ws_ml[(wrow + r) * 2 + 1] = have_o ? l : 0.0f;
      }
      if (n > 0) {
        // the softmax warps with rows meet here (uniform condition); rows
        // whose sum is zero carry stale stage data the merge never reads
        asm volatile("bar.sync 2, %0;\n" ::"r"(nact * 32) : "memory");
        for (int row = warp; row < rows_q; row += nact) {
          float* dst = P.ws_o + (wrow + row) * (2 * kHalf) + half * kHalf;
#pragma unroll
          for (int k = 0; k < 2; ++k) {
            const int j = k * 32 + lane;
            reinterpret_cast<float4*>(dst)[j] = *reinterpret_cast<const float4*>(stage + row * kHalf + ((j ^ (row & 7)) << 2));
          }
        }
      }
    }
  }

  // ---- teardown: free TMEM; neither CTA leaves while its peer may still
  // write into its shared memory ----
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
  cluster_sync();
}

}  // namespace

int launch_wide_attention(const AttnParams& P, bool prefill, int num_groups, int max_group_tokens, int* err,
                          cudaStream_t s) {
  using namespace tcw;
  static bool smem_set[2][kMaxDevices] = {};  // per kernel and device
  auto kernel = prefill ? hca_wide_attention_kernel<true> : hca_wide_attention_kernel<false>;
  if (set_func_attr_once(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes, smem_set[prefill]) != HCA_OK)
    return HCA_E_CUDA;
  const int tiles_per_group = prefill || P.sched ? 1 : (max_group_tokens + P.group_tokens - 1) / P.group_tokens;
  const int64_t pairs = prefill ? static_cast<int64_t>(num_groups)
                        : P.sched ? static_cast<int64_t>(P.sched_items)
                                  : static_cast<int64_t>(num_groups) * tiles_per_group * P.num_splits;
  if (pairs <= 0) return HCA_OK;
  if (2 * pairs > 0x7fffffff) return HCA_E_INVALID;
  kernel<<<dim3(static_cast<unsigned>(2 * pairs)), dim3(kThreads), kSmemBytes, s>>>(P, tiles_per_group, err);
  return HCA_LAUNCH_STATUS();
}

}  // namespace hca
