"""Torch-facing wrappers of the libhca_b200 kernels.

Names, argument meaning and return conventions mirror the reference ops the
kernels replace (cited per function).  Tensors must be CUDA tensors; every
call is stream-ordered on ``torch.cuda.current_stream()`` and allocates
only its documented outputs.  A failing status raises ``HcaError``.
"""

from __future__ import annotations

import torch

from ._lib import call, lib

FP8 = torch.float8_e4m3fn


def _s() -> int:
    return torch.cuda.current_stream().cuda_stream


def _p(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _check_cuda(*ts: torch.Tensor | None) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("libhca_b200 ops take CUDA tensors")


# ---------------------------------------------------------------------------
# metadata
# ---------------------------------------------------------------------------


def token_to_req_indices(query_start_loc: torch.Tensor, num_tokens: int,
                         out: torch.Tensor | None = None) -> torch.Tensor:
    """Device ``repeat_interleave(arange(R), query_lens)``
    (``V/v1/attention/backends/mla/sparse_swa.py:286-294``)."""
    _check_cuda(query_start_loc)
    out = out if out is not None else torch.empty(num_tokens, dtype=torch.int32, device=query_start_loc.device)
    call("hca_token_to_req", _p(out), _p(query_start_loc), query_start_loc.numel() - 1, num_tokens, _s())
    return out[:num_tokens]


def slot_mapping(query_start_loc, seq_lens, block_table, block_size: int, num_tokens: int,
                 out: torch.Tensor | None = None) -> torch.Tensor:
    """Per-token slot in a paged cache with ``block_size``-token pages."""
    _check_cuda(query_start_loc, seq_lens, block_table)
    out = out if out is not None else torch.empty(num_tokens, dtype=torch.int64, device=block_table.device)
    call("hca_slot_mapping", _p(out), _p(query_start_loc), _p(seq_lens), _p(block_table),
         block_table.stride(0), block_table.shape[0], block_size, _s())
    return out[:num_tokens]


def get_compressed_slot_mapping(num_tokens: int, query_start_loc, seq_lens, block_table,
                                block_size: int, compress_ratio: int,
                                out: torch.Tensor | None = None) -> torch.Tensor:
    """``V/v1/attention/backends/mla/compressor_utils.py:53-86``."""
    _check_cuda(query_start_loc, seq_lens, block_table)
    if out is None:
        out = torch.empty(num_tokens, dtype=torch.int64, device=block_table.device)
    call("hca_compressed_slot_mapping", _p(out), out.numel(), _p(query_start_loc), _p(seq_lens),
         _p(block_table), block_table.stride(0), block_table.shape[0], block_size, compress_ratio, _s())
    return out[:num_tokens]


def compute_swa_indices_and_lens(indices: torch.Tensor, lens: torch.Tensor, num_decode_tokens: int,
                                 window_size: int, query_start_loc, seq_lens, token_to_req,
                                 is_valid_token, block_table, block_size: int) -> None:
    """Fills the builder's persistent ``decode_swa_indices [max, W]`` and
    ``decode_swa_lens [max]`` (``V/v1/attention/backends/mla/sparse_swa.py:296-314,449-503``)."""
    _check_cuda(indices, lens, query_start_loc, seq_lens, token_to_req, is_valid_token, block_table)
    idx2 = indices.view(indices.shape[0], -1)
    call("hca_swa_indices_and_lens", _p(idx2), idx2.stride(0), _p(lens), lens.numel(),
         num_decode_tokens, window_size, _p(query_start_loc), _p(seq_lens), _p(token_to_req),
         _p(is_valid_token.view(torch.uint8)), _p(block_table), block_table.stride(0), block_size, _s())


def build_c128a_topk_metadata(positions, compress_ratio: int, num_decode_tokens: int,
                              token_to_req_indices, block_table, block_size: int, slot_mapping_,
                              global_decode_buffer, decode_lens_buffer, prefill_buffer,
                              max_compressed_tokens: int = 8192):
    """``V/v1/attention/backends/mla/flashmla_sparse.py:1032-1080``; returns
    ``(global_decode, decode_lens, prefill_local)`` slices of the buffers."""
    _check_cuda(positions, token_to_req_indices, block_table, slot_mapping_)
    n = positions.shape[0]
    call("hca_c128a_topk_metadata", _p(global_decode_buffer), global_decode_buffer.stride(0),
         _p(decode_lens_buffer), _p(prefill_buffer), prefill_buffer.stride(0), _p(positions), n,
         compress_ratio, max_compressed_tokens, num_decode_tokens, _p(token_to_req_indices),
         _p(block_table), block_table.stride(0), block_size, _p(slot_mapping_), _s())
    return (global_decode_buffer[:num_decode_tokens], decode_lens_buffer[:num_decode_tokens],
            prefill_buffer[: n - num_decode_tokens])


def compute_prefill_gather_lens(seq_lens, query_start_loc, num_prefills: int, num_decodes: int,
                                window_size: int) -> torch.Tensor:
    """``gather_len = q_len + min(prefix, W - 1)``
    (``V/v1/attention/backends/mla/sparse_swa.py:422-446``)."""
    out = torch.empty(num_prefills, dtype=torch.int32, device=seq_lens.device)
    call("hca_prefill_gather_lens", _p(out), _p(seq_lens), _p(query_start_loc), num_prefills,
         num_decodes, window_size, _s())
    return out


def combine_topk_swa_indices(topk_indices, query_start_loc, seq_lens, gather_lens, window_size: int,
                             compress_ratio: int, topk: int, M: int, N: int):
    """``V/models/deepseek_v4/common/ops/cache_utils.py:476-519``."""
    num_tokens = topk_indices.shape[0]
    width = (topk + window_size + 127) // 128 * 128
    comb = torch.empty((num_tokens, width), dtype=torch.int32, device=topk_indices.device)
    lens = torch.empty(num_tokens, dtype=torch.int32, device=topk_indices.device)
    call("hca_combine_topk_swa_indices", _p(comb), comb.stride(0), width, _p(lens), _p(topk_indices),
         topk_indices.stride(0), _p(query_start_loc), _p(seq_lens), _p(gather_lens),
         seq_lens.shape[0], num_tokens, window_size, compress_ratio, topk, M, N, _s())
    return comb, lens


# ---------------------------------------------------------------------------
# norms, cache write, compressor
# ---------------------------------------------------------------------------


def fused_q_kv_rmsnorm(qr, kv, q_weight, kv_weight, eps: float):
    """``V/models/deepseek_v4/common/ops/fused_qk_rmsnorm.py:57-96``."""
    _check_cuda(qr, kv, q_weight, kv_weight)
    qo, ko = torch.empty_like(qr), torch.empty_like(kv)
    if qr.shape[0]:
        call("hca_qk_rmsnorm", _p(qo), qo.stride(0), _p(qr), qr.stride(0), _p(q_weight), qr.shape[1],
             _p(ko), ko.stride(0), _p(kv), kv.stride(0), _p(kv_weight), kv.shape[1], qr.shape[0],
             eps, _s())
    return qo, ko


def fused_qnorm_rope_kv_insert(q, kv, swa_kv_cache, slot_mapping_, positions, cos_sin_cache,
                               padded_heads: int, eps: float, block_size: int, rope_dim: int = 64,
                               out: torch.Tensor | None = None) -> torch.Tensor:
    """Replacement of ``torch.ops._C.fused_deepseek_v4_qnorm_rope_kv_rope_quant_insert``
    (``V/models/deepseek_v4/attention.py:497-542``); returns the padded q."""
    _check_cuda(q, kv, swa_kv_cache, slot_mapping_, positions, cos_sin_cache)
    t, h, d = q.shape
    if out is None:
        out = torch.empty((t, padded_heads, d), dtype=q.dtype, device=q.device)
    n = slot_mapping_.shape[0]
    if n:
        call("hca_qnorm_rope_kv_insert", _p(out), out.stride(0), out.stride(1), padded_heads, _p(q),
             q.stride(0), q.stride(1), h, _p(kv), kv.stride(0), _p(swa_kv_cache), block_size,
             swa_kv_cache.stride(0), _p(slot_mapping_), _p(positions), _p(cos_sin_cache),
             cos_sin_cache.stride(0), n, d, rope_dim, eps, _s())
    return out


def quantize_and_insert_k_cache(k, k_cache, slot_mapping_, block_size: int = 64, rope_dim: int = 64):
    """``V/models/deepseek_v4/common/ops/cache_utils.py:142-194``."""
    _check_cuda(k, k_cache, slot_mapping_)
    n = slot_mapping_.shape[0]
    if n:
        call("hca_quantize_insert_k", _p(k_cache), block_size, k_cache.stride(0), _p(k), k.stride(0),
             _p(slot_mapping_), n, k.shape[1], rope_dim, _s())


def dequantize_and_gather_k_cache(out, k_cache, seq_lens, gather_lens, block_table, block_size: int,
                                  offset: int, rope_dim: int = 64) -> None:
    """``V/models/deepseek_v4/common/ops/cache_utils.py:355-380``."""
    _check_cuda(out, k_cache, seq_lens, block_table)
    call("hca_dequantize_gather_k", _p(out), out.stride(0), out.stride(1), _p(k_cache), block_size,
         k_cache.stride(0), _p(seq_lens), _p(gather_lens), _p(block_table), block_table.stride(0),
         seq_lens.shape[0], offset, out.shape[-1], rope_dim, _s())


def save_partial_states(kv, score, ape, positions, state_cache, slot_mapping_, block_size: int,
                        state_width: int, compress_ratio: int) -> None:
    """``V/models/deepseek_v4/common/ops/save_partial_states.py:9-45``."""
    _check_cuda(kv, score, ape, positions, state_cache, slot_mapping_)
    n = slot_mapping_.shape[0]
    if n:
        call("hca_save_partial_states", _p(state_cache), state_cache.stride(0), state_cache.stride(1),
             _p(kv), kv.stride(0), _p(score), score.stride(0), _p(ape), ape.stride(0), _p(positions),
             _p(slot_mapping_), n, block_size, kv.shape[-1], state_width, compress_ratio, _s())


def compress_norm_rope_store(state_cache, num_actual: int, token_to_req_indices, positions,
                             slot_mapping_, block_table, block_size: int, state_width: int,
                             cos_sin_cache, kv_cache, kv_slot_mapping, kv_block_size: int,
                             head_dim: int, rope_head_dim: int, compress_ratio: int,
                             rms_norm_weight, rms_norm_eps: float) -> None:
    """``compress_norm_rope_store_{triton,cutedsl}``
    (``V/models/deepseek_v4/common/ops/fused_compress_quant_cache.py:34-109``)."""
    _check_cuda(state_cache, token_to_req_indices, positions, slot_mapping_, block_table,
                cos_sin_cache, kv_cache, kv_slot_mapping, rms_norm_weight)
    if num_actual:
        call("hca_compress_norm_rope_store", _p(state_cache), state_cache.stride(0),
             state_cache.stride(1), state_width, _p(token_to_req_indices), _p(positions),
             _p(slot_mapping_), _p(block_table), block_table.stride(0), block_size,
             _p(rms_norm_weight), rms_norm_eps, _p(cos_sin_cache), cos_sin_cache.stride(0),
             _p(kv_cache), _p(kv_slot_mapping), kv_block_size, kv_cache.stride(0), num_actual,
             head_dim, rope_head_dim, compress_ratio, _s())


def decode_prep(q, kv, kv_score, ape, positions, cos_sin_cache, swa_kv_cache, swa_slot_mapping,
                swa_block_size: int, state_cache, state_slot_mapping, state_block_table, state_block_size: int,
                kv_cache, kv_slot_mapping, kv_block_size: int, rms_norm_weight, query_start_loc,
                token_to_req_indices, num_reqs: int, padded_heads: int, eps: float, compress_ratio: int,
                rope_dim: int = 64, out: torch.Tensor | None = None) -> torch.Tensor:
    """``fused_qnorm_rope_kv_insert`` + ``save_partial_states`` +
    ``compress_norm_rope_store`` of a decode-shaped batch (request r owns
    tokens ``query_start_loc[r] .. query_start_loc[r + 1]``) in one launch,
    with the same output bytes; returns the padded q.  ``kv_score`` is the
    compressor's fp32 ``[T, 2 D]`` (kv then score)."""
    _check_cuda(q, kv, kv_score, ape, positions, cos_sin_cache, swa_kv_cache, swa_slot_mapping, state_cache,
                state_slot_mapping, state_block_table, kv_cache, kv_slot_mapping, rms_norm_weight,
                query_start_loc, token_to_req_indices)
    t, h, d = q.shape
    if out is None:
        out = torch.empty((t, padded_heads, d), dtype=q.dtype, device=q.device)
    n = swa_slot_mapping.shape[0]
    if n:
        ks, sc = kv_score[:, :d], kv_score[:, d:]
        call("hca_decode_prep", _p(out), out.stride(0), out.stride(1), padded_heads, _p(q), q.stride(0),
             q.stride(1), h, _p(kv), kv.stride(0), _p(swa_kv_cache), swa_block_size, swa_kv_cache.stride(0),
             _p(swa_slot_mapping), _p(positions), _p(cos_sin_cache), cos_sin_cache.stride(0), _p(ks), ks.stride(0),
             _p(sc), sc.stride(0), _p(ape), ape.stride(0), _p(state_cache), state_cache.stride(0),
             state_cache.stride(1), d, state_block_size, _p(state_slot_mapping), _p(state_block_table),
             state_block_table.stride(0), _p(rms_norm_weight), _p(kv_cache), _p(kv_slot_mapping), kv_block_size,
             kv_cache.stride(0), _p(query_start_loc), _p(token_to_req_indices), num_reqs, n, d, rope_dim,
             compress_ratio, eps, _s())
    return out


# ---------------------------------------------------------------------------
# attention
# ---------------------------------------------------------------------------


def set_attention_wait_limit_ns(limit_ns: int) -> None:
    """Limit of every mbarrier wait of the head_dim-128 attention kernel for
    launches made from now on (``< 0``: the default 2 s; ``0``: a wait not
    already satisfied fails at once).  A diagnostic for testing the bounded
    waits; it has no counterpart in the reference."""
    call("hca_set_attention_wait_limit_ns", int(limit_ns))


def device_error(clear: bool = True) -> int:
    """The library's device error word (non-zero if a kernel gave up on a
    bounded wait); synchronous."""
    import ctypes

    v = ctypes.c_int32(0)
    call("hca_device_error", ctypes.addressof(v), 1 if clear else 0)
    return int(v.value)


class DecodeWorkspace:
    """Persistent zero-initialised split-K workspace, one buffer per device.

    A buffer's address is stable once a CUDA graph may hold it: it only
    grows while no stream on its device is capturing (a grown buffer would
    free the one a captured graph still points at); a request for more than
    it holds during capture raises instead.  Size it before capture by one
    eager call with the largest shapes (or ``reserve``)."""

    def __init__(self):
        self.bufs: dict[int, torch.Tensor] = {}

    def reserve(self, nbytes: int, device) -> None:
        self.get(nbytes, device)

    def get(self, nbytes: int, device) -> torch.Tensor | None:
        if nbytes == 0:
            return None
        device = torch.device(device)
        idx = device.index if device.index is not None else torch.cuda.current_device()
        buf = self.bufs.get(idx)
        if buf is None or buf.numel() < nbytes:
            if torch.cuda.is_current_stream_capturing():
                have = 0 if buf is None else buf.numel()
                raise RuntimeError(f"decode workspace on cuda:{idx} holds {have} bytes, {nbytes} needed while a "
                                   "CUDA graph is being captured; size it with an eager call (or reserve) first")
            buf = torch.zeros(nbytes, dtype=torch.uint8, device=torch.device("cuda", idx))
            self.bufs[idx] = buf
        return buf


_WS = DecodeWorkspace()


def decode_schedule(group_starts, num_tokens: int, swa_lens, comp_lens, max_items: int, out=None):
    """Per-step decode work list (the role of FlashMLA's ``get_mla_metadata``
    tile-scheduler metadata): ``int32[hca_decode_schedule_ints]``, valid for
    every layer of the step.  ``max_items`` = one wave of CTAs (the SM count,
    at least the number of groups)."""
    _check_cuda(swa_lens)
    num_groups = num_tokens if group_starts is None else group_starts.numel() - 1
    n = lib().hca_decode_schedule_ints(num_groups, max_items)
    if n <= 0:
        raise ValueError(f"decode schedule: max_items={max_items} must cover num_groups={num_groups}")
    if out is None or out.numel() != n:
        out = torch.empty(n, dtype=torch.int32, device=swa_lens.device)
    call("hca_decode_schedule", _p(out), max_items, _p(group_starts), num_groups, num_tokens, _p(swa_lens),
         _p(comp_lens), _s())
    return out


def sparse_decode(q, swa_cache, swa_block_size: int, swa_indices, swa_lens, comp_cache,
                  comp_block_size: int, comp_indices, comp_lens, softmax_scale: float, attn_sink,
                  out=None, group_starts=None, max_group_tokens: int = 1, num_splits: int = 1,
                  lse=None, rope_dim: int = 64, workspace: DecodeWorkspace | None = None,
                  schedule=None, max_items: int = 0):
    """Replacement of ``flash_mla_with_kvcache`` for the HCA decode call
    (``V/models/deepseek_v4/nvidia/flashmla.py:286-302``).  ``q`` is
    ``[T, H, D]`` bf16; ``swa_indices``/``comp_indices`` are the builders'
    ``[T, W]`` / ``[T, C]`` int32 tables (any extra middle dim of size 1 is
    accepted); ``group_starts`` groups consecutive-position tokens of one
    request.  With ``schedule`` (from ``decode_schedule``, same
    ``max_items``) the CTAs follow its balanced work list and ``num_splits``
    is unused; otherwise every group gets ``num_splits`` even splits."""
    _check_cuda(q, swa_cache, swa_indices, swa_lens)
    t, h, d = q.shape
    if out is None:
        out = torch.empty_like(q)
    si = swa_indices.reshape(swa_indices.shape[0], -1)
    ci = comp_indices.reshape(comp_indices.shape[0], -1) if comp_indices is not None else None
    num_groups = t if group_starts is None else group_starts.numel() - 1
    ws = None
    nbytes = 0
    slots = (1, max_items) if schedule is not None else (num_groups, num_splits)
    if slots[1] > 1:
        nbytes = lib().hca_sparse_decode_workspace_bytes(slots[0], max_group_tokens, h, d, slots[1])
        ws = (workspace or _WS).get(nbytes, q.device)
    common = (_p(out), out.stride(0), out.stride(1), _p(lse), _p(q), q.stride(0),
              q.stride(1), t, h, d, rope_dim, _p(swa_cache), swa_block_size, swa_cache.stride(0), _p(si),
              si.stride(0), _p(swa_lens), _p(comp_cache), comp_block_size,
              comp_cache.stride(0) if comp_cache is not None else 0, _p(ci),
              ci.stride(0) if ci is not None else 0, _p(comp_lens), _p(group_starts), num_groups,
              max_group_tokens, softmax_scale, _p(attn_sink))
    if schedule is not None:
        call("hca_sparse_decode_scheduled", *common, _p(schedule), max_items, _p(ws), nbytes, _s())
    else:
        call("hca_sparse_decode", *common, num_splits, _p(ws), nbytes, _s())
    return out


def sparse_prefill(q, query_start_loc, seq_lens, swa_cache, swa_block_size: int, swa_block_table,
                   comp_cache, comp_block_size: int, comp_block_table, window: int,
                   compress_ratio: int, softmax_scale: float, attn_sink, out=None,
                   rope_dim: int = 64):
    """Prefill attention straight from the fp8 caches (replaces the gather +
    ``flash_mla_sparse_fwd`` of ``V/models/deepseek_v4/nvidia/flashmla.py:304-424``)."""
    _check_cuda(q, query_start_loc, seq_lens, swa_cache, swa_block_table)
    t, h, d = q.shape
    if out is None:
        out = torch.empty_like(q)
    call("hca_sparse_prefill", _p(out), out.stride(0), out.stride(1), _p(q), q.stride(0), q.stride(1),
         h, d, rope_dim, _p(query_start_loc), _p(seq_lens), seq_lens.shape[0], t, _p(swa_cache),
         swa_block_size, swa_cache.stride(0), _p(swa_block_table), swa_block_table.stride(0),
         _p(comp_cache), comp_block_size, comp_cache.stride(0) if comp_cache is not None else 0,
         _p(comp_block_table), comp_block_table.stride(0) if comp_block_table is not None else 0,
         window, compress_ratio, softmax_scale, _p(attn_sink), _s())
    return out


# ---------------------------------------------------------------------------
# output path
# ---------------------------------------------------------------------------


def _aligned(n: int) -> int:
    return (n + 3) // 4 * 4


def _quant_out(out, scale, n_groups: int, t: int, hpg: int, d: int, device):
    """The ``(data [G, T, HPG*D] e4m3, scale [G, HPG, round_up(T, 4)] int32)``
    buffers of the VHA quant: the caller's or new ones."""
    if out is None:
        out = torch.empty((n_groups, t, hpg * d), dtype=FP8, device=device)
    if scale is None:
        scale = torch.empty((n_groups, hpg, _aligned(t)), dtype=torch.int32, device=device)
    assert out.shape == (n_groups, t, hpg * d) and out.dtype == FP8 and out.is_contiguous()
    assert scale.shape == (n_groups, hpg, _aligned(t)) and scale.dtype == torch.int32 and scale.is_contiguous()
    return out, scale


def vha_inv_rope_fp8_quant(o, mix, positions, cos_sin_cache, n_groups: int, nope_dim: int,
                           rope_dim: int, out=None, scale_out=None):
    """``E/nvidia/attention.py:232-285``: returns ``(data [T, G, HPG*D] e4m3,
    scale [T, G, HPG] int32)`` views with the plugin's strides (of ``out``
    ``[G, T, HPG*D]`` and ``scale_out`` ``[G, HPG, round_up(T, 4)]`` when
    given)."""
    _check_cuda(o, mix, positions, cos_sin_cache)
    t, h, d = o.shape
    assert d == nope_dim + rope_dim and o.stride(-1) == 1
    hpg = h // n_groups
    out, scale = _quant_out(out, scale_out, n_groups, t, hpg, d, o.device)
    if t:
        call("hca_vha_inv_rope_fp8_quant", _p(out), _p(scale), _p(o), o.stride(0), o.stride(1),
             _p(mix), _p(positions), _p(cos_sin_cache), cos_sin_cache.stride(0), t, h, n_groups, d,
             rope_dim, _s())
    return out.transpose(0, 1), scale.permute(2, 0, 1)[:t]


def sparse_decode_vha_fp8_quant(q, swa_cache, swa_block_size: int, swa_indices, swa_lens, comp_cache,
                                comp_block_size: int, comp_indices, comp_lens, softmax_scale: float,
                                attn_sink, group_starts, max_group_tokens: int, schedule, max_items: int,
                                mix, positions, cos_sin_cache, n_groups: int, rope_dim: int = 64,
                                workspace: DecodeWorkspace | None = None, out=None, scale_out=None):
    """Decode attention (scheduled) fused with the VHA mix, inverse RoPE and
    FP8 quant: ``sparse_decode`` followed by ``vha_inv_rope_fp8_quant`` in two
    launches, without the bf16 O round trip.  Returns the same
    ``(data [T, G, HPG*D] e4m3, scale [T, G, HPG] int32)`` views."""
    _check_cuda(q, swa_cache, swa_indices, swa_lens, mix, positions, cos_sin_cache, schedule)
    t, h, d = q.shape
    hpg = h // n_groups
    out, scale = _quant_out(out, scale_out, n_groups, t, hpg, d, q.device)
    if t == 0:
        return out.transpose(0, 1), scale.permute(2, 0, 1)[:t]
    si = swa_indices.reshape(swa_indices.shape[0], -1)
    ci = comp_indices.reshape(comp_indices.shape[0], -1) if comp_indices is not None else None
    num_groups = t if group_starts is None else group_starts.numel() - 1
    nbytes = lib().hca_sparse_decode_vha_workspace_bytes(max_items, max_group_tokens, h, d)
    ws = (workspace or _WS).get(nbytes, q.device)
    call("hca_sparse_decode_vha_fp8_quant", _p(out), _p(scale), _p(q), q.stride(0), q.stride(1), t, h, d,
         rope_dim, _p(swa_cache), swa_block_size, swa_cache.stride(0), _p(si), si.stride(0), _p(swa_lens),
         _p(comp_cache), comp_block_size, comp_cache.stride(0) if comp_cache is not None else 0, _p(ci),
         ci.stride(0) if ci is not None else 0, _p(comp_lens), _p(group_starts), num_groups, max_group_tokens,
         softmax_scale, _p(attn_sink), _p(schedule), max_items, _p(mix), _p(positions), _p(cos_sin_cache),
         cos_sin_cache.stride(0), n_groups, _p(ws), nbytes, _s())
    return out.transpose(0, 1), scale.permute(2, 0, 1)[:t]


def fused_inv_rope_fp8_quant(o, positions, cos_sin_cache, n_groups: int, heads_per_group: int,
                             nope_dim: int = 448, rope_dim: int = 64):
    """``V/models/deepseek_v4/common/ops/fused_inv_rope_fp8_quant.py:138-193``
    with ``tma_aligned_scales=True``: ``(fp8 [T, G, D'], scale [T, G, packs])``."""
    _check_cuda(o, positions, cos_sin_cache)
    t, h, d = o.shape
    dd = heads_per_group * d
    packs = (dd // 128 + 3) // 4
    out = torch.empty((n_groups, t, dd), dtype=FP8, device=o.device)
    al = _aligned(t)
    buf = torch.empty(n_groups * packs * al, dtype=torch.int32, device=o.device)
    if t:
        call("hca_inv_rope_fp8_quant", _p(out), _p(buf), _p(o), o.stride(0), o.stride(1),
             _p(positions), _p(cos_sin_cache), cos_sin_cache.stride(0), t, h, n_groups, d, rope_dim, _s())
    scale = buf.as_strided((n_groups, t, packs), (packs * al, 1, al))
    return out.transpose(0, 1), scale.transpose(0, 1)


def vha_inv_rope(o, mix, positions, cos_sin_cache, rope_dim: int = 64, out=None):
    """``inverse_rope(m @ o)`` in bf16 for the bf16 ``wo_a`` path."""
    _check_cuda(o, positions, cos_sin_cache)
    t, h, d = o.shape
    out = out if out is not None else torch.empty((t, h, d), dtype=o.dtype, device=o.device)
    if t:
        call("hca_vha_inv_rope", _p(out), out.stride(0), out.stride(1), _p(o), o.stride(0),
             o.stride(1), _p(mix), _p(positions), _p(cos_sin_cache), cos_sin_cache.stride(0), t, h, d,
             rope_dim, _s())
    return out


def sigmoid_mul_quant_fp8(x, gate):
    """``E/nvidia/attention.py:330-361``: ``(fp8 [rows, hidden], scale [rows, packs])``."""
    _check_cuda(x, gate)
    rows, hidden = x.shape
    assert gate.shape == x.shape and hidden % 512 == 0
    out = torch.empty((rows, hidden), dtype=FP8, device=x.device)
    packs = hidden // 512
    scale = torch.empty_strided((rows, packs), (1, _aligned(rows)), dtype=torch.int32, device=x.device)
    if rows:
        call("hca_sigmoid_mul_quant_fp8", _p(out), _p(scale), _p(x), x.stride(0), _p(gate),
             gate.stride(0), rows, hidden, _s())
    return out, scale




# split-K partial tiles of the FP8 GEMM (one buffer per device; calls are
# ordered on the current stream)
_GEMM_WS = DecodeWorkspace()


def fp8_grouped_gemm(x, x_scale, w, w_scale, out=None, workspace: DecodeWorkspace | None = None):
    """Block-scaled FP8 GEMM of the output path: the grouped ``wo_a`` einsum
    ``"bhr,hdr->bhd"`` (``V/models/deepseek_v4/attention.py:317-347``) for a
    3-D ``x [T, G, K]`` and ``w [G, N, K]``, or the gated ``wo_b`` linear
    (``E/nvidia/attention.py:364-395``) for a 2-D ``x [T, K]`` and ``w [N, K]``.
    ``x`` e4m3 with the int32 UE8M0 scales the quant kernels write
    (``[T, G, packs]`` or ``[T, packs]``, one or four 128-blocks per int32);
    ``w`` e4m3 with fp32 128 x 128 block scales ``[G, ceil(N/128), K/128]`` (or
    ``[ceil(N/128), K/128]``).  Returns bf16 ``[T, G, N]`` (or ``[T, N]``)."""
    _check_cuda(x, x_scale, w, w_scale)
    flat = x.dim() == 2
    if flat:
        x, x_scale, w, w_scale = x.unsqueeze(1), x_scale.unsqueeze(1), w.unsqueeze(0), w_scale.unsqueeze(0)
    t, g, k = x.shape
    n = w.shape[1]
    assert x.dtype == FP8 and w.dtype == FP8 and x.stride(2) == 1
    assert w.shape == (g, n, k) and w.is_contiguous()
    assert w_scale.dtype == torch.float32 and w_scale.is_contiguous() and w_scale.shape == (g, (n + 127) // 128, k // 128)
    assert x_scale.dtype == torch.int32 and x_scale.shape[:2] == (t, g) and k % 128 == 0
    per_int = (k // 128) // x_scale.shape[2]
    assert per_int in (1, 4) and per_int * x_scale.shape[2] == k // 128
    if out is None:
        out = torch.empty((t, g, n), dtype=torch.bfloat16, device=x.device)
    elif flat:
        out = out.unsqueeze(1)
    assert out.shape == (t, g, n) and out.dtype == torch.bfloat16 and out.stride(2) == 1
    if t:
        nbytes = lib().hca_fp8_grouped_gemm_workspace_bytes(t, g, n, k)
        ws = (workspace or _GEMM_WS).get(nbytes, x.device) if nbytes > 0 else None
        call("hca_fp8_grouped_gemm", _p(out), out.stride(0), out.stride(1) if g > 1 else 0, _p(x), x.stride(0),
             x.stride(1) if g > 1 else 0, _p(x_scale), x_scale.stride(0), x_scale.stride(1) if g > 1 else 0,
             x_scale.stride(2), per_int, _p(w), _p(w_scale), t, g, n, k, _p(ws), nbytes, _s())
    return out.squeeze(1) if flat else out


def quantize_weight_block_fp8(w: torch.Tensor, block: int = 128):
    """Load-time 128 x 128 block FP8 quant of a bf16 weight ``[..., N, K]``:
    power-of-two (UE8M0-valued) fp32 block scales, the format the Blackwell
    DeepGEMM path runs block-FP8 checkpoints in (``E/nvidia/quant_config.py``;
    ``dequantize_block_fp8`` there is its inverse).  Returns ``(w_fp8,
    scale [..., ceil(N/128), K/128])``.  A one-off weight transform, not a
    step of the forward pass."""
    *lead, n, k = w.shape
    assert k % block == 0
    nb = (n + block - 1) // block
    wf = torch.zeros((*lead, nb * block, k), dtype=torch.float32, device=w.device)
    wf[..., :n, :] = w.float()
    blocks = wf.view(*lead, nb, block, k // block, block)
    amax = blocks.abs().amax(dim=(-3, -1)).clamp_min(1e-10)
    e = torch.ceil(torch.log2(amax / 448.0))
    scale = torch.exp2(e)
    q = (blocks / scale[..., :, None, :, None]).clamp(-448.0, 448.0).to(FP8)
    return q.view(*lead, nb * block, k)[..., :n, :].contiguous(), scale.contiguous()
