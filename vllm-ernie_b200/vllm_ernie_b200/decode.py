"""The HCA decode hot path between the input projections and ``wo_a``.

Per step (shared by all HCA layers, as the reference builds attention
metadata once per step): slot mappings, window indices and C128A indices.
Per layer: Q head-norm + RoPE with the fp8 SWA insert, compressor state save
and block compression, sparse attention over ``[window || compressed]``, and
the VHA post-mix fused with inverse RoPE and the FP8 quant of ``wo_a``'s
input.  Mirrors ``DeepseekV4MultiHeadLatentAttentionWrapper.attention_impl``
(``V/models/deepseek_v4/attention.py:409-495``) + the HCA mixin's output path
(``E/nvidia/attention.py:471-539``) without the GEMMs.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import ops
from .backend import decode_group_rows
from .synthetic import DecodeBatch, HCADims, LayerCaches

SM_COUNT_B200 = 148


@dataclass
class DecodeMetadata:
    num_tokens: int
    token_to_req: torch.Tensor
    swa_slot: torch.Tensor
    state_slot: torch.Tensor
    comp_slot: torch.Tensor
    is_valid: torch.Tensor
    swa_indices: torch.Tensor
    swa_lens: torch.Tensor
    comp_indices: torch.Tensor
    comp_lens: torch.Tensor
    group_starts: torch.Tensor
    max_group_tokens: int
    num_splits: int
    schedule: torch.Tensor | None = None  # balanced work list (None: uniform num_splits)
    max_items: int = 0


def choose_num_splits(num_groups: int, sm_count: int = SM_COUNT_B200) -> int:
    """Split-K factor: as many splits per group as fit one wave of one CTA
    per SM (the decode kernel holds a whole SM: 512 TMEM columns, ~150 KB
    shared memory)."""
    if num_groups <= 0:
        return 1
    return max(1, min(16, sm_count // num_groups))


def build_decode_metadata(batch: DecodeBatch, max_compressed: int, num_splits: int | None = None,
                          buffers: dict | None = None, sm_count: int = SM_COUNT_B200,
                          max_items: int | None = None) -> DecodeMetadata:
    """All per-step index tables, on the device, through the library's
    builders (bit-exact with the reference's).  ``num_splits=None`` builds the
    balanced work list for one wave of ``sm_count`` CTAs (``max_items``
    overrides the item count); an integer forces that many uniform splits per
    group."""
    d = batch.dims
    dev = batch.device
    T = batch.num_tokens
    qsl, sl = batch.query_start_loc, batch.seq_lens
    buf = buffers if buffers is not None else {}

    def get(name, shape, dtype):
        t = buf.get(name)
        if t is None or t.shape != shape:
            t = torch.empty(shape, dtype=dtype, device=dev)
            buf[name] = t
        return t

    t2r = ops.token_to_req_indices(qsl, T, out=get("t2r", (T,), torch.int32))
    swa_slot = ops.slot_mapping(qsl, sl, batch.swa_bt, d.swa_page, T, out=get("swa_slot", (T,), torch.int64))
    state_slot = ops.slot_mapping(qsl, sl, batch.state_bt, d.state_page, T, out=get("state_slot", (T,), torch.int64))
    comp_slot = ops.get_compressed_slot_mapping(T, qsl, sl, batch.comp_bt, d.comp_page, d.ratio,
                                                out=get("comp_slot", (T,), torch.int64))
    is_valid = get("is_valid", (T,), torch.bool)
    torch.ge(swa_slot, 0, out=is_valid)
    swa_idx = get("swa_idx", (T, d.window), torch.int32)
    swa_lens = get("swa_lens", (T,), torch.int32)
    ops.compute_swa_indices_and_lens(swa_idx, swa_lens, T, d.window, qsl, sl, t2r, is_valid,
                                     batch.swa_bt, d.swa_page)
    cidx = get("comp_idx", (T, max_compressed), torch.int32)
    clens = get("comp_lens", (T,), torch.int32)
    pre = get("comp_prefill", (1, max_compressed), torch.int32)
    ops.build_c128a_topk_metadata(batch.positions, d.ratio, T, t2r, batch.comp_bt, d.comp_page,
                                  swa_slot, cidx, clens, pre, max_compressed)
    max_g = max(1, min(batch.q_per_seq, decode_group_rows(d.head_dim) // d.heads))
    if max_g < batch.q_per_seq:
        # split each request's tokens into sub-groups of max_g tokens (a fixed
        # table for the batch shape: built once, so steps stay graph-capturable)
        key = ("group_starts", batch.num_reqs, batch.q_per_seq, max_g)
        gs = buf.get(key)
        if gs is None:
            starts = [t for r in range(batch.num_reqs) for t in
                      range(r * batch.q_per_seq, (r + 1) * batch.q_per_seq, max_g)] + [T]
            gs = torch.tensor(starts, dtype=torch.int32, device=dev)
            buf[key] = gs
    else:
        gs = qsl
    ngroups = gs.numel() - 1
    if num_splits is not None:
        return DecodeMetadata(T, t2r, swa_slot, state_slot, comp_slot, is_valid, swa_idx, swa_lens,
                              cidx, clens, gs, max_g, num_splits)
    # one wave: a CTA per SM, or a CTA pair per two SMs at head_dim 512
    items = max(max_items or (sm_count if d.head_dim == 128 else sm_count // 2), ngroups)
    sched = ops.decode_schedule(gs, T, swa_lens, clens, items, out=buf.get("schedule"))
    buf["schedule"] = sched
    return DecodeMetadata(T, t2r, swa_slot, state_slot, comp_slot, is_valid, swa_idx, swa_lens,
                          cidx, clens, gs, max_g, 1, sched, items)


@dataclass
class LayerWeights:
    """The HCA weights the decode path touches (no GEMM weights)."""

    attn_sink: torch.Tensor          # [H] fp32
    ape: torch.Tensor                # [ratio, D] fp32
    comp_norm: torch.Tensor          # [D] fp32
    vha_mix: torch.Tensor            # [H, H] bf16 (I + V U^T)


def random_layer_weights(dims: HCADims, device, seed: int) -> LayerWeights:
    g = torch.Generator(device=device).manual_seed(seed)
    h, d = dims.heads, dims.head_dim
    u = torch.randn(h, 16, generator=g, device=device) * 0.02
    v = torch.randn(h, 16, generator=g, device=device) * 0.02
    return LayerWeights(
        attn_sink=torch.randn(h, generator=g, device=device),
        ape=torch.randn(dims.ratio, d, generator=g, device=device) * 0.02,
        comp_norm=1.0 + 0.02 * torch.randn(d, generator=g, device=device),
        vha_mix=(torch.eye(h, device=device) + v @ u.T).to(torch.bfloat16),
    )


def decode_layer(batch: DecodeBatch, md: DecodeMetadata, caches: LayerCaches, w: LayerWeights,
                 q_raw: torch.Tensor, kv: torch.Tensor, kv_score: torch.Tensor,
                 cos_sin: torch.Tensor, q_buf: torch.Tensor | None = None,
                 o_buf: torch.Tensor | None = None, quantize: bool = True):
    """One layer of the decode hot path.  Returns ``(fp8 [T, G, HPG*D],
    scale [T, G, HPG])`` (``quantize``) or the bf16 ``[T, H, D]`` output of
    VHA + inverse RoPE."""
    d = batch.dims
    # Q head-norm + RoPE, KV insert, state save and block compression: one
    # launch (the same bytes as the three ops in sequence)
    q = ops.decode_prep(q_raw, kv, kv_score, w.ape, batch.positions, cos_sin, caches.swa, md.swa_slot, d.swa_page,
                        caches.state, md.state_slot, batch.state_bt, d.state_page, caches.comp, md.comp_slot,
                        d.comp_page, w.comp_norm, batch.query_start_loc, md.token_to_req, batch.num_reqs, d.heads,
                        d.eps, d.ratio, d.rope_dim, out=q_buf)
    if quantize and md.schedule is not None and d.head_dim == 128:
        # attention + VHA + inverse RoPE + FP8 quant without the bf16 O round trip
        return ops.sparse_decode_vha_fp8_quant(
            q, caches.swa, d.swa_page, md.swa_indices, md.swa_lens, caches.comp, d.comp_page, md.comp_indices,
            md.comp_lens, d.head_dim ** -0.5, w.attn_sink, md.group_starts, md.max_group_tokens, md.schedule,
            md.max_items, w.vha_mix, batch.positions, cos_sin, d.n_groups, d.rope_dim)
    o = ops.sparse_decode(q, caches.swa, d.swa_page, md.swa_indices, md.swa_lens, caches.comp,
                          d.comp_page, md.comp_indices, md.comp_lens, d.head_dim ** -0.5, w.attn_sink,
                          out=o_buf, group_starts=md.group_starts, max_group_tokens=md.max_group_tokens,
                          num_splits=md.num_splits, rope_dim=d.rope_dim, schedule=md.schedule,
                          max_items=md.max_items)
    if not quantize:
        return ops.vha_inv_rope(o, w.vha_mix, batch.positions, cos_sin, d.rope_dim)
    return ops.vha_inv_rope_fp8_quant(o, w.vha_mix, batch.positions, cos_sin, d.n_groups, d.nope,
                                      d.rope_dim)


# ---------------------------------------------------------------------------
# chunked prefill (the same layer path over a chunk of tokens per request)
# ---------------------------------------------------------------------------


@dataclass
class PrefillMetadata:
    num_tokens: int
    token_to_req: torch.Tensor
    swa_slot: torch.Tensor
    state_slot: torch.Tensor
    comp_slot: torch.Tensor


def build_prefill_metadata(batch: DecodeBatch, buffers: dict | None = None) -> PrefillMetadata:
    """Per-step slot maps of a prefill chunk (the attention reads the caches
    through the block tables, so no index tables are built)."""
    d = batch.dims
    T = batch.num_tokens
    qsl, sl = batch.query_start_loc, batch.seq_lens
    buf = buffers if buffers is not None else {}

    def get(name, shape, dtype):
        t = buf.get(name)
        if t is None or t.shape != shape:
            t = torch.empty(shape, dtype=dtype, device=batch.device)
            buf[name] = t
        return t

    t2r = ops.token_to_req_indices(qsl, T, out=get("t2r", (T,), torch.int32))
    swa_slot = ops.slot_mapping(qsl, sl, batch.swa_bt, d.swa_page, T, out=get("swa_slot", (T,), torch.int64))
    state_slot = ops.slot_mapping(qsl, sl, batch.state_bt, d.state_page, T, out=get("state_slot", (T,), torch.int64))
    comp_slot = ops.get_compressed_slot_mapping(T, qsl, sl, batch.comp_bt, d.comp_page, d.ratio,
                                                out=get("comp_slot", (T,), torch.int64))
    return PrefillMetadata(T, t2r, swa_slot, state_slot, comp_slot)


def prefill_layer(batch: DecodeBatch, md: PrefillMetadata, caches: LayerCaches, w: LayerWeights,
                  q_raw: torch.Tensor, kv: torch.Tensor, kv_score: torch.Tensor, cos_sin: torch.Tensor,
                  q_buf: torch.Tensor | None = None, o_buf: torch.Tensor | None = None):
    """One layer of the chunked-prefill path: Q prep + SWA insert, state save,
    block compression (every completed 128-block of the chunk), attention
    straight from the fp8 caches, VHA + inverse RoPE + FP8 quant."""
    d = batch.dims
    T = md.num_tokens
    q = ops.fused_qnorm_rope_kv_insert(q_raw, kv, caches.swa, md.swa_slot, batch.positions, cos_sin,
                                       d.heads, d.eps, d.swa_page, d.rope_dim, out=q_buf)
    ops.save_partial_states(kv_score[:, : d.head_dim], kv_score[:, d.head_dim:], w.ape, batch.positions,
                            caches.state, md.state_slot, d.state_page, d.head_dim, d.ratio)
    ops.compress_norm_rope_store(caches.state, T, md.token_to_req, batch.positions, md.state_slot,
                                 batch.state_bt, d.state_page, d.head_dim, cos_sin, caches.comp,
                                 md.comp_slot, d.comp_page, d.head_dim, d.rope_dim, d.ratio,
                                 w.comp_norm, d.eps)
    o = ops.sparse_prefill(q, batch.query_start_loc, batch.seq_lens, caches.swa, d.swa_page, batch.swa_bt,
                           caches.comp, d.comp_page, batch.comp_bt, d.window, d.ratio, d.head_dim ** -0.5,
                           w.attn_sink, out=o_buf, rope_dim=d.rope_dim)
    return ops.vha_inv_rope_fp8_quant(o, w.vha_mix, batch.positions, cos_sin, d.n_groups, d.nope, d.rope_dim)
