"""Paged fp8 KV-cache layout, insert, gather and the block compressor (CPU oracle).

Layout (``fp8_ds_mla``, generalised from head_dim 512 to any
``D = N + R`` with ``N % 64 == 0``): a page of ``P`` tokens holds
``P`` data rows of ``N`` e4m3 bytes followed by ``R`` bf16 values, then
``P`` scale rows of ``N // 64`` UE8M0 bytes plus one zero pad byte
(``V/models/deepseek_v4/common/ops/cache_utils.py:42-51,149-159``;
``V/models/deepseek_v4/nvidia/flashmla.py:98-111``).  At D=512 that is the
reference's 576 + 8 = 584 bytes per token.

Caches are numpy ``uint8`` arrays ``[num_pages, page_stride]``.
"""

from __future__ import annotations

import numpy as np

from .fp8 import (
    bf16_bytes,
    bf16_from_bytes,
    bf16_round,
    e4m3_to_f32,
    encode_ue8m0,
    quantize_blocks,
)

QUANT_BLOCK = 64


def row_geometry(head_dim: int, rope_dim: int) -> tuple[int, int, int]:
    """``(nope, data_bytes, scale_bytes)`` of one cached row."""
    nope = head_dim - rope_dim
    assert nope % QUANT_BLOCK == 0 and rope_dim % 2 == 0
    return nope, nope + 2 * rope_dim, nope // QUANT_BLOCK + 1


def page_bytes(page_size: int, head_dim: int, rope_dim: int) -> int:
    _, data, scale = row_geometry(head_dim, rope_dim)
    return page_size * (data + scale)


def _row_views(cache: np.ndarray, slot: int, page_size: int, head_dim: int, rope_dim: int):
    nope, data, sbytes = row_geometry(head_dim, rope_dim)
    page, off = divmod(int(slot), page_size)
    base = cache[page]
    d0 = off * data
    s0 = page_size * data + off * sbytes
    return base, d0, s0, nope, data, sbytes


def insert_rows(
    cache: np.ndarray,
    slots: np.ndarray,
    k: np.ndarray,
    page_size: int,
    head_dim: int,
    rope_dim: int,
) -> None:
    """Quantise bf16-valued rows ``k [T, D]`` and write them at ``slots``.

    Restates ``quantize_and_insert_k_kernel``
    (``V/models/deepseek_v4/common/ops/cache_utils.py:23-139``): NoPE in
    64-wide blocks, amax floor 1e-4, ``amax / 448`` by division, RoPE dims
    copied as bf16, pad scale byte zero; ``slot == -1`` is skipped.
    """
    k = bf16_round(np.asarray(k, dtype=np.float32))
    nope, data, sbytes = row_geometry(head_dim, rope_dim)
    q, exp = quantize_blocks(k[:, :nope], QUANT_BLOCK, floor=1e-4, divide=True)
    sc = encode_ue8m0(exp)
    rope = bf16_bytes(k[:, nope:])
    for t, slot in enumerate(np.asarray(slots).tolist()):
        if slot < 0:
            continue
        base, d0, s0, *_ = _row_views(cache, slot, page_size, head_dim, rope_dim)
        base[d0 : d0 + nope] = q[t]
        base[d0 + nope : d0 + data] = rope[t]
        base[s0 : s0 + sbytes - 1] = sc[t]
        base[s0 + sbytes - 1] = 0


def read_rows(
    cache: np.ndarray, slots: np.ndarray, page_size: int, head_dim: int, rope_dim: int
) -> np.ndarray:
    """Dequantise rows at ``slots`` to fp32 ``[n, D]`` (exact in bf16).

    Restates ``_dequantize_and_gather_k_kernel``
    (``V/models/deepseek_v4/common/ops/cache_utils.py:197-320``).
    """
    nope, data, sbytes = row_geometry(head_dim, rope_dim)
    slots = np.asarray(slots, dtype=np.int64).reshape(-1)
    page, off = np.divmod(slots, page_size)
    d_idx = off[:, None] * data + np.arange(data)[None, :]
    s_idx = page_size * data + off[:, None] * sbytes + np.arange(nope // QUANT_BLOCK)[None, :]
    raw = cache[page[:, None], d_idx]  # [n, data]
    exps = cache[page[:, None], s_idx].astype(np.int32) - 127  # [n, nope/64]
    out = np.empty((slots.shape[0], head_dim), dtype=np.float32)
    vals = e4m3_to_f32(raw[:, :nope]).reshape(-1, nope // QUANT_BLOCK, QUANT_BLOCK)
    out[:, :nope] = (vals * np.ldexp(np.float32(1.0), exps)[..., None]).reshape(-1, nope)
    out[:, nope:] = bf16_from_bytes(raw[:, nope:])
    return out


def dequantize_and_gather(
    cache: np.ndarray,
    seq_lens: np.ndarray,
    gather_lens: np.ndarray | None,
    block_table: np.ndarray,
    page_size: int,
    offset: int,
    out: np.ndarray,
    head_dim: int,
    rope_dim: int,
) -> None:
    """Gather positions ``[seq_len - gather_len, seq_len)`` of each request
    into ``out[req, offset + i]`` as bf16-valued fp32.

    Restates ``dequantize_and_gather_k_cache``
    (``V/models/deepseek_v4/common/ops/cache_utils.py:197-320,323-380``).
    """
    for b in range(len(seq_lens)):
        sl = int(seq_lens[b])
        gl = sl if gather_lens is None else int(gather_lens[b])
        start = sl - gl
        for i in range(gl):
            pos = start + i
            slot = int(block_table[b, pos // page_size]) * page_size + pos % page_size
            out[b, offset + i] = read_rows(cache, [slot], page_size, head_dim, rope_dim)[0]


# ---------------------------------------------------------------------------
# RoPE (GPT-J / interleaved pairs on the last R dims)
# ---------------------------------------------------------------------------


def rope_cos_sin_cache(max_pos: int, rope_dim: int, theta: float) -> np.ndarray:
    """fp32 ``[max_pos, R]``: ``cos(p * f)`` then ``sin(p * f)``,
    ``f_i = theta ** (-2i / R)``
    (``V/model_executor/layers/rotary_embedding/base.py:69-92``)."""
    import torch

    inv = 1.0 / (theta ** (torch.arange(0, rope_dim, 2, dtype=torch.float) / rope_dim))
    t = torch.arange(max_pos, dtype=torch.float)
    freqs = torch.einsum("i,j->ij", t, inv)
    return torch.cat([freqs.cos(), freqs.sin()], -1).numpy().astype(np.float32)


def rope_gptj(x: np.ndarray, pos: np.ndarray, cos_sin: np.ndarray, rope_dim: int, inverse=False):
    """Rotate interleaved pairs of the last ``rope_dim`` dims of ``x [..., D]``.

    ``pos`` broadcasts against ``x.shape[:-1]`` (e.g. ``[T, 1]`` for
    ``[T, H, D]``).  Forward:
    ``e' = e cos - o sin, o' = o cos + e sin``
    (``V/models/deepseek_v4/common/ops/fused_compress_quant_cache.py:262-290``);
    inverse flips the sign of ``sin``
    (``V/models/deepseek_v4/common/ops/fused_inv_rope_fp8_quant.py:80-94``).
    """
    x = np.array(x, dtype=np.float32, copy=True)
    half = rope_dim // 2
    cs = cos_sin[np.asarray(pos)]
    cos, sin = cs[..., :half], cs[..., half:]
    r = x[..., -rope_dim:]
    e, o = r[..., 0::2].copy(), r[..., 1::2].copy()
    if inverse:
        sin = -sin
    r[..., 0::2] = e * cos - o * sin
    r[..., 1::2] = o * cos + e * sin
    return x


# ---------------------------------------------------------------------------
# Compressor state + block compressor
# ---------------------------------------------------------------------------


def save_partial_states(
    state: np.ndarray,
    kv: np.ndarray,
    score: np.ndarray,
    ape: np.ndarray,
    positions: np.ndarray,
    slot_mapping: np.ndarray,
    block_size: int,
    ratio: int,
) -> None:
    """``state[slot] = [kv, score + ape[pos % ratio]]`` (fp32), skipping
    ``slot < 0``.  ``state`` is ``[blocks, block_size, 2 * D]``.

    Restates ``_save_partial_states_kernel``
    (``V/models/deepseek_v4/common/ops/save_partial_states.py:48-101``).
    """
    d = kv.shape[-1]
    for t, slot in enumerate(np.asarray(slot_mapping).tolist()):
        if slot < 0:
            continue
        blk, off = divmod(slot, block_size)
        state[blk, off, :d] = kv[t]
        state[blk, off, d : 2 * d] = (
            np.float32(score[t]) + ape[int(positions[t]) % ratio]
        ).astype(np.float32)


def compress_norm_rope_store(
    state: np.ndarray,
    token_to_req: np.ndarray,
    positions: np.ndarray,
    state_slot_mapping: np.ndarray,
    state_block_table: np.ndarray,
    state_block_size: int,
    norm_weight: np.ndarray,
    eps: float,
    cos_sin: np.ndarray,
    kv_cache: np.ndarray,
    kv_slot_mapping: np.ndarray,
    kv_page_size: int,
    head_dim: int,
    rope_dim: int,
    ratio: int = 128,
) -> None:
    """Block compressor: at tokens with ``(p + 1) % ratio == 0`` pool the
    last ``ratio`` states with a per-channel softmax over tokens of the
    score, RMSNorm (fp32, weight), quantise the NoPE dims from the bf16
    rounding of the normed vector, rotate the RoPE dims of the (unrounded)
    normed vector at position ``(p // ratio) * ratio`` and store them as
    bf16, all into the compressed cache slot ``kv_slot_mapping[t]``.

    Restates ``_fused_kv_compress_norm_rope_insert_sparse_attn``
    (``V/models/deepseek_v4/common/ops/fused_compress_quant_cache.py:112-296``)
    with ``OVERLAP = False`` (ratio 128).
    """
    d = head_dim
    nope = d - rope_dim
    for t in range(len(positions)):
        if state_slot_mapping[t] < 0:
            continue
        p = int(positions[t])
        if (p + 1) % ratio != 0:
            continue
        req = int(token_to_req[t])
        pos = np.arange(p - ratio + 1, p + 1)
        valid = pos >= 0
        blk = np.where(valid, state_block_table[req, np.maximum(pos, 0) // state_block_size], 0)
        off = pos % state_block_size
        rows = state[blk, off]  # [ratio, 2D]
        score = np.where(valid[:, None], rows[:, d : 2 * d], -np.inf).astype(np.float64)
        kv = np.where(valid[:, None], rows[:, :d], 0.0).astype(np.float64)
        score = score - score.max(axis=0, keepdims=True)
        w = np.exp(score)
        w = w / w.sum(axis=0, keepdims=True)
        c = (w * kv).sum(axis=0).astype(np.float32)
        var = np.float32((c.astype(np.float64) ** 2).mean())
        normed = (c * np.float32(1.0 / np.sqrt(var + eps)) * norm_weight).astype(np.float32)
        slot = int(kv_slot_mapping[t])
        if slot < 0:
            continue
        q, exp = quantize_blocks(bf16_round(normed[None, :nope]), QUANT_BLOCK, 1e-4, divide=False)
        roped = rope_gptj(normed[None], np.array([(p // ratio) * ratio]), cos_sin, rope_dim)[0]
        base, d0, s0, _, data, sbytes = _row_views(kv_cache, slot, kv_page_size, d, rope_dim)
        base[d0 : d0 + nope] = q[0]
        base[d0 + nope : d0 + data] = bf16_bytes(roped[None, nope:])[0]
        base[s0 : s0 + sbytes - 1] = encode_ue8m0(exp[0])
        base[s0 + sbytes - 1] = 0
