"""Norms, Q/KV preparation and the HCA output path (CPU oracle)."""

from __future__ import annotations

import numpy as np

from .fp8 import bf16_round, e4m3_bytes, ue8m0_exponent
from .cache import rope_gptj


def rms_norm(x: np.ndarray, weight: np.ndarray | None, eps: float) -> np.ndarray:
    """fp32 RMSNorm with one rounding at the end left to the caller
    (``V/models/deepseek_v4/common/ops/fused_qk_rmsnorm.py:44-54``)."""
    x = np.asarray(x, dtype=np.float32)
    var = (x.astype(np.float64) ** 2).mean(axis=-1, keepdims=True)
    y = x * (1.0 / np.sqrt(var + eps)).astype(np.float32)
    if weight is not None:
        y = y * np.asarray(weight, dtype=np.float32)
    return y.astype(np.float32)


def q_prep(q: np.ndarray, positions: np.ndarray, cos_sin: np.ndarray, rope_dim: int, eps: float,
           padded_heads: int | None = None) -> np.ndarray:
    """Query side of the fused insert op: weightless per-head RMSNorm, GPT-J
    RoPE of the last R dims at the token position, bf16 output, heads
    zero-padded to ``padded_heads``
    (``V/models/deepseek_v4/attention.py:208-209,497-542``)."""
    t, h, d = q.shape
    y = rms_norm(q, None, eps)
    y = rope_gptj(y, np.asarray(positions)[:, None], cos_sin, rope_dim)
    y = bf16_round(y)
    if padded_heads is not None and padded_heads > h:
        y = np.concatenate([y, np.zeros((t, padded_heads - h, d), np.float32)], axis=1)
    return y


def kv_rope(kv: np.ndarray, positions: np.ndarray, cos_sin: np.ndarray, rope_dim: int) -> np.ndarray:
    """KV side of the fused insert op before quantisation: GPT-J RoPE of the
    last R dims in fp32, bf16 rounding (the readable insert spec then
    quantises this row: ``V/models/deepseek_v4/common/ops/cache_utils.py:23-139``)."""
    y = rope_gptj(np.asarray(kv, np.float32), np.asarray(positions), cos_sin, rope_dim)
    return bf16_round(y)


def vha_fold(u: np.ndarray, v: np.ndarray) -> np.ndarray:
    """``m = I + V U^T`` (``E/nvidia/attention.py:140-146``)."""
    return np.eye(u.shape[0], dtype=np.float32) + v.astype(np.float32) @ u.astype(np.float32).T


def inv_rope_fp8_quant(o: np.ndarray, positions: np.ndarray, cos_sin: np.ndarray,
                       n_groups: int, rope_dim: int, quant: bool = True):
    """Inverse GPT-J RoPE of the last R dims at the query position, then
    UE8M0 1x128 FP8 quant (amax floor 1e-10, multiply by fp32 1/448).

    Restates ``_fused_inv_rope_fp8_quant_per_head``
    (``V/models/deepseek_v4/common/ops/fused_inv_rope_fp8_quant.py:17-136``).
    Returns ``(fp8 [G, T, HPG * D] bytes, exponents [T, H, D // 128])`` or
    the rotated fp32 values when ``quant`` is False.
    """
    t, h, d = o.shape
    y = rope_gptj(np.asarray(o, np.float32), np.asarray(positions)[:, None], cos_sin, rope_dim,
                  inverse=True)
    if not quant:
        return y
    yb = y.reshape(t, h, d // 128, 128)
    exp = ue8m0_exponent(np.abs(yb).max(-1), 1e-10, divide=False)
    inv = np.ldexp(np.float32(1.0), -exp)
    q = e4m3_bytes(yb * inv[..., None]).reshape(t, h, d)
    hpg = h // n_groups
    q = q.reshape(t, n_groups, hpg * d).transpose(1, 0, 2).copy()
    return q, exp


def vha_inv_rope_fp8_quant(o: np.ndarray, mix_bf16: np.ndarray, positions: np.ndarray,
                           cos_sin: np.ndarray, n_groups: int, rope_dim: int):
    """The plugin's fused VHA + inverse RoPE + FP8 kernel: ``y = m @ o`` with
    bf16 operands and fp32 accumulation, inverse RoPE on ``y`` (fp32), per
    (head, 128-chunk) UE8M0 quant with amax floor 1e-10
    (``E/nvidia/attention.py:166-285``).  Returns ``(fp8 bytes [G, T, HPG*D],
    exponents [T, H, D // 128])``."""
    t, h, d = o.shape
    y = np.einsum("hg,tgd->thd", np.asarray(mix_bf16, np.float64),
                  np.asarray(o, np.float64)).astype(np.float32)
    return inv_rope_fp8_quant(y, positions, cos_sin, n_groups, rope_dim, quant=True)


def pack_scale_exponents(exp: np.ndarray) -> np.ndarray:
    """Pack per-128 exponents ``[T, H, C]`` as ``[T, H]`` int32 with byte
    ``c`` = ``exp + 127`` (``E/nvidia/attention.py:226-228``); unused
    bytes are zero."""
    t, h, c = exp.shape
    out = np.zeros((t, h), dtype=np.int64)
    for i in range(c):
        out |= (np.clip(exp[..., i] + 127, 0, 255).astype(np.int64) << (8 * i))
    return out.astype(np.uint32).view(np.int32)


def sigmoid_mul_quant_fp8(x: np.ndarray, gate: np.ndarray):
    """``x * sigmoid(gate)`` with the bf16 roundings of the unfused torch
    expression, then 1x128 UE8M0 FP8 with packed int32 exponents
    (``E/nvidia/attention.py:288-361``).  ``x``, ``gate`` hold bf16 values.
    Returns ``(fp8 bytes [rows, hidden], packed int32 [rows, hidden // 512])``.
    """
    import torch

    xt = torch.from_numpy(np.asarray(x, np.float32)).to(torch.bfloat16)
    gt = torch.from_numpy(np.asarray(gate, np.float32)).to(torch.bfloat16)
    s = torch.sigmoid(gt.float()).to(torch.bfloat16).float()
    y = (xt.float() * s).to(torch.bfloat16).float().numpy()
    rows, hidden = y.shape
    yb = y.reshape(rows, hidden // 128, 128)
    exp = ue8m0_exponent(np.abs(yb).max(-1), 1e-10, divide=False)
    q = e4m3_bytes(yb * np.ldexp(np.float32(1.0), -exp)[..., None]).reshape(rows, hidden)
    e4 = (exp + 127).astype(np.int64).reshape(rows, hidden // 512, 4)
    packed = (e4 << (np.arange(4) * 8)).sum(-1).astype(np.uint32).view(np.int32)
    return q, packed
