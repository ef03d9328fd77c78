"""FP8 e4m3 / UE8M0 emulation on the CPU (test infrastructure only).

The reference quantises with a power-of-two ("UE8M0") scale per block:
``scale = 2 ** ceil(log2(max(amax, floor) / 448))``, stores
``clamp(x / scale, -448, 448)`` as float8_e4m3fn (round to nearest even) and
the scale as the byte ``exponent + 127``
(``V/models/deepseek_v4/common/ops/cache_utils.py:88-118``,
``V/models/deepseek_v4/common/ops/fused_compress_quant_cache.py:235-257``).

The kernels differ in how they form ``amax / 448``: the KV insert divides
(``cache_utils.py:98``), every other kernel multiplies by the fp32 constant
``1/448`` (``fused_compress_quant_cache.py:247``,
``fused_inv_rope_fp8_quant.py:105``, ``E/nvidia/attention.py:223,318``).
The two differ by one ulp when ``amax`` is 448 times a power of two, so
both are modelled.  ``ceil(log2(.))`` is evaluated exactly.
"""

from __future__ import annotations

import numpy as np
import torch

FP8_MAX = 448.0
INV_FP8_MAX_F32 = np.float32(1.0) / np.float32(448.0)


def ceil_log2_exact(x: np.ndarray) -> np.ndarray:
    """``ceil(log2(x))`` for positive finite fp32 ``x``, exactly."""
    x = np.asarray(x, dtype=np.float32)
    m, e = np.frexp(x)  # x = m * 2**e, m in [0.5, 1)
    return np.where(m == 0.5, e - 1, e).astype(np.int32)


def ue8m0_exponent(amax: np.ndarray, floor: float, divide: bool) -> np.ndarray:
    """Exponent of the UE8M0 scale for a block with abs-max ``amax``."""
    a = np.maximum(np.asarray(amax, dtype=np.float32), np.float32(floor))
    if divide:
        raw = (a / np.float32(FP8_MAX)).astype(np.float32)
    else:
        raw = (a * INV_FP8_MAX_F32).astype(np.float32)
    return ceil_log2_exact(raw)


def encode_ue8m0(exponent: np.ndarray) -> np.ndarray:
    """Scale byte ``clamp(exponent + 127, 0, 255)``."""
    return np.clip(np.asarray(exponent) + 127, 0, 255).astype(np.uint8)


def e4m3_bytes(x_scaled: np.ndarray) -> np.ndarray:
    """Clamp to +-448 and round to float8_e4m3fn (nearest even); raw bytes."""
    t = torch.from_numpy(np.clip(np.asarray(x_scaled, dtype=np.float32), -FP8_MAX, FP8_MAX))
    return t.to(torch.float8_e4m3fn).view(torch.uint8).numpy()


def e4m3_to_f32(b: np.ndarray) -> np.ndarray:
    """Raw float8_e4m3fn bytes to fp32."""
    t = torch.from_numpy(np.ascontiguousarray(b, dtype=np.uint8))
    return t.view(torch.float8_e4m3fn).to(torch.float32).numpy()


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round fp32 to bf16 (nearest even) and back to fp32."""
    t = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32))
    return t.to(torch.bfloat16).to(torch.float32).numpy()


def bf16_bytes(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 raw little-endian bytes, shape ``[..., 2 * n]``."""
    t = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(torch.bfloat16)
    return t.view(torch.uint8).numpy().reshape(*x.shape[:-1], x.shape[-1] * 2)


def bf16_from_bytes(b: np.ndarray) -> np.ndarray:
    """bf16 raw bytes ``[..., 2 * n]`` to fp32 ``[..., n]``."""
    b = np.ascontiguousarray(b, dtype=np.uint8)
    if b.size == 0:
        return np.zeros(b.shape[:-1] + (b.shape[-1] // 2,), np.float32)
    return torch.from_numpy(b).view(torch.bfloat16).to(torch.float32).numpy()


def quantize_blocks(x: np.ndarray, block: int, floor: float, divide: bool):
    """UE8M0 block quantisation of the last axis.

    Returns ``(fp8_bytes, exponents)`` with exponents shaped
    ``[..., x.shape[-1] // block]``.
    """
    x = np.asarray(x, dtype=np.float32)
    n = x.shape[-1]
    assert n % block == 0
    xb = x.reshape(*x.shape[:-1], n // block, block)
    exp = ue8m0_exponent(np.abs(xb).max(axis=-1), floor, divide)
    inv = np.ldexp(np.float32(1.0), -exp).astype(np.float32)
    q = e4m3_bytes(xb * inv[..., None])
    return q.reshape(x.shape), exp
