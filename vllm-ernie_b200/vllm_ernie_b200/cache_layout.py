"""Byte layout of the paged fp8 HCA caches (host-side helpers).

One cached row ("fp8_ds_mla", generalised to ``D = N + R``): ``N`` e4m3
bytes then ``R`` bf16 values; a page of ``P`` rows stores the ``P`` data rows
first, then ``P`` scale rows of ``N / 64`` UE8M0 bytes plus one zero pad
byte (``V/models/deepseek_v4/common/ops/cache_utils.py:42-51``,
``V/models/deepseek_v4/nvidia/flashmla.py:98-111``).  At ``D = 512`` a row is
the reference's 584 bytes.
"""

from __future__ import annotations

QUANT_BLOCK = 64
SWA_BLOCK_SIZE = 64          # V/v1/attention/backends/mla/sparse_swa.py:70-75
KV_MANAGER_BLOCK = 256       # V/models/deepseek_v4/nvidia/flashmla.py:78-80
STATE_BLOCK_SIZE = 8         # V/models/deepseek_v4/compressor.py:146-155 (ratio 128)
FLASHMLA_ALIGNMENT = 576     # page alignment of every cache spec (compressor.py:163)


def row_geometry(head_dim: int, rope_dim: int) -> tuple[int, int, int]:
    """``(nope, data_bytes, scale_bytes)`` of one row."""
    nope = head_dim - rope_dim
    if nope <= 0 or nope % QUANT_BLOCK or rope_dim % 2:
        raise ValueError(f"unsupported HCA row geometry D={head_dim} R={rope_dim}")
    return nope, nope + 2 * rope_dim, nope // QUANT_BLOCK + 1


def row_bytes(head_dim: int, rope_dim: int) -> int:
    """Bytes per cached token (584 at D=512)."""
    _, data, scale = row_geometry(head_dim, rope_dim)
    return data + scale


def page_bytes(page_size: int, head_dim: int, rope_dim: int, align: int = 16) -> int:
    """Bytes of one page, rounded up to ``align`` (16 keeps vector loads aligned)."""
    b = page_size * row_bytes(head_dim, rope_dim)
    return (b + align - 1) // align * align


def compressed_page_size(compress_ratio: int, manager_block: int = KV_MANAGER_BLOCK) -> int:
    """Compressed entries per page: ``256 // 128 = 2``
    (``V/models/deepseek_v4/nvidia/flashmla.py:229``)."""
    return max(1, manager_block // compress_ratio)
