"""Integer metadata builders of the HCA path (CPU oracle, bit-exact target).

Each function restates one reference Triton kernel; inputs and outputs are
numpy integer arrays with the reference's dtypes.
"""

from __future__ import annotations

import numpy as np


def token_to_req_indices(query_start_loc: np.ndarray) -> np.ndarray:
    """``repeat_interleave(arange(num_reqs), query_lens)`` as int32
    (``V/v1/attention/backends/mla/sparse_swa.py:286-294``,
    ``V/models/deepseek_v4/compressor.py:107-112``)."""
    qsl = np.asarray(query_start_loc, dtype=np.int64)
    lens = qsl[1:] - qsl[:-1]
    return np.repeat(np.arange(len(lens), dtype=np.int32), lens)


def slot_mapping(
    query_start_loc: np.ndarray,
    seq_lens: np.ndarray,
    block_table: np.ndarray,
    block_size: int,
) -> np.ndarray:
    """Plain per-token slot ``bt[p // bs] * bs + p % bs`` (int64): the vLLM
    model runner's slot mapping for the SWA cache (64-token pages) and the
    compressor state cache (8-token pages)."""
    qsl = np.asarray(query_start_loc, dtype=np.int64)
    out = np.full(int(qsl[-1]), -1, dtype=np.int64)
    for b in range(len(qsl) - 1):
        ql = qsl[b + 1] - qsl[b]
        start = int(seq_lens[b]) - ql
        for i in range(ql):
            p = start + i
            out[qsl[b] + i] = int(block_table[b, p // block_size]) * block_size + p % block_size
    return out


def compressed_slot_mapping(
    num_tokens: int,
    query_start_loc: np.ndarray,
    seq_lens: np.ndarray,
    block_table: np.ndarray,
    block_size: int,
    compress_ratio: int,
) -> np.ndarray:
    """Slot of the compressed entry a token completes, else -1 (int64).

    Restates ``_compressed_slot_mapping_kernel`` /
    ``get_compressed_slot_mapping``
    (``V/v1/attention/backends/mla/compressor_utils.py:8-86``):
    ``slot = bt[(p // C) // bs] * bs + (p // C) % bs`` when
    ``(p + 1) % C == 0``.
    """
    out = np.full(num_tokens, -1, dtype=np.int64)
    qsl = np.asarray(query_start_loc, dtype=np.int64)
    for b in range(block_table.shape[0]):
        qs, qe = int(qsl[b]), int(qsl[b + 1])
        start = int(seq_lens[b]) - (qe - qs)
        for i in range(qe - qs):
            p = start + i
            if (p + 1) % compress_ratio != 0:
                continue
            c = p // compress_ratio
            out[qs + i] = int(block_table[b, c // block_size]) * block_size + c % block_size
    return out


def swa_indices_and_lens(
    num_decode_tokens: int,
    window_size: int,
    query_start_loc: np.ndarray,
    seq_lens: np.ndarray,
    token_to_req: np.ndarray,
    is_valid_token: np.ndarray,
    block_table: np.ndarray,
    block_size: int,
    out_indices: np.ndarray,
    out_lens: np.ndarray,
) -> None:
    """Window slots of each decode token, ``[max(p - W + 1, 0), p]``, and
    the window length; invalid tokens get length 0 and keep their row.

    Restates ``_compute_swa_indices_and_lens_kernel``
    (``V/v1/attention/backends/mla/sparse_swa.py:449-503``).
    ``out_indices`` is ``[max_tokens, W]`` int32 (the builder's persistent
    buffer) and ``out_lens`` ``[max_tokens]`` int32; lens past
    ``num_decode_tokens`` are zeroed (``sparse_swa.py:296``).
    """
    out_lens[num_decode_tokens:] = 0
    for t in range(num_decode_tokens):
        if not is_valid_token[t]:
            out_lens[t] = 0
            continue
        r = int(token_to_req[t])
        qs, qe = int(query_start_loc[r]), int(query_start_loc[r + 1])
        pos = int(seq_lens[r]) - (qe - qs) + t - qs
        start = max(pos - window_size + 1, 0)
        n = pos + 1 - start
        out_lens[t] = n
        for i in range(window_size):
            if i < n:
                p = start + i
                out_indices[t, i] = int(block_table[r, p // block_size]) * block_size + p % block_size
            else:
                out_indices[t, i] = -1


def c128a_topk_metadata(
    positions: np.ndarray,
    compress_ratio: int,
    num_decode_tokens: int,
    token_to_req: np.ndarray,
    block_table: np.ndarray,
    block_size: int,
    slot_mapping_: np.ndarray,
    global_decode: np.ndarray,
    decode_lens: np.ndarray,
    prefill_local: np.ndarray,
    max_compressed_tokens: int,
) -> None:
    """Compressed-entry indices for every token.

    Decode tokens: global slots of entries ``0 .. n - 1`` with
    ``n = min((p + 1) // C, max)`` (block-table lookup), ``-1`` beyond, and
    ``decode_lens = n`` (0 for invalid tokens).  Prefill tokens: local
    indices ``0 .. n - 1`` then ``-1``.

    Restates ``_build_c128a_topk_metadata_kernel``
    (``V/v1/attention/backends/mla/flashmla_sparse.py:1083-1149``).
    """
    w = max_compressed_tokens
    for t in range(len(positions)):
        p = int(positions[t])
        n = min((p + 1) // compress_ratio, w)
        ar = np.arange(w)
        if t < num_decode_tokens:
            valid_tok = int(slot_mapping_[t]) >= 0
            r = int(token_to_req[t])
            row = np.full(w, -1, dtype=np.int64)
            idx = ar[:n]
            row[:n] = block_table[r, idx // block_size].astype(np.int64) * block_size + idx % block_size
            global_decode[t, :w] = row.astype(np.int32)
            decode_lens[t] = n if valid_tok else 0
        else:
            prefill_local[t - num_decode_tokens, :w] = np.where(ar < n, ar, -1).astype(np.int32)


def prefill_gather_lens(
    seq_lens: np.ndarray,
    query_start_loc: np.ndarray,
    num_prefills: int,
    num_decodes: int,
    window_size: int,
) -> np.ndarray:
    """``gather_len = query_len + min(prefix_len, W - 1)`` per prefill
    request (``V/v1/attention/backends/mla/sparse_swa.py:422-446``)."""
    out = np.zeros(num_prefills, dtype=np.int32)
    for i in range(num_prefills):
        r = num_decodes + i
        ql = int(query_start_loc[r + 1]) - int(query_start_loc[r])
        prefix = int(seq_lens[r]) - ql
        out[i] = ql + min(prefix, window_size - 1)
    return out


def combine_topk_swa_indices(
    topk_indices: np.ndarray,
    query_start_loc: np.ndarray,
    seq_lens: np.ndarray,
    gather_lens: np.ndarray,
    window_size: int,
    compress_ratio: int,
    topk: int,
    M: int,
    N: int,
) -> tuple[np.ndarray, np.ndarray]:
    """``[compressed || window]`` indices into the per-chunk gathered
    workspace, width padded to a multiple of 128, ``-1`` filled.

    Restates ``combine_topk_swa_indices``
    (``V/models/deepseek_v4/common/ops/cache_utils.py:476-594``).
    """
    num_tokens = topk_indices.shape[0]
    width = (topk + window_size + 127) // 128 * 128
    comb = np.full((num_tokens, width), -1, dtype=np.int32)
    lens = np.zeros(num_tokens, dtype=np.int32)
    base = int(query_start_loc[0])
    for b in range(len(seq_lens)):
        qs = int(query_start_loc[b]) - base
        qe = int(query_start_loc[b + 1]) - base
        ql = qe - qs
        sl = int(seq_lens[b])
        gstart = sl - int(gather_lens[b])
        start_pos = sl - ql
        for t in range(qs, qe):
            pos = start_pos + (t - qs)
            tk = min((pos + 1) // compress_ratio, topk)
            sw = min(pos + 1, window_size)
            comb[t, :tk] = topk_indices[t, :tk] + M * b
            comb[t, tk : tk + sw] = M * b + N + np.arange(sw) + pos - sw + 1 - gstart
            lens[t] = tk + sw
    return comb, lens
