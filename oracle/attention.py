"""Sparse HCA attention with an attention sink (CPU oracle, fp32/fp64).

Semantics of FlashMLA's sparse decode/prefill as the reference calls them
(``V/models/deepseek_v4/nvidia/flashmla.py:286-302,416-424``) and as the
interface documents them
(``V/third_party/flashmla/flash_mla_interface.py:54-92,180-215``):

* each query token attends the leftmost ``topk_length`` entries of its
  window index row (SWA cache) and the leftmost ``extra_topk_length``
  entries of its compressed index row (compressed cache); negative indices
  are skipped;
* ``s_j = scale * q . k_j``; ``o = sum_j softmax(s)_j v_j`` with ``V = K``
  (the full dequantised row);
* the sink multiplies the output by ``exp(lse) / (exp(lse) + exp(sink_h))``;
  a token with no rows outputs zeros.

The closed FlashMLA binary is not run.  The restatement is pinned against
vLLM's readable DeepSeek-V4 sparse attention kernels for the same op, cache
layout and sink (``_sparse_attn_decode_ragged_kernel`` /
``_sparse_attn_prefill_ragged_kernel`` in
``vllm/v1/attention/ops/rocm_aiter_mla_sparse.py``, driven as in
``vllm/models/deepseek_v4/amd/rocm.py``): ``tests/golden/make_golden.py``
runs them under the Triton interpreter at D=512 and
``tests/test_oracle_golden.py`` checks this module against their outputs.
"""

from __future__ import annotations

import numpy as np

from .cache import read_rows


def sparse_attention_token(
    q: np.ndarray,
    k: np.ndarray,
    scale: float,
    sink: np.ndarray | None,
) -> np.ndarray:
    """One token: ``q [H, D]`` against rows ``k [n, D]`` (fp64 math)."""
    h, d = q.shape
    if k.shape[0] == 0:
        return np.zeros((h, d), dtype=np.float32)
    qd = q.astype(np.float64)
    kd = k.astype(np.float64)
    s = (qd @ kd.T) * scale  # [H, n]
    m = s.max(axis=1, keepdims=True)
    p = np.exp(s - m)
    l = p.sum(axis=1, keepdims=True)
    o = (p @ kd) / l
    if sink is not None:
        lse = (np.log(l) + m)[:, 0]
        sk = np.asarray(sink, dtype=np.float64)[:h]
        # exp(lse) / (exp(lse) + exp(sink)) = 1 / (1 + exp(sink - lse))
        with np.errstate(over="ignore"):
            f = 1.0 / (1.0 + np.exp(sk - lse))
        o = o * f[:, None]
    return o.astype(np.float32)


def sparse_decode(
    q: np.ndarray,
    swa_cache: np.ndarray,
    swa_page: int,
    swa_indices: np.ndarray,
    swa_lens: np.ndarray,
    comp_cache: np.ndarray | None,
    comp_page: int,
    comp_indices: np.ndarray | None,
    comp_lens: np.ndarray | None,
    scale: float,
    sink: np.ndarray | None,
    head_dim: int,
    rope_dim: int,
) -> np.ndarray:
    """``flash_mla_with_kvcache`` with ``indices``/``extra_indices`` over
    the two fp8 caches; ``q [T, H, D]`` (bf16 values) -> ``[T, H, D]`` fp32."""
    t_n, h, d = q.shape
    out = np.zeros((t_n, h, d), dtype=np.float32)
    for t in range(t_n):
        rows = []
        idx = np.asarray(swa_indices[t, : int(swa_lens[t])])
        idx = idx[idx >= 0]
        if idx.size:
            rows.append(read_rows(swa_cache, idx, swa_page, head_dim, rope_dim))
        if comp_cache is not None and comp_lens is not None:
            cidx = np.asarray(comp_indices[t, : int(comp_lens[t])])
            cidx = cidx[cidx >= 0]
            if cidx.size:
                rows.append(read_rows(comp_cache, cidx, comp_page, head_dim, rope_dim))
        k = np.concatenate(rows, 0) if rows else np.zeros((0, d), np.float32)
        out[t] = sparse_attention_token(q[t], k, scale, sink)
    return out


def sparse_prefill_workspace(
    q: np.ndarray,
    kv: np.ndarray,
    indices: np.ndarray,
    lens: np.ndarray,
    scale: float,
    sink: np.ndarray | None,
) -> np.ndarray:
    """``flash_mla_sparse_fwd`` over a gathered bf16 workspace
    ``kv [s_kv, D]`` with per-token ``indices [T, topk]`` (``-1`` or out of
    range skipped) and ``topk_length``
    (``V/third_party/flashmla/flash_mla_interface.py:180-215``)."""
    t_n, h, d = q.shape
    out = np.zeros((t_n, h, d), dtype=np.float32)
    for t in range(t_n):
        idx = np.asarray(indices[t, : int(lens[t])])
        idx = idx[(idx >= 0) & (idx < kv.shape[0])]
        out[t] = sparse_attention_token(q[t], kv[idx], scale, sink)
    return out


def sparse_prefill_paged(
    q: np.ndarray,
    positions: np.ndarray,
    token_to_req: np.ndarray,
    swa_cache: np.ndarray,
    swa_page: int,
    swa_bt: np.ndarray,
    comp_cache: np.ndarray | None,
    comp_page: int,
    comp_bt: np.ndarray | None,
    window: int,
    ratio: int,
    scale: float,
    sink: np.ndarray | None,
    head_dim: int,
    rope_dim: int,
) -> np.ndarray:
    """Prefill semantics of ``_forward_prefill``
    (``V/models/deepseek_v4/nvidia/flashmla.py:304-424``) evaluated straight on
    the paged caches: token at position ``p`` of request ``r`` attends
    compressed entries ``0 .. (p + 1) // ratio - 1`` and window positions
    ``max(p - W + 1, 0) .. p`` (``cache_utils.py:567-594``)."""
    t_n, h, d = q.shape
    out = np.zeros((t_n, h, d), dtype=np.float32)
    for t in range(t_n):
        p, r = int(positions[t]), int(token_to_req[t])
        wpos = np.arange(max(p - window + 1, 0), p + 1)
        wsl = swa_bt[r, wpos // swa_page].astype(np.int64) * swa_page + wpos % swa_page
        rows = [read_rows(swa_cache, wsl, swa_page, head_dim, rope_dim)]
        nc = (p + 1) // ratio if comp_cache is not None else 0
        if nc:
            ci = np.arange(nc)
            csl = comp_bt[r, ci // comp_page].astype(np.int64) * comp_page + ci % comp_page
            rows.append(read_rows(comp_cache, csl, comp_page, head_dim, rope_dim))
        out[t] = sparse_attention_token(q[t], np.concatenate(rows), scale, sink)
    return out


def hca_rows_for_position(p: int, window: int = 128, ratio: int = 128) -> tuple[int, int]:
    """``(compressed_entries, window_rows)`` a query at position ``p`` attends."""
    return (p + 1) // ratio, min(p + 1, window)
