"""Seeded synthetic HCA workloads on the GPU (the BASELINE configs' shapes).

Builds, per layer, the three paged caches the HCA path reads -- the fp8 SWA
cache (64-token pages), the fp8 compressed cache (2 entries per page) and the
fp32 compressor state cache (8-token pages) -- filled with N(0, 1) rows
quantised through the library's own insert kernel, plus block tables whose
pages are a random permutation (so reads are scattered like a real paged
pool).  No public dataset is involved: the configs are synthetic by
definition.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch

from . import ops
from .cache_layout import STATE_BLOCK_SIZE, SWA_BLOCK_SIZE, page_bytes


@dataclass
class HCADims:
    heads: int = 64
    head_dim: int = 128
    rope_dim: int = 64
    window: int = 128
    ratio: int = 128
    comp_page: int = 2
    swa_page: int = SWA_BLOCK_SIZE
    state_page: int = STATE_BLOCK_SIZE
    n_groups: int = 8
    eps: float = 1e-6
    rope_theta: float = 160000.0

    @property
    def nope(self) -> int:
        return self.head_dim - self.rope_dim


def rope_cos_sin_cache(max_pos: int, rope_dim: int, theta: float, device) -> torch.Tensor:
    """fp32 ``[max_pos, R]`` = ``cos | sin`` of ``p * theta^(-2i/R)``
    (``V/model_executor/layers/rotary_embedding/base.py:69-92``)."""
    inv = 1.0 / (theta ** (torch.arange(0, rope_dim, 2, dtype=torch.float, device=device) / rope_dim))
    t = torch.arange(max_pos, dtype=torch.float, device=device)
    f = torch.outer(t, inv)
    return torch.cat([f.cos(), f.sin()], -1).contiguous()


@dataclass
class LayerCaches:
    swa: torch.Tensor
    comp: torch.Tensor
    state: torch.Tensor


@dataclass
class DecodeBatch:
    """One decode step: ``q_per_seq`` query tokens per request appended at
    positions ``ctx_b .. ctx_b + q_per_seq - 1``."""

    dims: HCADims
    ctx: torch.Tensor            # [B] int64 cpu: tokens already cached
    q_per_seq: int
    device: torch.device
    query_start_loc: torch.Tensor = field(init=False)
    seq_lens: torch.Tensor = field(init=False)
    positions: torch.Tensor = field(init=False)
    swa_bt: torch.Tensor = field(init=False)
    comp_bt: torch.Tensor = field(init=False)
    state_bt: torch.Tensor = field(init=False)
    n_swa_pages: int = field(init=False)
    n_comp_pages: int = field(init=False)
    n_state_pages: int = field(init=False)

    @property
    def num_reqs(self) -> int:
        return int(self.ctx.numel())

    @property
    def num_tokens(self) -> int:
        return self.num_reqs * self.q_per_seq


def _block_table(need_lo: torch.Tensor, need_hi: torch.Tensor, page: int, width: int,
                 gen: torch.Generator) -> tuple[torch.Tensor, int]:
    """Pages for positions ``[lo, hi)`` of each request, physically shuffled;
    entries outside the live range are 0 (vLLM clamps them to 0)."""
    b = need_lo.numel()
    lo_p = (need_lo // page).tolist()
    hi_p = ((need_hi + page - 1) // page).tolist()
    total = sum(h - l for l, h in zip(lo_p, hi_p))
    perm = torch.randperm(max(total, 1), generator=gen).to(torch.int32)
    bt = torch.zeros((b, width), dtype=torch.int32)
    k = 0
    for r in range(b):
        n = hi_p[r] - lo_p[r]
        bt[r, lo_p[r]:hi_p[r]] = perm[k:k + n]
        k += n
    return bt, max(total, 1)


def make_decode_batch(ctx: list[int] | torch.Tensor, q_per_seq: int, dims: HCADims, device,
                      seed: int = 0, max_model_len: int | None = None) -> DecodeBatch:
    ctx = torch.as_tensor(ctx, dtype=torch.int64)
    b = DecodeBatch(dims, ctx, q_per_seq, torch.device(device))
    gen = torch.Generator().manual_seed(seed)
    end = ctx + q_per_seq  # seq_lens after the step
    max_len = int(end.max()) if max_model_len is None else max_model_len
    d = dims
    # SWA: window of the first query token .. last token
    swa_lo = torch.clamp(ctx - d.window + 1, min=0)
    b.swa_bt, b.n_swa_pages = _block_table(swa_lo, end, d.swa_page, (max_len + d.swa_page - 1) // d.swa_page, gen)
    # compressed entries 0 .. end // ratio (incl. ones this step completes)
    n_ent = end // d.ratio + 1
    b.comp_bt, b.n_comp_pages = _block_table(torch.zeros_like(n_ent), n_ent, d.comp_page,
                                             max_len // d.ratio // d.comp_page + 2, gen)
    # compressor state: the last `ratio` positions before each boundary
    st_lo = torch.clamp(ctx - d.ratio, min=0)
    b.state_bt, b.n_state_pages = _block_table(st_lo, end, d.state_page,
                                               (max_len + d.state_page - 1) // d.state_page, gen)
    qsl = torch.arange(0, b.num_reqs + 1, dtype=torch.int32) * q_per_seq
    b.query_start_loc = qsl.to(device)
    b.seq_lens = end.to(torch.int32).to(device)
    b.positions = (ctx[:, None] + torch.arange(q_per_seq)[None, :]).reshape(-1).to(device)
    b.swa_bt = b.swa_bt.to(device)
    b.comp_bt = b.comp_bt.to(device)
    b.state_bt = b.state_bt.to(device)
    return b


def alloc_layer_caches(batch: DecodeBatch, seed: int, fill: bool = True) -> LayerCaches:
    """Caches of one layer, filled with quantised N(0, 1) rows (and N(0, 1)
    fp32 compressor states) through the library's insert kernel."""
    d = batch.dims
    dev = batch.device
    g = torch.Generator(device=dev).manual_seed(seed)
    swa = torch.zeros((batch.n_swa_pages, page_bytes(d.swa_page, d.head_dim, d.rope_dim)), dtype=torch.uint8, device=dev)
    comp = torch.zeros((batch.n_comp_pages, page_bytes(d.comp_page, d.head_dim, d.rope_dim)), dtype=torch.uint8, device=dev)
    state = torch.randn((batch.n_state_pages, d.state_page, 2 * d.head_dim), generator=g, device=dev)
    if fill:
        for cache, page, n in ((swa, d.swa_page, batch.n_swa_pages), (comp, d.comp_page, batch.n_comp_pages)):
            slots = torch.arange(n * page, dtype=torch.int64, device=dev)
            rows = torch.randn((slots.numel(), d.head_dim), generator=g, device=dev).to(torch.bfloat16)
            ops.quantize_and_insert_k_cache(rows, cache, slots, block_size=page, rope_dim=d.rope_dim)
    return LayerCaches(swa, comp, state)
