"""Attention-backend side of the HCA path: KV-cache specs and per-step
metadata builders, mirroring what the vLLM 0.32 scheduler calls.

* ``get_kv_cache_spec`` of the three cache layers an HCA layer owns -- the
  compressed cache (``V/models/deepseek_v4/attention.py:704-718``), the SWA
  cache (``V/v1/attention/backends/mla/sparse_swa.py:78-88``) and the
  compressor state (``V/models/deepseek_v4/compressor.py:157-165``);
* ``*MetadataBuilder.build(common_prefix_len, common_attn_metadata)`` of the
  SWA, C128A and compressor groups, whose integer tables are produced on the
  device by the library's builders (bit-exact with the reference's).

The builders keep persistent buffers (fixed addresses for CUDA graphs) like
the reference's.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

from . import ops
from .cache_layout import (
    FLASHMLA_ALIGNMENT,
    KV_MANAGER_BLOCK,
    STATE_BLOCK_SIZE,
    SWA_BLOCK_SIZE,
    row_bytes,
)

C128A_TOPK_ALIGNMENT = 128  # V/v1/attention/backends/mla/flashmla_sparse.py:351-359


# ---------------------------------------------------------------------------
# KV cache specs
# ---------------------------------------------------------------------------


@dataclass(frozen=True)
class HCACacheSpec:
    """Fields of vLLM's ``MLAAttentionSpec`` / ``SlidingWindowMLASpec`` that
    the HCA caches set."""

    kind: str                 # "compressed" | "swa" | "compressor_state"
    block_size: int           # tokens per manager block (scheduler view)
    head_size: int            # bytes (uint8 caches) or fp32 elements per token
    dtype: torch.dtype
    num_kv_heads: int = 1
    compress_ratio: int = 1
    sliding_window: int | None = None
    cache_dtype_str: str = "fp8_ds_mla"
    alignment: int = FLASHMLA_ALIGNMENT

    @property
    def storage_block_size(self) -> int:
        """Rows per physical page (compressed: 256 // 128 = 2)."""
        return self.block_size // self.compress_ratio if self.kind == "compressed" else self.block_size

    @property
    def page_size_bytes(self) -> int:
        elem = torch.tensor([], dtype=self.dtype).element_size()
        raw = self.storage_block_size * self.head_size * elem
        return math.ceil(raw / self.alignment) * self.alignment


def hca_kv_cache_specs(head_dim: int, rope_dim: int, window: int = 128, compress_ratio: int = 128,
                       block_size: int = KV_MANAGER_BLOCK) -> dict[str, HCACacheSpec]:
    rb = row_bytes(head_dim, rope_dim)
    return {
        "compressed": HCACacheSpec("compressed", block_size, rb, torch.uint8, compress_ratio=compress_ratio),
        "swa": HCACacheSpec("swa", SWA_BLOCK_SIZE, rb, torch.uint8, sliding_window=window),
        "compressor_state": HCACacheSpec("compressor_state", STATE_BLOCK_SIZE, 2 * head_dim, torch.float32,
                                         sliding_window=compress_ratio, cache_dtype_str="auto"),
    }


def get_kv_cache_shape(num_blocks: int, block_size: int, num_kv_heads: int, head_size: int,
                       cache_dtype_str: str = "fp8_ds_mla") -> tuple[int, ...]:
    """``(blocks, block_size, row_bytes)`` (584 at D=512)
    (``V/models/deepseek_v4/nvidia/flashmla.py:98-111``)."""
    assert num_kv_heads == 1
    if cache_dtype_str == "fp8_ds_mla":
        return (num_blocks, block_size, row_bytes(head_size, 64))
    return (num_blocks, block_size, head_size)


def packed_block_stride_alignment(vllm_config) -> int:
    """Byte alignment shared by the pages of every layer in the hybrid KV
    group (HCA, DSA and indexer), read from
    ``vllm_config.model_config.hf_config`` (``E/nvidia/attention.py:561-571``)."""
    cfg = vllm_config.model_config.hf_config
    return math.lcm(512, cfg.head_dim * 2, (cfg.mla_kv_lora_rank + cfg.mla_qk_rope_head_dim) * 2)


# ---------------------------------------------------------------------------
# common metadata + split
# ---------------------------------------------------------------------------


@dataclass
class CommonAttentionMetadata:
    """The fields of vLLM's ``CommonAttentionMetadata`` the builders read."""

    query_start_loc: torch.Tensor        # [R + 1] int32, device
    query_start_loc_cpu: torch.Tensor    # [R + 1] int32, host
    seq_lens: torch.Tensor               # [R] int32, device
    num_reqs: int
    num_actual_tokens: int
    max_query_len: int
    block_table_tensor: torch.Tensor     # [R, pages] int32 of this cache group
    slot_mapping: torch.Tensor           # [T] int64 of this cache group
    positions: torch.Tensor | None = None  # [T] int64
    max_seq_len: int = 0


def split_decodes_and_prefills(cm: CommonAttentionMetadata, decode_threshold: int = 1):
    """``(num_decodes, num_prefills, num_decode_tokens, num_prefill_tokens)``
    for a batch reordered decodes-first
    (``vllm/v1/attention/backends/utils.py`` split_decodes_and_prefills)."""
    qsl = cm.query_start_loc_cpu.tolist()
    lens = [qsl[i + 1] - qsl[i] for i in range(cm.num_reqs)]
    nd = 0
    while nd < cm.num_reqs and lens[nd] <= decode_threshold:
        nd += 1
    ndt = qsl[nd]
    return nd, cm.num_reqs - nd, ndt, cm.num_actual_tokens - ndt


# ---------------------------------------------------------------------------
# metadata objects
# ---------------------------------------------------------------------------


@dataclass
class SWAMetadata:
    """``DeepseekSparseSWAMetadata`` (``V/v1/attention/backends/mla/sparse_swa.py:151-190``)
    plus the decode grouping our attention kernel uses."""

    block_table: torch.Tensor
    slot_mapping: torch.Tensor
    block_size: int
    seq_lens: torch.Tensor
    query_start_loc: torch.Tensor
    query_start_loc_cpu: torch.Tensor
    is_valid_token: torch.Tensor
    token_to_req_indices: torch.Tensor
    decode_swa_indices: torch.Tensor
    decode_swa_lens: torch.Tensor
    num_decodes: int = 0
    num_prefills: int = 0
    num_decode_tokens: int = 0
    num_prefill_tokens: int = 0
    prefill_seq_lens: torch.Tensor | None = None
    prefill_gather_lens: torch.Tensor | None = None
    decode_group_starts: torch.Tensor | None = None
    decode_max_group_tokens: int = 1


@dataclass
class C128AMetadata:
    """The C128A fields of ``FlashMLASparseMetadata``
    (``V/v1/attention/backends/mla/flashmla_sparse.py:565-687``)."""

    block_table: torch.Tensor
    slot_mapping: torch.Tensor          # compressed slot per token (-1 off-boundary)
    block_size: int                     # manager block (256)
    req_id_per_token: torch.Tensor
    c128a_global_decode_topk_indices: torch.Tensor | None = None
    c128a_decode_topk_lens: torch.Tensor | None = None
    c128a_prefill_topk_indices: torch.Tensor | None = None
    num_splits: int = 1
    # balanced decode work list of the step (built on first use, shared by
    # every layer): see ops.decode_schedule
    decode_schedule: torch.Tensor | None = None
    decode_items: int = 0


@dataclass
class CompressorMetadata:
    """``V/models/deepseek_v4/compressor.py:78-118``."""

    block_table: torch.Tensor
    slot_mapping: torch.Tensor
    block_size: int
    token_to_req_indices: torch.Tensor | None = None
    c128_boundary: bool | None = None


# ---------------------------------------------------------------------------
# builders
# ---------------------------------------------------------------------------


def decode_group_rows(head_dim: int) -> int:
    """Query rows (tokens x heads) one decode group may hold: two M=128 tiles
    of one CTA at head_dim 128, one tile of a CTA pair at head_dim 512."""
    return 256 if head_dim == 128 else 128


def _decode_groups(qsl_cpu: list[int], num_decodes: int, max_tokens: int, device) -> torch.Tensor:
    starts: list[int] = []
    for r in range(num_decodes):
        starts.extend(range(qsl_cpu[r], qsl_cpu[r + 1], max_tokens))
    starts.append(qsl_cpu[num_decodes])
    return torch.tensor(starts, dtype=torch.int32).to(device, non_blocking=True)


class SWAMetadataBuilder:
    """``DeepseekSparseSWAMetadataBuilder`` (``sparse_swa.py:193-446``)."""

    reorder_batch_threshold = 1

    def __init__(self, window_size: int, max_num_batched_tokens: int, num_heads: int,
                 num_speculative_tokens: int = 0, device="cuda", head_dim: int = 128):
        self.window_size = window_size
        self.head_dim = head_dim
        self.block_size = SWA_BLOCK_SIZE
        self.decode_threshold = self.reorder_batch_threshold + num_speculative_tokens
        self.num_heads = num_heads
        self.device = torch.device(device)
        self.token_to_req_indices = torch.zeros(max_num_batched_tokens, dtype=torch.int32, device=self.device)
        self.decode_swa_indices = torch.zeros((max_num_batched_tokens, 1, window_size), dtype=torch.int32,
                                              device=self.device)
        self.decode_swa_lens = torch.zeros(max_num_batched_tokens, dtype=torch.int32, device=self.device)
        self.is_valid_token = torch.zeros(max_num_batched_tokens, dtype=torch.bool, device=self.device)

    def build(self, common_prefix_len: int, cm: CommonAttentionMetadata, fast_build: bool = False) -> SWAMetadata:
        nd, npf, ndt, npt = split_decodes_and_prefills(cm, self.decode_threshold)
        n = cm.num_actual_tokens
        t2r = ops.token_to_req_indices(cm.query_start_loc, n, out=self.token_to_req_indices)
        is_valid = self.is_valid_token[: cm.slot_mapping.shape[0]]
        torch.ge(cm.slot_mapping, 0, out=is_valid)
        if ndt > 0:
            ops.compute_swa_indices_and_lens(self.decode_swa_indices, self.decode_swa_lens, ndt,
                                             self.window_size, cm.query_start_loc, cm.seq_lens, t2r, is_valid,
                                             cm.block_table_tensor, self.block_size)
        md = SWAMetadata(
            block_table=cm.block_table_tensor, slot_mapping=cm.slot_mapping, block_size=self.block_size,
            seq_lens=cm.seq_lens, query_start_loc=cm.query_start_loc,
            query_start_loc_cpu=cm.query_start_loc_cpu, is_valid_token=is_valid, token_to_req_indices=t2r,
            decode_swa_indices=self.decode_swa_indices[:ndt], decode_swa_lens=self.decode_swa_lens[:ndt],
            num_decodes=nd, num_prefills=npf, num_decode_tokens=ndt, num_prefill_tokens=npt)
        if npf > 0:
            md.prefill_seq_lens = cm.seq_lens[nd:]
            md.prefill_gather_lens = ops.compute_prefill_gather_lens(cm.seq_lens, cm.query_start_loc, npf, nd,
                                                                     self.window_size)
        if ndt > 0:
            max_g = max(1, decode_group_rows(self.head_dim) // self.num_heads)
            md.decode_max_group_tokens = min(max_g, self.decode_threshold)
            md.decode_group_starts = _decode_groups(cm.query_start_loc_cpu.tolist(), nd,
                                                    md.decode_max_group_tokens, self.device)
        return md


class C128AMetadataBuilder:
    """The C128A part of ``FlashMLASparseMetadataBuilder``
    (``flashmla_sparse.py:328-389,565-687``)."""

    def __init__(self, max_model_len: int, max_num_batched_tokens: int, compress_ratio: int = 128,
                 block_size: int = KV_MANAGER_BLOCK, num_speculative_tokens: int = 0, device="cuda",
                 sm_count: int | None = None):
        self.compress_ratio = compress_ratio
        self.block_size = block_size
        self.device = torch.device(device)
        self.decode_threshold = 1 + num_speculative_tokens
        maxc = math.ceil(max_model_len / compress_ratio)
        self.c128a_max_compressed = math.ceil(maxc / C128A_TOPK_ALIGNMENT) * C128A_TOPK_ALIGNMENT
        self.compressed_slot_mapping_buffer = torch.empty(max_num_batched_tokens, dtype=torch.int64, device=self.device)
        self.c128a_global_decode_buffer = torch.empty((max_num_batched_tokens, self.c128a_max_compressed),
                                                      dtype=torch.int32, device=self.device)
        self.c128a_decode_lens_buffer = torch.empty(max_num_batched_tokens, dtype=torch.int32, device=self.device)
        self.c128a_prefill_buffer = torch.empty((max_num_batched_tokens, self.c128a_max_compressed),
                                                dtype=torch.int32, device=self.device)
        self.sm_count = sm_count
        self.req_id_per_token_buffer = torch.zeros(max_num_batched_tokens, dtype=torch.int32, device=self.device)

    def build(self, common_prefix_len: int, cm: CommonAttentionMetadata, swa_slot_mapping: torch.Tensor,
              fast_build: bool = False) -> C128AMetadata:
        n = cm.num_actual_tokens
        storage = self.block_size // self.compress_ratio
        bt = cm.block_table_tensor.clamp(min=0)
        slot = ops.get_compressed_slot_mapping(n, cm.query_start_loc, cm.seq_lens, bt, storage,
                                               self.compress_ratio, out=self.compressed_slot_mapping_buffer)
        rid = ops.token_to_req_indices(cm.query_start_loc, n, out=self.req_id_per_token_buffer)
        md = C128AMetadata(block_table=cm.block_table_tensor, slot_mapping=slot, block_size=self.block_size,
                           req_id_per_token=rid)
        nd, _, ndt, npt = split_decodes_and_prefills(cm, self.decode_threshold)
        if n:
            assert cm.positions is not None, "positions is required for C128A metadata build"
            gd, dl, pl = ops.build_c128a_topk_metadata(
                cm.positions[:n], self.compress_ratio, ndt, rid, cm.block_table_tensor, storage,
                swa_slot_mapping, self.c128a_global_decode_buffer, self.c128a_decode_lens_buffer,
                self.c128a_prefill_buffer, self.c128a_max_compressed)
            if ndt:
                md.c128a_global_decode_topk_indices = gd.view(ndt, 1, -1)
                md.c128a_decode_topk_lens = dl
                from .decode import choose_num_splits

                md.num_splits = choose_num_splits(nd, self.sm_count or _sm_count(self.device))
            if npt:
                md.c128a_prefill_topk_indices = pl
        return md


class CompressorMetadataBuilder:
    """``V/models/deepseek_v4/compressor.py:90-118``."""

    def __init__(self, max_num_batched_tokens: int, block_size: int = STATE_BLOCK_SIZE, device="cuda"):
        self.block_size = block_size
        self.device = torch.device(device)
        self.token_to_req_indices = torch.zeros(max_num_batched_tokens, dtype=torch.int32, device=self.device)

    def build(self, common_prefix_len: int, cm: CommonAttentionMetadata, fast_build: bool = False):
        t2r = ops.token_to_req_indices(cm.query_start_loc, cm.num_actual_tokens, out=self.token_to_req_indices)
        return CompressorMetadata(block_table=cm.block_table_tensor.clamp_(min=0), slot_mapping=cm.slot_mapping,
                                  block_size=self.block_size, token_to_req_indices=t2r)


_SM = {}


def _sm_count(device) -> int:
    d = torch.device(device)
    if d.type != "cuda":
        return 148
    if d not in _SM:
        _SM[d] = torch.cuda.get_device_properties(d).multi_processor_count
    return _SM[d]


@dataclass
class HCAStepMetadata:
    """The three metadata objects of one HCA layer keyed like the reference's
    forward context: ``{prefix}``, ``{prefix}.swa_cache``,
    ``{prefix}.compressor.state_cache``."""

    swa: SWAMetadata
    c128a: C128AMetadata
    compressor: CompressorMetadata
    extra: dict = field(default_factory=dict)

    def as_forward_context(self, prefixes: list[str]) -> dict:
        out = {}
        for p in prefixes:
            out[p] = self.c128a
            out[f"{p}.swa_cache"] = self.swa
            out[f"{p}.compressor.state_cache"] = self.compressor
        return out
