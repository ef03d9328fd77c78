"""The ERNIE 5.5 HCA attention module, as the model code calls it.

Mirrors the plugin's module API (``E/nvidia/attention.py``):

* ``select_ernie5_5_hca_cls(kv_cache_dtype)`` (``:554-558``) returns the
  fp8 (``fp8_ds_mla``) HCA class;
* ``Ernie5_5HCAAttention(vllm_config, prefix, topk_indices_buffer=None,
  aux_stream_list=None)`` owns the parameters under the names the checkpoint
  mapper fills (``E/nvidia/model.py:656-704``) and exposes
  ``forward(positions, hidden_states, llama_4_scaling=None) -> [T, hidden]``
  (``:471-539``) reading per-step metadata from the forward context under
  ``{prefix}``, ``{prefix}.swa_cache`` and ``{prefix}.compressor.state_cache``;
* ``VHAPostMix`` / ``fold_vha`` (``:121-163``) including the TP branch
  (``o + V all_reduce(U^T o)`` in fp32 over this rank's heads).

The attention-side work is the library's CUDA kernels.  With a 128 x 128
block-FP8 quant config (``keeps_fp8_output``, the condition of
``keeps_fp8_wo_a`` in ``E/nvidia/quant_config.py``) the output path is the
reference's FP8 one: VHA + inverse RoPE + 1x128 UE8M0 quant (fused into the
decode attention launch on decode-only steps), the grouped ``wo_a`` einsum
and the gated ``wo_b`` on the library's tcgen05 FP8 GEMM, the gate's sigmoid
fused into ``wo_b``'s input quant.  Without it ``wo_a``/``wo_b`` stay bf16
(torch/cuBLAS), as the reference's non-FP8 path.  The input projections
(``fused_wqa_wkv``, ``wq_b``, compressor ``kv_score``, ``o_gate``) are
torch/cuBLAS GEMMs.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from types import SimpleNamespace
from typing import Any

import torch
import torch.distributed as dist
from torch import nn

from . import ops
from .backend import HCACacheSpec, _sm_count, hca_kv_cache_specs
from .cache_layout import SWA_BLOCK_SIZE, STATE_BLOCK_SIZE, compressed_page_size
from .forward_context import get_forward_context

VHA_RANK = 16


@dataclass
class Ernie5_5HCAConfig:
    """The HCA fields of ``Ernie5_5Config`` (``E/config.py:14-102``), same
    names and defaults."""

    hidden_size: int = 4096
    num_hidden_layers: int = 43
    num_attention_heads: int = 64
    num_key_value_heads: int = 1
    head_dim: int = 512
    q_lora_rank: int = 1024
    qk_rope_head_dim: int = 64
    o_groups: int = 8
    o_lora_rank: int = 1024
    sliding_window: int = 128
    compress_ratios: list[int] | None = None
    hybrid_mla_num_attention_heads: int = 64
    max_position_embeddings: int = 200192
    rope_theta: float = 2500000.0
    compress_rope_theta: float = 160000.0
    rms_norm_eps: float = 1e-6
    num_nextn_predict_layers: int = 1
    rope_parameters: dict = field(default_factory=lambda: {"rope_type": "default"})

    def __post_init__(self):
        if self.compress_ratios is None:
            self.compress_ratios = [128] * (self.num_hidden_layers + self.num_nextn_predict_layers)

    def is_dsa_layer(self, layer_id: int) -> bool:
        return layer_id < len(self.compress_ratios) and self.compress_ratios[layer_id] <= 0


def make_vllm_config(hf_config: Any, max_model_len: int = 131072, max_num_batched_tokens: int = 8192,
                     kv_cache_dtype: str = "fp8", num_speculative_tokens: int = 0,
                     quant_config: Any = None) -> SimpleNamespace:
    """A duck-typed stand-in for the ``VllmConfig`` fields the module reads."""
    spec = SimpleNamespace(num_speculative_tokens=num_speculative_tokens) if num_speculative_tokens else None
    return SimpleNamespace(
        model_config=SimpleNamespace(hf_config=hf_config, max_model_len=max_model_len),
        cache_config=SimpleNamespace(cache_dtype=kv_cache_dtype, block_size=256),
        scheduler_config=SimpleNamespace(max_num_batched_tokens=max_num_batched_tokens),
        speculative_config=spec, quant_config=quant_config)


def block_fp8_quant_config(ignored_layers: list[str] | None = None) -> SimpleNamespace:
    """The ``Fp8Config`` fields of a 128 x 128 block-FP8 checkpoint."""
    return SimpleNamespace(weight_block_size=[128, 128], ignored_layers=list(ignored_layers or []))


def keeps_fp8_output(quant_config: Any) -> bool:
    """Whether ``wo_a``/``wo_b`` run block FP8: a 128 x 128 block-FP8 config
    that does not ignore ``wo_a`` (``keeps_fp8_wo_a``,
    ``E/nvidia/quant_config.py``)."""
    if quant_config is None or list(getattr(quant_config, "weight_block_size", None) or []) != [128, 128]:
        return False
    ignored = getattr(quant_config, "ignored_layers", None) or []
    return not any(n.endswith(("linear_o_group_proj", ".attn.wo_a")) for n in ignored)


def _tp(group) -> tuple[int, int]:
    if group is None or not dist.is_available() or not dist.is_initialized():
        return 1, 0
    return dist.get_world_size(group), dist.get_rank(group)


def _check_attn_tp(config: Any, tp_size: int | None = None) -> None:
    """TP must divide ``o_groups`` and the head counts (``E/nvidia/attention.py:111-118``).
    ``tp_size`` defaults to the world size of the default process group (1
    when none is initialised), the tensor-parallel group of a TP-only run."""
    if tp_size is None:
        tp_size = dist.get_world_size() if dist.is_available() and dist.is_initialized() else 1
    for name in ("o_groups", "num_attention_heads", "hybrid_mla_num_attention_heads"):
        if getattr(config, name) % tp_size:
            raise ValueError(
                f"ERNIE 5.5 attention TP size {tp_size} must divide {name}={getattr(config, name)}.")


class VHAPostMix(nn.Module):
    """Head mixing ``o[h] <- sum_g m[h, g] o[g]`` with ``m = I + V U^T``
    (``E/nvidia/attention.py:121-157``)."""

    def __init__(self, num_heads: int, rank: int = VHA_RANK, tp_group=None):
        super().__init__()
        self.tp_group = tp_group
        self.tp_size, self.tp_rank = _tp(tp_group)
        local = num_heads // self.tp_size
        self.U = nn.Parameter(torch.zeros(local, rank), requires_grad=False)
        self.V = nn.Parameter(torch.zeros(local, rank), requires_grad=False)
        # checkpoint loaders call param.weight_loader(param, full_tensor)
        self.U.weight_loader = self.load_local_heads
        self.V.weight_loader = self.load_local_heads
        if self.tp_size == 1:
            self.register_buffer("m", torch.eye(num_heads), persistent=False)
            # the bf16 copy the fused VHA kernels read
            self.register_buffer("m_bf16", torch.eye(num_heads, dtype=torch.bfloat16), persistent=False)

    def load_local_heads(self, param: nn.Parameter, loaded: torch.Tensor) -> None:
        rows = param.shape[0]
        param.data.copy_(loaded[self.tp_rank * rows:(self.tp_rank + 1) * rows])

    def fold(self) -> None:
        """Idempotent, in place (graph-stable address)."""
        if self.tp_size != 1:
            return
        eye = torch.eye(self.U.shape[0], dtype=self.U.dtype, device=self.U.device)
        self.m.copy_(torch.addmm(eye, self.V, self.U.t()))
        self.m_bf16.copy_(self.m)

    def forward(self, o: torch.Tensor) -> torch.Tensor:
        if self.tp_size == 1:
            return torch.matmul(self.m.to(o.dtype), o)
        t = o.shape[0]
        u = self.U.t().to(o.dtype).expand(t, -1, -1)
        z = torch.bmm(u.float(), o.float())
        dist.all_reduce(z, group=self.tp_group)
        v = self.V.float().expand(t, -1, -1)
        return torch.bmm(v, z).add_(o.float()).to(o.dtype)


def fold_vha(model: nn.Module) -> None:
    for m in model.modules():
        if isinstance(m, VHAPostMix):
            m.fold()


class _Linear(nn.Module):
    def __init__(self, in_features: int, out_features: int, dtype):
        super().__init__()
        self.weight = nn.Parameter(torch.empty(out_features, in_features, dtype=dtype), requires_grad=False)

    def forward(self, x):
        return x @ self.weight.t()


class _FP8Linear(nn.Module):
    """Block-FP8 weight: ``weight`` e4m3 ``[N, K]`` and ``weight_scale_inv``
    fp32 ``[ceil(N / 128), K / 128]`` (the checkpoint names and layout of
    vLLM's block-FP8 linears)."""

    def __init__(self, in_features: int, out_features: int):
        super().__init__()
        self.weight = nn.Parameter(torch.empty(out_features, in_features, dtype=ops.FP8), requires_grad=False)
        self.weight_scale_inv = nn.Parameter(
            torch.empty((out_features + 127) // 128, in_features // 128, dtype=torch.float32), requires_grad=False)


class _RMSNorm(nn.Module):
    def __init__(self, n: int, dtype):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(n, dtype=dtype), requires_grad=False)


class _Compressor(nn.Module):
    """Parameters of ``DeepseekCompressor`` (``V/models/deepseek_v4/compressor.py:212-235``)."""

    def __init__(self, hidden: int, head_dim: int, ratio: int, dtype, prefix: str):
        super().__init__()
        self.compress_ratio = ratio
        self.head_dim = head_dim
        self.ape = nn.Parameter(torch.zeros(ratio, head_dim, dtype=torch.float32), requires_grad=False)
        self.fused_wkv_wgate = _Linear(hidden, 2 * head_dim, dtype)
        self.norm = _RMSNorm(head_dim, torch.float32)
        self.state_cache_prefix = f"{prefix}.state_cache"


# ---------------------------------------------------------------------------
# custom-op boundary
# ---------------------------------------------------------------------------
# The reference runs a layer's attention as ``torch.ops.vllm.deepseek_v4_attention(
# hidden_states, positions, out, layer_name)``: a custom op that mutates ``out``,
# with a fake implementation, which finds its layer by name in the forward
# context (``V/models/deepseek_v4/attention.py:545-571``).  Its counterpart here
# takes the layer's projected inputs.

_LAYERS: dict[str, nn.Module] = {}


def _register_layer(vllm_config: Any, name: str, layer: nn.Module) -> None:
    """Make the layer findable by name: in vLLM's static forward context when
    the config has one, and in this module's registry."""
    _LAYERS[name] = layer
    ctx = getattr(getattr(vllm_config, "compilation_config", None), "static_forward_context", None)
    if isinstance(ctx, dict):
        ctx[name] = layer


def _find_layer(name: str) -> nn.Module:
    try:
        layers = get_forward_context().no_compile_layers
    except RuntimeError:
        layers = {}
    layer = layers.get(name) if isinstance(layers, dict) else None
    if layer is None:
        layer = _LAYERS.get(name)
    if layer is None:
        raise KeyError(f"no HCA attention layer registered as {name!r}")
    return layer


@torch.library.custom_op("hca_b200::hca_attention", mutates_args=("out", "out_scale"))
def hca_attention(q: torch.Tensor, kv: torch.Tensor, kv_score: torch.Tensor, positions: torch.Tensor,
                  out: torch.Tensor, out_scale: torch.Tensor, layer_name: str) -> None:
    """The layer's attention (KV insert, compressor, sparse decode / prefill),
    reading this step's metadata from the forward context, into either
    ``out`` bf16 ``[T, H_local, D]`` (``out_scale`` empty), or, on the FP8
    output path, ``wo_a``'s quantised input: ``out`` e4m3 ``[G, T, HPG * D]``
    of VHA + inverse RoPE and ``out_scale`` int32 ``[G, HPG, round_up(T, 4)]``
    UE8M0 exponents."""
    layer = _find_layer(layer_name)
    layer._attention(q, kv, kv_score, positions, out, out_scale, get_forward_context().attn_metadata)


@hca_attention.register_fake
def _hca_attention_fake(q, kv, kv_score, positions, out, out_scale, layer_name):
    return None


class Ernie5_5HCAAttention(nn.Module):
    """One HCA layer on the fp8 ``fp8_ds_mla`` cache (replaces
    ``Ernie5_5HCAFlashMLAAttention``, ``E/nvidia/attention.py:548-551``)."""

    def __init__(self, vllm_config: Any, prefix: str, topk_indices_buffer=None,
                 aux_stream_list: list | None = None, tp_group=None, dtype=torch.bfloat16):
        super().__init__()
        cfg = vllm_config.model_config.hf_config
        self.tp_group = tp_group
        tp_size, self.tp_rank = _tp(tp_group)
        _check_attn_tp(cfg, tp_size)
        self.prefix = prefix
        self.layer_name = f"{prefix}.deepseek_v4_multi_head_latent_attention"
        _register_layer(vllm_config, self.layer_name, self)
        self.hidden_size = cfg.hidden_size
        self.n_heads = cfg.num_attention_heads
        self.n_local_heads = self.n_heads // tp_size
        self.head_dim = cfg.head_dim
        self.rope_head_dim = cfg.qk_rope_head_dim
        self.nope_head_dim = self.head_dim - self.rope_head_dim
        self.q_lora_rank = cfg.q_lora_rank
        self.o_lora_rank = cfg.o_lora_rank
        self.n_groups = cfg.o_groups
        self.n_local_groups = self.n_groups // tp_size
        self.window_size = cfg.sliding_window
        self.eps = cfg.rms_norm_eps
        layer_id = _layer_index(prefix)
        ratios = cfg.compress_ratios
        self.compress_ratio = max(1, ratios[layer_id]) if layer_id < cfg.num_hidden_layers else 1
        if self.compress_ratio != 128:
            raise ValueError(f"{prefix}: HCA layers compress 128 tokens per entry, got {self.compress_ratio}")
        self.scale = self.head_dim ** -0.5
        self.padded_heads = self.n_local_heads  # no head padding (FlashMLA pads to 64/128)
        self.aux_stream_list = aux_stream_list
        self.max_model_len = vllm_config.model_config.max_model_len

        self.fused_wqa_wkv = _Linear(self.hidden_size, self.q_lora_rank + self.head_dim, dtype)
        self.q_norm = _RMSNorm(self.q_lora_rank, dtype)
        self.wq_b = _Linear(self.q_lora_rank, self.n_local_heads * self.head_dim, dtype)
        self.kv_norm = _RMSNorm(self.head_dim, dtype)
        wo_a_in = self.n_heads * self.head_dim // self.n_groups
        # block-FP8 wo_a/wo_b where the reference keeps them FP8 and the
        # blocks tile the groups (o_lora_rank and the group width multiples
        # of 128; wo_b's input quant packs four 128-blocks per int32)
        self.fp8_output = (keeps_fp8_output(getattr(vllm_config, "quant_config", None))
                           and self.o_lora_rank % 128 == 0 and wo_a_in % (128 if tp_size == 1 else 512) == 0
                           and (self.n_local_groups * self.o_lora_rank) % 512 == 0)
        if self.fp8_output:
            self.wo_a = _FP8Linear(wo_a_in, self.n_local_groups * self.o_lora_rank)
            self.wo_b = _FP8Linear(self.n_local_groups * self.o_lora_rank, self.hidden_size)
        else:
            self.wo_a = _Linear(wo_a_in, self.n_local_groups * self.o_lora_rank, dtype)
            self.wo_b = _Linear(self.n_local_groups * self.o_lora_rank, self.hidden_size, dtype)
        self.o_gate = _Linear(self.q_lora_rank, self.n_local_groups * self.o_lora_rank, dtype)
        self.vha = VHAPostMix(self.n_heads, tp_group=tp_group)
        self.attn_sink = nn.Parameter(torch.full((max(self.n_local_heads, 64),), -float("inf")),
                                      requires_grad=False)
        self.compressor = _Compressor(self.hidden_size, self.head_dim, self.compress_ratio, dtype,
                                      f"{prefix}.compressor")
        theta = cfg.compress_rope_theta
        inv = 1.0 / (theta ** (torch.arange(0, self.rope_head_dim, 2, dtype=torch.float) / self.rope_head_dim))
        # the RoPE kernels index this table by position: every position the
        # model can reach must have a row (vLLM refuses such configs too)
        if self.max_model_len > cfg.max_position_embeddings:
            raise ValueError(f"max_model_len {self.max_model_len} exceeds max_position_embeddings "
                             f"{cfg.max_position_embeddings}")
        t = torch.arange(min(cfg.max_position_embeddings, self.max_model_len + 1), dtype=torch.float)
        f = torch.outer(t, inv)
        self.register_buffer("cos_sin_cache", torch.cat([f.cos(), f.sin()], -1), persistent=False)
        # caches are bound by the engine (bind_kv_cache)
        self.swa_cache = torch.tensor([])
        self.kv_cache = torch.tensor([])
        self.state_cache = torch.tensor([])
        self.comp_page = compressed_page_size(self.compress_ratio)

    # -- engine-facing -----------------------------------------------------
    def get_kv_cache_spec(self) -> dict[str, HCACacheSpec]:
        return hca_kv_cache_specs(self.head_dim, self.rope_head_dim, self.window_size, self.compress_ratio)

    def bind_kv_cache(self, swa_cache: torch.Tensor, kv_cache: torch.Tensor, state_cache: torch.Tensor) -> None:
        """``swa_cache``/``kv_cache``: uint8 ``[pages, ...]`` (page stride =
        ``stride(0)`` bytes); ``state_cache``: fp32 ``[pages, 8, 2 * D]``."""
        self.swa_cache, self.kv_cache, self.state_cache = swa_cache, kv_cache, state_cache

    def process_weights_after_loading(self) -> None:
        self.vha.fold()

    # -- forward -----------------------------------------------------------
    def forward(self, positions: torch.Tensor, hidden_states: torch.Tensor,
                llama_4_scaling: torch.Tensor | None = None) -> torch.Tensor:
        T = hidden_states.shape[0]
        d, r = self.head_dim, self.rope_head_dim
        aux = self._aux_streams(hidden_states)
        # input GEMMs: fused_wqa_wkv here, the compressor's kv_score on aux
        # stream 0 (V/models/deepseek_v4/attention.py:355-405)
        kv_score = self._on_aux(aux, 0, lambda: self._kv_score(hidden_states))
        qr_kv = self.fused_wqa_wkv(hidden_states)
        qr, kv = qr_kv.split([self.q_lora_rank, d], dim=-1)
        qr, kv = ops.fused_q_kv_rmsnorm(qr, kv, self.q_norm.weight, self.kv_norm.weight, self.eps)
        # the gate GEMM on aux stream 1 during attention (HCA has no
        # indexer: E/nvidia/attention.py:487-510); the FP8 path's wo_b input
        # quant applies the sigmoid itself
        gate = self._on_aux(aux, 1, lambda: self.o_gate(qr) if self.fp8_output else torch.sigmoid(self.o_gate(qr)))
        q = self.wq_b(qr).view(T, self.n_local_heads, d)
        kv_score = self._join(aux, 0, kv_score)
        attn_metadata = get_forward_context().attn_metadata
        dev = hidden_states.device
        if self.fp8_output and self.vha.tp_size == 1:
            # VHA + inverse RoPE + FP8 quant inside the attention op
            hpg = self.n_local_heads // self.n_local_groups
            o = torch.empty((self.n_local_groups, T, hpg * d), dtype=ops.FP8, device=dev)
            o_scale = torch.empty((self.n_local_groups, hpg, ops._aligned(T)), dtype=torch.int32, device=dev)
        else:
            o = torch.empty((T, self.n_local_heads, d), dtype=hidden_states.dtype, device=dev)
            o_scale = torch.empty(0, dtype=torch.int32, device=dev)
        if not isinstance(attn_metadata, dict):  # profile / dummy run
            o.view(torch.uint8).zero_() if o.dtype == ops.FP8 else o.zero_()
            o_scale.fill_(127)
        else:
            # the attention part is one opaque op that writes `o` in place (an
            # eager break under graph compilation, as the reference's)
            torch.ops.hca_b200.hca_attention(q, kv, kv_score, positions, o, o_scale, self.layer_name)
        gate = self._join(aux, 1, gate)
        if o.dtype == ops.FP8:
            return self._output_fp8(o.transpose(0, 1), o_scale.permute(2, 0, 1)[:T], gate)
        return self._output(o, positions, gate)

    def _kv_score(self, x: torch.Tensor) -> torch.Tensor:
        """fp32 ``x @ W^T`` of the bf16 compressor weight
        (``torch.mm(..., out_dtype=torch.float32)`` as the reference; the fp32
        matmul off the GPU)."""
        w = self.compressor.fused_wkv_wgate.weight
        if x.is_cuda:
            return torch.mm(x, w.t(), out_dtype=torch.float32)
        return x.float() @ w.float().t()

    def _aux_streams(self, x: torch.Tensor):
        """The first two aux streams when the caller passed them and the
        step runs on a GPU, else None (serial)."""
        if not x.is_cuda or not self.aux_stream_list or len(self.aux_stream_list) < 2:
            return None
        return self.aux_stream_list[:2]

    def _on_aux(self, aux, i: int, fn):
        """Run ``fn`` on aux stream ``i`` after the work queued so far on the
        current stream; None streams run it inline."""
        if aux is None:
            return fn()
        cur = torch.cuda.current_stream()
        aux[i].wait_stream(cur)
        with torch.cuda.stream(aux[i]):
            out = fn()
        return out

    def _join(self, aux, i: int, t: torch.Tensor) -> torch.Tensor:
        """Make the current stream wait for aux stream ``i``'s result ``t``."""
        if aux is None:
            return t
        cur = torch.cuda.current_stream()
        cur.wait_stream(aux[i])
        t.record_stream(cur)
        return t

    def _attention(self, q, kv, kv_score, positions, o, o_scale, md: dict) -> None:
        d, r = self.head_dim, self.rope_head_dim
        quant = o.dtype == ops.FP8  # o: wo_a's FP8 input [G, T, HPG*D], o_scale its exponents
        T = o.shape[1] if quant else o.shape[0]
        swa = md[f"{self.prefix}.swa_cache"]
        c128 = md[self.prefix]
        comp = md[self.compressor.state_cache_prefix]
        n = swa.slot_mapping.shape[0]
        if swa.num_prefills == 0:
            # decode-only step: the three cache ops below in one launch
            qp = ops.decode_prep(q, kv, kv_score, self.compressor.ape, positions, self.cos_sin_cache,
                                 self.swa_cache, swa.slot_mapping, SWA_BLOCK_SIZE, self.state_cache, comp.slot_mapping,
                                 comp.block_table, STATE_BLOCK_SIZE, self.kv_cache, c128.slot_mapping, self.comp_page,
                                 self.compressor.norm.weight, swa.query_start_loc, comp.token_to_req_indices,
                                 swa.num_decodes, self.padded_heads, self.eps, self.compress_ratio, r)
        else:
            qp = ops.fused_qnorm_rope_kv_insert(q, kv, self.swa_cache, swa.slot_mapping, positions,
                                                self.cos_sin_cache, self.padded_heads, self.eps, SWA_BLOCK_SIZE, r)
            ops.save_partial_states(kv_score[:, :d], kv_score[:, d:], self.compressor.ape, positions,
                                    self.state_cache, comp.slot_mapping, STATE_BLOCK_SIZE, d, self.compress_ratio)
            ops.compress_norm_rope_store(self.state_cache, n, comp.token_to_req_indices, positions,
                                         comp.slot_mapping, comp.block_table, STATE_BLOCK_SIZE, d, self.cos_sin_cache,
                                         self.kv_cache, c128.slot_mapping, self.comp_page, d, r, self.compress_ratio,
                                         self.compressor.norm.weight, self.eps)
        ndt, nd = swa.num_decode_tokens, swa.num_decodes
        sink = self.attn_sink[: self.n_local_heads].contiguous()
        if ndt:
            if c128.decode_schedule is None:
                # the step's balanced work list: one wave of CTAs over the SMs
                groups = swa.decode_group_starts.numel() - 1
                # (a CTA per SM; a CTA pair per two SMs at head_dim 512)
                sms = _sm_count(qp.device)
                c128.decode_items = max(sms if d == 128 else sms // 2, groups)
                c128.decode_schedule = ops.decode_schedule(swa.decode_group_starts, ndt, swa.decode_swa_lens,
                                                           c128.c128a_decode_topk_lens, c128.decode_items)
            if quant and ndt == T and d == 128 and self.n_local_heads % 16 == 0 and self.n_local_heads <= 64:
                # decode-only step: attention, split merge, VHA, inverse RoPE
                # and FP8 quant in two launches (no bf16 O round trip)
                ops.sparse_decode_vha_fp8_quant(
                    qp[:ndt], self.swa_cache, SWA_BLOCK_SIZE, swa.decode_swa_indices, swa.decode_swa_lens,
                    self.kv_cache, self.comp_page, c128.c128a_global_decode_topk_indices, c128.c128a_decode_topk_lens,
                    self.scale, sink, swa.decode_group_starts, swa.decode_max_group_tokens, c128.decode_schedule,
                    c128.decode_items, self.vha.m_bf16, positions, self.cos_sin_cache, self.n_local_groups, r,
                    out=o, scale_out=o_scale)
                return
        ob = torch.empty((T, self.n_local_heads, d), dtype=q.dtype, device=q.device) if quant else o
        if ndt:
            ops.sparse_decode(qp[:ndt], self.swa_cache, SWA_BLOCK_SIZE, swa.decode_swa_indices, swa.decode_swa_lens,
                              self.kv_cache, self.comp_page, c128.c128a_global_decode_topk_indices,
                              c128.c128a_decode_topk_lens, self.scale, sink, out=ob[:ndt],
                              group_starts=swa.decode_group_starts, max_group_tokens=swa.decode_max_group_tokens,
                              rope_dim=r, schedule=c128.decode_schedule, max_items=c128.decode_items)
        if swa.num_prefills:
            qsl = swa.query_start_loc[nd:] - ndt
            ops.sparse_prefill(qp[ndt:n], qsl, swa.seq_lens[nd:], self.swa_cache, SWA_BLOCK_SIZE,
                               swa.block_table[nd:], self.kv_cache, self.comp_page, c128.block_table[nd:],
                               self.window_size, self.compress_ratio, self.scale, sink, out=ob[ndt:n], rope_dim=r)
        if quant:
            if n < T:
                ob[n:].zero_()  # padding rows: finite values for the quant
            ops.vha_inv_rope_fp8_quant(ob, self.vha.m_bf16, positions, self.cos_sin_cache, self.n_local_groups,
                                       self.nope_head_dim, r, out=o, scale_out=o_scale)

    def _output(self, o, positions, gate):
        T = o.shape[0]
        if self.fp8_output:
            # head-sharded TP: VHA with its all-reduce, then inverse RoPE + quant
            x, xs = ops.fused_inv_rope_fp8_quant(self.vha(o), positions, self.cos_sin_cache, self.n_local_groups,
                                                 self.n_local_heads // self.n_local_groups, self.nope_head_dim,
                                                 self.rope_head_dim)
            return self._output_fp8(x, xs, gate)
        if self.vha.tp_size == 1:
            o = ops.vha_inv_rope(o, self.vha.m.to(o.dtype), positions, self.cos_sin_cache, self.rope_head_dim)
        else:
            o = ops.vha_inv_rope(self.vha(o), None, positions, self.cos_sin_cache, self.rope_head_dim)
        og = o.view(T, self.n_local_groups, -1).transpose(0, 1)            # [G, T, HPG*D]
        wa = self.wo_a.weight.view(self.n_local_groups, self.o_lora_rank, -1)  # [G, o_lora, HPG*D]
        z = torch.bmm(og, wa.transpose(1, 2)).transpose(0, 1).reshape(T, -1)  # [T, G*o_lora]
        y = self.wo_b(z * gate)
        if self.tp_group is not None and self.vha.tp_size > 1:
            dist.all_reduce(y, group=self.tp_group)
        return y

    def _output_fp8(self, x, xs, gate_logits):
        """The reference's FP8 output path (``V/models/deepseek_v4/attention.py:317-347``
        and the gated ``wo_b`` of ``E/nvidia/attention.py:364-395,466-469``):
        grouped ``wo_a`` on ``x`` (e4m3 ``[T, G, HPG*D]``, UE8M0 exponents
        ``xs`` ``[T, G, packs]``) -> ``z`` bf16 ``[T, G * o_lora]`` ->
        ``z * sigmoid(gate)`` quantised 1x128 -> ``wo_b`` (all-reduced over
        the TP group)."""
        G, L = self.n_local_groups, self.o_lora_rank
        T, K = x.shape[0], x.shape[2]
        z = ops.fp8_grouped_gemm(x, xs, self.wo_a.weight.view(G, L, K),
                                 self.wo_a.weight_scale_inv.view(G, L // 128, K // 128))
        zq, zs = ops.sigmoid_mul_quant_fp8(z.view(T, G * L), gate_logits)
        y = ops.fp8_grouped_gemm(zq, zs, self.wo_b.weight, self.wo_b.weight_scale_inv)
        if self.tp_group is not None and self.vha.tp_size > 1:
            dist.all_reduce(y, group=self.tp_group)
        return y

    # -- weights -----------------------------------------------------------
    def load_weights(self, weights) -> set[str]:
        """Load already-mapped names (``E/nvidia/model.py:656-704``); stacked
        shards arrive as ``(name, tensor, shard_id)``."""
        params = dict(self.named_parameters())
        loaded = set()
        for item in weights:
            name, w = item[0], item[1]
            shard = item[2] if len(item) > 2 else None
            p = params[name]
            if name in ("vha.U", "vha.V"):
                self.vha.load_local_heads(p, w)
            elif name == "attn_sink":
                p.data[: self.n_local_heads].copy_(w[self.tp_rank * self.n_local_heads:(self.tp_rank + 1) * self.n_local_heads])
            elif shard is not None:
                sizes = {"fused_wqa_wkv.weight": [self.q_lora_rank, self.head_dim],
                         "compressor.fused_wkv_wgate.weight": [self.head_dim, self.head_dim]}[name]
                off = sum(sizes[:shard])
                p.data[off:off + sizes[shard]].copy_(w)
            elif self.fp8_output and name in ("wo_a.weight", "wo_a.weight_scale_inv", "wo_b.weight",
                                              "wo_b.weight_scale_inv"):
                self._load_fp8(name, p, w)
            elif name in ("wq_b.weight", "wo_a.weight", "o_gate.weight"):
                rows = p.shape[0]
                p.data.copy_(w[self.tp_rank * rows:(self.tp_rank + 1) * rows])
            elif name == "wo_b.weight":
                cols = p.shape[1]
                p.data.copy_(w[:, self.tp_rank * cols:(self.tp_rank + 1) * cols])
            else:
                p.data.copy_(w)
            loaded.add(name)
        return loaded

    def _load_fp8(self, name: str, p: nn.Parameter, w: torch.Tensor) -> None:
        """This rank's slice of a block-FP8 ``wo_a`` (rows) or ``wo_b``
        (columns) weight or its block scales.  A weight that arrives in
        bf16/fp32 is quantised to 128 x 128 block FP8 here (power-of-two
        scales), filling ``weight_scale_inv`` too."""
        lin = self.wo_a if name.startswith("wo_a") else self.wo_b
        by_rows = name.startswith("wo_a")
        rows, cols = lin.weight.shape

        def local(t, block):
            if by_rows:
                n = rows // block
                return t[self.tp_rank * n:(self.tp_rank + 1) * n]
            n = cols // block
            return t[:, self.tp_rank * n:(self.tp_rank + 1) * n]

        if name.endswith("weight_scale_inv"):
            p.data.copy_(local(w, 128).float())
        elif w.dtype == ops.FP8:
            p.data.copy_(local(w, 1))
        else:
            q, sc = ops.quantize_weight_block_fp8(local(w, 1).to(torch.float32))
            lin.weight.data.copy_(q)
            lin.weight_scale_inv.data.copy_(sc)


def _layer_index(prefix: str) -> int:
    for part in prefix.split("."):
        if part.isdigit():
            return int(part)
    return 0


def select_ernie5_5_hca_cls(kv_cache_dtype: str) -> type[nn.Module]:
    """fp8 KV caches take this path (``E/nvidia/attention.py:554-558``);
    the bf16 FlashInfer variant is not part of this build."""
    if kv_cache_dtype.startswith("fp8"):
        return Ernie5_5HCAAttention
    raise ValueError(f"HCA on B200 stores fp8_ds_mla caches; kv_cache_dtype={kv_cache_dtype!r} is not supported")
