"""Whole HCA layer forward on the CPU in fp32 (config-1 oracle).

Restates ``Ernie5_5HCAAttentionMixin.forward``
(``E/nvidia/attention.py:471-539``) over the inherited DeepSeek-V4 MLA
wrapper (``V/models/deepseek_v4/attention.py:280-495``), compressor
(``V/models/deepseek_v4/compressor.py:270-380``) and FlashMLA sparse
attention (``V/models/deepseek_v4/nvidia/flashmla.py:130-424``), with the
unfused bf16 ``wo_a`` output path (the checkpoint is not 128x128 block FP8:
``E/nvidia/attention.py:417-428``, ``V/v1/attention/ops/rocm_aiter_mla_sparse.py:894-927``).

``fp8_output=True`` follows the reference's FP8 output path instead
(128 x 128 block-FP8 ``wo_a``/``wo_b``: ``E/nvidia/attention.py:417-428,
439-469``, ``V/models/deepseek_v4/attention.py:317-347``): the fused VHA +
inverse RoPE + 1x128 UE8M0 quant, the grouped ``wo_a`` on the dequantised
operands with one bf16 rounding, ``sigmoid_mul_quant_fp8`` and ``wo_b`` on
its dequantised output; ``wo_a.weight``/``wo_b.weight`` are then the
dequantised block-FP8 weights.

Two evaluations: ``emulate_quant=True`` runs the FP8/UE8M0 cache and the
bf16 roundings exactly as the reference kernels do (the comparison target
of the CUDA path); ``emulate_quant=False`` keeps everything fp32 (the
"exact" reference of the tolerance check).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import cache as C
from . import metadata as M
from .attention import sparse_attention_token
from .fp8 import bf16_round, e4m3_to_f32
from .output import kv_rope, q_prep, rms_norm, sigmoid_mul_quant_fp8, vha_fold, vha_inv_rope_fp8_quant


@dataclass
class HCAShape:
    hidden: int = 2048
    heads: int = 16
    head_dim: int = 128
    rope_dim: int = 64
    q_lora: int = 512
    o_groups: int = 4
    o_lora: int = 64
    vha_rank: int = 16
    window: int = 128
    ratio: int = 128
    eps: float = 1e-6
    rope_theta: float = 160000.0


def random_weights(shape: HCAShape, seed: int = 0, std: float = 0.02) -> dict[str, np.ndarray]:
    """N(0, std) weights under the plugin's parameter names
    (``E/nvidia/model.py:656-704``); norms are N(1, std), sinks N(0, 1)."""
    import torch

    g = torch.Generator().manual_seed(seed)
    s = shape

    def n(*sz, mean=0.0, sd=std):
        return (torch.randn(*sz, generator=g) * sd + mean).numpy().astype(np.float32)

    return {
        "fused_wqa_wkv.weight": n(s.q_lora + s.head_dim, s.hidden),
        "q_norm.weight": n(s.q_lora, mean=1.0),
        "wq_b.weight": n(s.heads * s.head_dim, s.q_lora),
        "kv_norm.weight": n(s.head_dim, mean=1.0),
        "wo_a.weight": n(s.o_groups * s.o_lora, s.heads * s.head_dim // s.o_groups),
        "wo_b.weight": n(s.hidden, s.o_groups * s.o_lora),
        "o_gate.weight": n(s.o_groups * s.o_lora, s.q_lora),
        "vha.U": n(s.heads, s.vha_rank),
        "vha.V": n(s.heads, s.vha_rank),
        "attn_sink": n(s.heads, sd=1.0),
        "compressor.ape": n(s.ratio, s.head_dim),
        "compressor.fused_wkv_wgate.weight": n(2 * s.head_dim, s.hidden),
        "compressor.norm.weight": n(s.head_dim, mean=1.0),
    }


class HCALayerOracle:
    """One HCA layer with its own paged caches (contiguous pages per request)."""

    SWA_PAGE = 64
    COMP_PAGE = 2  # 256-token manager block / ratio 128
    STATE_PAGE = 8

    def __init__(self, shape: HCAShape, weights: dict[str, np.ndarray], max_len: int,
                 num_reqs: int, emulate_quant: bool = True, fp8_output: bool = False):
        self.s = shape
        self.w = weights
        self.emulate = emulate_quant
        self.fp8_output = fp8_output
        assert emulate_quant or not fp8_output
        s = shape
        self.cos_sin = C.rope_cos_sin_cache(max_len + 1, s.rope_dim, s.rope_theta)
        sw_pages = (max_len + self.SWA_PAGE - 1) // self.SWA_PAGE
        c_pages = (max_len // s.ratio + self.COMP_PAGE) // self.COMP_PAGE + 1
        st_pages = (max_len + self.STATE_PAGE - 1) // self.STATE_PAGE
        self.swa_bt = np.arange(num_reqs * sw_pages, dtype=np.int32).reshape(num_reqs, sw_pages)
        self.comp_bt = np.arange(num_reqs * c_pages, dtype=np.int32).reshape(num_reqs, c_pages)
        self.state_bt = np.arange(num_reqs * st_pages, dtype=np.int32).reshape(num_reqs, st_pages)
        self.swa_cache = np.zeros((num_reqs * sw_pages, C.page_bytes(self.SWA_PAGE, s.head_dim, s.rope_dim)), np.uint8)
        self.comp_cache = np.zeros((num_reqs * c_pages, C.page_bytes(self.COMP_PAGE, s.head_dim, s.rope_dim)), np.uint8)
        self.state = np.zeros((num_reqs * st_pages, self.STATE_PAGE, 2 * s.head_dim), np.float32)
        # fp32 shadow of the caches for the exact evaluation
        self.swa_f32: dict[tuple[int, int], np.ndarray] = {}
        self.comp_f32: dict[tuple[int, int], np.ndarray] = {}

    # -- helpers ----------------------------------------------------------
    def _r(self, x):
        return bf16_round(x) if self.emulate else np.asarray(x, np.float32)

    def forward(self, hidden: np.ndarray, query_start_loc: np.ndarray, seq_lens: np.ndarray) -> np.ndarray:
        """All tokens of requests ``b`` occupy positions
        ``[seq_lens[b] - q_len_b, seq_lens[b])``.  Returns ``[T, hidden]``."""
        s, w = self.s, self.w
        qsl = np.asarray(query_start_loc)
        t2r = M.token_to_req_indices(qsl)
        positions = np.concatenate([
            np.arange(int(seq_lens[b]) - (qsl[b + 1] - qsl[b]), int(seq_lens[b]))
            for b in range(len(seq_lens))]).astype(np.int64)
        x = self._r(hidden)
        qr_kv = self._r(x @ w["fused_wqa_wkv.weight"].T)
        qr, kv = qr_kv[:, : s.q_lora], qr_kv[:, s.q_lora:]
        qr = self._r(rms_norm(qr, w["q_norm.weight"], s.eps))
        kv = self._r(rms_norm(kv, w["kv_norm.weight"], s.eps))
        kv_score = (x @ w["compressor.fused_wkv_wgate.weight"].T).astype(np.float32)
        q = self._r(qr @ w["wq_b.weight"].T).reshape(-1, s.heads, s.head_dim)
        q = q_prep(q, positions, self.cos_sin, s.rope_dim, s.eps) if self.emulate else \
            C.rope_gptj(rms_norm(q, None, s.eps), positions[:, None], self.cos_sin, s.rope_dim)
        k_rows = kv_rope(kv, positions, self.cos_sin, s.rope_dim) if self.emulate else \
            C.rope_gptj(kv, positions, self.cos_sin, s.rope_dim)

        # KV insert into the SWA cache.
        swa_slots = M.slot_mapping(qsl, seq_lens, self.swa_bt, self.SWA_PAGE)
        C.insert_rows(self.swa_cache, swa_slots, k_rows, self.SWA_PAGE, s.head_dim, s.rope_dim)
        for t, p in enumerate(positions):
            self.swa_f32[(int(t2r[t]), int(p))] = k_rows[t]

        # Compressor: state save, then compress at block boundaries.
        st_slots = M.slot_mapping(qsl, seq_lens, self.state_bt, self.STATE_PAGE)
        C.save_partial_states(self.state, kv_score[:, : s.head_dim], kv_score[:, s.head_dim:],
                              w["compressor.ape"], positions, st_slots, self.STATE_PAGE, s.ratio)
        c_slots = M.compressed_slot_mapping(len(positions), qsl, seq_lens, self.comp_bt,
                                            self.COMP_PAGE, s.ratio)
        C.compress_norm_rope_store(self.state, t2r, positions, st_slots, self.state_bt,
                                   self.STATE_PAGE, w["compressor.norm.weight"], s.eps,
                                   self.cos_sin, self.comp_cache, c_slots, self.COMP_PAGE,
                                   s.head_dim, s.rope_dim, s.ratio)
        if not self.emulate:
            self._compress_exact(t2r, positions, st_slots)

        # Attention over [window || compressed] rows with the sink.
        o = np.zeros((len(positions), s.heads, s.head_dim), np.float32)
        for t, p in enumerate(positions):
            r = int(t2r[t])
            nc, nw = (int(p) + 1) // s.ratio, min(int(p) + 1, s.window)
            wpos = np.arange(int(p) - nw + 1, int(p) + 1)
            if self.emulate:
                wsl = self.swa_bt[r, wpos // self.SWA_PAGE].astype(np.int64) * self.SWA_PAGE + wpos % self.SWA_PAGE
                ci = np.arange(nc)
                csl = self.comp_bt[r, ci // self.COMP_PAGE].astype(np.int64) * self.COMP_PAGE + ci % self.COMP_PAGE
                k = np.concatenate([
                    C.read_rows(self.swa_cache, wsl, self.SWA_PAGE, s.head_dim, s.rope_dim),
                    C.read_rows(self.comp_cache, csl, self.COMP_PAGE, s.head_dim, s.rope_dim),
                ])
            else:
                k = np.stack([self.swa_f32[(r, int(pp))] for pp in wpos] +
                             [self.comp_f32[(r, i)] for i in range(nc)])
            o[t] = sparse_attention_token(q[t], k, s.head_dim ** -0.5, w["attn_sink"])
        o = self._r(o)

        if self.fp8_output:
            return self.output_fp8(o, self._r(qr @ w["o_gate.weight"].T), positions)
        # Gate, VHA, inverse RoPE, grouped wo_a, gated wo_b.
        gate = self._r(1.0 / (1.0 + np.exp(-self._r(qr @ w["o_gate.weight"].T))))
        m = vha_fold(w["vha.U"], w["vha.V"])
        m = self._r(m)
        o = self._r(np.einsum("hg,tgd->thd", m, o))
        o = C.rope_gptj(o, positions[:, None], self.cos_sin, s.rope_dim, inverse=True)
        o = self._r(o).reshape(len(positions), s.o_groups, -1)
        wa = w["wo_a.weight"].reshape(s.o_groups, s.o_lora, -1)
        z = self._r(np.einsum("tgd,grd->tgr", o, wa)).reshape(len(positions), -1)
        zg = self._r(z * gate)
        return (zg @ w["wo_b.weight"].T).astype(np.float32)

    def output_fp8(self, o, gate_logits, positions):
        """The FP8 output path on the bf16 attention output ``o [T, H, D]``
        and the bf16 gate logits ``[T, G * o_lora]``."""
        s, w = self.s, self.w
        t = len(positions)
        m = bf16_round(vha_fold(w["vha.U"], w["vha.V"]))
        q8, exp = vha_inv_rope_fp8_quant(o, m, positions, self.cos_sin, s.o_groups, s.rope_dim)
        scale = np.ldexp(np.float32(1.0), np.repeat(exp, 128, axis=-1))        # [T, H, D]
        x = e4m3_to_f32(q8.transpose(1, 0, 2)).reshape(t, s.heads, s.head_dim) * scale
        x = x.reshape(t, s.o_groups, -1)
        wa = w["wo_a.weight"].reshape(s.o_groups, s.o_lora, -1)
        z = bf16_round(np.einsum("tgd,grd->tgr", x.astype(np.float64), wa.astype(np.float64))).reshape(t, -1)
        zq, packed = sigmoid_mul_quant_fp8(z, gate_logits)
        ez = np.stack([(packed.view(np.uint32) >> (8 * c)) & 0xFF for c in range(4)], -1).reshape(t, -1)
        zf = e4m3_to_f32(zq) * np.ldexp(np.float32(1.0), np.repeat(ez.astype(np.int64) - 127, 128, axis=-1))
        return bf16_round(zf.astype(np.float64) @ w["wo_b.weight"].T.astype(np.float64)).astype(np.float32)

    def _compress_exact(self, t2r, positions, st_slots):
        """fp32 compressed rows (no quantisation) for the exact evaluation."""
        s = self.s
        d = s.head_dim
        for t, p in enumerate(positions):
            p = int(p)
            if st_slots[t] < 0 or (p + 1) % s.ratio:
                continue
            r = int(t2r[t])
            pos = np.arange(p - s.ratio + 1, p + 1)
            rows = self.state[self.state_bt[r, pos // self.STATE_PAGE], pos % self.STATE_PAGE]
            sc = rows[:, d:].astype(np.float64)
            e = np.exp(sc - sc.max(0, keepdims=True))
            c = ((e / e.sum(0, keepdims=True)) * rows[:, :d]).sum(0).astype(np.float32)
            normed = rms_norm(c, self.w["compressor.norm.weight"], s.eps)
            roped = C.rope_gptj(normed[None], np.array([(p // s.ratio) * s.ratio]), self.cos_sin, s.rope_dim)[0]
            self.comp_f32[(r, p // s.ratio)] = roped
