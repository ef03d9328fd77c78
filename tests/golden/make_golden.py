"""Generate golden vectors by running the reference's own Triton kernels on
the CPU (Triton interpreter).  Run in the build container only:

    HCA_REFERENCE_ATTENTION=<plugin>/src/vllm_ernie/models/ernie5_5/nvidia/attention.py \
        TRITON_INTERPRET=1 python tests/golden/make_golden.py [insert|compressor|metadata|output|attention ...]

Sources executed:

* vLLM's DeepSeek-V4 HCA kernels that the plugin inherits (installed
  ``vllm`` package; the plugin pins vLLM 0.32.0, this container has 0.22.0):
  KV insert, dequant gather, partial-state save, block compressor, slot
  mapping, window indices, C128A indices, prefill gather lengths, combined
  prefill indices, QK RMSNorm, inverse RoPE + FP8 quant.
* The plugin's own ``_vha_inv_rope_quant_kernel`` and
  ``_sigmoid_mul_quant_kernel`` (``src/vllm_ernie/models/ernie5_5/nvidia/attention.py``
  of the reference checkout), loaded from the reference source at run time
  because the plugin module itself needs vLLM 0.32 to import.

Shapes are the reference's hard-coded D=512 layout (448 NoPE + 64 RoPE).
The output ``*.npz`` files are committed; nothing at test time needs the
reference or vLLM.
"""

from __future__ import annotations

import ast
import os
import sys
from pathlib import Path

os.environ.setdefault("TRITON_INTERPRET", "1")

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
# The plugin's ``src/vllm_ernie/models/ernie5_5/nvidia/attention.py`` (needed
# by the "output" fixtures only): set HCA_REFERENCE_ATTENTION to its path.
PLUGIN_ATTENTION_ENV = "HCA_REFERENCE_ATTENTION"

D, R, NOPE = 512, 64, 448


def save(name: str, **arrays) -> None:
    out = {}
    for k, v in arrays.items():
        if isinstance(v, torch.Tensor):
            v = v.detach().cpu()
            if v.dtype == torch.bfloat16:
                v = v.float()
            elif v.dtype == torch.float8_e4m3fn:
                v = v.view(torch.uint8)
            elif v.dtype == torch.bool:
                v = v.to(torch.uint8)
            v = v.numpy()
        out[k] = np.asarray(v)
    np.savez_compressed(HERE / f"{name}.npz", **out)
    print(f"wrote {name}.npz: " + ", ".join(f"{k}{tuple(v.shape)}" for k, v in out.items()))


def patch_interpreter() -> None:
    """Make the interpreter's float conversions and bf16 dots behave like the GPU.

    The stock Triton interpreter truncates fp32 -> bf16 and rounds fp8
    ties away from zero without carrying into the exponent, while the
    compiled kernels use round-to-nearest-even conversions (``cvt.rn``).
    Downcasts between float types are redone here through torch's RTNE
    casts; everything else is left to the interpreter.
    """
    from triton.language import core as tlc
    from triton.runtime import interpreter as interp

    torch_of = {
        "fp32": torch.float32, "bf16": torch.bfloat16, "fp16": torch.float16,
        "fp8e4nv": torch.float8_e4m3fn, "fp8e5": torch.float8_e5m2,
    }
    bits_of = {torch.float32: torch.int32, torch.bfloat16: torch.int16, torch.float16: torch.int16,
               torch.float8_e4m3fn: torch.uint8, torch.float8_e5m2: torch.uint8}
    stock = interp._convert_float

    def convert(input, input_dtype, output_dtype, rounding_mode):
        src_t, dst_t = torch_of.get(input_dtype.name), torch_of.get(output_dtype.name)
        if (src_t is None or dst_t is None
                or input_dtype.primitive_bitwidth <= output_dtype.primitive_bitwidth
                or rounding_mode not in (None, interp._ir.ROUNDING_MODE.RTNE)):
            return stock(input, input_dtype, output_dtype, rounding_mode)
        raw = torch.from_numpy(np.ascontiguousarray(input).copy())
        src = raw.view(bits_of[src_t]).view(src_t) if raw.dtype != src_t else raw
        out = src.to(dst_t).view(bits_of[dst_t]).numpy()
        out_np = np.dtype(f"uint{output_dtype.primitive_bitwidth}")
        return out.view(out_np).reshape(np.shape(input))

    assert isinstance(tlc.float32, tlc.dtype)
    interp._convert_float = convert

    # The stock interpreter multiplies bf16 dot operands as raw uint16 bit
    # patterns; widen them to fp32 (exact) and accumulate in fp32 as the
    # tensor cores do.
    stock_dot = interp.InterpreterBuilder.create_dot

    def create_dot(self, a, b, d, input_precision, max_num_imprecise_acc):
        if a.dtype.scalar.name == "bf16" or b.dtype.scalar.name == "bf16":
            def widen(h):
                if h.dtype.scalar.name != "bf16":
                    return h.data.astype(np.float32)
                return (h.data.astype(np.uint32) << 16).view(np.float32)
            out = np.matmul(widen(a), widen(b), dtype=np.float32) + d.data
            return interp.TensorHandle(out.astype(d.data.dtype), d.dtype.scalar)
        return stock_dot(self, a, b, d, input_precision, max_num_imprecise_acc)

    interp.InterpreterBuilder.create_dot = create_dot

    # Elementwise arithmetic on two bf16 tensors (e.g. the fp8 dequant
    # ``x.to(bf16) * scale.to(bf16)``) would also act on the raw bit
    # patterns: evaluate it in fp32 and round to bf16 (RTNE), as the compiled
    # kernel's fp32-promoted arithmetic does.
    stock_binary = interp.InterpreterBuilder.binary_op

    def binary_op(self, lhs, rhs, op):
        if lhs.dtype.scalar.name != "bf16" or rhs.dtype.scalar.name != "bf16":
            return stock_binary(self, lhs, rhs, op)
        widen = lambda h: (h.data.astype(np.uint32) << 16).view(np.float32)  # noqa: E731
        res = op(widen(lhs), widen(rhs))
        if res.dtype != np.float32:
            return interp.TensorHandle(res, lhs.dtype.scalar)
        bits = torch.from_numpy(np.ascontiguousarray(res)).to(torch.bfloat16).view(torch.int16).numpy()
        return interp.TensorHandle(bits.view(np.uint16).reshape(np.shape(res)), lhs.dtype.scalar)

    interp.InterpreterBuilder.binary_op = binary_op


def plugin_kernels():
    """Load the plugin's two @triton.jit kernels from its source file."""
    from vllm.triton_utils import tl, triton

    path = os.environ.get(PLUGIN_ATTENTION_ENV)
    if not path:
        raise SystemExit(f"set {PLUGIN_ATTENTION_ENV} to the plugin's ernie5_5/nvidia/attention.py")
    path = Path(path)
    tree = ast.parse(path.read_text())
    wanted = {"_vha_inv_rope_quant_kernel", "_sigmoid_mul_quant_kernel"}
    nodes = [n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name in wanted]
    assert {n.name for n in nodes} == wanted
    ns = {"tl": tl, "triton": triton}
    exec(compile(ast.Module(body=nodes, type_ignores=[]), str(path), "exec"), ns)
    return ns["_vha_inv_rope_quant_kernel"], ns["_sigmoid_mul_quant_kernel"]


def rope_cache(max_pos: int, theta: float = 160000.0) -> torch.Tensor:
    inv = 1.0 / (theta ** (torch.arange(0, R, 2, dtype=torch.float) / R))
    f = torch.arange(max_pos, dtype=torch.float)[:, None] * inv
    return torch.cat([f.cos(), f.sin()], -1)


def gen_insert_and_gather(g: torch.Generator) -> None:
    from vllm.models.deepseek_v4.common.ops.cache_utils import (
        dequantize_and_gather_k_cache_triton,
        quantize_and_insert_k_cache,
    )

    page, pages = 64, 5
    n = 40
    k = (torch.randn(n, D, generator=g) * torch.logspace(-3, 2, n)[:, None]).bfloat16()
    k[3, :64] = 0.0  # amax floor
    k[4, 64:128] = 448.0  # scale exactly a power of two
    slots = torch.randperm(pages * page, generator=g)[:n].to(torch.int64)
    slots[7] = -1
    cache = torch.zeros(pages, page * 584, dtype=torch.uint8)
    quantize_and_insert_k_cache(k, cache, slots, block_size=page)
    # gather two requests through a block table
    bt = torch.tensor([[2, 0, 4], [1, 3, 0]], dtype=torch.int32)
    seq_lens = torch.tensor([150, 100], dtype=torch.int32)
    gather_lens = torch.tensor([130, 100], dtype=torch.int32)
    out = torch.zeros(2, 200, D, dtype=torch.bfloat16)
    dequantize_and_gather_k_cache_triton(out, cache.view(pages, page, 584), seq_lens, gather_lens,
                                         bt, page, offset=5)
    save("kv_insert_gather", k=k, slots=slots, cache=cache, block_table=bt, seq_lens=seq_lens,
         gather_lens=gather_lens, gathered=out, page=np.int64(page))


def gen_compressor(g: torch.Generator) -> None:
    from vllm.models.deepseek_v4.common.ops.fused_compress_quant_cache import (
        compress_norm_rope_store_triton,
    )
    from vllm.models.deepseek_v4.common.ops.save_partial_states import save_partial_states

    ratio, sbs = 128, 8
    # two requests: positions [100, 260) and [440, 520) -> boundaries 127, 255, 511
    spans = [(100, 260), (440, 520)]
    positions = torch.cat([torch.arange(a, b) for a, b in spans]).to(torch.int64)
    t2r = torch.cat([torch.full((b - a,), i, dtype=torch.int32) for i, (a, b) in enumerate(spans)])
    T = positions.shape[0]
    n_pages = 56
    pages_per_req = 520 // sbs + 1
    state_bt = torch.zeros(2, pages_per_req, dtype=torch.int32)
    perm = torch.randperm(n_pages, generator=g).to(torch.int32)
    state_bt[0, :33] = perm[:33]  # positions 0..263
    state_bt[1, 48:] = perm[33 : 33 + pages_per_req - 48]  # positions 384..527
    # bf16-representable fp32 values keep the fixture small
    state = torch.randn(n_pages, sbs, 2 * D, generator=g).bfloat16().float()
    state_before = state.clone()
    slot = (state_bt[t2r.long(), positions // sbs].long() * sbs + positions % sbs)
    slot[5] = -1
    kv = torch.randn(T, D, generator=g).bfloat16().float()
    score = (torch.randn(T, D, generator=g) * 2).bfloat16().float()
    ape = (torch.randn(ratio, D, generator=g) * 0.5).bfloat16().float()
    save_partial_states(kv, score, ape, positions, state, slot, sbs, D, ratio)
    written = state.view(-1, 2 * D)[slot.clamp(min=0)]
    # compressed cache: 2 entries per page
    comp_bt = torch.stack([torch.randperm(16, generator=g)[:4] for _ in spans]).to(torch.int32)
    cpos = positions // ratio
    comp_slot = torch.where((positions + 1) % ratio == 0,
                            comp_bt[t2r.long(), cpos // 2].long() * 2 + cpos % 2,
                            torch.full_like(positions, -1))
    kv_cache = torch.zeros(16, 2, 584, dtype=torch.uint8)
    cos_sin = rope_cache(1024)
    w = 1.0 + 0.1 * torch.randn(D, generator=g)

    class Meta:
        slot_mapping = comp_slot

    compress_norm_rope_store_triton(
        state_cache=state, num_actual=T, token_to_req_indices=t2r, positions=positions,
        slot_mapping=slot, block_table=state_bt, block_size=sbs, state_width=D,
        cos_sin_cache=cos_sin, kv_cache=kv_cache, k_cache_metadata=Meta, pdl_kwargs={},
        head_dim=D, rope_head_dim=R, compress_ratio=ratio, overlap=False, use_fp4_cache=False,
        rms_norm_weight=w, rms_norm_eps=1e-6, quant_block=64, token_stride=576, scale_dim=8)
    save("compressor", positions=positions, token_to_req=t2r, state_block_table=state_bt,
         state_before=state_before, kv=kv, score=score, ape=ape, state_slot=slot,
         state_rows_written=written, comp_block_table=comp_bt, comp_slot=comp_slot,
         kv_cache=kv_cache.view(16, -1), cos_sin=cos_sin, norm_weight=w)


def gen_compressor_blocks(g: torch.Generator, d: int = D) -> None:
    """More compressed blocks at the model's head_dim (the reference's HCA
    compressor kernel is the head_dim-512 one; other head sizes take its
    indexer kernel and cache format): three requests whose spans cover 8
    block boundaries -- a whole 512-token prefix, a span starting mid-block
    on earlier-step states (its first block pools 108 states written before
    the step), and a span from an odd offset -- through state pages of 8
    tokens in shuffled order, so blocks straddle pages everywhere.  Stores the
    compressed rows with their UE8M0 scale bytes."""
    from vllm.models.deepseek_v4.common.ops.fused_compress_quant_cache import (
        compress_norm_rope_store_triton,
    )
    from vllm.models.deepseek_v4.common.ops.save_partial_states import save_partial_states

    ratio, sbs = 128, 8
    nope = d - R
    spans = [(0, 512), (1900, 2100), (4995, 5250)]
    positions = torch.cat([torch.arange(a, b) for a, b in spans]).to(torch.int64)
    t2r = torch.cat([torch.full((b - a,), i, dtype=torch.int32) for i, (a, b) in enumerate(spans)])
    T = positions.shape[0]
    width = 5250 // sbs + 1
    state_bt = torch.zeros(len(spans), width, dtype=torch.int32)
    need = [(a // ratio * ratio // sbs, (b + sbs - 1) // sbs) for a, b in spans]  # pages of the blocks touched
    n_pages = sum(hi - lo for lo, hi in need)
    perm = torch.randperm(n_pages, generator=g).to(torch.int32)
    k = 0
    for r, (lo, hi) in enumerate(need):
        state_bt[r, lo:hi] = perm[k:k + hi - lo]
        k += hi - lo
    # earlier-step states only where a block starts before the step (bf16-
    # representable values keep the fixture small); zeros elsewhere
    state = torch.zeros(n_pages, sbs, 2 * d)
    for r, (a, _) in enumerate(spans):
        for p0 in range(a // ratio * ratio, a):
            pg = int(state_bt[r, p0 // sbs])
            state[pg, p0 % sbs] = torch.randn(2 * d, generator=g).bfloat16().float()
    state_before = state.clone()
    slot = (state_bt[t2r.long(), positions // sbs].long() * sbs + positions % sbs)
    kv = torch.randn(T, d, generator=g).bfloat16().float()
    score = (torch.randn(T, d, generator=g) * 2).bfloat16().float()
    ape = (torch.randn(ratio, d, generator=g) * 0.5).bfloat16().float()
    save_partial_states(kv, score, ape, positions, state, slot, sbs, d, ratio)
    # compressed cache: 2 entries per page
    n_cpages = 32
    comp_bt = torch.stack([torch.randperm(n_cpages, generator=g)[:24] for _ in spans]).to(torch.int32)
    cpos = positions // ratio
    comp_slot = torch.where((positions + 1) % ratio == 0,
                            comp_bt[t2r.long(), cpos // 2].long() * 2 + cpos % 2,
                            torch.full_like(positions, -1))
    entry = nope + 2 * R + nope // 64 + 1
    kv_cache = torch.zeros(n_cpages, 2, entry, dtype=torch.uint8)
    cos_sin = rope_cache(6144)
    w = 1.0 + 0.1 * torch.randn(d, generator=g)

    class Meta:
        slot_mapping = comp_slot

    compress_norm_rope_store_triton(
        state_cache=state, num_actual=T, token_to_req_indices=t2r, positions=positions,
        slot_mapping=slot, block_table=state_bt, block_size=sbs, state_width=d,
        cos_sin_cache=cos_sin, kv_cache=kv_cache, k_cache_metadata=Meta, pdl_kwargs={},
        head_dim=d, rope_head_dim=R, compress_ratio=ratio, overlap=False, use_fp4_cache=False,
        rms_norm_weight=w, rms_norm_eps=1e-6, quant_block=64, token_stride=nope + 2 * R,
        scale_dim=nope // 64 + 1)
    assert int((comp_slot >= 0).sum()) == 8
    save(f"compressor_blocks_d{d}", positions=positions, token_to_req=t2r, state_block_table=state_bt,
         state_before=state_before, kv=kv, score=score, ape=ape, state_slot=slot, comp_block_table=comp_bt,
         comp_slot=comp_slot, kv_cache=kv_cache.view(n_cpages, -1), cos_sin=cos_sin, norm_weight=w)


def gen_metadata(g: torch.Generator) -> None:
    from vllm.models.deepseek_v4.common.ops.cache_utils import combine_topk_swa_indices
    from vllm.v1.attention.backends.mla.compressor_utils import get_compressed_slot_mapping
    from vllm.v1.attention.backends.mla.flashmla_sparse import build_c128a_topk_metadata
    from vllm.v1.attention.backends.mla.sparse_swa import (
        _compute_prefill_metadata_kernel,
        _compute_swa_indices_and_lens_kernel,
    )

    # 3 decode requests (q_len 3, 3, 1 incl. MTP) then 2 prefills.
    q_lens = [3, 3, 1, 70, 200]
    seq_lens = torch.tensor([5000, 130, 2, 300, 1200], dtype=torch.int32)
    qsl = torch.tensor(np.concatenate([[0], np.cumsum(q_lens)]), dtype=torch.int32)
    T = int(qsl[-1])
    t2r = torch.repeat_interleave(torch.arange(5, dtype=torch.int32), torch.tensor(q_lens))
    positions = torch.cat([torch.arange(int(s) - q, int(s)) for s, q in zip(seq_lens, q_lens)]).to(torch.int64)
    num_decodes, num_decode_tokens = 3, 7
    # SWA block table (64-token pages), compressed (2 entries per page)
    swa_bt = torch.randint(0, 10000, (5, 100), generator=g, dtype=torch.int32)
    comp_bt = torch.randint(0, 10000, (5, 40), generator=g, dtype=torch.int32)
    slot_mapping = (swa_bt[t2r.long(), positions // 64].long() * 64 + positions % 64)
    slot_mapping[5] = -1  # one invalid (padding) decode token
    is_valid = slot_mapping >= 0

    comp_slot = get_compressed_slot_mapping(T, qsl, seq_lens, comp_bt, 2, 128,
                                            out=torch.empty(T + 8, dtype=torch.int64))

    W = 128
    swa_idx = torch.full((T, 1, W), 777, dtype=torch.int32)
    swa_lens = torch.full((T,), 99, dtype=torch.int32)
    swa_lens[num_decode_tokens:] = 0
    _compute_swa_indices_and_lens_kernel[(num_decode_tokens,)](
        swa_idx, swa_idx.stride(0), swa_lens, W, qsl, seq_lens, t2r, is_valid, swa_bt,
        swa_bt.stride(0), 64, TRITON_BLOCK_SIZE=1024)

    maxc = 128  # round_up(ceil(max_model_len 16384 / 128), 128)
    gdec = torch.full((T, maxc), 555, dtype=torch.int32)
    dlens = torch.full((T,), 555, dtype=torch.int32)
    plocal = torch.full((T, maxc), 555, dtype=torch.int32)
    build_c128a_topk_metadata(positions, 128, num_decode_tokens, t2r, comp_bt[:num_decodes], 2,
                              slot_mapping, gdec, dlens, plocal, max_compressed_tokens=maxc)

    num_prefills = 2
    glens = torch.empty(num_prefills, dtype=torch.int32)
    _compute_prefill_metadata_kernel[(1,)](glens, seq_lens, qsl, num_prefills, num_decodes, W,
                                           BLOCK_SIZE=2)
    npt = T - num_decode_tokens
    Nc = 16384 // 128
    Mw = Nc + W + 512
    comb, clens = combine_topk_swa_indices(plocal[:npt], qsl[num_decodes:], seq_lens[num_decodes:],
                                           glens, W, 128, maxc, Mw, Nc)
    save("metadata", q_lens=np.array(q_lens), seq_lens=seq_lens, query_start_loc=qsl,
         token_to_req=t2r, positions=positions, swa_block_table=swa_bt, comp_block_table=comp_bt,
         slot_mapping=slot_mapping, comp_slot=comp_slot, swa_indices=swa_idx[:, 0],
         swa_lens=swa_lens, c128a_global=gdec, c128a_lens=dlens, c128a_prefill=plocal,
         gather_lens=glens, combined=comb, combined_lens=clens,
         num_decodes=np.int64(num_decodes), num_decode_tokens=np.int64(num_decode_tokens),
         M=np.int64(Mw), N=np.int64(Nc), max_compressed=np.int64(maxc))


def gen_norm_and_output(g: torch.Generator) -> None:
    from vllm.models.deepseek_v4.common.ops.fused_inv_rope_fp8_quant import (
        _fused_inv_rope_fp8_quant_kernel_impl,
    )
    from vllm.models.deepseek_v4.common.ops.fused_qk_rmsnorm import fused_q_kv_rmsnorm

    T = 9
    qr = (torch.randn(T, 1024, generator=g) * 3).bfloat16()
    kv = torch.randn(T, D, generator=g).bfloat16()
    qw = (1 + 0.1 * torch.randn(1024, generator=g)).bfloat16()
    kw = (1 + 0.1 * torch.randn(D, generator=g)).bfloat16()
    qn, kn = fused_q_kv_rmsnorm(qr, kv, qw, kw, 1e-6)
    save("qk_rmsnorm", qr=qr, kv=kv, q_weight=qw, kv_weight=kw, q_out=qn, kv_out=kn)

    H, G = 64, 8
    o = torch.randn(T, H, D, generator=g).bfloat16()
    positions = torch.randint(0, 512, (T,), generator=g)
    cos_sin = rope_cache(512, 10000.0)
    aligned = (T + 3) // 4 * 4
    fp8, scale = _fused_inv_rope_fp8_quant_kernel_impl(
        o, positions, cos_sin, H // G, 128, D // 128, NOPE % 128, R // 2, True, 448.0, aligned,
        T, G, (H // G) * D, ((H // G) * D // 128 + 3) // 4)
    save("inv_rope_fp8_quant", o=o, positions=positions, cos_sin=cos_sin, fp8=fp8,
         scale=scale.as_strided((G, aligned, scale.shape[-1]), (scale.stride(0), 1, scale.stride(2))).contiguous(),
         n_groups=np.int64(G))

    vha_kernel, sig_kernel = plugin_kernels()
    # Plugin VHA + inverse RoPE + FP8 (launch as vha_inv_rope_fp8_quant does).
    o_pad = torch.randn(T, 128, D, generator=g).bfloat16()
    o2 = o_pad[:, :H]
    u = torch.randn(H, 16, generator=g) / 8
    v = torch.randn(H, 16, generator=g) / 8
    mix = (torch.eye(H) + v @ u.T).bfloat16()
    hpg = H // G
    out = torch.zeros(G, T, hpg * D, dtype=torch.float8_e4m3fn)
    sc = torch.full((G, hpg, aligned), -1, dtype=torch.int32)
    vha_kernel[(aligned, D // 128)](
        o2, mix, positions, cos_sin, out, sc.view(torch.uint8), T, o2.stride(0), o2.stride(1),
        cos_sin.stride(0), out.stride(0), sc.stride(0), sc.stride(1), NUM_HEADS=H,
        HEADS_PER_GROUP=hpg, HEAD_DIM=D, NOPE_DIM=NOPE, HALF_ROPE=R // 2, BLOCK=128,
        FP8_MAX=448.0, num_warps=4)
    save("vha_inv_rope_fp8_quant", o=o2.contiguous(), mix=mix, positions=positions, cos_sin=cos_sin,
         fp8=out, scale=sc, n_groups=np.int64(G))

    # Plugin sigmoid gate + FP8 quant (launch as sigmoid_mul_quant_fp8 does).
    for rows, hidden in [(5, 1024), (13, 2048)]:
        x = (torch.randn(rows, hidden, generator=g) * 3).bfloat16()
        gate = (torch.randn(rows, hidden, generator=g) * 4).bfloat16()
        packs = hidden // 512
        al = (rows + 3) // 4 * 4
        q = torch.zeros(rows, hidden, dtype=torch.float8_e4m3fn)
        s = torch.empty_strided((rows, packs), (1, al), dtype=torch.int32)
        s.zero_()
        sig_kernel[(packs, (rows + 3) // 4)](
            x, gate, q, s, rows, x.stride(0), gate.stride(0), s.stride(1), HIDDEN=hidden,
            BLOCK=128, BLOCK_M=4, FP8_MAX=448.0, num_warps=4)
        save(f"sigmoid_mul_quant_{rows}x{hidden}", x=x, gate=gate, fp8=q, scale=s.contiguous())


def _bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def _fill_rows(cache: torch.Tensor, slots: np.ndarray, block: int, g: torch.Generator) -> None:
    """Write N(0, 1) rows (bf16, then the reference's fp8 insert) at ``slots``."""
    from vllm.models.deepseek_v4.common.ops.cache_utils import quantize_and_insert_k_cache

    slots = np.unique(slots[slots >= 0]).astype(np.int64)
    k = torch.randn(len(slots), D, generator=g).bfloat16()
    quantize_and_insert_k_cache(k, cache, torch.from_numpy(slots), block_size=block)


def gen_attention() -> None:
    """Sparse decode and prefill attention at D=512, through vLLM's readable
    DeepSeek-V4 Triton kernels ``_sparse_attn_decode_ragged_kernel`` and
    ``_sparse_attn_prefill_ragged_kernel``
    (``vllm/v1/attention/ops/rocm_aiter_mla_sparse.py``), fed the way
    ``vllm/models/deepseek_v4/amd/rocm.py`` ``_forward_decode`` /
    ``_forward_prefill`` feed them: builders' index tables, ragged packing,
    the bf16 gather workspace and ``combine_topk_swa_indices`` for prefill.
    Every step runs reference code; its own seed keeps the fixture
    independent of the other generators."""
    from vllm.models.deepseek_v4.common.ops.cache_utils import (
        combine_topk_swa_indices,
        dequantize_and_gather_k_cache_triton,
    )
    from vllm.v1.attention.backends.mla.flashmla_sparse import build_c128a_topk_metadata
    from vllm.v1.attention.backends.mla.sparse_swa import (
        _compute_prefill_metadata_kernel,
        _compute_swa_indices_and_lens_kernel,
    )
    from vllm.v1.attention.ops import rocm_aiter_mla_sparse as ra

    g = torch.Generator().manual_seed(5)
    H, W, ratio, swa_page, comp_page = 16, 128, 128, 64, 2
    comp_stride = 1728  # 2 x 584 bytes padded to the 576-byte page alignment
    scale = D ** -0.5
    maxc = 128  # compressed index width (max_model_len 16384)

    def caches(n_swa_pages: int, n_comp_pages: int):
        swa = torch.zeros(n_swa_pages, swa_page * 584, dtype=torch.uint8)
        comp = torch.zeros(n_comp_pages, comp_stride, dtype=torch.uint8)
        return swa, comp

    def as_pages(raw: torch.Tensor, block: int) -> torch.Tensor:
        return raw.as_strided((raw.shape[0], block, 584), (raw.stride(0), 584, 1))

    sinks = {
        "random": torch.randn(H, generator=g),
        "neginf": torch.full((H,), -float("inf")),
        "none": None,
    }

    # ---------------- decode: 4 requests, MTP-style consecutive tokens ----
    # r0 crosses a compression boundary between its tokens, r1 fills the
    # window exactly, r2 is window-only, r3's second token is padding.
    q_lens = [3, 3, 1, 2]
    seq_lens = torch.tensor([1025, 130, 5, 300], dtype=torch.int32)
    R_ = len(q_lens)
    qsl = torch.tensor(np.concatenate([[0], np.cumsum(q_lens)]), dtype=torch.int32)
    T = int(qsl[-1])
    t2r = torch.repeat_interleave(torch.arange(R_, dtype=torch.int32), torch.tensor(q_lens))
    positions = torch.cat([torch.arange(int(s) - q, int(s)) for s, q in zip(seq_lens, q_lens)]).to(torch.int64)
    n_swa_pages, n_comp_pages = 24, 8
    swa_bt = torch.stack([torch.randperm(n_swa_pages, generator=g)[:17] for _ in range(R_)]).to(torch.int32)
    comp_bt = torch.stack([torch.randperm(n_comp_pages, generator=g)[:8] for _ in range(R_)]).to(torch.int32)
    slot_mapping = swa_bt[t2r.long(), positions // swa_page].long() * swa_page + positions % swa_page
    slot_mapping[T - 1] = -1  # padding token
    is_valid = slot_mapping >= 0
    swa_idx = torch.full((T, 1, W), -1, dtype=torch.int32)
    swa_lens = torch.zeros(T, dtype=torch.int32)
    _compute_swa_indices_and_lens_kernel[(T,)](
        swa_idx, swa_idx.stride(0), swa_lens, W, qsl, seq_lens, t2r, is_valid, swa_bt,
        swa_bt.stride(0), swa_page, TRITON_BLOCK_SIZE=1024)
    gdec = torch.full((T, maxc), -1, dtype=torch.int32)
    dlens = torch.zeros(T, dtype=torch.int32)
    plocal = torch.full((1, maxc), -1, dtype=torch.int32)
    build_c128a_topk_metadata(positions, ratio, T, t2r, comp_bt, comp_page, slot_mapping, gdec, dlens,
                              plocal, max_compressed_tokens=maxc)
    swa_raw, comp_raw = caches(n_swa_pages, n_comp_pages)
    sidx = swa_idx[:, 0].numpy()
    _fill_rows(swa_raw, np.concatenate([sidx[t, : int(swa_lens[t])] for t in range(T)]), swa_page, g)
    gd = gdec.numpy()
    _fill_rows(comp_raw, np.concatenate([gd[t, : int(dlens[t])] for t in range(T)]), comp_page, g)
    q = torch.randn(T, H, D, generator=g).bfloat16()

    main_i, main_p = ra.build_ragged_indices_from_dense(swa_idx[:, 0], swa_lens,
                                                        num_rows=n_swa_pages * swa_page)
    extra_i, extra_p = ra.build_ragged_indices_from_dense(gdec, dlens, num_rows=n_comp_pages * comp_page)
    main_cache, extra_cache = as_pages(swa_raw, swa_page), as_pages(comp_raw, comp_page)
    outs = {}
    for name, sink in sinks.items():
        out = torch.empty(T, H, D, dtype=torch.bfloat16)
        ra._sparse_attn_decode_ragged_kernel[(T, triton_cdiv(H, 16))](
            q, main_cache, main_i, main_p, extra_cache, extra_i, extra_p,
            sink if sink is not None else torch.empty(1), out,
            q.stride(0), q.stride(1), out.stride(0), out.stride(1),
            main_cache.stride(0), extra_cache.stride(0),
            main_cache.shape[0] * main_cache.shape[1], extra_cache.shape[0] * extra_cache.shape[1],
            main_cache.shape[1], extra_cache.shape[1], scale, H,
            HAS_ATTN_SINK=sink is not None, HAS_EXTRA=True, NOPE_DIM=NOPE, NOPE_BLOCK=512,
            ROPE_DIM=R, IS_FNUZ=False, BLOCK_H=16, BLOCK_K=16, num_warps=8)
        outs[f"out_{name}"] = _bf16_bits(out)
    save("sparse_decode_d512", q=_bf16_bits(q), positions=positions, query_start_loc=qsl,
         seq_lens=seq_lens, swa_block_table=swa_bt, comp_block_table=comp_bt, slot_mapping=slot_mapping,
         swa_indices=swa_idx[:, 0], swa_lens=swa_lens, comp_indices=gdec, comp_lens=dlens,
         swa_cache=swa_raw, comp_cache=comp_raw, sink=sinks["random"], scale=np.float64(scale), **outs)

    # ---------------- prefill: 3 chunks, window-only / boundary-crossing ----
    chunks = [(0, 6), (1020, 6), (380, 5)]  # (prior context, chunk tokens)
    q_lens = [c for _, c in chunks]
    seq_lens = torch.tensor([p + c for p, c in chunks], dtype=torch.int32)
    R_ = len(chunks)
    qsl = torch.tensor(np.concatenate([[0], np.cumsum(q_lens)]), dtype=torch.int32)
    T = int(qsl[-1])
    t2r = torch.repeat_interleave(torch.arange(R_, dtype=torch.int32), torch.tensor(q_lens))
    positions = torch.cat([torch.arange(int(s) - q, int(s)) for s, q in zip(seq_lens, q_lens)]).to(torch.int64)
    swa_bt = torch.stack([torch.randperm(n_swa_pages, generator=g)[:17] for _ in range(R_)]).to(torch.int32)
    comp_bt = torch.stack([torch.randperm(n_comp_pages, generator=g)[:8] for _ in range(R_)]).to(torch.int32)
    slot_mapping = swa_bt[t2r.long(), positions // swa_page].long() * swa_page + positions % swa_page
    gather_lens = torch.empty(R_, dtype=torch.int32)
    _compute_prefill_metadata_kernel[(1,)](gather_lens, seq_lens, qsl, R_, 0, W, BLOCK_SIZE=4)
    gdec = torch.full((1, maxc), -1, dtype=torch.int32)
    dlens = torch.zeros(1, dtype=torch.int32)
    plocal = torch.full((T, maxc), -1, dtype=torch.int32)
    build_c128a_topk_metadata(positions, ratio, 0, t2r, comp_bt, comp_page, slot_mapping, gdec, dlens,
                              plocal, max_compressed_tokens=maxc)
    swa_raw, comp_raw = caches(n_swa_pages, n_comp_pages)
    # rows the gather reads: the last gather_len positions of each request,
    # and every compressed entry below seq_len // ratio
    wslots, cslots = [], []
    for r in range(R_):
        s, gl = int(seq_lens[r]), int(gather_lens[r])
        pos = np.arange(s - gl, s)
        wslots.append(swa_bt[r].numpy()[pos // swa_page].astype(np.int64) * swa_page + pos % swa_page)
        ce = np.arange(s // ratio)
        cslots.append(comp_bt[r].numpy()[ce // comp_page].astype(np.int64) * comp_page + ce % comp_page)
    _fill_rows(swa_raw, np.concatenate(wslots), swa_page, g)
    _fill_rows(comp_raw, np.concatenate(cslots), comp_page, g)
    q = torch.randn(T, H, D, generator=g).bfloat16()
    N = maxc
    M = N + W + T
    kv = torch.zeros(R_, M, D, dtype=torch.bfloat16)
    dequantize_and_gather_k_cache_triton(kv, as_pages(comp_raw, comp_page), seq_lens // ratio, None, comp_bt,
                                         comp_page, offset=0)
    dequantize_and_gather_k_cache_triton(kv, as_pages(swa_raw, swa_page), seq_lens, gather_lens, swa_bt,
                                         swa_page, offset=N)
    comb, comb_lens = combine_topk_swa_indices(plocal, qsl, seq_lens, gather_lens, W, ratio, maxc, M, N)
    rag_i, rag_p = ra.build_ragged_indices_from_dense(comb, comb_lens, num_rows=R_ * M)
    kv2 = kv.view(-1, D)
    outs = {}
    for name, sink in sinks.items():
        out = torch.empty(T, H, D, dtype=torch.bfloat16)
        ra._sparse_attn_prefill_ragged_kernel[(T, triton_cdiv(H, 16))](
            q, kv2, rag_i, rag_p, sink if sink is not None else torch.empty(1), out,
            q.stride(0), q.stride(1), q.stride(2), kv2.stride(0), kv2.stride(1),
            out.stride(0), out.stride(1), out.stride(2), H, D, kv2.shape[0], scale,
            HAS_ATTN_SINK=sink is not None, BLOCK_H=16, BLOCK_D=512, BLOCK_K=16, num_warps=8)
        outs[f"out_{name}"] = _bf16_bits(out)
    save("sparse_prefill_d512", q=_bf16_bits(q), positions=positions, query_start_loc=qsl, seq_lens=seq_lens,
         token_to_req=t2r, swa_block_table=swa_bt, comp_block_table=comp_bt, gather_lens=gather_lens,
         combined=comb, combined_lens=comb_lens, swa_cache=swa_raw, comp_cache=comp_raw,
         sink=sinks["random"], scale=np.float64(scale), **outs)


def triton_cdiv(a: int, b: int) -> int:
    return (a + b - 1) // b


def main() -> None:
    patch_interpreter()
    g = torch.Generator().manual_seed(0)
    which = sys.argv[1:] or ["insert", "compressor", "metadata", "output", "attention"]
    if "insert" in which:
        gen_insert_and_gather(g)
    if "compressor" in which:
        gen_compressor(g)
    if "compressor_blocks" in which:
        gen_compressor_blocks(torch.Generator().manual_seed(11))
    if "metadata" in which:
        gen_metadata(g)
    if "output" in which:
        gen_norm_and_output(g)
    if "attention" in which:
        gen_attention()


if __name__ == "__main__":
    main()
