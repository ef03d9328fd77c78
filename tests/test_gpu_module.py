"""The drop-in module on the GPU: ``Ernie5_5HCAAttention.forward`` through the
backend's metadata builders and the forward context, against the whole-layer
CPU oracle (config 1: hidden 2048, 16 heads x 128, and the same with the
model's head_dim 512; prefill of 1024 and 640 tokens from an empty cache, then
an ECHO/MTP decode step of 3 tokens per request on the caches the prefill
wrote, a verify step after partial acceptance that writes the rejected
drafts' positions again, and a one-token step).

Tolerance of the block-FP8 output path: relative L2 and max |err| / max
|ref| <= 6e-2.  Its two 1x128 e4m3 quant points (wo_a's and wo_b's inputs)
turn the ~0.5% attention-output difference into whole e4m3 steps (12.5%) on
the few percent of elements that sit near a rounding boundary, about 2.5%
of the output per quant point.  The chain after the attention is held to
relative L2 1e-2 on identical inputs (test_fp8_output_chain_matches_oracle).

Tolerance: the layer output (after wo_b) against the oracle's emulated
evaluation (the FP8/UE8M0 cache and bf16 roundings of the reference kernels)
within relative L2 3e-2 and max |err| <= 3e-2 x max |ref|.  The attention core
itself is held to the tighter bar (max |err| <= 2e-2, relative L2 <= 5e-3) in
test_gpu_attention.py; at the layer output five bf16 GEMMs, the bf16 gate and
FP8 rounding flips of cache rows (one e4m3 step where the GPU's and the
oracle's fp32 values straddle a rounding boundary) add up to about 1.5%.  The
oracle's own emulated and all-fp32 evaluations differ by up to 5%.
"""

import numpy as np
import pytest
import torch

from oracle.layer import HCALayerOracle, HCAShape, random_weights

pytestmark = pytest.mark.gpu

DEV = "cuda"
PREFIX = "model.layers.0.self_attn"


def _metadata(layer, swa_bt, comp_bt, st_bt, qsl, seq_lens, positions, spec_tokens):
    from vllm_ernie_b200 import ops
    from vllm_ernie_b200.backend import (C128AMetadataBuilder, CommonAttentionMetadata, CompressorMetadataBuilder,
                                         HCAStepMetadata, SWAMetadataBuilder)

    n = int(qsl[-1])
    q_lens = np.diff(qsl)
    qsl_d = torch.tensor(qsl, dtype=torch.int32, device=DEV)
    sl_d = torch.tensor(seq_lens, dtype=torch.int32, device=DEV)
    pos_d = torch.tensor(positions, dtype=torch.int64, device=DEV)

    def common(bt, page):
        bt_d = torch.tensor(bt, dtype=torch.int32, device=DEV)
        slot = ops.slot_mapping(qsl_d, sl_d, bt_d, page, n)
        return CommonAttentionMetadata(query_start_loc=qsl_d, query_start_loc_cpu=torch.tensor(qsl, dtype=torch.int32),
                                       seq_lens=sl_d, num_reqs=len(seq_lens), num_actual_tokens=n,
                                       max_query_len=int(q_lens.max()), block_table_tensor=bt_d, slot_mapping=slot,
                                       positions=pos_d, max_seq_len=int(max(seq_lens)))

    cm_swa, cm_comp, cm_st = common(swa_bt, 64), common(comp_bt, 256), common(st_bt, 8)
    swa = SWAMetadataBuilder(128, 4096, layer.n_local_heads, num_speculative_tokens=spec_tokens, device=DEV,
                             head_dim=layer.head_dim).build(0, cm_swa)
    c128 = C128AMetadataBuilder(layer.max_model_len, 4096, num_speculative_tokens=spec_tokens, device=DEV).build(
        0, cm_comp, cm_swa.slot_mapping)
    comp = CompressorMetadataBuilder(4096, device=DEV).build(0, cm_st)
    return HCAStepMetadata(swa, c128, comp).as_forward_context([PREFIX]), pos_d


def _block_fp8(weights: dict, names=("wo_a.weight", "wo_b.weight")):
    """Block-FP8 copies of ``names`` (e4m3 + ``weight_scale_inv``, as a 128 x 128
    block-FP8 checkpoint holds them) and the dequantised fp32 values."""
    from vllm_ernie_b200.ops import quantize_weight_block_fp8

    ckpt, deq = {}, dict(weights)
    for name in names:
        q, sc = quantize_weight_block_fp8(torch.from_numpy(weights[name]))
        ckpt[name], ckpt[name + "_scale_inv"] = q, sc
        full = sc.repeat_interleave(128, 0)[: q.shape[0]].repeat_interleave(128, 1)
        deq[name] = (q.float() * full).numpy()
    return ckpt, deq


@pytest.mark.parametrize("head_dim,fp8,aux", [(128, False, False), (512, False, False), (128, True, False),
                                              (512, True, False), (128, True, True)])
def test_module_forward_prefill_then_decode_matches_layer_oracle(head_dim, fp8, aux):
    """head_dim 128 is config 1; 512 is the model's own head size (the CTA-pair
    attention kernel, head_dim-512 cache rows, compressor and output path).
    ``fp8``: a 128 x 128 block-FP8 checkpoint (rank-128 groups), so the module
    runs the reference's FP8 output path (fused VHA + quant on the decode
    step, the tcgen05 FP8 GEMMs for wo_a and gated wo_b), against the
    oracle's FP8 output path on the same block-FP8 weights.  ``aux``: the
    model's two aux streams (kv_score beside fused_wqa_wkv, the gate beside
    attention); the output must equal the serial run's bit for bit."""
    from vllm_ernie_b200 import attention as A
    from vllm_ernie_b200.cache_layout import page_bytes
    from vllm_ernie_b200.forward_context import set_forward_context

    shape = HCAShape(head_dim=head_dim, o_lora=128 if fp8 else 64)
    weights = random_weights(shape, seed=0)
    ckpt = {k: torch.from_numpy(v) for k, v in weights.items()}
    if fp8:
        fp8_ckpt, weights = _block_fp8(weights)
        ckpt.update(fp8_ckpt)
    max_len = 1152
    oracle = HCALayerOracle(shape, weights, max_len=max_len, num_reqs=2, emulate_quant=True, fp8_output=fp8)

    cfg = A.Ernie5_5HCAConfig(hidden_size=2048, num_hidden_layers=2, num_attention_heads=16, head_dim=head_dim,
                              q_lora_rank=512, qk_rope_head_dim=64, o_groups=4, o_lora_rank=shape.o_lora,
                              hybrid_mla_num_attention_heads=16, num_nextn_predict_layers=0,
                              compress_rope_theta=shape.rope_theta)
    quant = A.block_fp8_quant_config() if fp8 else None
    streams = [torch.cuda.Stream(), torch.cuda.Stream()] if aux else None
    layer = A.Ernie5_5HCAAttention(A.make_vllm_config(cfg, max_model_len=max_len, num_speculative_tokens=2,
                                                      quant_config=quant), prefix=PREFIX,
                                   aux_stream_list=streams).to(DEV)
    assert layer.fp8_output == fp8
    loaded = layer.load_weights(list(ckpt.items()))
    assert loaded == set(ckpt)
    layer.process_weights_after_loading()
    # the oracle's page numbering (contiguous pages per request); the page
    # strides are the engine's: the compressed cache's pages (388 bytes at
    # head_dim 128, 1168 at 512) padded to the 576-byte alignment every HCA
    # cache spec uses
    cache_spec = layer.get_kv_cache_spec()
    swa = torch.zeros(oracle.swa_cache.shape, dtype=torch.uint8, device=DEV)
    comp = torch.zeros((oracle.comp_cache.shape[0], cache_spec["compressed"].page_size_bytes), dtype=torch.uint8,
                       device=DEV)
    state = torch.zeros(oracle.state.shape, dtype=torch.float32, device=DEV)
    assert swa.shape[1] == page_bytes(64, head_dim, 64) and comp.shape[1] % 576 == 0
    assert comp.shape[1] >= page_bytes(2, head_dim, 64)
    layer.bind_kv_cache(swa, comp, state)

    g = torch.Generator().manual_seed(1)
    steps = [  # (query_start_loc, seq_lens, speculative tokens)
        (np.array([0, 1024, 1664]), np.array([1024, 640]), 0),   # prefill from an empty cache
        (np.array([0, 3, 6]), np.array([1027, 643]), 2),         # decode, 3 tokens per request
        # ECHO/MTP verify after partial acceptance: request 0 kept 2 of its 3
        # tokens, request 1 kept 1, so the rejected drafts' positions (1026;
        # 641, 642) are written again with new values beside the next ones
        (np.array([0, 3, 6]), np.array([1029, 644]), 2),
        (np.array([0, 1, 2]), np.array([1030, 645]), 2),         # one token per request (a draft step)
    ]
    for qsl, seq_lens, spec in steps:
        n = int(qsl[-1])
        hidden = torch.randn(n, 2048, generator=g)
        hidden_bf16 = hidden.to(torch.bfloat16)
        ref = oracle.forward(hidden_bf16.float().numpy(), qsl, seq_lens)
        positions = np.concatenate([np.arange(seq_lens[b] - (qsl[b + 1] - qsl[b]), seq_lens[b])
                                    for b in range(len(seq_lens))])
        md, pos_d = _metadata(layer, oracle.swa_bt, oracle.comp_bt, oracle.state_bt, qsl, seq_lens, positions, spec)
        with set_forward_context(md):
            y = layer(pos_d, hidden_bf16.to(DEV))
            if aux:
                # the same step serially (the cache writes repeat the same bytes)
                layer.aux_stream_list = None
                y_serial = layer(pos_d, hidden_bf16.to(DEV))
                layer.aux_stream_list = streams
                torch.cuda.synchronize()
                assert torch.equal(y, y_serial)
        torch.cuda.synchronize()
        got = y.float().cpu().numpy()
        assert np.isfinite(got).all()
        err = np.abs(got - ref)
        rel = np.linalg.norm(got - ref) / np.linalg.norm(ref)
        tol = 6e-2 if fp8 else 3e-2
        assert rel <= tol, (rel, err.max())
        assert err.max() <= tol * np.abs(ref).max(), (rel, err.max(), np.abs(ref).max())


@pytest.mark.parametrize("head_dim,t", [(128, 6), (128, 300), (512, 37)])
def test_fp8_output_chain_matches_oracle(head_dim, t):
    """The module's FP8 output path on one bf16 attention output: VHA +
    inverse RoPE + quant, grouped wo_a, sigmoid gate + quant, wo_b, against
    the oracle's on the same input (differences: fp32 summation order only)."""
    from vllm_ernie_b200 import attention as A
    from vllm_ernie_b200 import ops

    shape = HCAShape(head_dim=head_dim, o_lora=128)
    fp8_ckpt, weights = _block_fp8(random_weights(shape, seed=3))
    ckpt = {k: torch.from_numpy(v) for k, v in random_weights(shape, seed=3).items()}
    ckpt.update(fp8_ckpt)
    oracle = HCALayerOracle(shape, weights, max_len=1152, num_reqs=2, emulate_quant=True, fp8_output=True)
    cfg = A.Ernie5_5HCAConfig(hidden_size=2048, num_hidden_layers=2, num_attention_heads=16, head_dim=head_dim,
                              q_lora_rank=512, qk_rope_head_dim=64, o_groups=4, o_lora_rank=128,
                              hybrid_mla_num_attention_heads=16, num_nextn_predict_layers=0,
                              compress_rope_theta=shape.rope_theta)
    layer = A.Ernie5_5HCAAttention(A.make_vllm_config(cfg, max_model_len=1152,
                                                      quant_config=A.block_fp8_quant_config()), prefix=PREFIX).to(DEV)
    layer.load_weights(list(ckpt.items()))
    layer.process_weights_after_loading()
    g = torch.Generator().manual_seed(t)
    o = torch.randn(t, 16, head_dim, generator=g).to(torch.bfloat16)
    gate = torch.randn(t, 4 * 128, generator=g).to(torch.bfloat16)
    pos = torch.randint(0, 1100, (t,), generator=g)
    x8, xs = ops.vha_inv_rope_fp8_quant(o.to(DEV), layer.vha.m_bf16, pos.to(DEV), layer.cos_sin_cache, 4,
                                        head_dim - 64, 64)
    y = layer._output_fp8(x8, xs, gate.to(DEV))
    torch.cuda.synchronize()
    ref = oracle.output_fp8(o.float().numpy(), gate.float().numpy(), pos.numpy())
    got = y.float().cpu().numpy()
    rel = np.linalg.norm(got - ref) / np.linalg.norm(ref)
    assert np.isfinite(got).all() and rel <= 1e-2, rel
    assert ops.device_error() == 0
