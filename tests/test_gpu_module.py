"""The drop-in module on the GPU: ``Ernie5_5HCAAttention.forward`` through the
backend's metadata builders and the forward context, against the whole-layer
CPU oracle (config 1: hidden 2048, 16 heads x 128, and the same with the
model's head_dim 512; prefill of 1024 and 640 tokens from an empty cache, then
an ECHO/MTP decode step of 3 tokens per request on the caches the prefill
wrote).

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


@pytest.mark.parametrize("head_dim", [128, 512])
def test_module_forward_prefill_then_decode_matches_layer_oracle(head_dim):
    """head_dim 128 is config 1; 512 is the model's own head size (the CTA-pair
    attention kernel, head_dim-512 cache rows, compressor and output path)."""
    from vllm_ernie_b200 import attention as A
    from vllm_ernie_b200.cache_layout import page_bytes
    from vllm_ernie_b200.forward_context import set_forward_context

    shape = HCAShape(head_dim=head_dim)
    weights = random_weights(shape, seed=0)
    max_len = 1152
    oracle = HCALayerOracle(shape, weights, max_len=max_len, num_reqs=2, emulate_quant=True)

    cfg = A.Ernie5_5HCAConfig(hidden_size=2048, num_hidden_layers=2, num_attention_heads=16, head_dim=head_dim,
                              q_lora_rank=512, qk_rope_head_dim=64, o_groups=4, o_lora_rank=64,
                              hybrid_mla_num_attention_heads=16, num_nextn_predict_layers=0,
                              compress_rope_theta=shape.rope_theta)
    layer = A.Ernie5_5HCAAttention(A.make_vllm_config(cfg, max_model_len=max_len, num_speculative_tokens=2),
                                   prefix=PREFIX).to(DEV)
    loaded = layer.load_weights([(k, torch.from_numpy(v)) for k, v in weights.items()])
    assert loaded == set(weights)
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
        torch.cuda.synchronize()
        got = y.float().cpu().numpy()
        assert np.isfinite(got).all()
        err = np.abs(got - ref)
        rel = np.linalg.norm(got - ref) / np.linalg.norm(ref)
        assert rel <= 3e-2, (rel, err.max())
        assert err.max() <= 3e-2 * np.abs(ref).max(), (rel, err.max(), np.abs(ref).max())
