"""Head-sharded tensor parallelism of the drop-in module over NCCL at TP =
2, 4 and 8: each rank holds 1/TP of the heads and output groups; the VHA
low-rank term and the ``wo_b`` output are all-reduced
(``E/nvidia/attention.py:121-157,466-469``).  Shape: hidden 2048, 32 heads x
128 in 8 output groups of rank 512 (every TP size divides the groups, and
the block-FP8 variant's group width and ``wo_b`` input tile its 128 x 128
blocks and 512-wide scale packs on every rank).  bf16 and block-FP8
``wo_a``/``wo_b``.  The layer output of every rank after the all-reduce must
match the whole-layer CPU oracle within the tolerance of the single-GPU
module test (relative L2 3e-2, max |err| <= 3e-2 x max |ref|; 6e-2 on the
block-FP8 path, whose two e4m3 quant points turn small upstream differences
into whole e4m3 steps), for a prefill step and an ECHO/MTP decode step, and
all ranks must hold the same output.
Skipped when the box has fewer GPUs than ranks.
"""

import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle.layer import HCALayerOracle, HCAShape, random_weights

pytestmark = pytest.mark.gpu

PREFIX = "model.layers.0.self_attn"
MAX_LEN = 1152
STEPS = [  # (query_start_loc, seq_lens, speculative tokens)
    (np.array([0, 1024, 1664]), np.array([1024, 640]), 0),
    (np.array([0, 3, 6]), np.array([1027, 643]), 2),
]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _hidden_states():
    g = torch.Generator().manual_seed(1)
    return [torch.randn(int(qsl[-1]), 2048, generator=g).to(torch.bfloat16) for qsl, _, _ in STEPS]


SHAPE = HCAShape(heads=32, o_groups=8, o_lora=512)


def _weights(fp8: bool):
    """Checkpoint tensors and the oracle's weights (dequantised block FP8)."""
    from test_gpu_module import _block_fp8

    weights = random_weights(SHAPE, seed=0)
    ckpt = {k: torch.from_numpy(v) for k, v in weights.items()}
    if fp8:
        fp8_ckpt, weights = _block_fp8(weights)
        ckpt.update(fp8_ckpt)
    return ckpt, weights


def _worker(rank, world, port, fp8, out):
    from test_gpu_module import _metadata
    from vllm_ernie_b200 import attention as A
    from vllm_ernie_b200.forward_context import set_forward_context

    torch.cuda.set_device(rank)
    dev = f"cuda:{rank}"
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=120))
    try:
        shape = SHAPE
        ckpt, weights = _weights(fp8)
        layout = HCALayerOracle(shape, weights, max_len=MAX_LEN, num_reqs=2, emulate_quant=True)  # page tables
        cfg = A.Ernie5_5HCAConfig(hidden_size=2048, num_hidden_layers=2, num_attention_heads=32, head_dim=128,
                                  q_lora_rank=512, qk_rope_head_dim=64, o_groups=8, o_lora_rank=512,
                                  hybrid_mla_num_attention_heads=32, num_nextn_predict_layers=0,
                                  compress_rope_theta=shape.rope_theta)
        quant = A.block_fp8_quant_config() if fp8 else None
        layer = A.Ernie5_5HCAAttention(A.make_vllm_config(cfg, max_model_len=MAX_LEN, num_speculative_tokens=2,
                                                          quant_config=quant),
                                       prefix=PREFIX, tp_group=dist.group.WORLD).to(dev)
        assert layer.n_local_heads == 32 // world and layer.fp8_output == fp8
        layer.load_weights(list(ckpt.items()))
        layer.process_weights_after_loading()
        spec = layer.get_kv_cache_spec()
        swa = torch.zeros(layout.swa_cache.shape, dtype=torch.uint8, device=dev)
        comp = torch.zeros((layout.comp_cache.shape[0], spec["compressed"].page_size_bytes), dtype=torch.uint8,
                           device=dev)
        state = torch.zeros(layout.state.shape, dtype=torch.float32, device=dev)
        layer.bind_kv_cache(swa, comp, state)
        # _metadata builds on the default "cuda" device: this rank's
        with torch.cuda.device(rank):
            for step, ((qsl, seq_lens, spec_tokens), hidden) in enumerate(zip(STEPS, _hidden_states())):
                positions = np.concatenate([np.arange(seq_lens[b] - (qsl[b + 1] - qsl[b]), seq_lens[b])
                                            for b in range(len(seq_lens))])
                md, pos_d = _metadata(layer, layout.swa_bt, layout.comp_bt, layout.state_bt, qsl, seq_lens, positions,
                                      spec_tokens)
                with set_forward_context(md):
                    y = layer(pos_d, hidden.to(dev))
                torch.cuda.synchronize()
                out[(rank, step)] = y.float().cpu().numpy()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("fp8", [False, True])
@pytest.mark.parametrize("world", [2, 4, 8])
def test_module_tp_nccl_matches_layer_oracle(world, fp8):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    _, weights = _weights(fp8)
    oracle = HCALayerOracle(SHAPE, weights, max_len=MAX_LEN, num_reqs=2, emulate_quant=True, fp8_output=fp8)
    refs = [oracle.forward(h.float().numpy(), qsl, seq_lens) for (qsl, seq_lens, _), h in zip(STEPS, _hidden_states())]
    with mp.get_context("spawn").Manager() as manager:
        out = manager.dict()
        mp.spawn(_worker, args=(world, _free_port(), fp8, out), nprocs=world)
        got = {k: v for k, v in out.items()}
    assert sorted(got) == [(r, k) for r in range(world) for k in range(len(STEPS))]
    for (rank, step), y in sorted(got.items()):
        ref = refs[step]
        assert np.isfinite(y).all()
        err = np.abs(y - ref)
        rel = np.linalg.norm(y - ref) / np.linalg.norm(ref)
        tol = 6e-2 if fp8 else 3e-2
        assert rel <= tol, (rank, step, rel, err.max())
        assert err.max() <= tol * np.abs(ref).max(), (rank, step, rel, err.max())
    # every rank holds the same all-reduced output
    for step in range(len(STEPS)):
        for rank in range(1, world):
            np.testing.assert_allclose(got[(0, step)], got[(rank, step)], rtol=0, atol=1e-6)
