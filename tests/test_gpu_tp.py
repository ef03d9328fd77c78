"""Head-sharded tensor parallelism of the drop-in module over NCCL, on two
GPUs: each rank holds half of config 1's heads and output groups; the VHA
low-rank term and the ``wo_b`` output are all-reduced
(``E/nvidia/attention.py:121-157,466-469``).  The layer output of both
ranks after the all-reduce must match the whole-layer CPU oracle within the
tolerance of the single-GPU module test (relative L2 3e-2, max |err| <=
3e-2 x max |ref|), for a prefill step and an ECHO/MTP decode step.  Skipped
with fewer than two GPUs.
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


def _worker(rank, world, port, out):
    from test_gpu_module import _metadata
    from vllm_ernie_b200 import attention as A
    from vllm_ernie_b200.forward_context import set_forward_context

    torch.cuda.set_device(rank)
    dev = f"cuda:{rank}"
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=120))
    try:
        shape = HCAShape()
        weights = random_weights(shape, seed=0)
        layout = HCALayerOracle(shape, weights, max_len=MAX_LEN, num_reqs=2, emulate_quant=True)  # page tables
        cfg = A.Ernie5_5HCAConfig(hidden_size=2048, num_hidden_layers=2, num_attention_heads=16, head_dim=128,
                                  q_lora_rank=512, qk_rope_head_dim=64, o_groups=4, o_lora_rank=64,
                                  hybrid_mla_num_attention_heads=16, num_nextn_predict_layers=0,
                                  compress_rope_theta=shape.rope_theta)
        layer = A.Ernie5_5HCAAttention(A.make_vllm_config(cfg, max_model_len=MAX_LEN, num_speculative_tokens=2),
                                       prefix=PREFIX, tp_group=dist.group.WORLD).to(dev)
        assert layer.n_local_heads == 16 // world
        layer.load_weights([(k, torch.from_numpy(v)) for k, v in weights.items()])
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


def test_module_tp2_nccl_matches_layer_oracle():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    shape = HCAShape()
    oracle = HCALayerOracle(shape, random_weights(shape, seed=0), max_len=MAX_LEN, num_reqs=2, emulate_quant=True)
    refs = [oracle.forward(h.float().numpy(), qsl, seq_lens) for (qsl, seq_lens, _), h in zip(STEPS, _hidden_states())]
    world = 2
    with mp.get_context("spawn").Manager() as manager:
        out = manager.dict()
        mp.spawn(_worker, args=(world, _free_port(), out), nprocs=world)
        got = {k: v for k, v in out.items()}
    assert sorted(got) == [(r, k) for r in range(world) for k in range(len(STEPS))]
    for (rank, step), y in sorted(got.items()):
        ref = refs[step]
        assert np.isfinite(y).all()
        err = np.abs(y - ref)
        rel = np.linalg.norm(y - ref) / np.linalg.norm(ref)
        assert rel <= 3e-2, (rank, step, rel, err.max())
        assert err.max() <= 3e-2 * np.abs(ref).max(), (rank, step, rel, err.max())
    # every rank holds the same all-reduced output
    for step in range(len(STEPS)):
        np.testing.assert_allclose(got[(0, step)], got[(1, step)], rtol=0, atol=1e-6)
