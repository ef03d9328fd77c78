"""GPU parity of the head_dim-512 sparse attention kernels against golden
vectors from the reference's own kernels.

``tests/golden/sparse_{decode,prefill}_d512.npz`` hold the inputs and
outputs of vLLM's readable DeepSeek-V4 sparse attention
(``_sparse_attn_decode_ragged_kernel`` / ``_sparse_attn_prefill_ragged_kernel``
in ``vllm/v1/attention/ops/rocm_aiter_mla_sparse.py``), run by
``tests/golden/make_golden.py`` under the Triton interpreter on the fp8
caches and the builders' index tables.  The CUDA kernels read the same cache
bytes and tables through the C ABI.

Tolerance (the parity bar for floating point): ``max |err| <= 2e-2`` and
relative L2 ``<= 5e-3`` against the golden bf16 output.
"""

import numpy as np
import pytest
import torch

from golden_io import load

pytestmark = pytest.mark.gpu

DEV = "cuda"
MAX_ABS, MAX_REL_L2 = 2e-2, 5e-3
D = 512


def _bf16(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16).to(DEV)


def _t(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def _sink(g, mode):
    if mode == "random":
        return _t(g["sink"].astype(np.float32))
    if mode == "neginf":
        return torch.full((g["sink"].shape[0],), -float("inf"), device=DEV)
    return None


def _check(out: torch.Tensor, ref_bits: np.ndarray) -> None:
    got = out.float().cpu().numpy().astype(np.float64)
    ref = (ref_bits.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    assert np.isfinite(got).all()
    err = np.abs(got - ref)
    rel = np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30)
    assert err.max() <= MAX_ABS and rel <= MAX_REL_L2, (err.max(), rel)


@pytest.mark.parametrize("sink", ["random", "neginf", "none"])
@pytest.mark.parametrize("layout", ["per_token_2_splits", "mtp_groups_scheduled"])
def test_decode_d512_matches_reference_kernel(sink, layout):
    from vllm_ernie_b200 import ops

    g = load("sparse_decode_d512")
    q = _bf16(g["q"])
    swa, comp = _t(g["swa_cache"]), _t(g["comp_cache"])
    si, sl = _t(g["swa_indices"]), _t(g["swa_lens"])
    ci, cl = _t(g["comp_indices"]), _t(g["comp_lens"])
    kw = {}
    if layout == "per_token_2_splits":
        kw = dict(num_splits=2)
    else:
        # a request's consecutive tokens share a group; a group is all valid
        # tokens or all padding (the entry points' contract), so the padding
        # token of the last request forms its own group
        qsl = g["query_start_loc"]
        starts = np.concatenate([qsl[:-1], [qsl[-1] - 1, qsl[-1]]]).astype(np.int32)
        assert g["swa_lens"][starts[-2]] == 0 and (g["swa_lens"][:starts[-2]] > 0).all()
        gs = _t(starts)
        max_items = 16
        sched = ops.decode_schedule(gs, q.shape[0], sl, cl, max_items)
        kw = dict(group_starts=gs, max_group_tokens=int(np.diff(starts).max()), schedule=sched,
                  max_items=max_items)
    out = ops.sparse_decode(q, swa, 64, si, sl, comp, 2, ci, cl, float(g["scale"]), _sink(g, sink), **kw)
    torch.cuda.synchronize()
    _check(out, g[f"out_{sink}"])
    empty = g["swa_lens"] == 0
    assert empty.any() and torch.count_nonzero(out[torch.from_numpy(empty).to(DEV)]).item() == 0
    assert ops.device_error() == 0


@pytest.mark.parametrize("sink", ["random", "neginf", "none"])
def test_prefill_d512_matches_reference_kernel(sink):
    from vllm_ernie_b200 import ops

    g = load("sparse_prefill_d512")
    q = _bf16(g["q"])
    out = ops.sparse_prefill(q, _t(g["query_start_loc"]), _t(g["seq_lens"]), _t(g["swa_cache"]), 64,
                             _t(g["swa_block_table"]), _t(g["comp_cache"]), 2, _t(g["comp_block_table"]), 128, 128,
                             float(g["scale"]), _sink(g, sink))
    torch.cuda.synchronize()
    _check(out, g[f"out_{sink}"])
    assert ops.device_error() == 0
