"""The allocation-free decode entry point, hca_sparse_decode_noalloc.

Some callers of this library cannot allocate device memory for the split-K
workspace of hca_sparse_decode: a serving runtime whose caching allocator owns
all device memory and must not be bypassed, or one that fixes its memory
budget before it starts serving.  hca_sparse_decode_noalloc keeps the partials
in a static device array instead.  These tests check, through the C ABI, that
two calls in a row give what hca_sparse_decode gives with a caller-supplied
workspace (the second call runs on top of the first call's leftovers in the
shared array), and that a problem larger than the array is refused.

This file is collected last on purpose: if it fails, a run that stops at the
first failure has already run every other test.
"""

import numpy as np
import pytest
import torch

from vllm_ernie_b200 import _lib

MAX_ABS, MAX_REL_L2 = 2e-2, 5e-3  # the parity tolerance of the attention tests
HCA_E_TOO_LARGE = -5


def _close(got: torch.Tensor, ref: torch.Tensor):
    g = got.float().cpu().numpy().astype(np.float64)
    r = ref.float().cpu().numpy().astype(np.float64)
    assert np.isfinite(g).all() and np.isfinite(r).all()
    err = np.abs(g - r).max()
    rel = np.linalg.norm(g - r) / max(np.linalg.norm(r), 1e-30)
    assert err <= MAX_ABS and rel <= MAX_REL_L2, (err, rel)


def _case(ctx, q_per_seq, splits, seed, head_dim=128):
    from vllm_ernie_b200.decode import build_decode_metadata
    from vllm_ernie_b200.synthetic import HCADims, alloc_layer_caches, make_decode_batch

    dims = HCADims(heads=64, head_dim=head_dim)
    b = make_decode_batch(ctx, q_per_seq, dims, "cuda", seed=seed, max_model_len=1024 * 128)
    caches = alloc_layer_caches(b, seed=seed + 1)
    md = build_decode_metadata(b, 1024, num_splits=splits)
    g = torch.Generator(device="cuda").manual_seed(seed + 2)
    q = torch.randn((b.num_tokens, 64, head_dim), generator=g, device="cuda").to(torch.bfloat16)
    sink = torch.randn(64, generator=g, device="cuda")
    return q, caches, md, sink


def _noalloc(q, caches, md, sink, out):
    from vllm_ernie_b200.ops import _p, _s

    t, h, d = q.shape
    si = md.swa_indices.reshape(t, -1)
    ci = md.comp_indices.reshape(t, -1)
    _lib.call("hca_sparse_decode_noalloc", _p(out), out.stride(0), out.stride(1), None, _p(q), q.stride(0),
              q.stride(1), t, h, d, 64, _p(caches.swa), 64, caches.swa.stride(0), _p(si), si.stride(0),
              _p(md.swa_lens), _p(caches.comp), 2, caches.comp.stride(0), _p(ci), ci.stride(0), _p(md.comp_lens),
              _p(md.group_starts), md.group_starts.numel() - 1, md.max_group_tokens, d ** -0.5, _p(sink),
              md.num_splits, _s())
    return out


@pytest.mark.gpu
def test_noalloc_matches_workspace_entry_point_on_consecutive_calls():
    from vllm_ernie_b200 import ops

    rng = np.random.default_rng(11)
    cases = [
        # 48 requests x 3 query tokens, 3 splits: a large share of the array
        (rng.integers(4096, 120000, size=48).tolist(), 3, 3, 101, 128),
        # then a smaller, differently shaped call over the first call's leftovers
        ([130, 1000, 7000, 65000, 200, 33000], 2, 2, 202, 128),
        # then head_dim 512 (the CTA-pair kernel writes its partials with its
        # own code), again over the leftovers of the larger first call
        ([300, 9000, 70000, 2000], 2, 3, 303, 512),
    ]
    for ctx, qps, splits, seed, hd in cases:
        q, caches, md, sink = _case(ctx, qps, splits, seed, hd)
        assert md.num_splits > 1
        ref = ops.sparse_decode(q, caches.swa, 64, md.swa_indices, md.swa_lens, caches.comp, 2, md.comp_indices,
                                md.comp_lens, hd ** -0.5, sink, group_starts=md.group_starts,
                                max_group_tokens=md.max_group_tokens, num_splits=md.num_splits)
        out = torch.full_like(q, float("nan"))
        _noalloc(q, caches, md, sink, out)
        torch.cuda.synchronize()
        assert ops.device_error() == 0
        _close(out, ref)


def test_noalloc_refuses_problems_larger_than_its_array():
    # 4096 groups x 16 splits x 192 rows of fp32 partials is far beyond the
    # static array: refused before any device work (the pointers below are
    # placeholders that are never touched)
    lib = _lib.lib()
    need = lib.hca_sparse_decode_workspace_bytes(4096, 3, 64, 128, 16)
    assert need > 16 * 1024 * 1024
    rc = lib.hca_sparse_decode_noalloc(256, 64 * 128, 128, None, 256, 64 * 128, 128, 3 * 4096, 64, 128, 64, 256,
                                       64, 12416, 256, 128, 256, None, 2, 0, None, 0, None, 256, 4096, 3, 0.1,
                                       None, 16, None)
    assert rc == HCA_E_TOO_LARGE
    assert b"HCA_NOALLOC_WORKSPACE_BYTES" in lib.hca_status_string(rc)


def test_noalloc_reports_argument_errors_before_the_size_check():
    # the same oversized problem with a bad split count or an unsupported
    # head_dim: the argument error, not HCA_E_TOO_LARGE (host-side checks,
    # no device work; the pointers are placeholders never touched)
    lib = _lib.lib()
    args = lambda splits, hd: (256, 64 * 128, 128, None, 256, 64 * 128, 128, 3 * 4096, 64, hd, 64, 256, 64, 12416,
                               256, 128, 256, None, 2, 0, None, 0, None, 256, 4096, 3, 0.1, None, splits, None)
    assert lib.hca_sparse_decode_noalloc(*args(17, 128)) == -1  # HCA_E_INVALID
    assert lib.hca_sparse_decode_noalloc(*args(16, 256)) == -2  # HCA_E_UNSUPPORTED
