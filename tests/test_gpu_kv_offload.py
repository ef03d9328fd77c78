"""KV pages survive an offload round trip: moved out to pinned host memory and
back into other page ids, the way a KV offload connector moves whole blocks
(``SimpleCPUOffloadConnector``, the reference README's "KV Cache Offload"),
they carry everything a decode step reads.

Every page of the three caches of a layer (window rows, compressed rows,
compressor states) goes to host memory; the device caches are then filled with
garbage and each page is written back at a new id ``perm[p]``, with the block
tables remapped through the same permutation.  A decode step over the moved
pages must give the same output bytes as the step over the original pages, and
leave every page it wrote (the new window rows, the states it saved, the
entries it compressed) equal to its counterpart.  Nothing outside the pages
(no side table of scales, no absolute slot) may carry state across steps.
"""

import copy

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _move_pages(cache: torch.Tensor, perm: torch.Tensor) -> torch.Tensor:
    """Offload every page to pinned host memory, then load page p back at
    perm[p] of a device cache that held garbage."""
    host = torch.empty(cache.shape, dtype=cache.dtype, pin_memory=True)
    host.copy_(cache, non_blocking=True)
    torch.cuda.synchronize()
    moved = torch.empty_like(cache)
    moved.view(torch.uint8).fill_(0xA5)
    moved[perm.to(DEV)] = host.to(DEV, non_blocking=True)
    return moved


def _remap(bt: torch.Tensor, perm: torch.Tensor) -> torch.Tensor:
    return perm.to(bt.device)[bt.long()].to(bt.dtype)


@pytest.mark.parametrize("head_dim", [128, 512])
def test_decode_step_over_offloaded_and_moved_pages(head_dim):
    from vllm_ernie_b200 import ops
    from vllm_ernie_b200.decode import build_decode_metadata, decode_layer, random_layer_weights
    from vllm_ernie_b200.synthetic import (HCADims, LayerCaches, alloc_layer_caches, make_decode_batch,
                                           rope_cos_sin_cache)

    heads = 64
    dims = HCADims(heads=heads, head_dim=head_dim)
    maxc = 160
    # contexts whose step completes a compressed block (ctx % 128 in
    # {125, 126, 127}) beside plain ones, short and long
    ctx = [125, 254, 3199, 0, 7, 130, 5000, 20000 - 3]
    b = make_decode_batch(ctx, 3, dims, DEV, seed=7, max_model_len=maxc * 128)
    caches = alloc_layer_caches(b, seed=8)
    w = random_layer_weights(dims, DEV, seed=9)
    n = b.num_tokens
    g = torch.Generator(device=DEV).manual_seed(10)
    q_raw = torch.randn((n, heads, head_dim), generator=g, device=DEV).to(torch.bfloat16)
    kv = torch.randn((n, head_dim), generator=g, device=DEV).to(torch.bfloat16)
    ks = torch.randn((n, 2 * head_dim), generator=g, device=DEV)
    cs = rope_cos_sin_cache(maxc * 128 + 8, dims.rope_dim, dims.rope_theta, DEV)
    quantize = head_dim == 128

    def step(batch, lc):
        md = build_decode_metadata(batch, maxc)
        out = decode_layer(batch, md, lc, w, q_raw, kv, ks, cs, quantize=quantize)
        torch.cuda.synchronize()
        return out

    # the step over the original pages (on copies: the step writes into them)
    ref_caches = LayerCaches(caches.swa.clone(), caches.comp.clone(), caches.state.clone())
    ref = step(b, ref_caches)

    # the step over pages moved through host memory to permuted ids
    gp = torch.Generator().manual_seed(11)
    perms = [torch.randperm(c.shape[0], generator=gp) for c in (caches.swa, caches.comp, caches.state)]
    moved = LayerCaches(*[_move_pages(c, p) for c, p in zip((caches.swa, caches.comp, caches.state), perms)])
    mb = copy.copy(b)
    mb.swa_bt = _remap(b.swa_bt, perms[0])
    mb.comp_bt = _remap(b.comp_bt, perms[1])
    mb.state_bt = _remap(b.state_bt, perms[2])
    got = step(mb, moved)
    assert ops.device_error() == 0

    if quantize:
        assert torch.equal(got[0].view(torch.uint8), ref[0].view(torch.uint8))
        assert torch.equal(got[1], ref[1])
    else:
        assert torch.equal(got.view(torch.int16), ref.view(torch.int16))
    # every page after the step, moved back to its original id, equals the
    # page the unmoved step left
    for name, p in zip(("swa", "comp", "state"), perms):
        after = getattr(moved, name)[p.to(DEV)]
        want = getattr(ref_caches, name)
        assert torch.equal(after.view(torch.uint8), want.view(torch.uint8)), name
