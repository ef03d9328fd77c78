"""GPU parity of the sparse HCA attention (decode and prefill) and of the
whole decode hot path, against the CPU oracle.

Tolerance (from the task's parity bar for floating point): the bf16 output
vs the oracle's fp64 evaluation on the same cached rows must have
``max |err| <= 2e-2`` and relative L2 ``<= 5e-3``.  Index tables are
checked bit-exactly against the oracle's builders first.
"""

import dataclasses

import numpy as np
import pytest
import torch

from oracle import attention as A
from oracle import cache as C
from oracle import metadata as M
from oracle import output as O
from oracle.fp8 import bf16_round

pytestmark = pytest.mark.gpu

DEV = "cuda"
MAX_ABS, MAX_REL_L2 = 2e-2, 5e-3


def check_close(got: np.ndarray, ref: np.ndarray, max_abs=MAX_ABS, max_rel=MAX_REL_L2):
    assert np.isfinite(ref).all(), f"oracle non-finite at {np.argwhere(~np.isfinite(ref))[:8].tolist()}"
    assert np.isfinite(got).all(), f"kernel non-finite at {np.argwhere(~np.isfinite(got))[:8].tolist()}"
    err = np.abs(got.astype(np.float64) - ref)
    rel = np.linalg.norm(got.astype(np.float64) - ref) / max(np.linalg.norm(ref), 1e-30)
    assert err.max() <= max_abs, (err.max(), rel)
    assert rel <= max_rel, (err.max(), rel)


def _decode_case(ctx, q_per_seq, heads, splits, seed, sink_mode="random", comp=True, sm_count=148, maxc=1024,
                 head_dim=128, whole_groups=False):
    """``splits=None``: the balanced work list for ``sm_count`` CTAs; ``maxc``:
    compressed-index width (context up to maxc * 128); ``whole_groups``: one
    group per request however many rows it has (uniform splits only)."""
    from vllm_ernie_b200 import ops
    from vllm_ernie_b200.decode import build_decode_metadata
    from vllm_ernie_b200.synthetic import HCADims, alloc_layer_caches, make_decode_batch

    dims = HCADims(heads=heads, head_dim=head_dim)
    b = make_decode_batch(ctx, q_per_seq, dims, DEV, seed=seed, max_model_len=maxc * 128)
    caches = alloc_layer_caches(b, seed=seed + 1)
    md = build_decode_metadata(b, maxc, num_splits=splits, sm_count=sm_count)
    if splits is None:
        check_schedule(md)
    if whole_groups:
        md = dataclasses.replace(md, group_starts=b.query_start_loc, max_group_tokens=q_per_seq)
    # index tables vs the oracle builders (bit-exact)
    qsl, sl = b.query_start_loc.cpu().numpy(), b.seq_lens.cpu().numpy()
    t2r = M.token_to_req_indices(qsl)
    swa_slot = M.slot_mapping(qsl, sl, b.swa_bt.cpu().numpy(), 64)
    assert np.array_equal(md.swa_slot.cpu().numpy(), swa_slot)
    n = b.num_tokens
    idx = np.full((n, 128), -7, np.int32)
    lens = np.zeros(n, np.int32)
    M.swa_indices_and_lens(n, 128, qsl, sl, t2r, swa_slot >= 0, b.swa_bt.cpu().numpy(), 64, idx, lens)
    assert np.array_equal(md.swa_lens.cpu().numpy(), lens)
    assert np.array_equal(md.swa_indices.cpu().numpy(), idx)
    gd = np.zeros((n, maxc), np.int32)
    dl = np.zeros(n, np.int32)
    M.c128a_topk_metadata(b.positions.cpu().numpy(), 128, n, t2r, b.comp_bt.cpu().numpy(), 2, swa_slot, gd,
                          dl, np.zeros((1, maxc), np.int32), maxc)
    assert np.array_equal(md.comp_lens.cpu().numpy(), dl)
    assert np.array_equal(md.comp_indices.cpu().numpy(), gd)

    g = torch.Generator(device=DEV).manual_seed(seed + 2)
    q = torch.randn((n, heads, head_dim), generator=g, device=DEV).to(torch.bfloat16)
    if sink_mode == "random":
        sink = torch.randn(heads, generator=g, device=DEV)
    elif sink_mode == "neginf":
        sink = torch.full((heads,), -float("inf"), device=DEV)
    else:
        sink = None
    out = ops.sparse_decode(q, caches.swa, 64, md.swa_indices, md.swa_lens,
                            caches.comp if comp else None, 2, md.comp_indices if comp else None,
                            md.comp_lens if comp else None, head_dim ** -0.5, sink,
                            group_starts=md.group_starts, max_group_tokens=md.max_group_tokens,
                            num_splits=md.num_splits, schedule=md.schedule, max_items=md.max_items)
    ref = A.sparse_decode(q.float().cpu().numpy(), caches.swa.cpu().numpy(), 64, idx, lens,
                          caches.comp.cpu().numpy() if comp else None, 2, gd if comp else None,
                          dl if comp else None, head_dim ** -0.5,
                          sink.cpu().numpy() if sink is not None else None, head_dim, 64)
    check_close(out.float().cpu().numpy(), ref)
    assert ops.device_error() == 0
    return out


def check_schedule(md):
    """The device work list equals this plain restatement of its rule: the
    smallest per-CTA chunk budget t (at most 16 CTAs per group) with
    sum_g max(1, ceil(c_g / t)) <= max_items; group g gets that many CTAs over
    even chunk ranges, numbered group by group; the rest are idle."""
    gs = md.group_starts.cpu().numpy()
    wl = md.swa_lens.cpu().numpy()
    cl = md.comp_lens.cpu().numpy()
    c = []
    for g in range(len(gs) - 1):
        t0, t1 = gs[g], gs[g + 1]
        if wl[t0] <= 0:
            c.append(0)
            continue
        rows = wl[t0] + min(t1 - t0 - 1, wl[t1 - 1]) + max(cl[t1 - 1], 0)
        c.append(-(-rows // 64))
    maxc = max(c + [1])
    t = max(1, -(-maxc // 16))
    while sum(max(1, -(-x // t)) for x in c) > md.max_items:
        t += 1
    items, groups = [], []
    for g, x in enumerate(c):
        s = max(1, -(-x // t))
        groups.append((len(items), s))
        items += [(g, k, k * x // s, (k + 1) * x // s) for k in range(s)]
    items += [(-1, 0, 0, 0)] * (md.max_items - len(items))
    got = md.schedule.cpu().numpy()
    n = md.max_items
    assert np.array_equal(got[: 4 * n].reshape(n, 4)[:, 0], np.array([i[0] for i in items]))
    live = [i for i in items if i[0] >= 0]
    assert np.array_equal(got[: 4 * len(live)].reshape(-1, 4), np.array(live))
    assert np.array_equal(got[4 * n:].reshape(-1, 2), np.array(groups))


@pytest.mark.parametrize("splits", [1, 3, None])
@pytest.mark.parametrize("q_per_seq", [1, 3])
def test_decode_mixed_contexts(q_per_seq, splits):
    # short (< window), boundary-crossing, and long contexts
    ctx = [0, 5, 126, 127, 128, 254, 1000, 9000, 40000, 130000]
    _decode_case(ctx, q_per_seq, 64, splits, seed=11 + q_per_seq + (splits or 7))


def test_decode_config2_shape_sample():
    """Config-2 geometry (64 heads x 128, 3 queries/seq) on a sample of 8
    requests with contexts drawn from U[4096, 131072]."""
    rng = np.random.default_rng(0)
    ctx = rng.integers(4096, 131072, size=8).tolist()
    _decode_case(ctx, 3, 64, 4, seed=3)


def test_decode_config2_shape_scheduled():
    """The bench's balanced work list on 64 config-2 requests: multi-CTA
    groups, single-CTA groups and idle CTAs in one launch."""
    rng = np.random.default_rng(1)
    ctx = rng.integers(4096, 131072, size=64).tolist()
    _decode_case(ctx, 3, 64, None, seed=4)


@pytest.mark.parametrize("sm_count", [3, 13, 40])
def test_decode_schedule_small_waves(sm_count):
    # few CTAs for many rows: budgets above the 16-split cap, groups with one CTA
    _decode_case([5, 126, 700, 4000, 9000, 33000, 60000, 131000][: max(1, min(8, sm_count))], 3, 64, None,
                 seed=17 + sm_count, sm_count=sm_count)


@pytest.mark.parametrize("sink_mode", ["neginf", "none"])
def test_decode_sink_variants(sink_mode):
    _decode_case([300, 77, 5000], 3, 64, 2, seed=5, sink_mode=sink_mode)


def test_decode_16_heads_window_only():
    _decode_case([3, 200, 2000], 3, 16, 1, seed=9, comp=False)


def test_decode_grid_has_idle_splits():
    # many splits relative to rows: empty splits must still combine correctly
    _decode_case([10, 150], 3, 64, 8, seed=13)


def test_prefill_matches_oracle():
    # prefill chunks: (prior context, chunk length)
    _prefill_case([(0, 300), (1000, 131), (128 * 7, 64)], 64, seed=22)


@pytest.mark.parametrize("heads", [8, 16, 64])
def test_prefill_long_prior_context(heads):
    # tiles of 32 (H=8, e.g. 16 heads under TP=2), 16 (H=16) or 4 (H=64)
    # tokens over many chunks of compressed rows
    _prefill_case([(20000, 70), (128 * 40 - 3, 9), (5, 250)], heads, seed=31 + heads)


def _prefill_case(reqs, heads, seed, head_dim=128):
    from vllm_ernie_b200 import ops

    q_lens = np.array([c for _, c in reqs])
    qsl = np.concatenate([[0], np.cumsum(q_lens)]).astype(np.int32)
    seq = np.array([p + c for p, c in reqs], np.int32)
    # pages: make every needed position mapped (window of the first token .. end)
    swa_bt = np.zeros((3, (seq.max() + 63) // 64 + 2), np.int32)
    comp_bt = np.zeros((3, seq.max() // 256 + 2), np.int32)
    k = 0
    for r, (p, c) in enumerate(reqs):
        lo, hi = max(p - 127, 0) // 64, (p + c + 63) // 64
        swa_bt[r, lo:hi] = np.arange(k, k + hi - lo)
        k += hi - lo
    n_swa = k
    k = 0
    for r, (p, c) in enumerate(reqs):
        hi = (p + c) // 128 // 2 + 1
        comp_bt[r, :hi] = np.arange(k, k + hi)
        k += hi
    n_comp = k
    from vllm_ernie_b200.cache_layout import page_bytes

    gen = torch.Generator(device=DEV).manual_seed(seed)
    swa = torch.zeros((n_swa, page_bytes(64, head_dim, 64)), dtype=torch.uint8, device=DEV)
    comp = torch.zeros((n_comp, page_bytes(2, head_dim, 64)), dtype=torch.uint8, device=DEV)
    for cache, page, npg in ((swa, 64, n_swa), (comp, 2, n_comp)):
        rows = torch.randn((npg * page, head_dim), generator=gen, device=DEV).to(torch.bfloat16)
        ops.quantize_and_insert_k_cache(rows, cache, torch.arange(npg * page, device=DEV), page)
    n = int(qsl[-1])
    q = torch.randn((n, heads, head_dim), generator=gen, device=DEV).to(torch.bfloat16)
    sink = torch.randn(heads, generator=gen, device=DEV)
    out = ops.sparse_prefill(q, torch.from_numpy(qsl).to(DEV), torch.from_numpy(seq).to(DEV), swa, 64,
                             torch.from_numpy(swa_bt).to(DEV), comp, 2, torch.from_numpy(comp_bt).to(DEV),
                             128, 128, head_dim ** -0.5, sink)
    t2r = M.token_to_req_indices(qsl)
    pos = np.concatenate([np.arange(p, p + c) for p, c in reqs])
    ref = A.sparse_prefill_paged(q.float().cpu().numpy(), pos, t2r, swa.cpu().numpy(), 64, swa_bt,
                                 comp.cpu().numpy(), 2, comp_bt, 128, 128, head_dim ** -0.5,
                                 sink.cpu().numpy(), head_dim, 64)
    check_close(out.float().cpu().numpy(), ref)
    assert ops.device_error() == 0


def test_decode_layer_hot_path_matches_oracle():
    """q prep + SWA insert, compressor, attention and VHA/inverse-RoPE/FP8 of
    one layer vs the oracle composition of the same steps."""
    from vllm_ernie_b200.decode import build_decode_metadata, decode_layer, random_layer_weights
    from vllm_ernie_b200.synthetic import HCADims, alloc_layer_caches, make_decode_batch, rope_cos_sin_cache

    dims = HCADims(heads=64)
    maxc = 256
    # contexts chosen so some query tokens complete a 128-block this step
    ctx = [125, 254, 1020, 5000, 30000]
    b = make_decode_batch(ctx, 3, dims, DEV, seed=31, max_model_len=maxc * 128)
    caches = alloc_layer_caches(b, seed=32)
    w = random_layer_weights(dims, DEV, seed=33)
    md = build_decode_metadata(b, maxc, num_splits=2)
    n = b.num_tokens
    g = torch.Generator(device=DEV).manual_seed(34)
    q_raw = torch.randn((n, 64, 128), generator=g, device=DEV).to(torch.bfloat16)
    kv = torch.randn((n, 128), generator=g, device=DEV).to(torch.bfloat16)
    kv_score = torch.randn((n, 256), generator=g, device=DEV)
    cos_sin = rope_cos_sin_cache(maxc * 128 + 8, 64, dims.rope_theta, DEV)
    swa0, comp0, state0 = (caches.swa.cpu().numpy(), caches.comp.cpu().numpy(), caches.state.cpu().numpy())
    y = decode_layer(b, md, caches, w, q_raw, kv, kv_score, cos_sin, quantize=False)
    torch.cuda.synchronize()

    # oracle composition
    pos = b.positions.cpu().numpy()
    cs = cos_sin.cpu().numpy()
    qsl, sl = b.query_start_loc.cpu().numpy(), b.seq_lens.cpu().numpy()
    t2r = M.token_to_req_indices(qsl)
    swa_bt, comp_bt, st_bt = b.swa_bt.cpu().numpy(), b.comp_bt.cpu().numpy(), b.state_bt.cpu().numpy()
    qp = O.q_prep(q_raw.float().cpu().numpy(), pos, cs, 64, 1e-6)
    swa_slot = M.slot_mapping(qsl, sl, swa_bt, 64)
    C.insert_rows(swa0, swa_slot, O.kv_rope(kv.float().cpu().numpy(), pos, cs, 64), 64, 128, 64)
    st_slot = M.slot_mapping(qsl, sl, st_bt, 8)
    ks = kv_score.cpu().numpy()
    C.save_partial_states(state0, ks[:, :128], ks[:, 128:], w.ape.cpu().numpy(), pos, st_slot, 8, 128)
    c_slot = M.compressed_slot_mapping(n, qsl, sl, comp_bt, 2, 128)
    assert (c_slot >= 0).sum() >= 2
    C.compress_norm_rope_store(state0, t2r, pos, st_slot, st_bt, 8, w.comp_norm.cpu().numpy(), 1e-6, cs,
                               comp0, c_slot, 2, 128, 64)
    idx = np.zeros((n, 128), np.int32)
    lens = np.zeros(n, np.int32)
    M.swa_indices_and_lens(n, 128, qsl, sl, t2r, swa_slot >= 0, swa_bt, 64, idx, lens)
    gd = np.zeros((n, maxc), np.int32)
    dl = np.zeros(n, np.int32)
    M.c128a_topk_metadata(pos, 128, n, t2r, comp_bt, 2, swa_slot, gd, dl, np.zeros((1, maxc), np.int32), maxc)
    o = A.sparse_decode(qp, swa0, 64, idx, lens, comp0, 2, gd, dl, 128 ** -0.5, w.attn_sink.cpu().numpy(), 128, 64)
    mix = w.vha_mix.float().cpu().numpy()
    y_ref = O.inv_rope_fp8_quant(np.einsum("hg,tgd->thd", mix, bf16_round(o)), pos, cs, 8, 64, quant=False)
    check_close(y.float().cpu().numpy(), y_ref)


def _dequant(data, scale):
    """e4m3 [T, G, HPG*D] x UE8M0 [T, G, HPG] -> fp32 [T, H, D]."""
    t, g, w = data.shape
    hpg = scale.shape[2]
    x = data.float().view(t, g, hpg, w // hpg)
    e = (scale.to(torch.int64) & 0xFF).float() - 127.0
    return (x * torch.exp2(e)[..., None]).reshape(t, g * hpg, w // hpg)


def test_decode_fused_vha_quant_matches_unfused():
    """Scheduled attention fused with the VHA mix + inverse RoPE + FP8 quant
    equals attention followed by hca_vha_inv_rope_fp8_quant up to roundings:
    both read the same bf16 split partials, but the fused merge adds them in
    another order and mixes in another kernel, so >= 95% of the e4m3 bytes
    agree, each element is within one e4m3 step or 2 units of its head's
    scale (near-zero elements where the splits cancel), and the dequantised
    outputs are within relative L2 2e-2."""
    from vllm_ernie_b200 import ops
    from vllm_ernie_b200.decode import build_decode_metadata, random_layer_weights
    from vllm_ernie_b200.synthetic import HCADims, alloc_layer_caches, make_decode_batch, rope_cos_sin_cache

    dims = HCADims(heads=64)
    rng = np.random.default_rng(5)
    ctx = [0, 3, 130] + rng.integers(4096, 131000, size=29).tolist()
    b = make_decode_batch(ctx, 3, dims, DEV, seed=41, max_model_len=1024 * 128)
    caches = alloc_layer_caches(b, seed=42)
    w = random_layer_weights(dims, DEV, seed=43)
    for sm_count in (148, 40):
        md = build_decode_metadata(b, 1024, sm_count=sm_count)
        g = torch.Generator(device=DEV).manual_seed(44)
        q = torch.randn((b.num_tokens, 64, 128), generator=g, device=DEV).to(torch.bfloat16)
        cs = rope_cos_sin_cache(1024 * 128 + 8, 64, dims.rope_theta, DEV)
        args = (q, caches.swa, 64, md.swa_indices, md.swa_lens, caches.comp, 2, md.comp_indices, md.comp_lens,
                128 ** -0.5, w.attn_sink)
        o = ops.sparse_decode(*args, group_starts=md.group_starts, max_group_tokens=md.max_group_tokens,
                              schedule=md.schedule, max_items=md.max_items)
        d_ref, s_ref = ops.vha_inv_rope_fp8_quant(o, w.vha_mix, b.positions, cs, 8, 64, 64)
        d_got, s_got = ops.sparse_decode_vha_fp8_quant(*args, md.group_starts, md.max_group_tokens, md.schedule,
                                                       md.max_items, w.vha_mix, b.positions, cs, 8)
        torch.cuda.synchronize()
        assert ops.device_error() == 0
        same = (d_ref.view(torch.uint8) == d_got.view(torch.uint8)).float().mean().item()
        assert same > 0.95, same
        assert (s_ref == s_got).float().mean().item() > 0.99
        a, r = _dequant(d_got, s_got), _dequant(d_ref, s_ref)
        assert torch.isfinite(a).all()
        # one e4m3 step (2^-3 of the larger value's binade), or 2 units of
        # the head's scale (1/224 of its e4m3 range)
        t, g, hpg = s_ref.shape
        unit = torch.exp2((torch.maximum(s_ref, s_got).to(torch.int64) & 0xFF).float() - 127.0)
        unit = unit.reshape(t, g * hpg, 1)
        assert ((a - r).abs() <= 0.125 * torch.maximum(a.abs(), r.abs()) + 2.0 * unit).all()
        assert ((a - r).norm() / r.norm()).item() <= 2e-2


@pytest.mark.parametrize("heads", [1, 8])
@pytest.mark.parametrize("splits", [1, None])
def test_decode_few_heads(heads, splits):
    """Tiles with fewer than 16 query rows (some TMEM lane quadrants empty),
    e.g. 8 heads per GPU under TP=8."""
    _decode_case([5, 300, 9000, 70000], 3, heads, splits, seed=23 + heads)


@pytest.mark.parametrize("splits", [None, 16])
def test_decode_million_token_context(splits):
    """Config 4 geometry: ~1M-token contexts, 8192 compressed entries plus the
    window per sequence, 3 queries per sequence; the split-K merge spans up to
    16 CTAs per request."""
    ctx = [1048573, 1048000, 900001, 1048575 - 128 * 5]
    _decode_case(ctx, 3, 64, splits, seed=51, maxc=8320)


# ---- head_dim 512 (the model's own head size): CTA-pair kernel ----


@pytest.mark.parametrize("splits", [1, 3, None])
@pytest.mark.parametrize("q_per_seq", [1, 3])
def test_decode_head_dim_512(q_per_seq, splits):
    """64 heads x 512: groups of at most 2 tokens (one 128-row tile of a CTA
    pair); None = the balanced work list."""
    ctx = [0, 5, 127, 128, 700, 9000, 40000]
    _decode_case(ctx, q_per_seq, 64, splits, seed=61 + q_per_seq + (splits or 5), maxc=320, head_dim=512)


@pytest.mark.parametrize("splits", [1, 4])
def test_decode_head_dim_512_whole_groups(splits):
    """A 3-token group of 64 heads (192 rows) spans two pair tiles, whose
    partials (or outputs) land in the group's rows."""
    ctx = [0, 5, 127, 128, 700, 9000, 40000]
    _decode_case(ctx, 3, 64, splits, seed=81 + splits, maxc=320, head_dim=512, whole_groups=True)


@pytest.mark.parametrize("sink_mode", ["neginf", "none"])
def test_decode_head_dim_512_16_heads(sink_mode):
    # 16 heads: all 3 tokens of a request in one 48-row tile; window-only rows
    _decode_case([3, 200, 2000], 3, 16, 2, seed=67, sink_mode=sink_mode, comp=False, maxc=32, head_dim=512)


def test_decode_head_dim_512_long_context():
    # many compressed rows per tile, split-K over 8 pairs
    _decode_case([130000, 65000], 3, 64, 8, seed=69, maxc=1024, head_dim=512)


@pytest.mark.parametrize("heads", [4, 16, 64])
def test_prefill_head_dim_512(heads):
    # 4 heads: tiles of 31 tokens (the most a row's token mask holds)
    _prefill_case([(0, 130), (3000, 67), (128 * 9 - 1, 5)], heads, seed=71 + heads, head_dim=512)


def test_bounded_wait_gives_up_and_next_launch_is_clean():
    """The attention kernel's mbarrier waits are bounded: with a wait limit of
    0 (a wait not already satisfied fails at once) the launch still ends, with
    its softmax error bit (value 8) set in the device error word; once the bit
    is cleared and the default limit restored, the next launch is correct and
    leaves the word zero."""
    from vllm_ernie_b200 import ops

    ops.device_error(clear=True)
    ops.set_attention_wait_limit_ns(0)
    try:
        with pytest.raises(AssertionError):
            _decode_case([300, 5000, 40000], 3, 64, None, seed=41)
        torch.cuda.synchronize()
    finally:
        ops.set_attention_wait_limit_ns(-1)
    err = ops.device_error(clear=True)
    assert err & 8, err
    assert ops.device_error() == 0
    _decode_case([300, 5000, 40000], 3, 64, None, seed=41)


def test_decode_workspace_per_device_and_stable_under_capture():
    """The split-K workspace keeps one buffer per device, reuses it for
    smaller requests, and refuses to grow while a CUDA graph is being
    captured (a regrown buffer would free the address the graph holds)."""
    from vllm_ernie_b200.ops import DecodeWorkspace

    ws = DecodeWorkspace()
    a = ws.get(1 << 20, "cuda:0")
    assert ws.get(1 << 10, "cuda:0").data_ptr() == a.data_ptr()
    s = torch.cuda.Stream()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        assert ws.get(1 << 20, "cuda:0").data_ptr() == a.data_ptr()
        with pytest.raises(RuntimeError):
            ws.get(1 << 21, "cuda:0")
    del g
    if torch.cuda.device_count() > 1:
        b = ws.get(1 << 20, "cuda:1")
        assert b.device.index == 1 and ws.get(1 << 20, "cuda:0").data_ptr() == a.data_ptr()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs in one process")
def test_decode_on_two_devices_in_one_process():
    """One process drives split-K decode on cuda:0 then cuda:1: each launch
    gets its own device's workspace and both give the same output."""
    from vllm_ernie_b200 import ops
    from vllm_ernie_b200.decode import build_decode_metadata
    from vllm_ernie_b200.synthetic import HCADims, alloc_layer_caches, make_decode_batch

    outs = []
    for dev in ("cuda:0", "cuda:1"):
        with torch.cuda.device(dev):
            dims = HCADims(heads=64)
            b = make_decode_batch([300, 5000, 40000], 3, dims, dev, seed=7, max_model_len=1024 * 128)
            caches = alloc_layer_caches(b, seed=8)
            md = build_decode_metadata(b, 1024, num_splits=3)
            g = torch.Generator(device=dev).manual_seed(9)
            q = torch.randn((b.num_tokens, 64, 128), generator=g, device=dev).to(torch.bfloat16)
            sink = torch.randn(64, generator=g, device=dev)
            o = ops.sparse_decode(q, caches.swa, 64, md.swa_indices, md.swa_lens, caches.comp, 2, md.comp_indices,
                                  md.comp_lens, 128 ** -0.5, sink, group_starts=md.group_starts,
                                  max_group_tokens=md.max_group_tokens, num_splits=3)
            torch.cuda.synchronize()
            outs.append(o.cpu())
    assert torch.equal(outs[0], outs[1])
