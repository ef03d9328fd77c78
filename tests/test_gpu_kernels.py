"""GPU parity of the metadata, cache, compressor and output kernels.

Each test runs the CUDA kernel through the C ABI (``vllm_ernie_b200.ops``)
and compares with the golden vectors of the reference's own kernels
(``tests/golden``, D=512) or with the CPU oracle (D=128).  Integer and
byte outputs must match bit-exactly; floating outputs within the tolerances
stated per test.
"""

import numpy as np
import pytest
import torch

from golden_io import load
from oracle import cache as C
from oracle import metadata as M
from oracle import output as O
from oracle.fp8 import bf16_round, e4m3_to_f32

pytestmark = pytest.mark.gpu

DEV = "cuda"


def T(x, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(x))
    if dtype is not None:
        t = t.to(dtype)
    return t.to(DEV)


@pytest.fixture(scope="module")
def ops():
    from vllm_ernie_b200 import ops as _ops

    return _ops


# --------------------------------------------------------------------------
# metadata (bit-exact vs reference kernels)
# --------------------------------------------------------------------------


def test_metadata_bit_exact(ops):
    g = load("metadata")
    qsl, sl = T(g["query_start_loc"]), T(g["seq_lens"])
    n = int(g["query_start_loc"][-1])
    nd, ndt = int(g["num_decodes"]), int(g["num_decode_tokens"])
    t2r = ops.token_to_req_indices(qsl, n)
    assert np.array_equal(t2r.cpu().numpy(), g["token_to_req"])
    cs = ops.get_compressed_slot_mapping(n, qsl, sl, T(g["comp_block_table"]), 2, 128,
                                         out=torch.empty(n + 8, dtype=torch.int64, device=DEV))
    assert np.array_equal(cs.cpu().numpy(), g["comp_slot"][:n])
    idx = torch.full((n, 128), 777, dtype=torch.int32, device=DEV)
    lens = torch.full((n,), 99, dtype=torch.int32, device=DEV)
    ops.compute_swa_indices_and_lens(idx, lens, ndt, 128, qsl, sl, t2r, T(g["slot_mapping"]) >= 0,
                                     T(g["swa_block_table"]), 64)
    assert np.array_equal(lens.cpu().numpy(), g["swa_lens"])
    assert np.array_equal(idx.cpu().numpy()[:ndt], g["swa_indices"][:ndt])
    maxc = int(g["max_compressed"])
    gd = torch.full((n, maxc), 555, dtype=torch.int32, device=DEV)
    dl = torch.full((n,), 555, dtype=torch.int32, device=DEV)
    pl = torch.full((n, maxc), 555, dtype=torch.int32, device=DEV)
    ops.build_c128a_topk_metadata(T(g["positions"]), 128, ndt, t2r, T(g["comp_block_table"][:nd]), 2,
                                  T(g["slot_mapping"]), gd, dl, pl, maxc)
    assert np.array_equal(gd.cpu().numpy()[:ndt], g["c128a_global"][:ndt])
    assert np.array_equal(dl.cpu().numpy()[:ndt], g["c128a_lens"][:ndt])
    assert np.array_equal(pl.cpu().numpy()[: n - ndt], g["c128a_prefill"][: n - ndt])
    gl = ops.compute_prefill_gather_lens(sl, qsl, 2, nd, 128)
    assert np.array_equal(gl.cpu().numpy(), g["gather_lens"])
    comb, clens = ops.combine_topk_swa_indices(T(g["c128a_prefill"][: n - ndt]), qsl[nd:], sl[nd:], gl,
                                               128, 128, maxc, int(g["M"]), int(g["N"]))
    assert np.array_equal(comb.cpu().numpy(), g["combined"])
    assert np.array_equal(clens.cpu().numpy(), g["combined_lens"])


def test_slot_mapping_matches_oracle(ops):
    rng = np.random.default_rng(1)
    q_lens = np.array([3, 1, 200, 3])
    seq = np.array([7000, 5, 900, 129], dtype=np.int32)
    qsl = np.concatenate([[0], np.cumsum(q_lens)]).astype(np.int32)
    bt = rng.integers(0, 1 << 20, size=(4, 1000), dtype=np.int32)
    for bs in (8, 64):
        ours = ops.slot_mapping(T(qsl), T(seq), T(bt), bs, int(qsl[-1])).cpu().numpy()
        assert np.array_equal(ours, M.slot_mapping(qsl, seq, bt, bs))


# --------------------------------------------------------------------------
# cache write / gather
# --------------------------------------------------------------------------


def test_quantize_insert_bytes_match_reference(ops):
    g = load("kv_insert_gather")
    cache = torch.zeros(g["cache"].shape, dtype=torch.uint8, device=DEV)
    ops.quantize_and_insert_k_cache(T(g["k"], torch.bfloat16), cache, T(g["slots"]), block_size=int(g["page"]))
    assert np.array_equal(cache.cpu().numpy(), g["cache"])


def test_dequant_gather_matches_reference(ops):
    g = load("kv_insert_gather")
    out = torch.zeros(g["gathered"].shape, dtype=torch.bfloat16, device=DEV)
    ops.dequantize_and_gather_k_cache(out, T(g["cache"]), T(g["seq_lens"]), T(g["gather_lens"]),
                                      T(g["block_table"]), int(g["page"]), 5)
    assert np.array_equal(out.float().cpu().numpy(), g["gathered"])


@pytest.mark.parametrize("head_dim", [128, 512])
def test_qnorm_rope_kv_insert_matches_oracle(ops, head_dim):
    rng = np.random.default_rng(head_dim)
    t, h, r, page = 37, 16, 64, 64
    q = bf16_round(rng.standard_normal((t, h, head_dim)).astype(np.float32) * 2)
    kv = bf16_round(rng.standard_normal((t, head_dim)).astype(np.float32))
    pos = rng.integers(0, 4000, size=t)
    cos_sin = C.rope_cos_sin_cache(4096, r, 160000.0)
    slots = rng.permutation(4 * page)[:t].astype(np.int64)
    slots[3] = -1
    pb = C.page_bytes(page, head_dim, r)
    cache = torch.zeros((4, pb), dtype=torch.uint8, device=DEV)
    qo = ops.fused_qnorm_rope_kv_insert(T(q, torch.bfloat16), T(kv, torch.bfloat16), cache, T(slots),
                                        T(pos), T(cos_sin), 64, 1e-6, page)
    ref_q = O.q_prep(q, pos, cos_sin, r, 1e-6, padded_heads=64)
    got_q = qo.float().cpu().numpy()
    np.testing.assert_allclose(got_q, ref_q, rtol=2 ** -7, atol=1e-6)
    assert (got_q == ref_q).mean() > 0.99
    ref_cache = np.zeros((4, pb), np.uint8)
    C.insert_rows(ref_cache, slots, O.kv_rope(kv, pos, cos_sin, r), page, head_dim, r)
    got = cache.cpu().numpy()
    # NoPE bytes and scales exact; RoPE bf16 within one ulp
    rows = C.read_rows(got, slots[slots >= 0], page, head_dim, r)
    ref_rows = C.read_rows(ref_cache, slots[slots >= 0], page, head_dim, r)
    nope = head_dim - r
    assert np.array_equal(rows[:, :nope], ref_rows[:, :nope])
    np.testing.assert_allclose(rows[:, nope:], ref_rows[:, nope:], rtol=2 ** -7, atol=1e-6)


@pytest.mark.parametrize("head_dim,heads,padded", [(128, 64, 64), (128, 16, 64), (512, 16, 64)])
def test_qnorm_rope_kv_insert_streamed_matches_per_token_kernel(ops, head_dim, heads, padded):
    """At >= 4096 tokens with contiguous heads the library takes the streamed
    kernel (bulk copies into a shared-memory ring); with a head stride != D
    it takes the per-token kernel.  Both must write identical bytes (q and
    the cache), and the q rows must match the oracle."""
    rng = np.random.default_rng(heads + head_dim)
    t, r, page = 4500, 64, 64
    q = bf16_round(rng.standard_normal((t, heads, head_dim)).astype(np.float32) * 2)
    kv = bf16_round(rng.standard_normal((t, head_dim)).astype(np.float32))
    pos = rng.integers(0, 8000, size=t)
    cos_sin = C.rope_cos_sin_cache(8192, r, 160000.0)
    n_pages = (t + page - 1) // page + 1
    slots = rng.permutation(n_pages * page)[:t].astype(np.int64)
    slots[::97] = -1
    pb = C.page_bytes(page, head_dim, r)
    q_dev = T(q, torch.bfloat16)
    # the same q with a head stride of D + 8: the per-token kernel
    q_wide = torch.zeros((t, heads, head_dim + 8), dtype=torch.bfloat16, device=DEV)
    q_wide[..., :head_dim] = q_dev
    q_strided = q_wide[..., :head_dim]
    assert q_strided.stride(1) != head_dim
    outs = []
    for qin in (q_dev, q_strided):
        cache = torch.zeros((n_pages, pb), dtype=torch.uint8, device=DEV)
        qo = ops.fused_qnorm_rope_kv_insert(qin, T(kv, torch.bfloat16), cache, T(slots), T(pos), T(cos_sin),
                                            padded, 1e-6, page)
        torch.cuda.synchronize()
        outs.append((qo.view(torch.int16).cpu().numpy(), cache.cpu().numpy()))
    assert np.array_equal(outs[0][0], outs[1][0])
    assert np.array_equal(outs[0][1], outs[1][1])
    assert ops.device_error() == 0
    ref_q = O.q_prep(q, pos, cos_sin, r, 1e-6, padded_heads=padded)
    got_q = outs[0][0].astype(np.int16).view(np.uint16).astype(np.uint32) << 16
    got_q = got_q.view(np.float32)
    np.testing.assert_allclose(got_q, ref_q, rtol=2 ** -7, atol=1e-6)
    assert (got_q == ref_q).mean() > 0.99
    assert not got_q[:, heads:].any()


# --------------------------------------------------------------------------
# compressor
# --------------------------------------------------------------------------


def test_save_partial_states_bit_exact(ops):
    g = load("compressor")
    state = T(g["state_before"])
    ops.save_partial_states(T(g["kv"]), T(g["score"]), T(g["ape"]), T(g["positions"]), state,
                            T(g["state_slot"]), 8, 512, 128)
    flat = state.view(-1, 1024).cpu().numpy()
    ok = g["state_slot"] >= 0
    assert np.array_equal(flat[g["state_slot"][ok]], g["state_rows_written"][ok])


def test_compressor_matches_reference_d512(ops):
    g = load("compressor")
    state = T(g["state_before"])
    ops.save_partial_states(T(g["kv"]), T(g["score"]), T(g["ape"]), T(g["positions"]), state,
                            T(g["state_slot"]), 8, 512, 128)
    cache = torch.zeros(g["kv_cache"].shape, dtype=torch.uint8, device=DEV)
    n = g["positions"].shape[0]
    ops.compress_norm_rope_store(state, n, T(g["token_to_req"]), T(g["positions"]), T(g["state_slot"]),
                                 T(g["state_block_table"]), 8, 512, T(g["cos_sin"]), cache,
                                 T(g["comp_slot"]), 2, 512, 64, 128, T(g["norm_weight"]), 1e-6)
    slots = g["comp_slot"][g["comp_slot"] >= 0]
    ours = C.read_rows(cache.cpu().numpy(), slots, 2, 512, 64)
    ref = C.read_rows(g["kv_cache"], slots, 2, 512, 64)
    assert np.linalg.norm(ours - ref) / np.linalg.norm(ref) < 2e-3
    np.testing.assert_allclose(ours, ref, rtol=2 ** -3, atol=1e-6)
    _, _, sc = _compressed_bytes(cache.cpu().numpy(), slots)
    _, _, rsc = _compressed_bytes(g["kv_cache"], slots)
    assert np.array_equal(sc, rsc)  # UE8M0 scale bytes


def _compressed_bytes(cache, slots, d=512, r=64):
    """(e4m3 NoPE codes, bf16 RoPE bytes, UE8M0 scale bytes) of each row at ``slots``."""
    nope = d - r
    row, srow = nope + 2 * r, nope // 64 + 1
    codes, rope, scales = [], [], []
    for sl in slots:
        page, off = divmod(int(sl), 2)
        codes.append(cache[page, off * row:off * row + nope])
        rope.append(cache[page, off * row + nope:(off + 1) * row])
        scales.append(cache[page, 2 * row + off * srow:2 * row + (off + 1) * srow])
    return np.array(codes), np.array(rope), np.array(scales)


def test_compressor_many_blocks_matches_reference(ops):
    """Eight blocks of the reference's head_dim-512 compressor (whole
    prefix, earlier-step states, odd offsets, shuffled state pages): the
    UE8M0 scale bytes equal, >= 99% of the e4m3 codes equal and the rest one
    step apart, RoPE within one bf16 ulp."""
    g = load("compressor_blocks_d512")
    state = T(g["state_before"])
    ops.save_partial_states(T(g["kv"]), T(g["score"]), T(g["ape"]), T(g["positions"]), state,
                            T(g["state_slot"]), 8, 512, 128)
    cache = torch.zeros(g["kv_cache"].shape, dtype=torch.uint8, device=DEV)
    n = g["positions"].shape[0]
    ops.compress_norm_rope_store(state, n, T(g["token_to_req"]), T(g["positions"]), T(g["state_slot"]),
                                 T(g["state_block_table"]), 8, 512, T(g["cos_sin"]), cache,
                                 T(g["comp_slot"]), 2, 512, 64, 128, T(g["norm_weight"]), 1e-6)
    torch.cuda.synchronize()
    slots = g["comp_slot"][g["comp_slot"] >= 0]
    assert len(slots) == 8
    got = cache.cpu().numpy()
    oc, _, osc = _compressed_bytes(got, slots)
    rc, _, rsc = _compressed_bytes(g["kv_cache"], slots)
    assert np.array_equal(osc, rsc)
    assert (oc == rc).mean() >= 0.99
    ours = C.read_rows(got, slots, 2, 512, 64)
    ref = C.read_rows(g["kv_cache"], slots, 2, 512, 64)
    np.testing.assert_allclose(ours, ref, rtol=2 ** -3, atol=1e-6)
    assert np.linalg.norm(ours - ref) / np.linalg.norm(ref) < 2e-3
    assert ops.device_error() == 0


def test_compressor_matches_oracle_d128(ops):
    rng = np.random.default_rng(5)
    d, r = 128, 64
    spans = [(0, 300), (1000, 1200)]
    pos = np.concatenate([np.arange(a, b) for a, b in spans]).astype(np.int64)
    t2r = np.concatenate([np.full(b - a, i, np.int32) for i, (a, b) in enumerate(spans)])
    bt = np.zeros((2, 160), np.int32)
    bt[0, :40] = rng.permutation(40)
    bt[1, 100:160] = 40 + rng.permutation(60)
    slot = bt[t2r, pos // 8].astype(np.int64) * 8 + pos % 8
    kv = rng.standard_normal((len(pos), d)).astype(np.float32)
    score = rng.standard_normal((len(pos), d)).astype(np.float32) * 2
    ape = rng.standard_normal((128, d)).astype(np.float32) * 0.3
    state0 = rng.standard_normal((100, 8, 2 * d)).astype(np.float32)
    cbt = rng.permutation(64).astype(np.int32).reshape(2, 32)
    cpos = pos // 128
    cslot = np.where((pos + 1) % 128 == 0, cbt[t2r, cpos // 2].astype(np.int64) * 2 + cpos % 2, -1)
    cos_sin = C.rope_cos_sin_cache(2048, r, 160000.0)
    w = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
    pb = C.page_bytes(2, d, r)
    state = T(state0)
    ops.save_partial_states(T(kv), T(score), T(ape), T(pos), state, T(slot), 8, d, 128)
    cache = torch.zeros((64, pb), dtype=torch.uint8, device=DEV)
    ops.compress_norm_rope_store(state, len(pos), T(t2r), T(pos), T(slot), T(bt), 8, d, T(cos_sin), cache,
                                 T(cslot), 2, d, r, 128, T(w), 1e-6)
    ref_state = state0.copy()
    C.save_partial_states(ref_state, kv, score, ape, pos, slot, 8, 128)
    assert np.array_equal(state.cpu().numpy(), ref_state)
    ref_cache = np.zeros((64, pb), np.uint8)
    C.compress_norm_rope_store(ref_state, t2r, pos, slot, bt, 8, w, 1e-6, cos_sin, ref_cache, cslot, 2, d, r)
    s = cslot[cslot >= 0]
    assert len(s) == 4  # boundaries 127, 255, 1023, 1151
    ours = C.read_rows(cache.cpu().numpy(), s, 2, d, r)
    ref = C.read_rows(ref_cache, s, 2, d, r)
    assert np.linalg.norm(ours - ref) / np.linalg.norm(ref) < 2e-3


# --------------------------------------------------------------------------
# norms and output path
# --------------------------------------------------------------------------


def test_qk_rmsnorm_matches_reference(ops):
    g = load("qk_rmsnorm")
    qn, kn = ops.fused_q_kv_rmsnorm(T(g["qr"], torch.bfloat16), T(g["kv"], torch.bfloat16),
                                    T(g["q_weight"], torch.bfloat16), T(g["kv_weight"], torch.bfloat16), 1e-6)
    for got, ref in ((qn, g["q_out"]), (kn, g["kv_out"])):
        got = got.float().cpu().numpy()
        np.testing.assert_allclose(got, ref, rtol=2 ** -7, atol=0)
        assert (got == ref).mean() > 0.98


def test_inv_rope_fp8_quant_matches_reference(ops):
    g = load("inv_rope_fp8_quant")
    G = int(g["n_groups"])
    o = T(g["o"], torch.bfloat16)
    t, h, d = o.shape
    data, scale = ops.fused_inv_rope_fp8_quant(o, T(g["positions"]), T(g["cos_sin"]), G, h // G, 448, 64)
    ref_data = g["fp8"].transpose(1, 0, 2)  # [T, G, D']
    got = data.contiguous().view(torch.uint8).cpu().numpy()
    assert (got == ref_data).mean() > 0.999
    got_s = scale.contiguous().cpu().numpy()  # [T, G, packs]
    ref_s = g["scale"][:, :t].transpose(1, 0, 2)
    assert np.array_equal(got_s, ref_s)


def test_vha_inv_rope_fp8_quant_matches_plugin_kernel(ops):
    g = load("vha_inv_rope_fp8_quant")
    G = int(g["n_groups"])
    o = T(g["o"], torch.bfloat16)
    t = o.shape[0]
    data, scale = ops.vha_inv_rope_fp8_quant(o, T(g["mix"], torch.bfloat16), T(g["positions"]),
                                             T(g["cos_sin"]), G, 448, 64)
    got = data.contiguous().view(torch.uint8).cpu().numpy()  # [T, G, D']
    ref = g["fp8"].transpose(1, 0, 2)
    assert (got == ref).mean() > 0.995
    got_s = scale.contiguous().cpu().numpy()  # [T, G, HPG]
    ref_s = g["scale"][:, :, :t].transpose(2, 0, 1)
    assert (got_s == ref_s).mean() > 0.99
    # dequantised relative L2 like the plugin's own test (< 0.03)
    deq = lambda q, s: (e4m3_to_f32(q).reshape(t, G, 8, 4, 128) *
                        np.exp2((np.ascontiguousarray(s).view(np.uint8).reshape(t, G, 8, 4).astype(np.float64)
                                 - 127))[..., None])
    a, b = deq(got, got_s), deq(ref, ref_s)
    assert np.linalg.norm(a - b) / np.linalg.norm(b) < 0.03


@pytest.mark.parametrize("head_dim,t", [(128, 13), (512, 13), (128, 1501), (512, 1501), (128, 4099)])
def test_vha_inv_rope_fp8_quant_matches_oracle(ops, head_dim, t):
    # 1501 / 4099 tokens: several tokens per CTA (double-buffered loads), ragged last CTA
    rng = np.random.default_rng(head_dim + 7 + t)
    h, G, r = 64, 8, 64
    o = bf16_round(rng.standard_normal((t, h, head_dim)).astype(np.float32))
    u = rng.standard_normal((h, 16)).astype(np.float32) / 8
    v = rng.standard_normal((h, 16)).astype(np.float32) / 8
    mix = bf16_round(np.eye(h, dtype=np.float32) + v @ u.T)
    pos = rng.integers(0, 4000, size=t)
    cos_sin = C.rope_cos_sin_cache(4096, r, 160000.0)
    data, scale = ops.vha_inv_rope_fp8_quant(T(o, torch.bfloat16), T(mix, torch.bfloat16), T(pos), T(cos_sin),
                                             G, head_dim - r, r)
    q_ref, exp_ref = O.vha_inv_rope_fp8_quant(o, mix, pos, cos_sin, G, r)
    got = data.contiguous().view(torch.uint8).cpu().numpy()
    assert (got == q_ref.transpose(1, 0, 2)).mean() > 0.995
    packed = O.pack_scale_exponents(exp_ref).reshape(t, G, h // G)
    assert (scale.contiguous().cpu().numpy() == packed).mean() > 0.99
    # bf16 output variant (no quant)
    y = ops.vha_inv_rope(T(o, torch.bfloat16), T(mix, torch.bfloat16), T(pos), T(cos_sin), r)
    y_ref = O.inv_rope_fp8_quant(np.einsum("hg,tgd->thd", mix, o), pos, cos_sin, G, r, quant=False)
    np.testing.assert_allclose(y.float().cpu().numpy(), y_ref, rtol=2 ** -7, atol=1e-5)


@pytest.mark.parametrize("heads,groups,t", [(64, 8, 1900), (32, 4, 1900), (16, 4, 1900), (64, 8, 1901)])
def test_vha_fp8_quant_streamed_matches_per_token_kernel(ops, heads, groups, t):
    """At >= 1024 tokens (D=128) the library takes the streamed VHA kernel
    (persistent CTAs, bulk row copies, 16 heads x 128 dims per warp, several
    token groups per CTA below 64 heads); below it the per-token-block
    kernel.  The same tokens run in calls of < 1024 tokens must give the
    identical e4m3 bytes and scales; the scale rows of the padding tokens up
    to the next multiple of 4 are zero."""
    rng = np.random.default_rng(heads + t)
    d, r = 128, 64
    o = T(bf16_round(rng.standard_normal((t, heads, d)).astype(np.float32)), torch.bfloat16)
    u = rng.standard_normal((heads, 16)).astype(np.float32) / 8
    v = rng.standard_normal((heads, 16)).astype(np.float32) / 8
    mix = T(bf16_round(np.eye(heads, dtype=np.float32) + v @ u.T), torch.bfloat16)
    pos = T(rng.integers(0, 4000, size=t))
    cs = T(C.rope_cos_sin_cache(4096, r, 160000.0))
    data, scale = ops.vha_inv_rope_fp8_quant(o, mix, pos, cs, groups, d - r, r)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    got_d = data.contiguous().view(torch.uint8).cpu().numpy()
    got_s = scale.contiguous().cpu().numpy()
    # scale is a [t] view of a [groups, hpg, aligned(t)] buffer: its padding columns
    full = torch.as_strided(scale, (groups, heads // groups, (t + 3) // 4 * 4),
                            (scale.stride(1), scale.stride(2), scale.stride(0))).cpu().numpy()
    assert not full[:, :, t:].any()
    for a, b in ((0, 1000), (1000, t)):
        d2, s2 = ops.vha_inv_rope_fp8_quant(o[a:b], mix, pos[a:b], cs, groups, d - r, r)
        assert np.array_equal(got_d[a:b], d2.contiguous().view(torch.uint8).cpu().numpy())
        assert np.array_equal(got_s[a:b], s2.contiguous().cpu().numpy())


@pytest.mark.parametrize("name", ["sigmoid_mul_quant_5x1024", "sigmoid_mul_quant_13x2048"])
def test_sigmoid_mul_quant_bitwise(ops, name):
    g = load(name)
    q, s = ops.sigmoid_mul_quant_fp8(T(g["x"], torch.bfloat16), T(g["gate"], torch.bfloat16))
    assert np.array_equal(s.cpu().numpy(), g["scale"])
    assert np.array_equal(q.view(torch.uint8).cpu().numpy(), g["fp8"])


def test_unsupported_dims_raise(ops):
    from vllm_ernie_b200 import HcaError

    k = torch.zeros((4, 96), dtype=torch.bfloat16, device=DEV)
    cache = torch.zeros((1, 4096), dtype=torch.uint8, device=DEV)
    with pytest.raises(HcaError):
        ops.quantize_and_insert_k_cache(k, cache, torch.zeros(4, dtype=torch.int64, device=DEV), 8, 32)


# --------------------------------------------------------------------------
# fused decode prep == the three cache ops in sequence (same bytes)
# --------------------------------------------------------------------------


@pytest.mark.parametrize("head_dim,heads,padded", [(128, 64, 64), (128, 16, 64), (512, 64, 64)])
def test_decode_prep_matches_three_ops(ops, head_dim, heads, padded):
    """q, SWA cache, compressor state and compressed cache after
    hca_decode_prep equal, byte for byte, those after
    hca_qnorm_rope_kv_insert + hca_save_partial_states +
    hca_compress_norm_rope_store on the same inputs.  Contexts put block
    boundaries on the first, middle and last query token of a request (the
    pooled states include ones saved in the same launch)."""
    from vllm_ernie_b200.decode import build_decode_metadata
    from vllm_ernie_b200.synthetic import HCADims, alloc_layer_caches, make_decode_batch, rope_cos_sin_cache

    dims = HCADims(heads=heads, head_dim=head_dim)
    ctx = [0, 125, 126, 127, 253, 1022, 5000, 130000 - 2, 77]
    b = make_decode_batch(ctx, 3, dims, DEV, seed=7, max_model_len=1024 * 128)
    caches = alloc_layer_caches(b, seed=8)
    md = build_decode_metadata(b, 1024, num_splits=1)
    n = b.num_tokens
    assert (((b.positions + 1) % 128 == 0).sum() >= 4)
    g = torch.Generator(device=DEV).manual_seed(9)
    q = torch.randn((n, heads, head_dim), generator=g, device=DEV).to(torch.bfloat16)
    kv = torch.randn((n, head_dim), generator=g, device=DEV).to(torch.bfloat16)
    ks = torch.randn((n, 2 * head_dim), generator=g, device=DEV)
    ape = torch.randn((128, head_dim), generator=g, device=DEV) * 0.1
    w = 1.0 + 0.05 * torch.randn(head_dim, generator=g, device=DEV)
    cs = rope_cos_sin_cache(1024 * 128 + 8, 64, dims.rope_theta, DEV)
    a = [t.clone() for t in (caches.swa, caches.state, caches.comp)]
    f = [t.clone() for t in (caches.swa, caches.state, caches.comp)]
    qa = ops.fused_qnorm_rope_kv_insert(q, kv, a[0], md.swa_slot, b.positions, cs, padded, 1e-6, 64, 64)
    ops.save_partial_states(ks[:, :head_dim], ks[:, head_dim:], ape, b.positions, a[1], md.state_slot, 8,
                            head_dim, 128)
    ops.compress_norm_rope_store(a[1], n, md.token_to_req, b.positions, md.state_slot, b.state_bt, 8, head_dim, cs,
                                 a[2], md.comp_slot, 2, head_dim, 64, 128, w, 1e-6)
    qf = ops.decode_prep(q, kv, ks, ape, b.positions, cs, f[0], md.swa_slot, 64, f[1], md.state_slot, b.state_bt, 8,
                         f[2], md.comp_slot, 2, w, b.query_start_loc, md.token_to_req, b.num_reqs, padded, 1e-6,
                         128, 64)
    torch.cuda.synchronize()
    assert torch.equal(qa.view(torch.int16), qf.view(torch.int16))
    for x, y in zip(a, f):
        assert torch.equal(x.view(torch.uint8), y.view(torch.uint8))
    # the launch did write: boundaries produced compressed rows, states moved
    assert not torch.equal(f[2], caches.comp) and not torch.equal(f[1], caches.state)


def test_decode_prep_ragged_requests_match_three_ops(ops):
    """Requests with 1, 2 or 3 query tokens in one batch (ragged
    query_start_loc), block ends on their first / last / only token: the
    fused launch still writes the bytes of the three separate ops."""
    from vllm_ernie_b200.decode import build_decode_metadata
    from vllm_ernie_b200.synthetic import HCADims, alloc_layer_caches, make_decode_batch, rope_cos_sin_cache

    dims = HCADims(heads=64, head_dim=128)
    ctx = [0, 125, 126, 127, 253, 1022, 5000, 77, 383]
    keep = [1, 3, 2, 1, 3, 2, 3, 1, 1]  # tokens kept per request
    b = make_decode_batch(ctx, 3, dims, DEV, seed=17, max_model_len=1024 * 128)
    caches = alloc_layer_caches(b, seed=18)
    md = build_decode_metadata(b, 1024, num_splits=1)
    sel = torch.tensor([r * 3 + j for r, k in enumerate(keep) for j in range(k)], device=DEV)
    qsl = torch.tensor(np.concatenate([[0], np.cumsum(keep)]), dtype=torch.int32, device=DEV)
    t2r = torch.tensor([r for r, k in enumerate(keep) for _ in range(k)], dtype=torch.int32, device=DEV)
    pos, swa_slot, st_slot, c_slot = (x[sel].contiguous() for x in (b.positions, md.swa_slot, md.state_slot, md.comp_slot))
    assert int(((pos + 1) % 128 == 0).sum()) >= 3
    n = sel.numel()
    g = torch.Generator(device=DEV).manual_seed(19)
    q = torch.randn((n, 64, 128), generator=g, device=DEV).to(torch.bfloat16)
    kv = torch.randn((n, 128), generator=g, device=DEV).to(torch.bfloat16)
    ks = torch.randn((n, 256), generator=g, device=DEV)
    ape = torch.randn((128, 128), generator=g, device=DEV) * 0.1
    w = 1.0 + 0.05 * torch.randn(128, generator=g, device=DEV)
    cs = rope_cos_sin_cache(1024 * 128 + 8, 64, dims.rope_theta, DEV)
    a = [t.clone() for t in (caches.swa, caches.state, caches.comp)]
    f = [t.clone() for t in (caches.swa, caches.state, caches.comp)]
    qa = ops.fused_qnorm_rope_kv_insert(q, kv, a[0], swa_slot, pos, cs, 64, 1e-6, 64, 64)
    ops.save_partial_states(ks[:, :128], ks[:, 128:], ape, pos, a[1], st_slot, 8, 128, 128)
    ops.compress_norm_rope_store(a[1], n, t2r, pos, st_slot, b.state_bt, 8, 128, cs, a[2], c_slot, 2, 128, 64, 128,
                                 w, 1e-6)
    qf = ops.decode_prep(q, kv, ks, ape, pos, cs, f[0], swa_slot, 64, f[1], st_slot, b.state_bt, 8, f[2], c_slot, 2, w,
                         qsl, t2r, len(keep), 64, 1e-6, 128, 64)
    torch.cuda.synchronize()
    assert torch.equal(qa.view(torch.int16), qf.view(torch.int16))
    for x, y in zip(a, f):
        assert torch.equal(x.view(torch.uint8), y.view(torch.uint8))


def test_decode_prep_rejected_drafts_are_rewritten(ops):
    """ECHO/MTP rewrites: step A writes a token and its two drafts (KV rows,
    compressor states, and any block a draft completes); the drafts are
    rejected and step B re-submits those positions with new values plus the
    next one.  The caches after A then B equal, byte for byte, those after
    writing only the accepted token and then B: a block completed by a
    rejected draft is recomputed from the rewritten states."""
    from vllm_ernie_b200.decode import build_decode_metadata
    from vllm_ernie_b200.synthetic import HCADims, alloc_layer_caches, make_decode_batch, rope_cos_sin_cache

    dims = HCADims(heads=64, head_dim=128)
    ctx = [124, 125, 126, 127, 1000, 5000]  # block ends on token 3, 2, 1, 0 (positions ctx .. ctx + 3)
    b = make_decode_batch(ctx, 4, dims, DEV, seed=27, max_model_len=64 * 128)
    caches = alloc_layer_caches(b, seed=28)
    md = build_decode_metadata(b, 64, num_splits=1)
    R = len(ctx)
    g = torch.Generator(device=DEV).manual_seed(29)
    ape = torch.randn((128, 128), generator=g, device=DEV) * 0.1
    w = 1.0 + 0.05 * torch.randn(128, generator=g, device=DEV)
    cs = rope_cos_sin_cache(64 * 128 + 8, 64, dims.rope_theta, DEV)

    def inputs(n):
        return (torch.randn((n, 64, 128), generator=g, device=DEV).to(torch.bfloat16),
                torch.randn((n, 128), generator=g, device=DEV).to(torch.bfloat16),
                torch.randn((n, 256), generator=g, device=DEV))

    def run(cache, tokens_per_req, first, inp):
        sel = torch.tensor([r * 4 + first + j for r in range(R) for j in range(tokens_per_req)], device=DEV)
        qsl = torch.arange(0, R + 1, dtype=torch.int32, device=DEV) * tokens_per_req
        t2r = torch.arange(R, dtype=torch.int32, device=DEV).repeat_interleave(tokens_per_req)
        q, kv, ks = inp
        ops.decode_prep(q, kv, ks, ape, b.positions[sel].contiguous(), cs, cache[0], md.swa_slot[sel].contiguous(),
                        64, cache[1], md.state_slot[sel].contiguous(), b.state_bt, 8, cache[2],
                        md.comp_slot[sel].contiguous(), 2, w, qsl, t2r, R, 64, 1e-6, 128, 64)

    a_in = inputs(3 * R)   # accepted token + two drafts per request
    b_in = inputs(3 * R)   # the rewrite: drafts' positions with new values, plus the next position
    first_only = tuple(x.view(R, 3, *x.shape[1:])[:, :1].reshape(R, *x.shape[1:]).contiguous() for x in a_in)
    got = [t.clone() for t in (caches.swa, caches.state, caches.comp)]
    ref = [t.clone() for t in (caches.swa, caches.state, caches.comp)]
    run(got, 3, 0, a_in)
    run(got, 3, 1, b_in)
    run(ref, 1, 0, first_only)
    run(ref, 3, 1, b_in)
    torch.cuda.synchronize()
    for x, y in zip(got, ref):
        assert torch.equal(x.view(torch.uint8), y.view(torch.uint8))
    # the drafts did write (a block completed by a draft was computed, then recomputed)
    mid = [t.clone() for t in (caches.swa, caches.state, caches.comp)]
    run(mid, 3, 0, a_in)
    torch.cuda.synchronize()
    assert not torch.equal(mid[2], ref[2])
