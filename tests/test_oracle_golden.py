"""Pin the CPU oracle against golden vectors from the reference's own kernels.

The fixtures under ``tests/golden`` were produced by
``tests/golden/make_golden.py`` (reference Triton kernels under the Triton
CPU interpreter).  Integer/byte outputs must match bit-exactly; floating
point outputs within the stated tolerances.
"""

import numpy as np
import pytest

from golden_io import load
from oracle import cache as C
from oracle import metadata as M
from oracle import output as O
from oracle.fp8 import bf16_round, e4m3_to_f32

D, R = 512, 64


def test_kv_insert_bytes_match_reference():
    g = load("kv_insert_gather")
    page = int(g["page"])
    cache = np.zeros_like(g["cache"])
    C.insert_rows(cache, g["slots"], g["k"], page, D, R)
    assert np.array_equal(cache, g["cache"])


def test_dequant_gather_matches_reference():
    g = load("kv_insert_gather")
    page = int(g["page"])
    out = np.zeros_like(g["gathered"])
    C.dequantize_and_gather(g["cache"], g["seq_lens"], g["gather_lens"], g["block_table"], page, 5,
                            out, D, R)
    assert np.array_equal(bf16_round(out), g["gathered"])


def test_save_partial_states_matches_reference():
    g = load("compressor")
    state = g["state_before"].copy()
    C.save_partial_states(state, g["kv"], g["score"], g["ape"], g["positions"], g["state_slot"], 8, 128)
    flat = state.reshape(-1, 2 * D)
    slots = g["state_slot"]
    ok = slots >= 0
    assert np.array_equal(flat[slots[ok]], g["state_rows_written"][ok])


def test_compressor_matches_reference():
    """Compressed rows: RoPE bf16 within 1 ulp, NoPE scale bytes equal and
    fp8 codes within one step (fp32 softmax/rsqrt ordering may differ)."""
    g = load("compressor")
    state = g["state_before"].copy()
    C.save_partial_states(state, g["kv"], g["score"], g["ape"], g["positions"], g["state_slot"], 8, 128)
    cache = np.zeros_like(g["kv_cache"])
    C.compress_norm_rope_store(state, g["token_to_req"], g["positions"], g["state_slot"],
                               g["state_block_table"], 8, g["norm_weight"], 1e-6, g["cos_sin"],
                               cache, g["comp_slot"], 2, D, R, 128)
    slots = g["comp_slot"][g["comp_slot"] >= 0]
    assert len(slots) == 3
    ours = C.read_rows(cache, slots, 2, D, R)
    ref = C.read_rows(g["kv_cache"], slots, 2, D, R)
    np.testing.assert_allclose(ours, ref, rtol=2 ** -3, atol=1e-6)
    rel = np.linalg.norm(ours - ref) / np.linalg.norm(ref)
    assert rel < 2e-3
    # scale bytes
    for s in slots:
        page, off = divmod(int(s), 2)
        sb = 2 * 576 + off * 8
        assert np.array_equal(cache[page, sb:sb + 8], g["kv_cache"][page, sb:sb + 8])


def _compressed_bytes(cache, slots, d=D, r=R):
    """(e4m3 NoPE codes, bf16 RoPE bytes, UE8M0 scale bytes) of each row at ``slots``."""
    nope = d - r
    row, srow = nope + 2 * r, nope // 64 + 1
    codes, rope, scales = [], [], []
    for s in slots:
        page, off = divmod(int(s), 2)
        base = off * row
        codes.append(cache[page, base:base + nope])
        rope.append(cache[page, base + nope:base + row])
        sb = 2 * row + off * srow
        scales.append(cache[page, sb:sb + srow])
    return np.array(codes), np.array(rope), np.array(scales)


def test_compressor_many_blocks_matches_reference():
    """Eight blocks (whole prefix, earlier-step states, odd offsets, shuffled
    state pages): UE8M0 scale bytes equal; e4m3 codes within one step with
    >= 99% equal; RoPE within one bf16 ulp."""
    g = load("compressor_blocks_d512")
    state = g["state_before"].copy()
    C.save_partial_states(state, g["kv"], g["score"], g["ape"], g["positions"], g["state_slot"], 8, 128)
    cache = np.zeros_like(g["kv_cache"])
    C.compress_norm_rope_store(state, g["token_to_req"], g["positions"], g["state_slot"],
                               g["state_block_table"], 8, g["norm_weight"], 1e-6, g["cos_sin"],
                               cache, g["comp_slot"], 2, D, R, 128)
    slots = g["comp_slot"][g["comp_slot"] >= 0]
    assert len(slots) == 8
    oc, orope, osc = _compressed_bytes(cache, slots)
    rc, rrope, rsc = _compressed_bytes(g["kv_cache"], slots)
    assert np.array_equal(osc, rsc)
    assert (oc == rc).mean() >= 0.99
    ours = C.read_rows(cache, slots, 2, D, R)
    ref = C.read_rows(g["kv_cache"], slots, 2, D, R)
    np.testing.assert_allclose(ours, ref, rtol=2 ** -3, atol=1e-6)
    assert np.linalg.norm(ours - ref) / np.linalg.norm(ref) < 2e-3


def test_metadata_builders_bit_exact():
    g = load("metadata")
    qsl, seq_lens = g["query_start_loc"], g["seq_lens"]
    T = int(qsl[-1])
    nd, ndt = int(g["num_decodes"]), int(g["num_decode_tokens"])
    t2r = M.token_to_req_indices(qsl)
    assert np.array_equal(t2r, g["token_to_req"])
    cs = M.compressed_slot_mapping(T, qsl, seq_lens, g["comp_block_table"], 2, 128)
    assert np.array_equal(cs, g["comp_slot"][:T])

    idx = np.full((T, 128), 777, np.int32)
    lens = np.full(T, 99, np.int32)
    M.swa_indices_and_lens(ndt, 128, qsl, seq_lens, t2r, g["slot_mapping"] >= 0,
                           g["swa_block_table"], 64, idx, lens)
    assert np.array_equal(lens, g["swa_lens"])
    assert np.array_equal(idx, g["swa_indices"])

    maxc = int(g["max_compressed"])
    gd = np.full((T, maxc), 555, np.int32)
    dl = np.full(T, 555, np.int32)
    pl = np.full((T, maxc), 555, np.int32)
    M.c128a_topk_metadata(g["positions"], 128, ndt, t2r, g["comp_block_table"][:nd], 2,
                          g["slot_mapping"], gd, dl, pl, maxc)
    assert np.array_equal(gd[:ndt], g["c128a_global"][:ndt])
    assert np.array_equal(dl[:ndt], g["c128a_lens"][:ndt])
    assert np.array_equal(pl[: T - ndt], g["c128a_prefill"][: T - ndt])

    gl = M.prefill_gather_lens(seq_lens, qsl, 2, nd, 128)
    assert np.array_equal(gl, g["gather_lens"])
    comb, clens = M.combine_topk_swa_indices(g["c128a_prefill"][: T - ndt], qsl[nd:], seq_lens[nd:],
                                             gl, 128, 128, maxc, int(g["M"]), int(g["N"]))
    assert np.array_equal(comb, g["combined"])
    assert np.array_equal(clens, g["combined_lens"])


def test_qk_rmsnorm_matches_reference():
    g = load("qk_rmsnorm")
    q = bf16_round(O.rms_norm(g["qr"], g["q_weight"], 1e-6))
    k = bf16_round(O.rms_norm(g["kv"], g["kv_weight"], 1e-6))
    # one bf16 ulp (rsqrt rounding)
    np.testing.assert_allclose(q, g["q_out"], rtol=2 ** -7, atol=0)
    np.testing.assert_allclose(k, g["kv_out"], rtol=2 ** -7, atol=0)
    assert (q == g["q_out"]).mean() > 0.98


def _dequant_groups(fp8, exp_bytes):
    return e4m3_to_f32(fp8) * np.ldexp(1.0, exp_bytes.astype(np.int32) - 127)


def test_inv_rope_fp8_quant_matches_reference():
    g = load("inv_rope_fp8_quant")
    G = int(g["n_groups"])
    q, exp = O.inv_rope_fp8_quant(g["o"], g["positions"], g["cos_sin"], G, R)
    T, H = g["o"].shape[:2]
    hpg = H // G
    # reference scale: [G, aligned_T, packs] int32, byte c of pack k = chunk 4k + c
    ref_bytes = g["scale"].view(np.uint8).reshape(G, -1, g["scale"].shape[-1] * 4)[:, :T]
    ours_bytes = (exp + 127).astype(np.uint8).reshape(T, G, hpg * (D // 128)).transpose(1, 0, 2)
    assert np.array_equal(ours_bytes, ref_bytes[..., : hpg * (D // 128)])
    assert (q == g["fp8"]).mean() > 0.999
    assert np.abs(e4m3_to_f32(q).astype(np.float64) - e4m3_to_f32(g["fp8"])).max() <= 32


def test_vha_inv_rope_fp8_quant_matches_plugin_kernel():
    g = load("vha_inv_rope_fp8_quant")
    G = int(g["n_groups"])
    q, exp = O.vha_inv_rope_fp8_quant(g["o"], g["mix"], g["positions"], g["cos_sin"], G, R)
    T, H = g["o"].shape[:2]
    hpg = H // G
    packed = O.pack_scale_exponents(exp)  # [T, H]
    ref = g["scale"][:, :, :T].transpose(2, 0, 1).reshape(T, H)
    assert (packed == ref).mean() > 0.99
    assert (q == g["fp8"]).mean() > 0.995


@pytest.mark.parametrize("name", ["sigmoid_mul_quant_5x1024", "sigmoid_mul_quant_13x2048"])
def test_sigmoid_mul_quant_matches_plugin_kernel(name):
    g = load(name)
    q, s = O.sigmoid_mul_quant_fp8(g["x"], g["gate"])
    assert np.array_equal(s, g["scale"])
    assert np.array_equal(q, g["fp8"])


def test_layer_oracle_emulated_vs_exact():
    """The whole-layer oracle (config 1, prefill 1024 + 640 from an empty
    cache): the evaluation with the reference kernels' FP8/UE8M0 and bf16
    roundings stays close to the all-fp32 one, and both are finite."""
    import torch

    from oracle.layer import HCALayerOracle, HCAShape, random_weights

    shape = HCAShape()
    w = random_weights(shape, seed=0)
    g = torch.Generator().manual_seed(1)
    h = torch.randn(1664, 2048, generator=g).to(torch.bfloat16).float().numpy()
    qsl, sl = np.array([0, 1024, 1664]), np.array([1024, 640])
    em = HCALayerOracle(shape, w, max_len=1152, num_reqs=2, emulate_quant=True).forward(h, qsl, sl)
    ex = HCALayerOracle(shape, w, max_len=1152, num_reqs=2, emulate_quant=False).forward(h, qsl, sl)
    assert np.isfinite(em).all() and np.isfinite(ex).all()
    assert np.linalg.norm(em - ex) / np.linalg.norm(ex) < 5e-2


def bf16_bits_to_f32(a: np.ndarray) -> np.ndarray:
    return (a.astype(np.uint32) << 16).view(np.float32)


# The attention fixtures run vLLM's readable DeepSeek-V4 sparse attention
# (rocm_aiter_mla_sparse.py, Triton) in fp32 with bf16 P and a bf16 output;
# the oracle evaluates in fp64.  Parity bar for the attention output:
ATTN_MAX_ABS, ATTN_MAX_REL_L2 = 2e-2, 5e-3


def _check_attn(ours: np.ndarray, ref: np.ndarray) -> None:
    assert np.isfinite(ours).all() and np.isfinite(ref).all()
    err = np.abs(ours.astype(np.float64) - ref)
    rel = np.linalg.norm(ours.astype(np.float64) - ref) / max(np.linalg.norm(ref), 1e-30)
    assert err.max() <= ATTN_MAX_ABS and rel <= ATTN_MAX_REL_L2, (err.max(), rel)


def test_decode_attention_index_tables_match_reference():
    """The decode fixture's window and compressed index tables, rebuilt by
    the oracle's builders (bit-exact)."""
    g = load("sparse_decode_d512")
    qsl, seq_lens = g["query_start_loc"], g["seq_lens"]
    T = int(qsl[-1])
    t2r = M.token_to_req_indices(qsl)
    idx = np.full((T, 128), -1, np.int32)
    lens = np.zeros(T, np.int32)
    M.swa_indices_and_lens(T, 128, qsl, seq_lens, t2r, g["slot_mapping"] >= 0, g["swa_block_table"], 64,
                           idx, lens)
    assert np.array_equal(lens, g["swa_lens"]) and np.array_equal(idx, g["swa_indices"])
    gd = np.full((T, 128), -1, np.int32)
    dl = np.zeros(T, np.int32)
    M.c128a_topk_metadata(g["positions"], 128, T, t2r, g["comp_block_table"], 2, g["slot_mapping"], gd, dl,
                          np.zeros((1, 128), np.int32), 128)
    assert np.array_equal(dl, g["comp_lens"]) and np.array_equal(gd, g["comp_indices"])
    # the cases the fixture is meant to hold
    assert (g["swa_lens"] == 0).any() and (g["comp_lens"] == 0).any() and g["swa_lens"].max() == 128
    assert len(set(g["comp_lens"][:3].tolist())) == 2  # a compression boundary between MTP tokens


@pytest.mark.parametrize("sink", ["random", "neginf", "none"])
def test_oracle_sparse_decode_matches_reference_kernel(sink):
    from oracle import attention as A

    g = load("sparse_decode_d512")
    q = bf16_bits_to_f32(g["q"])
    sk = {"random": g["sink"], "neginf": np.full_like(g["sink"], -np.inf), "none": None}[sink]
    ours = A.sparse_decode(q, g["swa_cache"], 64, g["swa_indices"], g["swa_lens"], g["comp_cache"], 2,
                           g["comp_indices"], g["comp_lens"], float(g["scale"]), sk, D, R)
    ref = bf16_bits_to_f32(g[f"out_{sink}"])
    _check_attn(ours, ref)
    empty = g["swa_lens"] == 0
    assert np.array_equal(ref[empty], np.zeros_like(ref[empty]))


@pytest.mark.parametrize("sink", ["random", "neginf", "none"])
def test_oracle_sparse_prefill_matches_reference_kernel(sink):
    """The oracle's prefill straight on the paged caches against the
    reference's gather-workspace pipeline (dequant gather, combined
    indices, sparse prefill kernel)."""
    from oracle import attention as A

    g = load("sparse_prefill_d512")
    q = bf16_bits_to_f32(g["q"])
    sk = {"random": g["sink"], "neginf": np.full_like(g["sink"], -np.inf), "none": None}[sink]
    ours = A.sparse_prefill_paged(q, g["positions"], g["token_to_req"], g["swa_cache"], 64,
                                  g["swa_block_table"], g["comp_cache"], 2, g["comp_block_table"], 128, 128,
                                  float(g["scale"]), sk, D, R)
    _check_attn(ours, bf16_bits_to_f32(g[f"out_{sink}"]))
