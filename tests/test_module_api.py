"""CPU checks of the drop-in module and backend API (no kernels launched).

Mirrors the reference's own tests of this boundary:
* page-stride alignment shared by every layer (``tests/models/ernie5_5/test_dsa_backend.py:40-55``);
* TP divisibility errors (``tests/models/ernie5_5/test_vha_tp.py:84-95``);
* VHA low-rank TP mixing vs the folded TP=1 mix (``test_vha_tp.py:55-81``), here
  as two ``gloo`` ranks on the CPU;
plus the KV-cache specs, class selection, parameter names the checkpoint mapper
fills, sharded weight loading and the decode/prefill split.
"""

import os
import socket
from types import SimpleNamespace

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from vllm_ernie_b200 import attention as A
from vllm_ernie_b200 import backend as B

NUM_HEADS = 64
RANK = 16


def _config1():
    return A.Ernie5_5HCAConfig(hidden_size=2048, num_hidden_layers=2, num_attention_heads=16, head_dim=128,
                               q_lora_rank=512, qk_rope_head_dim=64, o_groups=4, o_lora_rank=64,
                               hybrid_mla_num_attention_heads=16, num_nextn_predict_layers=0)


def test_kv_cache_specs_and_shapes():
    specs = B.hca_kv_cache_specs(512, 64)
    comp, swa, st = specs["compressed"], specs["swa"], specs["compressor_state"]
    assert comp.head_size == 584 and comp.compress_ratio == 128 and comp.block_size == 256
    assert comp.storage_block_size == 2 and comp.dtype == torch.uint8
    assert swa.block_size == 64 and swa.sliding_window == 128 and swa.head_size == 584
    assert st.dtype == torch.float32 and st.block_size == 8 and st.head_size == 1024 and st.sliding_window == 128
    for s in specs.values():
        assert s.page_size_bytes % 576 == 0
        assert s.page_size_bytes >= s.storage_block_size * s.head_size * (4 if s.dtype == torch.float32 else 1)
    assert B.get_kv_cache_shape(10, 64, 1, 512) == (10, 64, 584)
    assert B.hca_kv_cache_specs(128, 64)["swa"].head_size == 194


def test_packed_block_stride_alignment_fits_every_layer_row():
    cfg = SimpleNamespace(model_config=SimpleNamespace(
        hf_config=SimpleNamespace(head_dim=512, mla_kv_lora_rank=512, mla_qk_rope_head_dim=64)))
    a = B.packed_block_stride_alignment(cfg)
    assert a % 512 == 0 and a % (512 * 2) == 0 and a % ((512 + 64) * 2) == 0


@pytest.mark.parametrize("tp_size", [3, 16])
def test_attn_tp_must_divide_groups_and_heads(tp_size):
    config = SimpleNamespace(o_groups=8, num_attention_heads=64, hybrid_mla_num_attention_heads=64)
    with pytest.raises(ValueError, match=f"TP size {tp_size} must divide o_groups"):
        A._check_attn_tp(config, tp_size)


def test_attn_tp_divisors_accepted():
    config = SimpleNamespace(o_groups=8, num_attention_heads=64, hybrid_mla_num_attention_heads=64)
    for tp in (1, 2, 4, 8):
        A._check_attn_tp(config, tp)
    A._check_attn_tp(config)  # no process group: TP = 1


def test_select_class():
    assert A.select_ernie5_5_hca_cls("fp8") is A.Ernie5_5HCAAttention
    assert A.select_ernie5_5_hca_cls("fp8_ds_mla") is A.Ernie5_5HCAAttention
    with pytest.raises(ValueError):
        A.select_ernie5_5_hca_cls("auto")


def test_module_parameter_names_and_loading():
    cfg = _config1()
    vc = A.make_vllm_config(cfg, max_model_len=4096)
    layer = A.Ernie5_5HCAAttention(vc, prefix="model.layers.0.self_attn")
    names = set(dict(layer.named_parameters()))
    # the names the plugin's checkpoint mapper fills (E/nvidia/model.py:656-704)
    expected = {"fused_wqa_wkv.weight", "q_norm.weight", "wq_b.weight", "kv_norm.weight", "wo_a.weight",
                "wo_b.weight", "o_gate.weight", "vha.U", "vha.V", "attn_sink", "compressor.ape",
                "compressor.fused_wkv_wgate.weight", "compressor.norm.weight"}
    assert expected <= names, expected - names
    spec = layer.get_kv_cache_spec()
    assert spec["swa"].head_size == 194 and spec["compressed"].compress_ratio == 128
    g = torch.Generator().manual_seed(0)
    wq = torch.randn(512, 2048, generator=g).bfloat16()
    wkv = torch.randn(128, 2048, generator=g).bfloat16()
    loaded = layer.load_weights([("fused_wqa_wkv.weight", wq, 0), ("fused_wqa_wkv.weight", wkv, 1),
                                 ("attn_sink", torch.arange(16.0))])
    assert loaded == {"fused_wqa_wkv.weight", "attn_sink"}
    w = layer.fused_wqa_wkv.weight
    assert torch.equal(w[:512], wq) and torch.equal(w[512:], wkv)
    assert torch.equal(layer.attn_sink[:16], torch.arange(16.0))
    # a non-HCA compress ratio is refused
    cfg2 = _config1()
    cfg2.compress_ratios = [4, 4]
    with pytest.raises(ValueError):
        A.Ernie5_5HCAAttention(A.make_vllm_config(cfg2, max_model_len=4096), prefix="model.layers.1.self_attn")


def test_vha_fold_is_identity_plus_low_rank_and_idempotent():
    vha = A.VHAPostMix(NUM_HEADS)
    g = torch.Generator().manual_seed(1)
    u = torch.randn(NUM_HEADS, RANK, generator=g) * 0.1
    v = torch.randn(NUM_HEADS, RANK, generator=g) * 0.1
    vha.U.weight_loader(vha.U, u)
    vha.V.weight_loader(vha.V, v)
    vha.fold()
    addr = vha.m.data_ptr()
    vha.fold()
    assert vha.m.data_ptr() == addr
    torch.testing.assert_close(vha.m, torch.eye(NUM_HEADS) + v @ u.t())
    o = torch.randn(5, NUM_HEADS, 128, generator=g)
    torch.testing.assert_close(vha(o), vha.m @ o)


def test_split_decodes_and_prefills():
    qsl = torch.tensor([0, 3, 6, 9, 109, 209], dtype=torch.int32)
    cm = B.CommonAttentionMetadata(query_start_loc=qsl, query_start_loc_cpu=qsl, seq_lens=qsl[1:], num_reqs=5,
                                   num_actual_tokens=209, max_query_len=100, block_table_tensor=torch.zeros(5, 1),
                                   slot_mapping=torch.zeros(209, dtype=torch.int64))
    assert B.split_decodes_and_prefills(cm, decode_threshold=3) == (3, 2, 9, 200)
    assert B.split_decodes_and_prefills(cm, decode_threshold=1) == (0, 5, 0, 209)


# --------------------------------------------------------------------------- TP on gloo


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(num_tokens):
    g = torch.Generator().manual_seed(0)
    u = (torch.randn(NUM_HEADS, RANK, generator=g) * 0.1).bfloat16()
    v = (torch.randn(NUM_HEADS, RANK, generator=g) * 0.1).bfloat16()
    o = torch.randn(num_tokens, NUM_HEADS, 128, generator=g).bfloat16()
    return u, v, o


def _vha_tp_worker(rank, world_size, port, num_tokens, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world_size)
    try:
        vha = A.VHAPostMix(NUM_HEADS, tp_group=dist.group.WORLD).bfloat16()
        u, v, o = _inputs(num_tokens)
        vha.U.weight_loader(vha.U, u)
        vha.V.weight_loader(vha.V, v)
        vha.fold()  # a no-op under TP
        heads = NUM_HEADS // world_size
        out[rank] = vha(o[:, rank * heads:(rank + 1) * heads]).float()
        # the layer checks TP divisibility against the live group
        A._check_attn_tp(SimpleNamespace(o_groups=8, num_attention_heads=64, hybrid_mla_num_attention_heads=64))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("num_tokens", [1, 37])
def test_vha_tp_matches_folded_mix_gloo(num_tokens):
    world_size = 2
    with mp.get_context("spawn").Manager() as manager:
        out = manager.dict()
        mp.spawn(_vha_tp_worker, args=(world_size, _free_port(), num_tokens, out), nprocs=world_size)
        tp_out = torch.cat([out[r] for r in range(world_size)], dim=1)
    u, v, o = _inputs(num_tokens)
    eye = torch.eye(NUM_HEADS)
    exact = (eye + v.float() @ u.float().t()) @ o.float()
    m = torch.addmm(eye.bfloat16(), v, u.t())
    tp1 = torch.matmul(m, o).float()
    tp_err, tp1_err = (tp_out - exact).abs(), (tp1 - exact).abs()
    # TP mixes in fp32, so it is no less accurate than the bf16 m @ o
    assert tp_err.mean() <= tp1_err.mean()
    assert tp_err.max() <= tp1_err.max()
    torch.testing.assert_close(tp_out, tp1, atol=0.25, rtol=2e-2)


# --------------------------------------------------------------------------- custom-op boundary


def test_attention_custom_op_schema_and_fake():
    """The attention runs as ``torch.ops.hca_b200.hca_attention``: it mutates
    ``out`` (the schema marks it), has a fake implementation (shape
    propagation without running), and the layer registers itself by name."""
    from torch._subclasses.fake_tensor import FakeTensorMode

    op = torch.ops.hca_b200.hca_attention
    schema = str(op.default._schema)
    for name in ("out", "out_scale"):
        arg = next(a for a in op.default._schema.arguments if a.name == name)
        assert arg.alias_info is not None and arg.alias_info.is_write, schema
    assert schema.endswith("-> ()"), schema
    with FakeTensorMode():
        q = torch.empty(3, 16, 128, dtype=torch.bfloat16)
        kv = torch.empty(3, 128, dtype=torch.bfloat16)
        ks = torch.empty(3, 256)
        pos = torch.empty(3, dtype=torch.int64)
        out = torch.empty(3, 16, 128, dtype=torch.bfloat16)
        assert op(q, kv, ks, pos, out, torch.empty(0, dtype=torch.int32), "model.layers.0.self_attn.x") is None
        out8 = torch.empty(4, 3, 512, dtype=torch.float8_e4m3fn)
        sc = torch.empty(4, 4, 4, dtype=torch.int32)
        assert op(q, kv, ks, pos, out8, sc, "model.layers.0.self_attn.x") is None
    cfg = A.Ernie5_5HCAConfig(hidden_size=2048, num_hidden_layers=2, num_attention_heads=16, head_dim=128,
                              q_lora_rank=512, qk_rope_head_dim=64, o_groups=4, o_lora_rank=64,
                              hybrid_mla_num_attention_heads=16, num_nextn_predict_layers=0)
    vcfg = A.make_vllm_config(cfg, max_model_len=1152)
    vcfg.compilation_config = SimpleNamespace(static_forward_context={})
    layer = A.Ernie5_5HCAAttention(vcfg, prefix="model.layers.0.self_attn")
    assert vcfg.compilation_config.static_forward_context[layer.layer_name] is layer
    assert A._find_layer(layer.layer_name) is layer


# --------------------------------------------------------------------------- block-FP8 output path


def _fp8_cfg(**kw):
    base = dict(hidden_size=2048, num_hidden_layers=2, num_attention_heads=16, head_dim=128, q_lora_rank=512,
                qk_rope_head_dim=64, o_groups=4, o_lora_rank=128, hybrid_mla_num_attention_heads=16,
                num_nextn_predict_layers=0)
    base.update(kw)
    return A.Ernie5_5HCAConfig(**base)


def test_fp8_output_selection_follows_the_quant_config():
    """``wo_a``/``wo_b`` are block FP8 exactly when the reference keeps
    ``wo_a`` FP8 (a 128 x 128 block-FP8 config that does not ignore it) and the
    blocks tile the groups."""
    assert not A.keeps_fp8_output(None)
    assert not A.keeps_fp8_output(SimpleNamespace(weight_block_size=[32, 32], ignored_layers=[]))
    assert not A.keeps_fp8_output(A.block_fp8_quant_config(["model.layers.0.self_attn.attn.wo_a"]))
    assert A.keeps_fp8_output(A.block_fp8_quant_config())
    layer = A.Ernie5_5HCAAttention(A.make_vllm_config(_fp8_cfg(), max_model_len=1152,
                                                      quant_config=A.block_fp8_quant_config()),
                                   prefix="model.layers.0.self_attn")
    assert layer.fp8_output
    assert layer.wo_a.weight.dtype == torch.float8_e4m3fn and layer.wo_a.weight_scale_inv.shape == (4, 4)
    assert layer.wo_b.weight.shape == (2048, 512) and layer.wo_b.weight_scale_inv.shape == (16, 4)
    # rank-64 groups do not tile 128-row blocks: the bf16 path
    layer64 = A.Ernie5_5HCAAttention(A.make_vllm_config(_fp8_cfg(o_lora_rank=64), max_model_len=1152,
                                                        quant_config=A.block_fp8_quant_config()),
                                     prefix="model.layers.0.self_attn")
    assert not layer64.fp8_output and layer64.wo_a.weight.dtype == torch.bfloat16


def test_fp8_weights_load_from_block_fp8_or_quantise_on_load():
    """A block-FP8 checkpoint (e4m3 + ``weight_scale_inv``) loads as is; a
    bf16 weight is quantised to the same bytes and scales on load."""
    from vllm_ernie_b200.ops import quantize_weight_block_fp8

    vc = A.make_vllm_config(_fp8_cfg(), max_model_len=1152, quant_config=A.block_fp8_quant_config())
    g = torch.Generator().manual_seed(0)
    wa = torch.randn(512, 512, generator=g) * 0.02
    wb = torch.randn(2048, 512, generator=g) * 0.02
    qa, sa = quantize_weight_block_fp8(wa)
    qb, sb = quantize_weight_block_fp8(wb)
    assert torch.equal(sa, torch.exp2(torch.log2(sa))) and sa.shape == (4, 4)
    deq = qa.float() * sa.repeat_interleave(128, 0).repeat_interleave(128, 1)
    assert ((deq - wa).abs() <= wa.abs() * 2 ** -4 + sa.repeat_interleave(128, 0).repeat_interleave(128, 1) * 2 ** -9).all()
    a = A.Ernie5_5HCAAttention(vc, prefix="model.layers.0.self_attn")
    got = a.load_weights([("wo_a.weight", qa), ("wo_a.weight_scale_inv", sa), ("wo_b.weight", qb),
                          ("wo_b.weight_scale_inv", sb)])
    assert got == {"wo_a.weight", "wo_a.weight_scale_inv", "wo_b.weight", "wo_b.weight_scale_inv"}
    b = A.Ernie5_5HCAAttention(vc, prefix="model.layers.0.self_attn")
    b.load_weights([("wo_a.weight", wa), ("wo_b.weight", wb)])
    for x, y in ((a.wo_a, b.wo_a), (a.wo_b, b.wo_b)):
        assert torch.equal(x.weight.view(torch.uint8), y.weight.view(torch.uint8))
        assert torch.equal(x.weight_scale_inv, y.weight_scale_inv)


def test_max_model_len_beyond_rope_table_is_refused():
    """The RoPE kernels index the cos/sin table by position, so a context
    the table does not cover is refused at construction."""
    cfg = _fp8_cfg(max_position_embeddings=4096)
    with pytest.raises(ValueError, match="max_position_embeddings"):
        A.Ernie5_5HCAAttention(A.make_vllm_config(cfg, max_model_len=8192), prefix="model.layers.0.self_attn")
    layer = A.Ernie5_5HCAAttention(A.make_vllm_config(cfg, max_model_len=4096), prefix="model.layers.0.self_attn")
    assert layer.cos_sin_cache.shape[0] == 4096


def _fp8_shard_worker(rank, world_size, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world_size)
    try:
        from vllm_ernie_b200.ops import quantize_weight_block_fp8

        cfg = _fp8_cfg(num_attention_heads=32, hybrid_mla_num_attention_heads=32, o_groups=8, o_lora_rank=512)
        vc = A.make_vllm_config(cfg, max_model_len=1152, quant_config=A.block_fp8_quant_config())
        g = torch.Generator().manual_seed(4)
        wa = torch.randn(8 * 512, 512, generator=g) * 0.02   # [G * o_lora, H * D / G]
        wb = torch.randn(2048, 8 * 512, generator=g) * 0.02  # [hidden, G * o_lora]
        qa, sa = quantize_weight_block_fp8(wa)
        qb, sb = quantize_weight_block_fp8(wb)
        for form, items in (("fp8", [("wo_a.weight", qa), ("wo_a.weight_scale_inv", sa), ("wo_b.weight", qb),
                                     ("wo_b.weight_scale_inv", sb)]),
                            ("bf16", [("wo_a.weight", wa), ("wo_b.weight", wb)])):
            layer = A.Ernie5_5HCAAttention(vc, prefix="model.layers.0.self_attn", tp_group=dist.group.WORLD)
            assert layer.fp8_output and layer.n_local_groups == 8 // world_size
            layer.load_weights(items)
            out[(rank, form)] = (layer.wo_a.weight.view(torch.uint8).clone(), layer.wo_a.weight_scale_inv.clone(),
                                 layer.wo_b.weight.view(torch.uint8).clone(), layer.wo_b.weight_scale_inv.clone())
    finally:
        dist.destroy_process_group()


def test_fp8_weights_shard_by_rank_gloo():
    """Head-sharded TP of the block-FP8 output weights: wo_a by rows (output
    groups), wo_b by columns, the 128 x 128 scale blocks with them; loading
    the checkpoint's e4m3 + scales and quantising a bf16 weight on load give
    each rank the same bytes, the matching slice of the unsharded layer's."""
    from vllm_ernie_b200.ops import quantize_weight_block_fp8

    world_size = 2
    with mp.get_context("spawn").Manager() as manager:
        out = manager.dict()
        mp.spawn(_fp8_shard_worker, args=(world_size, _free_port(), out), nprocs=world_size)
        got = dict(out.items())
    g = torch.Generator().manual_seed(4)
    qa, sa = quantize_weight_block_fp8(torch.randn(8 * 512, 512, generator=g) * 0.02)
    qb, sb = quantize_weight_block_fp8(torch.randn(2048, 8 * 512, generator=g) * 0.02)
    ra, rb = qa.shape[0] // world_size, qb.shape[1] // world_size
    for r in range(world_size):
        want = (qa[r * ra:(r + 1) * ra].view(torch.uint8), sa[r * ra // 128:(r + 1) * ra // 128],
                qb[:, r * rb:(r + 1) * rb].view(torch.uint8), sb[:, r * rb // 128:(r + 1) * rb // 128])
        for form in ("fp8", "bf16"):
            for a, b in zip(got[(r, form)], want):
                assert torch.equal(a, b), (r, form)
