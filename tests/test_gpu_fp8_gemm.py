"""GPU parity of the block-scaled FP8 GEMM (grouped ``wo_a`` einsum and
gated ``wo_b`` linear, ``hca_fp8_grouped_gemm``) against an fp32 torch
reference on the dequantised operands.

Tolerance: the kernel accumulates in fp32 and rounds once to bf16, so
``|got - ref| <= 2^-8 |ref| + 1e-4 max|ref|`` (one bf16 rounding plus the
fp32 summation-order difference).
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"
FP8 = torch.float8_e4m3fn


def _aligned(n):
    return (n + 3) // 4 * 4


def _e4m3(shape, gen):
    return (torch.randn(shape, generator=gen, device=DEV) * 64).clamp(-448, 448).to(FP8)


def _exps(shape, gen):
    return torch.randint(118, 132, shape, generator=gen, device=DEV, dtype=torch.int32)


def _pack(e):
    """[..., blocks] exponent bytes -> [..., blocks / 4] int32, byte c of int k = block 4k + c."""
    e = e.view(*e.shape[:-1], -1, 4).to(torch.int64)
    v = e[..., 0] | (e[..., 1] << 8) | (e[..., 2] << 16) | (e[..., 3] << 24)
    return torch.where(v >= 2 ** 31, v - 2 ** 32, v).to(torch.int32)


def _reference(x, sx, w, sw):
    """fp32 ``out[t, g, n] = sum_k x sx w sw`` with sx [T, G, K/128] exponents."""
    t, g, k = x.shape
    n = w.shape[1]
    xf = x.float() * torch.exp2(sx.float() - 127).repeat_interleave(128, -1)
    swf = sw.repeat_interleave(128, 1)[:, :n].repeat_interleave(128, 2)
    wf = w.float() * swf
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        return torch.einsum("tgk,gnk->tgn", xf.double(), wf.double()).float()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def _check(got, ref):
    got = got.float()
    bound = 2.0 ** -8 * ref.abs() + 1e-4 * ref.abs().max()
    assert torch.isfinite(got).all()
    bad = (got - ref).abs() > bound
    assert not bad.any(), ((got - ref).abs().max().item(), int(bad.sum()))


@pytest.mark.parametrize("t,g,hpg,d,n", [
    (192, 8, 8, 128, 1024),   # config-1 decode wo_a: 64 heads x 128 in 8 groups, rank 1024
    (300, 2, 4, 128, 256),    # ragged token tiles
    (3, 4, 2, 512, 128),      # head_dim 512: four 128-blocks per int32
    (1, 1, 16, 128, 64),      # rank-64 group (CPU reference config shape)
])
def test_grouped_wo_a_matches_fp32(t, g, hpg, d, n):
    from vllm_ernie_b200 import ops

    gen = torch.Generator(device=DEV).manual_seed(t * 7 + g)
    k = hpg * d
    # activation layout of hca_vha_inv_rope_fp8_quant: data [G, T, K]
    # viewed [T, G, K]; scales int32 [G, HPG, aligned_T] viewed [T, G, HPG]
    x = _e4m3((g, t, k), gen).transpose(0, 1)
    blocks = k // 128
    ex = _exps((t, g, blocks), gen)
    per_int = d // 128
    packed = ex if per_int == 1 else _pack(ex)
    sbuf = torch.zeros((g, hpg, _aligned(t)), dtype=torch.int32, device=DEV)
    sbuf.permute(2, 0, 1)[:t].copy_(packed)
    sx = sbuf.permute(2, 0, 1)[:t]
    w = _e4m3((g, n, k), gen)
    sw = torch.rand((g, (n + 127) // 128, blocks), generator=gen, device=DEV) * 2 ** -6 + 2 ** -8
    out = ops.fp8_grouped_gemm(x, sx, w, sw)
    torch.cuda.synchronize()
    _check(out, _reference(x, ex, w, sw))
    assert ops.device_error() == 0


@pytest.mark.parametrize("t,hidden,k", [(192, 4096, 8192), (37, 1024, 2048)])
def test_gated_wo_b_matches_fp32(t, hidden, k):
    """``wo_b(z * sigmoid(gate))`` through the fused gate quant and the GEMM."""
    from vllm_ernie_b200 import ops

    gen = torch.Generator(device=DEV).manual_seed(t)
    z = torch.randn((t, k), generator=gen, device=DEV).bfloat16()
    gate = torch.randn((t, k), generator=gen, device=DEV).bfloat16()
    wbf = (torch.randn((hidden, k), generator=gen, device=DEV) * 0.02).bfloat16()
    w, sw = ops.quantize_weight_block_fp8(wbf)
    assert torch.equal(sw, torch.exp2(torch.log2(sw)))  # power-of-two block scales
    xq, xs = ops.sigmoid_mul_quant_fp8(z, gate)
    out = ops.fp8_grouped_gemm(xq, xs, w, sw)
    torch.cuda.synchronize()
    assert out.shape == (t, hidden)
    ex = torch.stack([(xs >> (8 * c)) & 0xFF for c in range(4)], -1).reshape(t, -1)
    _check(out, _reference(xq.unsqueeze(1), ex.unsqueeze(1), w.unsqueeze(0), sw.unsqueeze(0)).squeeze(1))
    # and close to the bf16 GEMM it replaces (the FP8 quant error only)
    ref_bf16 = (z.float() * torch.sigmoid(gate.float())) @ wbf.float().t()
    rel = (out.float() - ref_bf16).norm() / ref_bf16.norm()
    assert rel < 0.05, rel.item()
    assert ops.device_error() == 0


def test_fp8_gemm_empty_and_unsupported_shapes():
    from vllm_ernie_b200 import ops
    from vllm_ernie_b200._lib import HcaError

    x = torch.zeros((0, 256), dtype=FP8, device=DEV)
    xs = torch.zeros((0, 1), dtype=torch.int32, device=DEV)
    w = torch.zeros((128, 256), dtype=FP8, device=DEV)
    sw = torch.ones((1, 2), device=DEV)
    # 256 = two 128-blocks, scales must cover them in one int32 of four
    xs4 = torch.zeros((0, 1), dtype=torch.int32, device=DEV)
    with pytest.raises(AssertionError):
        ops.fp8_grouped_gemm(x, xs4, w, sw)  # 2 blocks cannot be 1 or 4 per int32 of one pack
    x = torch.zeros((0, 512), dtype=FP8, device=DEV)
    w = torch.zeros((128, 512), dtype=FP8, device=DEV)
    sw = torch.ones((1, 4), device=DEV)
    assert ops.fp8_grouped_gemm(x, xs, w, sw).shape == (0, 128)
    # N not a multiple of 64: refused by the library, nothing launched
    x = torch.zeros((4, 512), dtype=FP8, device=DEV)
    xs = torch.zeros((4, 1), dtype=torch.int32, device=DEV)
    w = torch.zeros((96, 512), dtype=FP8, device=DEV)
    sw = torch.ones((1, 4), device=DEV)
    with pytest.raises(HcaError):
        ops.fp8_grouped_gemm(x, xs, w, sw)
    torch.cuda.synchronize()
    assert ops.device_error() == 0


def test_fp8_gemm_split_k_workspace_checked_before_launch():
    """A split-K call needs its workspace: missing or too small, the library
    refuses it before launching (HCA_E_INVALID / HCA_E_WORKSPACE)."""
    from vllm_ernie_b200 import ops
    from vllm_ernie_b200._lib import HcaError, call, lib

    t, n, k = 48, 4096, 8192
    need = lib().hca_fp8_grouped_gemm_workspace_bytes(t, 1, n, k)
    assert need > 0  # 32 weight tiles: split K over a cluster
    x = torch.zeros((t, k), dtype=FP8, device=DEV)
    xs = torch.zeros((t, k // 512), dtype=torch.int32, device=DEV)
    w = torch.zeros((n, k), dtype=FP8, device=DEV)
    sw = torch.ones((n // 128, k // 128), device=DEV)
    out = torch.empty((t, n), dtype=torch.bfloat16, device=DEV)
    small = torch.empty(need // 4 - 4, dtype=torch.float32, device=DEV)
    s = torch.cuda.current_stream().cuda_stream
    args = (out.data_ptr(), n, 0, x.data_ptr(), k, 0, xs.data_ptr(), 1, 0, t, 4, w.data_ptr(), sw.data_ptr(),
            t, 1, n, k)
    with pytest.raises(HcaError) as e:
        call("hca_fp8_grouped_gemm", *args, small.data_ptr(), small.numel() * 4, s)
    assert e.value.status == -4
    with pytest.raises(HcaError) as e:
        call("hca_fp8_grouped_gemm", *args, None, 0, s)
    assert e.value.status == -1
    torch.cuda.synchronize()
    assert ops.device_error() == 0
