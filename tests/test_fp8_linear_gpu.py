"""FP8 linear layers on the GPU (lbq_fp8_quant_rows, lbq_fp8_gemm, lingbot_b200.fp8_linear.FP8Linear):
codes and scales bit-exact against the oracle (pinned to the reference's FP8Linear by golden vectors);
the GEMM against torch._scaled_mm with rowwise scales — the reference's own call — and against a
float64 product of the same FP8 operands."""
import pytest
import torch

from oracle import fp8_linear as F8

pytestmark = pytest.mark.gpu


def _rnd(g, *shape, scale=1.0):
    return torch.randn(*shape, generator=g) * scale


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_quant_rows_bit_exact(dtype):
    from lingbot_b200 import fp8_linear as L
    g = torch.Generator().manual_seed(1)
    x = (_rnd(g, 300, 1536, scale=4) * (1 + 30 * (torch.rand(300, 1536, generator=g) > 0.999))).to(dtype)
    x[7] = 0
    q, s = L.quant_rows(x.cuda())
    qr, sr = F8.quant_rows(x)
    torch.cuda.synchronize()
    assert torch.equal(q.cpu().view(torch.uint8), qr.view(torch.uint8))
    assert torch.equal(s.cpu().view(torch.int32), sr[:, 0].contiguous().view(torch.int32))


SHAPES = [(6032, 1536, 1536), (6032, 8960, 1536), (6032, 1536, 8960), (300, 96, 48), (1, 32, 16), (513, 800, 272)]


@pytest.mark.parametrize("m,n,k", SHAPES, ids=[f"m{m}n{n}k{k}" for m, n, k in SHAPES])
@pytest.mark.parametrize("with_bias", [False, True], ids=["nobias", "bias"])
def test_gemm_matches_scaled_mm_and_float64(m, n, k, with_bias):
    """Same e4m3 operands and scales into lbq_fp8_gemm and torch._scaled_mm: the bf16 outputs agree to
    within one bf16 rounding of each other (both accumulate in fp32, in their own orders), and both
    within one bf16 rounding of the float64 product."""
    from lingbot_b200 import _lib
    from lingbot_b200 import fp8_linear as L
    g = torch.Generator().manual_seed(m + n + k)
    x = _rnd(g, m, k).bfloat16().cuda()
    w = _rnd(g, n, k, scale=0.05).bfloat16().cuda()
    bias = _rnd(g, n, scale=0.1).bfloat16().cuda() if with_bias else None
    qx, sx = L.quant_rows(x)
    qw, sw = L.quant_rows(w)
    y = L.gemm(qx, sx, qw, sw, bias)
    ref = torch._scaled_mm(qx, qw.t(), scale_a=sx.reshape(-1, 1), scale_b=sw.reshape(1, -1), bias=bias,
                           out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    exact = F8.gemm(qx.cpu(), sx.cpu(), qw.cpu(), sw.cpu(), None if bias is None else bias.cpu())
    _check_against_exact(y, ref, exact)


def test_gemm_into_a_strided_output():
    """Output rows 16- but not 32-byte aligned (row stride N + 8): the epilogue's 16-byte store path, and
    the padding columns left untouched."""
    from lingbot_b200 import fp8_linear as L
    g = torch.Generator().manual_seed(5)
    m, n, k = 257, 256, 128
    qx, sx = L.quant_rows(_rnd(g, m, k).bfloat16().cuda())
    qw, sw = L.quant_rows(_rnd(g, n, k, scale=0.05).bfloat16().cuda())
    big = torch.full((m, n + 8), 7.0, dtype=torch.bfloat16, device="cuda")
    y = L.gemm(qx, sx, qw, sw, out=big[:, :n])
    ref = torch._scaled_mm(qx, qw.t(), scale_a=sx.reshape(-1, 1), scale_b=sw.reshape(1, -1), out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    assert y.stride(0) == n + 8
    assert bool((big[:, n:] == 7.0).all())
    _check_against_exact(y, ref, F8.gemm(qx.cpu(), sx.cpu(), qw.cpu(), sw.cpu()))


def _check_against_exact(y, ref, exact):
    """Each output within half a bf16 ulp of the float64 product plus an fp32-accumulation allowance,
    for this kernel; torch._scaled_mm's own error is reported beside it."""
    yd, rd = y.double().cpu(), ref.double().cpu()
    scale = exact.abs().max()
    tol = exact.abs() * 2.0 ** -8 + scale * 2.0 ** -14
    err, err_ref = (yd - exact).abs(), (rd - exact).abs()
    info = dict(ours_max_rel=float((err / (exact.abs() + scale * 1e-3)).max()),
                scaled_mm_max_rel=float((err_ref / (exact.abs() + scale * 1e-3)).max()),
                ours_over=float((err - tol).max()), scaled_mm_over=float((err_ref - tol).max()),
                differ=float((yd != rd).double().mean()))
    assert (err <= tol).all(), info
    assert (err_ref <= 4 * tol).all(), info


def test_module_matches_the_reference_forward():
    """FP8Linear(lin)(x) against the reference's forward written out and run by torch on the GPU
    (linear.py:14-31: weight and per-token scales, torch._scaled_mm with rowwise scales and the bf16
    bias), over a [B, L, C] input: the e4m3 codes and scales bit for bit (torch's CUDA rule for the
    scalar division), the output within half a bf16 ulp of the exact product."""
    from lingbot_b200 import fp8_linear as L
    from lingbot_b200.fp8_linear import FP8Linear
    torch.manual_seed(0)
    lin = torch.nn.Linear(1536, 8960).bfloat16().cuda()
    x = torch.randn(2, 1000, 1536, device="cuda").bfloat16()
    mod = FP8Linear(lin)
    got = mod(x)
    w = lin.weight.detach()
    w_scale = (w.abs().amax(dim=1, keepdim=True).float() / 448.0).clamp(min=1e-12)
    w8 = (w.float() / w_scale).to(torch.float8_e4m3fn)
    x2 = x.reshape(-1, 1536)
    x_scale = (x2.abs().amax(dim=1, keepdim=True).float() / 448.0).clamp(min=1e-12)
    x8 = (x2.float() / x_scale).to(torch.float8_e4m3fn)
    want = torch._scaled_mm(x8, w8.t(), scale_a=x_scale, scale_b=w_scale.t().contiguous(),
                            bias=lin.bias.to(torch.bfloat16), out_dtype=torch.bfloat16).reshape(2, 1000, 8960)
    ours_x8, ours_xs = L.quant_rows(x2)
    torch.cuda.synchronize()
    assert torch.equal(mod.w8.view(torch.uint8), w8.view(torch.uint8))
    assert torch.equal(mod.w_scale.view(torch.int32), w_scale[:, 0].contiguous().view(torch.int32))
    assert torch.equal(ours_x8.view(torch.uint8), x8.view(torch.uint8))
    assert torch.equal(ours_xs.view(torch.int32), x_scale[:, 0].contiguous().view(torch.int32))
    exact = F8.gemm(x8.cpu(), x_scale.cpu(), w8.cpu(), w_scale.cpu(), lin.bias.detach().cpu())
    _check_against_exact(got.reshape(-1, 8960), want.reshape(-1, 8960), exact)
