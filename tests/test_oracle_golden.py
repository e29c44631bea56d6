"""The CPU oracle against the reference's own quantizer outputs (golden fixtures): bit for bit."""
import pytest
import torch

from oracle import sage_semantics as O
from tests._golden import quant_cases

CASES = quant_cases()
IDS = [c["meta"]["name"] for c in CASES]


@pytest.mark.parametrize("case", CASES, ids=IDS)
def test_q_codes_and_scales_bit_exact(case):
    codes, scale = O.quant_q(case["q"])
    assert torch.equal(codes, case["q_codes"])
    assert torch.equal(scale.view(torch.int32), case["q_scale"].view(torch.int32))


@pytest.mark.parametrize("case", CASES, ids=IDS)
def test_k_mean_within_one_bf16_ulp(case):
    km = O.k_mean(case["k"])
    a = km.view(torch.int16).int()
    b = case["km"].view(torch.int16).int()
    assert (a - b).abs().max().item() <= 1


@pytest.mark.parametrize("case", CASES, ids=IDS)
def test_k_codes_bit_exact_given_reference_mean(case):
    codes, scale = O.quant_k(case["k"], case["km"])
    assert torch.equal(codes, case["k_codes"])
    assert torch.equal(scale.view(torch.int32), case["k_scale"].view(torch.int32))


@pytest.mark.parametrize("case", CASES, ids=IDS)
def test_v_codes_bit_exact(case):
    am = O.v_amax(case["v"])
    assert torch.equal(am, case["v_amax"])
    codes, vs = O.quant_v(case["v"], am)
    assert torch.equal(vs.view(torch.int32), case["v_scale"].view(torch.int32))
    n = codes.shape[1]
    e16 = (n + 15) // 16 * 16
    padded = torch.nn.functional.pad(codes, (0, 0, 0, 0, 0, e16 - n))   # pad code 0 == +0.0
    assert torch.equal(O.sage_layout(padded).contiguous(), case["v_codes_sage"])


def test_attention_emulation_close_to_fp32():
    """Sanity: the kernel emulation is a faithful attention (reference reports cos 0.99925 vs fp32
    on randn at its own shape, results/h2_cfg_base.json)."""
    g = torch.Generator().manual_seed(0)
    q = torch.randn(1, 256, 2, 128, generator=g).bfloat16()
    k = (torch.randn(1, 640, 2, 128, generator=g) + 3 * torch.randn(1, 1, 2, 128, generator=g)).bfloat16()
    v = torch.randn(1, 640, 2, 128, generator=g).bfloat16()
    o = O.sage_attention(q, k, v)
    ref = O.sdpa_fp32(q, k, v)
    m = O.compare(o, ref)
    assert m["cos"] > 0.998, m
