"""The drop-in boundary on the GPU: fp16 activations through `dtype`, causal calls refused by the C ABI
(LBQ_ERR_UNSUPPORTED) and routed to the reference's non-Sage branch by attention(), and the custom op
`lbq::sage_attn` under torch.compile(fullgraph=True, dynamic=True) and torch.library.opcheck."""
import pytest
import torch
import torch.nn.functional as F

from oracle import sage_semantics as O
from tests._gpu import bits, k_codes_nhd, k_scale_ref, q_codes_nhd, v_codes_nhd
from tests.test_attn_gpu import check_parity

pytestmark = pytest.mark.gpu


def qkv(seed, b, h, lq, lk, dtype):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(b, lq, h, 128, generator=g)
    k = torch.randn(b, lk, h, 128, generator=g) + 3 * torch.randn(b, 1, h, 128, generator=g)
    v = torch.randn(b, lk, h, 128, generator=g)
    return q.to(dtype), k.to(dtype), v.to(dtype)


@pytest.mark.parametrize("shape", [(1, 2, 300, 1000), (2, 3, 129, 777)], ids=["q300k1000", "b2q129k777"])
def test_fp16_codes_match_the_oracle(shape):
    """lbq_quant_qkv with fp16 activations: Q/K/V codes, scales and km (rounded to fp16) bit-exact."""
    from lingbot_b200 import ops
    b, h, lq, lk = shape
    q, k, v = qkv(3, b, h, lq, lk, torch.float16)
    w = ops.quantize_qkv(q.cuda(), k.cuda(), v.cuda())
    ref = O.quantize_qkv(q, k, v)
    torch.cuda.synchronize()
    assert w.dtype == torch.float16 and w.km.dtype == torch.float16
    assert torch.equal(q_codes_nhd(w), ref["q_codes"])
    nq = (lq + 31) // 32
    assert torch.equal(bits(w.q_scale[:, :, :nq].cpu()), bits(ref["q_scale"][:, :, :nq]))
    assert torch.equal(w.km.cpu().view(torch.int16), ref["km"][:, 0].contiguous().view(torch.int16))
    assert torch.equal(k_codes_nhd(w), ref["k_codes"])
    assert torch.equal(bits(k_scale_ref(w)), bits(ref["k_scale"]))
    assert torch.equal(v_codes_nhd(w), ref["v_codes"])
    assert torch.equal(bits(w.v_scale.cpu()), bits(ref["v_scale"]))


@pytest.mark.parametrize("splits", [1, 3])
def test_fp16_attention_matches_the_oracle(splits):
    """fp16 in, fp16 out (one pass and split-KV with its combine), held to the same tolerance as the
    bf16 path against the Sage emulation."""
    from lingbot_b200 import _lib, ops
    q, k, v = qkv(4, 1, 2, 300, 1000, torch.float16)
    w = ops.quantize_qkv(q.cuda(), k.cuda(), v.cuda())
    out = ops.attn_from_codes(w, num_splits=splits)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    assert out.dtype == torch.float16
    check_parity(out.float().cpu(), w, splits=splits)


def test_drop_in_attention_casts_to_dtype():
    """attention(q, k, v, dtype=torch.float16) with bf16 inputs runs the fp16 path and returns bf16:
    the reference casts to `dtype` before Sage and back to q's dtype after (attention.py:30-36)."""
    from lingbot_b200 import ops
    from lingbot_b200.attention import attention
    q, k, v = qkv(5, 1, 2, 256, 640, torch.bfloat16)
    q, k, v = q.cuda(), k.cuda(), v.cuda()
    got = attention(q, k, v, dtype=torch.float16)
    want = ops.sage_attn(q.half(), k.half(), v.half()).to(torch.bfloat16)
    assert got.dtype == torch.bfloat16
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))


def test_causal_is_refused_by_the_kernel_and_routed_by_attention():
    from lingbot_b200 import _lib, ops
    from lingbot_b200.attention import attention
    q, k, v = qkv(6, 1, 2, 256, 256, torch.bfloat16)
    q, k, v = q.cuda(), k.cuda(), v.cuda()
    with pytest.raises(_lib.LbqError, match="causal"):
        ops.sage_attn(q, k, v, is_causal=True)
    assert _lib.load().lbq_last_error() is not None
    got = attention(q, k, v, causal=True)
    want = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                          is_causal=True).transpose(1, 2)
    assert torch.equal(got, want.to(got.dtype))


def test_torch_compile_keeps_one_graph():
    """torch.compile(attention, fullgraph=True, dynamic=True) traces through lbq::sage_attn (its fake
    implementation) without a graph break, over two shapes, with the eager call's bits."""
    from lingbot_b200.attention import attention
    torch._dynamo.reset()
    fn = torch.compile(attention, fullgraph=True, dynamic=True)
    for shape in [(1, 2, 256, 640), (1, 2, 384, 1000)]:
        q, k, v = qkv(7, *shape, torch.bfloat16)
        q, k, v = q.cuda(), k.cuda(), v.cuda()
        got = fn(q, k, v)
        want = attention(q, k, v)
        torch.cuda.synchronize()
        assert torch.equal(got.view(torch.int16), want.view(torch.int16)), shape


def test_opcheck_sage_attn():
    from lingbot_b200.attention import sage_attn
    q, k, v = qkv(8, 1, 2, 128, 256, torch.bfloat16)
    torch.library.opcheck(sage_attn, (q.cuda(), k.cuda(), v.cuda(), 0.0))
