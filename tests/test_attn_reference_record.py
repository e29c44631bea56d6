"""Attention accuracy against the reference's own measurement of the stock Sage INT8 kernel.

The reference's protocol (experiments/bench_attn/sage3_build.md:123-141): torch.manual_seed(0), then
q [1, 6032, 12, 128] and k, v [1, 27144, 12, 128] drawn with CUDA randn in bf16, in that order; output
compared with fp32 scaled_dot_product_attention by the cosine of the flattened tensors. The stock
SageAttention-2 INT8 kernel the reference calls (qk_int8_sv_f8_accum_f16_fuse_v_scale_attn_inst_buf)
recorded cos 0.9992457628 and max-abs 0.0023489 on exactly this setup
(experiments/bench_attn/results/h2_cfg_base.json). The reference notes that every INT8 kernel variant it
tried moved only the fourth decimal of this cosine; this kernel lands 7e-6 from it. The bound is
two-sided: a much better cosine would mean different (lighter) quantization, a worse one a defect.
"""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

REF_COS = 0.9992457628250122
REF_MAX_ABS = 0.002348925918340683


def test_accuracy_matches_the_recorded_sage_kernel():
    from lingbot_b200 import _lib, attention
    torch.manual_seed(0)
    b, lq, lkv, h, d = 1, 6032, 27144, 12, 128
    q = torch.randn(b, lq, h, d, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(b, lkv, h, d, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(b, lkv, h, d, device="cuda", dtype=torch.bfloat16)
    ref = F.scaled_dot_product_attention(q.transpose(1, 2).float(), k.transpose(1, 2).float(),
                                         v.transpose(1, 2).float(), is_causal=False).transpose(1, 2)
    out = attention.attention(q, k, v)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    cos = F.cosine_similarity(ref.flatten().float(), out.flatten().float(), dim=0).item()
    max_abs = (ref - out.float()).abs().max().item()
    print(f"cos {cos:.7f} (reference Sage kernel {REF_COS:.7f}), max-abs {max_abs:.3e} ({REF_MAX_ABS:.3e})")
    # measured on B200: cos 0.9992384, max-abs 2.342e-3
    assert abs(cos - REF_COS) <= 1e-4, (cos, REF_COS)
    assert 0.8 * REF_MAX_ABS <= max_abs <= 1.25 * REF_MAX_ABS, (max_abs, REF_MAX_ABS)
