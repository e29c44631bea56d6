"""The drop-in attention entry points' routing, without a GPU (the kernels themselves are covered by the
GPU tests)."""
import pytest
import torch


def test_cross_attention_routing_without_a_gpu():
    """flash_attention is the paper's attention by default (CPU SDPA here); in the "sage" mode its plain
    calls go to the quantized kernels, which refuse CPU tensors (no fallback), while masked calls stay
    on the paper's attention."""
    import torch.nn.functional as F
    from lingbot_b200 import attention
    g = torch.Generator().manual_seed(0)
    q = torch.randn(1, 40, 2, 128, generator=g).bfloat16()
    k = torch.randn(1, 24, 2, 128, generator=g).bfloat16()
    v = torch.randn(1, 24, 2, 128, generator=g).bfloat16()
    ref = F.scaled_dot_product_attention(*(x.transpose(1, 2) for x in (q, k, v))).transpose(1, 2)
    assert torch.equal(attention.flash_attention(q, k, v), ref)
    with pytest.raises(ValueError):
        attention.set_cross_attention("fp8")
    try:
        attention.set_cross_attention("sage")
        with pytest.raises(ValueError, match="CUDA"):
            attention.flash_attention(q, k, v)
        assert attention.flash_attention(q, k, v, k_lens=torch.tensor([24])).shape == q.shape
    finally:
        attention.set_cross_attention("paper")
