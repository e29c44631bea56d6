"""The fused producers on the GPU: RoPE + Q quantization (lbq_rope_quant_q) and the KV-cache write
with its block statistics (lbq_cache_write), against the oracle (RoPE pinned to the reference by
tests/golden/rope_grid2x4x6.npz) and against the unfused path (bf16 copy + lbq_kv_block_stats),
bit for bit."""
import pytest
import torch

from oracle import rope as R
from oracle import sage_semantics as O
from tests._gpu import bits

pytestmark = pytest.mark.gpu


def tables(grid, start_frame, device="cuda"):
    cos, sin = R.rope_tables(grid, R.freqs_table(128), start_frame)
    return cos.to(device), sin.to(device)


@pytest.mark.parametrize("grid,heads", [([(3, 10, 10), (3, 10, 10)], 3), ([(1, 1, 1)], 1), ([(2, 7, 9)], 12)],
                         ids=["b2_q300", "q1", "q126_h12"])
def test_rope_quant_q_matches_rope_then_quant(grid, heads):
    """Codes and scales of lbq_rope_quant_q(q) equal the oracle's quant_q(rope_apply(q)) and the
    unfused GPU path (lbq_quant_q of the oracle-roped bf16)."""
    from lingbot_b200 import _lib, kv_cache, ops
    b = len(grid)
    lq = grid[0][0] * grid[0][1] * grid[0][2]
    g = torch.Generator().manual_seed(5)
    q = (torch.randn(b, lq, heads, 128, generator=g) * 2).bfloat16()
    cos, sin = tables(grid, start_frame=4)
    qz = kv_cache.WindowQuantizer().buffers(b, heads, lq, 64, "cuda")
    rc, rs, sr_b, sr_l = kv_cache._rope_args((cos, sin))
    qd = q.cuda()
    _lib.call("lbq_rope_quant_q", ops._ptr(qd), *qd.stride()[:3], rc, rs, sr_b, sr_l, b, heads, lq,
              ops._ptr(qz.q_codes), ops._ptr(qz.q_scale), ops._stream())
    roped = R.rope_apply(q, cos.cpu(), sin.cpu())
    ref_codes, ref_scale = O.quant_q(roped)
    nq = (lq + 31) // 32
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    assert torch.equal(qz.q_codes[:, :, :lq].permute(0, 2, 1, 3).cpu(), ref_codes)
    assert torch.equal(bits(qz.q_scale[:, :, :nq].cpu()), bits(ref_scale[:, :, :nq]))
    unf_codes, unf_scale = ops.alloc_q(b, heads, lq, "cuda")
    rd = roped.cuda()
    _lib.call("lbq_quant_q", ops._ptr(rd), *rd.stride()[:3], b, heads, lq, ops._ptr(unf_codes), ops._ptr(unf_scale),
              ops._stream())
    assert torch.equal(unf_codes, qz.q_codes) and torch.equal(bits(unf_scale), bits(qz.q_scale))


@pytest.mark.parametrize("tok_begin,n", [(0, 300), (237, 300), (64, 128), (999, 1), (700, 300)])
@pytest.mark.parametrize("with_rope", [False, True], ids=["plain", "roped"])
def test_cache_write_matches_copy_then_block_stats(tok_begin, n, with_rope):
    """lbq_cache_write leaves the cache and the statistics tables bit-identical to the unfused path:
    K (roped by the oracle when `with_rope`) and V copied in, then lbq_kv_block_stats over the blocks
    covering [tok_begin, tok_begin + n)."""
    from lingbot_b200 import _lib, kv_cache
    b, h, size = 2, 3, 1000
    g = torch.Generator().manual_seed(tok_begin + n)
    fused = kv_cache.allocate(1, [b, size, h, 128], torch.bfloat16, "cuda")[0]
    base_k = (torch.randn(b, size, h, 128, generator=g) + 3 * torch.randn(1, 1, h, 128, generator=g)).bfloat16()
    base_v = torch.randn(b, size, h, 128, generator=g).bfloat16()
    fused["k"].copy_(base_k)
    fused["v"].copy_(base_v)
    kv_cache.refresh_stats(fused, 0, size)
    plain = {key: (t.clone() if torch.is_tensor(t) else t) for key, t in fused.items()}
    k = (torch.randn(b, n, h, 128, generator=g) * 2).bfloat16()
    v = torch.randn(b, n, h, 128, generator=g).bfloat16()
    rope = None
    k_in = k
    if with_rope:
        frames = max(1, n // 4)
        grid = [(frames, 2, 2)] * b
        cos, sin = tables(grid, start_frame=3)
        cos, sin = cos[:, :n].contiguous(), sin[:, :n].contiguous()
        rope = (cos, sin)
        k_in = R.rope_apply(k, cos.cpu(), sin.cpu())
    kv_cache.store(fused, k.cuda(), v.cuda(), tok_begin, rope)
    plain["k"][:, tok_begin:tok_begin + n] = k_in.cuda()
    plain["v"][:, tok_begin:tok_begin + n] = v.cuda()
    kv_cache.refresh_stats(plain, tok_begin, tok_begin + n)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    assert torch.equal(fused["k"].view(torch.int16), plain["k"].view(torch.int16))
    assert torch.equal(fused["v"].view(torch.int16), plain["v"].view(torch.int16))
    assert torch.equal(fused["lbq_ksum"].view(torch.int64), plain["lbq_ksum"].view(torch.int64))
    assert torch.equal(fused["lbq_vamax"].view(torch.int32), plain["lbq_vamax"].view(torch.int32))


def test_roped_window_attention_matches_the_unfused_call():
    """The whole call with the producers fused (K roped in the cache write, Q roped in its quantizer)
    equals roping on the host, writing, and quantizing the roped Q: same codes, same output bits."""
    from lingbot_b200 import kv_cache
    b, h, mem, n = 1, 2, 640, 300
    grid = [(3, 10, 10)]
    cos, sin = tables(grid, start_frame=6)
    g = torch.Generator().manual_seed(9)
    mk = (torch.randn(b, mem, h, 128, generator=g) + 2 * torch.randn(1, 1, h, 128, generator=g)).bfloat16().cuda()
    mv = torch.randn(b, mem, h, 128, generator=g).bfloat16().cuda()
    q = torch.randn(b, n, h, 128, generator=g).bfloat16()
    k = torch.randn(b, n, h, 128, generator=g).bfloat16()
    v = torch.randn(b, n, h, 128, generator=g).bfloat16()
    outs = []
    for fused in (True, False):
        c = kv_cache.allocate(1, [b, mem + n, h, 128], torch.bfloat16, "cuda")[0]
        kv_cache.store(c, mk, mv, 0)
        if fused:
            kv_cache.store(c, k.cuda(), v.cuda(), mem, (cos, sin))
            out = kv_cache.attend(q.cuda(), c, mem, mem + n, quantizer=kv_cache.WindowQuantizer(), rope=(cos, sin))
        else:
            kr = R.rope_apply(k, cos.cpu(), sin.cpu()).cuda()
            qr = R.rope_apply(q, cos.cpu(), sin.cpu()).cuda()
            kv_cache.store(c, kr, v.cuda(), mem)
            out = kv_cache.attend(qr, c, mem, mem + n, quantizer=kv_cache.WindowQuantizer())
        outs.append(out.clone())
    torch.cuda.synchronize()
    assert torch.equal(outs[0].view(torch.int16), outs[1].view(torch.int16))
