"""The overlapped sequence-split attention (lingbot_b200.split.SplitAttention) on one GPU: a one-rank
NCCL group exercises the share totals, the all-reduce, the asynchronous gather and the two-segment window
(memory part quantized before the chunk arrives). Its codes must equal quantizing the window in one
piece, and its output must equal (128-aligned memory) or match within tolerance (64-aligned memory) the
single-segment attention."""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist

from oracle import sage_semantics as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def one_rank_group():
    if dist.is_initialized():
        yield
        return
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("nccl", rank=0, world_size=1, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", 0))
    yield
    dist.destroy_process_group()


@pytest.mark.parametrize("mem,n", [(640, 300), (576, 257)], ids=["mem128aligned", "mem64aligned"])
def test_split_attention_matches_single_segment(one_rank_group, mem, n):
    from lingbot_b200 import kv_cache, ops, split
    torch.manual_seed(0)
    dev, H = torch.device("cuda"), 2
    kc = kv_cache.allocate(1, [1, mem + n, H, 128], torch.bfloat16, dev)[0]
    kc["k"][:, :mem] = (torch.randn(1, mem, H, 128, device=dev) + 3 * torch.randn(1, 1, H, 128, device=dev)).bfloat16()
    kc["v"][:, :mem] = torch.randn(1, mem, H, 128, device=dev).bfloat16()
    kv_cache.refresh_stats(kc, 0, mem)
    q = torch.randn(1, n, H, 128, device=dev).bfloat16()
    kcur = (torch.randn(1, n, H, 128, device=dev) + 1.5).bfloat16()
    vcur = torch.randn(1, n, H, 128, device=dev).bfloat16()
    sp = split.SplitAttention(1, H, n, mem, n, dev)
    sp.memory_changed(kc)
    out = torch.empty(1, n, H, 128, dtype=torch.bfloat16, device=dev)
    sp(q, kc, kcur, vcur, out)
    torch.cuda.synchronize()
    # the chunk landed in the cache
    assert torch.equal(kc["k"][:, mem:], kcur) and torch.equal(kc["v"][:, mem:], vcur)
    w = ops.quantize_qkv(q, kc["k"], kc["v"])
    ref = ops.attn_from_codes(w)
    torch.cuda.synchronize()
    # codes: segment 0 = tokens [0, mem), segment 1 = tokens [mem, mem + n) of the one-piece window
    assert torch.equal(sp.k_codes[0][:, :, :mem], w.k_codes[0][:, :, :mem])
    assert torch.equal(sp.k_codes[1][:, :, :n], w.k_codes[0][:, :, mem:mem + n])
    assert torch.equal(sp.vt_codes[0][..., :mem], w.vt_codes[0][..., :mem])
    assert torch.equal(sp.vt_codes[1][..., :n], w.vt_codes[0][..., mem:mem + n])
    assert torch.equal(sp.k_scale[0][:, :, :mem // 64], w.k_scale[0][:, :, :mem // 64])
    assert torch.equal(sp.k_scale[1][:, :, :(n + 63) // 64], w.k_scale[0][:, :, mem // 64:(mem + n + 63) // 64])
    assert torch.equal(sp.v_scale, w.v_scale) and torch.equal(sp.km, w.km)
    assert torch.equal(sp.q_codes[:, :, :n], w.q_codes[:, :, :n])
    if mem % 128 == 0:
        assert torch.equal(out, ref)       # same key tiles -> same result
    else:
        m = O.compare(out.float().cpu(), ref.float().cpu())
        assert m["cos"] >= 0.9999 and m["max_abs"] <= 2e-2, m
