"""The peer-memory sequence-split attention (lingbot_b200.split.SplitAttention).

On one GPU a one-rank group exercises the exchange kernels (statistics push, window totals, share push
into the cache replica, peer wait), the two-segment window and CUDA-graph replay (the signal counters
and the slot parity advance on the device). Its codes must equal quantizing the window in one piece, its
cache writes must equal kv_cache.write's, and its output must equal (128-aligned memory) or match within
tolerance (64-aligned memory) the single-segment attention. With two or more GPUs,
`test_two_ranks_match_one_gpu` runs tests/_split_worker.py under torch.distributed.run."""
import datetime
import os
import socket
import subprocess
import sys

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


def _inputs(seed, mem, n, H, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    q = torch.randn(1, n, H, 128, device=dev, generator=g).bfloat16()
    kcur = (torch.randn(1, n, H, 128, device=dev, generator=g) + 1.5).bfloat16()
    vcur = torch.randn(1, n, H, 128, device=dev, generator=g).bfloat16()
    return q, kcur, vcur


def _check_against_one_piece(sp, kc, q, kcur, vcur, out, mem, n, persisted=True):
    from lingbot_b200 import kv_cache, ops
    if persisted:
        # the chunk landed in the cache, with the block statistics kv_cache.write keeps
        assert torch.equal(kc["k"][:, mem:mem + n], kcur) and torch.equal(kc["v"][:, mem:mem + n], vcur)
        ref_stats = {"k": kc["k"], "v": kc["v"]}
        kv_cache.refresh_stats(ref_stats, 0, mem + n)
        nb = (mem + n + 63) // 64
        assert torch.equal(kc["lbq_ksum"][:, :nb], ref_stats["lbq_ksum"][:, :nb])
        assert torch.equal(kc["lbq_vamax"][:, :nb], ref_stats["lbq_vamax"][:, :nb])
    kwin = torch.cat([kc["k"][:, :mem], kcur], dim=1)
    vwin = torch.cat([kc["v"][:, :mem], vcur], dim=1)
    w = ops.quantize_qkv(q, kwin, vwin)
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


def _setup(mem, n, H, dev, layers=1):
    from lingbot_b200 import kv_cache, peer, split
    heap = peer.PeerHeap(kv_cache.heap_bytes(layers, [1, mem + n, H, 128], torch.bfloat16)
                         + split.SplitAttention.heap_bytes(1, H, mem, n, 1), dev)
    caches = kv_cache.allocate(layers, [1, mem + n, H, 128], torch.bfloat16, dev, heap=heap)
    g = torch.Generator(device=dev).manual_seed(7)
    for kc in caches:
        kc["k"][:, :mem] = (torch.randn(1, mem, H, 128, device=dev, generator=g)
                            + 3 * torch.randn(1, 1, H, 128, device=dev, generator=g)).bfloat16()
        kc["v"][:, :mem] = torch.randn(1, mem, H, 128, device=dev, generator=g).bfloat16()
        kv_cache.refresh_stats(kc, 0, mem)
    sp = split.SplitAttention(1, H, n, mem, n, dev, heap)
    for kc in caches:
        sp.memory_changed(kc)
    torch.cuda.synchronize()
    return heap, caches, sp


@pytest.mark.parametrize("mem,n", [(640, 300), (576, 257)], ids=["mem128aligned", "mem64aligned"])
def test_split_attention_matches_single_segment(one_rank_group, mem, n):
    from lingbot_b200 import _lib
    dev, H = torch.device("cuda"), 2
    heap, (kc,), sp = _setup(mem, n, H, dev)
    for seed, persist in ((0, True), (1, False), (2, False), (3, True)):   # counters and slot parity advance
        q, kcur, vcur = _inputs(seed, mem, n, H, dev)
        before = kc["k"][:, mem:mem + n].clone()
        out = torch.empty(1, n, H, 128, dtype=torch.bfloat16, device=dev)
        sp(q, kc, kcur, vcur, out, persist=persist)
        torch.cuda.synchronize()
        assert _lib.device_status() == 0
        if not persist:                       # a denoise pass leaves the cache's chunk region alone
            assert torch.equal(kc["k"][:, mem:mem + n], before)
        _check_against_one_piece(sp, kc, q, kcur, vcur, out, mem, n, persisted=persist)


def test_split_attention_graph_replay(one_rank_group):
    """Three layers captured once in a CUDA graph, replayed with new inputs each time."""
    from lingbot_b200 import _lib
    dev, H, mem, n, L = torch.device("cuda"), 2, 640, 300, 3
    heap, caches, sp = _setup(mem, n, H, dev, layers=L)
    q = torch.zeros(L, 1, n, H, 128, dtype=torch.bfloat16, device=dev)
    kp, vp = torch.zeros_like(q), torch.zeros_like(q)
    out = torch.empty_like(q)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):             # warm-up call outside the graph
        for li in range(L):
            sp(q[li], caches[li], kp[li], vp[li], out[li])
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for li in range(L):
            sp(q[li], caches[li], kp[li], vp[li], out[li])
    for seed in (10, 11):
        for li in range(L):
            a, b, c = _inputs(seed * 10 + li, mem, n, H, dev)
            q[li].copy_(a)
            kp[li].copy_(b)
            vp[li].copy_(c)
        graph.replay()
        torch.cuda.synchronize()
        assert _lib.device_status() == 0
        for li in range(L):
            if li == L - 1:                   # the code buffers hold the last layer's window
                _check_against_one_piece(sp, caches[li], q[li], kp[li], vp[li], out[li], mem, n)
            else:
                assert torch.equal(caches[li]["k"][:, mem:], kp[li]) and torch.equal(caches[li]["v"][:, mem:], vp[li])
    del graph


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_ranks_match_one_gpu():
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={port}", os.path.join(root, "tests", "_split_worker.py")]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(["timeout", "-k", "30", "300", *cmd], cwd=root, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert r.stdout.count("RANK OK") == 2, r.stdout[-3000:]
