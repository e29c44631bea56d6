"""The key-range sequence split (lingbot_b200.split.KeySplitAttention; lbq_attn_fwd_keys, lbq_q_push,
lbq_keys_combine, lbq_quant_kv_tiles).

* One rank (one GPU): the whole window is this rank's key range; its codes must equal quantizing the
  window in one piece and its merged output must match the single-piece attention.
* Several ranks emulated on one GPU through the C ABI, with no waits: rank r's attention runs over its
  key ranges and stores its partials into per-owner receive buffers (regions of one device buffer
  standing in for the ranks' heaps), then each owner's rows are merged. The result must match the
  CPU emulation of the same key ranges (tolerance of the attention tests) and the one-piece output
  within the Sage tolerance.
* Two or more GPUs: tests/_split_worker.py --keys under torch.distributed.run.
"""
import ctypes
import datetime
import os
import socket
import subprocess
import sys

import pytest
import torch
import torch.distributed as dist

from oracle import sage_semantics as O
from tests._gpu import k_codes_nhd, q_codes_nhd, v_codes_nhd

pytestmark = pytest.mark.gpu

COS_MIN, MAX_ABS = 0.9995, 2e-2


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


def _window(seed, mem, n, H, dev):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(1, n, H, 128, generator=g)
    k = torch.randn(1, mem + n, H, 128, generator=g) + 3 * torch.randn(1, 1, H, 128, generator=g)
    v = torch.randn(1, mem + n, H, 128, generator=g)
    return tuple(x.bfloat16().to(dev) for x in (q, k, v))


@pytest.mark.parametrize("mem,n", [(640, 300), (576, 257), (0, 300)], ids=["mem128", "mem64", "nomem"])
def test_one_rank_key_split(one_rank_group, mem, n):
    from lingbot_b200 import _lib, kv_cache, ops, peer, split
    dev, H = torch.device("cuda"), 2
    heap = peer.PeerHeap(kv_cache.heap_bytes(1, [1, mem + n, H, 128], torch.bfloat16)
                         + split.KeySplitAttention.heap_bytes(1, H, mem, n, 1), dev)
    (kc,) = kv_cache.allocate(1, [1, mem + n, H, 128], torch.bfloat16, dev, heap=heap)
    q, kwin, vwin = _window(3, mem, n, H, dev)
    kc["k"][:, :mem] = kwin[:, :mem]
    kc["v"][:, :mem] = vwin[:, :mem]
    kv_cache.refresh_stats(kc, 0, mem)
    sp = split.KeySplitAttention(1, H, n, mem, n, dev, heap)
    sp.memory_changed(kc)
    torch.cuda.synchronize()
    w = ops.quantize_qkv(q, kwin, vwin)
    ref = ops.attn_from_codes(w)
    for persist in (True, False, True):          # counters advance across calls
        out = torch.empty(1, n, H, 128, dtype=torch.bfloat16, device=dev)
        sp(q, kc, kwin[:, mem:], vwin[:, mem:], out, persist=persist)
        torch.cuda.synchronize()
        assert _lib.device_status() == 0
        s = 1 if mem else 0                      # the chunk's code segment
        assert torch.equal(sp.k_codes[s][:, :, :n], w.k_codes[0][:, :, mem:mem + n])
        assert torch.equal(sp.vt_codes[s][..., :n], w.vt_codes[0][..., mem:mem + n])
        assert torch.equal(sp.k_scale[s][:, :, :(n + 63) // 64], w.k_scale[0][:, :, mem // 64:(mem + n + 63) // 64])
        if mem:
            assert torch.equal(sp.k_codes[0][:, :, :mem], w.k_codes[0][:, :, :mem])
            assert torch.equal(sp.vt_codes[0][..., :mem], w.vt_codes[0][..., :mem])
            assert torch.equal(sp.k_scale[0][:, :, :mem // 64], w.k_scale[0][:, :, :mem // 64])
        assert torch.equal(sp.v_scale, w.v_scale) and torch.equal(sp.km, w.km)
        assert torch.equal(sp.q_all[:, :, :n], w.q_codes[:, :, :n])
        m = O.compare(out.float().cpu(), ref.float().cpu())
        # fp16 partials (and, with 64-aligned memory, different key tiles) against the one-piece kernel
        assert m["cos"] >= 0.9999 and m["max_abs"] <= MAX_ABS, m
        if persist:
            assert torch.equal(kc["k"][:, mem:mem + n], kwin[:, mem:])


def _ranges(mem, n, world, rank):
    """Rank `rank`'s (tile start, tiles, valid keys) per code segment, and its keys in window coordinates."""
    from lingbot_b200 import split
    part = split.share_part(n, world)
    lo = min(n, rank * part)
    hi = min(n, lo + part)
    chunk = (lo // 128, -(-hi // 128) - lo // 128 if hi > lo else 0, n)
    if mem == 0:
        return [chunk], [(lo, hi)]
    t0, t1 = split.key_tiles(mem, world, rank)
    return [(t0, t1 - t0, mem), chunk], [(t0 * 128, min(mem, t1 * 128)), (mem + lo, mem + hi)]


@pytest.mark.parametrize("world", [2, 3, 8])
@pytest.mark.parametrize("mem,n", [(1280, 700), (1216, 643), (0, 1100)], ids=["mem128", "mem64", "nomem"])
def test_key_ranges_emulated_on_one_gpu(world, mem, n):
    from lingbot_b200 import _lib, ops, split
    dev, H = torch.device("cuda"), 3
    q, kwin, vwin = _window(11 + world, mem, n, H, dev)
    w = ops.quantize_qkv(q, kwin, vwin)
    ref = ops.attn_from_codes(w)
    # (memory, chunk) code segments cut from the one-piece codes (memory a whole number of 64-key blocks)
    nseg = 2 if mem else 1
    seg_len = mem if mem else n
    seg_pad = ops.round_up(seg_len, 128)
    kc = torch.zeros(nseg, 1, H, seg_pad, 128, dtype=torch.int8, device=dev)
    ks = torch.zeros(nseg, 1, H, seg_pad // 64, dtype=torch.float32, device=dev)
    vt = torch.zeros(nseg, 1, H, 128, seg_pad, dtype=torch.uint8, device=dev)
    for s, (t0, t1) in enumerate([(0, mem), (mem, mem + n)][2 - nseg:]):
        kc[s][:, :, :t1 - t0] = w.k_codes[0][:, :, t0:t1]
        vt[s][..., :t1 - t0] = w.vt_codes[0][..., t0:t1]
        ks[s][:, :, :(t1 - t0 + 63) // 64] = w.k_scale[0][:, :, t0 // 64:(t1 + 63) // 64]
    part = split.share_part(n, world)
    if mem == 0 and n <= (world - 1) * part:
        pytest.skip("the last ranks would hold no keys (KeySplitAttention rejects this split)")
    q_pad = world * part
    q_all = torch.zeros(1, H, q_pad, 128, dtype=torch.int8, device=dev)
    q_all_scale = torch.zeros(1, H, q_pad // 32, dtype=torch.float32, device=dev)
    q_all[:, :, :w.q_codes.shape[2]] = w.q_codes
    q_all_scale[:, :, :w.q_scale.shape[2]] = w.q_scale
    # one region per emulated rank: exchange area, receive slots
    lib = _lib.load()
    up = lambda x: (x + 255) // 256 * 256  # noqa: E731
    xbytes = up(lib.lbq_exchange_bytes(world, 1, H))
    o_bytes, ml_bytes = up(world * H * part * 256), up(world * H * part * 8)
    delta = xbytes + o_bytes + ml_bytes
    region = torch.zeros(world * delta, dtype=torch.uint8, device=dev)
    peers = torch.tensor([region.data_ptr() + p * delta for p in range(world)], dtype=torch.int64, device=dev)
    window_ranges = []
    for r in range(world):
        rg, keys = _ranges(mem, n, world, r)
        window_ranges.append(keys)
        arr = ctypes.c_int * len(rg)
        _lib.call("lbq_attn_fwd_keys", ops._ptr(q_all), ops._ptr(q_all_scale), n, q_pad, ops._ptr(kc), ops._ptr(ks),
                  ops._ptr(vt), nseg, seg_len, 1, H, 0.0, arr(*[x[0] for x in rg]), arr(*[x[1] for x in rg]),
                  arr(*[x[2] for x in rg]), ops._ptr(peers), world, r, 0, part, xbytes, xbytes + o_bytes,
                  ops._stream())
    out = torch.zeros(1, n, H, 128, dtype=torch.bfloat16, device=dev)
    for p in range(world):
        lo, hi = min(n, p * part), min(n, (p + 1) * part)
        base = region.data_ptr() + p * delta
        o = out[:, lo:hi]
        _lib.call("lbq_keys_combine", ctypes.c_void_p(base + xbytes), ctypes.c_void_p(base + xbytes + o_bytes), world,
                  part, hi - lo, ops._ptr(w.v_scale), 1, H, ops._ptr(o), *o.stride()[:3], ops._stream())
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    got = out.float().cpu()
    nb = (w.kv_len + 63) // 64
    emu = O.attn_from_codes(q_codes_nhd(w), w.q_scale.cpu(), k_codes_nhd(w), w.k_scale[0][:, :, :nb].cpu(),
                            v_codes_nhd(w), w.v_scale.cpu(), pv_accum="fp32", key_ranges=window_ranges,
                            partial_fp16=True)
    exact = O.compare(got, emu)
    assert exact["cos"] >= 0.99999 and exact["max_abs"] <= MAX_ABS, exact
    one_piece = O.compare(got, ref.float().cpu())
    assert one_piece["cos"] >= COS_MIN and one_piece["max_abs"] <= MAX_ABS, one_piece


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_ranks_key_split_match_one_gpu():
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={port}", os.path.join(root, "tests", "_split_worker.py"),
           "--keys"]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(["timeout", "-k", "30", "300", *cmd], cwd=root, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert r.stdout.count("RANK OK") == 2, r.stdout[-3000:]
