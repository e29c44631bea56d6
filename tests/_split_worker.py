"""One rank of the multi-GPU SplitAttention check (launched by tests/test_split_gpu.py with
torch.distributed.run, one process per GPU). Every rank builds the same inputs, attends its query slice
through the peer-memory split (eagerly, then from a CUDA graph) and compares it with the single-GPU
quantized attention of the whole window; prints "RANK OK" on success. With --keys (launched by
tests/test_keysplit_gpu.py) the split is KeySplitAttention, whose output matches within tolerance
(per-rank key-range partials) instead of bit for bit."""
import datetime
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "lingbot-world-v2-realtime_b200"))
sys.path.insert(0, ROOT)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def main():
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    world, rank = dist.get_world_size(), dist.get_rank()
    from lingbot_b200 import _lib, kv_cache, ops, peer, split
    from oracle import sage_semantics as O
    keys = "--keys" in sys.argv
    cls = split.KeySplitAttention if keys else split.SplitAttention
    H, mem, n, L = 3, 1280, 700, 2
    heap = peer.PeerHeap(kv_cache.heap_bytes(L, [1, mem + n, H, 128], torch.bfloat16)
                         + cls.heap_bytes(1, H, mem, n, world), dev)
    caches = kv_cache.allocate(L, [1, mem + n, H, 128], torch.bfloat16, dev, heap=heap)
    g = torch.Generator().manual_seed(3)
    for kc in caches:
        kc["k"][:, :mem] = (torch.randn(1, mem, H, 128, generator=g) + 3 * torch.randn(1, 1, H, 128, generator=g)).bfloat16().to(dev)
        kc["v"][:, :mem] = torch.randn(1, mem, H, 128, generator=g).bfloat16().to(dev)
        kv_cache.refresh_stats(kc, 0, mem)
    r0, r1 = split.shard_rows(n, world, rank)
    sp = cls(1, H, r1 - r0, mem, n, dev, heap)
    assert sp.lo == r0 and sp.share_valid == r1 - r0
    for kc in caches:
        sp.memory_changed(kc)
    torch.cuda.synchronize()
    dist.barrier()

    def inputs(seed):
        gi = torch.Generator().manual_seed(seed)
        q = torch.randn(1, n, H, 128, generator=gi).bfloat16().to(dev)
        k = (torch.randn(1, n, H, 128, generator=gi) + 1.5).bfloat16().to(dev)
        v = torch.randn(1, n, H, 128, generator=gi).bfloat16().to(dev)
        return q, k, v

    def check(kc, q, k, v, out_rows, persisted=True):
        if persisted:
            assert torch.equal(kc["k"][:, mem:], k) and torch.equal(kc["v"][:, mem:], v), "cache replica differs"
            ref_stats = {"k": kc["k"], "v": kc["v"]}
            kv_cache.refresh_stats(ref_stats, 0, mem + n)
            assert torch.equal(kc["lbq_ksum"], ref_stats["lbq_ksum"]), "block K sums differ"
            assert torch.equal(kc["lbq_vamax"], ref_stats["lbq_vamax"]), "block V maxima differ"
        w = ops.quantize_qkv(q, torch.cat([kc["k"][:, :mem], k], 1), torch.cat([kc["v"][:, :mem], v], 1))
        ref = ops.attn_from_codes(w)
        torch.cuda.synchronize()
        if keys:
            m = O.compare(out_rows.float().cpu(), ref[:, r0:r1].float().cpu())
            assert m["cos"] >= 0.9995 and m["max_abs"] <= 2e-2, f"key split far from the one-GPU output: {m}"
        else:
            assert torch.equal(out_rows, ref[:, r0:r1]), "split output differs from the one-GPU output"

    # eager calls over both layers (denoise passes do not persist their K/V)
    for seed in range(3):
        persist = seed != 1
        for li, kc in enumerate(caches):
            q, k, v = inputs(100 * seed + li)
            out = torch.empty(1, r1 - r0, H, 128, dtype=torch.bfloat16, device=dev)
            sp(q[:, r0:r1], kc, k[:, r0:r1], v[:, r0:r1], out, persist=persist)
            torch.cuda.synchronize()
            assert _lib.device_status() == 0
            check(kc, q, k, v, out, persisted=persist)
    # graph replay
    part = sp.part
    qs = torch.zeros(L, 1, r1 - r0, H, 128, dtype=torch.bfloat16, device=dev)
    ks = torch.zeros(L, 1, part, H, 128, dtype=torch.bfloat16, device=dev)
    vs = torch.zeros_like(ks)
    outs = torch.empty_like(qs)
    full = {}
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for li in range(L):
            sp(qs[li], caches[li], ks[li], vs[li], outs[li])
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    dist.barrier()
    with torch.cuda.graph(graph):
        for li in range(L):
            sp(qs[li], caches[li], ks[li], vs[li], outs[li])
    for seed in (7, 8, 9):
        for li in range(L):
            q, k, v = inputs(1000 * seed + li)
            full[li] = (q, k, v)
            qs[li].copy_(q[:, r0:r1])
            ks[li, :, :r1 - r0].copy_(k[:, r0:r1])
            vs[li, :, :r1 - r0].copy_(v[:, r0:r1])
        graph.replay()
        torch.cuda.synchronize()
        assert _lib.device_status() == 0
        check(caches[L - 1], *full[L - 1], outs[L - 1])
        for li in range(L - 1):
            assert torch.equal(caches[li]["k"][:, mem:], full[li][1])
    del graph
    torch.cuda.synchronize()
    dist.barrier()
    heap.close()
    print(f"RANK OK {rank}", flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
