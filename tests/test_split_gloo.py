"""Host-side logic of the sequence split on CPU ranks (gloo, world size 2): query slices, token shares,
the set-up's exchange of peer-heap records (the split's one collective), and that a rank leaving before it
makes the others' call fail instead of hang."""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from lingbot_b200 import peer, split


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=60):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))


def _exchange_worker(rank, world, port, sizes, q):
    _init(rank, world, port)
    try:
        rec = (bytes([rank]) * 64, 4096 * rank, sizes[rank])
        try:
            got = peer.exchange_records(rec)
            q.put((rank, [(h[0], o, n) for h, o, n in got]))
        except ValueError as e:
            q.put((rank, "mismatch:" + str(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("sizes", [(1 << 21, 1 << 21), (1 << 21, 1 << 22)], ids=["same", "mismatched"])
def test_peer_records_are_exchanged_in_rank_order(sizes):
    """PeerHeap's set-up exchange: every rank receives every rank's record in rank order, and a heap size
    that differs between ranks is rejected on every rank."""
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_exchange_worker, args=(r, world, port, sizes, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(60)
    if sizes[0] == sizes[1]:
        assert res == {r: [(0, 0, sizes[0]), (1, 4096, sizes[1])] for r in range(world)}
    else:
        assert all(str(v).startswith("mismatch:") for v in res.values()), res


def _leaver_worker(rank, world, port, q):
    _init(rank, world, port, timeout_s=5)
    if rank == 1:
        # leaves before the set-up, with nothing in flight (flush the report first: _exit skips it)
        q.put((rank, "left"))
        q.close()
        q.join_thread()
        os._exit(0)
    try:
        peer.exchange_records((bytes(64), 0, 1 << 21))
        q.put((rank, "completed"))
    except Exception as e:          # the survivor learns of it through the collective's error
        q.put((rank, "error:" + type(e).__name__))


def test_rank_leaving_fails_the_setup_not_hangs():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_leaver_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(60)
        if p.is_alive():
            p.kill()
    assert res[1] == "left"
    assert res[0].startswith("error:"), res


@pytest.mark.parametrize("q_len,world", [(6032, 1), (6032, 2), (6032, 8), (300, 4), (129, 8)])
def test_shard_rows_cover_the_chunk_in_tiles(q_len, world):
    spans = [split.shard_rows(q_len, world, r) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == q_len
    for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
        assert a1 == b0
    for r0, r1 in spans:
        assert (r0 % 128 == 0 or r0 == q_len) and r1 >= r0


def test_share_parts_partition_the_chunk_in_tiles():
    """share_part: whole 128-token tiles per rank, covering the chunk once (a rank's share and its query
    slice are the same tokens)."""
    for n, world in [(6032, 8), (6032, 2), (7, 2), (300, 4)]:
        part = split.share_part(n, world)
        assert part % 128 == 0 and part * world >= n > part * (world - 1) - 128
        spans = [(min(n, r * part), min(n, (r + 1) * part)) for r in range(world)]
        assert sum(hi - lo for lo, hi in spans) == n
        assert [s[0] for s in spans] == [split.shard_rows(n, world, r)[0] for r in range(world)]


def test_parallel_config_allows_any_degree():
    """The reference requires the degree to divide the 12 heads (lingbot/parallel/config.py:16-17);
    a query split does not."""
    split.ParallelConfig(sp=8).validate(12, 8)
    with pytest.raises(ValueError):
        split.ParallelConfig(sp=8).validate(12, 4)
