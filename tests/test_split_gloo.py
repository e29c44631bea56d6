"""Host-side logic of the sequence split on CPU ranks (gloo, world size 2): query slices, token shares,
the all-gather's token order, and that a rank leaving makes the others' collective fail instead of hang."""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from lingbot_b200 import split


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=60):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))


def _gather_worker(rank, world, port, n, q):
    _init(rank, world, port)
    try:
        g = torch.Generator().manual_seed(0)
        full = torch.randn(1, n, 3, 8, generator=g)
        got = split.gather_tokens(split.pad_share(full, world, rank), n)
        q.put((rank, bool(torch.equal(got, full))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n", [6032, 7, 1])
def test_gather_tokens_restores_token_order(n):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_worker, args=(r, world, port, n, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(60)
    assert res == {0: True, 1: True}


def _leaver_worker(rank, world, port, q):
    _init(rank, world, port, timeout_s=5)
    if rank == 1:
        # leaves between steps, with nothing in flight (flush the report first: _exit skips it)
        q.put((rank, "left"))
        q.close()
        q.join_thread()
        os._exit(0)
    try:
        dist.all_gather(list(torch.empty(world, 4).unbind(0)), torch.ones(4))
        q.put((rank, "completed"))
    except Exception as e:          # the survivor learns of it through the collective's error
        q.put((rank, "error:" + type(e).__name__))


def test_rank_leaving_fails_the_collective_not_hangs():
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


def test_token_shards_partition_the_chunk():
    for n, world in [(6032, 8), (7, 2), (1, 4)]:
        spans = [split.token_shard(n, world, r) for r in range(world)]
        covered = sum(hi - lo for lo, hi in spans)
        assert covered == n and spans[0][0] == 0


def test_parallel_config_allows_any_degree():
    """The reference requires the degree to divide the 12 heads (lingbot/parallel/config.py:16-17);
    a query split does not."""
    split.ParallelConfig(sp=8).validate(12, 8)
    with pytest.raises(ValueError):
        split.ParallelConfig(sp=8).validate(12, 4)
