"""Host side of the sequence split over peer memory, without a GPU: the C ABI's argument checks for the
exchange entry points, the ctypes argument types against the header, the peer-heap carving and its size
accounting, and the agreement of the K/V shares with the query slices."""
import ctypes
import datetime
import os
import re
import socket

import pytest
import torch
import torch.distributed as dist

from lingbot_b200 import _lib, kv_cache, peer, split

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

_C_TO_CTYPES = {"int": ctypes.c_int, "int64_t": ctypes.c_int64, "uint64_t": ctypes.c_uint64,
                "size_t": ctypes.c_size_t, "float": ctypes.c_float}


def _declarations():
    src = open(os.path.join(ROOT, "include", "lbq.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    out = {}
    for m in re.finditer(r"LBQ_API\s+[\w\s\*]+?\b(lbq_\w+)\s*\(([^)]*)\)\s*;", src):
        params = [p.strip() for p in m.group(2).replace("\n", " ").split(",") if p.strip() not in ("", "void")]
        out[m.group(1)] = params
    return out


def _expected_ctype(param):
    decl = re.sub(r"\b(const|struct)\b", "", param).strip()
    if "*" in decl:
        return "pointer"
    ctype = decl.rsplit(" ", 1)[0].strip()
    return _C_TO_CTYPES[ctype]


def test_ctypes_argument_types_match_the_header():
    decls = _declarations()
    assert set(decls) == set(_lib.SIGNATURES)
    for name, params in decls.items():
        argtypes = _lib.SIGNATURES[name][1]
        assert len(argtypes) == len(params), f"{name}: {len(argtypes)} ctypes args, header has {len(params)}"
        for i, (p, t) in enumerate(zip(params, argtypes)):
            exp = _expected_ctype(p)
            if exp == "pointer":
                assert t is ctypes.c_void_p or issubclass(t, ctypes._Pointer), f"{name} arg {i} ({p}) is {t}"
            else:
                assert t is exp, f"{name} arg {i} ({p}): ctypes {t}, header {exp}"


def _err():
    return _lib._lib.lbq_last_error()


def test_exchange_entry_points_check_their_arguments_before_any_cuda_call():
    lib = _lib.load()
    fake = ctypes.c_void_p(0x10000)          # never dereferenced: the checks fail first
    assert lib.lbq_exchange_bytes(1, 1, 12) == 256 + 2 * 1 * 3 * 1536 * 8
    assert lib.lbq_exchange_bytes(9, 1, 12) == -1 and lib.lbq_exchange_bytes(0, 1, 12) == -1
    # group checks
    assert lib.lbq_chunk_totals(None, 2, 0, 0, 1, 12, fake, fake, fake, fake, 0, None) == 1
    assert b"peers" in _err()
    assert lib.lbq_chunk_totals(fake, 9, 0, 0, 1, 12, fake, fake, fake, fake, 0, None) == 1
    assert b"nranks" in _err()
    assert lib.lbq_chunk_totals(fake, 2, 2, 0, 1, 12, fake, fake, fake, fake, 0, None) == 1
    assert b"rank" in _err()
    assert lib.lbq_chunk_totals(fake, 2, 0, 100, 1, 12, fake, fake, fake, fake, 0, None) == 2
    assert b"xchg_off" in _err()
    # totals push: table rows must cover the share
    assert lib.lbq_share_totals_push(fake, fake, 10, 8, 4, 1, 12, fake, 2, 0, 0, None) == 1
    assert b"rows" in _err()
    # share push: destination must start on a 64-token block and fit the cache
    share = (fake, 1536, 1536, 128, fake, 1536, 1536, 128)
    assert lib.lbq_share_push(*share, 1, 12, 64, 1, fake, 2, 0, 0, 0, 256, 100, 36, 0, 256, 2, 0, None) == 1
    assert b"64-token" in _err()
    # share quant push: the share must start on a 128-token tile
    assert lib.lbq_share_quant_push(*share, 1, 12, 64, 64, 128, 1, 2, 640, 1280, fake, fake, fake, fake, fake,
                                    fake, fake, 0, fake, 2, 0, 0, 0, None) == 1
    assert b"multiples of 128" in _err()
    assert lib.lbq_peer_wait(fake, 2, 0, 0, 3, 0, None) == 1
    assert b"signals" in _err()


def test_peer_heap_carving_on_one_rank():
    heap = peer.PeerHeap(1 << 20, torch.device("cpu"))
    assert heap.world == 1 and heap.peer_ptrs == [heap.buf.data_ptr()]
    a = heap.carve((3, 5), torch.float64)
    b = heap.carve((7,), torch.int8)
    c = heap.carve((2, 2), torch.float32)
    for t in (a, b, c):
        assert heap.offset(t) % peer.ALIGN == 0 and not t.any()
    assert heap.offset(b) >= heap.offset(a) + 3 * 5 * 8 and heap.offset(c) >= heap.offset(b) + 7
    with pytest.raises(MemoryError):                 # the request is rounded up to 2 MiB
        heap.carve((heap.nbytes,), torch.uint8)
    with pytest.raises(ValueError):
        heap.offset(torch.zeros(4))


@pytest.fixture
def one_rank_gloo():
    if dist.is_initialized():
        pytest.skip("a process group is already initialised")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=1,
                            timeout=datetime.timedelta(seconds=30))
    yield
    dist.destroy_process_group()


@pytest.mark.parametrize("cls", [split.SplitAttention, split.KeySplitAttention], ids=["queries", "keys"])
@pytest.mark.parametrize("mem,n,heads,layers", [(24128, 6032, 12, 2), (640, 300, 2, 3), (0, 300, 2, 1)])
def test_heap_bytes_cover_the_caches_and_the_split(one_rank_gloo, cls, mem, n, heads, layers):
    """kv_cache.heap_bytes + <split>.heap_bytes is exactly what the carves take."""
    need = kv_cache.heap_bytes(layers, [1, mem + n, heads, 128], torch.bfloat16)
    need += cls.heap_bytes(1, heads, mem, n, 1)
    heap = peer.PeerHeap(need, torch.device("cpu"))
    heap.nbytes = need                        # no slack from the 2 MiB rounding
    caches = kv_cache.allocate(layers, [1, mem + n, heads, 128], torch.bfloat16, "cpu", heap=heap)
    sp = cls(1, heads, n, mem, n, torch.device("cpu"), heap)
    assert heap.top <= need
    for c in caches:
        for key in ("k", "v", "lbq_ksum", "lbq_vamax"):
            heap.offset(c[key])
    assert sp.xchg_off % 256 == 0 and sp.nseg == (2 if mem else 1)
    assert sp.k_codes.shape == (sp.nseg, 1, heads, -(-sp.seg_len // 128) * 128, 128)


@pytest.mark.parametrize("world", range(1, 9))
def test_shares_are_the_query_slices(world):
    """Rank r's K/V share [r*part, (r+1)*part) is its query slice, for every N up to a node."""
    n = 6032
    part = split.share_part(n, world)
    assert part % 128 == 0 and part * world >= n
    covered = 0
    for r in range(world):
        r0, r1 = split.shard_rows(n, world, r)
        lo = min(n, r * part)
        assert (r0, r1) == (lo, min(n, lo + part))
        covered += r1 - r0
    assert covered == n
