"""Failure detection on the GPU without a fault: every device-side wait of the sequence split is bounded.
A wait whose flag nothing sets gives up after its time limit, records a status code that the host reads
(lbq_device_status), and leaves the context usable. Here a one-process "group" of two ranks waits for a
rank 1 that never sends: the window-totals wait (tagged words, code 0x201) and the data-signal wait
(counters, code 0x202), each with a 50 ms limit."""
import ctypes
import time

import pytest
import torch

from oracle import sage_semantics as O
from tests._gpu import make_qkv

pytestmark = pytest.mark.gpu

TIMEOUT_NS = 50_000_000


def test_waits_give_up_with_a_status_and_the_context_stays_usable():
    from lingbot_b200 import _lib, ops
    lib = _lib.load()
    b, h = 1, 2
    up = lambda x: (x + 255) // 256 * 256  # noqa: E731
    xbytes = up(lib.lbq_exchange_bytes(2, b, h))
    area = torch.zeros(2 * xbytes, dtype=torch.uint8, device="cuda")          # rank 0's and "rank 1's" areas
    peers = torch.tensor([area.data_ptr(), area.data_ptr() + xbytes], dtype=torch.int64, device="cuda")
    cols = b * h * 128
    mem_ksum = torch.zeros(cols, dtype=torch.float64, device="cuda")
    mem_vamax = torch.zeros(cols, dtype=torch.float32, device="cuda")
    tot_ksum, tot_vamax = torch.empty_like(mem_ksum), torch.empty_like(mem_vamax)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    try:
        t0 = time.monotonic()
        _lib.call("lbq_chunk_totals", ops._ptr(peers), 2, 0, 0, b, h, ops._ptr(mem_ksum), ops._ptr(mem_vamax),
                  ops._ptr(tot_ksum), ops._ptr(tot_vamax), ctypes.c_uint64(TIMEOUT_NS), ops._stream())
        torch.cuda.synchronize()
        assert _lib.device_status() == 0x201               # a rank's share statistics never arrived
        _lib.call("lbq_peer_wait", ops._ptr(peers), 2, 0, 0, 1, ctypes.c_uint64(TIMEOUT_NS), ops._stream())
        torch.cuda.synchronize()
        assert _lib.device_status() == 0x202               # a rank's data never arrived
        assert time.monotonic() - t0 < 30                  # bounded by the limits, not by a hang
    finally:
        _lib.device_status()                               # leave the status word clear for other tests
    # the context still works
    q, k, v = make_qkv(3, 1, 2, 200, 700)
    out = ops.sage_attn(q, k, v)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    m = O.compare(out.float().cpu(), O.sage_attention(q.cpu(), k.cpu(), v.cpu()).float())
    assert m["cos"] >= 0.9995, m
