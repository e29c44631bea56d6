"""Sequence split of the DiT's self-attention across GPUs — replaces the head/token split of
lingbot/parallel/split_dit.py:366-445 and the head-divisibility rule of lingbot/parallel/config.py:13-17.

The reference splits attention heads across cards, so its degree must divide the 12 heads, which 8 GPUs
do not. Here every rank keeps all heads. Projections are token-sharded in whole 128-token tiles
(`share_part`), so each rank holds a contiguous share of the current chunk's q/k/v.

* `SplitAttention` (query split): rank r attends its own query rows against the whole window. The
  memory part of the window is replicated on every rank (it was replicated when it was the current
  chunk); the chunk's per-channel statistics and quantized codes cross NVLink as peer-memory stores
  into the other ranks' buffers (`peer.PeerHeap`, csrc/peer.cu), with no collective on the data path.
* `KeySplitAttention` (key-range split): rank r quantizes and attends only its tiles of the window for
  every query row, and the partial outputs go to the owners of the rows, which merge them.

The process group serves only the set-up (the exchange of the peer heaps' IPC handles, `peer.PeerHeap`)
and barriers between calls.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

Q_ALIGN = 128   # query-slice granularity: whole 128-row Q tiles, so per-warp Q scales (32 rows) match


@dataclass(frozen=True)
class ParallelConfig:
    """How one run is laid out across GPUs (the role of lingbot/parallel/config.py:6-17).
    `sp` ranks split the query tokens; there is no head-divisibility requirement."""
    sp: int = 1

    @property
    def world_size(self):
        return self.sp

    def validate(self, num_heads, world_size):
        if self.world_size != world_size:
            raise ValueError(f"{self} needs {self.world_size} processes, got {world_size}")
        if self.sp < 1:
            raise ValueError(f"sequence split degree must be >= 1, got {self.sp}")
        if num_heads < 1:
            raise ValueError("need at least one attention head")


def shard_rows(q_len, world, rank, align=Q_ALIGN):
    """Rank `rank`'s query rows [r0, r1): 128-row tiles dealt out contiguously, the last rank taking the
    remainder (it may be empty when world > tiles)."""
    tiles = (q_len + align - 1) // align
    per = -(-tiles // world)
    r0 = min(q_len, rank * per * align)
    r1 = min(q_len, (rank + 1) * per * align)
    return r0, r1


def token_part(n, world):
    """Tokens per rank of a token-sharded chunk of n tokens (the last share is zero-padded)."""
    return -(-n // world)


def pad_share(x_full, world, rank, part=None):
    """This rank's zero-padded share [B, part, H, D] of a chunk [B, n, H, D] (test and bench helper);
    shares are `token_part` tokens unless `part` is given (e.g. `share_part`)."""
    b, n, h, d = x_full.shape
    part = token_part(n, world) if part is None else part
    lo = min(n, rank * part)
    hi = min(n, lo + part)
    share = torch.zeros(b, part, h, d, dtype=x_full.dtype, device=x_full.device)
    share[:, :hi - lo] = x_full[:, lo:hi]
    return share


def share_part(n, world, align=Q_ALIGN):
    """Tokens per rank of the peer-memory split: whole 128-token tiles, so that a rank's K/V share and
    its query slice (`shard_rows`) are the same tokens and every share starts on a 64-token K block."""
    tiles = (n + align - 1) // align
    return -(-tiles // world) * align


class SplitAttention:
    """One rank's sequence-split self-attention for one layer of a chunk, exchanging over NVLink peer
    memory (replaces the head split + host-staged q/k/v exchange of lingbot/parallel/split_dit.py:366-445).

    The window is the replicated memory part of the cache (tokens [0, mem_len)) plus the current chunk
    of n_tokens, token-sharded across ranks in `share_part` slices (rank r holds chunk tokens
    [r*part, (r+1)*part) as k/v shares, and attends the same query rows). Per call, on this rank:

      1. lbq_kv_block_stats    — block statistics of the share into this rank's cache tables;
      2. lbq_share_totals_push — the share's per-channel totals -> every rank's exchange area;
         lbq_chunk_totals      — wait for every rank's totals; window totals (memory + shares in rank
                                 order, identical on every rank);
      3. quantize the memory segment (K mean-smoothed int8, V e4m3) locally, while on a side stream
         lbq_share_quant_push  — this rank's share is quantized into its chunk segment and the codes
                                 copied into every other rank's,
         lbq_share_push        — (persist=True) the bf16 share and its block statistics -> every rank's
                                 cache replica and tables,
         and the query slice is quantized;
      4. lbq_peer_wait         — wait for the other ranks' pushes;
      5. attention over the two segments (memory, chunk).

    Codes and scales are identical to quantizing the whole window in one piece (mem_len % 64 == 0
    keeps the 64-token K blocks those of the whole window). `persist=False` skips the bf16 replication
    of the chunk into the caches: for the denoise passes of a chunk, whose K/V the next pass of the same
    chunk overwrites before anything reads them (only the memory-write pass's K/V stay in the cache);
    with persist=True a call leaves every rank's cache as kv_cache.write would. The caches and this
    object's code buffers are carved from `heap` (kv_cache.allocate(..., heap=heap), then this
    constructor), identically on every rank; size the heap with `heap_bytes`. Every launch is on the
    current stream (plus one forked side stream), without host synchronisation, so a call can be
    captured in a CUDA graph and replayed. `memory_changed(cache)` must be called whenever the memory
    part of a cache changes.
    """

    @staticmethod
    def heap_bytes(batch, heads, mem_len, n_tokens, world):
        """Peer-heap bytes this object carves (code buffers and exchange area, 256-byte aligned)."""
        from . import _lib
        seg_pad = -(-(mem_len if mem_len > 0 else n_tokens) // 128) * 128
        nseg = 2 if mem_len > 0 else 1
        up = lambda x: (x + 255) // 256 * 256  # noqa: E731
        per_seg = batch * heads * seg_pad
        return (up(nseg * per_seg * 128) + up(nseg * per_seg // 64 * 4) + up(nseg * per_seg * 128)
                + up(_lib.load().lbq_exchange_bytes(world, batch, heads)))

    def __init__(self, batch, heads, q_rows, mem_len, n_tokens, device, heap, group=None, timeout_s=4.0):
        from . import _lib, ops
        if mem_len % 64:
            raise ValueError("the memory part must be a whole number of 64-token blocks")
        if 0 < mem_len < n_tokens:
            raise ValueError("the chunk segment cannot be longer than the memory segment")
        self.group, self.heap = group, heap
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if heap.world != self.world or heap.rank != self.rank:
            raise ValueError("the peer heap was built for another group")
        self.b, self.h, self.q_rows = batch, heads, q_rows
        self.mem_len, self.n = mem_len, n_tokens
        self.part = share_part(n_tokens, self.world)
        self.nb_part = self.part // 64
        lo = min(n_tokens, self.rank * self.part)
        self.share_valid = min(n_tokens, lo + self.part) - lo
        self.lo = lo
        self._lo = lo if self.share_valid > 0 else 0     # an empty share writes nothing; any aligned start
        self.timeout_ns = int(timeout_s * 1e9)
        self.nseg = 2 if mem_len > 0 else 1
        self.seg_len = mem_len if mem_len > 0 else n_tokens
        seg_pad = -(-self.seg_len // 128) * 128
        cols = batch * heads * 128
        # the code buffers live in the heap: every rank stores its share's codes into every rank's copy
        self.k_codes = heap.carve((self.nseg, batch, heads, seg_pad, 128), torch.int8)
        self.k_scale = heap.carve((self.nseg, batch, heads, seg_pad // 64), torch.float32)
        self.vt_codes = heap.carve((self.nseg, batch, heads, 128, seg_pad), torch.uint8)
        xbytes = _lib.load().lbq_exchange_bytes(self.world, batch, heads)
        if xbytes <= 0:
            raise ValueError(f"no exchange layout for {self.world} ranks")
        self.xchg = heap.carve((xbytes,), torch.uint8)          # zeroed; caller barriers before first use
        self.xchg_off = heap.offset(self.xchg)
        self.q_codes, self.q_scale = ops.alloc_q(batch, heads, max(q_rows, 1), device)
        self.v_scale = torch.empty(batch, heads, 128, dtype=torch.float32, device=device)
        self.km = torch.empty(batch, heads, 128, dtype=torch.bfloat16, device=device)
        self.tot_ksum = torch.zeros(cols, dtype=torch.float64, device=device)
        self.tot_vamax = torch.zeros(cols, dtype=torch.float32, device=device)
        # high priority: the small push kernels get SMs as soon as a quantizer CTA retires
        self.side = self.fork = self.join = None
        if torch.device(device).type == "cuda":
            self.side = torch.cuda.Stream(device=device, priority=-1)
            self.fork, self.join = torch.cuda.Event(), torch.cuda.Event()
        self.push_ctas = 64      # CTAs of the bf16 share push; the same on every rank
        self.code_ctas = 32      # CTAs of the code push (few: it shares the GPU with the memory quantizer)

    def memory_changed(self, cache):
        """Per-channel totals of the memory part from the cache's block statistics, kept in the cache
        dict (one SplitAttention, i.e. one set of code buffers, can serve every layer)."""
        from . import _lib, ops
        ksum, vamax = cache["lbq_ksum"], cache["lbq_vamax"]
        cols = self.b * self.h * 128
        if "lbq_mem_ksum" not in cache:
            cache["lbq_mem_ksum"] = torch.zeros(cols, dtype=torch.float64, device=ksum.device)
            cache["lbq_mem_vamax"] = torch.zeros(cols, dtype=torch.float32, device=ksum.device)
        if self.mem_len == 0:
            cache["lbq_mem_ksum"].zero_()
            cache["lbq_mem_vamax"].zero_()
            return
        _lib.call("lbq_kv_window_sums", ops._ptr(ksum), ops._ptr(vamax), self.b, self.h, 0, self.mem_len // 64,
                  ksum.shape[1], ops._ptr(cache["lbq_mem_ksum"]), ops._ptr(cache["lbq_mem_vamax"]), ops._stream())

    def _check_cache(self, cache):
        k = cache["k"]
        b, lk, h, d = k.shape
        if (b, h, d) != (self.b, self.h, 128) or not (k.is_contiguous() and cache["v"].is_contiguous()):
            raise ValueError("cache K/V must be contiguous [B, tokens, H, 128] buffers of this split")
        if lk < self.mem_len + self.n:
            raise ValueError(f"cache of {lk} tokens cannot hold {self.mem_len} memory + {self.n} chunk tokens")
        return self.heap.offset(k), self.heap.offset(cache["v"]), lk

    def _group(self):
        from . import ops
        return (ops._ptr(self.heap.peers), self.world, self.rank, self.xchg_off)

    @staticmethod
    def _share(k_part, v_part):
        from . import ops
        return (ops._ptr(k_part), *k_part.stride()[:3], ops._ptr(v_part), *v_part.stride()[:3])

    def _codes(self):
        from . import ops
        return (ops._ptr(self.tot_ksum), ops._ptr(self.tot_vamax), ops._ptr(self.k_codes), ops._ptr(self.k_scale),
                ops._ptr(self.vt_codes), ops._ptr(self.km), ops._ptr(self.v_scale))

    def _window_totals(self, cache, k_part, v_part, stp):
        """Steps 1-2 of a call: the share's block statistics into this rank's tables, its per-channel
        totals to every rank, and the window totals (memory + every share in rank order, identical on
        every rank) into tot_ksum / tot_vamax."""
        from . import _lib, ops
        if k_part.shape[1] < self.share_valid or v_part.shape[1] < self.share_valid:
            raise ValueError(f"shares of {k_part.shape[1]} tokens, expected {self.part}")
        b, h = self.b, self.h
        ksum, vamax = cache["lbq_ksum"], cache["lbq_vamax"]
        max_blocks = ksum.shape[1]
        row0 = (self.mem_len + self._lo) // 64
        nb_valid = (self.share_valid + 63) // 64
        group = self._group()
        if nb_valid > 0:
            _lib.call("lbq_kv_block_stats", *self._share(k_part, v_part), b, h, self.share_valid, 0, nb_valid,
                      max_blocks, ksum.data_ptr() + row0 * h * 128 * 8, vamax.data_ptr() + row0 * h * 128 * 4,
                      0, 0, 0, stp)
        _lib.call("lbq_share_totals_push", ops._ptr(ksum), ops._ptr(vamax), max_blocks, row0, nb_valid, b, h,
                  *group, stp)
        _lib.call("lbq_chunk_totals", *group, b, h, ops._ptr(cache["lbq_mem_ksum"]), ops._ptr(cache["lbq_mem_vamax"]),
                  ops._ptr(self.tot_ksum), ops._ptr(self.tot_vamax), self.timeout_ns, stp)

    def __call__(self, q_rows, cache, k_part, v_part, out, sm_scale=None, num_splits=None, attn_events=None,
                 persist=True):
        """q_rows [B, rows, H, 128] (this rank's query slice), k_part/v_part [B, part, H, 128] (this rank's
        share of the chunk, rows past the chunk's end ignored) -> out [B, rows, H, 128]. With persist=True
        the whole chunk also lands in `cache` at [mem_len, mem_len + n_tokens), with its block statistics,
        on every rank (as kv_cache.write does). Every rank makes the same calls with the same `persist`."""
        from . import _lib, ops
        st = torch.cuda.current_stream()
        stp = st.cuda_stream
        b, h = self.b, self.h
        k_off, v_off, lk = self._check_cache(cache)
        ksum, vamax = cache["lbq_ksum"], cache["lbq_vamax"]
        max_blocks = ksum.shape[1]
        group = self._group()
        share = self._share(k_part, v_part)
        kv_len = self.mem_len + self.n
        rows = q_rows.shape[1]
        nseg = self.nseg
        codes = self._codes()
        # 1.-2. block statistics of the share, window totals
        self._window_totals(cache, k_part, v_part, stp)
        # 3. side stream: the share's codes (and, persisting, its bf16) -> every rank; the query slice
        self.fork.record(st)
        self.side.wait_event(self.fork)
        sst = self.side.cuda_stream
        _lib.call("lbq_share_quant_push", *share, b, h, self._lo, self.share_valid, self.part, nseg - 1, nseg,
                  self.seg_len, kv_len, *codes, int(self.mem_len == 0), *group, self.code_ctas, sst)
        if persist:
            _lib.call("lbq_share_push", *share, b, h, self.share_valid, self.nb_part, *group, k_off, v_off, lk,
                      self.mem_len + self._lo, self.heap.offset(ksum), self.heap.offset(vamax), max_blocks,
                      self.push_ctas, sst)
        if rows > 0:
            _lib.call("lbq_quant_q", ops._ptr(q_rows), *q_rows.stride()[:3], b, h, rows, ops._ptr(self.q_codes),
                      ops._ptr(self.q_scale), sst)
        self.join.record(self.side)
        # ... while the memory segment is quantized here
        if self.mem_len > 0:
            kc, vc = cache["k"], cache["v"]
            _lib.call("lbq_quant_kv", ops._ptr(kc), *kc.stride()[:3], ops._ptr(vc), *vc.stride()[:3], b, h, 0, 0, 2,
                      self.mem_len, self.mem_len, kv_len, *codes, 1, stp)
        # 4. every rank's pushes have landed
        st.wait_event(self.join)
        _lib.call("lbq_peer_wait", *group, 1 + int(bool(persist)), self.timeout_ns, stp)
        if rows == 0:
            return out
        # 5. attention over (memory, chunk)
        w = ops.QuantWindow(self.q_codes, self.q_scale, self.k_codes, self.k_scale, self.vt_codes, self.v_scale,
                            self.km, rows, kv_len, self.seg_len, nseg)
        if attn_events is not None:
            attn_events[0].record()
        ops.attn_from_codes(w, sm_scale=sm_scale, out=out, num_splits=num_splits)
        if attn_events is not None:
            attn_events[1].record()
        return out

    def launches(self, num_splits, persist=True):
        """Our kernels per call: share block stats, totals push, window totals, share K/V quantizer, code
        push (more than one rank), bf16 share push (persist), Q quantizer, memory K/V quantizer, peer
        wait, attention (+ split-KV combine)."""
        rows = self.q_rows > 0
        return (int(self.share_valid > 0) + 2 + 1 + int(self.world > 1) + int(bool(persist)) + int(rows)
                + int(self.mem_len > 0) + 1 + int(rows) + int(num_splits > 1 and rows))


def key_tiles(mem_len, world, rank):
    """Rank `rank`'s 128-token tiles [t0, t1) of the memory segment under the key-range split: the
    ceil(mem_len / 128) tiles dealt out contiguously, as evenly as whole tiles allow."""
    tiles = -(-mem_len // 128)
    return rank * tiles // world, (rank + 1) * tiles // world


def key_ranges(mem_len, n_tokens, world, rank):
    """Rank `rank`'s keys under the key-range split, as (tile start, tiles, valid keys) per code segment
    (memory, then chunk; chunk only without a memory part): its `key_tiles` of the memory part and the
    128-token tiles of its own chunk share (none when the share is empty)."""
    part = share_part(n_tokens, world)
    lo = min(n_tokens, rank * part)
    valid = min(n_tokens, lo + part) - lo
    lo = lo if valid > 0 else 0
    chunk = (lo // 128, -(-(lo + valid) // 128) - lo // 128 if valid else 0, n_tokens)
    if mem_len == 0:
        return [chunk]
    m0, m1 = key_tiles(mem_len, world, rank)
    return [(m0, m1 - m0, mem_len), chunk]


class KeySplitAttention(SplitAttention):
    """One rank's self-attention for one layer of a chunk under the key-range split: the rank attends
    EVERY query row of the chunk, but only against its own keys — its slice of the memory part
    (`key_tiles`) and its own share of the chunk — and sends each query tile's partial result to the
    rank that owns those rows, which merges the partials of all ranks.

    Against the query split (SplitAttention) this removes the one step that does not shrink with N: the
    re-quantization of the whole memory part on every rank (Sage's codes depend on the window-global K
    mean and V absmax, so memory codes change with every call). Here a rank quantizes 1/N of the memory
    and its own share and never sends K/V codes; the exchange is the query codes (all-gathered through
    peer memory) and the partial outputs (fp16 O / row sum plus the row's (max, sum), stored by the
    attention kernel itself into the owner's receive slots). Codes are identical to quantizing the whole
    window in one piece; the merged output equals the split-KV combine over N key ranges.

    Per call, on this rank (every launch on the current stream or one forked side stream, no host
    synchronisation, so a call can be captured in a CUDA graph):

      0. side stream, from the start: lbq_quant_q of the query slice, lbq_q_push into every rank's full
         query buffers;
      1.-2. block statistics of the share and window totals, as SplitAttention;
      3. side stream: lbq_share_push (persist=True) of the bf16 share into every rank's cache replica;
         main stream: lbq_quant_kv_tiles of this rank's memory tiles and of its chunk share;
      4. lbq_peer_wait (query codes, shares);
      5. lbq_attn_fwd_keys — partials into the owners' receive slots, then a signal per rank;
      6. lbq_peer_wait (partials); lbq_keys_combine -> this rank's output rows.

    Requirements beyond SplitAttention's: with a memory part, at least one memory tile per rank; without
    one, a non-empty chunk share per rank (every rank needs a key tile).
    """

    @staticmethod
    def heap_bytes(batch, heads, mem_len, n_tokens, world):
        """Peer-heap bytes this object carves: SplitAttention's plus the full query buffers and the
        receive slots."""
        part = share_part(n_tokens, world)
        q_pad = world * part
        up = lambda x: (x + 255) // 256 * 256  # noqa: E731
        bh = batch * heads
        return (SplitAttention.heap_bytes(batch, heads, mem_len, n_tokens, world) + up(bh * q_pad * 128)
                + up(bh * q_pad // 32 * 4) + up(world * bh * part * 128 * 2) + up(world * bh * part * 8))

    def __init__(self, batch, heads, q_rows, mem_len, n_tokens, device, heap, group=None, timeout_s=4.0):
        super().__init__(batch, heads, q_rows, mem_len, n_tokens, device, heap, group=group, timeout_s=timeout_s)
        if mem_len > 0 and -(-mem_len // 128) < self.world:
            raise ValueError(f"a {mem_len}-token memory part has fewer 128-token tiles than {self.world} ranks")
        if mem_len == 0 and n_tokens <= (self.world - 1) * self.part:
            raise ValueError(f"a {n_tokens}-token chunk leaves rank {self.world - 1} without keys")
        self.q_pad = self.world * self.part
        bh = batch * heads
        self.mem_tiles = key_tiles(mem_len, self.world, self.rank) if mem_len > 0 else (0, 0)
        self.q_all = heap.carve((batch, heads, self.q_pad, 128), torch.int8)
        self.q_all_scale = heap.carve((batch, heads, self.q_pad // 32), torch.float32)
        self.recv_o = heap.carve((self.world, bh, self.part, 128), torch.float16)
        self.recv_ml = heap.carve((self.world, bh, self.part, 2), torch.float32)
        self.q_ctas = 32          # CTAs of the query-code push (few: it runs beside the quantizers)
        self.totals_done = torch.cuda.Event() if self.side is not None else None

    def ranges(self):
        """(tile start, tiles, valid keys) of each code segment this rank attends."""
        return key_ranges(self.mem_len, self.n, self.world, self.rank)

    def __call__(self, q_rows, cache, k_part, v_part, out, sm_scale=None, num_splits=None, attn_events=None,
                 persist=True):
        """q_rows [B, rows, H, 128] (this rank's query slice, rows = its share of the chunk), k_part /
        v_part [B, part, H, 128] (its share, rows past the chunk's end ignored) -> out [B, rows, H, 128].
        `num_splits` is ignored (one partial per rank). persist=True also lands the whole chunk in every
        rank's `cache` at [mem_len, mem_len + n_tokens), as kv_cache.write would."""
        import ctypes
        from . import _lib, ops
        st = torch.cuda.current_stream()
        stp = st.cuda_stream
        b, h = self.b, self.h
        k_off, v_off, lk = self._check_cache(cache)
        ksum, vamax = cache["lbq_ksum"], cache["lbq_vamax"]
        max_blocks = ksum.shape[1]
        group = self._group()
        share = self._share(k_part, v_part)
        kv_len = self.mem_len + self.n
        rows = q_rows.shape[1]
        if rows > self.part:
            raise ValueError(f"{rows} query rows, the slice holds {self.part}")
        nseg = self.nseg
        codes = self._codes()
        # side stream, from the start of the call: the query slice -> every rank. Every rank has finished
        # its previous attention, the last reader of the query buffers: this rank's previous merge waited
        # for every rank's partials, which each rank signals after its attention's last CTA.
        self.fork.record(st)
        self.side.wait_event(self.fork)
        sst = self.side.cuda_stream
        rows_pad = ops.round_up(rows, 128)
        if rows > 0:
            _lib.call("lbq_quant_q", ops._ptr(q_rows), *q_rows.stride()[:3], b, h, rows, ops._ptr(self.q_codes),
                      ops._ptr(self.q_scale), sst)
        _lib.call("lbq_q_push", ops._ptr(self.q_codes), ops._ptr(self.q_scale), rows_pad, self.rank * self.part,
                  self.q_pad, b, h, self.heap.offset(self.q_all), self.heap.offset(self.q_all_scale), *group,
                  self.q_ctas, sst)
        # 1.-2. block statistics of the share, window totals
        self._window_totals(cache, k_part, v_part, stp)
        if persist:
            # the bf16 share -> every rank's cache, after the window totals (every rank is past its
            # previous call's reads of its cache)
            self.totals_done.record(st)
            self.side.wait_event(self.totals_done)
            _lib.call("lbq_share_push", *share, b, h, self.share_valid, self.nb_part, *group, k_off, v_off, lk,
                      self.mem_len + self._lo, self.heap.offset(ksum), self.heap.offset(vamax), max_blocks,
                      self.push_ctas, sst)
        self.join.record(self.side)
        # ... while this rank's keys are quantized here: its memory tiles, then its chunk share
        if self.mem_len > 0:
            m0, m1 = self.mem_tiles
            kc, vc = cache["k"], cache["v"]
            _lib.call("lbq_quant_kv_tiles", ops._ptr(kc), *kc.stride()[:3], ops._ptr(vc), *vc.stride()[:3], b, h, 0, 0,
                      nseg, self.mem_len, self.mem_len, kv_len, *codes, 1, m0, m1, stp)
        if self.share_valid > 0:
            t0 = self._lo // 128
            _lib.call("lbq_quant_kv_tiles", *share, b, h, -self._lo, nseg - 1, nseg, self._lo + self.share_valid,
                      self.seg_len, kv_len, *codes, int(self.mem_len == 0), t0,
                      -(-(self._lo + self.share_valid) // 128), stp)
        # 4. every rank's query codes (and shares) have landed
        st.wait_event(self.join)
        _lib.call("lbq_peer_wait", *group, 1 + int(bool(persist)), self.timeout_ns, stp)
        # 5. partials of every query tile over this rank's keys -> the tiles' owners
        rg = self.ranges()
        arr = ctypes.c_int * len(rg)
        if attn_events is not None:
            attn_events[0].record()
        _lib.call("lbq_attn_fwd_keys", ops._ptr(self.q_all), ops._ptr(self.q_all_scale), self.n, self.q_pad,
                  ops._ptr(self.k_codes), ops._ptr(self.k_scale), ops._ptr(self.vt_codes), nseg, self.seg_len, b, h,
                  float(sm_scale or 0.0), arr(*[r[0] for r in rg]), arr(*[r[1] for r in rg]),
                  arr(*[r[2] for r in rg]), *group, self.part, self.heap.offset(self.recv_o),
                  self.heap.offset(self.recv_ml), stp)
        if attn_events is not None:
            attn_events[1].record()
        # 6. every rank's partials for this rank's rows -> out
        _lib.call("lbq_peer_wait", *group, 1, self.timeout_ns, stp)
        if rows > 0:
            _lib.call("lbq_keys_combine", ops._ptr(self.recv_o), ops._ptr(self.recv_ml), self.world, self.part, rows,
                      ops._ptr(self.v_scale), b, h, ops._ptr(out), *out.stride()[:3], stp)
        return out

    def launches(self, num_splits=1, persist=True):
        """Our kernels per call: share block stats, totals push, window totals, Q quantizer, query push,
        bf16 share push (persist), memory-tile quantizer, share quantizer, peer wait, attention, peer
        wait, combine."""
        rows = self.q_rows > 0
        return (int(self.share_valid > 0) + 2 + int(rows) + 1 + int(bool(persist)) + int(self.mem_len > 0)
                + int(self.share_valid > 0) + 1 + 1 + 1 + int(rows))
