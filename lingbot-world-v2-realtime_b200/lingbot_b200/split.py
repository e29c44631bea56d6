"""Sequence split of the DiT's self-attention across GPUs — replaces the head/token split of
lingbot/parallel/split_dit.py:366-445 and the head-divisibility rule of lingbot/parallel/config.py:13-17.

The reference splits attention heads across cards (Ulysses), so its degree must divide the 12 heads,
which 8 GPUs do not. Here every rank keeps all heads and a 128-row slice of the chunk's queries: query
rows are independent given the full key window. Projections are token-sharded, so each rank holds a
contiguous share of the current chunk's K/V; `gather_tokens` all-gathers it (NCCL over NVLink on the
GPU, gloo on the CPU) into the rank's replica of the cache. The memory part of the window is already
replicated on every rank: it was gathered when it was the current chunk.
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


def token_shard(n, world, rank):
    """Rank `rank`'s contiguous token share [lo, hi) of a chunk of n tokens."""
    part = token_part(n, world)
    lo = min(n, rank * part)
    return lo, min(n, lo + part)


def gather_tokens(x_part, n, group=None, out=None):
    """All-gather token shares [B, part, H, D] (zero-padded to `token_part(n, world)`) into the whole
    chunk [B, n, H, D], in token order (rank-major == token order)."""
    world = dist.get_world_size(group)
    b, part, h, d = x_part.shape
    if part != token_part(n, world):
        raise ValueError(f"share of {part} tokens, expected {token_part(n, world)} for n={n}, world={world}")
    buf = out if out is not None else torch.empty(world, b, part, h, d, dtype=x_part.dtype, device=x_part.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(buf, x_part.contiguous(), group=group)
    else:
        dist.all_gather(list(buf.unbind(0)), x_part.contiguous(), group=group)
    return buf.permute(1, 0, 2, 3, 4).reshape(b, world * part, h, d)[:, :n]


def pad_share(x_full, world, rank):
    """This rank's zero-padded share [B, part, H, D] of a chunk [B, n, H, D] (test and bench helper)."""
    b, n, h, d = x_full.shape
    part = token_part(n, world)
    lo, hi = token_shard(n, world, rank)
    share = torch.zeros(b, part, h, d, dtype=x_full.dtype, device=x_full.device)
    share[:, :hi - lo] = x_full[:, lo:hi]
    return share


def attend_split(q_rows, cache, k_part, v_part, current_start, sink_tokens, local_attn_size,
                 max_attention_size, n_tokens, group=None, sm_scale=None):
    """One rank's self-attention for a chunk: gather the chunk's K/V shares, write them into this rank's
    cache replica (kv_cache.write, which refreshes the block statistics), quantize the window and attend
    this rank's query rows `q_rows` [B, r1-r0, H, 128]. Returns (out_rows, local_end, current_end);
    the caller commits (kv_cache.commit) after the chunk's forward, as the reference does."""
    from . import kv_cache
    k = gather_tokens(k_part, n_tokens, group)
    v = gather_tokens(v_part, n_tokens, group)
    end, cur_end = kv_cache.write(cache, k, v, current_start, sink_tokens, local_attn_size)
    if end > max_attention_size:
        raise NotImplementedError("the window must start at token 0 of the cache (kv_size <= max_attention_size)")
    out = kv_cache.attend(q_rows, cache, end - n_tokens, end, sm_scale=sm_scale)
    return out, end, cur_end
