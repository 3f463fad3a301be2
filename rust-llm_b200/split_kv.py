"""Long-context decode with the KV sequence split across the GPUs of one box.

Each rank holds a contiguous range of the sequence's positions in its own
bf16 cache (one rl_ctx per GPU, `rl_set_shard`).  A decode row then takes
three steps per layer:

  1. every rank walks its own positions (`rl_full_attn_partial`), the rank
     whose range holds the new position also appending its key and value,
     and leaves a partial [n_head][head_dim + 2]: unnormalised output, max
     (log2 units) and sum of weights, 16,512 bytes at the Qwen3.5 shapes;
  2. one all-gather over NCCL (NVLink) collects the world's partials;
  3. every rank merges them with the log-sum-exp rule and applies the output
     gate (`rl_merge_partials`), so each holds the `heads` row.

This is the reference's Exec::full_attn for one decode row
(crates/rust-llm/src/forward.rs:1259-1340) with its single pass over the
cache cut into ranges; nothing else of the row changes.

The orchestration is written against two small interfaces so that its host
logic (range arithmetic, gather order, merge) is testable on CPU ranks over
gloo: `Shard` (the GPU context, or a stand-in in tests) and the process
group.
"""
from __future__ import annotations

from dataclasses import dataclass


def shard_range(seq_context: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous split of seq_context positions over `world` ranks: rank r
    holds positions [lo, lo + n).  Ranges are whole multiples of 64 positions
    (the walk's tile) except the last, which takes the remainder."""
    if world < 1 or not 0 <= rank < world or seq_context < 1:
        raise ValueError(f"bad split: seq_context={seq_context} world={world} rank={rank}")
    tiles = (seq_context + 63) // 64
    per = (tiles + world - 1) // world * 64
    lo = min(rank * per, seq_context)
    hi = min(lo + per, seq_context)
    return lo, hi - lo


def owner_of(pos: int, seq_context: int, world: int) -> int:
    """The rank whose range holds sequence position `pos`."""
    for r in range(world):
        lo, n = shard_range(seq_context, world, r)
        if lo <= pos < lo + n:
            return r
    raise ValueError(f"position {pos} outside a sequence of {seq_context}")


@dataclass
class SplitDecoder:
    """Runs split decode rows on one rank.

    shard: object with partial(layer, pos, qg, k, v, out_partial) and
           merge(parts, qg, out) (rlcuda.Context-backed on GPUs);
    group: torch.distributed process group (NCCL on GPUs, gloo in tests);
    make:  allocator make(shape) for the partial and gather buffers on the
           rank's device."""

    shard: object
    world: int
    rank: int
    n_head: int
    head_dim: int
    group: object = None
    make: object = None

    def __post_init__(self):
        width = self.head_dim + 2
        self.partial = self.make((self.n_head, width))
        # gathered along dim 0, [world * n_head][width], viewed per rank
        self.gathered_flat = self.make((self.world * self.n_head, width))
        self.gathered = self.gathered_flat.view(self.world, self.n_head, width)

    def step(self, layer: int, pos: int, qg, k, v, out):
        import torch.distributed as dist
        if getattr(self.shard, "exchange", False):
            # the partials cross NVLink as peer-memory stores (no NCCL)
            self.shard.split(layer, pos, qg, k, v, out)
            return out
        self.shard.partial(layer, pos, qg, k, v, self.partial)
        if self.world > 1:
            dist.all_gather_into_tensor(self.gathered_flat, self.partial, group=self.group)
        else:
            self.gathered[0].copy_(self.partial)
        self.shard.merge(self.gathered, qg, out)
        return out


class GpuShard:
    """The GPU side of a SplitDecoder: one rl_ctx holding this rank's range.
    With `exchange`, the partials cross between GPUs through peer memory
    (rl_exchange_*, rl_full_attn_split) instead of an NCCL all-gather; the
    ranks swap their buffers' CUDA IPC handles once over the process group."""

    def __init__(self, ctx, lo: int, seq_context: int, exchange: bool = False,
                 rank: int = 0, world: int = 1, group=None):
        self.ctx = ctx
        self.exchange = exchange
        ctx.set_shard(lo, seq_context)
        if exchange:
            handle = ctx.exchange_init(rank, world)
            handles = connect_handles(handle, world, group)
            ctx.exchange_connect(handles)

    def partial(self, layer, pos, qg, k, v, out_partial):
        self.ctx.full_attn_partial(layer, pos, qg, k, v, out_partial)

    def merge(self, parts, qg, out):
        self.ctx.merge_partials(parts, qg, out)

    def split(self, layer, pos, qg, k, v, out):
        self.ctx.full_attn_split(layer, pos, qg, k, v, out)


def connect_handles(handle: bytes, world: int, group=None) -> list:
    """Every rank's exchange handle, in rank order (an all-gather of small
    host objects over the process group; the handle itself for world 1)."""
    if world == 1:
        return [handle]
    import torch.distributed as dist
    out = [None] * world
    dist.all_gather_object(out, handle, group=group)
    return out


def partition_sequences(lengths, world: int) -> list[list[int]]:
    """Independent sequences of a batch over `world` GPUs, no collective:
    longest first, each to the GPU with the least total context so far (ties
    to the lowest rank).  Returns each rank's sequence indices in the order
    they were dealt.  Decode cost is proportional to context, so this
    balances every GPU's cache traffic per step."""
    order = sorted(range(len(lengths)), key=lambda i: (-lengths[i], i))
    load = [0] * world
    parts: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        r = min(range(world), key=lambda k: (load[k], k))
        parts[r].append(i)
        load[r] += lengths[i]
    return parts
