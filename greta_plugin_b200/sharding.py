"""Channel sharding of the dynamic convolution across GPUs.

The conv is depthwise: channel d only ever reads channel d of x and of the
cache-slot state, and its filter f = d // G. Splitting the channels into
contiguous, group-aligned shards (rank r owns channels [lo, hi) with
lo, hi multiples of G) therefore needs no communication for the conv itself:
each rank runs the same kernels on its slice of x, gate, the filter columns
[lo/G, hi/G) and the state channels. This is the layout of vLLM's
column-parallel in_proj / gate_proj / kernel_proj (the reference adapter is
single-GPU only, greta_vllm/model.py:51-55; TP is new work), where the
all-reduce happens after the row-parallel out_proj, outside this op.
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class ChannelShard:
    rank: int
    world: int
    lo: int  # first channel
    hi: int  # one past the last channel
    group_size: int

    @property
    def channels(self) -> int:
        return self.hi - self.lo

    @property
    def filters(self) -> slice:
        return slice(self.lo // self.group_size, self.hi // self.group_size)

    @property
    def chan(self) -> slice:
        return slice(self.lo, self.hi)


def channel_shard(channels: int, group_size: int, world: int, rank: int) -> ChannelShard:
    """Contiguous group-aligned shard of `channels` for `rank` of `world`.

    Groups are dealt as evenly as possible (the first `groups % world` ranks
    get one extra group). Raises ValueError when a rank would get no group."""
    if channels % group_size:
        raise ValueError(f"group_size={group_size} must divide channels={channels}")
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} out of range for world size {world}")
    groups = channels // group_size
    if groups < world:
        raise ValueError(f"{groups} channel groups cannot be split over {world} ranks")
    base, extra = divmod(groups, world)
    g0 = rank * base + min(rank, extra)
    g1 = g0 + base + (1 if rank < extra else 0)
    return ChannelShard(rank, world, g0 * group_size, g1 * group_size, group_size)


def shard_packed_inputs(shard: ChannelShard, x, weights, gate, state):
    """Views (x, weights, gate, state) of a vLLM packed batch restricted to a
    shard: x / gate [T, D] -> [T, D_r]; weights [T, W, D/G] -> [T, W, D_r/G];
    state [slots, D, W-1] -> [slots, D_r, W-1] (a strided view, updated in place
    by the kernels)."""
    xs = x[:, shard.chan]
    ws = weights[:, :, shard.filters]
    gs = gate[:, shard.chan] if gate is not None else None
    ss = state[:, shard.chan, :]
    return xs, ws, gs, ss


def shard_training_inputs(shard: ChannelShard, x, weight, gate):
    """Views of training inputs x [1, T, D], weight [T, W, D/G], gate [1, T, D]."""
    xs = x[:, :, shard.chan]
    ws = weight[:, :, shard.filters]
    gs = gate[:, :, shard.chan] if gate is not None else None
    return xs, ws, gs


__all__ = ["ChannelShard", "channel_shard", "shard_packed_inputs", "shard_training_inputs"]
