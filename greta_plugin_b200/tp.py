"""Tensor-parallel Greta convolution layer (vLLM's column- / row-parallel split).

The reference vLLM adapter runs on one GPU only: `validate_config` rejects
tensor_parallel_size != 1 (greta_vllm/model.py:51-55) and the conv state is
sized with tp_world_size=1 (greta_vllm/model.py:272-276). This module is the
tensor-parallel form of its GretaConv layer (greta_vllm/model.py:85-182):

  in_proj, gate_proj, kernel_proj  column-parallel: rank r computes the conv
                                   inputs, gates and filters of its channel
                                   shard from the full hidden states;
  the convolution                  the B200 packed kernel on the rank's
                                   channels and on its slice of the cache
                                   state [slots, D/N, W-1] -- the conv is
                                   depthwise, so it needs no communication;
  out_proj                         row-parallel: each rank multiplies its
                                   channels' outputs by its column block of
                                   out_proj and the partial sums are
                                   all-reduced (NCCL) into the layer output.

kernel_proj's output row is tap-major, index k * F + f for tap k and filter
f (the `.view(n, kernel_size, num_conv_filters)` of greta_vllm/model.py:121-
122), so a rank's filters are not one contiguous block of its weight rows:
`shard_layer_weights` gathers rows k * F + [f0, f1) for every tap into one
[W * F_r, hidden] block (and the bias likewise), so that the rank's GEMM
writes its filters directly in the compact [T, W, F_r] layout the kernel
reads.

Optionally (`fused=True`) the three column-parallel projections are one GEMM
over the concatenated weight [D_r | D_r | W * F_r (+ padding), hidden]; the
convolution reads x, gate and filters in place from that one output through
its row strides (no split copies). That saves two GEMM launches and two reads
of the hidden states per layer call.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

from .sharding import channel_shard


def validate_tp(hidden_dim: int, group_size: int, kernel_size: int, tp_world_size: int) -> None:
    """The conditions under which GretaConv splits over `tp_world_size` ranks
    with vLLM's even division (`divide(intermediate_size, tp_world_size)` in
    MambaStateShapeCalculator.short_conv_state_shape): whole filter groups
    per rank, the same number on every rank. Replaces the reference's
    tensor_parallel_size == 1 requirement (greta_vllm/model.py:51-55)."""
    if tp_world_size < 1:
        raise ValueError("tensor_parallel_size must be >= 1")
    if kernel_size < 2:
        raise ValueError("This Greta adapter requires kernel_size >= 2 for its state cache")
    if hidden_dim % group_size:
        raise ValueError("hidden_dim must be divisible by num_k_heads")
    filters = hidden_dim // group_size
    if filters % tp_world_size:
        raise ValueError(f"Greta tensor parallelism needs the {filters} convolution filter groups to split evenly "
                         f"over tensor_parallel_size={tp_world_size}")


def conv_state_shape(hidden_dim: int, kernel_size: int, tp_world_size: int = 1, dim_first: bool = True):
    """Per-rank conv-state shape of one cache slot: (D / tp, W - 1) in the
    dim-first (DS) orientation, else (W - 1, D / tp) -- the shape
    greta_vllm/model.py:272-276 computes with tp_world_size=1."""
    if hidden_dim % tp_world_size:
        raise ValueError(f"hidden_dim={hidden_dim} is not divisible by tensor_parallel_size={tp_world_size}")
    d = hidden_dim // tp_world_size
    return (d, kernel_size - 1) if dim_first else (kernel_size - 1, d)


@dataclass
class TPConvWeights:
    """One rank's shard of a GretaConv layer's weights."""
    in_proj: torch.Tensor       # [D_r, hidden]
    gate_proj: torch.Tensor     # [D_r, hidden]
    kernel_proj: torch.Tensor   # [W * F_r, hidden], rows tap-major (k * F_r + f)
    kernel_bias: torch.Tensor   # [W * F_r]
    out_proj: torch.Tensor      # [hidden, D_r] (a contiguous column block)
    lo: int                     # first channel of the shard
    hi: int                     # one past the last channel


def shard_layer_weights(in_proj, gate_proj, kernel_proj, kernel_bias, out_proj, kernel_size: int, group_size: int,
                        rank: int, world: int) -> TPConvWeights:
    """Column-parallel shards of in_proj / gate_proj / kernel_proj and the
    row-parallel shard of out_proj for `rank` of `world` (full weights in the
    reference's nn.Linear layout, [out_features, in_features])."""
    D = in_proj.shape[0]
    validate_tp(D, group_size, kernel_size, world)
    sh = channel_shard(D, group_size, world, rank)
    Fn = D // group_size
    f0, f1 = sh.filters.start, sh.filters.stop
    rows = torch.cat([torch.arange(k * Fn + f0, k * Fn + f1) for k in range(kernel_size)]).to(kernel_proj.device)
    return TPConvWeights(
        in_proj=in_proj[sh.lo:sh.hi].contiguous(),
        gate_proj=gate_proj[sh.lo:sh.hi].contiguous(),
        kernel_proj=kernel_proj.index_select(0, rows).contiguous(),
        kernel_bias=kernel_bias.index_select(0, rows).contiguous(),
        out_proj=out_proj[:, sh.lo:sh.hi].contiguous(),
        lo=sh.lo, hi=sh.hi)


def _default_conv():
    from .vllm_conv import packed_dynamic_conv_triton

    return packed_dynamic_conv_triton


class TPGretaConv(torch.nn.Module):
    """One rank's part of a GretaConv layer under tensor parallelism.

    forward(hidden_states [T, hidden], state, starts, slots, has_initial)
    returns the layer output [T, hidden] (the out_proj partial sums
    all-reduced over `group` when world > 1). `state` is the rank's slice of
    the cache, [slots, D/N, W-1] in any strides (DS or SD orientation), and is
    updated in place; starts / slots / has_initial are the packed-batch
    metadata of greta_vllm.conv.metadata_to_batch, the same on every rank.

    `conv` is the packed convolution, packed_dynamic_conv_triton of this
    package by default (tests pass the reference's torch form to check the
    sharding on CPU).
    """

    def __init__(self, weights: TPConvWeights, kernel_size: int, group_size: int, norm: bool = True,
                 eps: float = 1e-6, world: int = 1, group=None, conv=None, fused: bool = False):
        super().__init__()
        self.w = weights
        self.kernel_size = kernel_size
        self.group_size = group_size
        self.norm = norm
        self.eps = eps
        self.world = world
        self.group = group
        self.conv = conv if conv is not None else _default_conv()
        self.channels = weights.hi - weights.lo
        self.filters = self.channels // group_size
        self.fused = fused
        if fused:
            # one GEMM over [in | gate | kernel] rows, padded so that the
            # output row stride is a multiple of 8 elements (16-byte rows)
            nk = kernel_size * self.filters
            width = 2 * self.channels + nk
            self.row = (width + 7) // 8 * 8
            hidden = weights.in_proj.shape[1]
            wcat = weights.in_proj.new_zeros(self.row, hidden)
            wcat[:self.channels] = weights.in_proj
            wcat[self.channels:2 * self.channels] = weights.gate_proj
            wcat[2 * self.channels:width] = weights.kernel_proj
            bcat = weights.kernel_bias.new_zeros(self.row)
            bcat[2 * self.channels:width] = weights.kernel_bias
            self.wcat, self.bcat = wcat, bcat

    @classmethod
    def from_layer(cls, layer, rank: int, world: int, group=None, conv=None, fused: bool = False):
        """From a reference GretaConv (vLLM) or GretaDynamicConv (HF) module:
        both hold in_proj / gate_proj / kernel_proj (with bias) / out_proj as
        nn.Linear (greta_vllm/model.py:91-95, greta/modeling_greta.py:426-433)."""
        cfg = getattr(layer, "config", None)
        W = cfg.kernel_size if cfg is not None else layer.kernel_size
        G = cfg.conv_group_size if cfg is not None else layer.group_size
        norm = cfg.dynconv_norm if cfg is not None else layer.norm
        eps = cfg.dynconv_norm_eps if cfg is not None else layer.norm_eps
        with torch.no_grad():
            w = shard_layer_weights(layer.in_proj.weight, layer.gate_proj.weight, layer.kernel_proj.weight,
                                    layer.kernel_proj.bias, layer.out_proj.weight, W, G, rank, world)
        return cls(w, W, G, norm, eps, world, group, conv, fused)

    def projections(self, hidden_states):
        """(x [T, D_r], filters [T, W, F_r], gate [T, D_r]) of the rank's
        channels; with fused=True all three are strided views of one GEMM
        output."""
        T = hidden_states.shape[0]
        if self.fused:
            out = F.linear(hidden_states, self.wcat, self.bcat)
            c = self.channels
            x = out[:, :c]
            gate = out[:, c:2 * c]
            filt = out[:, 2 * c:2 * c + self.kernel_size * self.filters].unflatten(1, (self.kernel_size,
                                                                                       self.filters))
            return x, filt, gate
        x = F.linear(hidden_states, self.w.in_proj)
        gate = F.linear(hidden_states, self.w.gate_proj)
        filt = F.linear(hidden_states, self.w.kernel_proj, self.w.kernel_bias).view(T, self.kernel_size, self.filters)
        return x, filt, gate

    def forward(self, hidden_states, state, starts, slots, has_initial, reduce: bool = True):
        """The layer output; with reduce=False, this rank's out_proj partial
        sum (the caller reduces)."""
        x, filt, gate = self.projections(hidden_states)
        mixed = self.conv(x, filt, gate, state, starts, slots, has_initial, self.group_size, self.norm, self.eps)
        y = F.linear(mixed, self.w.out_proj)
        if reduce and self.world > 1:
            import torch.distributed as dist

            dist.all_reduce(y, group=self.group)
        return y


__all__ = ["validate_tp", "conv_state_shape", "TPConvWeights", "shard_layer_weights", "TPGretaConv"]
