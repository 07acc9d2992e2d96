"""Host-side logic without a GPU: the drop-in entry points raise the reference's
errors before any launch, the plugin installer rebinds exactly the reference's
names, and channel sharding splits a batch into group-aligned shards whose
results (oracle on each shard, gathered over a world-size-2 gloo group)
equal the unsharded result."""
import os
import socket
import sys
import types

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from greta_plugin_b200 import (dynamic_causal_conv1d, dynamic_causal_conv1d_decode, dynamic_causal_conv1d_inference,
                               packed_dynamic_conv_triton)
from greta_plugin_b200.sharding import channel_shard, shard_packed_inputs, shard_training_inputs

# ---------------------------------------------------------------- drop-in errors


def test_training_shape_errors_match_reference():
    x = torch.randn(1, 8, 64)
    with pytest.raises(ValueError, match="physical batch size B=1"):
        dynamic_causal_conv1d(torch.randn(2, 8, 64), torch.randn(8, 4, 64), None, None, 1)
    with pytest.raises(ValueError, match=r"weight must be \[T, W, D // group_size\]"):
        dynamic_causal_conv1d(x, torch.randn(8, 4, 32), None, None, 1)
    with pytest.raises(ValueError, match="must divide one of BD"):
        dynamic_causal_conv1d(torch.randn(1, 8, 96), torch.randn(8, 4, 32), None, None, 3)
    with pytest.raises(ValueError, match="gate shape"):
        dynamic_causal_conv1d(x, torch.randn(8, 4, 64), torch.randn(1, 7, 64), None, 1)
    with pytest.raises(ValueError, match="requires CUDA tensors"):
        dynamic_causal_conv1d(x, torch.randn(8, 4, 64), None, None, 1)


def test_inference_and_decode_shape_errors_match_reference():
    """Like the reference, these entry points test for CUDA tensors first
    (greta/dynamic_conv.py:657-658, :737-738), then the shapes."""
    from greta_plugin_b200.dynamic_conv import _check_decode_shapes, _check_inference_shapes

    with pytest.raises(ValueError, match="requires CUDA tensors"):
        dynamic_causal_conv1d_inference(torch.randn(2, 11, 64), torch.randn(2, 8, 4, 64), None, 1)
    with pytest.raises(ValueError, match="requires CUDA tensors"):
        dynamic_causal_conv1d_decode(torch.randn(2, 64), torch.randn(2, 4, 64), torch.randn(2, 64, 3), None, 1)
    with pytest.raises(ValueError, match="exactly W-1 history tokens"):
        _check_inference_shapes(torch.randn(2, 10, 64), torch.randn(2, 8, 4, 64), None, 1)
    with pytest.raises(ValueError, match="does not match weight batch"):
        _check_inference_shapes(torch.randn(2, 11, 64), torch.randn(3, 8, 4, 64), None, 1)
    with pytest.raises(ValueError, match="expected hidden_size // group_size=32"):
        _check_inference_shapes(torch.randn(2, 11, 64), torch.randn(2, 8, 4, 64), None, 2)
    assert _check_inference_shapes(torch.randn(2, 11, 64), torch.randn(2, 8, 4, 32), torch.randn(2, 8, 64), 2) == \
        (2, 8, 64, 4)
    with pytest.raises(ValueError, match="kernel_size >= 2"):
        _check_decode_shapes(torch.randn(2, 64), torch.randn(2, 1, 64), None, torch.randn(2, 64, 0), 1)
    with pytest.raises(ValueError, match=r"conv_state must be \(2, 64, 3\)"):
        _check_decode_shapes(torch.randn(2, 64), torch.randn(2, 4, 64), None, torch.randn(2, 64, 2), 1)
    with pytest.raises(ValueError, match="divide 128"):
        _check_decode_shapes(torch.randn(2, 512), torch.randn(2, 4, 2), None, torch.randn(2, 512, 3), 256)
    assert _check_decode_shapes(torch.randn(2, 64), torch.randn(2, 4, 64), None, torch.randn(2, 64, 3), 1) == (2, 64, 4)


def test_packed_errors_match_reference():
    x, st = torch.randn(5, 64), torch.randn(4, 64, 3)
    starts, slots, ini = torch.tensor([0, 5]), torch.tensor([1]), torch.tensor([1])
    with pytest.raises(ValueError, match="power-of-two group size"):
        packed_dynamic_conv_triton(x, torch.randn(5, 4, 64 // 4), None, st, starts, slots, ini, 3)
    with pytest.raises(ValueError, match="weight/group dimensions"):
        packed_dynamic_conv_triton(x, torch.randn(5, 4, 32), None, st, starts, slots, ini, 1)
    with pytest.raises(ValueError, match="cache has the wrong shape"):
        packed_dynamic_conv_triton(x, torch.randn(5, 4, 64), None, torch.randn(4, 64, 2), starts, slots, ini, 1)
    with pytest.raises(ValueError, match="requires CUDA tensors"):
        packed_dynamic_conv_triton(x, torch.randn(5, 4, 64), None, st, starts, slots, ini, 1)
    # T == 0 returns the (empty) output without touching anything
    out = packed_dynamic_conv_triton(torch.empty(0, 64), torch.empty(0, 4, 64), None, st, torch.tensor([0, 0]),
                                     slots, ini, 1)
    assert out.shape == (0, 64)


# ---------------------------------------------------------------- plugin installation


def _fake_reference(monkeypatch):
    """Modules named like the reference plugin's, holding placeholders."""
    sentinel = object()
    mods = {}
    for name, attrs in {
        "greta": [],
        "greta.dynamic_conv": ["dynamic_causal_conv1d", "dynamic_causal_conv1d_decode",
                               "dynamic_causal_conv1d_inference", "DynamicCausalConv1dFunction", "dynconv_fwd",
                               "dynconv_bwd"],
        "greta.modeling_greta": ["_TRITON_DYNAMIC_CAUSAL_CONV1D", "_TRITON_DYNAMIC_CAUSAL_CONV1D_DECODE",
                                 "_TRITON_DYNAMIC_CAUSAL_CONV1D_INFERENCE",
                                 "triton_dynamic_causal_conv1d_autograd_from_context"],
        "greta_vllm": [],
        "greta_vllm.triton_conv": ["packed_dynamic_conv_triton", "supports"],
        "greta_vllm.model": ["packed_dynamic_conv_triton", "triton_supports"],
    }.items():
        m = types.ModuleType(name)
        for a in attrs:
            setattr(m, a, sentinel)
        mods[name] = m
        monkeypatch.setitem(sys.modules, name, m)
    class GretaDynamicConv:
        def forward(self, hidden_states, past_key_values=None, use_cache=False, attention_mask=None):
            return "reference forward"

    mods["greta.modeling_greta"].GretaDynamicConv = GretaDynamicConv
    calls = []
    mods["greta_vllm"].register = lambda: calls.append("reference register")
    return mods, sentinel, calls


def test_install_rebinds_reference_names(monkeypatch):
    from greta_plugin_b200 import integration

    mods, sentinel, calls = _fake_reference(monkeypatch)
    integration.register()
    assert calls == ["reference register"]
    for name in ("greta.dynamic_conv", "greta.modeling_greta", "greta_vllm.triton_conv", "greta_vllm.model"):
        for attr, v in vars(mods[name]).items():
            if not attr.startswith("__"):
                assert v is not sentinel, f"{name}.{attr} was not rebound"
    assert mods["greta_vllm.model"].triton_supports(128, 4096)
    assert mods["greta.modeling_greta"]._TRITON_DYNAMIC_CAUSAL_CONV1D is dynamic_causal_conv1d
    # the cached-prefill wrapper is installed once and keeps the reference
    # forward for everything it does not take (here: no cache)
    cls = mods["greta.modeling_greta"].GretaDynamicConv
    assert getattr(cls.forward, "__greta_b200__", False)
    wrapped = cls.forward
    integration.install_hf()
    assert cls.forward is wrapped
    assert cls().forward(torch.zeros(1, 2, 4)) == "reference forward"


def test_install_refuses_unknown_reference_version(monkeypatch):
    from greta_plugin_b200 import integration

    mods, _, _ = _fake_reference(monkeypatch)
    delattr(mods["greta_vllm.model"], "triton_supports")
    with pytest.raises(AttributeError, match="unexpected reference version"):
        integration.install_vllm()


# ---------------------------------------------------------------- channel sharding


@pytest.mark.parametrize("D,G,world", [(4096, 1, 2), (4096, 128, 8), (384, 128, 2), (640, 64, 3), (256, 256, 1)])
def test_channel_shards_tile_the_channels(D, G, world):
    shards = [channel_shard(D, G, world, r) for r in range(world)]
    assert shards[0].lo == 0 and shards[-1].hi == D
    for a, b in zip(shards, shards[1:]):
        assert a.hi == b.lo
    for s in shards:
        assert s.lo % G == 0 and s.hi % G == 0 and s.channels > 0
    sizes = [s.channels // G for s in shards]
    assert max(sizes) - min(sizes) <= 1


def test_channel_shard_rejects_bad_splits():
    with pytest.raises(ValueError):
        channel_shard(256, 128, 4, 0)  # two groups over four ranks
    with pytest.raises(ValueError):
        channel_shard(100, 8, 2, 0)
    with pytest.raises(ValueError):
        channel_shard(256, 1, 2, 2)


def _packed_case(seed=0, D=384, W=4, G=64):
    from oracle import oracle  # noqa: F401  (build before the ranks start)

    rng = np.random.default_rng(seed)
    lens = [1, 1, 7, 0, 40, 3]
    T = sum(lens)
    slots = np.array([2, -1, 0, 5, 3, 1])
    init = np.array([1, 0, 1, 0, 1, 0])
    starts = np.concatenate([[0], np.cumsum(lens)])
    x = rng.standard_normal((T, D)).astype(np.float32)
    w = (0.5 * rng.standard_normal((T, W, D // G))).astype(np.float32)
    gate = rng.standard_normal((T, D)).astype(np.float32)
    state = rng.standard_normal((6, D, W - 1)).astype(np.float32)
    return x, w, gate, state, starts, slots, init, G


def _rank_main(rank, world, port, result_dir):
    from oracle import oracle

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        x, w, gate, state, starts, slots, init, G = _packed_case()
        D = x.shape[1]
        sh = channel_shard(D, G, world, rank)
        xs, ws, gs, ss = shard_packed_inputs(sh, torch.from_numpy(x), torch.from_numpy(w), torch.from_numpy(gate),
                                             torch.from_numpy(state))
        y, st = oracle.packed(xs.numpy(), ws.numpy(), gs.numpy(), ss.numpy(), starts, slots, init, G, 2)
        # training inputs shard the same way
        xt, wt, gt = shard_training_inputs(sh, torch.from_numpy(x)[None], torch.from_numpy(w),
                                           torch.from_numpy(gate)[None])
        yt, _ = oracle.fwd(xt[0].numpy(), wt.numpy(), gt[0].numpy(), starts, G, 1)
        outs = {}
        for name, t in (("y", torch.from_numpy(y)), ("state", torch.from_numpy(st)), ("train", torch.from_numpy(yt))):
            parts = [None] * world
            dist.all_gather_object(parts, t)
            outs[name] = torch.cat(parts, dim=1)
        if rank == 0:
            torch.save(outs, os.path.join(result_dir, "gathered.pt"))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_channel_sharded_packed_batch_matches_unsharded(tmp_path):
    """Two gloo ranks each run their channel shard of a packed vLLM batch and
    of a training forward; the gathered outputs and slot states equal the
    unsharded results bit for bit (the conv and the group norm never cross a
    group-aligned shard boundary)."""
    from oracle import oracle

    x, w, gate, state, starts, slots, init, G = _packed_case()
    y_full, st_full = oracle.packed(x, w, gate, state, starts, slots, init, G, 2)
    yt_full, _ = oracle.fwd(x, w, gate, starts, G, 1)
    mp.start_processes(_rank_main, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    got = torch.load(tmp_path / "gathered.pt")
    assert np.array_equal(got["y"].numpy(), y_full)
    assert np.array_equal(got["state"].numpy(), st_full)
    assert np.array_equal(got["train"].numpy(), yt_full)
