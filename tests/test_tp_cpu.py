"""Tensor-parallel GretaConv (greta_plugin_b200.tp) on CPU.

* the weight shards: column-parallel in/gate/kernel projections (kernel_proj's
  tap-major rows gathered per rank) and the row-parallel out_proj block
  reproduce the unsharded layer's per-channel quantities;
* two gloo ranks run the reference's own vLLM GretaConv layer
  (greta_vllm/model.py:85-182, installed in baseline/_ref) split by
  TPGretaConv.from_layer, with the reference's torch packed_dynamic_conv
  (greta_vllm/conv.py:10-70) as each rank's convolution; the all-reduced
  output equals the reference layer's own forward through its vLLM custom op,
  and the ranks' state slices equal its cache after the call.

Skipped when the reference is not installed in baseline/_ref."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from greta_plugin_b200.tp import TPGretaConv, conv_state_shape, shard_layer_weights, validate_tp

import reference_harness as rh


def test_validate_and_state_shape():
    validate_tp(2048, 128, 7, 8)  # Greta defaults: 16 filter groups over 8 ranks
    with pytest.raises(ValueError, match="split evenly"):
        validate_tp(2048, 128, 7, 32)
    with pytest.raises(ValueError, match="kernel_size >= 2"):
        validate_tp(2048, 128, 1, 2)
    assert conv_state_shape(2048, 7, 4) == (512, 6)
    assert conv_state_shape(2048, 7, 4, dim_first=False) == (6, 512)


@pytest.mark.parametrize("world", [1, 2, 4])
def test_weight_shards_reproduce_the_layer(world):
    hidden, D, W, G = 64, 64, 3, 8
    Fn = D // G
    g = torch.Generator().manual_seed(0)
    in_w, gate_w, out_w = (torch.randn(D, hidden, generator=g) for _ in range(3))
    k_w, k_b = torch.randn(W * Fn, hidden, generator=g), torch.randn(W * Fn, generator=g)
    h = torch.randn(5, hidden, generator=g)
    full_k = (h @ k_w.T + k_b).view(5, W, Fn)
    mixed = torch.randn(5, D, generator=g)
    partial = torch.zeros(5, hidden)
    for r in range(world):
        s = shard_layer_weights(in_w, gate_w, k_w, k_b, out_w, W, G, r, world)
        torch.testing.assert_close(h @ s.in_proj.T, (h @ in_w.T)[:, s.lo:s.hi])
        torch.testing.assert_close(h @ s.gate_proj.T, (h @ gate_w.T)[:, s.lo:s.hi])
        kr = (h @ s.kernel_proj.T + s.kernel_bias).view(5, W, (s.hi - s.lo) // G)
        torch.testing.assert_close(kr, full_k[:, :, s.lo // G:s.hi // G])
        partial += mixed[:, s.lo:s.hi] @ s.out_proj.T
    torch.testing.assert_close(partial, mixed @ out_w.T, rtol=1e-5, atol=1e-4)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


HIDDEN = 256


def _case(vm, cg):
    cfg, layer, prefix = rh.make_vllm_conv(vm, cg, torch.float32, "cpu", 3, 8, hidden_dim=HIDDEN, num_k_heads=32,
                                           kernel_size=4)
    md = rh.short_conv_metadata(vm, [3, 5], [4, 6], [0, 7], [True, False], "cpu")
    pos = torch.tensor([5, 0] + list(range(2, 6)) + list(range(6)))
    hs = torch.randn(12, HIDDEN, generator=torch.Generator().manual_seed(4))
    return cfg, layer, prefix, md, pos, hs


def _rank_main(rank, world, port, result_dir, reference_dir):
    import sys

    sys.path.insert(0, reference_dir)
    import greta.configuration_greta as cg
    import greta_vllm.conv as vconv
    import greta_vllm.model as vm

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        cfg, layer, prefix, md, pos, hs = _case(vm, cg)
        tp = TPGretaConv.from_layer(layer, rank, world, conv=vconv.packed_dynamic_conv,
                                    fused=bool(int(os.environ.get("GRETA_TP_TEST_FUSED", "0"))))
        state = layer.kv_cache[0]
        view = state if vm.is_conv_state_dim_first() else state.transpose(-1, -2)
        starts, _, slots, initial, n = vconv.metadata_to_batch(md, pos)
        local = view[:, tp.w.lo:tp.w.hi, :]
        with torch.no_grad():
            y = tp(hs[:n], local, starts, slots, initial)
        parts = [None] * world
        dist.all_gather_object(parts, local.clone())
        if rank == 0:
            torch.save({"y": y, "state": torch.cat(parts, dim=1)}, os.path.join(result_dir, "tp.pt"))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("fused", [False, True])
def test_tp_layer_on_two_gloo_ranks_matches_the_reference_layer(tmp_path, monkeypatch, fused):
    rdc, mg, cg = rh.reference_modules(triton=False)
    vconv, vtc, vm = rh.vllm_reference_modules()
    import conftest

    cfg, layer, prefix, md, pos, hs = _case(vm, cg)
    with torch.no_grad(), rh.forward_context(vm, layer, prefix, md):
        ref = layer(hs, pos)
    ref_state = layer.kv_cache[0]
    ref_view = ref_state if vm.is_conv_state_dim_first() else ref_state.transpose(-1, -2)
    monkeypatch.setenv("GRETA_TP_TEST_FUSED", "1" if fused else "0")
    mp.start_processes(_rank_main, args=(2, _free_port(), str(tmp_path), str(conftest.REFERENCE_DIR)), nprocs=2,
                       join=True, start_method="spawn")
    got = torch.load(tmp_path / "tp.pt")
    # fp32 GEMMs over a different split of the out_proj reduction
    torch.testing.assert_close(got["y"], ref[:got["y"].shape[0]], rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(got["state"], ref_view, rtol=1e-5, atol=1e-5)
