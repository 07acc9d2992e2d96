"""CPU checks of the harness that runs the reference's own dispatch code
(tests/reference_harness.py), so that the GPU tests built on it compare like
with like:

* the transformers-5.17 cache stand-in: prefill with the cache, then one-token
  decodes, equals the cache-free forward of the same tokens in the
  reference's GretaDynamicConv (greta/modeling_greta.py:437-569);
* install / restore of the B200 kernel names in the real reference modules
  (greta/modeling_greta.py:25-34, greta_vllm/model.py:160-161);
* greta_vllm.conv.metadata_to_batch (greta_vllm/conv.py:73-103) on the
  metadata the harness builds (decodes first, initial = positions > 0);
* GretaConv.forward through the vLLM custom op (greta_vllm/model.py:115-182)
  on CPU equals the reference's packed_dynamic_conv called directly.

Skipped when the reference is not installed in baseline/_ref."""
import pytest
import torch

import reference_harness as rh


def test_cache_stand_in_matches_cache_free_forward():
    rdc, mg, cg = rh.reference_modules()
    cfg, mod = rh.make_hf_conv(mg, cg, torch.float32, "cpu", 0, False, hidden_dim=256)
    cache = rh.make_cache(mg, cfg)
    g = torch.Generator().manual_seed(1)
    h = torch.randn(2, 12, 256, generator=g)
    li = rh.conv_layer_index(cfg)
    with torch.no_grad():
        full = mod(h)
        outs = [mod(h[:, :9], past_key_values=cache, use_cache=True)]
        assert cache.get_conv_state_for_decode(li) is not None
        for t in range(9, 12):
            outs.append(mod(h[:, t:t + 1], past_key_values=cache, use_cache=True))
    torch.testing.assert_close(torch.cat(outs, 1), full, rtol=1e-5, atol=1e-5)
    # the cached state is the last W-1 projected inputs, channel first (the
    # projection of a token slice may round differently from the whole batch's)
    with torch.no_grad():
        last = mod.in_proj(h[:, -(cfg.kernel_size - 1):]).transpose(1, 2)
    torch.testing.assert_close(cache.layers[li].conv_states[0], last, rtol=1e-5, atol=1e-5)


def test_install_rebinds_and_restores_reference_names():
    rdc, mg, cg = rh.reference_modules()
    vconv, vtc, vm = rh.vllm_reference_modules()
    from greta_plugin_b200 import dynamic_conv as bdc
    from greta_plugin_b200 import vllm_conv as bvc

    before = (mg._TRITON_DYNAMIC_CAUSAL_CONV1D_DECODE, vm.packed_dynamic_conv_triton, vm.triton_supports,
              rdc.dynconv_fwd, mg.GretaDynamicConv.forward)
    with rh.installed(hf=True, vllm=True):
        assert getattr(mg.GretaDynamicConv.forward, "__greta_b200__", False)
        assert mg._TRITON_DYNAMIC_CAUSAL_CONV1D is bdc.dynamic_causal_conv1d
        assert mg._TRITON_DYNAMIC_CAUSAL_CONV1D_DECODE is bdc.dynamic_causal_conv1d_decode
        assert mg._TRITON_DYNAMIC_CAUSAL_CONV1D_INFERENCE is bdc.dynamic_causal_conv1d_inference
        assert mg.triton_dynamic_causal_conv1d_autograd_from_context is \
            bdc.triton_dynamic_causal_conv1d_autograd_from_context
        assert vm.packed_dynamic_conv_triton is bvc.packed_dynamic_conv_triton
        assert vm.triton_supports is bvc.supports
        assert vtc.packed_dynamic_conv_triton is bvc.packed_dynamic_conv_triton
        assert rdc.dynconv_fwd is bdc.dynconv_fwd
    after = (mg._TRITON_DYNAMIC_CAUSAL_CONV1D_DECODE, vm.packed_dynamic_conv_triton, vm.triton_supports,
             rdc.dynconv_fwd, mg.GretaDynamicConv.forward)
    assert all(a is b for a, b in zip(before, after))


def test_metadata_to_batch_on_harness_metadata():
    vconv, vtc, vm = rh.vllm_reference_modules()
    md = rh.short_conv_metadata(vm, [3, 5, 1], [4, 6], [0, 7], [True, False], "cpu")
    pos = torch.tensor([5, 0, 9] + list(range(2, 6)) + list(range(6)))
    starts, seq_idx, slots, initial, n = vconv.metadata_to_batch(md, pos)
    assert starts.tolist() == [0, 1, 2, 3, 7, 13]
    assert seq_idx is None
    assert slots.tolist() == [3, 5, 1, 0, 7]
    assert initial.tolist() == [1, 0, 1, 1, 0]
    assert n == 13


def test_vllm_layer_forward_on_cpu_is_the_torch_path():
    rdc, mg, cg = rh.reference_modules()
    vconv, vtc, vm = rh.vllm_reference_modules()
    cfg, layer, prefix = rh.make_vllm_conv(vm, cg, torch.float32, "cpu", 1, 8, hidden_dim=256)
    md = rh.short_conv_metadata(vm, [3, 5], [4, 6], [0, 7], [True, False], "cpu")
    pos = torch.tensor([5, 0] + list(range(2, 6)) + list(range(6)))
    g = torch.Generator().manual_seed(2)
    hs = torch.randn(12, 256, generator=g)
    state0 = layer.kv_cache[0].clone()
    with torch.no_grad(), rh.forward_context(vm, layer, prefix, md):
        y = layer(hs, pos)
    # the same call by hand
    with torch.no_grad():
        x, gate = layer.in_proj(hs), layer.gate_proj(hs)
        w = layer.kernel_proj(hs).view(12, cfg.kernel_size, cfg.num_conv_filters)
        state = state0.clone()
        view = state if vm.is_conv_state_dim_first() else state.transpose(-1, -2)
        starts, _, slots, initial, n = vconv.metadata_to_batch(md, pos)
        mixed = vconv.packed_dynamic_conv(x, w, gate, view, starts, slots, initial, cfg.conv_group_size,
                                          cfg.dynconv_norm, cfg.dynconv_norm_eps)
        ref = layer.out_proj(mixed)
    torch.testing.assert_close(y, ref, rtol=0, atol=0)
    assert torch.equal(layer.kv_cache[0], state)


def test_vllm_fused_projection_forward_on_cpu():
    """install_vllm(fused_projection=True) replaces GretaConv.forward's three
    projections by one GEMM whose column views go to the reference's custom op
    (on CPU: its torch packed_dynamic_conv); output and cache equal the
    reference forward's (fp32, the GEMMs' summation order aside)."""
    rdc, mg, cg = rh.reference_modules()
    vconv, vtc, vm = rh.vllm_reference_modules()
    from greta_plugin_b200 import integration

    cfg, layer, prefix = rh.make_vllm_conv(vm, cg, torch.float32, "cpu", 1, 8, hidden_dim=256)
    md = rh.short_conv_metadata(vm, [3, 5], [4, 6], [0, 7], [True, False], "cpu")
    pos = torch.tensor([5, 0] + list(range(2, 6)) + list(range(6)))
    hs = torch.randn(12, 256, generator=torch.Generator().manual_seed(2))
    state0 = layer.kv_cache[0].clone()
    with torch.no_grad(), rh.forward_context(vm, layer, prefix, md):
        y_ref = layer(hs, pos)
        s_ref = layer.kv_cache[0].clone()
        layer.kv_cache[0].copy_(state0)
        saved = vm.GretaConv.forward
        try:
            with rh.installed(vllm=True):
                integration.install_vllm(fused_projection=True)
                assert getattr(vm.GretaConv.forward, "__greta_b200__", False)
                y_f = layer(hs, pos)
        finally:
            vm.GretaConv.forward = saved
    torch.testing.assert_close(y_f, y_ref, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(layer.kv_cache[0], s_ref, rtol=1e-5, atol=1e-5)


def test_harness_skips_cleanly_without_reference(monkeypatch, tmp_path):
    import conftest

    monkeypatch.setattr(conftest, "REFERENCE_DIR", tmp_path)
    assert not conftest.reference_available()
    with pytest.raises(pytest.skip.Exception):
        conftest.import_reference_path()


def test_wrapped_forward_falls_back_to_the_reference_on_cpu():
    """Off the GPU (and without a live cache state) the wrapped forward is the
    reference's own: same output as the unwrapped module, cache state included."""
    rdc, mg, cg = rh.reference_modules()
    cfg, mod = rh.make_hf_conv(mg, cg, torch.float32, "cpu", 0, False, hidden_dim=256)
    g = torch.Generator().manual_seed(7)
    h = torch.randn(2, 10, 256, generator=g)
    c1, c2 = rh.make_cache(mg, cfg), rh.make_cache(mg, cfg)
    with torch.no_grad():
        ref = [mod(h[:, :6], past_key_values=c1, use_cache=True), mod(h[:, 6:], past_key_values=c1, use_cache=True)]
        with rh.installed(hf=True):
            got = [mod(h[:, :6], past_key_values=c2, use_cache=True),
                   mod(h[:, 6:], past_key_values=c2, use_cache=True)]
    for a, b in zip(got, ref):
        torch.testing.assert_close(a, b, rtol=0, atol=0)
    li = rh.conv_layer_index(cfg)
    assert torch.equal(c1.layers[li].conv_states[0], c2.layers[li].conv_states[0])
