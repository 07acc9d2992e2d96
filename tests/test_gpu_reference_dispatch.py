"""The B200 kernels behind the reference's OWN dispatch code, on the GPU.

The unmodified reference (baseline/_ref) is driven through its entry points
with the B200 kernels installed by greta_plugin_b200.integration, and compared
with the same reference code on its own paths, on the same device and inputs:

* HF GretaDynamicConv.forward (greta/modeling_greta.py:437-569) at Greta's
  defaults (hidden 2048, kernel 7, 128-channel groups, norm, gate): training
  (autograd, modeling_greta.py:378-414), inference without a cache, and cached
  prefill (update_conv_inputs, :214-248) followed by cached decode steps
  (:467-508), against use_triton_kernels=False (the torch paths, :287-355).
  The cached conv state must stay bit-identical.
* vLLM GretaConv.forward (greta_vllm/model.py:115-163) through the
  vllm::greta_dynamic_conv custom op and metadata_to_batch (conv.py:73-103)
  on a mixed decodes-first batch with CUDA-graph padding tokens, against the
  reference's torch fallback (conv.py:10-70) chosen by its own dispatch.
* The reference's Triton kernels themselves on this GPU
  (greta_vllm/triton_conv.py:128-173, greta/dynamic_conv.py:722-931) against
  the B200 kernels: outputs within the bf16 tolerance, conv state bit-exact.

Skipped when the reference is not installed in baseline/_ref."""
import numpy as np
import pytest
import torch

import reference_harness as rh
from gpu_helpers import DEV, assert_close

pytestmark = pytest.mark.gpu


def rel_err(a, b):
    a, b = a.detach().double(), b.detach().double()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def close(got, ref, dtype):
    assert_close(got, ref, dtype)


# ---------------------------------------------------------------------------
# HF
# ---------------------------------------------------------------------------
def _twin_modules(dtype, **cfg):
    """The same GretaDynamicConv weights twice: the reference's torch paths and
    the kernel paths (use_triton_kernels), the latter dispatching to the B200
    kernels once installed."""
    rdc, mg, cg = rh.reference_modules()
    c_ref, m_ref = rh.make_hf_conv(mg, cg, dtype, DEV, 0, False, **cfg)
    c_k, m_k = rh.make_hf_conv(mg, cg, dtype, DEV, 0, True, **cfg)
    m_k.load_state_dict(m_ref.state_dict())
    return mg, (c_ref, m_ref), (c_k, m_k)


def _train_step(m, h0, dy, install):
    h = h0.clone().requires_grad_()
    with rh.installed(hf=install):
        y = m(h)
        y.backward(dy)
    return [y, h.grad] + [p.grad for _, p in m.named_parameters()]


def test_hf_training_autograd_through_reference_forward_fp32():
    """fp32: the B200 training kernels under the reference's autograd dispatch
    equal its torch path to fp32 rounding (output, input grad, every weight grad)."""
    mg, (c_ref, m_ref), (c_k, m_k) = _twin_modules(torch.float32)
    g = torch.Generator().manual_seed(3)
    h0 = torch.randn(2, 37, c_ref.hidden_dim, generator=g).to(DEV)
    dy = torch.randn(2, 37, c_ref.hidden_dim, generator=g).to(DEV)
    ref = _train_step(m_ref, h0, dy, False)
    got = _train_step(m_k, h0, dy, True)
    close(got[0], ref[0], torch.float32)
    close(got[1], ref[1], torch.float32)
    for a, b in zip(got[2:], ref[2:]):
        assert rel_err(a, b) < 1e-4


def test_hf_training_autograd_through_reference_forward_bf16():
    """bf16: a whole layer (three bf16 GEMMs around the conv) differs between
    any two bf16 pipelines by a few bf16 ulps, so both -- the reference's own
    torch path and the B200 kernels under its dispatch -- are measured against
    the same layer in fp32 (same weights), and the B200 path must be as close
    to it as the reference's path is (relative L2 error within 1.25x + 1e-3)."""
    mg, (c_ref, m_ref), (c_k, m_k) = _twin_modules(torch.bfloat16)
    rdc, mg, cg = rh.reference_modules()
    c32, m32 = rh.make_hf_conv(mg, cg, torch.float32, DEV, 0, False)
    m32.load_state_dict({k: v.float() for k, v in m_ref.state_dict().items()})
    g = torch.Generator().manual_seed(3)
    h0 = torch.randn(2, 37, c_ref.hidden_dim, generator=g).to(DEV, torch.bfloat16)
    dy = torch.randn(2, 37, c_ref.hidden_dim, generator=g).to(DEV, torch.bfloat16)
    exact = _train_step(m32, h0.float(), dy.float(), False)
    ref = _train_step(m_ref, h0, dy, False)
    got = _train_step(m_k, h0, dy, True)
    for i, (a, b, e) in enumerate(zip(got, ref, exact)):
        e_got, e_ref = rel_err(a, e), rel_err(b, e)
        assert e_got <= 1.25 * e_ref + 1e-3, (i, e_got, e_ref)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_hf_training_fused_projection(dtype):
    """install_hf(fused_projection=True): the reference forward's training
    branch with the three projections as one GEMM (the conv reading and its
    backward writing in place) against the same module on the B200 kernels
    with three GEMMs: output, input gradient and every parameter's gradient,
    with an attention mask."""
    mg, (c_ref, m_ref), (c_k, m_k) = _twin_modules(dtype)
    from greta_plugin_b200 import integration

    g = torch.Generator().manual_seed(4)
    h0 = torch.randn(2, 37, c_ref.hidden_dim, generator=g).to(DEV, dtype)
    dy = torch.randn(2, 37, c_ref.hidden_dim, generator=g).to(DEV, dtype)
    mask = torch.ones(2, 37, dtype=torch.bool, device=DEV)
    mask[1, 30:] = False

    def step(m, fused):
        h = h0.clone().requires_grad_()
        saved = mg.GretaDynamicConv.forward
        try:
            with rh.installed(hf=True):
                if fused:
                    integration.install_hf(fused_projection=True)
                    assert getattr(mg.GretaDynamicConv.forward, "__greta_b200_fused__", False)
                y = m(h, attention_mask=mask)
                y.backward(dy)
        finally:
            mg.GretaDynamicConv.forward = saved
        return [y, h.grad] + [p.grad for _, p in m.named_parameters()]

    rdc, mg, cg = rh.reference_modules()
    c2, m2 = rh.make_hf_conv(mg, cg, dtype, DEV, 0, True)  # a second kernel-path module, same weights
    m2.load_state_dict(m_ref.state_dict())
    three = step(m_k, False)
    fused = step(m2, True)
    bound = 1e-4 if dtype == torch.float32 else 1e-2  # summation order of one GEMM vs three
    for i, (a, b) in enumerate(zip(fused, three)):
        assert rel_err(a, b) < bound, (i, rel_err(a, b))


def test_hf_inference_without_cache_with_mask():
    mg, (c_ref, m_ref), (c_k, m_k) = _twin_modules(torch.bfloat16)
    g = torch.Generator().manual_seed(4)
    h = torch.randn(3, 29, c_ref.hidden_dim, generator=g).to(DEV, torch.bfloat16)
    mask = torch.ones(3, 29, dtype=torch.bool)
    mask[1, :5] = False  # left padding of row 1
    mask = mask.to(DEV)
    with torch.no_grad():
        y_r = m_ref(h, attention_mask=mask)
        with rh.installed(hf=True):
            y_k = m_k(h, attention_mask=mask)
    close(y_k, y_r, torch.bfloat16)


def test_hf_cached_prefill_then_decode_steps():
    """Prefill 16 tokens into the cache, then 4 one-token decode steps that
    shift the cached state in place (the B200 decode kernel under the
    reference's get_conv_state_for_decode). States stay bit-identical."""
    mg, (c_ref, m_ref), (c_k, m_k) = _twin_modules(torch.bfloat16)
    li = rh.conv_layer_index(c_ref)
    cache_r, cache_k = rh.make_cache(mg, c_ref), rh.make_cache(mg, c_k)
    g = torch.Generator().manual_seed(5)
    h = torch.randn(3, 20, c_ref.hidden_dim, generator=g).to(DEV, torch.bfloat16)
    with torch.no_grad():
        spans = [(0, 16)] + [(t, t + 1) for t in range(16, 20)]
        for a, b in spans:
            y_r = m_ref(h[:, a:b], past_key_values=cache_r, use_cache=True)
            with rh.installed(hf=True):
                y_k = m_k(h[:, a:b], past_key_values=cache_k, use_cache=True)
            close(y_k, y_r, torch.bfloat16)
            s_r = cache_r.layers[li].conv_states[0]
            s_k = cache_k.layers[li].conv_states[0]
            assert torch.equal(s_k, s_r), f"conv state differs after tokens [{a}, {b})"


def test_hf_chunked_prefill_with_cache_is_one_launch_on_the_cache_state():
    """A prefill in two chunks (16 + 24 tokens) then decode steps, through the
    reference's GretaDynamicConv.forward and cache: the second chunk continues
    a cached sequence, which the installed forward runs as one launch on the
    cache's channel-first state (no context tensor). Against the reference's
    torch path and its own Triton kernels: outputs within tolerance, the cache
    state bit-identical after every call."""
    rdc, mg, cg = rh.reference_modules()
    c_ref, m_ref = rh.make_hf_conv(mg, cg, torch.bfloat16, DEV, 0, False)
    c_tri, m_tri = rh.make_hf_conv(mg, cg, torch.bfloat16, DEV, 0, True)
    c_k, m_k = rh.make_hf_conv(mg, cg, torch.bfloat16, DEV, 0, True)
    m_tri.load_state_dict(m_ref.state_dict())
    m_k.load_state_dict(m_ref.state_dict())
    li = rh.conv_layer_index(c_ref)
    caches = [rh.make_cache(mg, c) for c in (c_ref, c_tri, c_k)]
    g = torch.Generator().manual_seed(15)
    h = torch.randn(3, 43, c_ref.hidden_dim, generator=g).to(DEV, torch.bfloat16)
    spans = [(0, 16), (16, 40), (40, 41), (41, 42), (42, 43)]
    from greta_plugin_b200 import dynamic_conv as bdc

    calls = []
    orig = bdc.dynamic_causal_conv1d_prefill_with_state

    def counting(*a, **k):
        calls.append(1)
        return orig(*a, **k)

    bdc.dynamic_causal_conv1d_prefill_with_state = counting
    try:
        with torch.no_grad():
            for a, b in spans:
                y_r = m_ref(h[:, a:b], past_key_values=caches[0], use_cache=True)
                y_t = m_tri(h[:, a:b], past_key_values=caches[1], use_cache=True)
                with rh.installed(hf=True):
                    y_k = m_k(h[:, a:b], past_key_values=caches[2], use_cache=True)
                close(y_k, y_r, torch.bfloat16)
                close(y_k, y_t, torch.bfloat16)
                s_r, s_t, s_k = (c.layers[li].conv_states[0] for c in caches)
                assert torch.equal(s_k, s_r) and torch.equal(s_k, s_t), f"state differs after [{a}, {b})"
    finally:
        bdc.dynamic_causal_conv1d_prefill_with_state = orig
    assert len(calls) == 1  # the second prefill chunk


@pytest.mark.parametrize("has_previous", [True, False])
@pytest.mark.parametrize("Q", [1, 2, 9])
def test_prefill_with_state_against_reference_cache_and_kernel(has_previous, Q):
    """dynamic_causal_conv1d_prefill_with_state against the reference's two
    steps: the cache's update_conv_inputs (context and new state) and its
    Triton inference kernel on that context; chunks shorter than W-1 included."""
    rdc, mg, cg = rh.reference_modules()
    from greta_plugin_b200 import dynamic_causal_conv1d_prefill_with_state

    cfg = rh.greta_config(cg)
    li = rh.conv_layer_index(cfg)
    B, D, W, G = 3, cfg.hidden_dim, cfg.kernel_size, cfg.conv_group_size
    g = torch.Generator().manual_seed(16 + Q)
    x = torch.randn(B, Q, D, generator=g).bfloat16().to(DEV)
    wq = (torch.randn(B, Q, W, D // G, generator=g) * (1.0 / W) ** 0.5).bfloat16().to(DEV)
    gq = torch.randn(B, Q, D, generator=g).bfloat16().to(DEV)
    cache = rh.make_cache(mg, cfg)
    if has_previous:  # a cached sequence: the state of an earlier chunk
        cache.update_conv_inputs(torch.randn(B, 8, D, generator=g).bfloat16().to(DEV), li, W)
    state = cache.layers[li].conv_states[0].clone() if has_previous else torch.zeros(B, D, W - 1, dtype=x.dtype,
                                                                                    device=DEV)
    ctx = cache.update_conv_inputs(x, li, W)
    y_ref = rdc.dynamic_causal_conv1d_inference(ctx, wq, gq, G, True, 1e-6)
    y = dynamic_causal_conv1d_prefill_with_state(x, wq, state, has_previous, gq, G, True, 1e-6)
    close(y, y_ref, torch.bfloat16)
    if Q >= W - 1 or has_previous:
        assert torch.equal(state, cache.layers[li].conv_states[0]), "the new conv state must be bit-exact"


# ---------------------------------------------------------------------------
# vLLM
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("num_k_heads", [128, 512])  # 512: groups wider than a warp's 256 channels
def test_vllm_layer_forward_through_custom_op(num_k_heads):
    """GretaConv.forward -> vllm::greta_dynamic_conv -> run_conv ->
    metadata_to_batch -> packed_dynamic_conv_triton (the B200 kernel once
    installed), on 3 decodes (one a new prompt at position 0) then 2 prefill
    chunks (one with history), followed by 3 CUDA-graph padding tokens; against
    the reference's torch fallback chosen by run_conv itself."""
    rdc, mg, cg = rh.reference_modules()
    vconv, vtc, vm = rh.vllm_reference_modules()
    cfg, layer, prefix = rh.make_vllm_conv(vm, cg, torch.bfloat16, DEV, 7, 16, num_k_heads=num_k_heads)
    D = cfg.hidden_dim
    md = rh.short_conv_metadata(vm, [3, 9, 1], [5, 40], [0, 12], [True, False], DEV)
    pos = torch.tensor([11, 0, 30] + list(range(7, 12)) + list(range(40)) + [0, 0, 0], device=DEV)
    n_tok = pos.numel()
    g = torch.Generator().manual_seed(8)
    hs = torch.randn(n_tok, D, generator=g).to(DEV, torch.bfloat16)
    state0 = layer.kv_cache[0].clone()
    with torch.no_grad(), rh.forward_context(vm, layer, prefix, md):
        with rh.installed(vllm=True):
            assert vm.triton_supports(cfg.conv_group_size, D)
            y_k = layer(hs, pos)
        s_k = layer.kv_cache[0].clone()
        layer.kv_cache[0].copy_(state0)
        saved = vm.triton_supports
        vm.triton_supports = lambda *a: False  # the reference's own fallback branch
        try:
            y_r = layer(hs, pos)
        finally:
            vm.triton_supports = saved
        s_r = layer.kv_cache[0].clone()
    close(y_k, y_r, torch.bfloat16)
    assert torch.equal(s_k, s_r), "conv state must be bit-exact"
    named = {3, 9, 1, 0, 12}
    for s in range(state0.shape[0]):
        if s not in named:
            assert torch.equal(s_k[s], state0[s])


def test_vllm_layer_fused_projection_through_custom_op():
    """install_vllm(fused_projection=True): GretaConv.forward computes its
    three projections as one GEMM and hands column views of its output to the
    reference's custom op, which passes them (strided, not copied) to the
    B200 kernel; against the same layer with three GEMMs on the B200 kernel.
    Outputs within bf16 tolerance, the cache within one GEMM rounding, the
    slots no request names untouched."""
    rdc, mg, cg = rh.reference_modules()
    vconv, vtc, vm = rh.vllm_reference_modules()
    from greta_plugin_b200 import integration

    cfg, layer, prefix = rh.make_vllm_conv(vm, cg, torch.bfloat16, DEV, 7, 16)
    D = cfg.hidden_dim
    md = rh.short_conv_metadata(vm, [3, 9, 1], [5, 40], [0, 12], [True, False], DEV)
    pos = torch.tensor([11, 0, 30] + list(range(7, 12)) + list(range(40)) + [0, 0, 0], device=DEV)
    g = torch.Generator().manual_seed(9)
    hs = torch.randn(pos.numel(), D, generator=g).to(DEV, torch.bfloat16)
    state0 = layer.kv_cache[0].clone()
    seen = []
    saved_fwd = vm.GretaConv.forward
    with torch.no_grad(), rh.forward_context(vm, layer, prefix, md):
        with rh.installed(vllm=True):
            y_3 = layer(hs, pos)
            s_3 = layer.kv_cache[0].clone()
            layer.kv_cache[0].copy_(state0)
            kernel = vm.packed_dynamic_conv_triton

            def spy(x, weights, gate, *a, **k):
                seen.append((x.is_contiguous(), weights.is_contiguous(), gate.is_contiguous()))
                return kernel(x, weights, gate, *a, **k)

            vm.packed_dynamic_conv_triton = spy
            try:
                integration.install_vllm(fused_projection=True)
                vm.packed_dynamic_conv_triton = spy
                y_f = layer(hs, pos)
            finally:
                vm.GretaConv.forward = saved_fwd
        s_f = layer.kv_cache[0].clone()
    assert seen == [(False, False, False)], seen  # column views of one GEMM output reached the kernel
    close(y_f, y_3, torch.bfloat16)
    torch.testing.assert_close(s_f.float(), s_3.float(), rtol=1e-2, atol=1e-2)
    named = {3, 9, 1, 0, 12}
    for s in range(state0.shape[0]):
        if s not in named:
            assert torch.equal(s_f[s], state0[s])


def _packed_case(D, W, G, lengths, slots, n_slots, norm, gate_on, seed, layout):
    g = torch.Generator().manual_seed(seed)
    T = sum(lengths)
    x = torch.randn(T, D, generator=g).bfloat16()
    w = (torch.randn(T, W, D // G, generator=g) * (1.0 / W) ** 0.5).bfloat16()
    gate = torch.randn(T, D, generator=g).bfloat16() if gate_on else None
    logical = torch.randn(n_slots, D, W - 1, generator=g).bfloat16()
    if layout == "SD":
        store = logical.transpose(1, 2).contiguous().to(DEV)
        view = lambda s: s.transpose(1, 2)  # noqa: E731
    else:
        store = logical.to(DEV)
        view = lambda s: s  # noqa: E731
    starts = torch.tensor([0] + list(np.cumsum(lengths)), dtype=torch.int32, device=DEV)
    slots_t = torch.tensor(slots, dtype=torch.int32, device=DEV)
    init = torch.tensor([1 if i % 3 else 0 for i in range(len(lengths))], dtype=torch.int8, device=DEV)
    return dict(x=x.to(DEV), w=w.to(DEV), gate=None if gate is None else gate.to(DEV), store=store, view=view,
                starts=starts, slots=slots_t, init=init, G=G, norm=norm)


@pytest.mark.parametrize("case", [
    dict(D=4096, W=4, G=1, lengths=[179, 87, 54, 114, 71, 90, 148, 155], slots=[5, 17, 2, 40, 63, 0, 9, 33],
         n_slots=64, norm=False, gate_on=False),  # the headline prefill's shape
    dict(D=4096, W=4, G=1, lengths=[1] * 64, slots=[(7 * i) % 97 if i % 10 else -1 for i in range(64)],
         n_slots=97, norm=False, gate_on=False),  # decode, padding slots
    dict(D=2048, W=7, G=128, lengths=[1, 1, 1, 2, 6, 9, 40, 131], slots=[3, -1, 7, 0, 11, 5, 2, 9], n_slots=12,
         norm=True, gate_on=True),  # Greta's layer shape, mixed
    dict(D=4096, W=7, G=1024, lengths=[1, 1, 2, 6, 33], slots=[3, -1, 0, 11, 5], n_slots=12, norm=True,
         gate_on=True),  # a group wider than 256 channels
])
@pytest.mark.parametrize("layout", ["DS", "SD"])
def test_vllm_packed_against_reference_triton_kernels(case, layout):
    vconv, vtc, vm = rh.vllm_reference_modules()
    from greta_plugin_b200 import packed_dynamic_conv_triton as b200_packed

    ref_packed = vtc.packed_dynamic_conv_triton  # the reference's Triton launcher (not installed over)
    assert ref_packed is not b200_packed
    b = _packed_case(seed=11, layout=layout, **case)
    s_r, s_k = b["store"].clone(), b["store"].clone()
    y_r = ref_packed(b["x"], b["w"], b["gate"], b["view"](s_r), b["starts"], b["slots"], b["init"], b["G"],
                     norm=b["norm"])
    y_k = b200_packed(b["x"], b["w"], b["gate"], b["view"](s_k), b["starts"], b["slots"], b["init"], b["G"],
                      norm=b["norm"])
    torch.cuda.synchronize()
    close(y_k, y_r, torch.bfloat16)
    assert torch.equal(s_k, s_r), "conv state must be bit-exact against the reference kernel"


# ---------------------------------------------------------------------------
# training and HF kernels against the reference's Triton kernels
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("D,W,G,norm,gate_on,lens", [
    (2048, 7, 128, True, True, [300, 212]),  # Greta's layer shape
    (4096, 4, 1, False, False, [256, 256]),  # the training headline's shape (shorter)
])
def test_training_against_reference_triton_kernels(D, W, G, norm, gate_on, lens):
    rdc, mg, cg = rh.reference_modules()
    from greta_plugin_b200 import dynamic_causal_conv1d as b200_conv

    ref_conv = rdc.dynamic_causal_conv1d
    assert ref_conv is not b200_conv
    T = sum(lens)
    g = torch.Generator().manual_seed(12)
    x = torch.randn(1, T, D, generator=g).bfloat16().to(DEV)
    w = (torch.randn(T, W, D // G, generator=g) * (1.0 / W) ** 0.5).bfloat16().to(DEV)
    gate = torch.randn(1, T, D, generator=g).bfloat16().to(DEV) if gate_on else None
    dy = torch.randn(1, T, D, generator=g).bfloat16().to(DEV)
    cu = torch.tensor([0] + list(np.cumsum(lens)), dtype=torch.int32, device=DEV)
    res = []
    for fn in (ref_conv, b200_conv):
        xs, ws = x.clone().requires_grad_(), w.clone().requires_grad_()
        gs = gate.clone().requires_grad_() if gate_on else None
        y = fn(xs, ws, gs, cu, G, norm, 1e-6)
        y.backward(dy)
        res.append((y, xs.grad, ws.grad, gs.grad if gate_on else None))
    (y_r, dx_r, dw_r, dg_r), (y_k, dx_k, dw_k, dg_k) = res
    close(y_k, y_r, torch.bfloat16)
    close(dx_k, dx_r, torch.bfloat16)
    close(dw_k, dw_r, torch.bfloat16)
    if gate_on:
        close(dg_k, dg_r, torch.bfloat16)


def test_hf_decode_and_inference_against_reference_triton_kernels():
    rdc, mg, cg = rh.reference_modules()
    from greta_plugin_b200 import dynamic_causal_conv1d_decode as b200_decode
    from greta_plugin_b200 import dynamic_causal_conv1d_inference as b200_inf

    D, W, G, B, Q = 2048, 7, 128, 6, 33
    g = torch.Generator().manual_seed(13)
    x = torch.randn(B, D, generator=g).bfloat16().to(DEV)
    w = (torch.randn(B, W, D // G, generator=g) * (1.0 / W) ** 0.5).bfloat16().to(DEV)
    gate = torch.randn(B, D, generator=g).bfloat16().to(DEV)
    st0 = torch.randn(B, D, W - 1, generator=g).bfloat16().to(DEV)
    s_r, s_k = st0.clone(), st0.clone()
    y_r = rdc.dynamic_causal_conv1d_decode(x, w, s_r, gate, G, True, 1e-6)
    y_k = b200_decode(x, w, s_k, gate, G, True, 1e-6)
    close(y_k, y_r, torch.bfloat16)
    assert torch.equal(s_k, s_r), "decode state shift must be bit-exact"
    ctx = torch.randn(B, Q + W - 1, D, generator=g).bfloat16().to(DEV)
    wq = (torch.randn(B, Q, W, D // G, generator=g) * (1.0 / W) ** 0.5).bfloat16().to(DEV)
    gq = torch.randn(B, Q, D, generator=g).bfloat16().to(DEV)
    close(b200_inf(ctx, wq, gq, G, True, 1e-6), rdc.dynamic_causal_conv1d_inference(ctx, wq, gq, G, True, 1e-6),
          torch.bfloat16)
