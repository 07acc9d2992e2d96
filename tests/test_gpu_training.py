"""Training path (greta/dynamic_conv.py fwd/bwd) on the GPU vs the CPU oracle on
the same seeded inputs: ragged packing, every group-size class, W from 1 to
16, norm and gate on/off, bf16/fp16/fp32, misaligned and odd-width inputs,
and the full-size training configuration through per-sequence properties."""
import numpy as np
import pytest
import torch

from gpu_helpers import DEV, assert_close, rand, ragged_cu, to_np
from oracle import oracle

pytestmark = pytest.mark.gpu


def run_case(T_lens, D, W, G, norm, gate_on, dtype, seed=0, cu_dtype=torch.int32, use_cu=True):
    """Forward (saving the pre-norm output) and backward through the drop-in
    layer, compared with the oracle. The oracle backward reads the same saved
    pre-norm output as the kernel, as the reference backward kernel does. The
    autograd path must reproduce the explicit calls bit for bit."""
    from greta_plugin_b200 import dynamic_causal_conv1d
    from greta_plugin_b200.dynamic_conv import dynconv_bwd, dynconv_fwd

    g = torch.Generator().manual_seed(seed)
    T = int(sum(T_lens))
    x = rand(g, 1, T, D, dtype=dtype)
    w = rand(g, T, W, D // G, scale=(1.0 / W) ** 0.5, dtype=dtype)
    gate = rand(g, 1, T, D, dtype=dtype) if gate_on else None
    dout = rand(g, 1, T, D, dtype=dtype)
    cu = ragged_cu(T_lens).to(cu_dtype) if use_cu else None
    xd, wd, dd = x.to(DEV), w.to(DEV), dout.to(DEV)
    gd = gate.to(DEV) if gate_on else None
    cud = cu.to(DEV) if use_cu else None
    y, yr, BT, ci = dynconv_fwd(xd, wd, gd, cud, G, norm=norm, eps=1e-6, save_pre=True)
    dx, dw, dg = dynconv_bwd(xd, wd, gd, yr, dd, cud, G, norm, 1e-6, BT, ci)
    assert y.dtype == dtype and dw.dtype == dtype

    cu_np = cu.numpy() if use_cu else None
    gn = to_np(gate[0]) if gate_on else None
    yo, yro = oracle.fwd(to_np(x[0]), to_np(w), gn, cu_np, G, int(norm), save_pre=True)
    assert_close(y[0], yo, dtype)
    if norm:
        assert_close(yr[0], yro, dtype)
    dxo, dwo, dgo = oracle.bwd(to_np(x[0]), to_np(w), gn, to_np(dout[0]), cu_np, G, int(norm),
                               yr=to_np(yr[0]) if norm else None)
    assert_close(dx[0], dxo, dtype)
    assert_close(dw, dwo, dtype)
    if gate_on:
        assert_close(dg[0], dgo, dtype)

    xa, wa = xd.clone().requires_grad_(), wd.clone().requires_grad_()
    ga = gd.clone().requires_grad_() if gate_on else None
    ya = dynamic_causal_conv1d(xa, wa, ga, cud, G, norm, 1e-6)
    ya.backward(dd)
    assert torch.equal(ya, y)
    assert torch.equal(xa.grad, dx) and torch.equal(wa.grad, dw)
    if gate_on:
        assert torch.equal(ga.grad, dg)


@pytest.mark.parametrize("G", [1, 2, 4, 8, 16, 32, 64, 128])
@pytest.mark.parametrize("norm,gate_on", [(False, False), (True, True), (False, True), (True, False)])
def test_group_sizes_bf16(G, norm, gate_on):
    run_case([1, 2, 3, 50, 7, 130], 256, 4, G, norm, gate_on, torch.bfloat16, seed=G)


@pytest.mark.parametrize("W", [1, 2, 3, 4, 5, 6, 7, 8, 9, 12, 16])
def test_kernel_sizes(W):
    run_case([1, W - 1 if W > 1 else 1, W, 3 * W + 5, 70], 64, W, 4, True, True, torch.bfloat16, seed=100 + W)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("W,G", [(4, 1), (7, 128), (3, 8)])
def test_dtypes(dtype, W, G):
    run_case([5, 64, 200], 256, W, G, True, True, dtype, seed=7)


def test_int64_cu_seqlens_and_single_sequence():
    run_case([40, 90], 128, 4, 1, False, True, torch.bfloat16, cu_dtype=torch.int64)
    run_case([300], 128, 4, 1, True, True, torch.bfloat16, use_cu=False)


def test_odd_width_uses_scalar_path():
    # D % 8 != 0: one channel per thread
    run_case([3, 33, 17], 36, 4, 4, True, True, torch.bfloat16)
    run_case([3, 33, 17], 20, 7, 2, False, True, torch.float32)


def test_misaligned_views_are_handled():
    """Inputs offset by one element (not 16-byte aligned) must still be right."""
    from greta_plugin_b200 import dynamic_causal_conv1d

    g = torch.Generator().manual_seed(3)
    T, D, W, G = 50, 64, 4, 2
    xb = rand(g, 1, T * D + 1, dtype=torch.bfloat16)
    w = rand(g, T, W, D // G, scale=0.5, dtype=torch.bfloat16)
    cu = ragged_cu([20, 30])
    xd = xb.to(DEV)[:, 1:].reshape(1, T, D)  # storage offset of one element
    assert xd.data_ptr() % 16 != 0
    y = dynamic_causal_conv1d(xd, w.to(DEV), None, cu.to(DEV), G, False)
    yo, _ = oracle.fwd(to_np(xb[:, 1:].reshape(T, D)), to_np(w), None, cu.numpy(), G, 0)
    assert_close(y[0], yo, torch.bfloat16)


def test_empty_inputs():
    from greta_plugin_b200 import dynamic_causal_conv1d, dynamic_causal_conv1d_inference

    x = torch.zeros(1, 0, 64, device=DEV, dtype=torch.bfloat16)
    w = torch.zeros(0, 4, 64, device=DEV, dtype=torch.bfloat16)
    assert dynamic_causal_conv1d(x, w, None, torch.tensor([0], device=DEV), 1).shape == (1, 0, 64)
    ctx = torch.zeros(2, 3, 64, device=DEV, dtype=torch.bfloat16)
    wq = torch.zeros(2, 0, 4, 64, device=DEV, dtype=torch.bfloat16)
    assert dynamic_causal_conv1d_inference(ctx, wq).shape == (2, 0, 64)


def test_empty_sequences_inside_cu_seqlens():
    run_case([5, 0, 9, 0, 0, 30], 64, 4, 1, True, True, torch.bfloat16)


def test_sequence_independence_at_training_size():
    """Full-size training configuration: x [1, 8*4096, 4096], w [T, 4, 4096]
    bf16, dy ~ N(0,1). Sequences are independent, so each packed sequence's
    output and gradients equal those of that sequence run alone; two of the
    eight sequences are checked against the oracle."""
    from greta_plugin_b200 import dynamic_causal_conv1d

    g = torch.Generator(device=DEV).manual_seed(0)
    S, L, D, W = 8, 4096, 4096, 4
    T = S * L
    x = torch.randn(1, T, D, device=DEV, generator=g).bfloat16().requires_grad_()
    w = (torch.randn(T, W, D, device=DEV, generator=g) * 0.5).bfloat16().requires_grad_()
    dout = torch.randn(1, T, D, device=DEV, generator=g).bfloat16()
    cu = torch.arange(0, T + 1, L, device=DEV, dtype=torch.int32)
    y = dynamic_causal_conv1d(x, w, None, cu, 1)
    y.backward(dout)
    for s in (0, 5):
        sl = slice(s * L, (s + 1) * L)
        xs, ws, ds = to_np(x[0, sl]), to_np(w[sl]), to_np(dout[0, sl])
        yo, _ = oracle.fwd(xs, ws, None, None, 1, 0)
        dxo, dwo, _ = oracle.bwd(xs, ws, None, ds, None, 1, 0)
        assert_close(y[0, sl], yo, torch.bfloat16)
        assert_close(x.grad[0, sl], dxo, torch.bfloat16)
        assert_close(w.grad[sl], dwo, torch.bfloat16)


def test_bad_shapes_raise_reference_errors():
    from greta_plugin_b200 import dynamic_causal_conv1d

    x = torch.zeros(2, 8, 64, device=DEV)
    w = torch.zeros(8, 4, 64, device=DEV)
    with pytest.raises(ValueError, match="requires physical batch size B=1"):
        dynamic_causal_conv1d(x, w)
    with pytest.raises(ValueError, match="must divide one of BD"):
        dynamic_causal_conv1d(torch.zeros(1, 8, 768, device=DEV), torch.zeros(8, 4, 2, device=DEV),
                              group_size=384)
    with pytest.raises(ValueError, match="weight must be"):
        dynamic_causal_conv1d(x[:1], torch.zeros(7, 4, 64, device=DEV))


def test_config1_fp32_against_reference_checksums():
    """Configuration 1 exactly: fp32, B=2 x T=256 packed with cu_seqlens
    [0, 256, 512], C=512, K=4, x ~ N(0,1), w ~ N(0, 1/K), zero initial state,
    forward only, seed 0. Checked on the GPU against the checksums and sampled
    outputs of the reference's torch path (tests/golden/config1_stats.json,
    made by tests/golden/make_golden.py) and elementwise against the oracle."""
    import json

    from conftest import GOLDEN
    from greta_plugin_b200 import dynamic_causal_conv1d

    s = json.loads((GOLDEN / "config1_stats.json").read_text())
    g = torch.Generator().manual_seed(s["seed"])
    x = torch.randn(*s["shape_x"], generator=g)
    w = torch.randn(*s["shape_w"], generator=g) * s["w_scale"]
    assert abs(float(x.double().sum()) - s["x_sum"]) < 1e-6 * max(1.0, abs(s["x_sum"]))
    cu = torch.tensor(s["cu_seqlens"], dtype=torch.int32)
    y = dynamic_causal_conv1d(x.to(DEV), w.to(DEV), None, cu.to(DEV), 1, False)
    assert y.dtype == torch.float32 and y.shape == x.shape
    yd = y.double().cpu()
    assert abs(float(yd.sum()) - s["y_sum"]) < 1e-3
    assert abs(float(yd.square().sum()) - s["y_sq"]) < 1e-6 * s["y_sq"]
    assert abs(float(yd.abs().sum()) - s["y_abs"]) < 1e-6 * s["y_abs"]
    np.testing.assert_allclose(y.reshape(-1)[s["sample_idx"]].cpu().numpy(), s["sample_val"], rtol=1e-5, atol=1e-6)
    yo, _ = oracle.fwd(x[0].numpy(), w.numpy(), None, np.array(s["cu_seqlens"]), 1, 0)
    assert_close(y[0], yo, torch.float32)
