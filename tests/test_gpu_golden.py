"""The CUDA kernels, called through the drop-in Python layer and the C ABI, on
the golden vectors that the REFERENCE produced (tests/golden/make_golden.py).
fp32 cases are compared with the reference's fp32 outputs; bf16 cases with the
reference kernels' bf16 outputs; conv state must be bit-exact."""
import numpy as np
import pytest
import torch

from conftest import bf16_bits_to_f32, load_golden
from gpu_helpers import DEV, bf16_bits, f32_to_bf16_bits
from oracle import oracle

pytestmark = pytest.mark.gpu

TRAIN_CASES = ["train_g1_w4_plain", "train_g4_w4_norm_gate", "train_g16_w7_norm_gate",
               "train_g128_w7_norm_gate", "train_g2_w3_gate"]
PACKED_CASES = ["packed_stable_gate_mixed", "packed_all_valid_torchcheck", "packed_sd_layout_w7_g16",
                "packed_nonorm_nogate_g1"]


def t(a, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV, dtype)


def close32(got, ref, rtol=1e-4, atol=5e-5):
    r = np.asarray(ref, np.float32)
    np.testing.assert_allclose(got.detach().float().cpu().numpy(), r, rtol=rtol,
                               atol=atol * max(1.0, float(np.abs(r).max())))


@pytest.mark.parametrize("name", TRAIN_CASES)
def test_training_autograd_matches_reference(name):
    from greta_plugin_b200 import dynamic_causal_conv1d

    z = load_golden(name)
    G, norm, eps = int(z["G"]), bool(z["norm"]), float(z["eps"])
    x = t(z["x"])[None].requires_grad_()
    w = t(z["w"]).requires_grad_()
    gate = t(z["gate"])[None].requires_grad_() if "gate" in z else None
    cu = torch.from_numpy(z["cu_seqlens"]).to(DEV, torch.int32)
    y = dynamic_causal_conv1d(x, w, gate, cu, G, norm, eps)
    y.backward(t(z["dout"])[None])
    close32(y[0], z["y_torch"])
    close32(y[0], z["y_triton"])
    close32(x.grad[0], z["dx_triton"])
    close32(w.grad, z["dw_triton"])
    close32(x.grad[0], z["dx_torch"])
    close32(w.grad, z["dw_torch"])
    if gate is not None:
        close32(gate.grad[0], z["dg_triton"])
        close32(gate.grad[0], z["dg_torch"])


@pytest.mark.parametrize("name", TRAIN_CASES)
def test_training_fwd_saves_prenorm(name):
    from greta_plugin_b200.dynamic_conv import dynconv_fwd

    z = load_golden(name)
    if not int(z["norm"]):
        pytest.skip("no pre-norm output without norm")
    gate = t(z["gate"])[None] if "gate" in z else None
    y, yr, _, _ = dynconv_fwd(t(z["x"])[None], t(z["w"]), gate, torch.from_numpy(z["cu_seqlens"]).to(DEV),
                              int(z["G"]), norm=True, eps=float(z["eps"]), save_pre=True)
    close32(yr[0], z["yr_triton"])


def test_training_fwd_bf16_matches_reference_kernel():
    from greta_plugin_b200 import dynamic_causal_conv1d

    z = load_golden("train_bf16_g8_w4_norm_gate")
    x, w, g = (torch.from_numpy(bf16_bits_to_f32(z[k])).to(DEV, torch.bfloat16)
               for k in ("x_bits", "w_bits", "gate_bits"))
    cu = torch.from_numpy(z["cu_seqlens"]).to(DEV)
    y = dynamic_causal_conv1d(x[None], w, g[None], cu, int(z["G"]), True, float(z["eps"]))
    got = bf16_bits(y[0])
    ref = z["y_bits"]
    # the interpreted reference truncates; ours rounds to nearest even: <= 1 ulp
    np.testing.assert_allclose(bf16_bits_to_f32(got), bf16_bits_to_f32(ref), rtol=2 ** -7, atol=1e-6)
    # against the oracle rounded the same way (RTNE) it is bit-exact up to fp32 ties
    yo, _ = oracle.fwd(x.float().cpu().numpy(), w.float().cpu().numpy(), g.float().cpu().numpy(),
                       z["cu_seqlens"], int(z["G"]), 1, float(z["eps"]))
    assert np.mean(f32_to_bf16_bits(yo) == got) > 0.99


def test_inference_matches_reference():
    from greta_plugin_b200 import dynamic_causal_conv1d_inference

    z = load_golden("inference_g8_w4_norm_gate")
    y = dynamic_causal_conv1d_inference(t(z["context"]), t(z["w"]), t(z["gate"]), int(z["G"]), True,
                                        float(z["eps"]))
    close32(y, z["y_triton"])
    close32(y, z["y_torch"])


@pytest.mark.parametrize("name", ["decode_rows_g4_w4_norm_gate", "decode_rows_g1_w2_gate"])
def test_decode_rows_matches_reference(name):
    from greta_plugin_b200 import dynamic_causal_conv1d_decode

    z = load_golden(name)
    state = t(z["state"])
    y = dynamic_causal_conv1d_decode(t(z["x"]), t(z["w"]), state, t(z["gate"]), int(z["G"]), bool(z["norm"]),
                                     float(z["eps"]))
    close32(y, z["y_triton"])
    assert np.array_equal(state.cpu().numpy(), z["state_triton"]), "conv state must be bit-exact"


@pytest.mark.parametrize("name", PACKED_CASES)
def test_packed_matches_reference(name):
    from greta_plugin_b200 import packed_dynamic_conv_triton

    z = load_golden(name)
    D, W = int(z["D"]), int(z["W"])
    if int(z["sd_layout"]):
        storage = t(z["state"].transpose(0, 2, 1))  # [slots, W-1, D]
        state = storage.transpose(1, 2)
    else:
        state = t(z["state"])
    gate = t(z["gate"]) if "gate" in z else None
    y = packed_dynamic_conv_triton(t(z["x"]), t(z["w"]), gate, state, torch.from_numpy(z["starts"]),
                                   torch.from_numpy(z["slots"]), torch.from_numpy(z["has_initial"]), int(z["G"]),
                                   norm=bool(z["norm"]), eps=float(z["eps"]))
    close32(y, z["y_triton"])
    assert np.array_equal(state.cpu().numpy(), z["state_triton"]), "conv state must be bit-exact"


def test_packed_bf16_matches_reference_kernel():
    from greta_plugin_b200 import packed_dynamic_conv_triton

    z = load_golden("packed_bf16_stable_gate")
    x, w, g, s = (torch.from_numpy(bf16_bits_to_f32(z[k])).to(DEV, torch.bfloat16)
                  for k in ("x_bits", "w_bits", "gate_bits", "state_bits"))
    y = packed_dynamic_conv_triton(x, w, g, s, torch.from_numpy(z["starts"]), torch.from_numpy(z["slots"]),
                                   torch.from_numpy(z["has_initial"]), int(z["G"]), norm=True, eps=float(z["eps"]))
    np.testing.assert_allclose(bf16_bits_to_f32(bf16_bits(y)), bf16_bits_to_f32(z["y_bits"]), rtol=2 ** -7,
                               atol=1e-6)
    assert np.array_equal(bf16_bits(s), z["state_out_bits"]), "conv state must be bit-exact"
