"""Pin the CPU oracle to the reference: every oracle function is checked
against golden vectors that the reference's own code produced
(tests/golden/make_golden.py: its torch paths and its Triton kernels run by
the Triton CPU interpreter). CPU only."""
import json

import numpy as np
import pytest

from conftest import GOLDEN, bf16_bits_to_f32, f32_to_bf16_bits, load_golden
from oracle import oracle

TRAIN_CASES = ["train_g1_w4_plain", "train_g4_w4_norm_gate", "train_g16_w7_norm_gate",
               "train_g128_w7_norm_gate", "train_g2_w3_gate"]
PACKED_CASES = ["packed_stable_gate_mixed", "packed_all_valid_torchcheck", "packed_sd_layout_w7_g16",
                "packed_nonorm_nogate_g1"]

# fp32 reference paths vs a double-precision oracle. Group sums over G = 128
# channels carry fp32 cancellation error in the reference itself, so the
# absolute tolerance scales with the array's magnitude.
TOL = dict(rtol=1e-4, atol=2e-5)


def close(got, ref, rtol=1e-4, atol=5e-5):
    np.testing.assert_allclose(got, ref, rtol=rtol, atol=atol * max(1.0, float(np.abs(ref).max())))


@pytest.mark.parametrize("name", TRAIN_CASES)
def test_train_fwd_bwd_matches_reference(name):
    z = load_golden(name)
    G, norm, eps = int(z["G"]), int(z["norm"]), float(z["eps"])
    gate = z.get("gate")
    y, yr = oracle.fwd(z["x"], z["w"], gate, z["cu_seqlens"], G, norm, eps, save_pre=True)
    np.testing.assert_allclose(y, z["y_torch"], **TOL)
    np.testing.assert_allclose(y, z["y_triton"], **TOL)
    if norm:
        np.testing.assert_allclose(yr, z["yr_triton"], **TOL)
    dx, dw, dg = oracle.bwd(z["x"], z["w"], gate, z["dout"], z["cu_seqlens"], G, norm, eps)
    for ref in ("torch", "triton"):
        close(dx, z[f"dx_{ref}"])
        close(dw, z[f"dw_{ref}"])
        if gate is not None:
            close(dg, z[f"dg_{ref}"])


def trunc_bits(a):
    """fp32 -> bf16 by truncation: the Triton CPU interpreter's cast (it does
    not honour the kernels' rtne request; GPU Triton and torch round to
    nearest even, as the CUDA kernels do)."""
    return (np.ascontiguousarray(a, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)


def test_train_fwd_bf16_matches_reference_kernel():
    z = load_golden("train_bf16_g8_w4_norm_gate")
    x, w, g = (bf16_bits_to_f32(z[k]) for k in ("x_bits", "w_bits", "gate_bits"))
    y, yr = oracle.fwd(x, w, g, z["cu_seqlens"], int(z["G"]), int(z["norm"]), float(z["eps"]), save_pre=True)
    for got, key in ((y, "y_bits"), (yr, "yr_bits")):
        # bit-for-bit with the interpreted kernel under its truncating cast
        assert np.mean(trunc_bits(got) == z[key]) > 0.995
        # and within one bf16 ulp under round-to-nearest-even
        np.testing.assert_allclose(bf16_bits_to_f32(f32_to_bf16_bits(got)), bf16_bits_to_f32(z[key]),
                                   rtol=2 ** -7, atol=1e-6)


def test_inference_matches_reference():
    z = load_golden("inference_g8_w4_norm_gate")
    y = oracle.inference(z["context"], z["w"], z["gate"], int(z["G"]), int(z["norm"]), float(z["eps"]))
    np.testing.assert_allclose(y, z["y_triton"], **TOL)
    np.testing.assert_allclose(y, z["y_torch"], **TOL)


@pytest.mark.parametrize("name", ["decode_rows_g4_w4_norm_gate", "decode_rows_g1_w2_gate"])
def test_decode_rows_matches_reference(name):
    z = load_golden(name)
    y, st = oracle.decode_rows(z["x"], z["w"], z["gate"], z["state"], int(z["G"]), int(z["norm"]),
                               float(z["eps"]))
    np.testing.assert_allclose(y, z["y_triton"], **TOL)
    np.testing.assert_allclose(y, z["y_torch"], **TOL)
    assert np.array_equal(st, z["state_triton"])
    assert np.array_equal(st, z["state_torch"])


@pytest.mark.parametrize("name", PACKED_CASES)
def test_packed_matches_reference(name):
    z = load_golden(name)
    y, st = oracle.packed(z["x"], z["w"], z.get("gate"), z["state"], z["starts"], z["slots"], z["has_initial"],
                          int(z["G"]), int(z["norm"]), float(z["eps"]))
    np.testing.assert_allclose(y, z["y_triton"], **TOL)
    assert np.array_equal(st, z["state_triton"]), "conv state must be bit-exact"
    if "y_torch" in z:
        np.testing.assert_allclose(y, z["y_torch"], **TOL)
        assert np.array_equal(st, z["state_torch"])


def test_packed_sd_strides_match_logical_layout():
    """The same case addressed through the transposed ("SD") storage strides."""
    z = load_golden("packed_sd_layout_w7_g16")
    D, W = int(z["D"]), int(z["W"])
    H = W - 1
    storage = np.ascontiguousarray(z["state"].transpose(0, 2, 1))  # [slots, H, D]
    y, st = oracle.packed(z["x"], z["w"], z["gate"], storage.reshape(-1), z["starts"], z["slots"],
                          z["has_initial"], int(z["G"]), int(z["norm"]), float(z["eps"]),
                          state_strides=(H * D, 1, D))
    np.testing.assert_allclose(y, z["y_triton"], **TOL)
    got = st.reshape(-1, H, D).transpose(0, 2, 1)
    assert np.array_equal(got, z["state_triton"])


def test_packed_bf16_matches_reference_kernel():
    z = load_golden("packed_bf16_stable_gate")
    x, w, g, s0 = (bf16_bits_to_f32(z[k]) for k in ("x_bits", "w_bits", "gate_bits", "state_bits"))
    y, st = oracle.packed(x, w, g, s0, z["starts"], z["slots"], z["has_initial"], int(z["G"]), int(z["norm"]),
                          float(z["eps"]))
    assert np.mean(trunc_bits(y) == z["y_bits"]) > 0.995
    np.testing.assert_allclose(bf16_bits_to_f32(f32_to_bf16_bits(y)), bf16_bits_to_f32(z["y_bits"]),
                               rtol=2 ** -7, atol=1e-6)
    assert np.array_equal(f32_to_bf16_bits(st), z["state_out_bits"]), "conv state must be bit-exact"


def test_config1_full_size_against_reference_checksums():
    """Config 1 (fp32, 2 x 256 packed, C=512, K=4, forward, seed 0) at full size."""
    torch = pytest.importorskip("torch")
    s = json.loads((GOLDEN / "config1_stats.json").read_text())
    g = torch.Generator().manual_seed(s["seed"])
    x = torch.randn(*s["shape_x"], generator=g)
    w = torch.randn(*s["shape_w"], generator=g) * s["w_scale"]
    assert abs(float(x.double().sum()) - s["x_sum"]) < 1e-6 * max(1.0, abs(s["x_sum"]))
    assert abs(float(w.double().square().sum()) - s["w_sq"]) < 1e-9 * s["w_sq"]
    y, _ = oracle.fwd(x[0].numpy(), w.numpy(), None, np.array(s["cu_seqlens"]), 1, 0)
    yd = y.astype(np.float64)
    assert abs(yd.sum() - s["y_sum"]) < 1e-3
    assert abs((yd * yd).sum() - s["y_sq"]) < 1e-6 * s["y_sq"]
    np.testing.assert_allclose(y.reshape(-1)[s["sample_idx"]], s["sample_val"], rtol=1e-5, atol=1e-6)


def test_oracle_edge_cases():
    """Empty sequences and zero-length requests behave like the reference kernels."""
    rng = np.random.default_rng(0)
    D, W, G = 16, 4, 2
    x = rng.standard_normal((5, D)).astype(np.float32)
    w = rng.standard_normal((5, W, D // G)).astype(np.float32)
    # an empty sequence in the middle of cu_seqlens is harmless
    y1, _ = oracle.fwd(x, w, None, [0, 2, 2, 5], G)
    y2, _ = oracle.fwd(x, w, None, [0, 2, 5], G)
    np.testing.assert_array_equal(y1, y2)
    # a zero-length request with history keeps its slot; without history it
    # clears it (greta_vllm/triton_conv.py:106-116 with length 0)
    state = rng.standard_normal((3, D, W - 1)).astype(np.float32)
    _, st = oracle.packed(x, w, None, state, [0, 0, 5], [1, 2], [1, 0], G)
    assert np.array_equal(st[0], state[0])
    assert np.array_equal(st[1], state[1])  # slot 1: unchanged (length 0, history on)
    assert np.array_equal(st[2, :, :], x[2:5].T)  # slot 2: last W-1 inputs of request 1
