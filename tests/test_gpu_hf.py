"""HF Transformers paths (greta/dynamic_conv.py inference-from-context and
single-token decode) on the GPU vs the CPU oracle."""
import numpy as np
import pytest
import torch

from gpu_helpers import DEV, assert_close, rand, to_np
from oracle import oracle

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("W,G,norm,gate_on", [(4, 1, False, False), (7, 128, True, True), (3, 4, True, False),
                                              (5, 8, False, True), (1, 2, True, True)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_inference_from_context(W, G, norm, gate_on, dtype):
    from greta_plugin_b200 import dynamic_causal_conv1d_inference

    g = torch.Generator().manual_seed(W * 10 + G)
    B, Q, D = 3, 77, 256
    ctx = rand(g, B, Q + W - 1, D, dtype=dtype)
    w = rand(g, B, Q, W, D // G, scale=0.5, dtype=dtype)
    gate = rand(g, B, Q, D, dtype=dtype) if gate_on else None
    y = dynamic_causal_conv1d_inference(ctx.to(DEV), w.to(DEV), None if gate is None else gate.to(DEV), G, norm)
    yo = oracle.inference(to_np(ctx), to_np(w), to_np(gate), G, int(norm))
    assert_close(y, yo, dtype)


@pytest.mark.parametrize("W,G,norm,gate_on", [(4, 1, False, False), (7, 128, True, True), (2, 4, True, False),
                                              (8, 16, False, True), (12, 2, True, True)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_decode_rows(W, G, norm, gate_on, dtype):
    from greta_plugin_b200 import dynamic_causal_conv1d_decode

    g = torch.Generator().manual_seed(W * 7 + G)
    B, D = 19, 512
    x = rand(g, B, D, dtype=dtype)
    w = rand(g, B, W, D // G, scale=0.5, dtype=dtype)
    gate = rand(g, B, D, dtype=dtype) if gate_on else None
    state0 = rand(g, B, D, W - 1, dtype=dtype)
    state = state0.to(DEV).clone()
    y = dynamic_causal_conv1d_decode(x.to(DEV), w.to(DEV), state, None if gate is None else gate.to(DEV), G, norm)
    yo, so = oracle.decode_rows(to_np(x), to_np(w), to_np(gate), to_np(state0), G, int(norm))
    assert_close(y, yo, dtype)
    assert np.array_equal(state.float().cpu().numpy(), so), "conv state must be bit-exact"


def test_decode_errors_match_reference():
    from greta_plugin_b200 import dynamic_causal_conv1d_decode

    x = torch.zeros(2, 64, device=DEV)
    w = torch.zeros(2, 4, 64, device=DEV)
    st = torch.zeros(2, 64, 3, device=DEV)
    with pytest.raises(ValueError, match="must be contiguous"):
        dynamic_causal_conv1d_decode(x, w, torch.zeros(2, 3, 64, device=DEV).transpose(1, 2))
    with pytest.raises(ValueError, match="kernel_size >= 2"):
        dynamic_causal_conv1d_decode(x, torch.zeros(2, 1, 64, device=DEV), torch.zeros(2, 64, 0, device=DEV))
    with pytest.raises(ValueError, match="divide 128"):
        dynamic_causal_conv1d_decode(torch.zeros(2, 512, device=DEV), torch.zeros(2, 4, 2, device=DEV),
                                     torch.zeros(2, 512, 3, device=DEV), group_size=256)
    with pytest.raises(ValueError, match="requires CUDA tensors"):
        dynamic_causal_conv1d_decode(x.cpu(), w.cpu(), st.cpu())


def test_hf_decode_sequence_matches_prefill():
    """Prefill a context, then decode token by token: the decode outputs equal
    the inference kernel's outputs on the full context (same plain norm)."""
    from greta_plugin_b200 import dynamic_causal_conv1d_decode, dynamic_causal_conv1d_inference

    g = torch.Generator().manual_seed(21)
    B, Q, D, W, G = 2, 12, 256, 4, 8
    ctx = rand(g, B, Q + W - 1, D).to(DEV)
    w = rand(g, B, Q, W, D // G, scale=0.5).to(DEV)
    gate = rand(g, B, Q, D).to(DEV)
    y_full = dynamic_causal_conv1d_inference(ctx, w, gate, G, True)
    state = ctx[:, : W - 1].transpose(1, 2).contiguous()
    for q in range(Q):
        yq = dynamic_causal_conv1d_decode(ctx[:, W - 1 + q].contiguous(), w[:, q].contiguous(), state,
                                          gate[:, q].contiguous(), G, True)
        torch.testing.assert_close(yq, y_full[:, q], rtol=0, atol=0)


def _autograd_from_context_per_row(context, weights, gate, group_size, norm, eps):
    """The reference's algorithm (greta/modeling_greta.py:378-414): one
    training-kernel call per batch row on that row's context, filters and gate
    zero-padded over the history rows, keeping the last Q outputs."""
    from greta_plugin_b200 import dynamic_causal_conv1d

    B, Q, W, F = weights.shape
    L = context.shape[1]
    outs = []
    for b in range(B):
        pw = weights.new_zeros((L, W, F))
        pw[-Q:] = weights[b]
        pg = None
        if gate is not None:
            pg = gate.new_zeros((1, L, gate.shape[-1]))
            pg[:, -Q:] = gate[b:b + 1]
        full = dynamic_causal_conv1d(context[b:b + 1].contiguous(), pw.contiguous(), pg, None, group_size, norm, eps)
        outs.append(full[:, -Q:])
    return torch.cat(outs, dim=0)


@pytest.mark.parametrize("W,G,norm,gate_on", [(7, 128, True, True), (4, 1, False, False), (3, 8, True, False)])
def test_autograd_from_context_one_packed_call(W, G, norm, gate_on):
    """triton_dynamic_causal_conv1d_autograd_from_context as one packed call:
    output and the gradients of context, weights and gate equal the per-row
    loop of the reference's helper (within bf16 tolerance), and the output
    matches the oracle's inference from context."""
    from greta_plugin_b200.dynamic_conv import triton_dynamic_causal_conv1d_autograd_from_context as packed

    g = torch.Generator().manual_seed(W * 13 + G)
    B, Q, D = 3, 45, 256
    ctx0 = rand(g, B, Q + W - 1, D)
    w0 = rand(g, B, Q, W, D // G, scale=0.5)
    g0 = rand(g, B, Q, D) if gate_on else None
    dout = rand(g, B, Q, D).to(DEV)
    results = []
    for fn in (packed, _autograd_from_context_per_row):
        ctx = ctx0.to(DEV).requires_grad_()
        w = w0.to(DEV).requires_grad_()
        gt = g0.to(DEV).requires_grad_() if gate_on else None
        y = fn(ctx, w, gt, G, norm, 1e-6)
        y.backward(dout)
        results.append((y.detach(), ctx.grad, w.grad, None if gt is None else gt.grad))
    for a, b in zip(results[0], results[1]):
        if a is not None:
            assert_close(a, b, torch.bfloat16)
    yo = oracle.inference(to_np(ctx0), to_np(w0), to_np(g0), G, int(norm))
    assert_close(results[0][0], yo, torch.bfloat16)


@pytest.mark.parametrize("W,G,norm,gate_on", [(4, 1, False, False), (7, 128, True, True), (4, 8, True, True)])
def test_decode_rows_kernels_bit_identical(W, G, norm, gate_on):
    """HF decode rows run on the decode kernel (W = 4 or 7, contiguous state);
    a 256-thread CTA shape, which that kernel does not take, forces the
    register kernel: y and the shifted state agree bit for bit."""
    from greta_plugin_b200 import _capi, dynamic_causal_conv1d_decode

    g = torch.Generator().manual_seed(W + G)
    B, D = 37, 1024
    x = rand(g, B, D).to(DEV)
    w = rand(g, B, W, D // G, scale=0.5).to(DEV)
    gate = rand(g, B, D).to(DEV) if gate_on else None
    state0 = rand(g, B, D, W - 1).to(DEV)
    outs = []
    for shape in ((0, 0, 0), (256, 1, 1)):
        with _capi.launch_options(block_x=shape[0], block_y=shape[1], tokens=shape[2]):
            st = state0.clone()
            y = dynamic_causal_conv1d_decode(x, w, st, gate, G, norm)
            outs.append((y, st))
    assert torch.equal(outs[0][0].view(torch.int16), outs[1][0].view(torch.int16))
    assert torch.equal(outs[0][1].view(torch.int16), outs[1][1].view(torch.int16))
