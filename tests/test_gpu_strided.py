"""Strided inputs of the vLLM packed path and the tensor-parallel GretaConv
layer on the GPU.

* x, gate and filters as column blocks of ONE projection output
  [T, D | D | W*D/G (+ padding)] (greta_dynconv_packed_state_ld_ex): every
  kernel family (row-streaming prefill, decode, register-staged, wide-group)
  gives the same bits as the contiguous call, and the same conv state;
  unaligned row strides fall back to contiguous copies;
* greta_plugin_b200.tp.TPGretaConv: the fused one-GEMM projection equals the
  three-GEMM form, and two channel shards run on one GPU (their out_proj
  partial sums added, the all-reduce of a 2-rank group) equal the unsharded
  layer, against the oracle's convolution."""
import numpy as np
import pytest
import torch

from gpu_helpers import DEV, assert_close, rand
from greta_plugin_b200 import _capi
from greta_plugin_b200.vllm_conv import packed_dynamic_conv_triton
from oracle import oracle

pytestmark = pytest.mark.gpu


def fused_inputs(g, T, D, W, G, pad, dtype=torch.bfloat16):
    """x, w, gate as views of one [T, 2D + W*D/G + pad] buffer, and their
    contiguous copies."""
    DC = D // G
    row = 2 * D + W * DC + pad
    buf = rand(g, T, row, dtype=dtype).to(DEV)
    buf[:, 2 * D:2 * D + W * DC] *= (1.0 / W) ** 0.5
    x, gate = buf[:, :D], buf[:, D:2 * D]
    w = buf[:, 2 * D:2 * D + W * DC].unflatten(1, (W, DC))
    return (x, w, gate), (x.contiguous(), w.contiguous(), gate.contiguous())


def batch(g, lengths, n_slots, D, W, dtype=torch.bfloat16):
    N = len(lengths)
    starts = torch.tensor([0] + list(np.cumsum(lengths)), dtype=torch.int32, device=DEV)
    slots = torch.randperm(n_slots, generator=g)[:N].to(torch.int32)
    slots[::5] = -1
    init = (torch.arange(N) % 3 != 1).to(torch.int8)
    state = rand(g, n_slots, D, W - 1, dtype=dtype).to(DEV)
    return starts, slots.to(DEV), init.to(DEV), state


CASES = [
    # lengths, D, W, G, pad, kernel family, dtype
    ([37, 1, 90, 5, 200, 3], 1024, 4, 1, 0, "auto", torch.bfloat16),       # prefill-like: row streaming
    ([37, 1, 90, 5, 200, 3], 1024, 4, 1, 8, "register", torch.bfloat16),
    ([1] * 40 + [9], 2048, 7, 128, 8, "auto", torch.bfloat16),            # decode-like: decode kernel
    ([1] * 40 + [9], 2048, 7, 128, 0, "register", torch.bfloat16),
    ([60, 2, 33], 2048, 7, 128, 8, "auto", torch.bfloat16),                # Greta layer prefill
    ([60, 2, 33], 2048, 7, 512, 8, "auto", torch.bfloat16),                # wide groups
    ([17, 4], 512, 3, 8, 24, "auto", torch.bfloat16),
    ([33, 1, 70], 512, 4, 16, 8, "auto", torch.float16),
    ([1] * 12 + [40], 512, 7, 64, 4, "auto", torch.float32),
]


@pytest.mark.parametrize("lengths,D,W,G,pad,kernel,dtype", CASES)
def test_strided_inputs_give_the_contiguous_bits(lengths, D, W, G, pad, kernel, dtype):
    g = torch.Generator().manual_seed(D + W + G + pad)
    T = sum(lengths)
    (xs, ws, gs), (xc, wc, gc) = fused_inputs(g, T, D, W, G, pad, dtype)
    assert xs.stride(0) != D
    starts, slots, init, state = batch(g, lengths, 64, D, W, dtype)
    s1, s2 = state.clone(), state.clone()
    with _capi.launch_options(kernel=kernel):
        y1 = packed_dynamic_conv_triton(xc, wc, gc, s1, starts, slots, init, G, norm=True)
        y2 = packed_dynamic_conv_triton(xs, ws, gs, s2, starts, slots, init, G, norm=True)
    assert torch.equal(y1, y2)
    assert torch.equal(s1, s2)
    yo, so = oracle.packed(xc.float().cpu().numpy(), wc.float().cpu().numpy(), gc.float().cpu().numpy(),
                           state.float().cpu().numpy(), starts.cpu().numpy(), slots.cpu().numpy(),
                           init.cpu().numpy(), G, oracle.NORM_STABLE)
    assert_close(y2, yo, dtype)
    assert np.array_equal(s2.float().cpu().numpy(), so)


def test_unaligned_row_stride_falls_back_to_a_copy():
    g = torch.Generator().manual_seed(3)
    D, W, G = 256, 4, 8
    (xs, ws, gs), (xc, wc, gc) = fused_inputs(g, 50, D, W, G, pad=3)  # row of 2*256 + 128 + 3 elements
    starts, slots, init, state = batch(g, [20, 30], 8, D, W)
    s1, s2 = state.clone(), state.clone()
    y1 = packed_dynamic_conv_triton(xc, wc, gc, s1, starts, slots, init, G)
    y2 = packed_dynamic_conv_triton(xs, ws, gs, s2, starts, slots, init, G)
    assert torch.equal(y1, y2) and torch.equal(s1, s2)


class _Layer(torch.nn.Module):
    """The parameter layout of the reference's GretaConv
    (greta_vllm/model.py:91-95)."""

    def __init__(self, hidden, D, W, G, dtype):
        super().__init__()
        self.kernel_proj = torch.nn.Linear(hidden, (D // G) * W, bias=True)
        self.gate_proj = torch.nn.Linear(hidden, D, bias=False)
        self.in_proj = torch.nn.Linear(hidden, D, bias=False)
        self.out_proj = torch.nn.Linear(D, hidden, bias=False)
        self.kernel_size, self.group_size, self.norm, self.norm_eps = W, G, True, 1e-6
        self.to(device=DEV, dtype=dtype)


@pytest.mark.parametrize("lengths", [[1] * 24 + [30], [50, 70, 3]])
def test_tp_layer_shards_and_fused_projection(lengths):
    from greta_plugin_b200.tp import TPGretaConv

    torch.manual_seed(7)
    hidden, D, W, G = 512, 512, 7, 64
    layer = _Layer(hidden, D, W, G, torch.bfloat16)
    g = torch.Generator().manual_seed(8)
    T = sum(lengths)
    h = rand(g, T, hidden, scale=0.5).to(DEV)
    starts, slots, init, state = batch(g, lengths, 32, D, W)

    # the unsharded layer with the oracle's convolution (fp32 on the host)
    with torch.no_grad():
        x = layer.in_proj(h).float()
        gate = layer.gate_proj(h).float()
        w = layer.kernel_proj(h).float().view(T, W, D // G)
    yo, so = oracle.packed(x.cpu().numpy(), w.cpu().numpy(), gate.cpu().numpy(), state.float().cpu().numpy(),
                           starts.cpu().numpy(), slots.cpu().numpy(), init.cpu().numpy(), G, oracle.NORM_STABLE)
    with torch.no_grad():
        ref = torch.from_numpy(yo).to(DEV) @ layer.out_proj.weight.float().T

    outs = {}
    for fused in (False, True):
        st = state.clone()
        total = torch.zeros(T, hidden, device=DEV)
        for rank in range(2):
            tp = TPGretaConv.from_layer(layer, rank, 2, fused=fused)
            with torch.no_grad():
                total += tp(h, st[:, tp.w.lo:tp.w.hi, :], starts, slots, init, reduce=False).float()
        outs[fused] = total
        # the state holds the rank's projected inputs, which its own (sharded
        # or concatenated) GEMM may round differently from the full one
        np.testing.assert_allclose(st.float().cpu().numpy(), so, rtol=1e-2, atol=1e-2)
    scale = float(ref.abs().max())
    for fused, y in outs.items():
        np.testing.assert_allclose(y.cpu().numpy(), ref.cpu().numpy(), rtol=2e-2, atol=2e-2 * scale)
    np.testing.assert_allclose(outs[True].cpu().numpy(), outs[False].cpu().numpy(), rtol=2e-2, atol=2e-2 * scale)
