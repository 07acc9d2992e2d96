"""The training layer with its three input projections fused into one GEMM
(greta_plugin_b200.fused_layer) against the reference layer's structure --
three projections, the convolution (dynamic_causal_conv1d, itself checked
against the oracle elsewhere), out_proj -- with the same weights: output and
every gradient (hidden states, the three projection weights, kernel_proj's
bias, out_proj). Also the strided training entry points directly: the conv
reading x, gate and filters from one projection output and writing dx, dg, dw
into one gradient buffer gives the contiguous calls' bits."""
import numpy as np
import pytest
import torch

from gpu_helpers import DEV, rand
from greta_plugin_b200 import dynamic_causal_conv1d
from greta_plugin_b200.dynamic_conv import dynconv_bwd, dynconv_fwd
from greta_plugin_b200.fused_layer import FusedGretaConv, conv_backward_inplace, conv_forward_inplace

pytestmark = pytest.mark.gpu


class _RefLayer(torch.nn.Module):
    """The parameters of the reference's GretaDynamicConv
    (greta/modeling_greta.py:426-433) and its training forward on packed
    sequences: three projections, the conv, out_proj."""

    def __init__(self, hidden, D, W, G, norm, dtype):
        super().__init__()
        self.kernel_proj = torch.nn.Linear(hidden, (D // G) * W, bias=True)
        self.gate_proj = torch.nn.Linear(hidden, D, bias=False)
        self.in_proj = torch.nn.Linear(hidden, D, bias=False)
        self.out_proj = torch.nn.Linear(D, hidden, bias=False)
        self.kernel_size, self.group_size, self.norm, self.norm_eps = W, G, norm, 1e-6
        self.to(device=DEV, dtype=dtype)

    def forward(self, h, cu):
        T = h.shape[0]
        w = self.kernel_proj(h).view(T, self.kernel_size, -1)
        y = dynamic_causal_conv1d(self.in_proj(h)[None], w, self.gate_proj(h)[None], cu, self.group_size,
                                  self.norm, self.norm_eps)
        return self.out_proj(y[0])


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("hidden,D,W,G,norm,lens", [
    (256, 256, 7, 128, True, [40, 3, 90, 1]),
    (512, 512, 4, 8, False, [200, 57]),
    (256, 512, 3, 32, True, [17, 1, 2, 64]),
])
def test_fused_layer_matches_three_projections(dtype, hidden, D, W, G, norm, lens):
    torch.manual_seed(hidden + D + W)
    ref = _RefLayer(hidden, D, W, G, norm, dtype)
    fused = FusedGretaConv.from_module(ref)
    g = torch.Generator().manual_seed(3)
    T = sum(lens)
    cu = torch.tensor([0] + list(np.cumsum(lens)), dtype=torch.int32, device=DEV)
    h0 = rand(g, T, hidden, dtype=dtype).to(DEV)
    dout = rand(g, T, hidden, dtype=dtype).to(DEV)

    h1 = h0.clone().requires_grad_()
    y1 = ref(h1, cu)
    y1.backward(dout)
    h2 = h0.clone().requires_grad_()
    y2 = fused(h2, cu)
    y2.backward(dout)

    tol = dict(rtol=1e-4, atol=1e-4) if dtype == torch.float32 else dict(rtol=2e-2, atol=2e-2)

    def close(a, b):
        a, b = a.detach().float(), b.detach().float()
        scale = max(1.0, float(b.abs().max()))
        torch.testing.assert_close(a, b, rtol=tol["rtol"], atol=tol["atol"] * scale)

    close(y2, y1)
    close(h2.grad, h1.grad)
    close(fused.proj.grad[:D], ref.in_proj.weight.grad)
    close(fused.proj.grad[D:2 * D], ref.gate_proj.weight.grad)
    close(fused.proj.grad[2 * D:2 * D + W * (D // G)], ref.kernel_proj.weight.grad)
    close(fused.kernel_bias.grad, ref.kernel_proj.bias.grad)
    close(fused.out_proj.weight.grad, ref.out_proj.weight.grad)
    assert torch.count_nonzero(fused.proj.grad[2 * D + W * (D // G):]) == 0  # padding rows


@pytest.mark.parametrize("kernel", ["auto", "register"])
@pytest.mark.parametrize("D,W,G,norm,lens", [(2048, 7, 128, True, [300, 5, 1000]), (1024, 4, 1, False, [77, 400])])
def test_strided_training_calls_give_the_contiguous_bits(kernel, D, W, G, norm, lens):
    from greta_plugin_b200 import _capi

    g = torch.Generator().manual_seed(D + W)
    T = sum(lens)
    nk = W * (D // G)
    R = (2 * D + nk + 7) // 8 * 8
    cat = rand(g, T, R).to(DEV)
    cat[:, 2 * D:] *= (1.0 / W) ** 0.5
    x, gate, w = cat[:, :D], cat[:, D:2 * D], cat[:, 2 * D:2 * D + nk].unflatten(1, (W, D // G))
    dout = rand(g, T, D).to(DEV)
    cu = torch.tensor([0] + list(np.cumsum(lens)), dtype=torch.int32, device=DEV)
    with _capi.launch_options(kernel=kernel):
        y1, yr1, _, _ = dynconv_fwd(x.contiguous()[None], w.contiguous(), gate.contiguous()[None], cu, G, norm=norm,
                                    save_pre=True)
        y2, yr2 = conv_forward_inplace(cat, D, W, G, cu, norm, 1e-6, save_pre=True)
        assert torch.equal(y1[0], y2)
        if norm:
            assert torch.equal(yr1[0], yr2)
        dx1, dw1, dg1 = dynconv_bwd(x.contiguous()[None], w.contiguous(), gate.contiguous()[None],
                                    yr1 if norm else None, dout[None], cu, G, norm, 1e-6, 64, None)
        dcat = torch.full_like(cat, 7.0)
        conv_backward_inplace(cat, yr2, dout, dcat, D, W, G, cu, norm, 1e-6)
    assert torch.equal(dx1[0], dcat[:, :D])
    assert torch.equal(dg1[0], dcat[:, D:2 * D])
    assert torch.equal(dw1, dcat[:, 2 * D:2 * D + nk].unflatten(1, (W, D // G)))
    assert bool((dcat[:, 2 * D + nk:] == 7.0).all())  # the padding columns are untouched
