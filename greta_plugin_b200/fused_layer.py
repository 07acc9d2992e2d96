"""Greta's convolution layer with its three input projections fused into one
GEMM, for training (the HF path) -- the forward and backward sides of
fusing the conv with its neighbouring projections.

The reference layer (greta/modeling_greta.py:426-459, GretaDynamicConv)
computes x = in_proj(h), gate = gate_proj(h) and filters = kernel_proj(h)
as three GEMMs over the same hidden states, and autograd runs three backward
GEMM pairs for them. Here the three weights are one matrix

    proj = [in_proj | gate_proj | kernel_proj | zero rows]   [R, hidden]

(R = 2D + W*D/G rounded up to a multiple of 8, so that every row of the
output is 16-byte aligned), so that

  forward   cat = h @ proj^T + bias   ONE GEMM; the conv kernel reads x, gate
                                      and filters in place from `cat` through
                                      row strides (greta_dynconv_fwd_ld_ex)
  backward  the conv backward writes dx, dg and dw straight into the column
            blocks of one gradient buffer dcat (greta_dynconv_bwd_ld_ex), so
            d(hidden) = dcat @ proj and d(proj) = dcat^T @ h are ONE GEMM
            each, instead of three of each.

out_proj stays an nn.Linear. The layer keeps the reference's parameter
shapes through views of `proj` (in_proj_weight, gate_proj_weight,
kernel_proj_weight), and `from_module` loads a reference GretaDynamicConv.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from . import _capi


def _rows(D: int, W: int, G: int) -> int:
    return (2 * D + W * (D // G) + 7) // 8 * 8


def _norm_code(norm: bool) -> int:
    return _capi.NORM_PLAIN if norm else _capi.NORM_NONE


def conv_forward_inplace(cat, D, W, G, cu_seqlens, norm, eps, save_pre):
    """The conv over x = cat[:, :D], gate = cat[:, D:2D], filters =
    cat[:, 2D:2D+W*D/G] viewed [T, W, D/G]: returns (y, yr) (yr None unless
    norm and save_pre)."""
    T, R = cat.shape
    y = torch.empty(T, D, device=cat.device, dtype=cat.dtype)
    yr = torch.empty_like(y) if (norm and save_pre) else None
    if T == 0:
        return y, yr
    es = cat.element_size()
    base = cat.data_ptr()
    with torch.cuda.device(cat.device.index):
        st = _capi.lib().greta_dynconv_fwd_ld_ex(
            _capi.dtype_code(cat), base, R, base + 2 * D * es, R, base + D * es, R, _capi.ptr(y), _capi.ptr(yr),
            _capi.ptr(cu_seqlens), 0 if cu_seqlens is None else int(cu_seqlens.dtype == torch.int64),
            0 if cu_seqlens is None else cu_seqlens.numel() - 1, T, D, W, G, _norm_code(norm), float(eps),
            _capi.stream_of(cat), _capi.options())
    _capi.check("greta_dynconv_fwd_ld_ex", st)
    return y, yr


def conv_backward_inplace(cat, yr, dout, dcat, D, W, G, cu_seqlens, norm, eps):
    """The conv backward for the inputs held in `cat`, writing dx, dg and dw
    into the matching column blocks of `dcat` (same shape as cat)."""
    T, R = cat.shape
    if T == 0:
        return
    es = cat.element_size()
    b, db = cat.data_ptr(), dcat.data_ptr()
    dout = dout.contiguous()
    with torch.cuda.device(cat.device.index):
        st = _capi.lib().greta_dynconv_bwd_ld_ex(
            _capi.dtype_code(cat), b, R, b + 2 * D * es, R, b + D * es, R, _capi.ptr(yr), _capi.ptr(dout),
            db, R, db + 2 * D * es, R, db + D * es, R, _capi.ptr(cu_seqlens),
            0 if cu_seqlens is None else int(cu_seqlens.dtype == torch.int64),
            0 if cu_seqlens is None else cu_seqlens.numel() - 1, T, D, W, G, _norm_code(norm), float(eps),
            _capi.stream_of(cat), _capi.options())
    _capi.check("greta_dynconv_bwd_ld_ex", st)


class FusedProjConvFunction(torch.autograd.Function):
    """(h [T, hidden], proj [R, hidden], bias [W*D/G]) -> conv output [T, D]."""

    @staticmethod
    def forward(ctx, h, proj, bias, cu_seqlens, D, W, G, norm, eps):
        R = proj.shape[0]
        nk = W * (D // G)
        bcat = torch.zeros(R, device=h.device, dtype=h.dtype)
        bcat[2 * D:2 * D + nk] = bias
        cat = F.linear(h, proj, bcat)
        y, yr = conv_forward_inplace(cat, D, W, G, cu_seqlens, norm, eps, save_pre=True)
        ctx.save_for_backward(h, proj, cat, yr, cu_seqlens)
        ctx.dims = (D, W, G, norm, eps)
        return y

    @staticmethod
    def backward(ctx, dy):
        h, proj, cat, yr, cu_seqlens = ctx.saved_tensors
        D, W, G, norm, eps = ctx.dims
        nk = W * (D // G)
        dcat = torch.empty_like(cat)
        if dcat.shape[1] > 2 * D + nk:
            dcat[:, 2 * D + nk:].zero_()
        conv_backward_inplace(cat, yr, dy, dcat, D, W, G, cu_seqlens, norm, eps)
        dh = dcat @ proj                     # one GEMM for all three projections
        dproj = dcat.t() @ h                 # and one for their weights
        dbias = dcat[:, 2 * D:2 * D + nk].sum(0)
        return dh, dproj, dbias, None, None, None, None, None, None


class FusedGretaConv(torch.nn.Module):
    """GretaDynamicConv's training forward on packed sequences with the three
    input projections as one GEMM: forward(h [T, hidden], cu_seqlens) ->
    out_proj(conv(...)) [T, hidden]."""

    def __init__(self, hidden, D, W, G, norm=True, eps=1e-6, device=None, dtype=None):
        super().__init__()
        self.D, self.W, self.G, self.norm, self.eps = D, W, G, norm, eps
        kw = dict(device=device, dtype=dtype)
        self.proj = torch.nn.Parameter(torch.zeros(_rows(D, W, G), hidden, **kw))
        self.kernel_bias = torch.nn.Parameter(torch.zeros(W * (D // G), **kw))
        self.out_proj = torch.nn.Linear(D, hidden, bias=False, **kw)

    # the reference's parameters, as views of the fused matrix
    @property
    def in_proj_weight(self):
        return self.proj[:self.D]

    @property
    def gate_proj_weight(self):
        return self.proj[self.D:2 * self.D]

    @property
    def kernel_proj_weight(self):
        return self.proj[2 * self.D:2 * self.D + self.W * (self.D // self.G)]

    @classmethod
    def from_module(cls, m):
        """From a reference GretaDynamicConv (greta/modeling_greta.py:415-433)."""
        hidden = m.in_proj.weight.shape[1]
        D, W, G = m.in_proj.weight.shape[0], m.kernel_size, m.group_size
        p = m.in_proj.weight
        out = cls(hidden, D, W, G, m.norm, m.norm_eps, device=p.device, dtype=p.dtype)
        with torch.no_grad():
            out.in_proj_weight.copy_(m.in_proj.weight)
            out.gate_proj_weight.copy_(m.gate_proj.weight)
            out.kernel_proj_weight.copy_(m.kernel_proj.weight)
            out.kernel_bias.copy_(m.kernel_proj.bias)
            out.out_proj.weight.copy_(m.out_proj.weight)
        return out

    def forward(self, h, cu_seqlens=None):
        if not h.is_cuda:
            raise ValueError("FusedGretaConv requires CUDA tensors")
        y = FusedProjConvFunction.apply(h, self.proj, self.kernel_bias, cu_seqlens, self.D, self.W, self.G,
                                        self.norm, self.eps)
        return self.out_proj(y)


__all__ = ["FusedGretaConv", "FusedProjConvFunction", "conv_forward_inplace", "conv_backward_inplace"]
