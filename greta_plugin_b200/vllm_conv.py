"""Drop-in replacements for the vLLM conv path of the reference on B200.

  packed_dynamic_conv_triton   greta_vllm/triton_conv.py:128-173 -> greta_dynconv_packed_state
                               (its _conv_kernel and _state_kernel fused in one launch)
  supports                     greta_vllm/triton_conv.py:119-121

A vLLM batch is a flat run of T tokens from N requests (`starts` holds the
cumulative offsets, decodes first). Each request owns a cache slot holding its
last W-1 projected inputs; a negative slot means no history and no
write-back. The conv reads history from earlier tokens of the same request or
from the slot, applies the overflow-safe group RMS norm and the SiLU gate, and
the slot is rewritten with the request's last W-1 inputs, bit-exact.

The launch uses device values and tensor shapes only -- no allocation (given
`out`), no host synchronisation -- so a decode step can be captured in a CUDA
graph. `seq_idx` is accepted for signature compatibility and not needed: each
CTA finds its request from `starts` on the device.
"""
from __future__ import annotations

import torch

from . import _capi

def supports(group_size: int, channels: int) -> bool:
    """The reference's rule (greta_vllm/triton_conv.py:119-121): a power-of-two
    group size dividing the channels. Groups of up to 256 channels run within
    one warp; wider ones on a kernel that gives each CTA one whole group."""
    return group_size > 0 and group_size & (group_size - 1) == 0 and channels % group_size == 0


def _aligned_rows(t, row_stride):
    """Rows that start on whole 8-element vectors (the kernels load a
    thread's 8 channels as one aligned pack: 16 bytes for 16-bit types, 32
    for fp32)."""
    return t.data_ptr() % (8 * t.element_size()) == 0 and row_stride % 8 == 0


def _rows(t, channels):
    """A [T, D] input as (tensor, row stride): a view whose rows are
    contiguous and 16-byte aligned (e.g. a column block of one projection
    GEMM's output) is read in place, anything else is made contiguous."""
    if t.stride(1) == 1 and t.stride(0) >= channels and _aligned_rows(t, t.stride(0)):
        return t, t.stride(0)
    return t.contiguous(), channels


def _filter_rows(w):
    """Filters [T, W, D/G] as (tensor, token-row stride): each token's W
    filter rows must be contiguous (tap-major compact); the token rows may be
    spaced (a column block of a concatenated projection output)."""
    T, W, DC = w.shape
    if w.stride(2) == 1 and (W == 1 or w.stride(1) == DC) and w.stride(0) >= W * DC and \
            _aligned_rows(w, w.stride(0)):
        return w, w.stride(0)
    return w.contiguous(), W * DC


def _launch(x, weights, gate, state, starts, slots, has_initial, group_size, norm, eps, out, flags):
    tokens, channels = x.shape
    width = weights.shape[1]
    if out is None:
        out = torch.empty_like(x)
    if tokens == 0:
        return out
    if not supports(group_size, channels):
        raise ValueError('Triton dynamic convolution needs a power-of-two group size dividing D')
    if weights.shape != (tokens, width, channels // group_size):
        raise ValueError('Incompatible dynamic-convolution weight/group dimensions')
    if state.shape[1:] != (channels, width - 1):
        raise ValueError('Convolution cache has the wrong shape')
    if not x.is_cuda:
        raise ValueError('packed_dynamic_conv_triton requires CUDA tensors')
    if state.dtype != x.dtype:
        raise ValueError(f'Convolution cache dtype {state.dtype} must match x dtype {x.dtype}')
    if out.dtype != x.dtype or out.shape != x.shape or not out.is_contiguous():
        raise ValueError('out must be a contiguous tensor shaped and typed like x')
    x, ldx = _rows(x, channels)
    if weights.dtype != x.dtype:
        weights = weights.to(x.dtype)
    weights, ldw = _filter_rows(weights)
    ldg = channels
    if gate is not None:
        if gate.dtype != x.dtype:
            gate = gate.to(x.dtype)
        gate, ldg = _rows(gate, channels)
    starts = starts.to(device=x.device, dtype=torch.int32).contiguous()
    slots = slots.to(device=x.device, dtype=torch.int32).reshape(-1).contiguous()
    has_initial = has_initial.to(device=x.device, dtype=torch.int8).reshape(-1).contiguous()
    s_slot, s_d, s_h = state.stride()
    with torch.cuda.device(x.device.index):
        st = _capi.lib().greta_dynconv_packed_state_ld_ex(
            _capi.dtype_code(x), _capi.ptr(x), ldx, _capi.ptr(weights), ldw, _capi.ptr(gate), ldg, _capi.ptr(out),
            _capi.ptr(state) if state.numel() else None, state.shape[0], s_slot, s_d, s_h, _capi.ptr(starts),
            _capi.ptr(slots), _capi.ptr(has_initial), slots.numel(), tokens, channels, width, group_size,
            _capi.NORM_STABLE if norm else _capi.NORM_NONE, float(eps), _capi.ptr(flags), _capi.stream_of(x),
            _capi.options())
    _capi.check("greta_dynconv_packed_state", st)
    return out


def packed_dynamic_conv_triton(x, weights, gate, state, starts, slots, has_initial,
                               group_size, norm=True, eps=1e-6, seq_idx=None, out=None):
    """B200 version of ``conv.packed_dynamic_conv`` (same arguments and result).

    x: [T, D]; weights: [T, W, D/G]; gate: [T, D] or None; state: [slots, D, W-1]
    (any strides). starts: [N+1]; slots, has_initial: [N]. seq_idx: accepted,
    unused. A negative slot means no history and no write-back. ``out`` ([T, D])
    is filled in place when given.
    """
    return _launch(x, weights, gate, state, starts, slots, has_initial, group_size, norm, eps, out, None)


def packed_dynamic_conv_checked(x, weights, gate, state, starts, slots, has_initial, group_size, norm=True,
                                eps=1e-6, out=None):
    """packed_dynamic_conv_triton plus device checks.

    Slots >= state.shape[0] are skipped by the kernel (no read, no write-back)
    and reported here as IndexError. A pipeline wait of a row-streaming kernel
    that ran out (the kernel then returns with part of `out` unwritten) is
    reported as GretaKernelError. The checks synchronise the device, so this
    is for debugging and tests, not for the serving loop.
    """
    flags = torch.zeros(1, dtype=torch.int32, device=x.device)
    out = _launch(x, weights, gate, state, starts, slots, has_initial, group_size, norm, eps, out, flags)
    if int(flags.item()) & 1:
        raise IndexError(f"a cache slot index is >= the number of cache slots ({state.shape[0]})")
    with torch.cuda.device(x.device.index):
        _capi.check_device_errors("packed_dynamic_conv_checked")
    return out


__all__ = ["packed_dynamic_conv_triton", "packed_dynamic_conv_checked", "supports"]
