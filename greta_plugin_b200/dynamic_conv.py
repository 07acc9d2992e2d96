"""Drop-in replacements for greta/dynamic_conv.py on B200 (sm_100a CUDA kernels).

Same names, signatures, shapes, dtypes, return values and error messages as
the reference module; the Triton launches are replaced by calls into
libgreta_dynconv.so:

  dynconv_fwd                       greta/dynamic_conv.py:786-823  -> greta_dynconv_fwd
  dynconv_bwd                       greta/dynamic_conv.py:826-864  -> greta_dynconv_bwd
  DynamicCausalConv1dFunction       greta/dynamic_conv.py:867-893
  dynamic_causal_conv1d             greta/dynamic_conv.py:896-931
  dynamic_causal_conv1d_inference   greta/dynamic_conv.py:643-687  -> greta_dynconv_inference
  dynamic_causal_conv1d_decode      greta/dynamic_conv.py:722-765  -> greta_dynconv_decode_rows

Differences that callers can observe:
  * no host synchronisation: sequences are resolved on the device, so
    `cu_seqlens_cpu` is accepted and ignored, and the `chunk_indices` element
    returned by dynconv_fwd is None (dynconv_bwd accepts and ignores it);
  * outputs are rounded to the I/O dtype with round-to-nearest-even, as the
    reference kernels request (`fp_downcast_rounding="rtne"`).
There is no CPU fallback: non-CUDA tensors raise ValueError like the reference.
"""
from __future__ import annotations

import contextlib
import functools
import inspect
from typing import Optional

import torch

from . import _capi

BD_AUTOTUNE = [16, 32, 64, 128]
_TRAIN_CHUNK = 64  # tokens per CTA in the forward (reported as BT)


def custom_device_ctx(index: int):
    return torch.cuda.device(index)


def input_guard(fn=None, *, no_guard_contiguous=False):
    """Make tensor arguments contiguous and run under the first tensor's
    device (greta/dynamic_conv.py:44-96)."""

    def decorator(fn):
        names = list(inspect.signature(fn).parameters.keys())
        skip = set(no_guard_contiguous) if isinstance(no_guard_contiguous, list) else set()

        def fix(name, v):
            if isinstance(v, torch.Tensor) and not (no_guard_contiguous is True or name in skip):
                return v.contiguous()
            return v

        @functools.wraps(fn)
        def wrapper(*args, **kwargs):
            args = [fix(names[i] if i < len(names) else f"__arg_{i}", a) for i, a in enumerate(args)]
            kwargs = {k: fix(k, v) for k, v in kwargs.items()}
            tensor = next((a for a in list(args) + list(kwargs.values()) if isinstance(a, torch.Tensor)), None)
            ctx = custom_device_ctx(tensor.device.index) if tensor is not None and tensor.is_cuda \
                else contextlib.nullcontext()
            with ctx:
                return fn(*args, **kwargs)

        return wrapper

    return decorator(fn) if fn is not None else decorator


def _check_group(G: int) -> None:
    """Group sizes the reference training/inference kernels accept
    (greta/dynamic_conv.py:136-155: G must divide one of BD_AUTOTUNE)."""
    if not any(bd % G == 0 for bd in BD_AUTOTUNE) or G <= 0:
        raise ValueError(
            f"group_size={G} must divide one of BD={BD_AUTOTUNE} "
            f"(i.e. be a power of two <= {max(BD_AUTOTUNE)}).")


def _check_shapes(x, weight, gate, group_size):
    """greta/dynamic_conv.py:768-783."""
    if x.dim() != 3:
        raise ValueError(f"x must be [1, T, D], got {tuple(x.shape)}")
    B, T, D = x.shape
    if B != 1:
        raise ValueError("the packed dynamic-convolution training kernel requires physical batch size B=1")
    if D % group_size != 0:
        raise ValueError(f"group_size={group_size} must divide D={D}")
    DC = D // group_size
    if weight.dim() != 3 or weight.shape[0] != T or weight.shape[2] != DC:
        raise ValueError(
            f"weight must be [T, W, D // group_size] = [{T}, *, {DC}], got {tuple(weight.shape)}")
    if gate is not None and gate.shape != x.shape:
        raise ValueError(f"gate shape {tuple(gate.shape)} must match x {tuple(x.shape)}")
    return B, T, D, weight.shape[1]


def _check_inference_shapes(context, weight, gate, group_size):
    """greta/dynamic_conv.py:614-640."""
    if context.dim() != 3:
        raise ValueError(f"context must be [B, Q + W - 1, D], got {tuple(context.shape)}")
    if weight.dim() != 4:
        raise ValueError(f"weight must be [B, Q, W, D // group_size], got {tuple(weight.shape)}")
    batch_size, context_length, hidden_size = context.shape
    weight_batch, query_length, kernel_size, num_filters = weight.shape
    if batch_size != weight_batch:
        raise ValueError(f"context batch={batch_size} does not match weight batch={weight_batch}")
    if hidden_size % group_size != 0:
        raise ValueError(f"group_size={group_size} must divide hidden_size={hidden_size}")
    if num_filters != hidden_size // group_size:
        raise ValueError(
            f"weight has {num_filters} filters, expected hidden_size // group_size="
            f"{hidden_size // group_size}")
    if context_length != query_length + kernel_size - 1:
        raise ValueError(
            "context must contain exactly W-1 history tokens followed by the query chunk; "
            f"got context_length={context_length}, query_length={query_length}, kernel_size={kernel_size}")
    if gate is not None and gate.shape != (batch_size, query_length, hidden_size):
        raise ValueError(
            f"gate must be [{batch_size}, {query_length}, {hidden_size}], got {tuple(gate.shape)}")
    return batch_size, query_length, hidden_size, kernel_size


def _check_decode_shapes(x, weight, gate, conv_state, group_size):
    """greta/dynamic_conv.py:690-719."""
    if x.dim() != 2:
        raise ValueError(f"x must be [B, D], got {tuple(x.shape)}")
    if weight.dim() != 3:
        raise ValueError(f"weight must be [B, W, D // group_size], got {tuple(weight.shape)}")
    if conv_state.dim() != 3:
        raise ValueError(f"conv_state must be [B, D, W - 1], got {tuple(conv_state.shape)}")
    batch_size, hidden_size = x.shape
    weight_batch, kernel_size, num_filters = weight.shape
    if kernel_size < 2:
        raise ValueError("cached decode requires kernel_size >= 2")
    if weight_batch != batch_size:
        raise ValueError(f"x batch={batch_size} does not match weight batch={weight_batch}")
    if hidden_size % group_size != 0:
        raise ValueError(f"group_size={group_size} must divide hidden_size={hidden_size}")
    if num_filters != hidden_size // group_size:
        raise ValueError(f"weight has {num_filters} filters, expected {hidden_size // group_size}")
    expected_state = (batch_size, hidden_size, kernel_size - 1)
    if tuple(conv_state.shape) != expected_state:
        raise ValueError(f"conv_state must be {expected_state}, got {tuple(conv_state.shape)}")
    if gate is not None and gate.shape != x.shape:
        raise ValueError(f"gate shape {tuple(gate.shape)} must match x {tuple(x.shape)}")
    if 128 % group_size != 0:
        raise ValueError(f"cached decode currently requires group_size to divide 128, got {group_size}")
    return batch_size, hidden_size, kernel_size


def _as(t: Optional[torch.Tensor], dtype: torch.dtype) -> Optional[torch.Tensor]:
    if t is None:
        return None
    return (t if t.dtype == dtype else t.to(dtype)).contiguous()


def _flat3(x, gate):
    if x.dim() > 3:
        x = x.flatten(2)
        if gate is not None and gate.dim() > 3:
            gate = gate.flatten(2)
    return x, gate


def _cu(cu_seqlens, device):
    if cu_seqlens is None:
        return None, 0, 0
    cu = cu_seqlens.to(device=device)
    if cu.dtype not in (torch.int32, torch.int64):
        cu = cu.to(torch.int64)
    cu = cu.contiguous()
    return cu, int(cu.dtype == torch.int64), cu.numel() - 1


def dynconv_fwd(
    x: torch.Tensor,
    weight: torch.Tensor,
    gate: Optional[torch.Tensor],
    cu_seqlens: Optional[torch.Tensor],
    group_size: int,
    norm: bool = False,
    eps: float = 1e-6,
    save_pre: bool = False,
    BT: Optional[int] = None,
    chunk_indices: Optional[torch.Tensor] = None,
    cu_seqlens_cpu: Optional[torch.Tensor] = None,
):
    """Returns (y, yr, BT, chunk_indices) like greta/dynamic_conv.py:786-823;
    chunk_indices is None (sequences are resolved on the device)."""
    shape_x = x.shape
    x, gate = _flat3(x, gate)
    B, T, D, W = _check_shapes(x, weight, gate, group_size)
    _check_group(group_size)
    if not x.is_cuda:
        raise ValueError("dynamic_causal_conv1d requires CUDA tensors")
    x = x.contiguous()
    wk = _as(weight, x.dtype)
    gk = _as(gate, x.dtype)
    y = torch.empty_like(x)
    yr = torch.empty_like(x) if (norm and save_pre) else None
    cu, cu64, nseq = _cu(cu_seqlens, x.device)
    with custom_device_ctx(x.device.index):
        st = _capi.lib().greta_dynconv_fwd_ex(
            _capi.dtype_code(x), _capi.ptr(x), _capi.ptr(wk), _capi.ptr(gk), _capi.ptr(y), _capi.ptr(yr),
            _capi.ptr(cu), cu64, nseq, T, D, W, group_size, _capi.NORM_PLAIN if norm else _capi.NORM_NONE,
            float(eps), _capi.stream_of(x), _capi.options())
    _capi.check("greta_dynconv_fwd", st)
    return y.view(shape_x), yr, (BT if BT is not None else _TRAIN_CHUNK), None


def dynconv_bwd(
    x: torch.Tensor,
    weight: torch.Tensor,
    gate: Optional[torch.Tensor],
    yr: Optional[torch.Tensor],
    dout: torch.Tensor,
    cu_seqlens: Optional[torch.Tensor],
    group_size: int,
    norm: bool,
    eps: float,
    BT: int,
    chunk_indices: Optional[torch.Tensor],
):
    """Returns (dx, dw, dg) like greta/dynamic_conv.py:826-864."""
    shape_x = x.shape
    if x.dim() > 3:
        x = x.flatten(2)
        dout = dout.flatten(2)
        if gate is not None and gate.dim() > 3:
            gate = gate.flatten(2)
    B, T, D, W = _check_shapes(x, weight, gate, group_size)
    if norm and yr is None:
        raise RuntimeError("norm=True backward requires the saved pre-norm output")
    _check_group(group_size)
    if not x.is_cuda:
        raise ValueError("dynamic_causal_conv1d requires CUDA tensors")
    x = x.contiguous()
    dt = x.dtype
    wk, gk, yk, dk = _as(weight, dt), _as(gate, dt), _as(yr, dt), _as(dout, dt)
    dx = torch.empty_like(x)
    dw = torch.empty_like(wk)
    dg = torch.empty_like(gk) if gk is not None else None
    cu, cu64, nseq = _cu(cu_seqlens, x.device)
    with custom_device_ctx(x.device.index):
        st = _capi.lib().greta_dynconv_bwd_ex(
            _capi.dtype_code(x), _capi.ptr(x), _capi.ptr(wk), _capi.ptr(gk), _capi.ptr(yk if norm else None),
            _capi.ptr(dk), _capi.ptr(dx), _capi.ptr(dw), _capi.ptr(dg), _capi.ptr(cu), cu64, nseq, T, D, W,
            group_size, _capi.NORM_PLAIN if norm else _capi.NORM_NONE, float(eps), _capi.stream_of(x),
            _capi.options())
    _capi.check("greta_dynconv_bwd", st)
    if dw.dtype != weight.dtype:
        dw = dw.to(weight.dtype)
    if dg is not None and dg.dtype != gate.dtype:
        dg = dg.to(gate.dtype)
    return dx.view(shape_x), dw, dg


class DynamicCausalConv1dFunction(torch.autograd.Function):
    """greta/dynamic_conv.py:867-893 on the B200 kernels."""

    @staticmethod
    @input_guard
    def forward(ctx, x, weight, gate, cu_seqlens, group_size, norm, eps, cu_seqlens_cpu=None):
        y, yr, BT, chunk_indices = dynconv_fwd(
            x, weight, gate, cu_seqlens, group_size, norm=norm, eps=eps, save_pre=True,
            cu_seqlens_cpu=cu_seqlens_cpu)
        ctx.save_for_backward(x, weight, gate, yr)
        ctx.cu_seqlens = cu_seqlens
        ctx.chunk_indices = chunk_indices
        ctx.BT = BT
        ctx.group_size = group_size
        ctx.norm = norm
        ctx.eps = eps
        return y

    @staticmethod
    @input_guard
    def backward(ctx, dout):
        x, weight, gate, yr = ctx.saved_tensors
        dx, dw, dg = dynconv_bwd(x, weight, gate, yr, dout, ctx.cu_seqlens, ctx.group_size, ctx.norm, ctx.eps,
                                 ctx.BT, ctx.chunk_indices)
        return dx, dw, dg, None, None, None, None, None


@torch.compiler.disable(recursive=True)
def dynamic_causal_conv1d(
    x: torch.Tensor,
    weight: torch.Tensor,
    gate: Optional[torch.Tensor] = None,
    cu_seqlens: Optional[torch.Tensor] = None,
    group_size: int = 1,
    norm: bool = False,
    norm_eps: float = 1e-6,
    cu_seqlens_cpu: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """
    x:      [1, T, D]
    weight: [T, W, D // group_size]   (tap-major, compact; channel j uses filter j // group_size)
    gate:   [1, T, D] or None
    norm:   per-group (G channels) weightless RMSNorm on the conv output, before the gate

    out = RMSNorm_group(conv(x, w)) * silu(gate)      (greta/dynamic_conv.py:896-931)
    """
    needs_grad = torch.is_grad_enabled() and (
        x.requires_grad or weight.requires_grad or (gate is not None and gate.requires_grad))
    if needs_grad:
        return DynamicCausalConv1dFunction.apply(x, weight, gate, cu_seqlens, group_size, norm, norm_eps,
                                                 cu_seqlens_cpu)
    ctx = custom_device_ctx(x.device.index) if x.is_cuda else contextlib.nullcontext()
    with ctx:
        y, _, _, _ = dynconv_fwd(
            x.contiguous(), weight.contiguous(), gate.contiguous() if gate is not None else None,
            cu_seqlens, group_size, norm=norm, eps=norm_eps, save_pre=False, cu_seqlens_cpu=cu_seqlens_cpu)
    return y


@torch.compiler.disable(recursive=True)
def dynamic_causal_conv1d_inference(
    context: torch.Tensor,
    weight: torch.Tensor,
    gate: Optional[torch.Tensor] = None,
    group_size: int = 1,
    norm: bool = False,
    norm_eps: float = 1e-6,
) -> torch.Tensor:
    """Batched forward-only dynamic convolution for Hugging Face inference.

    `context` contains `W - 1` left-context tokens followed by the `Q` query tokens
    (greta/dynamic_conv.py:643-687).
    """
    if not context.is_cuda or not weight.is_cuda or (gate is not None and not gate.is_cuda):
        raise ValueError("dynamic_causal_conv1d_inference requires CUDA tensors")
    context = context.contiguous()
    weight = weight.contiguous()
    gate = gate.contiguous() if gate is not None else None
    B, Q, D, W = _check_inference_shapes(context, weight, gate, group_size)
    if Q == 0:
        return context.new_empty((B, 0, D))
    _check_group(group_size)
    wk, gk = _as(weight, context.dtype), _as(gate, context.dtype)
    y = context.new_empty((B, Q, D))
    with custom_device_ctx(context.device.index):
        st = _capi.lib().greta_dynconv_inference_ex(
            _capi.dtype_code(context), _capi.ptr(context), _capi.ptr(wk), _capi.ptr(gk), _capi.ptr(y), B, Q, D, W,
            group_size, _capi.NORM_PLAIN if norm else _capi.NORM_NONE, float(norm_eps),
            _capi.stream_of(context), _capi.options())
    _capi.check("greta_dynconv_inference", st)
    return y


@torch.compiler.disable(recursive=True)
def dynamic_causal_conv1d_decode(
    x: torch.Tensor,
    weight: torch.Tensor,
    conv_state: torch.Tensor,
    gate: Optional[torch.Tensor] = None,
    group_size: int = 1,
    norm: bool = False,
    norm_eps: float = 1e-6,
) -> torch.Tensor:
    """Single-token cached decode with an in-place fixed-size convolution state update.

    `x` is the current projected token `[B, D]`; `conv_state` contains the previous
    `W - 1` projected inputs in chronological order and is updated in-place
    (greta/dynamic_conv.py:722-765).
    """
    if not x.is_cuda or not weight.is_cuda or not conv_state.is_cuda or (gate is not None and not gate.is_cuda):
        raise ValueError("dynamic_causal_conv1d_decode requires CUDA tensors")
    x = x.contiguous()
    weight = weight.contiguous()
    gate = gate.contiguous() if gate is not None else None
    if not conv_state.is_contiguous():
        raise ValueError("conv_state must be contiguous because it is updated in-place")
    B, D, W = _check_decode_shapes(x, weight, gate, conv_state, group_size)
    if conv_state.dtype != x.dtype:
        raise ValueError(f"conv_state dtype {conv_state.dtype} must match x dtype {x.dtype}")
    wk, gk = _as(weight, x.dtype), _as(gate, x.dtype)
    y = torch.empty_like(x)
    with custom_device_ctx(x.device.index):
        st = _capi.lib().greta_dynconv_decode_rows_ex(
            _capi.dtype_code(x), _capi.ptr(x), _capi.ptr(wk), _capi.ptr(gk), _capi.ptr(conv_state), _capi.ptr(y),
            B, D, W, group_size, _capi.NORM_PLAIN if norm else _capi.NORM_NONE, float(norm_eps),
            _capi.stream_of(x), _capi.options())
    _capi.check("greta_dynconv_decode_rows", st)
    return y


@torch.compiler.disable(recursive=True)
def dynamic_causal_conv1d_prefill_with_state(
    x: torch.Tensor,
    weight: torch.Tensor,
    conv_state: torch.Tensor,
    has_previous: bool,
    gate: Optional[torch.Tensor] = None,
    group_size: int = 1,
    norm: bool = False,
    norm_eps: float = 1e-6,
) -> torch.Tensor:
    """HF prefill chunk with a channel-first conv state, in one launch.

    The reference does this in two steps: GretaDynamicCache.update_conv_inputs
    (greta/modeling_greta.py:214-248) transposes the chunk to channel-first,
    concatenates it with the cached state into [B, D, W-1+Q], keeps the last
    W-1 columns as the new state and transposes the concatenation back into a
    [B, Q+W-1, D] context, which dynamic_causal_conv1d_inference
    (greta/dynamic_conv.py:643-687) then convolves. Here the kernel reads the
    history of each batch row straight from conv_state (when has_previous;
    zeros otherwise) and writes the row's last W-1 inputs back into it, bit
    for bit: the same outputs (the same plain group RMS norm as the inference
    kernel) and the same new state, with no context tensor.

    x: [B, Q, D]; weight: [B, Q, W, D // group_size]; gate: [B, Q, D] or None;
    conv_state: [B, D, W-1], contiguous, updated in place. Returns [B, Q, D].
    """
    for t in (x, weight, conv_state, gate):
        if t is not None and not t.is_cuda:
            raise ValueError("dynamic_causal_conv1d_prefill_with_state requires CUDA tensors")
    if x.ndim != 3 or weight.ndim != 4:
        raise ValueError(f"x must be [B, Q, D] and weight [B, Q, W, D // group_size], got "
                         f"{tuple(x.shape)} and {tuple(weight.shape)}")
    B, Q, D = x.shape
    W = weight.shape[2]
    _check_group(group_size)
    if D % group_size != 0 or tuple(weight.shape) != (B, Q, W, D // group_size):
        raise ValueError(f"weight must be [B, Q, W, D // group_size], got {tuple(weight.shape)}")
    if W < 2:
        raise ValueError("a conv state needs kernel_size >= 2")
    if tuple(conv_state.shape) != (B, D, W - 1):
        raise ValueError(f"conv_state must be {(B, D, W - 1)}, got {tuple(conv_state.shape)}")
    if not conv_state.is_contiguous():
        raise ValueError("conv_state must be contiguous because it is updated in-place")
    if conv_state.dtype != x.dtype:
        raise ValueError(f"conv_state dtype {conv_state.dtype} must match x dtype {x.dtype}")
    if gate is not None and tuple(gate.shape) != (B, Q, D):
        raise ValueError(f"gate shape {tuple(gate.shape)} must match x {tuple(x.shape)}")
    y = torch.empty_like(x)
    if B == 0 or Q == 0:
        return y
    # each batch row is one request of Q tokens whose cache slot is its state row
    xk = x.contiguous().view(B * Q, D)
    wk = _as(weight, x.dtype).contiguous().view(B * Q, W, D // group_size)
    gk = None if gate is None else _as(gate, x.dtype).contiguous().view(B * Q, D)
    dev = x.device
    starts = torch.arange(0, B * Q + 1, Q, dtype=torch.int32, device=dev)
    slots = torch.arange(B, dtype=torch.int32, device=dev)
    init = torch.full((B,), 1 if has_previous else 0, dtype=torch.int8, device=dev)
    s_slot, s_d, s_h = conv_state.stride()
    with custom_device_ctx(dev.index):
        st = _capi.lib().greta_dynconv_packed_state_ex(
            _capi.dtype_code(x), _capi.ptr(xk), _capi.ptr(wk), _capi.ptr(gk), _capi.ptr(y), _capi.ptr(conv_state), B,
            s_slot, s_d, s_h, _capi.ptr(starts), _capi.ptr(slots), _capi.ptr(init), B, B * Q, D, W, group_size,
            _capi.NORM_PLAIN if norm else _capi.NORM_NONE, float(norm_eps), None, _capi.stream_of(x),
            _capi.options())
    _capi.check("greta_dynconv_packed_state", st)
    return y


def triton_dynamic_causal_conv1d_autograd_from_context(
    context: torch.Tensor,
    weights: torch.Tensor,
    gate: Optional[torch.Tensor],
    group_size: int,
    norm: bool,
    eps: float,
) -> torch.Tensor:
    """HF autograd path from an explicit context, as ONE packed call.

    Same signature, result and gradients as the reference's
    triton_dynamic_causal_conv1d_autograd_from_context
    (greta/modeling_greta.py:378-414), which runs the training kernel once per
    batch row on that row's context ([Q + W - 1] rows, weights and gate
    zero-padded over the W - 1 history rows) and keeps the last Q outputs.
    Here the B context rows are packed into one stream of B sequences of
    L = Q + W - 1 tokens (cu_seqlens = 0, L, 2L, ...): each sequence starts
    with zero history, exactly like the per-row calls, so one forward and one
    backward launch replace B of each.

    context: [B, Q + W - 1, D]; weights: [B, Q, W, D // group_size];
    gate: [B, Q, D] or None. Returns [B, Q, D].
    """
    B, Q, W, F = weights.shape
    L = context.shape[1]
    if context.ndim != 3 or context.shape[0] != B or L < Q:
        raise ValueError(
            f"context {tuple(context.shape)} must be [B, Q + W - 1, D] for weights {tuple(weights.shape)}")
    H = L - Q  # history rows of each context row (W - 1)
    D = context.shape[2]
    # zero filters (and gates) on the history rows, as the per-row padding does
    w_full = torch.nn.functional.pad(weights, (0, 0, 0, 0, H, 0)).reshape(B * L, W, F)
    g_full = None
    if gate is not None:
        g_full = torch.nn.functional.pad(gate, (0, 0, H, 0)).reshape(1, B * L, D)
    cu = torch.arange(0, B * L + 1, L, dtype=torch.int32, device=context.device)
    out = dynamic_causal_conv1d(context.reshape(1, B * L, D), w_full, g_full, cu, group_size, norm, eps)
    return out.view(B, L, D)[:, H:]


__all__ = [
    "dynamic_causal_conv1d_prefill_with_state",
    "triton_dynamic_causal_conv1d_autograd_from_context",
    "dynamic_causal_conv1d",
    "dynamic_causal_conv1d_decode",
    "dynamic_causal_conv1d_inference",
    "DynamicCausalConv1dFunction",
    "dynconv_fwd",
    "dynconv_bwd",
]
