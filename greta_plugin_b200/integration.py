"""Install the B200 kernels into the reference plugins, leaving their dispatch
and state plumbing unchanged.

Hugging Face: greta/modeling_greta.py binds the Triton entry points to
module globals at import (modeling_greta.py:25-34) and GretaDynamicConv.forward
(:437-569) calls them; install_hf() rebinds those globals (and the names in
greta/dynamic_conv.py) to the functions of greta_plugin_b200.dynamic_conv, and
replaces the per-batch-row autograd helper (modeling_greta.py:378-414) with a
single packed call.

vLLM: GretaConv.run_conv (greta_vllm/model.py:142-163) calls
packed_dynamic_conv_triton when `triton_supports(G, D)` holds; install_vllm()
rebinds both names in greta_vllm.model and greta_vllm.triton_conv.

register() is a drop-in for the reference's vLLM general-plugin entry point
(greta_vllm/__init__.py:3-24): it runs the reference registration, then
installs the kernels. Point `vllm.general_plugins` at
`greta_plugin_b200.integration:register` instead of `greta_vllm:register`.
"""
from __future__ import annotations

import functools
import importlib

import torch

from . import dynamic_conv as _dc
from . import vllm_conv as _vc

HF_GLOBALS = {
    "_TRITON_DYNAMIC_CAUSAL_CONV1D": _dc.dynamic_causal_conv1d,
    "_TRITON_DYNAMIC_CAUSAL_CONV1D_DECODE": _dc.dynamic_causal_conv1d_decode,
    "_TRITON_DYNAMIC_CAUSAL_CONV1D_INFERENCE": _dc.dynamic_causal_conv1d_inference,
    # one packed call instead of the reference's loop over batch rows
    # (greta/modeling_greta.py:378-414)
    "triton_dynamic_causal_conv1d_autograd_from_context": _dc.triton_dynamic_causal_conv1d_autograd_from_context,
}

DYNAMIC_CONV_NAMES = {
    "dynamic_causal_conv1d": _dc.dynamic_causal_conv1d,
    "dynamic_causal_conv1d_decode": _dc.dynamic_causal_conv1d_decode,
    "dynamic_causal_conv1d_inference": _dc.dynamic_causal_conv1d_inference,
    "DynamicCausalConv1dFunction": _dc.DynamicCausalConv1dFunction,
    "dynconv_fwd": _dc.dynconv_fwd,
    "dynconv_bwd": _dc.dynconv_bwd,
}

VLLM_NAMES = {
    "greta_vllm.triton_conv": {"packed_dynamic_conv_triton": _vc.packed_dynamic_conv_triton,
                               "supports": _vc.supports},
    "greta_vllm.model": {"packed_dynamic_conv_triton": _vc.packed_dynamic_conv_triton,
                         "triton_supports": _vc.supports},
}


def _rebind(module_name: str, names: dict) -> list[str]:
    mod = importlib.import_module(module_name)
    done = []
    for name, fn in names.items():
        if not hasattr(mod, name):
            raise AttributeError(f"{module_name} has no attribute {name!r}; unexpected reference version")
        setattr(mod, name, fn)
        done.append(f"{module_name}.{name}")
    return done


def _live_conv_state(module, mg, hidden_states, past_key_values, use_cache):
    """The cache's conv state [B, D, W-1] for a prefill chunk that continues
    a cached sequence, when the reference would run the Triton inference
    kernel on it (GretaDynamicConv.forward, greta/modeling_greta.py:437-569:
    a cache with a previous state, several query tokens, no gradient, CUDA,
    use_triton_kernels); None otherwise."""
    if not (use_cache and isinstance(past_key_values, mg.GretaDynamicCache)):
        return None
    if hidden_states.ndim != 3 or hidden_states.shape[1] < 2 or not hidden_states.is_cuda:
        return None
    if module.kernel_size < 2 or not module.config.use_triton_kernels:
        return None
    if torch.is_grad_enabled() and (hidden_states.requires_grad or any(p.requires_grad for p in module.parameters())):
        return None
    state = past_key_values.get_conv_state_for_decode(module.layer_idx)
    if state is None or state.device != hidden_states.device or not state.is_contiguous():
        return None
    if state.dtype != module.in_proj.weight.dtype:
        return None
    return state


def _fused_cached_prefill(original):
    """GretaDynamicConv.forward in which a prefill chunk that continues a
    cached sequence runs as ONE launch (dynamic_causal_conv1d_prefill_with_state:
    history read from the channel-first cache state, the new last W-1 inputs
    written back into it) instead of the cache's transpose / concatenate /
    transpose context (greta/modeling_greta.py:229-247) followed by the
    inference kernel. Every other case runs the reference's own forward."""
    if getattr(original, "__greta_b200__", False):
        return original

    @functools.wraps(original)
    def forward(self, hidden_states, past_key_values=None, use_cache=False, attention_mask=None):
        import greta.modeling_greta as mg

        state = _live_conv_state(self, mg, hidden_states, past_key_values, use_cache)
        if state is None:
            return original(self, hidden_states, past_key_values=past_key_values, use_cache=use_cache,
                            attention_mask=attention_mask)
        # the projections of greta/modeling_greta.py:444-459
        batch_size, query_length, _ = hidden_states.shape
        if attention_mask is not None:
            if attention_mask.ndim != 2 or attention_mask.shape != (batch_size, query_length):
                raise ValueError("Convolution attention_mask must match [batch, query_length]")
            hidden_states = hidden_states.masked_fill(~attention_mask.bool().unsqueeze(-1), 0)
        weights = self.kernel_proj(hidden_states).view(batch_size, query_length, self.kernel_size,
                                                       self.num_filters)
        conv_inputs = self.in_proj(hidden_states)
        gate = self.gate_proj(hidden_states)
        output = _dc.dynamic_causal_conv1d_prefill_with_state(conv_inputs, weights.to(conv_inputs.dtype), state, True,
                                                              gate, self.group_size, self.norm, self.norm_eps)
        return self.out_proj(output)

    forward.__greta_b200__ = True
    return forward


def _fused_training_applies(module, hidden_states, past_key_values, use_cache):
    """The reference forward's autograd branch (greta/modeling_greta.py:517-552:
    no cache update, a gradient needed, CUDA, use_triton_kernels), with a group
    size its training kernel takes (greta/dynamic_conv.py:136-155: at most 128)."""
    if use_cache and past_key_values is not None:
        return False
    if hidden_states.ndim != 3 or not hidden_states.is_cuda or not module.config.use_triton_kernels:
        return False
    if not torch.is_grad_enabled() or not (hidden_states.requires_grad or
                                           any(p.requires_grad for p in module.parameters())):
        return False
    if module.kernel_proj.bias is None or module.group_size > 128:
        return False
    return hidden_states.dtype == module.in_proj.weight.dtype


def _fused_projection_training(original):
    """GretaDynamicConv.forward whose training branch computes in_proj,
    gate_proj and kernel_proj as ONE GEMM over their concatenated weights
    (fused_layer.FusedProjConvFunction: the conv reads x, gate and filters in
    place from that output, and its backward writes dx, dg and dw into one
    gradient buffer, so that the projections' backward is one GEMM for the
    hidden states' gradient and one for the weights'); the B batch rows run
    as one packed call of B sequences. Autograd splits the concatenated
    weights' gradient back into the module's own parameters. Every other case
    runs the forward it wraps."""
    if getattr(original, "__greta_b200_fused__", False):
        return original

    @functools.wraps(original)
    def forward(self, hidden_states, past_key_values=None, use_cache=False, attention_mask=None):
        if not _fused_training_applies(self, hidden_states, past_key_values, use_cache):
            return original(self, hidden_states, past_key_values=past_key_values, use_cache=use_cache,
                            attention_mask=attention_mask)
        from .fused_layer import FusedProjConvFunction

        B, Q, hidden = hidden_states.shape
        if attention_mask is not None:
            if attention_mask.ndim != 2 or attention_mask.shape != (B, Q):
                raise ValueError("Convolution attention_mask must match [batch, query_length]")
            hidden_states = hidden_states.masked_fill(~attention_mask.bool().unsqueeze(-1), 0)
        D, nk = self.in_proj.weight.shape[0], self.kernel_proj.weight.shape[0]
        pad = (2 * D + nk + 7) // 8 * 8 - (2 * D + nk)
        proj = torch.cat([self.in_proj.weight, self.gate_proj.weight, self.kernel_proj.weight,
                          self.in_proj.weight.new_zeros(pad, hidden)])
        cu = torch.arange(0, B * Q + 1, Q, dtype=torch.int32, device=hidden_states.device)
        y = FusedProjConvFunction.apply(hidden_states.reshape(B * Q, hidden), proj, self.kernel_proj.bias, cu, D,
                                        self.kernel_size, self.group_size, self.norm, self.norm_eps)
        return self.out_proj(y.view(B, Q, D))

    forward.__greta_b200_fused__ = True
    return forward


def install_hf(fused_cache_prefill: bool = True, fused_projection: bool = False) -> list[str]:
    """Route the HF Transformers plugin's conv calls to the B200 kernels.

    With fused_cache_prefill, GretaDynamicConv.forward is also wrapped so
    that a prefill chunk continuing a cached sequence is one launch on the
    cache's own state tensor (see _fused_cached_prefill). With
    fused_projection, its training branch computes the three input
    projections as one GEMM (see _fused_projection_training); its rounding
    then differs from three separate GEMMs' by the GEMM's summation order."""
    done = _rebind("greta.dynamic_conv", DYNAMIC_CONV_NAMES)
    done += _rebind("greta.modeling_greta", HF_GLOBALS)
    if fused_cache_prefill or fused_projection:
        mg = importlib.import_module("greta.modeling_greta")
        if not hasattr(mg, "GretaDynamicConv"):
            raise AttributeError("greta.modeling_greta has no attribute 'GretaDynamicConv'; "
                                 "unexpected reference version")
        if fused_cache_prefill:
            mg.GretaDynamicConv.forward = _fused_cached_prefill(mg.GretaDynamicConv.forward)
        if fused_projection:
            mg.GretaDynamicConv.forward = _fused_projection_training(mg.GretaDynamicConv.forward)
        done.append("greta.modeling_greta.GretaDynamicConv.forward")
    return done


def _concat_projection(layer):
    """[in_proj | gate_proj | kernel_proj | zero rows] of a GretaConv layer,
    rows padded to a multiple of 8 so that every row of the GEMM's output
    starts on a whole 8-element vector, and the matching bias (kernel_proj's;
    zeros elsewhere). Built once and rebuilt only when a weight changes."""
    params = (layer.in_proj.weight, layer.gate_proj.weight, layer.kernel_proj.weight, layer.kernel_proj.bias)
    key = tuple((t.data_ptr(), t._version) for t in params)
    cached = getattr(layer, "_b200_projection", None)
    if cached is not None and cached[0] == key:
        return cached[1], cached[2]
    D, nk = layer.in_proj.weight.shape[0], layer.kernel_proj.weight.shape[0]
    rows = (2 * D + nk + 7) // 8 * 8
    with torch.no_grad():
        w = layer.in_proj.weight.new_zeros(rows, layer.in_proj.weight.shape[1])
        w[:D] = layer.in_proj.weight
        w[D:2 * D] = layer.gate_proj.weight
        w[2 * D:2 * D + nk] = layer.kernel_proj.weight
        b = layer.kernel_proj.bias.new_zeros(rows)
        b[2 * D:2 * D + nk] = layer.kernel_proj.bias
    layer._b200_projection = (key, w, b)
    return w, b


def _fused_projection_forward(original):
    """GretaConv.forward (greta_vllm/model.py:115-124) with in_proj, gate_proj
    and kernel_proj as ONE GEMM over the concatenated weights; x, gate and the
    filters handed to the reference's own custom op (and from there to the
    B200 packed kernel) are column views of that one output, which the kernel
    reads in place through their row strides. Everything after the
    projections -- the op, run_conv, the cache plumbing, out_proj -- is the
    reference's."""
    if getattr(original, "__greta_b200__", False):
        return original

    @functools.wraps(original)
    def forward(self, hidden_states, positions):
        w, b = _concat_projection(self)
        n, D = hidden_states.shape[0], self.config.hidden_dim
        W, F = self.config.kernel_size, self.config.num_conv_filters
        cat = torch.nn.functional.linear(hidden_states, w, b)
        x, gate = cat[:, :D], cat[:, D:2 * D]
        weights = cat[:, 2 * D:2 * D + W * F].unflatten(1, (W, F))
        mixed = torch.empty((n, D), dtype=cat.dtype, device=cat.device)
        torch.ops.vllm.greta_dynamic_conv(x, weights, gate, positions, mixed, self.prefix)
        return self.out_proj(mixed)

    forward.__greta_b200__ = True
    return forward


def install_vllm(fused_projection: bool = False) -> list[str]:
    """Route the vLLM plugin's packed conv to the B200 kernel. With
    fused_projection, GretaConv.forward also computes its three input
    projections as one GEMM whose output the kernel reads in place
    (_fused_projection_forward); its rounding then differs from three
    separate GEMMs' by the GEMM's summation order."""
    done = []
    for module_name, names in VLLM_NAMES.items():
        done += _rebind(module_name, names)
    if fused_projection:
        vm = importlib.import_module("greta_vllm.model")
        if not hasattr(vm, "GretaConv"):
            raise AttributeError("greta_vllm.model has no attribute 'GretaConv'; unexpected reference version")
        vm.GretaConv.forward = _fused_projection_forward(vm.GretaConv.forward)
        done.append("greta_vllm.model.GretaConv.forward")
    return done


def register() -> None:
    """vLLM general-plugin entry point: reference registration + B200 kernels."""
    import greta_vllm

    greta_vllm.register()
    install_vllm()
    install_hf()
