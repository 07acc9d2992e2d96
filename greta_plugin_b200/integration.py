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

import importlib

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


def install_hf() -> list[str]:
    """Route the HF Transformers plugin's conv calls to the B200 kernels."""
    done = _rebind("greta.dynamic_conv", DYNAMIC_CONV_NAMES)
    done += _rebind("greta.modeling_greta", HF_GLOBALS)
    return done


def install_vllm() -> list[str]:
    """Route the vLLM plugin's packed conv to the B200 kernel."""
    done = []
    for module_name, names in VLLM_NAMES.items():
        done += _rebind(module_name, names)
    return done


def register() -> None:
    """vLLM general-plugin entry point: reference registration + B200 kernels."""
    import greta_vllm

    greta_vllm.register()
    install_vllm()
    install_hf()
