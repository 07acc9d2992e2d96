"""Helpers that drive the UNMODIFIED reference (Garbo-AI/greta-plugin, installed
into baseline/_ref) through its own dispatch code, with the B200 kernels
installed by greta_plugin_b200.integration or with the reference's own paths.

Test infrastructure only. Two gaps between the reference's pinned
dependencies and this image are bridged here, and nothing else:

* transformers: the reference pins 5.17 (pyproject.toml:10) and its
  GretaDynamicCache (greta/modeling_greta.py:179-248) inherits that version's
  multi-state linear-attention cache API (`number_of_states`,
  `has_previous_state(layer_idx, state_idx)`,
  `update_conv_state(states, layer_idx, state_idx, conv_kernel_size)`), which
  the installed transformers 5.5 does not have. `ConvCache517` supplies those
  three methods with the semantics the reference's callers rely on
  (modeling_greta.py:214-248: the first update stores the last W-1 inputs;
  later updates return the old state followed by the new inputs,
  [B, D, W-1+Q], and keep its last W-1 columns), so that the reference's own
  update_conv_inputs / get_conv_state_for_decode / GretaDynamicConv.forward
  run unchanged on top of it. tests/test_reference_dispatch_cpu.py checks the
  stand-in against the cache-free forward of the same tokens.
* vLLM: the reference targets 0.30; 0.22 is installed. Its
  ShortConvAttentionMetadata has the fields metadata_to_batch reads, and
  GretaConv constructs with a minimal vllm_config; only the forward context is
  supplied here (get_forward_context patched in greta_vllm.model).
"""
from __future__ import annotations

import contextlib
import dataclasses
import types

import torch

from conftest import import_reference_path


def reference_modules(triton=True):
    """(greta.dynamic_conv, greta.modeling_greta, greta.configuration_greta) of
    the installed reference; skips the test when it (or Triton) is missing."""
    import pytest

    import_reference_path()
    try:
        import greta.configuration_greta as cg
        import greta.dynamic_conv as rdc
        import greta.modeling_greta as mg
    except ImportError as exc:  # Triton or transformers missing on this machine
        pytest.skip(f"the reference does not import here: {exc}")
    return rdc, mg, cg


def vllm_reference_modules():
    import pytest

    import_reference_path()
    try:
        import greta_vllm.conv as vconv
        import greta_vllm.model as vm
        import greta_vllm.triton_conv as vtc
    except Exception as exc:  # vLLM missing or incompatible
        pytest.skip(f"greta_vllm does not import here: {exc}")
    return vconv, vtc, vm


# ---------------------------------------------------------------------------
# install / restore the B200 kernels in the reference modules
# ---------------------------------------------------------------------------
@contextlib.contextmanager
def installed(hf=False, vllm=False):
    """Rebind the reference's kernel names to the B200 drop-ins (the way a user
    would, through greta_plugin_b200.integration) and restore them afterwards."""
    from greta_plugin_b200 import integration

    saved = []
    targets = []
    if hf:
        targets += [("greta.dynamic_conv", integration.DYNAMIC_CONV_NAMES),
                    ("greta.modeling_greta", integration.HF_GLOBALS)]
    if vllm:
        targets += list(integration.VLLM_NAMES.items())
    import importlib

    for mod_name, names in targets:
        mod = importlib.import_module(mod_name)
        for n in names:
            saved.append((mod, n, getattr(mod, n)))
    if hf:
        conv_cls = importlib.import_module("greta.modeling_greta").GretaDynamicConv
        saved.append((conv_cls, "forward", conv_cls.forward))
    try:
        if hf:
            integration.install_hf()
        if vllm:
            integration.install_vllm()
        yield
    finally:
        for mod, n, v in saved:
            setattr(mod, n, v)


# ---------------------------------------------------------------------------
# HF: the transformers-5.17 cache methods GretaDynamicCache relies on
# ---------------------------------------------------------------------------
def make_cache(mg, config):
    """A GretaDynamicCache (the reference class, so its isinstance checks and
    update_conv_inputs / get_conv_state_for_decode run as written) whose base
    methods follow transformers 5.17's linear-attention cache."""

    class ConvCache517(mg.GretaDynamicCache):
        def __init__(self, config):  # noqa: D401 -- 5.5's DynamicCache.__init__ cannot build these layers
            self.layers = []
            for layer_type in config.layer_types:
                if layer_type == "linear_attention":
                    layer = mg.GretaConvCacheLayer.__new__(mg.GretaConvCacheLayer)
                    layer.record_past = False
                    layer.number_of_states = 1
                    layer.conv_states = [None]
                    layer.recurrent_states = [None]
                    layer.is_conv_states_initialized = [False]
                    layer.is_recurrent_states_initialized = [False]
                    layer.previous = [False]
                    self.layers.append(layer)
                else:
                    self.layers.append(None)

        def has_previous_state(self, layer_idx=None, state_idx=0):
            layer = self.layers[layer_idx]
            return layer is not None and layer.previous[state_idx]

        def update_conv_state(self, conv_states, layer_idx, state_idx=0, conv_kernel_size=None):
            layer = self.layers[layer_idx]
            H = conv_kernel_size
            if not layer.previous[state_idx]:
                new = conv_states[..., -H:]
                if new.shape[-1] < H:
                    new = torch.nn.functional.pad(new, (H - new.shape[-1], 0))
                layer.conv_states[state_idx] = new.contiguous().clone()
                layer.is_conv_states_initialized[state_idx] = True
                layer.previous[state_idx] = True
                return layer.conv_states[state_idx]
            full = torch.cat((layer.conv_states[state_idx], conv_states), dim=-1)
            layer.conv_states[state_idx].copy_(full[..., -H:])
            return full

    return ConvCache517(config)


def conv_layer_index(config):
    return config.layer_types.index("linear_attention")


def greta_config(cg, **kw):
    """GretaConfig with overrides; a smaller hidden_dim also sets embedding_dim
    (the configuration requires them equal)."""
    if "hidden_dim" in kw:
        kw.setdefault("embedding_dim", kw["hidden_dim"])
    return cg.GretaConfig(**kw)


def make_hf_conv(mg, cg, dtype, device, seed, use_triton, **cfg_kwargs):
    """GretaDynamicConv at the configuration defaults (hidden 2048, kernel 7,
    128-channel groups, norm on) with seeded random weights."""
    cfg = greta_config(cg, **cfg_kwargs)
    cfg.use_triton_kernels = use_triton
    torch.manual_seed(seed)
    mod = mg.GretaDynamicConv(cfg, conv_layer_index(cfg)).to(device=device, dtype=dtype)
    return cfg, mod


# ---------------------------------------------------------------------------
# vLLM: SHORT_CONV metadata for a decodes-first mixed batch
# ---------------------------------------------------------------------------
def short_conv_metadata(vm, decode_slots, prefill_lens, prefill_slots, prefill_initial, device):
    """vLLM's ShortConvAttentionMetadata (the installed version's class) for a
    batch of one-token decodes followed by prefill chunks."""
    M = vm.ShortConvAttentionMetadata
    d, p = len(decode_slots), len(prefill_lens)
    qsl = torch.tensor([0] + list(torch.tensor(prefill_lens).cumsum(0).tolist()), dtype=torch.int32, device=device)
    fields = {f.name: None for f in dataclasses.fields(M)}
    fields.update(
        num_prefills=p, num_prefill_tokens=int(sum(prefill_lens)), num_decodes=d, num_decode_tokens=d,
        num_reqs=d + p,
        has_initial_states_p=torch.tensor(prefill_initial, dtype=torch.bool, device=device) if p else None,
        query_start_loc_p=qsl if p else None,
        state_indices_tensor_p=torch.tensor(prefill_slots, dtype=torch.int32, device=device) if p else None,
        state_indices_tensor_d=torch.tensor(decode_slots, dtype=torch.int32, device=device) if d else None,
        num_accepted_tokens=None)
    return M(**fields)


@contextlib.contextmanager
def forward_context(vm, layer, prefix, metadata):
    """greta_vllm.model.get_forward_context answering for one layer."""
    ctx = types.SimpleNamespace(attn_metadata=None if metadata is None else {prefix: metadata},
                                no_compile_layers={prefix: layer})
    saved = vm.get_forward_context
    vm.get_forward_context = lambda: ctx
    try:
        yield ctx
    finally:
        vm.get_forward_context = saved


def make_vllm_conv(vm, cg, dtype, device, seed, n_slots, prefix="model.layers.0.conv", **cfg_kwargs):
    """GretaConv (greta_vllm/model.py:85-163) with seeded weights and a conv
    cache of n_slots in vLLM's layout for this build (is_conv_state_dim_first:
    [slots, D, W-1], else [slots, W-1, D])."""
    cfg = greta_config(cg, **cfg_kwargs)
    vcfg = types.SimpleNamespace(compilation_config=types.SimpleNamespace(static_forward_context={}))
    torch.manual_seed(seed)
    layer = vm.GretaConv(cfg, vcfg, prefix).to(device=device, dtype=dtype)
    D, H = cfg.hidden_dim, cfg.kernel_size - 1
    g = torch.Generator().manual_seed(seed + 1)
    if vm.is_conv_state_dim_first():
        state = torch.randn(n_slots, D, H, generator=g)
    else:
        state = torch.randn(n_slots, H, D, generator=g)
    layer.kv_cache = (state.to(device=device, dtype=dtype),)
    return cfg, layer, prefix
