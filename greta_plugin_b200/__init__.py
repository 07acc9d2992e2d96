"""B200-native (sm_100a) Greta dynamic causal depthwise convolution.

Hand-written CUDA kernels behind a C ABI (include/greta_dynconv.h,
greta_plugin_b200/_lib/libgreta_dynconv.so), with drop-in Python entry points
that keep the reference plugin's signatures:

  greta_plugin_b200.dynamic_conv  -- greta/dynamic_conv.py (training autograd,
                                     HF inference from context, HF decode, HF
                                     prefill on the cache's own state)
  greta_plugin_b200.vllm_conv     -- greta_vllm/triton_conv.py (vLLM packed
                                     prefill/decode with cache-slot state)
  greta_plugin_b200.integration   -- installs them into the reference plugins
  greta_plugin_b200.sharding      -- channel sharding across GPUs (no collective)
"""
from .dynamic_conv import (  # noqa: F401
    DynamicCausalConv1dFunction,
    dynamic_causal_conv1d,
    dynamic_causal_conv1d_decode,
    dynamic_causal_conv1d_inference,
    dynamic_causal_conv1d_prefill_with_state,
    dynconv_bwd,
    dynconv_fwd,
)
from .vllm_conv import packed_dynamic_conv_triton, supports  # noqa: F401

__version__ = "0.2.0"
