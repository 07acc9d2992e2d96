"""CPU oracle of the dynamic causal depthwise convolution (test infrastructure only)."""
