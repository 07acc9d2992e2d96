"""Helpers shared by the GPU parity tests (inputs, tolerances, oracle glue)."""
import numpy as np
import torch

DEV = "cuda"

# Tolerance of the CUDA kernels against the fp32/fp64 reference math:
# 16-bit I/O: rtol = atol = 1e-2 (one rounding of the output to bf16/fp16);
# fp32 I/O: tight, the kernels accumulate in fp32 like the reference kernels.
TOL = {torch.bfloat16: dict(rtol=1e-2, atol=1e-2), torch.float16: dict(rtol=1e-2, atol=1e-2),
       torch.float32: dict(rtol=1e-4, atol=5e-5)}


def assert_close(got, ref, dtype, scale_atol=True):
    """got: torch tensor (any device); ref: numpy/torch fp32. The absolute
    tolerance scales with the reference's magnitude for group sums (dw)."""
    g = got.detach().float().cpu().numpy() if isinstance(got, torch.Tensor) else np.asarray(got, np.float32)
    r = ref.detach().float().cpu().numpy() if isinstance(ref, torch.Tensor) else np.asarray(ref, np.float32)
    tol = dict(TOL[dtype])
    if scale_atol:
        tol["atol"] = tol["atol"] * max(1.0, float(np.abs(r).max()) / 4.0)
    np.testing.assert_allclose(g, r, **tol)


def to_np(t):
    return None if t is None else t.detach().float().cpu().numpy()


def rand(gen, *shape, scale=1.0, dtype=torch.bfloat16):
    return (torch.randn(*shape, generator=gen) * scale).to(dtype)


def ragged_cu(lengths):
    return torch.tensor([0] + list(np.cumsum(lengths)), dtype=torch.int32)


def f32_to_bf16_bits(a):
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def bf16_bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)
