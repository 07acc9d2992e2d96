"""ctypes binding of libgreta_dynconv.so (the C ABI in include/greta_dynconv.h).

The library is built in-tree (python -m greta_plugin_b200.build). There is no
fallback: if the library is missing or a call fails, an exception is raised.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libgreta_dynconv.so"

DT_F32, DT_F16, DT_BF16 = 0, 1, 2
NORM_NONE, NORM_PLAIN, NORM_STABLE = 0, 1, 2
OK, ERR_INVALID_ARG, ERR_UNSUPPORTED, ERR_ALIGNMENT, ERR_LAUNCH = 0, 1, 2, 3, 4

_DTYPES = {torch.float32: DT_F32, torch.float16: DT_F16, torch.bfloat16: DT_BF16}

_lib = None


class GretaKernelError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, fn: str, status: int, msg: str):
        super().__init__(f"{fn} failed with status {status}: {msg}")
        self.status = status


def lib() -> ctypes.CDLL:
    """Load the shared library once (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise RuntimeError(
            f"{LIB_PATH} is missing: build the CUDA kernels with `python -m greta_plugin_b200.build` "
            "(there is no CPU or Triton fallback)")
    L = ctypes.CDLL(str(LIB_PATH))
    P, I64, I32, F = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float
    L.greta_dynconv_fwd.argtypes = [I32, P, P, P, P, P, P, I32, I64, I64, I64, I64, I64, I32, F, P]
    L.greta_dynconv_bwd.argtypes = [I32, P, P, P, P, P, P, P, P, P, I32, I64, I64, I64, I64, I64, I32, F, P]
    L.greta_dynconv_inference.argtypes = [I32, P, P, P, P, I64, I64, I64, I64, I64, I32, F, P]
    L.greta_dynconv_decode_rows.argtypes = [I32, P, P, P, P, P, I64, I64, I64, I64, I32, F, P]
    L.greta_dynconv_packed_state.argtypes = [I32, P, P, P, P, P, I64, I64, I64, I64, P, P, P, I64, I64, I64, I64,
                                             I64, I32, F, P, P]
    L.greta_dynconv_supports.argtypes = [I64, I64]
    L.greta_dynconv_set_launch_shape.argtypes = [I32, I32, I32, I32]
    L.greta_dynconv_set_tma.argtypes = [I32]
    L.greta_dynconv_device_errors.argtypes = [I32]
    L.greta_dynconv_status_string.argtypes = [I32]
    L.greta_dynconv_status_string.restype = ctypes.c_char_p
    L.greta_dynconv_version.restype = I32
    for name in ("fwd", "bwd", "inference", "decode_rows", "packed_state", "supports", "set_launch_shape", "set_tma",
                 "device_errors"):
        getattr(L, f"greta_dynconv_{name}").restype = I32
    _lib = L
    return L


def dtype_code(t: torch.Tensor) -> int:
    try:
        return _DTYPES[t.dtype]
    except KeyError:
        raise ValueError(f"unsupported dtype {t.dtype}; expected float32, float16 or bfloat16") from None


def ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_of(t: torch.Tensor):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def check(fn: str, status: int) -> None:
    if status != OK:
        msg = lib().greta_dynconv_status_string(status).decode()
        if status in (ERR_INVALID_ARG, ERR_UNSUPPORTED, ERR_ALIGNMENT):
            raise ValueError(f"{fn}: {msg}")
        raise GretaKernelError(fn, status, msg)


PATH_FWD, PATH_BWD, PATH_INFERENCE, PATH_DECODE_ROWS, PATH_PACKED_PREFILL, PATH_PACKED_DECODE = range(6)


def set_launch_shape(path: int, block_x: int = 0, block_y: int = 0, tokens: int = 0) -> None:
    """Override (or, with zeros, restore) the CTA shape of one launch path."""
    check("greta_dynconv_set_launch_shape", lib().greta_dynconv_set_launch_shape(path, block_x, block_y, tokens))


def set_tma(enable: bool) -> None:
    """Use (default) or bypass the TMA-staged forward for long token streams."""
    lib().greta_dynconv_set_tma(1 if enable else 0)


def device_errors(clear: bool = True) -> int:
    """Device-side error bits of earlier kernels (synchronises the device)."""
    return int(lib().greta_dynconv_device_errors(1 if clear else 0))


def version() -> int:
    return int(lib().greta_dynconv_version())


def loaded_path() -> str:
    lib()
    return os.fspath(LIB_PATH)
