"""ctypes binding of libgreta_dynconv.so (the C ABI in include/greta_dynconv.h).

The library is built in-tree (python -m greta_plugin_b200.build). There is no
fallback: if the library is missing or a call fails, an exception is raised.
"""
from __future__ import annotations

import contextlib
import ctypes
import os
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libgreta_dynconv.so"

DT_F32, DT_F16, DT_BF16 = 0, 1, 2
NORM_NONE, NORM_PLAIN, NORM_STABLE = 0, 1, 2
OK, ERR_INVALID_ARG, ERR_UNSUPPORTED, ERR_ALIGNMENT, ERR_LAUNCH = 0, 1, 2, 3, 4

_DTYPES = {torch.float32: DT_F32, torch.float16: DT_F16, torch.bfloat16: DT_BF16}

_lib = None


class Options(ctypes.Structure):
    """greta_dynconv_options: per-call launch choices of the `_ex` entry points."""
    _fields_ = [("size", ctypes.c_int), ("kernel", ctypes.c_int), ("block_x", ctypes.c_int),
                ("block_y", ctypes.c_int), ("tokens", ctypes.c_int), ("wait_limit_log2", ctypes.c_int),
                ("test_withhold_release", ctypes.c_int), ("rows_channels", ctypes.c_int),
                ("rows_ranges", ctypes.c_int), ("rows_smem_kb", ctypes.c_int)]


_local = threading.local()


KERNELS = {"auto": 0, "register": 1, "rows": 2}  # GRETA_KERNEL_*


@contextlib.contextmanager
def launch_options(kernel="auto", block_x=0, block_y=0, tokens=0, wait_limit_log2=0, test_withhold_release=False,
                   rows_channels=0, rows_ranges=0, rows_smem_kb=0):
    """Launch choices for the C-ABI calls this thread makes inside the block
    (tests and tuning sweeps): the kernel family ("auto", "register", "rows"
    for the row-streaming bulk-copy kernels), the register kernels' CTA
    shape, the pipeline wait bound, the row-streaming kernels' channel slice,
    token ranges and stage-ring budget. They
    travel with each call as its options argument; nothing is set in the
    library."""
    o = Options(ctypes.sizeof(Options), KERNELS[kernel], block_x, block_y, tokens, wait_limit_log2,
                int(bool(test_withhold_release)), rows_channels, rows_ranges, rows_smem_kb)
    prev = getattr(_local, "opts", None)
    _local.opts = o
    try:
        yield o
    finally:
        _local.opts = prev


def options():
    """The options of the enclosing launch_options block (None = defaults)."""
    o = getattr(_local, "opts", None)
    return None if o is None else ctypes.byref(o)


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
    sig = {
        "fwd": [I32, P, P, P, P, P, P, I32, I64, I64, I64, I64, I64, I32, F, P],
        "bwd": [I32, P, P, P, P, P, P, P, P, P, I32, I64, I64, I64, I64, I64, I32, F, P],
        "inference": [I32, P, P, P, P, I64, I64, I64, I64, I64, I32, F, P],
        "decode_rows": [I32, P, P, P, P, P, I64, I64, I64, I64, I32, F, P],
        "packed_state": [I32, P, P, P, P, P, I64, I64, I64, I64, P, P, P, I64, I64, I64, I64, I64, I32, F, P, P],
    }
    for name, args in sig.items():
        getattr(L, f"greta_dynconv_{name}").argtypes = args
        getattr(L, f"greta_dynconv_{name}_ex").argtypes = args + [P]
        getattr(L, f"greta_dynconv_{name}").restype = I32
        getattr(L, f"greta_dynconv_{name}_ex").restype = I32
    # packed_state with row strides: x, ldx, w, ldw, gate, ldg, then as packed_state from y on
    L.greta_dynconv_packed_state_ld_ex.argtypes = [I32, P, I64, P, I64, P, I64] + sig["packed_state"][4:] + [P]
    L.greta_dynconv_packed_state_ld_ex.restype = I32
    L.greta_dynconv_fwd_ld_ex.argtypes = [I32, P, I64, P, I64, P, I64, P, P, P, I32, I64, I64, I64, I64, I64, I32,
                                          F, P, P]
    L.greta_dynconv_fwd_ld_ex.restype = I32
    L.greta_dynconv_bwd_ld_ex.argtypes = [I32, P, I64, P, I64, P, I64, P, P, P, I64, P, I64, P, I64, P, I32, I64,
                                          I64, I64, I64, I64, I32, F, P, P]
    L.greta_dynconv_bwd_ld_ex.restype = I32
    L.greta_dynconv_supports.argtypes = [I64, I64]
    L.greta_dynconv_device_errors.argtypes = [I32]
    L.greta_dynconv_status_string.argtypes = [I32]
    L.greta_dynconv_status_string.restype = ctypes.c_char_p
    L.greta_dynconv_version.restype = I32
    for name in ("supports", "device_errors"):
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


ERR_BIT_TIMEOUT = 2  # a pipeline wait of a row-streaming kernel ran out


def check_device_errors(fn: str) -> None:
    """Raise GretaKernelError when an earlier kernel on the current device
    recorded an error (clears the bits; synchronises the device)."""
    bits = device_errors(clear=True)
    if bits < 0:
        raise GretaKernelError(fn, ERR_LAUNCH, "the device error word could not be read")
    if bits & ERR_BIT_TIMEOUT:
        raise GretaKernelError(fn, ERR_LAUNCH, "a pipeline wait timed out; the kernel returned with its outputs "
                               "partly unwritten")


def device_errors(clear: bool = True) -> int:
    """Device-side error bits of earlier kernels (synchronises the device)."""
    return int(lib().greta_dynconv_device_errors(1 if clear else 0))


def version() -> int:
    return int(lib().greta_dynconv_version())


def loaded_path() -> str:
    lib()
    return os.fspath(LIB_PATH)
