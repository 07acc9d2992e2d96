"""CPU oracle for the dynamic causal depthwise convolution -- TEST INFRASTRUCTURE.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline arm may use
this module, and only as the checker or the timed CPU baseline; the product
path never imports it.

It wraps oracle/_build/libdynconv_oracle.so (built from dynconv_oracle.c by
oracle/Makefile), a double-precision restatement of the reference's
algorithms:

  fwd          greta/dynamic_conv.py:937-962  torch_dynamic_causal_conv1d
               (+ the pre-norm save of dynconv_fwd_kernel, :247-249)
  bwd          greta/dynamic_conv.py:319-428  dynconv_bwd_kernel math
  inference    greta/dynamic_conv.py:467-506  dynconv_inference_kernel
  decode_rows  greta/dynamic_conv.py:536-602  dynconv_decode_kernel
  packed       greta_vllm/triton_conv.py:41-116 (_conv_kernel + _state_kernel)

Parity is pinned: tests/test_oracle_golden.py checks every function against
golden vectors produced by the reference itself (tests/golden/make_golden.py).

All inputs are numpy arrays (any float dtype; converted to fp32), outputs are
fp32 numpy arrays. Norm kinds: 0 none, 1 plain, 2 stable.
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "libdynconv_oracle.so"

NORM_NONE, NORM_PLAIN, NORM_STABLE = 0, 1, 2

_lib = None


def build() -> Path:
    """Compile the C restatement (make -C oracle)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def _load():
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        build()
    lib = ctypes.CDLL(str(LIB_PATH))
    P = ctypes.c_void_p
    I = ctypes.c_int64
    lib.oracle_fwd.argtypes = [P, P, P, P, I, I, I, I, I, ctypes.c_int, ctypes.c_double, P, P, ctypes.c_int]
    lib.oracle_bwd.argtypes = [P, P, P, P, P, P, I, I, I, I, I, ctypes.c_int, ctypes.c_double, P, P, P,
                               ctypes.c_int]
    lib.oracle_inference.argtypes = [P, P, P, I, I, I, I, I, ctypes.c_int, ctypes.c_double, P, ctypes.c_int]
    lib.oracle_decode_rows.argtypes = [P, P, P, P, I, I, I, I, ctypes.c_int, ctypes.c_double, P, ctypes.c_int]
    lib.oracle_packed.argtypes = [P, P, P, P, I, I, I, I, P, P, P, I, I, I, I, I, ctypes.c_int, ctypes.c_double,
                                  P, ctypes.c_int]
    lib.oracle_max_threads.restype = ctypes.c_int
    _lib = lib
    return lib


def max_threads() -> int:
    return int(_load().oracle_max_threads())


def _f32(a):
    if a is None:
        return None
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def _i64(a):
    if a is None:
        return None
    return np.ascontiguousarray(np.asarray(a, dtype=np.int64))


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def fwd(x, w, gate, cu_seqlens, group_size, norm=NORM_NONE, eps=1e-6, save_pre=False, threads=0):
    """x [T, D], w [T, W, D/G], gate [T, D] or None, cu_seqlens [N+1] or None.

    Returns (y, yr); yr is the pre-norm output when save_pre and norm != 0."""
    x, w, gate, cu = _f32(x), _f32(w), _f32(gate), _i64(cu_seqlens)
    T, D = x.shape
    W = w.shape[1]
    y = np.zeros((T, D), np.float32)
    yr = np.zeros((T, D), np.float32) if (save_pre and norm) else None
    nseq = 0 if cu is None else cu.shape[0] - 1
    _load().oracle_fwd(_p(x), _p(w), _p(gate), _p(cu), nseq, T, D, W, group_size, norm, eps, _p(y), _p(yr),
                       threads)
    return y, yr


def bwd(x, w, gate, dout, cu_seqlens, group_size, norm=NORM_NONE, eps=1e-6, yr=None, threads=0):
    """Returns (dx [T, D], dw [T, W, D/G], dg [T, D] or None).

    yr: the pre-norm output as saved by the forward (I/O precision), which the
    reference backward kernel reads; None recomputes it in double precision."""
    x, w, gate, dout, cu, yr = _f32(x), _f32(w), _f32(gate), _f32(dout), _i64(cu_seqlens), _f32(yr)
    T, D = x.shape
    W = w.shape[1]
    dx = np.zeros((T, D), np.float32)
    dw = np.zeros(w.shape, np.float32)
    dg = np.zeros((T, D), np.float32) if gate is not None else None
    nseq = 0 if cu is None else cu.shape[0] - 1
    _load().oracle_bwd(_p(x), _p(w), _p(gate), _p(dout), _p(yr), _p(cu), nseq, T, D, W, group_size, norm, eps,
                       _p(dx), _p(dw), _p(dg), threads)
    return dx, dw, dg


def inference(context, w, gate, group_size, norm=NORM_NONE, eps=1e-6, threads=0):
    """context [B, Q+W-1, D], w [B, Q, W, D/G], gate [B, Q, D] -> y [B, Q, D]."""
    ctx, w, gate = _f32(context), _f32(w), _f32(gate)
    B, Q, W, _ = w.shape
    D = ctx.shape[2]
    y = np.zeros((B, Q, D), np.float32)
    _load().oracle_inference(_p(ctx), _p(w), _p(gate), B, Q, D, W, group_size, norm, eps, _p(y), threads)
    return y


def decode_rows(x, w, gate, state, group_size, norm=NORM_NONE, eps=1e-6, threads=0):
    """x [B, D], w [B, W, D/G], state [B, D, W-1] -> (y [B, D], new state)."""
    x, w, gate = _f32(x), _f32(w), _f32(gate)
    st = np.array(state, dtype=np.float32, copy=True, order="C")
    B, D = x.shape
    W = w.shape[1]
    y = np.zeros((B, D), np.float32)
    _load().oracle_decode_rows(_p(x), _p(w), _p(gate), _p(st), B, D, W, group_size, norm, eps, _p(y), threads)
    return y, st


def packed(x, w, gate, state, starts, slots, has_initial, group_size, norm=NORM_STABLE, eps=1e-6,
           state_strides=None, threads=0):
    """vLLM packed batch. state is a [slots, D, W-1] array (copied); when
    state_strides (element strides of a [slots, D, W-1] view) are given, state
    must be the flat backing storage. Returns (y [T, D], new state)."""
    x, w, gate = _f32(x), _f32(w), _f32(gate)
    starts, slots, init = _i64(starts), _i64(slots), _i64(has_initial)
    T, D = x.shape
    W = w.shape[1]
    st = np.array(state, dtype=np.float32, copy=True, order="C")
    if state_strides is None:
        num_slots = st.shape[0] if st.ndim == 3 else 0
        s_slot, s_d, s_h = D * (W - 1), W - 1, 1
    else:
        s_slot, s_d, s_h = state_strides
        num_slots = st.size // s_slot if s_slot else 0
    y = np.zeros((T, D), np.float32)
    N = slots.shape[0]
    _load().oracle_packed(_p(x), _p(w), _p(gate), _p(st) if st.size else None, num_slots, s_slot, s_d, s_h,
                          _p(starts), _p(slots), _p(init), N, T, D, W, group_size, norm, eps, _p(y), threads)
    return y, st


__all__ = ["fwd", "bwd", "inference", "decode_rows", "packed", "build", "max_threads", "NORM_NONE", "NORM_PLAIN",
           "NORM_STABLE", "LIB_PATH"]
