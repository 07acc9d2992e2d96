"""C ABI without a GPU: the library loads, exports every entry point that
include/greta_dynconv.h declares, and rejects bad arguments before touching
CUDA (no kernel is launched in this file)."""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "greta_dynconv.h"


@pytest.fixture(scope="module")
def lib():
    from greta_plugin_b200 import _capi

    return _capi.lib()


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"GRETA_API\s+[\w\s\*]+?\b(greta_dynconv_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared_symbols()
    for n in ("greta_dynconv_fwd", "greta_dynconv_bwd", "greta_dynconv_inference", "greta_dynconv_decode_rows",
              "greta_dynconv_packed_state", "greta_dynconv_supports", "greta_dynconv_status_string",
              "greta_dynconv_version"):
        assert n in names


def test_library_exports_every_declared_symbol(lib):
    for name in declared_symbols():
        assert hasattr(lib, name), f"{name} declared in {HEADER.name} but not exported"


def test_status_strings_and_version(lib):
    from greta_plugin_b200 import _capi

    for code in range(5):
        assert lib.greta_dynconv_status_string(code)
    assert b"unknown" in lib.greta_dynconv_status_string(99)
    assert _capi.version() == 10000


def test_supports_mirrors_reference_rule(lib):
    from greta_plugin_b200 import supports

    for g, d, want in [(1, 4096, True), (128, 2048, True), (256, 4096, True), (3, 48, False), (0, 64, False),
                       (512, 4096, False), (16, 40, False), (64, 64, True)]:
        assert bool(lib.greta_dynconv_supports(g, d)) == want
        assert supports(g, d) == want


P = ctypes.c_void_p
FAKE = P(0x1000)  # never dereferenced: validation fails before any use


def test_fwd_rejects_bad_arguments(lib):
    from greta_plugin_b200 import _capi as C

    f = lib.greta_dynconv_fwd
    # null tensors with work to do
    assert f(C.DT_BF16, None, FAKE, None, FAKE, None, None, 0, 0, 10, 64, 4, 1, 0, 1e-6, None) == C.ERR_INVALID_ARG
    # group size not a power of two / too large, kernel size too large, dtype, norm kind
    assert f(C.DT_BF16, FAKE, FAKE, None, FAKE, None, None, 0, 0, 10, 96, 4, 3, 0, 1e-6, None) == C.ERR_UNSUPPORTED
    assert f(C.DT_BF16, FAKE, FAKE, None, FAKE, None, None, 0, 0, 10, 1024, 4, 512, 0, 1e-6, None) == \
        C.ERR_UNSUPPORTED
    assert f(C.DT_BF16, FAKE, FAKE, None, FAKE, None, None, 0, 0, 10, 64, 17, 1, 0, 1e-6, None) == C.ERR_UNSUPPORTED
    assert f(7, FAKE, FAKE, None, FAKE, None, None, 0, 0, 10, 64, 4, 1, 0, 1e-6, None) == C.ERR_UNSUPPORTED
    assert f(C.DT_BF16, FAKE, FAKE, None, FAKE, None, None, 0, 0, 10, 64, 4, 1, 9, 1e-6, None) == C.ERR_UNSUPPORTED
    # G must divide D
    assert f(C.DT_BF16, FAKE, FAKE, None, FAKE, None, None, 0, 0, 10, 60, 4, 8, 0, 1e-6, None) == C.ERR_INVALID_ARG
    # empty work is a no-op, even with null pointers
    assert f(C.DT_BF16, None, None, None, None, None, None, 0, 0, 0, 64, 4, 1, 0, 1e-6, None) == C.OK


def test_bwd_rejects_bad_arguments(lib):
    from greta_plugin_b200 import _capi as C

    f = lib.greta_dynconv_bwd
    # stable norm has no backward; norm needs yr; gate and dg come together
    assert f(C.DT_BF16, FAKE, FAKE, None, None, FAKE, FAKE, FAKE, None, None, 0, 0, 10, 64, 4, 1, 2, 1e-6,
             None) == C.ERR_UNSUPPORTED
    assert f(C.DT_BF16, FAKE, FAKE, None, None, FAKE, FAKE, FAKE, None, None, 0, 0, 10, 64, 4, 1, 1, 1e-6,
             None) == C.ERR_INVALID_ARG
    assert f(C.DT_BF16, FAKE, FAKE, FAKE, None, FAKE, FAKE, FAKE, None, None, 0, 0, 10, 64, 4, 1, 0, 1e-6,
             None) == C.ERR_INVALID_ARG


def test_decode_and_packed_reject_bad_arguments(lib):
    from greta_plugin_b200 import _capi as C

    d = lib.greta_dynconv_decode_rows
    assert d(C.DT_BF16, FAKE, FAKE, None, FAKE, FAKE, 4, 64, 1, 1, 0, 1e-6, None) == C.ERR_INVALID_ARG  # W < 2
    assert d(C.DT_BF16, FAKE, FAKE, None, None, FAKE, 4, 64, 4, 1, 0, 1e-6, None) == C.ERR_INVALID_ARG
    assert d(C.DT_BF16, None, None, None, None, None, 0, 64, 4, 1, 0, 1e-6, None) == C.OK
    p = lib.greta_dynconv_packed_state
    # missing metadata
    assert p(C.DT_BF16, FAKE, FAKE, None, FAKE, FAKE, 8, 192, 3, 1, None, FAKE, FAKE, 2, 5, 64, 4, 1, 2, 1e-6, None,
             None) == C.ERR_INVALID_ARG
    # a state cache is required when W > 1 and there are slots
    assert p(C.DT_BF16, FAKE, FAKE, None, FAKE, None, 8, 192, 3, 1, FAKE, FAKE, FAKE, 2, 5, 64, 4, 1, 2, 1e-6, None,
             None) == C.ERR_INVALID_ARG
    # T == 0 returns at once (greta_vllm/triton_conv.py:142-143)
    assert p(C.DT_BF16, None, None, None, None, None, 8, 192, 3, 1, None, None, None, 2, 0, 64, 4, 1, 2, 1e-6, None,
             None) == C.OK


def test_launch_shape_knob_validates(lib):
    from greta_plugin_b200 import _capi as C

    s = lib.greta_dynconv_set_launch_shape
    assert s(99, 32, 4, 8) == C.ERR_INVALID_ARG
    assert s(C.PATH_FWD, 48, 4, 8) == C.ERR_INVALID_ARG  # not a multiple of 32
    assert s(C.PATH_FWD, 128, 4, 8) == C.ERR_INVALID_ARG  # more than 256 threads
    assert s(C.PATH_DECODE_ROWS, 64, 2, 1) == C.ERR_INVALID_ARG
    assert s(C.PATH_FWD, 64, 2, 8) == C.OK
    assert s(C.PATH_FWD, 0, 0, 0) == C.OK  # restore
