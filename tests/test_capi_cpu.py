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
    assert _capi.version() == 10100


SUPPORT_CASES = [(1, 4096, True), (128, 2048, True), (256, 4096, True), (3, 48, False), (0, 64, False),
                 (512, 4096, True), (1024, 2048, True), (4096, 4096, True), (8192, 4096, False), (16, 40, False),
                 (64, 64, True)]


def test_supports_mirrors_reference_rule(lib):
    """greta_vllm/triton_conv.py:119-121: any power-of-two G dividing D."""
    from greta_plugin_b200 import supports

    for g, d, want in SUPPORT_CASES:
        assert bool(lib.greta_dynconv_supports(g, d)) == want
        assert supports(g, d) == want


def test_supports_equals_the_installed_reference():
    import reference_harness as rh

    vconv, vtc, vm = rh.vllm_reference_modules()
    from greta_plugin_b200 import supports

    for g in [0, 1, 2, 3, 8, 96, 128, 256, 512, 1024, 2048, 4096, 8192]:
        for d in [64, 512, 2048, 4096, 6144]:
            assert supports(g, d) == bool(vtc.supports(g, d)), (g, d)


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


def test_launch_options_validate(lib):
    """The `_ex` entry points check their options before anything else; an
    empty launch (T = 0) with valid options returns OK without a GPU."""
    from greta_plugin_b200 import _capi as C

    def fwd(opt, T=0):
        return lib.greta_dynconv_fwd_ex(C.DT_BF16, FAKE, FAKE, None, FAKE, None, None, 0, 0, T, 256, 4, 1, 0, 1e-6,
                                        None, None if opt is None else ctypes.byref(opt))

    def opts(**kw):
        o = C.Options(ctypes.sizeof(C.Options), 0, 0, 0, 0, 0, 0)
        for k, v in kw.items():
            setattr(o, k, v)
        return o

    assert fwd(None) == C.OK
    assert fwd(opts()) == C.OK
    assert fwd(opts(size=4)) == C.ERR_INVALID_ARG  # wrong struct size
    assert fwd(opts(block_x=48, block_y=4, tokens=8)) == C.ERR_INVALID_ARG  # not a multiple of 32
    assert fwd(opts(block_x=128, block_y=4, tokens=8)) == C.ERR_INVALID_ARG  # more than 256 threads
    assert fwd(opts(wait_limit_log2=4)) == C.ERR_INVALID_ARG
    assert fwd(opts(wait_limit_log2=25)) == C.ERR_INVALID_ARG
    assert fwd(opts(kernel=3)) == C.ERR_INVALID_ARG
    assert fwd(opts(block_x=64, block_y=2, tokens=8, wait_limit_log2=12, kernel=1)) == C.OK
    # no process-wide knobs remain in the ABI
    for gone in ("greta_dynconv_set_tma", "greta_dynconv_set_launch_shape"):
        assert not hasattr(lib, gone)


def test_wide_groups_only_on_the_packed_entry_point(lib):
    from greta_plugin_b200 import _capi as C

    # G = 512 > 256: the training forward rejects it as unsupported ...
    assert lib.greta_dynconv_fwd(C.DT_BF16, FAKE, FAKE, None, FAKE, None, None, 0, 0, 5, 4096, 4, 512, 0, 1e-6,
                                 None) == C.ERR_UNSUPPORTED
    # ... the packed (vLLM) entry point takes any power of two dividing D
    assert lib.greta_dynconv_packed_state(C.DT_BF16, None, None, None, None, None, 8, 12288, 3, 1, None, None, None,
                                          2, 0, 4096, 4, 4096, 2, 1e-6, None, None) == C.OK
    assert lib.greta_dynconv_packed_state(C.DT_BF16, None, None, None, None, None, 8, 12288, 3, 1, None, None, None,
                                          2, 0, 4096, 4, 8192, 2, 1e-6, None, None) == C.ERR_INVALID_ARG
