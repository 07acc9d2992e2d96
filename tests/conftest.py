"""Shared test configuration.

Markers:
  gpu  -- needs a CUDA device (B200, sm_100a). Everything else runs on CPU.
"""
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: requires a CUDA GPU (B200, sm_100a)")


@pytest.fixture(autouse=True)
def _no_device_errors(request):
    """After every GPU test: no kernel of the library recorded a device error
    (a pipeline wait that ran out). Tests that cause one on purpose clear it."""
    yield
    if request.node.get_closest_marker("gpu") is None:
        return
    import torch

    if not torch.cuda.is_available():
        return
    from greta_plugin_b200 import _capi

    bits = _capi.device_errors(clear=True)
    assert bits == 0, f"a kernel recorded device error bits {bits:#x}"


@pytest.fixture(scope="session")
def golden_dir():
    return GOLDEN


def load_golden(name):
    import numpy as np

    with np.load(GOLDEN / f"{name}.npz") as z:
        return {k: z[k] for k in z.files}


def bf16_bits_to_f32(bits):
    """uint16 bf16 bit patterns -> float32 numpy array (exact)."""
    import numpy as np

    return (bits.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(a):
    """float32 -> bf16 bits with round-to-nearest-even (numpy; matches torch)."""
    import numpy as np

    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return r


# The unmodified reference (Garbo-AI/greta-plugin) as installed into
# baseline/_ref by `pip install --target baseline/_ref <checkout>`; the
# GRETA_REFERENCE environment variable may point at another installed copy.
REFERENCE_DIR = Path(os.environ.get("GRETA_REFERENCE") or (ROOT / "baseline" / "_ref"))


def reference_available():
    return (REFERENCE_DIR / "greta" / "dynamic_conv.py").is_file() and (REFERENCE_DIR / "greta_vllm").is_dir()


def import_reference_path():
    """Put the installed reference on sys.path (tests that use it skip without it)."""
    if not reference_available():
        pytest.skip(f"the reference is not installed at {REFERENCE_DIR}")
    if str(REFERENCE_DIR) not in sys.path:
        sys.path.insert(0, str(REFERENCE_DIR))
