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


def reference_available():
    return Path(os.environ.get("GRETA_REFERENCE", "/root/reference")).is_dir()
