"""Build libgreta_dynconv.so in-tree (greta_plugin_b200/_lib/) with nvcc for sm_100a.

Each .cu under csrc/ is compiled to an object in parallel, then linked into one
shared library exposing the C ABI declared in include/greta_dynconv.h. The
library links the shared CUDA runtime, so inside a PyTorch process it uses the
same runtime instance (and therefore the same current device) as torch.

Usage: python -m greta_plugin_b200.build [--force] [--verbose-ptxas]
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
LIBDIR = PKG / "_lib"
BUILDDIR = PKG / "_build"
LIBNAME = "libgreta_dynconv.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "--cudart",
    "shared",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build the kernels")
    return cand


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _compile(src: Path, verbose_ptxas: bool) -> tuple[Path, str]:
    obj = BUILDDIR / (src.stem + ".o")
    cmd = [nvcc(), *ARCH_FLAGS, *COMMON_FLAGS, f"-I{INCLUDE}", f"-I{CSRC}", "-c", str(src), "-o", str(obj)]
    if verbose_ptxas:
        cmd += ["-Xptxas", "-v"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    return obj, res.stderr


def build(force: bool = False, verbose_ptxas: bool = False, quiet: bool = True) -> Path:
    """Compile every csrc/*.cu and link the shared library; returns its path."""
    LIBDIR.mkdir(exist_ok=True)
    BUILDDIR.mkdir(exist_ok=True)
    lib = LIBDIR / LIBNAME
    sources = sorted(CSRC.glob("*.cu"))
    headers = _headers()
    todo = [s for s in sources if force or verbose_ptxas or _stale(BUILDDIR / (s.stem + ".o"), [s, *headers])]
    logs = []
    if todo:
        workers = min(len(todo), os.cpu_count() or 1)
        with cf.ThreadPoolExecutor(workers) as ex:
            for obj, log in ex.map(lambda s: _compile(s, verbose_ptxas), todo):
                logs.append((obj, log))
    objs = [BUILDDIR / (s.stem + ".o") for s in sources]
    if todo or _stale(lib, objs):
        tmp = lib.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH_FLAGS, "--cudart", "shared", "-shared", *map(str, objs), "-o", str(tmp),
               "-Xlinker", "-rpath,/usr/local/cuda/lib64"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, lib)
    if not quiet or verbose_ptxas:
        for obj, log in logs:
            if log.strip():
                print(f"== {obj.name}\n{log}", file=sys.stderr)
    return lib


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose-ptxas", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose_ptxas=a.verbose_ptxas, quiet=False))


if __name__ == "__main__":
    main()
