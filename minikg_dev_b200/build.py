"""Builds the in-tree CUDA library ``_lib/libminikg_b200.so`` for sm_100a with nvcc.

    python -m minikg_dev_b200.build [--verbose-ptxas] [--force]

Each ``csrc/*.cu`` compiles to an object under ``_build/`` (skipped when newer than its
sources), then one shared library links them.  No JIT cache is involved: the ``.so``
lives next to the package so it travels with the source tree.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
BUILD = ROOT / "_build"
LIB_DIR = PKG / "_lib"
LIB = LIB_DIR / "libminikg_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
              "--expt-relaxed-constexpr", "-DNDEBUG"]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; the CUDA 12.9 toolkit is required to build minikg_b200")
    return cand


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _compile(src: Path, verbose_ptxas: bool) -> tuple[Path, str]:
    obj = BUILD / (src.stem + ".o")
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-I", str(INCLUDE), "-I", str(CSRC), "-c", str(src), "-o", str(obj)]
    if verbose_ptxas:
        cmd[1:1] = ["-Xptxas", "-v"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stderr}\n{res.stdout}")
    return obj, res.stderr


def build(force: bool = False, verbose_ptxas: bool = False, quiet: bool = True) -> Path:
    BUILD.mkdir(exist_ok=True)
    LIB_DIR.mkdir(exist_ok=True)
    srcs = sources()
    hdrs = headers()
    todo = [s for s in srcs if force or verbose_ptxas or _stale(BUILD / (s.stem + ".o"), [s, *hdrs])]
    logs = []
    if todo:
        with ThreadPoolExecutor(max_workers=min(8, len(todo))) as ex:
            for obj, log in ex.map(lambda s: _compile(s, verbose_ptxas), todo):
                logs.append((obj, log))
    objs = [BUILD / (s.stem + ".o") for s in srcs]
    if force or todo or _stale(LIB, objs):
        # shared cudart: in a torch process the already-loaded libcudart.so.12 is reused, so
        # the library sees torch's current device; the rpath covers loading it on its own
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "shared", "-o", str(LIB), *map(str, objs),
               "-Xlinker", "-rpath=/usr/local/cuda/lib64"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stderr}\n{res.stdout}")
    if not quiet or verbose_ptxas:
        for obj, log in logs:
            if log.strip():
                print(f"== {obj.name}\n{log}", file=sys.stderr)
    return LIB


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose-ptxas", action="store_true")
    a = ap.parse_args(argv)
    lib = build(force=a.force, verbose_ptxas=a.verbose_ptxas, quiet=False)
    print(lib)


if __name__ == "__main__":
    main()
