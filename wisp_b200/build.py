"""Build libwisp_b200.so in-tree for sm_100a (B200).

    python -m wisp_b200.build          # incremental
    python -m wisp_b200.build --clean

Every CUDA translation unit under wisp_b200/csrc is compiled with
``-gencode arch=compute_100a,code=sm_100a -lineinfo -O3`` into
``wisp_b200/_build`` and linked into ``wisp_b200/libwisp_b200.so``. The
library has no PyTorch dependency: its ABI is include/wisp_b200.h.
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
BUILD = PKG / "_build"
LIB = PKG / "libwisp_b200.so"

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    f"-I{INCLUDE}", f"-I{CSRC}",
]
HOST_CXX = "/usr/bin/g++" if Path("/usr/bin/g++").exists() else "g++"


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _headers() -> list[Path]:
    return sorted(list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h")))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _compile(src: Path, verbose: bool) -> Path:
    obj = BUILD / (src.stem + ".o")
    if not _stale(obj, [src] + _headers()):
        return obj
    cmd = [NVCC, *NVCC_FLAGS, "-ccbin", HOST_CXX, "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
    if verbose and r.stderr:
        print(r.stderr, file=sys.stderr)
    return obj


def build(verbose: bool = False, clean: bool = False) -> Path:
    if clean and BUILD.exists():
        shutil.rmtree(BUILD)
    BUILD.mkdir(exist_ok=True)
    srcs = _sources()
    with ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), srcs))
    if _stale(LIB, objs):
        cmd = [NVCC, *ARCH, "-shared", "-ccbin", HOST_CXX, "-o", str(LIB), *map(str, objs),
               "-Xcompiler", "-fPIC"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


def reference_dir() -> Path | None:
    """The reference project's checkout: $WISP_REFERENCE_DIR, else a
    ``reference`` directory beside this repository; None when neither holds
    the reference's C engine."""
    cands = [os.environ.get("WISP_REFERENCE_DIR"), str(ROOT.parent / "reference")]
    for c in cands:
        if c and (Path(c) / "csrc" / "core" / "wisp_engine.c").exists():
            return Path(c)
    return None


def build_oracle() -> None:
    """Build the test-only oracle libraries (oracle/_ref). The reference CPU
    path is compiled only where the reference sources are present."""
    make = shutil.which("make") or "make"
    cmd = [make, "-C", str(ROOT / "oracle"), "all"]
    ref = reference_dir()
    if ref is not None:
        cmd.append(f"REF_DIR={ref}")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{r.stdout}\n{r.stderr}")


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--clean", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true", help="print ptxas resource usage")
    a = ap.parse_args()
    print(build(verbose=a.verbose, clean=a.clean))
