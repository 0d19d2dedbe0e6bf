"""Build libexl3b200.so (the C ABI in include/exl3_b200.h) from csrc/*.cu for sm_100a.

    python -m omlx_exl3_b200.build [--force] [--verbose]

Every translation unit is compiled by nvcc with `-gencode arch=compute_100a,code=sm_100a` (the
architecture-specific target: tcgen05 / TMA instructions need the `a` variant), objects go to
omlx_exl3_b200/_build/, and the shared library is linked in-tree next to this file so that it
travels with the repository snapshot. nvcc cross-compiles; no GPU is needed to build.
"""
from __future__ import annotations

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
LIB = PKG / "libexl3b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
              "-Xcompiler", "-fvisibility=hidden", "-DEXL3_BUILD"]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    return cand


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _deps() -> list[Path]:
    return sources() + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in _deps())


def _compile(src: Path, verbose: bool) -> Path:
    obj = BUILD / (src.stem + ".o")
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, f"-I{INCLUDE}", f"-I{CSRC}", "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
    if verbose and r.stderr:
        print(r.stderr, flush=True)
    return obj


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile (when sources changed) and return the path of libexl3b200.so."""
    if not force and up_to_date():
        return LIB
    BUILD.mkdir(exist_ok=True)
    srcs = sources()
    with ThreadPoolExecutor(max_workers=max(1, min(len(srcs), os.cpu_count() or 4))) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), srcs))
    tmp = LIB.with_suffix(f".so.{os.getpid()}.tmp")
    cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-lcudart"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="--verbose" in sys.argv))
