"""Build libdkv_b200.so (sm_100a) in-tree with nvcc.

Each ``csrc/*.cu`` is compiled to an object under ``deltakv_b200/_build`` (skipped when
it is newer than its source and every header), then linked into
``deltakv_b200/libdkv_b200.so``.  ``python -m deltakv_b200.build`` rebuilds; ``--ptxas``
prints register / spill / shared-memory usage per kernel.
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
BUILD = PKG / "_build"
LIB = PKG / "libdkv_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put the CUDA toolkit on PATH")


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted((ROOT / "include").glob("*.h"))


def _flags() -> list[str]:
    return [
        *ARCH,
        "-O3",
        "-lineinfo",
        "-std=c++17",
        "-Xcompiler",
        "-fPIC",
        "-I",
        str(ROOT / "include"),
        "--expt-relaxed-constexpr",
    ]


def _compile(src: Path, ptxas: bool) -> tuple[Path, str]:
    obj = BUILD / (src.stem + ".o")
    newest_dep = max([src.stat().st_mtime] + [h.stat().st_mtime for h in _headers()])
    if not ptxas and obj.exists() and obj.stat().st_mtime >= newest_dep:
        return obj, ""
    cmd = [_nvcc(), *_flags(), "-c", str(src), "-o", str(obj)]
    if ptxas:
        cmd += ["-Xptxas", "-v"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    return obj, res.stderr


def build(ptxas: bool = False, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    with ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        results = list(ex.map(lambda s: _compile(s, ptxas), srcs))
    if ptxas or verbose:
        for _, log in results:
            if log:
                print(log, file=sys.stderr)
    objs = [o for o, _ in results]
    newest = max(o.stat().st_mtime for o in objs)
    if LIB.exists() and LIB.stat().st_mtime >= newest and not ptxas:
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [_nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    out = build(ptxas="--ptxas" in sys.argv, verbose=True)
    print(out)
