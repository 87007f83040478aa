"""Build the sm_100a C-ABI library ``libb200packed.so`` in-tree with nvcc.

Every ``*.cu`` file in this directory is compiled in parallel to an object under
``_build/`` at the repository root and linked into ``tinygrad_dx12_b200/libb200packed.so``.
Rebuilds only what changed (source or header newer than its object).
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import pathlib
import shutil
import subprocess
import sys

HERE = pathlib.Path(__file__).resolve().parent
PKG = HERE.parent
ROOT = PKG.parent
BUILD = ROOT / "_build"
LIB = PKG / "libb200packed.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
         "--expt-relaxed-constexpr", "-I", str(ROOT / "include")]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and pathlib.Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _compile(src: pathlib.Path, extra: list[str]) -> pathlib.Path:
    obj = BUILD / (src.stem + ".o")
    headers = list(HERE.glob("*.cuh")) + list(HERE.glob("*.h")) + list((ROOT / "include").glob("*.h"))
    newest = max([src.stat().st_mtime] + [h.stat().st_mtime for h in headers])
    if obj.exists() and obj.stat().st_mtime >= newest and not extra:
        return obj
    cmd = [nvcc(), *ARCH, *FLAGS, *extra, "-c", str(src), "-o", str(obj)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    if res.stderr.strip():
        sys.stderr.write(res.stderr)
    return obj


def build(verbose: bool = False, extra: list[str] | None = None) -> pathlib.Path:
    BUILD.mkdir(exist_ok=True)
    sources = sorted(HERE.glob("*.cu"))
    extra = list(extra or [])
    with cf.ThreadPoolExecutor(max_workers=min(8, len(sources))) as ex:
        objs = list(ex.map(lambda s: _compile(s, extra), sources))
    if LIB.exists() and all(LIB.stat().st_mtime >= o.stat().st_mtime for o in objs) and not extra:
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-lcuda"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB)
    if verbose:
        print(f"built {LIB}")
    return LIB


if __name__ == "__main__":
    extra = sys.argv[1:]
    build(verbose=True, extra=extra)
