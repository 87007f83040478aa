"""Build the oracle's C restatement (``cpu_ref.c``) into ``oracle/libpackedref.so``.

TEST INFRASTRUCTURE ONLY. The reference itself (tinygrad-dx12) is Python over an
un-vendored tinygrad and has no C/C++ sources, so there is no ``oracle/_ref`` build:
only this restatement is compiled.
"""

from __future__ import annotations

import pathlib
import subprocess

HERE = pathlib.Path(__file__).resolve().parent
SRC = HERE / "cpu_ref.c"
LIB = HERE / "libpackedref.so"


def build(verbose: bool = False) -> pathlib.Path:
    if LIB.exists() and LIB.stat().st_mtime >= SRC.stat().st_mtime:
        return LIB
    cmd = ["gcc", "-O3", "-march=x86-64-v2", "-fopenmp", "-fPIC", "-shared", "-o", str(LIB), str(SRC), "-lm"]
    subprocess.run(cmd, check=True)
    if verbose:
        print(f"built {LIB}")
    return LIB


def load():
    import ctypes

    lib = ctypes.CDLL(str(build()))
    P, I64, I32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
    lib.oref_dequant_f32.argtypes = [P, I64, I32, I64, I64, P, I32, I64, P]
    lib.oref_linear.argtypes = [P, I64, I32, I64, I64, P, I32, I64, P, I32, I64, P, I32]
    lib.oref_max_threads.restype = I32
    return lib


if __name__ == "__main__":
    build(verbose=True)
