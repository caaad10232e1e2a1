"""Build recipe of the C oracle (test infrastructure only; see oracle/__init__.py):
oracle/hsd_oracle.c -> oracle/_build/liboracle.so (gcc, OpenMP, x86-64-v3).

The reference has no C, C++ or CUDA code (its kernels are Metal Shading Language strings
JIT-compiled by MLX on Apple silicon), so there is no oracle/_ref build: the C file here is
this repository's restatement of the reference's algorithm.
"""
import ctypes
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "hsd_oracle.c")
OUT_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(OUT_DIR, "liboracle.so")


def build(force=False):
    os.makedirs(OUT_DIR, exist_ok=True)
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < os.path.getmtime(SRC):
        cmd = ["gcc", "-O3", "-march=x86-64-v3", "-fopenmp", "-fPIC", "-shared", SRC, "-o", LIB]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"oracle build failed:\n{r.stderr}")
    return LIB


_lib = None


def load():
    """The C oracle library (built on demand)."""
    global _lib
    if _lib is None:
        L = ctypes.CDLL(build())
        P, I, Q = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64
        L.oracle_nibble_transpose.argtypes = [P, P, Q, Q, Q]
        L.oracle_sparse_down.argtypes = [P] * 10 + [I] * 7
        L.oracle_dense_down.argtypes = [P] * 10 + [I] * 6
        for f in (L.oracle_nibble_transpose, L.oracle_sparse_down, L.oracle_dense_down):
            f.restype = None
        _lib = L
    return _lib


if __name__ == "__main__":
    print(build(force=True))
