"""Build and load the C oracle (test infrastructure; see oracle/__init__.py).

``build()`` compiles ``cref.c`` with gcc into ``oracle/libcref.so``.  The
reference itself (Python on a pinned tinygrad fork, no C/C++ sources) cannot
be compiled here, so there is no ``oracle/_ref`` build.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "cref.c")
LIB = os.path.join(HERE, "libcref.so")


def build(force=False):
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= os.path.getmtime(SRC):
        return LIB
    cmd = ["gcc", "-O3", "-march=x86-64-v2", "-fopenmp", "-ffp-contract=off", "-fPIC",
           "-shared", "-o", LIB, SRC, "-lm"]
    subprocess.run(cmd, check=True)
    return LIB


_lib = None


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(LIB)
        vp, l, i, f = ctypes.c_void_p, ctypes.c_long, ctypes.c_int, ctypes.c_float
        L.cref_gemm_chain.argtypes = [vp, vp, vp, l, l, l, i, i]
        L.cref_reduce.argtypes = [vp, vp, vp, l, l, i]
        L.cref_fill.argtypes = [ctypes.c_uint64, ctypes.c_uint64, l, f, vp, vp, i]
        L.cref_f16_to_f32.argtypes = [vp, vp, l, i]
        _lib = L
    return _lib


def nthreads():
    return os.cpu_count() or 1


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def gemm_chain(A, B, C, b_kmajor, threads=None):
    A = np.ascontiguousarray(A, np.float16)
    B = np.ascontiguousarray(B, np.float16)
    C = np.ascontiguousarray(C, np.float32).copy()
    M, K = A.shape
    N = B.shape[0] if b_kmajor else B.shape[1]
    lib().cref_gemm_chain(_p(A), _p(B), _p(C), M, N, K, int(b_kmajor), threads or nthreads())
    return C


def reduce_rows(x2d, w, threads=None):
    x2d = np.ascontiguousarray(x2d, np.float16)
    w = np.ascontiguousarray(w, np.float16).reshape(-1)
    rows, n = x2d.shape
    assert w.size == n
    out = np.zeros(rows, np.float32)
    lib().cref_reduce(_p(x2d), _p(w), _p(out), rows, n, threads or nthreads())
    return out


def fill(seed, tid, count, bound, f16=True, threads=None):
    out = np.empty(count, np.float16 if f16 else np.float32)
    if f16:
        lib().cref_fill(seed, tid, count, bound, _p(out), None, threads or nthreads())
    else:
        lib().cref_fill(seed, tid, count, bound, None, _p(out), threads or nthreads())
    return out
