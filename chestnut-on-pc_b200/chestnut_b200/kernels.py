"""Kernel-level entry points (device pointers), mirroring the reference's
per-kernel A/B harnesses (``bench_r62.py``, ``bench_alu.py``): the same
kernel launched on caller-provided buffers."""
from ._lib import check, lib


def gemm_wmma_f16(A, B, C, M, N, K, b_kmajor, bn=0, splits=0, stream=None):
    """C[M][N] += A[M][K] * B (device pointers); WMMA semantics D = C + A*B."""
    check(lib().cn_gemm_wmma_f16(A, B, C, M, N, K, int(b_kmajor), bn, splits, stream), "cn_gemm_wmma_f16")


def reduce_rows_f16(x, w, out, rows, length, chunks_per_row=0, stream=None):
    """out[r] = sum_i x[r][i] * w[i] (device pointers)."""
    check(lib().cn_reduce_rows_f16(x, w, out, rows, length, chunks_per_row, stream), "cn_reduce_rows_f16")


def border_gather_s2(act, G, B, H, W, C, out, stream=None):
    check(lib().cn_border_gather_s2(act, G, B, H, W, C, out, stream), "cn_border_gather_s2")


def synchronize(device=0):
    check(lib().cn_device_synchronize(device), "cn_device_synchronize")


def device_error():
    import ctypes
    c = ctypes.c_int(0)
    check(lib().cn_device_error(ctypes.byref(c)), "cn_device_error")
    return c.value
