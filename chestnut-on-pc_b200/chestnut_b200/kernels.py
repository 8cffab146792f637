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


def warp_frames(frame, big_frame, tfm, big_tfm, width, height, stride, y_height, uv_height, out,
                model_w=512, model_h=256, stream=None):
    """Road + wide NV12 frames (device pointers) -> model input u8[2,6,model_h/2,model_w/2]
    at device pointer out.  tfm / big_tfm: 3x3 inverse transforms (anything numpy
    turns into 9 float32 values, row-major)."""
    import numpy as np
    m0 = np.ascontiguousarray(np.asarray(tfm, np.float32).reshape(9))
    m1 = np.ascontiguousarray(np.asarray(big_tfm, np.float32).reshape(9))
    check(lib().cn_warp_frames(frame, big_frame, m0.ctypes.data, m1.ctypes.data, width, height, stride, y_height,
                               uv_height, model_w, model_h, out, stream), "cn_warp_frames")


def synchronize(device=0):
    check(lib().cn_device_synchronize(device), "cn_device_synchronize")


def device_error():
    import ctypes
    c = ctypes.c_int(0)
    check(lib().cn_device_error(ctypes.byref(c)), "cn_device_error")
    return c.value
