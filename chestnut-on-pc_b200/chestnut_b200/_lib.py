"""ctypes binding of libchestnut.so (the C ABI declared in include/chestnut.h).

No PyTorch here: the engine's only compute path is the CUDA library.  If the
library is missing or cannot load, every call raises -- there is no CPU
fallback.
"""
import ctypes
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libchestnut.so")
HEADER = os.path.join(HERE, "..", "..", "include", "chestnut.h")

CN_MODEL_39M = 0
CN_MODEL_1B = 1
FRAME_BYTES = 2 * 6 * 128 * 256
PACKED = 524
N_OUT = 3323


class cn_config(ctypes.Structure):
    _fields_ = [("model", ctypes.c_int), ("device", ctypes.c_int), ("batch", ctypes.c_int),
                ("use_graph", ctypes.c_int), ("carry_hidden", ctypes.c_int), ("seed", ctypes.c_uint64)]


class cn_kernel_info(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 64), ("grid", ctypes.c_uint * 3), ("block", ctypes.c_uint * 3),
                ("cluster", ctypes.c_uint * 3), ("smem_bytes", ctypes.c_uint)]


class cn_slice(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 16), ("start", ctypes.c_int), ("stop", ctypes.c_int)]


class cn_decode_field(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_int), ("raw_off", ctypes.c_int), ("raw_len", ctypes.c_int), ("in_n", ctypes.c_int),
                ("out_n", ctypes.c_int), ("width", ctypes.c_int), ("out_off", ctypes.c_int)]


class ChestnutError(RuntimeError):
    pass


_vp, _i, _ll, _sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong, ctypes.c_size_t
_SIGS = {
    "cn_last_error": ([], ctypes.c_char_p),
    "cn_version": ([], _i),
    "cn_engine_create": ([ctypes.POINTER(cn_config), ctypes.POINTER(_vp)], _i),
    "cn_engine_destroy": ([_vp], _i),
    "cn_run_frame": ([_vp, _vp, _vp, _vp], _i),
    "cn_stage_input": ([_vp, _vp], _i),
    "cn_run_staged": ([_vp, _vp, _vp], _i),
    "cn_run_staged_async": ([_vp, _vp, _vp], _i),
    "cn_wait_output": ([_vp], _i),
    "cn_run_frames": ([_vp, _i, _vp, _vp, _vp], _i),
    "cn_run_frame_device": ([_vp, _vp, _vp], _i),
    "cn_read_output": ([_vp, _vp], _i),
    "cn_sync": ([_vp], _i),
    "cn_state_bytes": ([], _sz),
    "cn_get_state": ([_vp, _i, _vp, _sz], _i),
    "cn_set_state": ([_vp, _i, _vp, _sz], _i),
    "cn_reset_state": ([_vp], _i),
    "cn_kernel_list": ([_vp, ctypes.POINTER(cn_kernel_info), ctypes.POINTER(_i)], _i),
    "cn_profile_frame": ([_vp, _vp, _vp, ctypes.POINTER(ctypes.c_float), ctypes.POINTER(_i)], _i),
    "cn_set_timed_class": ([_vp, ctypes.c_char_p], _i),
    "cn_timed_class_ms": ([_vp, ctypes.POINTER(ctypes.c_float), ctypes.POINTER(_i)], _i),
    "cn_engine_info": ([_vp, ctypes.POINTER(_ll), ctypes.POINTER(_ll), ctypes.POINTER(_i)], _i),
    "cn_output_slices": ([ctypes.POINTER(cn_slice), ctypes.POINTER(_i)], _i),
    "cn_param_count": ([_i], _i),
    "cn_param_info": ([_i, _i, ctypes.c_char_p, _i, ctypes.POINTER(_i), ctypes.POINTER(_ll), ctypes.POINTER(_ll),
                       ctypes.POINTER(_ll), ctypes.POINTER(_i)], _i),
    "cn_gemm_wmma_f16": ([_vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _vp], _i),
    "cn_gemm_wmma_f16_noalloc": ([_vp, _vp, _vp, _i, _i, _i, _i, _vp], _i),
    "cn_reduce_rows_f16": ([_vp, _vp, _vp, _ll, _ll, _i, _vp], _i),
    "cn_border_gather_s2": ([_vp, _i, _i, _i, _i, _i, _vp, _vp], _i),
    "cn_warp_frames": ([_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _vp, _vp], _i),
    "cn_decode_layout": ([ctypes.POINTER(cn_decode_field), _i, ctypes.POINTER(_i)], _i),
    "cn_decode_outputs": ([_vp, _i, _i, ctypes.POINTER(cn_decode_field), _i, _vp, _i, _vp], _i),
    "cn_decode_frame": ([_vp, ctypes.POINTER(cn_decode_field), _i, _vp], _i),
    "cn_device_error": ([ctypes.POINTER(_i)], _i),
    "cn_selftest_bounded_wait": ([_i, ctypes.POINTER(_i)], _i),
    "cn_dev_alloc": ([ctypes.POINTER(_vp), _sz, _i], _i),
    "cn_dev_free": ([_vp], _i),
    "cn_host_alloc_pinned": ([ctypes.POINTER(_vp), _sz], _i),
    "cn_host_free_pinned": ([_vp], _i),
    "cn_memcpy": ([_vp, _vp, _sz, _i], _i),
    "cn_memset": ([_vp, _i, _sz], _i),
    "cn_device_synchronize": ([_i], _i),
    "cn_engine_stream": ([_vp, ctypes.POINTER(_vp)], _i),
}

_lib = None


def declared_symbols():
    """Function names declared in include/chestnut.h."""
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:int|size_t|const char\*)\s+(cn_\w+)\s*\(", text, re.M)))


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ChestnutError(f"{LIB_PATH} is missing: build it with chestnut-on-pc_b200/build.py "
                                "(the engine has no CPU fallback)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (args, res) in _SIGS.items():
            f = getattr(L, name)
            f.argtypes = args
            f.restype = res
        _lib = L
    return _lib


def check(rc, what=""):
    if rc != 0:
        msg = lib().cn_last_error().decode(errors="replace")
        raise ChestnutError(f"{what or 'chestnut call'} failed ({rc}): {msg}")
    return rc


class PinnedArray:
    """A numpy array over page-locked host memory (cn_host_alloc_pinned), so
    the engine's copies to and from it are asynchronous.  .array is the view;
    free() releases the memory (the view must not be used after it)."""

    def __init__(self, shape, dtype):
        import numpy as np
        dt = np.dtype(dtype)
        n = int(np.prod(shape)) * dt.itemsize
        p = ctypes.c_void_p()
        check(lib().cn_host_alloc_pinned(ctypes.byref(p), max(n, 1)), "cn_host_alloc_pinned")
        self.ptr = p
        self.array = np.frombuffer((ctypes.c_uint8 * max(n, 1)).from_address(p.value), dt, count=int(np.prod(shape))
                                   ).reshape(shape)

    def free(self):
        if self.ptr is not None and self.ptr.value:
            lib().cn_host_free_pinned(self.ptr)
        self.ptr = None


class DeviceBuffer:
    """Raw device allocation owned by Python (for kernel-level entry points)."""

    def __init__(self, nbytes, device=0):
        self.nbytes = int(nbytes)
        p = ctypes.c_void_p()
        check(lib().cn_dev_alloc(ctypes.byref(p), max(self.nbytes, 1), device), "cn_dev_alloc")
        self.ptr = p.value

    def upload(self, arr):
        import numpy as np
        a = np.ascontiguousarray(arr)
        assert a.nbytes <= self.nbytes
        check(lib().cn_memcpy(self.ptr, a.ctypes.data, a.nbytes, 0), "cn_memcpy H2D")
        return self

    def download(self, dtype, shape):
        import numpy as np
        out = np.empty(shape, dtype)
        check(lib().cn_memcpy(out.ctypes.data, self.ptr, out.nbytes, 1), "cn_memcpy D2H")
        return out

    def zero(self):
        check(lib().cn_memset(self.ptr, 0, self.nbytes), "cn_memset")
        return self

    def free(self):
        if self.ptr:
            lib().cn_dev_free(self.ptr)
            self.ptr = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass
