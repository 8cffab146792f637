"""Python host surface of the B200 chestnut frame engine.

Mirrors the reference's frame contract (``run_pinned2.py:1462``):
``run_frame(warped u8[2,6,128,256], packed f32[524]) -> f32[N_out]`` with
``out_slices`` naming the heads, plus queue state and the kernel list.  All
compute goes through libchestnut.so (ctypes); nothing here touches a GPU
directly and there is no CPU fallback.
"""
import ctypes

import numpy as np

from . import _lib
from ._lib import check, lib

MODELS = {"39m": _lib.CN_MODEL_39M, "1b": _lib.CN_MODEL_1B}


def output_slices():
    n = ctypes.c_int(8)
    arr = (_lib.cn_slice * 8)()
    check(lib().cn_output_slices(arr, ctypes.byref(n)), "cn_output_slices")
    return {arr[i].name.decode(): slice(arr[i].start, arr[i].stop) for i in range(n.value)}


def param_table(model):
    """[(name, tensor_id, rows, cols, valid_cols, kind)] as the engine lays them out."""
    m = MODELS[model] if isinstance(model, str) else model
    out = []
    for i in range(lib().cn_param_count(m)):
        name = ctypes.create_string_buffer(96)
        tid, kind = ctypes.c_int(), ctypes.c_int()
        r, c, v = ctypes.c_longlong(), ctypes.c_longlong(), ctypes.c_longlong()
        check(lib().cn_param_info(m, i, name, 96, ctypes.byref(tid), ctypes.byref(r), ctypes.byref(c),
                                  ctypes.byref(v), ctypes.byref(kind)), "cn_param_info")
        out.append((name.value.decode(), tid.value, r.value, c.value, v.value, kind.value))
    return out


STATE_LAYOUT = (
    ("img_q", np.uint8, (5, 6, 128, 256)),
    ("big_img_q", np.uint8, (5, 6, 128, 256)),
    ("feat_q", np.float32, (96, 1, 512)),
    ("desire_q", np.float32, (100, 1, 8)),
    ("hidden", np.float32, (512,)),
)


class Engine:
    """One engine = one device, ``batch`` independent clips, one CUDA graph."""

    def __init__(self, model="1b", device=0, batch=1, seed=0, use_graph=True, carry_hidden=False):
        self.model = model
        self.batch = int(batch)
        self.device = int(device)
        cfg = _lib.cn_config(MODELS[model], self.device, self.batch, int(bool(use_graph)),
                             int(bool(carry_hidden)), int(seed))
        h = ctypes.c_void_p()
        check(lib().cn_engine_create(ctypes.byref(cfg), ctypes.byref(h)), "cn_engine_create")
        self._h = h
        self.carry_hidden = bool(carry_hidden)
        self.out_slices = output_slices()
        self.n_out = _lib.N_OUT

    # -- frames ------------------------------------------------------------
    def run_frame(self, warped, packed, out=None):
        w = np.ascontiguousarray(warped, np.uint8)
        p = np.ascontiguousarray(packed, np.float32)
        assert w.size == self.batch * _lib.FRAME_BYTES, w.shape
        assert p.size == self.batch * _lib.PACKED, p.shape
        if out is None:
            out = np.empty((self.batch, self.n_out) if self.batch > 1 else (self.n_out,), np.float32)
        check(lib().cn_run_frame(self._h, w.ctypes.data, p.ctypes.data, out.ctypes.data), "cn_run_frame")
        return out

    def stage(self, warped):
        """Start uploading the next frame's warped bytes (double-buffered; the
        array must stay alive and unchanged until run_staged consumes it, and
        be in pinned memory for the copy to overlap compute)."""
        w = warped if isinstance(warped, int) else np.ascontiguousarray(warped, np.uint8)
        if not isinstance(w, int):
            assert w.size == self.batch * _lib.FRAME_BYTES, w.shape
        check(lib().cn_stage_input(self._h, w if isinstance(w, int) else w.ctypes.data), "cn_stage_input")

    def run_staged(self, packed, out=None):
        """run_frame on the oldest staged input."""
        p = np.ascontiguousarray(packed, np.float32)
        assert p.size == self.batch * _lib.PACKED, p.shape
        if out is None:
            out = np.empty((self.batch, self.n_out) if self.batch > 1 else (self.n_out,), np.float32)
        check(lib().cn_run_staged(self._h, p.ctypes.data, out.ctypes.data), "cn_run_staged")
        return out

    def run_staged_async(self, packed, out):
        """Queue a frame on the oldest staged input; its output lands in
        `out` (a pinned array, see PinnedArray) once wait_output returns."""
        p = np.ascontiguousarray(packed, np.float32)
        assert p.size == self.batch * _lib.PACKED, p.shape
        assert out.size == self.batch * self.n_out and out.dtype == np.float32
        check(lib().cn_run_staged_async(self._h, p.ctypes.data, out.ctypes.data), "cn_run_staged_async")

    def wait_output(self):
        check(lib().cn_wait_output(self._h), "cn_wait_output")

    def run_frame_async(self, warped_ptr, packed_ptr):
        """Host pointers (ideally pinned); output stays on the device."""
        check(lib().cn_run_frame(self._h, warped_ptr, packed_ptr, None), "cn_run_frame")

    def run_frame_device(self, d_warped, d_packed):
        check(lib().cn_run_frame_device(self._h, d_warped, d_packed), "cn_run_frame_device")

    def read_output(self, out=None):
        if out is None:
            out = np.empty((self.batch, self.n_out), np.float32)
        check(lib().cn_read_output(self._h, out.ctypes.data), "cn_read_output")
        return out

    def sync(self):
        check(lib().cn_sync(self._h), "cn_sync")

    def stream_handle(self):
        s = ctypes.c_void_p()
        check(lib().cn_engine_stream(self._h, ctypes.byref(s)), "cn_engine_stream")
        return s.value or 0

    # -- state -------------------------------------------------------------
    def get_state(self, clip=0):
        n = lib().cn_state_bytes()
        buf = np.empty(n, np.uint8)
        check(lib().cn_get_state(self._h, clip, buf.ctypes.data, n), "cn_get_state")
        out, o = {}, 0
        for name, dt, shape in STATE_LAYOUT:
            nb = int(np.prod(shape)) * np.dtype(dt).itemsize
            out[name] = buf[o:o + nb].view(dt).reshape(shape).copy()
            o += nb
        return out

    def set_state(self, state, clip=0):
        parts = [np.ascontiguousarray(state[name], dt).reshape(-1).view(np.uint8) for name, dt, _ in STATE_LAYOUT]
        buf = np.concatenate(parts)
        check(lib().cn_set_state(self._h, clip, buf.ctypes.data, buf.nbytes), "cn_set_state")

    def reset(self):
        """Start new clips: zero the queues, carried hidden state and frame counter."""
        check(lib().cn_reset_state(self._h), "cn_reset_state")

    # -- introspection -----------------------------------------------------
    def kernel_list(self):
        n = ctypes.c_int(0)
        check(lib().cn_kernel_list(self._h, None, ctypes.byref(n)), "cn_kernel_list")
        arr = (_lib.cn_kernel_info * n.value)()
        check(lib().cn_kernel_list(self._h, arr, ctypes.byref(n)), "cn_kernel_list")
        return [dict(name=k.name.decode(), grid=tuple(k.grid), block=tuple(k.block), cluster=tuple(k.cluster),
                     smem=k.smem_bytes) for k in arr]

    def profile_frame(self, warped, packed):
        w = np.ascontiguousarray(warped, np.uint8)
        p = np.ascontiguousarray(packed, np.float32)
        n = ctypes.c_int(0)
        check(lib().cn_profile_frame(self._h, w.ctypes.data, p.ctypes.data, None, ctypes.byref(n)), "profile")
        ms = (ctypes.c_float * n.value)()
        check(lib().cn_profile_frame(self._h, w.ctypes.data, p.ctypes.data, ms, ctypes.byref(n)), "profile")
        names = [k["name"] for k in self.kernel_list()]
        return list(zip(names, list(ms)))

    def set_timed_class(self, prefix):
        check(lib().cn_set_timed_class(self._h, prefix.encode()), "cn_set_timed_class")

    def timed_class_ms(self):
        n = ctypes.c_int(0)
        check(lib().cn_timed_class_ms(self._h, None, ctypes.byref(n)), "cn_timed_class_ms")
        ms = (ctypes.c_float * max(n.value, 1))()
        check(lib().cn_timed_class_ms(self._h, ms, ctypes.byref(n)), "cn_timed_class_ms")
        return list(ms)[:n.value]

    def info(self):
        p, w, k = ctypes.c_longlong(), ctypes.c_longlong(), ctypes.c_int()
        check(lib().cn_engine_info(self._h, ctypes.byref(p), ctypes.byref(w), ctypes.byref(k)), "cn_engine_info")
        return {"n_params": p.value, "weight_bytes": w.value, "n_kernels": k.value}

    def close(self):
        if getattr(self, "_h", None):
            lib().cn_engine_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
