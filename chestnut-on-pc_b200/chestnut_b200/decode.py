"""On-device output decode: the reference's Parser (parse_model_outputs.py:1-120)
run on the GPU by libchestnut.so (cn_decode_outputs / cn_decode_frame).

A layout is a sequence of fields ``(kind, name, raw_off, raw_len, in_n, out_n,
width)`` over one frame's raw output vector:

* ``"mdn"``: ``Parser.parse_mdn(name, in_N=in_n, out_N=out_n)``; decoded into
  ``name`` (best hypothesis mean per selection column), ``name + '_stds'`` and,
  with in_n > 1, ``name + '_weights'``, ``'_hypotheses'``,
  ``'_stds_hypotheses'`` -- the keys Parser writes;
* ``"sigmoid"``: ``parse_binary_crossentropy``;
* ``"softmax"``: ``parse_categorical_crossentropy`` over groups of ``width``.

The synthetic models' heads are laid out so that this decode applies to them
(``SYNTHETIC_LAYOUT``): plan = 5 hypotheses x [247 mean | 247 log-std | 1
weight logit]; lane_lines = [132 mean | 132 log-std]; lead = 3 hypotheses x
[11 mean | 11 log-std | 2 selection logits].
"""
import ctypes

import numpy as np

from . import _lib
from ._lib import check, lib

KINDS = {"mdn": 0, "sigmoid": 1, "softmax": 2}

SYNTHETIC_LAYOUT = (
    ("mdn", "plan", 0, 2475, 5, 1, 0),
    ("mdn", "lane_lines", 2475, 264, 0, 0, 0),
    ("mdn", "lead", 2739, 72, 3, 2, 0),
)


def fields(layout):
    """(ctypes array of cn_decode_field with out_off set, decoded floats per frame)."""
    arr = (_lib.cn_decode_field * len(layout))()
    for i, (kind, _name, off, length, in_n, out_n, width) in enumerate(layout):
        arr[i] = _lib.cn_decode_field(KINDS[kind], off, length, in_n, out_n, width, 0)
    n = ctypes.c_int(0)
    check(lib().cn_decode_layout(arr, len(layout), ctypes.byref(n)), "cn_decode_layout")
    return arr, n.value


def unflatten(flat, layout, arr):
    """Decoded values of one frame -> {key: array}, keyed as Parser keys them."""
    out = {}
    for i, (kind, name, _off, length, in_n, out_n, _w) in enumerate(layout):
        o = arr[i].out_off
        if kind != "mdn":
            out[name] = flat[o:o + length].copy()
            continue
        rows = max(in_n, 1)
        n = (length // rows - out_n) // 2
        if in_n > 1:
            out[name + "_weights"] = flat[o:o + in_n * out_n].reshape(in_n, out_n).copy()
            o += in_n * out_n
            out[name + "_hypotheses"] = flat[o:o + in_n * n].reshape(in_n, n).copy()
            o += in_n * n
            out[name + "_stds_hypotheses"] = flat[o:o + in_n * n].reshape(in_n, n).copy()
            o += in_n * n
        sel = max(out_n, 1)
        mu = flat[o:o + sel * n].reshape(sel, n)
        sd = flat[o + sel * n:o + 2 * sel * n].reshape(sel, n)
        out[name] = (mu if out_n > 1 else mu[0]).copy()
        out[name + "_stds"] = (sd if out_n > 1 else sd[0]).copy()
    return out


def decode_frame(engine, layout=SYNTHETIC_LAYOUT):
    """Decode the engine's last frame output on the GPU -> one dict per clip."""
    arr, n = fields(layout)
    host = np.empty((engine.batch, n), np.float32)
    check(lib().cn_decode_frame(engine._h, arr, len(layout), host.ctypes.data), "cn_decode_frame")
    return [unflatten(host[b], layout, arr) for b in range(engine.batch)]
