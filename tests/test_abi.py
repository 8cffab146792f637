"""CPU checks of the C ABI: the library loads, exports every declared symbol,
and its host-only model description matches the oracle's spec."""
import ctypes
import subprocess

import pytest

from chestnut_b200 import _lib, engine
from oracle import spec


def test_library_loads_and_exports_every_declared_symbol():
    L = _lib.lib()
    declared = _lib.declared_symbols()
    assert len(declared) >= 30
    missing = [s for s in declared if not hasattr(L, s)]
    assert not missing, missing
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    assert set(declared) <= exported


def test_every_declared_symbol_has_a_ctypes_signature():
    assert set(_lib.declared_symbols()) <= set(_lib._SIGS)


def test_output_slices_match_spec():
    assert engine.output_slices() == spec.out_slices()


@pytest.mark.parametrize("name,model", [("39m", 0), ("1b", 1)])
def test_param_table_matches_oracle(name, model):
    eng = engine.param_table(model)
    ora = spec.param_table(spec.CONFIGS[name])
    assert len(eng) == len(ora)
    kinds = {"w": 0, "b": 1, "pos": 2}
    for (en, etid, rows, cols, valid, kind), (on, otid, shape, fan_in, okind) in zip(eng, ora):
        assert en == on and etid == otid and kinds[okind] == kind
        if len(shape) == 1:
            assert (rows, cols) == (1, shape[0])
        else:
            assert (rows, cols) == shape
        if en.endswith("s0.conv3.w"):
            assert valid == spec.K0
        elif en == "cond.w":
            assert valid == spec.COND
        else:
            assert valid == cols


def test_state_bytes():
    assert _lib.lib().cn_state_bytes() == 2 * 5 * 6 * 128 * 256 + 96 * 512 * 4 + 100 * 8 * 4 + 512 * 4


def test_bad_arguments_return_errors_not_crashes():
    L = _lib.lib()
    assert L.cn_engine_create(None, None) == -2
    cfg = _lib.cn_config(7, 0, 1, 1, 0, 0)
    h = ctypes.c_void_p()
    assert L.cn_engine_create(ctypes.byref(cfg), ctypes.byref(h)) == -2
    assert b"bad config" in L.cn_last_error()
    assert L.cn_param_count(9) == -1
    assert L.cn_reduce_rows_f16(None, None, None, 1, 8, 0, None) == -2
    assert L.cn_gemm_wmma_f16(None, None, None, 1, 1, 64, 1, 0, 0, None) == -2
    assert L.cn_border_gather_s2(None, 1, 1, 2, 2, 8, None, None) == -2


def test_engine_create_without_gpu_fails_cleanly():
    try:
        import torch
        if torch.cuda.is_available():
            pytest.skip("GPU present")
    except Exception:
        pass
    cfg = _lib.cn_config(0, 0, 1, 1, 0, 0)
    h = ctypes.c_void_p()
    rc = _lib.lib().cn_engine_create(ctypes.byref(cfg), ctypes.byref(h))
    assert rc != 0 and not h.value
    assert _lib.lib().cn_last_error()


def test_shim_has_prefix_marker():
    import os
    path = os.path.join(os.path.dirname(_lib.HERE), "run_pinned2.py")
    src = open(path).read()
    assert "# --- smoke run" in src
    prefix = src.split("# --- smoke run")[0]
    for name in ("def run_frame", "out_slices", "ish", "img", "PACKED", "queues", "def make_warped", "_LIN_BY_NAME",
                 "jit", "cap", "rewrite_uop_list"):
        assert name in prefix, name
