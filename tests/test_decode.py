"""Output decode (parse_model_outputs.py:1-120): the oracle restatement and the
C-ABI layout check (CPU).  The GPU decoder is compared with the oracle in
tests/test_gpu_decode.py."""
import ctypes

import numpy as np
import pytest

from chestnut_b200 import _lib, decode
from oracle import parse


def test_safe_exp_clips_at_11_and_sigmoid_softmax_values():
    assert parse.safe_exp(np.float32(20.0)) == np.float32(np.exp(np.float32(11.0)))
    np.testing.assert_allclose(parse.sigmoid(np.array([0.0, 2.0, -30.0], np.float32)),
                               [0.5, 1 / (1 + np.exp(-2.0)), 1 / (1 + np.exp(11.0))], rtol=1e-6)
    s = parse.softmax(np.array([[1.0, 2.0, 3.0]], np.float32))
    np.testing.assert_allclose(s[0], np.exp([1.0, 2.0, 3.0]) / np.exp([1.0, 2.0, 3.0]).sum(), rtol=1e-6)


def test_mdn_single_selection_sorts_hypotheses_by_weight():
    # 3 hypotheses x [mu 2 | log-std 2 | logit]: logits 0, 2, 1 -> order 1, 2, 0
    raw = np.array([[10, 11, 0, 0, 0.0], [20, 21, 1, 1, 2.0], [30, 31, 2, 2, 1.0]], np.float32).reshape(-1)
    d = parse.mdn(raw, 3, 1)
    np.testing.assert_array_equal(d["hypotheses"], [[20, 21], [30, 31], [10, 11]])
    np.testing.assert_array_equal(d["mu"], [[20, 21]])
    w = np.exp([2.0, 1.0, 0.0]) / np.exp([0.0, 1.0, 2.0]).sum()
    np.testing.assert_allclose(d["weights"][:, 0], w, rtol=1e-6)
    np.testing.assert_allclose(d["std"], np.exp([[1.0, 1.0]]), rtol=1e-6)


def test_mdn_multi_selection_picks_per_column_and_keeps_order():
    # 2 hypotheses x [mu 1 | log-std 1 | 2 logits]: column 0 prefers h1, column 1 prefers h0
    raw = np.array([[5, 0, 0.0, 3.0], [7, 0, 1.0, 0.0]], np.float32).reshape(-1)
    d = parse.mdn(raw, 2, 2)
    np.testing.assert_array_equal(d["hypotheses"], [[5], [7]])
    np.testing.assert_array_equal(d["mu"], [[7], [5]])


def test_mdn_ties_follow_stable_argsort_reversed():
    raw = np.array([[1, 0, 0.0], [2, 0, 0.0]], np.float32).reshape(-1)   # equal logits
    d = parse.mdn(raw, 2, 1)
    np.testing.assert_array_equal(d["hypotheses"], [[2], [1]])          # higher index ranked first
    np.testing.assert_array_equal(d["mu"], [[1]])                       # then the later position is selected


def test_mdn_without_hypotheses_splits_mean_and_log_std():
    d = parse.mdn(np.array([1, 2, 0, np.log(3)], np.float32), 0, 0)
    np.testing.assert_array_equal(d["mu"], [[1, 2]])
    np.testing.assert_allclose(d["std"], [[1, 3]], rtol=1e-6)


def test_layout_offsets_from_the_library_match_the_oracle_order():
    arr, n = decode.fields(decode.SYNTHETIC_LAYOUT)
    rs = np.random.default_rng(0)
    raw = rs.standard_normal(3323).astype(np.float32)
    flat = parse.flatten(parse.decode(raw, decode.SYNTHETIC_LAYOUT), decode.SYNTHETIC_LAYOUT)
    assert flat.size == n
    assert [arr[i].out_off for i in range(3)] == [0, 2969, 3233]
    got = decode.unflatten(flat, decode.SYNTHETIC_LAYOUT, arr)
    ref = parse.decode(raw, decode.SYNTHETIC_LAYOUT)
    np.testing.assert_array_equal(got["plan"], ref["plan"]["mu"][0])
    np.testing.assert_array_equal(got["lead_weights"], ref["lead"]["weights"])


@pytest.mark.parametrize("field", [
    (0, 0, 10, 3, 1, 0),      # 10 values do not split into 3 hypothesis rows
    (0, 0, 12, 3, 0, 0),      # in_n > 1 needs a selection column
    (0, 0, 12, 0, 2, 0),      # in_n <= 1 has none
    (2, 0, 10, 0, 0, 4),      # softmax groups of 4 do not tile 10 values
    (7, 0, 8, 0, 0, 0),       # unknown kind
])
def test_bad_layouts_are_rejected(field):
    f = (_lib.cn_decode_field * 1)(_lib.cn_decode_field(*field, 0))
    n = ctypes.c_int(0)
    assert _lib.lib().cn_decode_layout(f, 1, ctypes.byref(n)) == -2
    assert b"not decodable" in _lib.lib().cn_last_error()
