"""GPU output decode against the oracle restatement of the reference's Parser
(parse_model_outputs.py:1-120).

Means and selections are copies (compared bit for bit); exp, sigmoid and
softmax values within 2e-6 relative (CUDA's expf and numpy's float32 exp are
both within a couple of ulp; the decoder divides with IEEE division)."""
import numpy as np
import pytest

from chestnut_b200 import DeviceBuffer, Engine, _lib, decode, kernels
from oracle import model as omodel
from oracle import parse, spec

pytestmark = pytest.mark.gpu

# openpilot-like field shapes: a 5-hypothesis plan (33 x 15 per hypothesis,
# one weight logit), a 2-hypothesis lead with 3 selection columns (6 x 4),
# lane lines without hypotheses, probabilities, a categorical desire field
OP_LAYOUT = (
    ("mdn", "plan", 0, 5 * (2 * 495 + 1), 5, 1, 0),
    ("mdn", "lead", 4955, 2 * (2 * 24 + 3), 2, 3, 0),
    ("mdn", "lane_lines", 5057, 2 * 264, 0, 0, 0),
    ("sigmoid", "lane_lines_prob", 5585, 8, 0, 0, 0),
    ("softmax", "desire_state", 5593, 8, 0, 0, 8),
    ("softmax", "desire_pred", 5601, 32, 0, 0, 8),
)
RAW = 5633


def _close(got, ref):
    return np.all(np.abs(got - ref) <= 2e-6 * np.abs(ref) + 1e-30)


@pytest.mark.parametrize("layout,raw_len", [(OP_LAYOUT, RAW), (decode.SYNTHETIC_LAYOUT, 3323)])
def test_device_decode_matches_the_oracle(layout, raw_len):
    rs = np.random.default_rng(raw_len)
    B = 3
    raw = (rs.standard_normal((B, raw_len)) * 3).astype(np.float32)
    raw[1, 10:20] = 40.0          # exercises the clip at 11 in exp
    arr, n = decode.fields(layout)
    dr, do = DeviceBuffer(raw.nbytes).upload(raw), DeviceBuffer(B * n * 4)
    _lib.check(_lib.lib().cn_decode_outputs(dr.ptr, B, raw_len, arr, len(layout), do.ptr, n, None), "decode")
    kernels.synchronize()
    got = do.download(np.float32, (B, n))
    for b in range(B):
        ref = parse.flatten(parse.decode(raw[b], layout), layout)
        assert _close(got[b], ref), (b, float(np.max(np.abs(got[b] - ref) / (np.abs(ref) + 1e-30))))
        g = decode.unflatten(got[b], layout, arr)
        r = parse.decode(raw[b], layout)
        for kind, name, *_ in layout:
            if kind == "mdn":
                np.testing.assert_array_equal(g[name].reshape(-1), r[name]["mu"].reshape(-1))   # copies


def test_engine_frame_decode_and_model_state():
    from chestnut_b200.modeld import ModelState
    rs = np.random.default_rng(9)
    w = rs.integers(0, 256, (2, 6, 128, 256), dtype=np.uint8)
    eng = Engine("39m", seed=4)
    ms = ModelState(engine=eng, decode=decode.SYNTHETIC_LAYOUT)
    inputs = {"desire_pulse": np.eye(8, dtype=np.float32)[2], "traffic_convention": np.array([1, 0], np.float32),
              "action_t": np.zeros(2, np.float32)}
    res = ms.run(w, inputs)
    raw = ms.last_output
    ref = parse.decode(raw, decode.SYNTHETIC_LAYOUT)
    np.testing.assert_array_equal(res["plan"][0], ref["plan"]["mu"][0])
    assert _close(res["plan_weights"][0], ref["plan"]["weights"])
    assert _close(res["lead_stds"][0], ref["lead"]["std"])
    assert res["plan_hypotheses"].shape == (1, 5, 247) and res["lead"].shape == (1, 2, 11)
    # the decoded frame is the oracle's frame, within the frame tolerance (ModelState
    # sent desire one-hot 2 as a rising edge, traffic convention [1, 0], no features yet)
    pk = np.zeros(524, np.float32)
    pk[2] = 1.0
    pk[8] = 1.0
    oref = omodel.Clip("39m", 4).run_frame(w, pk)
    sl = spec.out_slices()["plan"]
    assert np.all(np.abs(raw[sl] - oref[sl]) <= 2e-2 + 1e-2 * np.abs(oref[sl]))
