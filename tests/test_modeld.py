"""CPU tests of the ModelState host semantics (modeld.py:165-200) with a fake engine."""
import numpy as np

from chestnut_b200.modeld import ModelState
from oracle import spec


class RecordingEngine:
    def __init__(self, bad_frames=()):
        self.out_slices = spec.out_slices()
        self.calls = []
        self.bad = set(bad_frames)

    def run_frame(self, warped, packed):
        self.calls.append(np.array(packed, copy=True))
        n = len(self.calls)
        out = np.full(spec.N_OUT, 0.01 * n, np.float32)
        out[spec.out_slices()["hidden_state"]] = np.arange(512, dtype=np.float32) * n
        if n in self.bad:
            out[5] = np.nan
        return out


def test_desire_is_a_rising_edge_pulse_and_features_are_carried():
    eng = RecordingEngine()
    ms = ModelState(engine=eng)
    w = np.zeros((2, 6, 128, 256), np.uint8)
    d = np.zeros(8, np.float32)
    tc = np.array([1.0, 0.0], np.float32)
    at = np.array([0.5, -0.5], np.float32)
    d[3] = 1.0
    out = ms.run(w, {"desire_pulse": d, "traffic_convention": tc, "action_t": at})
    assert set(out) == set(spec.out_slices()) and out["plan"].shape == (1, 2475)
    assert eng.calls[0][3] == 1.0 and eng.calls[0][8] == 1.0 and eng.calls[0][10] == 0.5
    assert (eng.calls[0][12:] == 0).all()
    ms.run(w, {"desire_pulse": d, "traffic_convention": tc, "action_t": at})   # held -> no pulse
    assert eng.calls[1][3] == 0.0
    assert np.array_equal(eng.calls[1][12:], np.arange(512, dtype=np.float32))  # carried hidden state
    d0 = d.copy()
    d0[0] = 1.0                                   # desire[0] is forced to 0 (modeld.py:177)
    d0[3] = 0.0
    ms.run(w, {"desire_pulse": d0, "traffic_convention": tc, "action_t": at})
    assert eng.calls[2][0] == 0.0


def test_non_finite_frames_are_dropped_and_not_carried():
    eng = RecordingEngine(bad_frames={2})
    ms = ModelState(engine=eng)
    w = np.zeros((2, 6, 128, 256), np.uint8)
    inp = {"desire_pulse": np.zeros(8, np.float32), "traffic_convention": np.array([1, 0], np.float32),
           "action_t": np.zeros(2, np.float32)}
    assert ms.run(w, inp) is not None
    assert ms.run(w, inp) is None
    ms.run(w, inp)
    assert np.array_equal(eng.calls[2][12:], np.arange(512, dtype=np.float32) * 1)  # still frame 1's features
