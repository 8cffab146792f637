"""Headless video_check-style harness (video_check.py:50-94): per-frame plan
rows from NV12 camera frames.  CPU: plan selection, rows and summary on
constructed outputs.  GPU: the harness's rows (GPU frame warp + engine) against
rows computed from the oracle's warp and frame, frame by frame."""
import numpy as np
import pytest

from chestnut_b200 import video_check as vc
from oracle import spec

SL = spec.out_slices()
ATOL, RTOL = 2e-2, 1e-2  # per-head frame tolerance (north star)


def _out_with_plan(plan):
    out = np.zeros(spec.N_OUT, np.float32)
    out[SL["plan"]] = plan.reshape(-1)
    return out


def test_parse_plan_picks_the_laterally_closest_hypothesis():
    plan = np.zeros(vc.PLAN_SHAPE, np.float32)
    plan[:, -1, 1] = [3.0, -0.5, 0.2, -0.1, 4.0]
    plan[3, :, 0] = 7.0
    tr = vc.parse_plan(_out_with_plan(plan), SL)
    assert np.all(tr[:, 0] == 7.0)


def test_frame_row_and_summary():
    plan = np.zeros(vc.PLAN_SHAPE, np.float32)
    plan[0, vc.PLAN_IDX - 1, 3:6] = [3.0, 4.0, 0.0]      # v_now = 5
    plan[0, vc.PLAN_IDX, 3:6] = [0.0, 0.0, 0.5]          # v_next = 0.5 (a stop, and a decel)
    plan[0, vc.PLAN_IDX, 1] = 3.0                        # steer clipped to +1
    row = vc.frame_row(7, _out_with_plan(plan), SL)
    assert row[0] == 7 and row[1] == pytest.approx(5.0) and row[2] == pytest.approx(3.0)
    assert row[3] == pytest.approx(0.5) and row[4] == 1.0
    s = vc.summary([row, (8, 1.0, 0.0, 1.0, 0.0)])
    assert s["frames"] == 2 and s["stop_frames"] == 1 and s["decel_frames"] == 1
    assert s["steer_max"] == 1.0 and s["steer_min"] == 0.0


@pytest.mark.gpu
def test_gpu_rows_match_the_oracle_rows():
    from chestnut_b200.modeld import ModelState
    from oracle import model as omodel
    from oracle import warp as W
    geom = (256, 128, 256, 128, 64)   # a small NV12 camera keeps the CPU oracle quick
    frames = list(vc.synthetic_frames(8, geom, seed=7))
    # the model image reads the camera at scale 0.5 with a little roll and perspective
    tf = {"img": vc.calibration(0.5, 0.05, 1e-4, 3.0, 2.0), "big_img": vc.calibration(0.45, -0.04, -1e-4, 10.0, 5.0)}
    ms = ModelState(model="39m", seed=3, nv12=geom)
    rows = vc.run(frames, transforms=tf, state=ms)
    clip = omodel.Clip("39m", 3)
    pk = np.zeros(524, np.float32)
    checked = 0
    for i, (road, wide) in enumerate(frames):
        inp = vc.inputs_for(i)
        pk[8:10] = inp["traffic_convention"]
        warped = W.make_warp(road, wide, tf["img"], tf["big_img"], geom[0], geom[1], geom[2], geom[3])
        ref = clip.run_frame(warped, pk.copy())
        pk[12:] = ref[SL["hidden_state"]]
        plan = ref[SL["plan"]].reshape(vc.PLAN_SHAPE)
        lat = np.sort(np.abs(plan[:, -1, 1]))
        if lat[1] - lat[0] <= 2 * (ATOL + RTOL * lat[1]):
            continue   # the best hypothesis is within tolerance of the next: selection may differ
        want = vc.frame_row(i, ref, SL)
        got = rows[i]
        assert got[0] == i
        for g, w in zip(got[1:], want[1:]):
            assert abs(g - w) <= ATOL + RTOL * abs(w), (i, got, want)
        checked += 1
    assert checked >= 3, checked
    # the last frame's whole output, head by head (rows carry the state of every frame before it)
    for name, sl in SL.items():
        d = np.abs(ms.last_output[sl] - ref[sl])
        assert np.all(d <= ATOL + RTOL * np.abs(ref[sl])), (name, float(d.max()))
