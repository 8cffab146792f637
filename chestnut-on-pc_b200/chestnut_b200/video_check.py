"""Headless frame-rows harness in the style of the reference's ``video_check.py``.

The reference (``video_check.py:50-94``) decodes footage, prepares each frame,
runs ``run_frame`` with the hidden state carried (``pk[12:] = out[hidden_state]``),
picks the best plan hypothesis (``parse_plan``, ``:34-36``) and records one row
per frame, ``(frame, v_now, lateral, v_next, steer)`` at the ~2 s plan index
(``:61-66``), then prints summary lines and saves the rows (``:88-94``).  The
rows are its regression gate between engine builds.

Here the camera frames are NV12 buffers, prepared on the GPU by the frame warp
(``ModelState.run(bufs, transforms, inputs)`` -> ``cn_warp_frames``), so the
whole path from camera bytes to plan rows runs on the engine.  The reference's
footage and its OpenCV decode are not available, so seeded synthetic NV12
frames stand in unless a raw NV12 file is given (``--nv12``: consecutive frames
of the given geometry).  There is no video overlay (headless).

    python -m chestnut_b200.video_check [--model 39m|1b] [--frames N] [--nv12 FILE]
                                        [--width W --height H --stride S --y-height Y --uv-height U]
                                        [--rows OUT.npy]

The synthetic models' ``plan`` head is 5 x 33 x 15 (the reference's real plan is
5 x 33 x 6); ``parse_plan`` uses the same columns: 1 = lateral, 3..5 = velocity.
"""
import argparse
import time

import numpy as np

PLAN_SHAPE = (5, 33, 15)
PLAN_IDX = 8  # ~2 s into the plan (video_check.py:61)

# a 1928 x 1208 camera in NV12: 2048-byte rows, Y padded to 1216 rows, 608 UV rows
DEFAULT_NV12 = (1928, 1208, 2048, 1216, 608)


def calibration(scale, roll, persp, tx, ty):
    """A 3x3 inverse warp (model pixel -> camera pixel) of the kind modeld receives."""
    c, s = np.cos(roll), np.sin(roll)
    return np.array([[scale * c, -scale * s, tx], [scale * s, scale * c, ty], [persp, 0.0, 1.0]], np.float32)


DEFAULT_TRANSFORMS = {"img": calibration(3.6, 0.02, 2e-5, 40.0, 300.0),
                      "big_img": calibration(2.1, -0.03, -3e-5, 420.0, 350.0)}


def parse_plan(out, out_slices):
    """Best plan hypothesis: the one whose last point is laterally closest to 0
    (``video_check.py:34-36``)."""
    plan = np.asarray(out)[out_slices["plan"]].reshape(PLAN_SHAPE)
    return plan[int(np.argmin(np.abs(plan[:, -1, 1])))]


def frame_row(i, out, out_slices):
    """(frame, v_now, lateral, v_next, steer) at the ~2 s plan point (``video_check.py:61-66``)."""
    tr = parse_plan(out, out_slices)
    li = PLAN_IDX
    v_now = float(np.linalg.norm(tr[max(1, li - 1), 3:6]))
    v_next = float(np.linalg.norm(tr[li, 3:6]))
    steer = max(-1.0, min(1.0, float(tr[li, 1]) / 2.0))
    return (i, v_now, float(tr[li, 1]), v_next, steer)


def summary(rows):
    """The reference's closing summary (``video_check.py:88-93``) as a dict."""
    rows = np.asarray(rows, np.float64)
    return {"frames": int(len(rows)),
            "v_next_mean": float(rows[:, 3].mean()), "v_next_min": float(rows[:, 3].min()),
            "v_next_max": float(rows[:, 3].max()),
            "steer_mean": float(rows[:, 4].mean()), "steer_min": float(rows[:, 4].min()),
            "steer_max": float(rows[:, 4].max()),
            "decel_frames": int((rows[:, 3] < rows[:, 1] * 0.9).sum()),
            "stop_frames": int((rows[:, 3] < 1).sum())}


def synthetic_frames(n, nv12=DEFAULT_NV12, seed=0):
    """n seeded (road, wide) NV12 frame pairs, u8 buffers of stride * (y_height + uv_height) bytes."""
    _, _, stride, yh, uvh = nv12
    rs = np.random.default_rng(seed)
    for _ in range(n):
        yield (rs.integers(0, 256, stride * (yh + uvh), dtype=np.uint8),
               rs.integers(0, 256, stride * (yh + uvh), dtype=np.uint8))


def file_frames(path, nv12=DEFAULT_NV12):
    """Consecutive NV12 frames of a raw file; each frame feeds both cameras (as
    video_check.py:59 feeds the same channels to both)."""
    _, _, stride, yh, uvh = nv12
    size = stride * (yh + uvh)
    with open(path, "rb") as f:
        while True:
            b = f.read(size)
            if len(b) < size:
                return
            a = np.frombuffer(b, np.uint8)
            yield a, a


def inputs_for(i):
    """Inputs of frame i: no desire, traffic convention (1, 0) and action_t 0, as
    video_check.py:47-48 sets the packed vector."""
    return {"desire_pulse": np.zeros(8, np.float32), "traffic_convention": np.array([1.0, 0.0], np.float32),
            "action_t": np.zeros(2, np.float32)}


def run(frames, model="39m", nv12=DEFAULT_NV12, transforms=None, seed=0, state=None):
    """Rows of every frame pair in `frames` through ModelState's NV12 path."""
    from .modeld import ModelState
    ms = state if state is not None else ModelState(model=model, seed=seed, nv12=nv12)
    tf = transforms or DEFAULT_TRANSFORMS
    rows = []
    for i, (road, wide) in enumerate(frames):
        if ms.run({"img": road, "big_img": wide}, tf, inputs_for(i)) is None:
            continue  # non-finite frame dropped (modeld.py:191-194)
        flat = ms.last_output
        rows.append(frame_row(i, flat, ms.output_slices))
    return np.array(rows, np.float64)


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--model", default="39m", choices=["39m", "1b"])
    ap.add_argument("--frames", type=int, default=120)
    ap.add_argument("--nv12", default="")
    ap.add_argument("--width", type=int, default=DEFAULT_NV12[0])
    ap.add_argument("--height", type=int, default=DEFAULT_NV12[1])
    ap.add_argument("--stride", type=int, default=DEFAULT_NV12[2])
    ap.add_argument("--y-height", type=int, default=DEFAULT_NV12[3])
    ap.add_argument("--uv-height", type=int, default=DEFAULT_NV12[4])
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--rows", default="video_check_rows.npy")
    a = ap.parse_args()
    geom = (a.width, a.height, a.stride, a.y_height, a.uv_height)
    frames = file_frames(a.nv12, geom) if a.nv12 else synthetic_frames(a.frames, geom, a.seed)
    if a.nv12:
        frames = (f for i, f in zip(range(a.frames), frames))
    t0 = time.time()
    rows = run(frames, a.model, geom, seed=a.seed)
    s = summary(rows)
    print(f"processed {s['frames']} frames in {time.time() - t0:.1f}s -> {a.rows}")
    print(f"planned speed@2s: mean={s['v_next_mean']:.1f} min={s['v_next_min']:.1f} max={s['v_next_max']:.1f}")
    print(f"steer: mean={s['steer_mean']:+.3f} min={s['steer_min']:+.3f} max={s['steer_max']:+.3f}")
    print(f"decel frames (v@2s < v@prev-step*0.9): {s['decel_frames']}")
    print(f"stop frames (v@2s < 1): {s['stop_frames']}")
    np.save(a.rows, rows)


if __name__ == "__main__":
    main()
