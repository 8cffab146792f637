"""Input queues and packed-vector split (oracle side, test infrastructure).

Restates ``compile_modeld.py``:
  * ``shift_and_sample`` (:166-168): drop the oldest row, append the new one.
  * ``sample_skip`` (:171-172): every FS-th row, then flatten(0,1).
  * ``sample_desire`` (:175-176): max over groups of FS rows.
  * ``run_policy`` (:199-221): img/big_img from warped[0]/warped[1]; packed =
    desire | traffic_convention | action_t | prev_feat.
Queue shapes follow ``run_pinned2.py:1373-1389``.  All of this is index /
copy work: the engine must match it bit for bit.
"""
import numpy as np

from . import spec as S


def new_state():
    return {
        "img_q": np.zeros((S.IMG_Q, S.CH, S.H, S.W), np.uint8),
        "big_img_q": np.zeros((S.IMG_Q, S.CH, S.H, S.W), np.uint8),
        "feat_q": np.zeros((S.FEAT_Q, 1, S.FEAT), np.float32),
        "desire_q": np.zeros((S.DESIRE_Q, 1, S.DESIRE), np.float32),
    }


def shift_and_sample(buf, new_val, sample_fn):
    buf[:] = np.concatenate([buf[1:], new_val], axis=0)
    return sample_fn(buf)


def sample_skip(buf):
    s = buf[::S.FS]
    return s.reshape((s.shape[0] * s.shape[1],) + s.shape[2:])[None]


def sample_desire(buf):
    r = buf.reshape((-1, S.FS) + buf.shape[1:]).max(axis=1)
    return r.reshape((r.shape[0] * r.shape[1],) + r.shape[2:])[None]


def split_packed(packed):
    p = np.asarray(packed, np.float32)
    o = 0
    desire = p[o:o + S.DESIRE]; o += S.DESIRE
    tc = p[o:o + S.TC]; o += S.TC
    at = p[o:o + S.AT]; o += S.AT
    prev_feat = p[o:o + S.FEAT]
    return desire, tc, at, prev_feat


def step(state, warped, packed):
    """One frame of queue updates; returns the model inputs (run_policy)."""
    warped = np.asarray(warped, np.uint8)
    img = shift_and_sample(state["img_q"], warped[0:1], sample_skip)
    big_img = shift_and_sample(state["big_img_q"], warped[1:2], sample_skip)
    desire, tc, at, prev_feat = split_packed(packed)
    desire_buf = shift_and_sample(state["desire_q"], desire.reshape(1, 1, -1), sample_desire)
    feat_buf = shift_and_sample(state["feat_q"], prev_feat.reshape(1, 1, -1), sample_skip)
    return {
        "img": img,                    # u8 (1, 12, 128, 256)
        "big_img": big_img,            # u8 (1, 12, 128, 256)
        "features_buffer": feat_buf,   # f32 (1, 24, 512)
        "desire_pulse": desire_buf,    # f32 (1, 25, 8)
        "traffic_convention": tc.reshape(1, -1),
        "action_t": at.reshape(1, -1),
    }
