"""Synthetic chestnut frame forward pass (oracle side, test infrastructure).

Restates, in numpy f32 with f16 rounding at the same points as the engine, one
frame of the path the reference runs in ``run_pinned2.py:1462-1565``:
queues (``compile_modeld.py:199-221``) -> two camera conv stems reading the
image through the zero-border rule -> 88-token pre-LN transformer ->
hidden_state / plan / lane_lines / lead heads.  The caller carries the hidden
state exactly as ``video_check.py:60`` does: ``packed[12:] = out[hidden_state]``.

Numerics (mirrored by the engine):
  * activations between kernels are f16; the residual stream is f32;
  * every contraction accumulates in f32 (order differs on the GPU -> tolerance);
  * LayerNorm: f32 mean/var over the row, eps 1e-5, no affine, f16 out;
  * attention: f32 scores * 1/sqrt(hd), f32 softmax, f32 P @ V, f16 out;
  * GELU is the erf form; hidden_state = f16(tanh(.)).
"""
import math

import numpy as np

from . import rng, spec as S
from .border import im2col_frame, im2col_s2
from .queues import new_state, step as queue_step

try:
    from scipy.special import erf as _erf
except Exception:  # pragma: no cover
    _erf = np.vectorize(math.erf)


def _fill(seed, tid, count, bound, f16):
    """C restatement when it builds (fast); numpy restatement otherwise.
    Both are the same function (checked by tests/test_oracle.py)."""
    try:
        from . import build
        return build.fill(seed, tid, count, bound, f16)
    except Exception:
        return rng.fill(seed, tid, count, bound, np.float16 if f16 else np.float32)


def gen_params(cfg, seed):
    """All parameters, generated with the hash RNG exactly as the engine does."""
    P = {}
    for name, tid, shape, fan_in, kind in S.param_table(cfg):
        count = int(np.prod(shape))
        if kind == "w":
            v = _fill(seed, tid, count, math.sqrt(6.0 / fan_in), True).reshape(shape)
            if name.endswith("s0.conv3.w"):
                v[:, S.K0:] = 0
            if name == "cond.w":
                v[:, S.COND:] = 0
        elif kind == "b":
            v = _fill(seed, tid, count, 1.0 / math.sqrt(fan_in), False).reshape(shape)
        else:
            v = _fill(seed, tid, count, 0.5, False).reshape(shape)
        P[name] = v
    return P


def _mm(a16, w16):
    """f16 [M,K] x f16 [N,K]^T -> f32 [M,N] (f32 accumulate)."""
    return a16.astype(np.float32) @ w16.astype(np.float32).T


def layernorm(x):
    mean = x.mean(axis=-1, keepdims=True, dtype=np.float32)
    xc = x - mean
    var = (xc * xc).mean(axis=-1, keepdims=True, dtype=np.float32)
    return (xc * (1.0 / np.sqrt(var + np.float32(S.LN_EPS)))).astype(np.float16)


def gelu(x):
    return (0.5 * x * (1.0 + _erf(x / np.float32(math.sqrt(2.0))))).astype(np.float32)


def stem(P, cam, img12, cfg):
    """One camera's conv stem -> f16 [32, C4] (row = 4x8 position)."""
    a = im2col_frame(img12)
    hh, ww = S.H // 2, S.W // 2
    act = None
    for s, c in enumerate(cfg.stem):
        if s > 0:
            a = im2col_s2(act.reshape(hh * 2, ww * 2, -1))
        pre = _mm(a, P[f"cam{cam}.s{s}.conv3.w"]) + P[f"cam{cam}.s{s}.conv3.b"]
        y = np.maximum(pre, 0).astype(np.float16)
        pre = _mm(y, P[f"cam{cam}.s{s}.conv1.w"]) + P[f"cam{cam}.s{s}.conv1.b"]
        act = np.maximum(pre, 0).astype(np.float16)      # [hh*ww, c], NHWC
        if s + 1 < len(cfg.stem):
            hh, ww = hh // 2, ww // 2
    return act


def cond_vector(inp):
    v = np.zeros(S.COND_PAD, np.float32)
    v[:S.N_DESIRE * S.DESIRE] = inp["desire_pulse"].reshape(-1)
    v[S.N_DESIRE * S.DESIRE:S.N_DESIRE * S.DESIRE + S.TC] = inp["traffic_convention"].reshape(-1)
    v[S.N_DESIRE * S.DESIRE + S.TC:S.COND] = inp["action_t"].reshape(-1)
    return v.astype(np.float16)


def embed(P, inp, cfg):
    """Residual stream x f32 [88, d] at layer 0."""
    cond = (_mm(cond_vector(inp)[None], P["cond.w"]) + P["cond.b"])[0]
    x = np.zeros((S.T, cfg.d), np.float32)
    for cam, key in enumerate(("img", "big_img")):
        act = stem(P, cam, inp[key][0], cfg)
        x[cam * 32:(cam + 1) * 32] = _mm(act, P[f"cam{cam}.vis.w"]) + P[f"cam{cam}.vis.b"]
    feats = inp["features_buffer"][0].astype(np.float16)
    x[S.N_VIS:] = _mm(feats, P["temp.w"]) + P["temp.b"]
    return ((x + P["pos"]) + cond).astype(np.float32)


def attention(qkv, cfg):
    d, hd = cfg.d, cfg.hd
    q = qkv[:, :d].astype(np.float32)
    k = qkv[:, d:2 * d].astype(np.float32)
    v = qkv[:, 2 * d:].astype(np.float32)
    out = np.zeros((qkv.shape[0], d), np.float32)
    scale = np.float32(1.0 / math.sqrt(hd))
    for h in range(cfg.heads):
        sl = slice(h * hd, (h + 1) * hd)
        s = (q[:, sl] @ k[:, sl].T) * scale
        s = s - s.max(axis=-1, keepdims=True)
        p = np.exp(s)
        p = p / p.sum(axis=-1, keepdims=True)
        out[:, sl] = p @ v[:, sl]
    return out.astype(np.float16)


def layer(P, l, x, cfg):
    h = layernorm(x)
    qkv = (_mm(h, P[f"l{l}.qkv.w"]) + P[f"l{l}.qkv.b"]).astype(np.float16)
    o = attention(qkv, cfg)
    x = x + (_mm(o, P[f"l{l}.o.w"]) + P[f"l{l}.o.b"])
    h = layernorm(x)
    u = gelu(_mm(h, P[f"l{l}.fc1.w"]) + P[f"l{l}.fc1.b"]).astype(np.float16)
    return x + (_mm(u, P[f"l{l}.fc2.w"]) + P[f"l{l}.fc2.b"])


def heads(P, x):
    y = layernorm(x).astype(np.float32)
    feat = y.mean(axis=0).astype(np.float16)
    hid = np.tanh(_mm(feat[None], P["hid.w"]) + P["hid.b"]).astype(np.float16)
    z = np.maximum(_mm(hid, P["trunk.w"]) + P["trunk.b"], 0).astype(np.float16)
    hv = (_mm(z, P["heads.w"]) + P["heads.b"]).astype(np.float32)
    return np.concatenate([hv[0], hid[0].astype(np.float32)])


def forward(P, inp, cfg, trace=None):
    x = embed(P, inp, cfg)
    if trace is not None:
        trace["x0"] = x.copy()
    for l in range(cfg.layers):
        x = layer(P, l, x, cfg)
    if trace is not None:
        trace["xL"] = x.copy()
    return heads(P, x)


class Clip:
    """One clip's recurrent state + frame step (the oracle's run_frame)."""

    def __init__(self, cfg_name, seed, params=None):
        self.cfg = S.CONFIGS[cfg_name]
        self.P = params if params is not None else gen_params(self.cfg, seed)
        self.state = new_state()

    def run_frame(self, warped, packed, trace=None):
        inp = queue_step(self.state, warped, packed)
        if trace is not None:
            trace["inputs"] = inp
        return forward(self.P, inp, self.cfg, trace)
