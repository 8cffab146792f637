"""Output decode (oracle side, TEST INFRASTRUCTURE).

Restates the reference's host-side output parser ``Parser``
(``parse_model_outputs.py:1-120``) for one raw output vector per frame, in
numpy float32 as the reference computes it:

* ``safe_exp(x) = exp(min(x, 11))`` (``:4-6``);
* ``sigmoid(x) = 1 / (1 + safe_exp(-x))`` (``:8-9``);
* ``softmax`` over the last axis with the row max subtracted (``:11-18``);
* ``parse_mdn(in_N, out_N)`` (``:42-87``): each of max(in_N, 1) hypothesis
  rows is [mu n | log-std n | ... | out_N selection logits]; std =
  safe_exp(log-std); with in_N > 1 the selection logits are softmaxed across
  hypotheses, for out_N == 1 the hypotheses are reordered by weight,
  descending, and every output column takes the hypothesis of largest weight.

numpy's argsort of a short array is stable, so after ``[::-1]`` equal weights
rank the higher hypothesis index first; that is the tie rule here too.

A decode layout is a list of (kind, name, raw offset, raw length, in_N,
out_N, width): kind "mdn", "sigmoid" or "softmax" (softmax over consecutive
groups of ``width`` values, ``parse_categorical_crossentropy``'s last axis).
"""
import numpy as np

CLIP = np.float32(11.0)


def safe_exp(x):
    return np.exp(np.minimum(np.asarray(x, np.float32), CLIP)).astype(np.float32)


def sigmoid(x):
    return (np.float32(1.0) / (np.float32(1.0) + safe_exp(-np.asarray(x, np.float32)))).astype(np.float32)


def softmax(x, axis=-1):
    x = np.asarray(x, np.float32)
    x = x - np.max(x, axis=axis, keepdims=True)
    e = safe_exp(x)
    return (e / np.sum(e, axis=axis, keepdims=True, dtype=np.float32)).astype(np.float32)


def mdn(raw, in_n, out_n):
    """raw f32 [L] -> dict (weights [in_N, out_N] | hypotheses / stds_hypotheses
    [in_N, n] | mu / std [max(out_N,1), n]).  parse_model_outputs.py:42-87."""
    rows = max(in_n, 1)
    r = np.asarray(raw, np.float32).reshape(rows, -1)
    n = (r.shape[1] - out_n) // 2
    mu = r[:, :n].copy()
    std = safe_exp(r[:, n:2 * n])
    out = {}
    if in_n > 1:
        w = np.zeros((in_n, out_n), np.float32)
        for i in range(out_n):
            w[:, i - out_n] = softmax(r[:, i - out_n], axis=-1)
        if out_n == 1:
            idx = np.argsort(w[:, 0], kind="stable")[::-1]
            w, mu, std = w[idx], mu[idx], std[idx]
        out["weights"] = w
        out["hypotheses"] = mu
        out["stds_hypotheses"] = std
        fm = np.zeros((out_n, n), np.float32)
        fs = np.zeros((out_n, n), np.float32)
        for h in range(out_n):
            best = np.argsort(w[:, h], kind="stable")[::-1][0]
            fm[h] = mu[best]
            fs[h] = std[best]
        out["mu"], out["std"] = fm, fs
    else:
        out["mu"], out["std"] = mu, std
    return out


def decode(raw, layout):
    """Decode one frame's raw vector with a layout -> {name: array or dict}."""
    raw = np.asarray(raw, np.float32)
    res = {}
    for kind, name, off, length, in_n, out_n, width in layout:
        x = raw[off:off + length]
        if kind == "mdn":
            res[name] = mdn(x, in_n, out_n)
        elif kind == "sigmoid":
            res[name] = sigmoid(x)
        elif kind == "softmax":
            res[name] = softmax(x.reshape(-1, width), axis=-1).reshape(-1)
        else:
            raise ValueError(kind)
    return res


def flatten(decoded, layout):
    """The decoded values in the device decoder's output order (per field, in
    layout order): mdn -> weights, hypotheses, stds_hypotheses (in_N > 1 only),
    then mu, std; sigmoid / softmax -> the values."""
    parts = []
    for kind, name, *_ in layout:
        d = decoded[name]
        if kind == "mdn":
            for k in ("weights", "hypotheses", "stds_hypotheses", "mu", "std"):
                if k in d:
                    parts.append(d[k].reshape(-1))
        else:
            parts.append(d.reshape(-1))
    return np.concatenate(parts).astype(np.float32)
