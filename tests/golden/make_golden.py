"""Generate the golden vectors under tests/golden (run: python tests/golden/make_golden.py).

The reference ships no golden data (its .gitignore drops *.npy/*.npz/*.json and
its cubins).  Its known-answer tests are hardware probes whose inputs and
expected outputs are defined in the probe sources; this script restates those
constructions independently of ``oracle/`` so that the oracle can be pinned
against them:

  wmma_kat.npz   consumer_probe.py:131-154 / ffma_probe.py:112-127: lane l
                 fragment element j holds f16 bits (l*8 + j + 1); A[l%16][kj]
                 = B[kj][l%16] = that value; expected D = A @ B (numpy f64);
                 the probe accepts max |gpu-ref| / max(1,|ref|) <= 1e-5.
                 A second case shifts the bits into the normal f16 range
                 (0x3C00 + l*8 + j + 1) so the check has teeth.
  mma_kat.npz    mma_probe.py:86-105: A[r][k] = f16 bits (r*16+k) (16x8),
                 B[k][n] = f16 bits (n*16+k) (8x8), expected D = A @ B.
  sampler_kat.json  research/probe_sampler.py:12-23,34: a 2x1 RGBA float
                 image holding 1..8 read with CLK_ADDRESS_CLAMP at
                 (-1,0), (2,0), (0,-1), (0,1), (0,0), (1,0).  OpenCL defines
                 the out-of-range reads as the zero border colour.
  queue_golden.npz  compile_modeld.py:166-176,199-213: a scripted sequence of
                 pushes through Tensor.cat-style shift queues, sampled with
                 buf[::4] and max over groups of 4, written out explicitly.
"""
import json
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def kj(t, j):  # consumer_probe.py:14-19
    if j < 4:
        return j if t < 16 else j + 4
    return j + 4 if t < 16 else j + 8


def wmma_case(offset):
    vbits = np.zeros((32, 8), np.uint16)
    for lane in range(32):
        for j in range(8):
            vbits[lane, j] = offset + lane * 8 + j + 1
    vf = vbits.view(np.float16).astype(np.float64)
    A = np.zeros((16, 16))
    Bm = np.zeros((16, 16))
    for lane in range(32):
        for j in range(8):
            k = kj(lane, j)
            A[lane % 16, k] = vf[lane, j]
            Bm[k, lane % 16] = vf[lane, j]
    D = A @ Bm
    dfrag = np.zeros((32, 8), np.float64)
    for lane in range(32):
        for e in range(8):
            dfrag[lane, e] = D[(lane // 16) * 8 + e, lane % 16]
    return vbits, dfrag


def mma_case():
    bits = np.arange(256, dtype=np.uint16)
    f = bits.view(np.float16).astype(np.float64)
    A = np.empty((16, 8))
    B = np.empty((8, 8))
    for r in range(16):
        for k in range(8):
            A[r, k] = f[r * 16 + k]
    for k in range(8):
        for n in range(8):
            B[k, n] = f[n * 16 + k]
    Ab = np.array([[r * 16 + k for k in range(8)] for r in range(16)], np.uint16)
    Bb = np.array([[n * 16 + k for n in range(8)] for k in range(8)], np.uint16)
    return Ab, Bb, A @ B


def queue_script(steps=11, seed=5):
    """Explicit shift queues: buf <- concat(buf[1:], new); sample as the model does."""
    rng = np.random.default_rng(seed)
    img_q = np.zeros((5, 6, 4, 8), np.uint8)          # small planes: semantics are shape-free
    desire_q = np.zeros((100, 1, 8), np.float32)
    feat_q = np.zeros((96, 1, 16), np.float32)
    pushes_img, pushes_des, pushes_feat = [], [], []
    exp_img, exp_des, exp_feat = [], [], []
    for _ in range(steps):
        f = rng.integers(0, 256, (1, 6, 4, 8), dtype=np.uint8)
        d = rng.standard_normal((1, 1, 8)).astype(np.float32)
        ft = rng.standard_normal((1, 1, 16)).astype(np.float32)
        img_q = np.concatenate([img_q[1:], f], 0)
        desire_q = np.concatenate([desire_q[1:], d], 0)
        feat_q = np.concatenate([feat_q[1:], ft], 0)
        s = img_q[::4]
        exp_img.append(s.reshape(-1, 4, 8)[None])                   # (1, 12, 4, 8)
        dd = desire_q.reshape(25, 4, 1, 8).max(1).reshape(25, 8)[None]
        exp_des.append(dd)
        exp_feat.append(feat_q[::4].reshape(24, 16)[None])
        pushes_img.append(f[0])
        pushes_des.append(d.reshape(8))
        pushes_feat.append(ft.reshape(16))
    return dict(push_img=np.array(pushes_img), push_desire=np.array(pushes_des), push_feat=np.array(pushes_feat),
                exp_img=np.array(exp_img), exp_desire=np.array(exp_des), exp_feat=np.array(exp_feat),
                final_img_q=img_q, final_desire_q=desire_q, final_feat_q=feat_q)


def main():
    a0, d0 = wmma_case(0)
    a1, d1 = wmma_case(0x3C00)
    np.savez(os.path.join(HERE, "wmma_kat.npz"), frag_bits_subnormal=a0, d_subnormal=d0, frag_bits_normal=a1,
             d_normal=d1)
    Ab, Bb, D = mma_case()
    np.savez(os.path.join(HERE, "mma_kat.npz"), a_bits=Ab, b_bits=Bb, d=D)
    sampler = {
        "image_rgba_2x1": [1, 2, 3, 4, 5, 6, 7, 8],
        "reads": [[-1, 0], [2, 0], [0, -1], [0, 1], [0, 0], [1, 0]],
        "expected": [[0, 0, 0, 0], [0, 0, 0, 0], [0, 0, 0, 0], [0, 0, 0, 0], [1, 2, 3, 4], [5, 6, 7, 8]],
    }
    with open(os.path.join(HERE, "sampler_kat.json"), "w") as f:
        json.dump(sampler, f, indent=1)
    np.savez(os.path.join(HERE, "queue_golden.npz"), **queue_script())


if __name__ == "__main__":
    main()
