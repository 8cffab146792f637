"""RDNA4 ((16,16,16), half, 'AMD', 32) WMMA semantics (oracle side, test infrastructure).

Restates the fragment maps of ``run_pinned2.py:100-117`` (and the probes'
``kj`` map, ``consumer_probe.py:14-19``) and the FFMA reference consumer
(``run_pinned2.py:158-192``): D = C + sum_k A[m][k] * B[k][n] as an
``fma.rn.f32`` chain in k order 0..15 whose first step adds C.  Because an
f16*f16 product is exact in f32, ``fma.rn(a, b, c) == f32(a*b) + c`` in numpy,
so the chain is reproduced bit for bit (the reference notes the FFMA consumer
is bit-exact with tinygrad's Python spec, ``NOTES.md:27-33``).

A K-chained GEMM (config 1: 384 WMMA steps of K=16, C zero-initialised) is
therefore one sequential f32 accumulation over k = 0..K-1; ``gemm_chain`` does
exactly that.  The tcgen05 engine reassociates the sum (like the reference's
mma.sync consumer) and is compared within a stated tolerance.
"""
import numpy as np


def kj(lane, j):
    """Lane ``lane`` fragment element ``j`` -> k index (consumer_probe.py:14-19)."""
    if j < 4:
        return j if lane < 16 else j + 4
    return j + 4 if lane < 16 else j + 8


def frags_to_matrices(a_frag, b_frag):
    """a_frag, b_frag: f16 [32, 8] per-lane fragments -> A [16,16], B [16,16]."""
    A = np.zeros((16, 16), np.float16)
    B = np.zeros((16, 16), np.float16)
    for lane in range(32):
        for j in range(8):
            k = kj(lane, j)
            A[lane % 16, k] = a_frag[lane, j]
            B[k, lane % 16] = b_frag[lane, j]
    return A, B


def d_to_frag(D):
    """D [16,16] -> per-lane f32 [32, 8]: lane l elem e = D[(l//16)*8+e][l%16]."""
    out = np.zeros((32, 8), np.float32)
    for lane in range(32):
        for e in range(8):
            out[lane, e] = D[(lane // 16) * 8 + e, lane % 16]
    return out


def tile_ffma(A, B, C):
    """One WMMA with the FFMA reference consumer: f32 chain over k=0..15."""
    acc = C.astype(np.float32).copy()
    Af = A.astype(np.float32)
    Bf = B.astype(np.float32)
    for k in range(16):
        acc = (np.outer(Af[:, k], Bf[k, :]).astype(np.float32) + acc).astype(np.float32)
    return acc


def consume(a_frag, b_frag, c_frag):
    """Lane-level WMMA: fragments in, D fragment out (FFMA order)."""
    A, B = frags_to_matrices(a_frag, b_frag)
    C = np.zeros((16, 16), np.float32)
    for lane in range(32):
        for e in range(8):
            C[(lane // 16) * 8 + e, lane % 16] = c_frag[lane, e]
    return d_to_frag(tile_ffma(A, B, C))


def gemm_chain(A, B, C=None):
    """C + A @ B with A f16 [M,K], B f16 [K,N]; K consumed in 16-wide WMMA steps,
    each step an FFMA chain continuing from the previous accumulator."""
    M, K = A.shape
    N = B.shape[1]
    assert K % 16 == 0
    acc = np.zeros((M, N), np.float32) if C is None else np.asarray(C, np.float32).copy()
    Af = A.astype(np.float32)
    Bf = B.astype(np.float32)
    for k in range(K):
        acc += np.outer(Af[:, k], Bf[k, :])   # product exact in f32, one rounding per add
    return acc
