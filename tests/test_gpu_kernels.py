"""GPU parity of the kernel-level entry points against the CPU oracle.

Config 1 (r_6_2 shape GEMM) is compared with the FFMA-chain oracle
(oracle/cref.c, the reference's bit-exact py-spec order) within a stated
reassociation tolerance; config 2 (r_32_32_3_12288_32 shape reduce) at its
full size against the C oracle; the zero-border gather bit for bit.
"""
import numpy as np
import pytest

from chestnut_b200 import DeviceBuffer, kernels
from oracle import border
from oracle import build as cref

pytestmark = pytest.mark.gpu

# f32 reassociation tolerance, relative to sum_k |a_k b_k| of each output
GEMM_RTOL = 5e-5


def _gemm(M, N, K, b_kmajor, bn=0, splits=0, seed=0, c_init=False):
    rs = np.random.default_rng(seed)
    A = (rs.standard_normal((M, K)) / np.sqrt(K)).astype(np.float16)
    B = (rs.standard_normal((K, N)) / np.sqrt(K)).astype(np.float16)
    Bst = np.ascontiguousarray(B.T) if b_kmajor else B
    C = rs.standard_normal((M, N)).astype(np.float32) if c_init else np.zeros((M, N), np.float32)
    dA, dB, dC = DeviceBuffer(A.nbytes).upload(A), DeviceBuffer(Bst.nbytes).upload(Bst), DeviceBuffer(C.nbytes)
    dC.upload(C)
    kernels.gemm_wmma_f16(dA.ptr, dB.ptr, dC.ptr, M, N, K, b_kmajor, bn, splits)
    kernels.synchronize()
    got = dC.download(np.float32, (M, N))
    assert kernels.device_error() == 0
    ref = cref.gemm_chain(A, Bst, C, b_kmajor)
    mag = np.abs(A.astype(np.float32)) @ np.abs(B.astype(np.float32))
    return got, ref, mag, (dA, dB, dC)


def _check(got, ref, mag):
    err = np.abs(got - ref)
    assert np.all(err <= GEMM_RTOL * mag + 1e-6), float((err / (mag + 1e-6)).max())


@pytest.mark.parametrize("b_kmajor", [1, 0])
@pytest.mark.parametrize("bn,splits", [(0, 0), (64, 6), (128, 8), (256, 1), (256, 8), (256, 3), (256, 16), (128, 12), (128, 1), (64, 3), (128, 5)])
def test_gemm_config1_full_shape(b_kmajor, bn, splits):
    got, ref, mag, _ = _gemm(768, 256, 6144, b_kmajor, bn, splits)
    _check(got, ref, mag)


@pytest.mark.parametrize("M,N,K,b_kmajor,bn,splits", [
    (88, 2048, 2048, 1, 128, 8),     # batch-1 transformer projection, partial M tile
    (1, 512, 2048, 1, 64, 4),        # heads: one row
    (200, 200, 64, 1, 64, 1),        # partial M and N tiles, single k-block
    (130, 72, 192, 0, 64, 3),        # MN-major B with partial tiles
    (704, 1536, 512, 1, 0, 0),       # batch-8 clip shape (39M qkv)
    (64, 2811, 1024, 1, 0, 0),       # odd N (heads output width)
    (1000, 32, 32, 1, 0, 0),         # K=32: half a k-block, zero-filled by TMA (39M stem 1x1 conv)
    (300, 64, 288, 1, 64, 3),        # K=288 = 4.5 k-blocks (39M stem 3x3 conv)
    (96, 40, 136, 0, 64, 2),         # MN-major B with a partial k-block
])
def test_gemm_edge_shapes(M, N, K, b_kmajor, bn, splits):
    got, ref, mag, _ = _gemm(M, N, K, b_kmajor, bn, splits, seed=M + N)
    _check(got, ref, mag)


def test_gemm_rejects_unsupported_tilings():
    from chestnut_b200 import ChestnutError
    dA, dB, dC = DeviceBuffer(768 * 6144 * 2), DeviceBuffer(256 * 6144 * 2), DeviceBuffer(768 * 256 * 4)
    with pytest.raises(ChestnutError, match="unsupported tiling"):
        kernels.gemm_wmma_f16(dA.ptr, dB.ptr, dC.ptr, 768, 256, 6144, 1, 96, 2)      # bn not 64/128/256
    with pytest.raises(ChestnutError, match="unsupported tiling"):
        kernels.gemm_wmma_f16(dA.ptr, dB.ptr, dC.ptr, 768, 256, 64, 1, 128, 2)       # more splits than k-blocks
    with pytest.raises(ChestnutError, match="unsupported tiling"):
        kernels.gemm_wmma_f16(dA.ptr, dB.ptr, dC.ptr, 768, 256, 6144, 1, 128, 17)    # cluster larger than 16
    assert kernels.device_error() == 0


def test_gemm_accumulates_onto_c():
    got, ref, mag, _ = _gemm(256, 128, 512, 1, 128, 2, c_init=True)
    _check(got, ref, mag)


def test_gemm_deterministic_split_k():
    rs = np.random.default_rng(9)
    M, N, K = 768, 256, 6144
    A = (rs.standard_normal((M, K)) / 78).astype(np.float16)
    B = (rs.standard_normal((N, K)) / 78).astype(np.float16)
    dA, dB = DeviceBuffer(A.nbytes).upload(A), DeviceBuffer(B.nbytes).upload(B)
    outs = []
    for _ in range(3):
        dC = DeviceBuffer(M * N * 4).zero()
        kernels.gemm_wmma_f16(dA.ptr, dB.ptr, dC.ptr, M, N, K, 1, 128, 8)
        kernels.synchronize()
        outs.append(dC.download(np.float32, (M, N)))
    assert np.array_equal(outs[0], outs[1]) and np.array_equal(outs[0], outs[2])


def _reduce_inputs(rows, length, seed):
    rs = np.random.default_rng(seed)
    x = np.empty((rows, length), np.float16)
    step = max(1, (1 << 26) // length)
    for r in range(0, rows, step):
        n = min(step, rows - r)
        x[r:r + n] = (rs.random((n, length), dtype=np.float32) * 2 - 1).astype(np.float16)
    w = (rs.random(length, dtype=np.float32) * 2 - 1).astype(np.float16)
    return x, w


def _reduce_tol(x, w):
    return 2e-6 * (np.abs(x.astype(np.float32)) @ np.abs(w.astype(np.float32))) + 1e-6


def test_reduce_config2_full_size():
    rows, length = 32 * 32 * 3, 12288 * 32
    x, w = _reduce_inputs(rows, length, 0)
    dx, dw, do = DeviceBuffer(x.nbytes).upload(x), DeviceBuffer(w.nbytes).upload(w), DeviceBuffer(rows * 4)
    kernels.reduce_rows_f16(dx.ptr, dw.ptr, do.ptr, rows, length)
    kernels.synchronize()
    got = do.download(np.float32, (rows,))
    ref = cref.reduce_rows(x, w)
    assert np.all(np.abs(got - ref) <= _reduce_tol(x, w))
    # determinism: a second launch is bit-identical
    kernels.reduce_rows_f16(dx.ptr, dw.ptr, do.ptr, rows, length)
    kernels.synchronize()
    assert np.array_equal(got, do.download(np.float32, (rows,)))


@pytest.mark.parametrize("rows,length,cpr", [(1, 8, 1), (7, 8 * 1000, 2), (33, 8 * 4097, 4), (5, 393216, 8),
                                             (64, 2056, 8)])
def test_reduce_small_and_ragged(rows, length, cpr):
    x, w = _reduce_inputs(rows, length, rows)
    dx, dw, do = DeviceBuffer(x.nbytes).upload(x), DeviceBuffer(w.nbytes).upload(w), DeviceBuffer(rows * 4)
    kernels.reduce_rows_f16(dx.ptr, dw.ptr, do.ptr, rows, length, cpr)
    kernels.synchronize()
    got = do.download(np.float32, (rows,))
    assert np.all(np.abs(got - cref.reduce_rows(x, w)) <= _reduce_tol(x, w))


@pytest.mark.parametrize("G,B,H,W,C", [(2, 1, 64, 128, 32), (2, 3, 8, 16, 64), (1, 1, 2, 2, 8), (2, 2, 4, 8, 512)])
def test_border_gather_bit_exact(G, B, H, W, C):
    rs = np.random.default_rng(H * W + C)
    act = rs.standard_normal((G, B, H, W, C)).astype(np.float16)
    Ho, Wo = H // 2, W // 2
    da = DeviceBuffer(act.nbytes).upload(act)
    do = DeviceBuffer(G * B * Ho * Wo * 9 * C * 2)
    kernels.border_gather_s2(da.ptr, G, B, H, W, C, do.ptr)
    kernels.synchronize()
    got = do.download(np.float16, (G, B * Ho * Wo, 9 * C))
    for g in range(G):
        ref = np.concatenate([border.im2col_s2(act[g, b]) for b in range(B)], 0)
        assert np.array_equal(got[g].view(np.uint16), ref.view(np.uint16))
