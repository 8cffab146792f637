"""GPU test of cn_gemm_wmma_f16_noalloc, the GEMM entry point for callers that
cannot allocate device memory (their GPU memory belongs to another allocator,
or an allocation's implicit synchronisation is not allowed where they call).

It keeps its split-K scratch in a static device array inside the library, so
the only buffers are the caller's A, B and C.  The test calls it through the C
ABI twice in a row on the same C (C += A*B each time) and compares C with the
existing entry point cn_gemm_wmma_f16 run the same way, within the GEMM
reassociation tolerance of the kernel tests (5e-5 of sum |a*b| per output
against the oracle, so 1e-4 between two GPU results).  It also checks that
sizes beyond the static array are refused.  The file name makes pytest collect
it last.
"""
import numpy as np
import pytest

from chestnut_b200 import DeviceBuffer, _lib, kernels

pytestmark = pytest.mark.gpu

RTOL = 1e-4
CN_ERR_ARG = -2


@pytest.mark.parametrize("M,N,K,splits", [
    (768, 256, 6144, 8),    # config-1 shape
    (768, 256, 6144, 1),    # no split: direct accumulate
    (200, 130, 200, 3),     # partial M / N tiles, partial last k-block
])
def test_noalloc_gemm_matches_existing_entry_point_on_two_calls(M, N, K, splits):
    rs = np.random.default_rng(M + N + K + splits)
    A = (rs.standard_normal((M, K)) / np.sqrt(K)).astype(np.float16)
    Bt = (rs.standard_normal((N, K)) / np.sqrt(K)).astype(np.float16)   # B as [N][K]
    C0 = rs.standard_normal((M, N)).astype(np.float32)
    dA, dB = DeviceBuffer(A.nbytes).upload(A), DeviceBuffer(Bt.nbytes).upload(Bt)
    ref_c, got_c = DeviceBuffer(C0.nbytes).upload(C0), DeviceBuffer(C0.nbytes).upload(C0)
    L = _lib.lib()
    mag = np.abs(A.astype(np.float32)) @ np.abs(Bt.astype(np.float32)).T
    for call in range(2):
        kernels.gemm_wmma_f16(dA.ptr, dB.ptr, ref_c.ptr, M, N, K, 1)
        rc = L.cn_gemm_wmma_f16_noalloc(dA.ptr, dB.ptr, got_c.ptr, M, N, K, splits, None)
        assert rc == 0, _lib.lib().cn_last_error()
        kernels.synchronize()
        assert kernels.device_error() == 0
        ref = ref_c.download(np.float32, (M, N))
        got = got_c.download(np.float32, (M, N))
        err = np.abs(got - ref)
        assert np.all(err <= RTOL * (call + 1) * mag + 1e-5), (call, float((err / (mag + 1e-6)).max()))


def test_noalloc_gemm_refuses_sizes_beyond_its_static_scratch():
    L = _lib.lib()
    a = DeviceBuffer(256)
    # 4096 x 4096 output x 16 splits needs 1 GiB of partial tiles
    assert L.cn_gemm_wmma_f16_noalloc(a.ptr, a.ptr, a.ptr, 4096, 4096, 4096, 16, None) == CN_ERR_ARG
    assert b"static scratch" in L.cn_last_error()
    # 33 x 33 = 1089 output tiles with splits > 1: more tiles than the scratch has counters
    assert L.cn_gemm_wmma_f16_noalloc(a.ptr, a.ptr, a.ptr, 4224, 4224, 128, 2, None) == CN_ERR_ARG
    assert b"tile limit" in L.cn_last_error()
    assert L.cn_gemm_wmma_f16_noalloc(a.ptr, a.ptr, a.ptr, 128, 128, 64, 2, None) == CN_ERR_ARG  # splits > K/64
