"""CPU checks of the oracle against the reference-derived golden vectors."""
import json
import os

import numpy as np
import pytest

from oracle import border, build, queues, rng, spec, wmma


def test_wmma_kat_consumer_probe(golden_dir):
    """consumer_probe.py / ffma_probe.py known answers through the oracle's
    fragment maps and FFMA chain."""
    z = np.load(os.path.join(golden_dir, "wmma_kat.npz"))
    for case in ("subnormal", "normal"):
        bits = z[f"frag_bits_{case}"]
        frag = bits.view(np.float16)
        d = wmma.consume(frag, frag, np.zeros((32, 8), np.float32))
        ref = z[f"d_{case}"]
        rel = np.abs(d - ref) / np.maximum(1.0, np.abs(ref))
        assert rel.max() <= 1e-5          # the probe's own criterion
        # and, stronger: f32 accumulation of exact products, relative to scale
        assert np.abs(d - ref).max() <= 1e-6 * max(1.0, np.abs(ref).max()) + 1e-30


def test_wmma_kat_mma_probe(golden_dir):
    z = np.load(os.path.join(golden_dir, "mma_kat.npz"))
    A = z["a_bits"].view(np.float16)
    B = z["b_bits"].view(np.float16)
    Ap = np.zeros((16, 16), np.float16)
    Bp = np.zeros((16, 16), np.float16)
    Ap[:, :8] = A
    Bp[:8, :8] = B
    D = wmma.tile_ffma(Ap, Bp, np.zeros((16, 16), np.float32))[:, :8]
    assert np.abs(D - z["d"]).max() <= 0.5     # mma_probe.py:99 tolerance
    assert np.abs(D - z["d"]).max() <= 1e-6 * np.abs(z["d"]).max()


def test_fragment_map_roundtrip():
    rs = np.random.default_rng(0)
    A = rs.standard_normal((16, 16)).astype(np.float16)
    B = rs.standard_normal((16, 16)).astype(np.float16)
    af = np.zeros((32, 8), np.float16)
    bf = np.zeros((32, 8), np.float16)
    for lane in range(32):
        for j in range(8):
            k = wmma.kj(lane, j)
            af[lane, j] = A[lane % 16, k]
            bf[lane, j] = B[k, lane % 16]
    A2, B2 = wmma.frags_to_matrices(af, bf)
    assert np.array_equal(A2, A) and np.array_equal(B2, B)
    # every (row, k) covered exactly once across the 32 lanes
    cover = np.zeros((16, 16), int)
    for lane in range(32):
        for j in range(8):
            cover[lane % 16, wmma.kj(lane, j)] += 1
    assert (cover == 1).all()


def test_sampler_kat(golden_dir):
    kat = json.load(open(os.path.join(golden_dir, "sampler_kat.json")))
    img = np.array(kat["image_rgba_2x1"], np.float32).reshape(1, 2, 4)   # (A=1 row, B=2, C=4)
    for (x, y), exp in zip(kat["reads"], kat["expected"]):
        assert border.read_texel(img, y, x).tolist() == exp


def test_queue_golden(golden_dir):
    z = np.load(os.path.join(golden_dir, "queue_golden.npz"))
    img_q = np.zeros((5, 6, 4, 8), np.uint8)
    des_q = np.zeros((100, 1, 8), np.float32)
    feat_q = np.zeros((96, 1, 16), np.float32)
    for i in range(len(z["push_img"])):
        got = queues.shift_and_sample(img_q, z["push_img"][i][None], queues.sample_skip)
        assert np.array_equal(got, z["exp_img"][i])
        got = queues.shift_and_sample(des_q, z["push_desire"][i].reshape(1, 1, 8), queues.sample_desire)
        assert np.array_equal(got, z["exp_desire"][i])
        got = queues.shift_and_sample(feat_q, z["push_feat"][i].reshape(1, 1, 16), queues.sample_skip)
        assert np.array_equal(got, z["exp_feat"][i])
    assert np.array_equal(img_q, z["final_img_q"])
    assert np.array_equal(des_q, z["final_desire_q"])
    assert np.array_equal(feat_q, z["final_feat_q"])


def test_packed_split():
    p = np.arange(524, dtype=np.float32)
    d, tc, at, pf = queues.split_packed(p)
    assert d.tolist() == list(range(8)) and tc.tolist() == [8, 9] and at.tolist() == [10, 11]
    assert pf[0] == 12 and pf.size == 512


def test_rng_c_matches_numpy():
    for tid, bound, f16 in ((3, 0.05, True), (9, 0.5, False), (17, 1e-4, True), (2, 3.0, True)):
        a = rng.fill(11, tid, 1 << 18, bound, np.float16 if f16 else np.float32)
        b = build.fill(11, tid, 1 << 18, bound, f16)
        assert np.array_equal(a.view(np.uint8), b.view(np.uint8))


def test_rng_uniform_range_and_exactness():
    u = rng.uniform(1, 2, 0, 1 << 16)
    assert u.min() >= -1.0 and u.max() < 1.0
    m = (u.astype(np.float64) + 1.0) * 2 ** 23
    assert np.array_equal(m, np.round(m))


def test_gemm_chain_c_vs_numpy():
    rs = np.random.default_rng(1)
    A = (rs.standard_normal((40, 64)) / 8).astype(np.float16)
    B = (rs.standard_normal((64, 24)) / 8).astype(np.float16)
    C0 = rs.standard_normal((40, 24)).astype(np.float32)
    ref = wmma.gemm_chain(A, B, C0)
    got = build.gemm_chain(A, B, C0, b_kmajor=False)
    assert np.array_equal(ref, got)                      # same chain, bit for bit
    got_k = build.gemm_chain(A, np.ascontiguousarray(B.T), C0, b_kmajor=True)
    assert np.array_equal(ref, got_k)


def test_reduce_c_vs_numpy():
    rs = np.random.default_rng(2)
    x = rs.uniform(-1, 1, (12, 1024)).astype(np.float16)
    w = rs.uniform(-1, 1, 1024).astype(np.float16)
    got = build.reduce_rows(x, w)
    ref = (x.astype(np.float64) * w.astype(np.float64)).sum(1)
    assert np.abs(got - ref).max() <= 1e-5 * np.abs(x.astype(np.float64) * w).sum(1).max()


def test_im2col_border_matches_texel_rule():
    rs = np.random.default_rng(3)
    act = rs.standard_normal((6, 10, 8)).astype(np.float16)
    cols = border.im2col_s2(act)
    C = 8
    for oy in range(3):
        for ox in range(5):
            row = cols[oy * 5 + ox]
            for tap in range(9):
                y, x = 2 * oy + tap // 3 - 1, 2 * ox + tap % 3 - 1
                exp = border.read_texel(act, y, x)
                assert np.array_equal(row[tap * C:(tap + 1) * C], exp)


def test_im2col_frame_normalisation():
    img = np.arange(12 * 128 * 256, dtype=np.int64).reshape(12, 128, 256) % 256
    cols = border.im2col_frame(img.astype(np.uint8))
    assert cols.shape == (64 * 128, 128)
    assert (cols[:, 108:] == 0).all()
    # interior tap 4 (centre) of position (1, 1) reads texel (2, 2) of every plane
    row = cols[1 * 128 + 1]
    exp = ((img[:, 2, 2].astype(np.float32) - 128) / 64).astype(np.float16)
    assert np.array_equal(row[4 * 12:5 * 12], exp)
    # corner position (0, 0) tap 0 is out of range -> zeros
    assert (cols[0, 0:12] == 0).all()


@pytest.mark.parametrize("name", ["39m", "1b"])
def test_spec_param_counts(name):
    cfg = spec.CONFIGS[name]
    n = spec.n_params(cfg)
    per_layer = 4 * cfg.d * cfg.d + 2 * cfg.d * cfg.mlp
    assert n > cfg.layers * per_layer
    if name == "1b":
        assert 1.0e9 < n < 1.05e9


def test_out_slices_layout():
    s = spec.out_slices()
    assert s["plan"] == slice(0, 2475) and s["hidden_state"] == slice(2811, 3323)
    assert spec.N_OUT == 3323
