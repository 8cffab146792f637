"""GPU parity of the frame engine against the oracle frame (configs 3/4).

Tolerances (per output head, against the oracle's fp32-accumulate frame):
|gpu - ref| <= 2e-2 + 1e-2 * |ref|.  Index / copy work (queues, hidden-state
carry, graph vs eager replay) is compared bit for bit.
"""
import numpy as np
import pytest

from chestnut_b200 import Engine
from oracle import model as omodel
from oracle import spec

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-2, 1e-2


def frame_inputs(rs, n):
    w = rs.integers(0, 256, (n, 2, 6, 128, 256), dtype=np.uint8)
    pk = np.zeros((n, 524), np.float32)
    for i in range(n):
        pk[i, rs.integers(0, 8)] = 1.0      # desire one-hot
        pk[i, 8 + rs.integers(0, 2)] = 1.0  # traffic convention one-hot
        pk[i, 10:12] = rs.standard_normal(2)
    return w, pk


def head_errors(got, ref):
    out = {}
    for name, sl in spec.out_slices().items():
        d = np.abs(got[sl] - ref[sl])
        out[name] = (float(d.max()), bool(np.all(d <= ATOL + RTOL * np.abs(ref[sl]))))
    return out


@pytest.fixture(scope="module")
def params39():
    return omodel.gen_params(spec.CONFIGS["39m"], 3)


@pytest.mark.parametrize("mode", ["persistent", "per-layer stem", "per-layer trunk", "per-layer"])
def test_39m_frames_match_oracle_with_hidden_carry(params39, mode, monkeypatch):
    # single-clip engines run the conv stem and the transformer as one
    # persistent kernel each unless CN_STEM=0 / CN_TRUNK=0 ("per-layer trunk"
    # is the combination batched clips run)
    trunk = mode in ("persistent", "per-layer stem")
    stem = mode in ("persistent", "per-layer trunk")
    monkeypatch.setenv("CN_TRUNK", "1" if trunk else "0")
    monkeypatch.setenv("CN_STEM", "1" if stem else "0")
    rs = np.random.default_rng(0)
    w, pk = frame_inputs(rs, 12)
    eng = Engine("39m", seed=3)
    names = [k["name"] for k in eng.kernel_list()]
    assert ("transformer_trunk" in names) == trunk
    assert ("conv_stem" in names) == stem
    clip = omodel.Clip("39m", 3, params39)
    pg, po = pk[0].copy(), pk[0].copy()
    for f in range(len(w)):
        pg[:12] = pk[f, :12]
        po[:12] = pk[f, :12]
        got = eng.run_frame(w[f], pg)
        ref = clip.run_frame(w[f], po)
        errs = head_errors(got, ref)
        assert all(ok for _, ok in errs.values()), (f, errs)
        pg[12:] = got[spec.out_slices()["hidden_state"]]   # video_check.py:60 carry, each side its own
        po[12:] = ref[spec.out_slices()["hidden_state"]]


def test_queue_state_bit_exact_teacher_forced(params39):
    rs = np.random.default_rng(1)
    w, pk = frame_inputs(rs, 7)
    pk[:, 12:] = rs.standard_normal((7, 512)).astype(np.float32)
    eng = Engine("39m", seed=3)
    clip = omodel.Clip("39m", 3, params39)
    for f in range(7):
        eng.run_frame(w[f], pk[f])
        from oracle.queues import step
        step(clip.state, w[f], pk[f])
    st = eng.get_state(0)
    for k in ("img_q", "big_img_q", "feat_q", "desire_q"):
        assert np.array_equal(st[k], clip.state[k]), k
    # set_state round trip: a fresh engine given this state continues identically
    eng2 = Engine("39m", seed=3)
    eng2.set_state(st)
    st2 = eng2.get_state(0)
    for k in ("img_q", "big_img_q", "feat_q", "desire_q"):
        assert np.array_equal(st2[k], st[k]), k
    a = eng.run_frame(w[0], pk[0])
    b = eng2.run_frame(w[0], pk[0])
    assert np.array_equal(a, b)


def test_graph_replay_equals_eager():
    rs = np.random.default_rng(2)
    w, pk = frame_inputs(rs, 4)
    g = Engine("39m", seed=5, use_graph=True)
    e = Engine("39m", seed=5, use_graph=False)
    for f in range(4):
        assert np.array_equal(g.run_frame(w[f], pk[f]), e.run_frame(w[f], pk[f]))


def test_device_hidden_carry_equals_host_carry():
    rs = np.random.default_rng(3)
    w, pk = frame_inputs(rs, 6)
    host = Engine("39m", seed=7)
    dev = Engine("39m", seed=7, carry_hidden=True)
    ph = pk[0].copy()
    ph[12:] = 0
    for f in range(6):
        ph[:12] = pk[f, :12]
        pd = pk[f].copy()
        pd[12:] = 12345.0          # ignored in device-carry mode
        a = host.run_frame(w[f], ph)
        b = dev.run_frame(w[f], pd)
        assert np.array_equal(a, b), f
        ph[12:] = a[spec.out_slices()["hidden_state"]]


def test_batched_clips_match_single_clip_engines():
    rs = np.random.default_rng(4)
    n, B = 3, 4
    w = rs.integers(0, 256, (n, B, 2, 6, 128, 256), dtype=np.uint8)
    pk = np.zeros((n, B, 524), np.float32)
    pk[:, :, 8] = 1
    batched = Engine("39m", seed=2, batch=B)
    singles = [Engine("39m", seed=2) for _ in range(B)]
    for f in range(n):
        ob = batched.run_frame(w[f], pk[f])
        for b in range(B):
            os_ = singles[b].run_frame(w[f, b], pk[f, b])
            errs = head_errors(ob[b], os_)
            assert all(ok for _, ok in errs.values()), (f, b, errs)


@pytest.mark.parametrize("B", [5, 16])
def test_batched_persistent_stem_matches_per_layer_stem(B, monkeypatch):
    # 5 clips: ragged tiles (stage 4's 160 rows, 120 temporal-token rows, 5
    # cond rows) and 128-row tiles spanning several images; 16: whole tiles
    rs = np.random.default_rng(11)
    n = 3
    w = rs.integers(0, 256, (n, B, 2, 6, 128, 256), dtype=np.uint8)
    pk = np.zeros((n, B, 524), np.float32)
    pk[:, :, 8] = 1
    pk[:, :, 10:12] = rs.standard_normal((n, B, 2))
    for f in range(n):
        for b in range(B):
            pk[f, b, (f + b) % 8] = 1
    a, c = Engine("39m", seed=7, batch=B), Engine("39m", seed=7, batch=B, use_graph=False)
    assert "conv_stem" in [k["name"] for k in a.kernel_list()]
    monkeypatch.setenv("CN_STEM", "0")
    ref = Engine("39m", seed=7, batch=B)
    assert "conv_stem" not in [k["name"] for k in ref.kernel_list()]
    for f in range(n):
        oa, oc, orf = a.run_frame(w[f], pk[f]), c.run_frame(w[f], pk[f]), ref.run_frame(w[f], pk[f])
        assert np.array_equal(oa, oc), f          # graph replay == eager, run to run identical
        for b in range(B):
            errs = head_errors(oa[b], orf[b])
            assert all(ok for _, ok in errs.values()), (f, b, errs)


def test_kernel_list_describes_the_frame(monkeypatch):
    # the conv stem with the cond and token embeddings as one persistent
    # launch; the transformer, the final LayerNorm, the token mean and the
    # three head products as another
    eng = Engine("39m", seed=0)
    ks = eng.kernel_list()
    names = [k["name"] for k in ks]
    assert names == ["queue_push", "border_gather0", "conv_stem", "transformer_trunk"]
    assert eng.info()["n_kernels"] == len(ks)
    # per-layer stem: 10 conv GEMMs (4 im2col gathers) + cond / tokens 3 GEMMs
    monkeypatch.setenv("CN_STEM", "0")
    names = [k["name"] for k in Engine("39m", seed=0).kernel_list()]
    assert sum(n.startswith("gemm_tc") for n in names) == 10 + 3
    assert sum(n.startswith("border_gather_s2") for n in names) == 4
    assert names.count("transformer_trunk") == 1
    assert "token_mean_pool" not in names and "layernorm:final" not in names
    # per-layer kernels: 4 GEMMs per layer, then final LN, pool and 3 head GEMMs
    monkeypatch.setenv("CN_TRUNK", "0")
    names = [k["name"] for k in Engine("39m", seed=0).kernel_list()]
    assert sum(n.startswith("gemm_tc") for n in names) == 10 + 3 + 4 * 4 + 3
    assert "transformer_trunk" not in names
    assert "token_mean_pool" in names and "layernorm:final" in names
    # the persistent stem before the per-layer transformer kernels
    monkeypatch.delenv("CN_STEM")
    names = [k["name"] for k in Engine("39m", seed=0).kernel_list()]
    assert names[:3] == ["queue_push", "border_gather0", "conv_stem"]
    assert sum(n.startswith("gemm_tc") for n in names) == 4 * 4 + 3
    monkeypatch.delenv("CN_TRUNK")
    # batched clips: the persistent stem, then the per-layer transformer kernels
    names = [k["name"] for k in Engine("39m", seed=0, batch=3).kernel_list()]
    assert names[:3] == ["queue_push", "border_gather0", "conv_stem"]
    assert "transformer_trunk" not in names and not any(n.startswith("border_gather_s2") for n in names)


@pytest.mark.parametrize("cfg", ["39m", "1b"])
def test_persistent_kernels_are_deterministic_and_match_per_layer_kernels(cfg, monkeypatch):
    rs = np.random.default_rng(8)
    w, pk = frame_inputs(rs, 4)
    a, b = Engine(cfg, seed=5), Engine(cfg, seed=5, use_graph=False)
    monkeypatch.setenv("CN_TRUNK", "0")
    monkeypatch.setenv("CN_STEM", "0")
    ref = Engine(cfg, seed=5)
    for f in range(4):
        oa, ob, orf = a.run_frame(w[f], pk[f]), b.run_frame(w[f], pk[f]), ref.run_frame(w[f], pk[f])
        assert np.array_equal(oa, ob), f          # graph replay == eager, run to run identical
        errs = head_errors(oa, orf)
        assert all(ok for _, ok in errs.values()), (f, errs)
    assert a.run_frame(w[0], pk[0]).shape == (spec.N_OUT,)


@pytest.mark.slow
def test_1b_frames_match_oracle():
    rs = np.random.default_rng(6)
    w, pk = frame_inputs(rs, 3)
    eng = Engine("1b", seed=1)
    clip = omodel.Clip("1b", 1)
    pg, po = pk[0].copy(), pk[0].copy()
    for f in range(3):
        pg[:12] = pk[f, :12]
        po[:12] = pk[f, :12]
        got = eng.run_frame(w[f], pg)
        ref = clip.run_frame(w[f], po)
        errs = head_errors(got, ref)
        assert all(ok for _, ok in errs.values()), (f, errs)
        pg[12:] = got[spec.out_slices()["hidden_state"]]
        po[12:] = ref[spec.out_slices()["hidden_state"]]


def test_staged_input_equals_run_frame():
    # cn_stage_input / cn_run_staged: the next frame's upload overlaps the
    # current frame; the outputs are those of cn_run_frame, bit for bit
    from chestnut_b200._lib import ChestnutError
    rs = np.random.default_rng(14)
    B = 2
    w = rs.integers(0, 256, (5, B, 2, 6, 128, 256), dtype=np.uint8)
    pk = np.zeros((5, B, 524), np.float32)
    pk[:, :, 3] = 1.0
    pk[:, :, 8] = 1.0
    a, b = Engine("39m", seed=4, batch=B), Engine("39m", seed=4, batch=B)
    with pytest.raises(ChestnutError):
        b.run_staged(pk[0])                      # nothing staged yet
    b.stage(w[0])
    for f in range(5):
        if f + 1 < 5:
            b.stage(w[f + 1])
        if f == 0:
            with pytest.raises(ChestnutError):
                b.stage(w[0])                    # at most two inputs ahead
        oa = a.run_frame(w[f], pk[f])
        ob = b.run_staged(pk[f])
        assert np.array_equal(oa, ob), f


def test_pipelined_clip_runner_equals_run_frame_runner():
    # device-carried hidden state + queued frames (cn_run_staged_async /
    # cn_wait_output) give the host-carry run_frame results bit for bit
    from chestnut_b200 import PinnedArray, clips
    rs = np.random.default_rng(21)
    pool = rs.integers(0, 256, (3, 2, 6, 128, 256), dtype=np.uint8)
    pins = []

    def alloc(shape, dtype):
        pins.append(PinnedArray(shape, dtype))
        return pins[-1].array

    staged = {}

    def batch_source(group, f):
        key = (tuple(group), f % 3)
        if key not in staged:
            w = alloc((len(group), 2, 6, 128, 256), np.uint8)
            w[:] = np.stack([pool[(c + f) % 3] for c in group])
            pk = np.zeros((len(group), 524), np.float32)
            for i, c in enumerate(group):
                pk[i, c % 8] = 1.0
                pk[i, 8] = 1.0
            staged[key] = (w, pk)
        w, pk = staged[key]
        return w, pk.copy()

    group = [0, 1, 2]
    ref = clips.run_rank(lambda n: Engine("39m", seed=6, batch=n), None, group, 7, 3, batch_source)
    got = clips.run_rank_pipelined(lambda n: Engine("39m", seed=6, batch=n, carry_hidden=True), group, 7, 3,
                                   batch_source, alloc)
    for c in group:
        assert np.array_equal(ref[c][0], got[c][0]), c
        assert np.array_equal(ref[c][1], got[c][1]), c
    for p in pins:
        p.free()
