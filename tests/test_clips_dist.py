"""CPU tests of the clip-sharding host logic, with world_size-2 gloo ranks.

A fake engine stands in for the GPU: it is a deterministic function of the
frame inputs and the carried hidden state, so a sharded run must reproduce the
single-process run bit for bit.  The clip-end gather goes through a gloo
transport with the same ``allgather`` contract as clips.NcclGather (which
needs GPUs); the NCCL library itself is checked for its exports and its
argument errors here, and run for real by the multi-GPU bench.
"""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from chestnut_b200 import clips

N_OUT = 3323


class FakeEngine:
    def __init__(self, batch):
        self.batch = batch

    def run_frame(self, warped, packed):
        w = warped.reshape(self.batch, -1).astype(np.float64)
        h = packed[:, 12:].astype(np.float64)
        base = w[:, ::4097][:, :N_OUT - 512].mean(axis=1, keepdims=True) / 255.0
        head = np.tile(base, (1, N_OUT - 512)) + np.arange(N_OUT - 512) * 1e-4
        hid = np.tanh(0.5 * h + base)
        return np.concatenate([head, hid], axis=1).astype(np.float32)


def frame_source(clip, frame):
    rs = np.random.default_rng(1000 * clip + frame)
    w = rs.integers(0, 256, (2, 6, 128, 256), dtype=np.uint8)
    pk = np.zeros(524, np.float32)
    pk[clip % 8] = 1.0
    pk[8] = 1.0
    return w, pk


def test_assign_round_robin_covers_every_clip_once():
    n, world = 64, 8
    owned = [clips.assign(n, world, r) for r in range(world)]
    flat = sorted(c for o in owned for c in o)
    assert flat == list(range(n))
    assert all(len(o) == n // world for o in owned)
    assert clips.batches(owned[0], 8) == [owned[0]]
    assert clips.batches(list(range(10)), 4) == [[0, 1, 2, 3], [4, 5, 6, 7], [8, 9]]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class GlooTransport:
    """clips.NcclGather's allgather contract over a gloo process group."""

    def __init__(self, dist):
        self.dist = dist

    def allgather(self, arr):
        import torch
        t = torch.from_numpy(np.ascontiguousarray(arr, np.float64))
        parts = [torch.zeros_like(t) for _ in range(self.dist.get_world_size())]
        self.dist.all_gather(parts, t)
        return torch.stack(parts).numpy()


def _rank_main(rank, world, port, n_clips, n_frames, batch, out_path):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    mine = clips.assign(n_clips, world, rank)
    res = clips.run_rank(FakeEngine, frame_source, mine, n_frames, batch)
    sums, finals = clips.gather(res, n_clips, n_frames, N_OUT, GlooTransport(dist))
    if rank == 0:
        np.savez(out_path, sums=sums, finals=finals)
    dist.barrier()
    dist.destroy_process_group()


def test_sharded_run_equals_single_process(tmp_path):
    n_clips, n_frames, batch, world = 6, 4, 2, 2
    ref = clips.run_rank(FakeEngine, frame_source, list(range(n_clips)), n_frames, batch)
    ref_s, ref_f = clips.gather(ref, n_clips, n_frames, N_OUT, None)
    out_path = str(tmp_path / "gathered.npz")
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, n_clips, n_frames, batch, out_path))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    z = np.load(out_path)
    assert np.array_equal(z["sums"], ref_s)
    assert np.array_equal(z["finals"], ref_f)


def test_batching_does_not_change_results():
    a = clips.run_rank(FakeEngine, frame_source, [0, 1, 2], 3, 1)
    b = clips.run_rank(FakeEngine, frame_source, [0, 1, 2], 3, 3)
    for c in (0, 1, 2):
        assert np.array_equal(a[c][0], b[c][0]) and np.array_equal(a[c][1], b[c][1])


def test_comm_library_exports_and_argument_errors():
    import ctypes
    from chestnut_b200.clips import comm_lib
    L = comm_lib()
    v = ctypes.c_int(0)
    assert L.cn_comm_nccl_version(ctypes.byref(v)) == 0 and v.value >= 22000
    assert L.cn_comm_unique_id(None) == -2
    h = ctypes.c_void_p()
    assert L.cn_comm_init(ctypes.byref(h), 0, 2, 5, b"x" * 128, 1000) == -2   # rank outside [0, nranks)
    assert b"bad arguments" in L.cn_comm_last_error()
    assert L.cn_comm_allgather_f64(None, None, None, 1, 1000) == -2
    assert L.cn_comm_destroy(None) == 0
    hdr = open(os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include",
                            "chestnut_comm.h")).read()
    import re
    for name in re.findall(r"^int (cn_comm_\w+)\(", hdr, re.M):
        assert hasattr(L, name), name


class FakeQueuedEngine(FakeEngine):
    """FakeEngine with the queued interface: staged inputs, the hidden state
    carried on the 'device' (the previous output), outputs written into the
    caller's buffers only when waited for, as the asynchronous copies would."""

    def __init__(self, batch):
        super().__init__(batch)
        self.staged, self.queued = [], []
        self.prev = np.zeros((batch, N_OUT), np.float32)

    def reset(self):
        self.prev = np.zeros((self.batch, N_OUT), np.float32)

    def stage(self, warped):
        assert len(self.staged) < 2
        self.staged.append(np.array(warped, copy=True))

    def run_staged_async(self, packed, out):
        assert len(self.queued) < 2
        pk = np.array(packed, copy=True)
        pk[:, 12:] = self.prev[:, -512:]
        res = self.run_frame(self.staged.pop(0), pk)
        self.prev = res
        self.queued.append((out, res))

    def wait_output(self):
        out, res = self.queued.pop(0)
        out[:] = res


def test_pipelined_runner_equals_host_carry_runner():
    group = [3, 5, 8, 11, 12]
    cache = {}

    def batch_source(g, f):
        key = (tuple(g), f)
        if key not in cache:
            ws, pks = zip(*(frame_source(c, f) for c in g))
            cache[key] = (np.stack(ws), np.stack(pks))
        w, pk = cache[key]
        return w, pk.copy()

    ref = clips.run_rank(FakeEngine, None, group, 6, 2, batch_source)
    got = clips.run_rank_pipelined(FakeQueuedEngine, group, 6, 2, batch_source, lambda s, d: np.zeros(s, d))
    assert sorted(ref) == sorted(got) == sorted(group)
    for c in group:
        assert np.array_equal(ref[c][0], got[c][0]), c
        assert np.array_equal(ref[c][1], got[c][1]), c
