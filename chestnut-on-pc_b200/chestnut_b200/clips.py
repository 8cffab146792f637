"""Clip sharding across GPUs (one process per GPU).

Independent clips -- each with its own recurrent state (queues + hidden state)
-- are the only axis the frame path shards on: clip c runs on rank c % world,
``batch`` clips per engine launch.  No collective runs on the per-frame path;
each rank's per-clip results are gathered to every rank (rank 0 reports) once,
at clip end, through a transport: ``NcclGather`` drives NCCL from C++
(libcncomm.so, include/chestnut_comm.h) over NVLink; anything with the same
``allgather`` method (a test's gloo transport, say) works too.  The reference
has no multi-GPU path; this follows the clip-parallel plan of its
``video_check.py:50-94`` loop (per clip: frames -> run_frame -> carried hidden
state -> per-frame rows).  No PyTorch here.
"""
import ctypes
import os

import numpy as np

FRAME_OUT = 3323  # floats of one frame's flat output (plan | lane_lines | lead | hidden_state)


def assign(n_clips, world, rank):
    """Clip ids owned by `rank` (round robin)."""
    return [c for c in range(n_clips) if c % world == rank]


def batches(clips, batch):
    """Split a rank's clip list into launch batches of at most `batch` clips."""
    return [clips[i:i + batch] for i in range(0, len(clips), batch)]


def run_rank(engine_factory, frame_source, clips, n_frames, batch, batch_source=None):
    """Run this rank's clips: returns {clip: (per-frame checksum f64[n_frames], final output f32[N_OUT])}.

    engine_factory(batch) -> object with run_frame(warped[B,2,6,128,256], packed[B,524]) -> out[B,N_OUT];
    frame_source(clip, frame) -> (warped u8[2,6,128,256], packed f32[524]) with packed[12:] ignored
    (the hidden state is carried here exactly as video_check.py:60 does);
    batch_source(group, frame), when given, returns the whole batch at once
    (warped u8[B,2,6,128,256], packed f32[B,524]) so callers can pre-assemble
    inputs; with an engine that stages inputs (stage / run_staged), the next
    frame's warped batch is then uploaded while the current frame runs (the
    warped bytes do not depend on the carried hidden state).
    """
    results = {}
    engines = {}
    for group in batches(clips, batch):
        B = len(group)
        eng = engines.get(B)
        if eng is None:
            eng = engines[B] = engine_factory(B)
        elif hasattr(eng, "reset"):
            eng.reset()  # a new clip group starts from empty queues
        hidden = np.zeros((B, 512), np.float32)
        sums = np.zeros((B, n_frames), np.float64)
        out = None
        staged = batch_source is not None and hasattr(eng, "stage")
        if staged and n_frames > 0:
            eng.stage(batch_source(group, 0)[0])
        for f in range(n_frames):
            if staged:
                if f + 1 < n_frames:
                    eng.stage(batch_source(group, f + 1)[0])
                pk = batch_source(group, f)[1]
                pk[:, 12:] = hidden
                out = np.asarray(eng.run_staged(pk)).reshape(B, -1)
                hidden = out[:, -512:].copy()
                sums[:, f] = out.astype(np.float64).sum(axis=1)
                continue
            if batch_source is not None:
                w, pk = batch_source(group, f)
            else:
                w = np.empty((B, 2, 6, 128, 256), np.uint8)
                pk = np.empty((B, 524), np.float32)
                for i, c in enumerate(group):
                    w[i], pk[i] = frame_source(c, f)
            pk[:, 12:] = hidden
            out = np.asarray(eng.run_frame(w, pk)).reshape(B, -1)
            hidden = out[:, -512:].copy()
            sums[:, f] = out.astype(np.float64).sum(axis=1)
        for i, c in enumerate(group):
            results[c] = (sums[i], out[i].copy())
    return results


def run_rank_pipelined(engine_factory, clips, n_frames, batch, batch_source, alloc):
    """run_rank for engines that carry the hidden state on the device and
    queue frames (stage / run_staged_async / wait_output): frame f+1 is
    uploaded and queued before the host reads frame f's output, so the host's
    per-frame work overlaps the GPU.  Same results as run_rank (the device
    carry equals the host carry bit for bit).  alloc(shape, dtype) returns an
    array in pinned host memory (outputs and packed vectors are copied
    asynchronously)."""
    results = {}
    engines = {}
    bufs = {}
    for group in batches(clips, batch):
        B = len(group)
        eng = engines.get(B)
        if eng is None:
            eng = engines[B] = engine_factory(B)
        elif hasattr(eng, "reset"):
            eng.reset()  # a new clip group starts from empty queues and a zero hidden state
        if B not in bufs:
            bufs[B] = ([alloc((B, FRAME_OUT), np.float32) for _ in range(2)],
                       [alloc((B, 524), np.float32) for _ in range(2)])
        outs, pks = bufs[B]
        sums = np.zeros((B, n_frames), np.float64)
        if n_frames == 0:
            continue
        eng.stage(batch_source(group, 0)[0])
        for f in range(n_frames):
            if f + 1 < n_frames:
                eng.stage(batch_source(group, f + 1)[0])
            pks[f % 2][:] = batch_source(group, f)[1]
            eng.run_staged_async(pks[f % 2], outs[f % 2])
            if f > 0:
                eng.wait_output()
                sums[:, f - 1] = outs[(f - 1) % 2].sum(axis=1, dtype=np.float64)
        eng.wait_output()
        last = outs[(n_frames - 1) % 2]
        sums[:, n_frames - 1] = last.sum(axis=1, dtype=np.float64)
        for i, c in enumerate(group):
            results[c] = (sums[i], last[i].copy())
    return results


class CommError(RuntimeError):
    pass


_COMM = None


def comm_lib():
    """libcncomm.so (ctypes); raises CommError if it is missing."""
    global _COMM
    if _COMM is None:
        path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libcncomm.so")
        if not os.path.exists(path):
            raise CommError(f"{path} is missing: build it with chestnut-on-pc_b200/build.py")
        L = ctypes.CDLL(path)
        vp, i, sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t
        sigs = {"cn_comm_last_error": ([], ctypes.c_char_p), "cn_comm_nccl_version": ([ctypes.POINTER(i)], i),
                "cn_comm_unique_id": ([vp], i), "cn_comm_init": ([ctypes.POINTER(vp), i, i, i, vp, i], i),
                "cn_comm_allgather_f64": ([vp, vp, vp, sz, i], i), "cn_comm_destroy": ([vp], i)}
        for name, (args, res) in sigs.items():
            f = getattr(L, name)
            f.argtypes, f.restype = args, res
        _COMM = L
    return _COMM


ID_BYTES = 128


def _check(rc, what):
    if rc != 0:
        raise CommError(f"{what} failed ({rc}): {comm_lib().cn_comm_last_error().decode(errors='replace')}")


class NcclGather:
    """Clip-end all-gather over NCCL, driven from C++ (one process per GPU).

    ``unique_id``: the CN_COMM_ID_BYTES rendezvous bytes made on rank 0 by
    ``NcclGather.new_id()`` and handed to every rank by the host's own
    launcher (a key-value store, a broadcast, a file).  A rank that does not
    arrive within ``timeout_s`` turns into a CommError instead of a hang.
    """

    def __init__(self, rank, world, device, unique_id, timeout_s=60.0):
        if len(unique_id) != ID_BYTES:
            raise CommError(f"unique id must be {ID_BYTES} bytes")
        self.world, self.rank = int(world), int(rank)
        self.timeout_ms = int(timeout_s * 1000)
        h = ctypes.c_void_p()
        buf = ctypes.create_string_buffer(bytes(unique_id), ID_BYTES)
        _check(comm_lib().cn_comm_init(ctypes.byref(h), int(device), self.world, self.rank, buf, self.timeout_ms),
               "cn_comm_init")
        self._h = h

    @staticmethod
    def new_id():
        buf = ctypes.create_string_buffer(ID_BYTES)
        _check(comm_lib().cn_comm_unique_id(buf), "cn_comm_unique_id")
        return buf.raw

    def allgather(self, arr):
        """f64 array on every rank -> f64 [world, *arr.shape], rank r's array in row r."""
        a = np.ascontiguousarray(arr, np.float64)
        out = np.empty((self.world,) + a.shape, np.float64)
        _check(comm_lib().cn_comm_allgather_f64(self._h, a.ctypes.data, out.ctypes.data, a.size, self.timeout_ms),
               "cn_comm_allgather_f64")
        return out

    def close(self):
        if getattr(self, "_h", None) is not None and self._h.value:
            comm_lib().cn_comm_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def gather(results, n_clips, n_frames, n_out, transport=None):
    """All-gather every rank's per-clip results (one collective, at clip end).

    Returns (checksums f64[n_clips, n_frames], finals f32[n_clips, n_out]) on
    every rank.  Clips a rank does not own are zero in its contribution, so the
    gather is a sum over ranks of disjoint rows (exact: every row has one
    non-zero contributor).  ``transport`` None means a single process.
    """
    local_s = np.zeros((n_clips, n_frames), np.float64)
    local_f = np.zeros((n_clips, n_out), np.float64)
    for c, (s, f) in results.items():
        local_s[c] = s
        local_f[c] = f
    packed = np.concatenate([local_s, local_f], axis=1)
    total = transport.allgather(packed).sum(0) if transport is not None else packed
    return total[:, :n_frames], total[:, n_frames:].astype(np.float32)
