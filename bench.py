"""Benchmark: synthetic 1B big-driving frame on the B200 engine.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python bench.py --kernel gemm|reduce|frame39m|warp   (one kernel-level leg alone)

Workload (clip-sharded per config 5): every rank drives
its own recurrent clip of the 1B synthetic model at batch 1, one CUDA-graph
replay per frame.  A step = one frame of every clip.  `value` = frames of all
ranks / max-over-ranks device time (inputs resident in HBM); `latency_ms`
holds the per-frame p50/p90/p99 (graph launch -> outputs ready on device);
`e2e` = the same frames through the public run_frame call with pinned host
buffers (H2D of warped+packed and D2H of the output inside the timed region).
No collective runs per frame; each rank's clip digest is gathered once at the
end.

Further legs on the same line:
  latency_1200     config 4's own latency definition: p50/p90/p99 over 1,200
                   recurrent frames (hidden state carried on the device);
  clip_throughput  config 5: 64 39M clips x 1,200 frames, 8 clips per graph
                   launch, round-robin over the ranks, frames from pinned host
                   memory through the public run_frame, one gather at clip end;
  kernels          (1 GPU) configs 1 and 2 at kernel level (the B200
                   counterparts of the reference's bench_r62.py / bench_alu.py),
                   config 3 (39M single-frame p50) and the frame warp, each
                   with its roofline fraction and, for configs 1-3, a CPU
                   baseline timed on the host cores.

--impl reference times the reference-semantics CPU implementation of the same
frame (the numpy oracle restatement: the reference's own tinygrad CPU
backend is not importable here) on all host threads, rank 0 only.
"""
import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "chestnut-on-pc_b200"))
sys.path.insert(0, ROOT)

METRIC = "1B-model frame latency p50 ms (1×B200); clip frames/s at 1/2/4/8 GPUs"
PUBLISHED_MS = 84.0        # the reference's published 1B frame time on an RTX 2080 (README.md:19,39)
PUBLISHED_39M_MS = 8.6     # the reference's published 39M frame time on an RTX 2080 (README.md:18)
MEASURED = os.path.join(ROOT, "MEASURED_PEAKS.json")
N_OUT = 3323
FRAME = 2 * 6 * 128 * 256
MODEL_DIMS = {  # stem channels, d, mlp, layers (the synthetic configs 3 and 4)
    "39m": ((32, 64, 128, 256, 512), 512, 2048, 4),
    "1b": ((64, 128, 256, 512, 1024), 2048, 8192, 20),
}


def peaks():
    try:
        with open(MEASURED) as f:
            p = json.load(f)
        return p["hbm_gbs"], p["bf16_tflops"], "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


def pct(xs, q):
    xs = sorted(xs)
    return xs[min(len(xs) - 1, int(len(xs) * q))]


class Clocks:
    """nvidia-smi sampler (200 ms period) around the timed legs."""

    NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def __init__(self, index):
        self.index = index
        self.p = None
        self.path = f"/tmp/cn_clocks_{os.getpid()}.csv"

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}",
                                       "--format=csv,noheader,nounits", "-lms", "200"],
                                      stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        time.sleep(0.25)  # one more period, so a short region still gets a sample
        if self.p:
            self.p.terminate()
            self.p.wait()

    def summary(self):
        rows = []
        try:
            for line in open(self.path).read().strip().splitlines():
                r = [x.strip() for x in line.split(",")]
                if len(r) >= 9:
                    try:
                        rows.append((float(r[1]), float(r[2]), float(r[3]), r[5:9]))
                    except ValueError:
                        continue
        except OSError:
            pass
        if not rows:
            return {"error": "no nvidia-smi samples", "samples": 0}
        # samples under load: power above the midpoint of the region's range
        pw = [r[2] for r in rows]
        cut = (min(pw) + max(pw)) / 2
        load = [r for r in rows if r[2] >= cut] or rows
        reasons = sorted({self.NAMES[i] for r in rows for i in range(4) if r[3][i] == "Active"})
        return {"sm_mhz": statistics.median(r[0] for r in load), "sm_max_mhz": rows[0][1], "reasons": reasons,
                "samples": len(rows), "samples_under_load": len(load), "power_w_max": max(pw)}


def frame_inputs(rng, n, batch):
    w = rng.integers(0, 256, (n, batch, 2, 6, 128, 256), dtype=np.uint8)
    pk = np.zeros((n, batch, 524), np.float32)
    pk[:, :, 8] = 1.0
    for i in range(n):
        pk[i, :, rng.integers(0, 8)] = 1.0
    return w, pk


def ncu_traffic(model):
    """DRAM bytes (read + write) per trunk launch from the committed ncu capture
    (profiles/trunk_1b_ncu.json, made with the command in profiles/trunk_1b.md)."""
    path = os.path.join(ROOT, "profiles", "trunk_%s_ncu.json" % model)
    try:
        with open(path) as f:
            d = json.load(f)
        return d["dram_bytes_read"] + d["dram_bytes_write"]
    except (OSError, KeyError, ValueError):
        return None


def trunk_bytes(d, mlp, rows, layers):
    """Algorithmic HBM bytes of one trunk launch: every layer's f16 weights and
    f32 biases, read once.  The activations of a single clip (88 token rows,
    a few MB per layer) stay in the 126 MB L2 and are not counted."""
    del rows
    return layers * ((3 * d * d + d * d + 2 * d * mlp) * 2 + (3 * d + d + mlp + d) * 4)


def frame_flops(model):
    """Multiply-add FLOPs (x2) of one frame of the synthetic model: the two
    cameras' conv stems (3x3/s2 conv + 1x1 conv per stage, im2col K padded as
    the engine runs it), the token embeddings, the transformer over 88 tokens
    (projections + attention scores / values) and the head products."""
    stem, d, mlp, layers = MODEL_DIMS[model]
    macs = 0
    pos, cin = 64 * 128, None
    for s, c in enumerate(stem):
        k = 128 if s == 0 else 9 * cin
        macs += pos * k * c + pos * c * c
        cin = c
        if s + 1 < len(stem):
            pos //= 4
    macs *= 2                                    # two cameras
    macs += 64 * stem[-1] * d + 24 * 512 * d + 256 * d
    T = 88
    macs += layers * (T * (4 * d * d + 2 * d * mlp) + 2 * T * T * d)
    macs += d * 512 + 512 * 1024 + 1024 * 2811
    return 2 * macs


def stem_weight_bytes(model):
    """f16 weight bytes the persistent stem streams per frame: both cameras'
    conv stages (first conv K padded to 128), the cond embedding (K padded to
    256), the temporal and visual token embeddings."""
    stem, d, _, _ = MODEL_DIMS[model]
    n, cin = 0, None
    for s, c in enumerate(stem):
        k = 128 if s == 0 else 9 * cin
        n += 2 * (c * k + c * c)
        cin = c
    n += 2 * d * stem[-1] + 256 * d + 512 * d
    return 2 * n


# ------------------------------------------------------------ kernel-level legs
def bench_gemm(reps=50, bn=0, splits=0, b_kmajor=0):
    """Config 1: C f32[768x256] += A f16[768x6144] x B f16[6144x256] ([K][N], the
    BASELINE layout), A, B ~ N(0,1)/sqrt(6144).  Back-to-back launches captured in
    a CUDA graph (launch latency exceeds the kernel), operands L2-warm: the
    tensor roofline bounds it (2.416 GFLOP per call)."""
    import torch
    from chestnut_b200 import kernels
    M, N, K = 768, 256, 6144
    g = torch.Generator(device="cuda").manual_seed(0)
    A = (torch.randn(M, K, device="cuda", generator=g) / K ** 0.5).half()
    B = (torch.randn(K, N, device="cuda", generator=g) / K ** 0.5).half()
    if b_kmajor:
        B = B.t().contiguous()
    C = torch.zeros(M, N, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    for _ in range(3):
        kernels.gemm_wmma_f16(A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K, b_kmajor, bn, splits, st)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        s = torch.cuda.current_stream().cuda_stream
        for _ in range(reps):
            kernels.gemm_wmma_f16(A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K, b_kmajor, bn, splits, s)
    graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(4):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    assert kernels.device_error() == 0
    us = e0.elapsed_time(e1) * 1e3 / (4 * reps)
    flops = 2.0 * M * N * K
    hbm, tf, src = peaks()
    ach = flops / (us * 1e-6) / 1e12
    byts = M * K * 2 + K * N * 2 + M * N * 4 * 2
    return {"kernel": "gemm_tc (config 1, r_6_2 shape)", "shape": [M, N, K],
            "b_layout": "[N][K]" if b_kmajor else "[K][N]", "us_per_call": us, "tflops": ach,
            "l2": "operands L2-warm (13.4 MB), back-to-back graph replays",
            "roofline": {"bound": "tensor", "achieved": ach, "peak": tf, "unit": "TFLOP/s", "frac": ach / tf,
                         "peak_source": src},
            "hbm_view": {"algorithmic_bytes": byts, "frac_of_hbm": byts / (us * 1e-6) / 1e9 / hbm}}


def bench_reduce(reps=10, cpr=0, rows=32 * 32 * 3):
    """Config 2: out f32[3072] = x f16[3072x393216] . w f16[393216], U(-1,1).  The
    L2 is flushed between launches (x is 2.4 GB anyway): HBM roofline,
    2,416,717,824 algorithmic bytes per call.  `rows` < 3072 runs a smaller case
    of the same kernel (profiling)."""
    import torch
    from chestnut_b200 import kernels
    L = 12288 * 32
    g = torch.Generator(device="cuda").manual_seed(0)
    x = (torch.rand(rows * L, device="cuda", generator=g, dtype=torch.float16) * 2 - 1)
    w = (torch.rand(L, device="cuda", generator=g, dtype=torch.float16) * 2 - 1)
    out = torch.empty(rows, device="cuda")
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    for _ in range(3):
        kernels.reduce_rows_f16(x.data_ptr(), w.data_ptr(), out.data_ptr(), rows, L, cpr, st)
    torch.cuda.synchronize()
    ts = []
    for _ in range(reps):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        kernels.reduce_rows_f16(x.data_ptr(), w.data_ptr(), out.data_ptr(), rows, L, cpr, st)
        e1.record()
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1) * 1e3)
    assert kernels.device_error() == 0
    us = float(np.median(ts))
    byts = rows * L * 2 + L * 2 + rows * 4
    hbm, tf, src = peaks()
    ach = byts / (us * 1e-6) / 1e9
    del x, flush
    torch.cuda.empty_cache()
    return {"kernel": "row_dot (config 2, r_32_32_3_12288_32 shape)", "shape": [rows, L], "us_per_call": us,
            "l2": "flushed (256 MB write) before every call",
            "roofline": {"bound": "hbm", "achieved": ach, "peak": hbm, "unit": "GB/s", "frac": ach / hbm,
                         "peak_source": src, "algorithmic_bytes": byts}}


def bench_warp(reps=64, pairs=32):
    """Frame preparation (cn_warp_frames): road + wide NV12 frames of a 1928 x 1208
    camera (stride 2048) -> u8[2,6,128,256].  Back-to-back calls in a graph over
    `pairs` distinct frame pairs (7.5 MB each, more than the L2 in total), so the
    sampled source bytes come from HBM.  Algorithmic bytes per call: the output
    (393,216 B) plus one source byte per output byte."""
    import torch
    from chestnut_b200 import kernels
    width, height, stride, yh, uvh = 1928, 1208, 2048, 1216, 608
    fbytes = stride * (yh + uvh)
    g = torch.Generator(device="cuda").manual_seed(0)
    frames = torch.randint(0, 256, (pairs, 2, fbytes), device="cuda", generator=g, dtype=torch.uint8)
    out = torch.empty(FRAME, device="cuda", dtype=torch.uint8)
    c, s_ = np.cos(0.02), np.sin(0.02)
    ma = np.array([[3.6 * c, -3.6 * s_, 40.0], [3.6 * s_, 3.6 * c, 300.0], [2e-5, 0.0, 1.0]], np.float32)
    mb = np.array([[2.1, 0.05, 420.0], [-0.05, 2.1, 350.0], [-3e-5, 0.0, 1.0]], np.float32)

    def call(i, st):
        kernels.warp_frames(frames[i % pairs, 0].data_ptr(), frames[i % pairs, 1].data_ptr(), ma, mb, width, height,
                            stride, yh, uvh, out.data_ptr(), stream=st)
    st = torch.cuda.current_stream().cuda_stream
    for i in range(3):
        call(i, st)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        s = torch.cuda.current_stream().cuda_stream
        for i in range(reps):
            call(i, s)
    graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(4):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    assert kernels.device_error() == 0
    us = e0.elapsed_time(e1) * 1e3 / (4 * reps)
    byts = 2 * FRAME
    hbm, tf, src = peaks()
    ach = byts / (us * 1e-6) / 1e9
    return {"kernel": "warp_nv12 (frame preparation, 2 cameras)", "camera": [width, height, stride],
            "model": [512, 256], "us_per_call": us, "frame_pairs_per_s": 1e6 / us,
            "roofline": {"bound": "hbm", "achieved": ach, "peak": hbm, "unit": "GB/s", "frac": ach / hbm,
                         "peak_source": src, "algorithmic_bytes": byts}}


def bench_frame(model, dev=0, frames=300, warmup=10):
    """Single-clip frame latency (config 3 for the 39M model): device-resident
    inputs, one graph replay per frame, hidden state carried on the device,
    per-frame CUDA events on the engine's stream."""
    import torch
    from chestnut_b200 import DeviceBuffer, Engine
    eng = Engine(model, device=dev, batch=1, seed=0, carry_hidden=True)
    stream = torch.cuda.ExternalStream(eng.stream_handle(), device=dev)
    rng = np.random.default_rng(5)
    w, pk = frame_inputs(rng, 8, 1)
    dW = [DeviceBuffer(w[i].nbytes, dev).upload(w[i]) for i in range(8)]
    dP = [DeviceBuffer(pk[i].nbytes, dev).upload(pk[i]) for i in range(8)]
    for i in range(warmup):
        eng.run_frame_device(dW[i % 8].ptr, dP[i % 8].ptr)
    eng.sync()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(frames)]
    for i in range(frames):
        evs[i][0].record(stream)
        eng.run_frame_device(dW[i % 8].ptr, dP[i % 8].ptr)
        evs[i][1].record(stream)
    eng.sync()
    torch.cuda.synchronize(dev)
    lat = [a.elapsed_time(b) for a, b in evs]
    info = eng.info()
    eng.close()
    hbm, tf, src = peaks()
    fl = frame_flops(model)
    t_hbm = info["weight_bytes"] / (hbm * 1e9) * 1e3
    t_tc = fl / (tf * 1e12) * 1e3
    floor = max(t_hbm, t_tc)
    p50 = pct(lat, 0.5)
    return {"model": model, "frames": frames, "p50_ms": p50, "p90_ms": pct(lat, 0.9), "p99_ms": pct(lat, 0.99),
            "launches_per_frame": info["n_kernels"],
            "roofline": {"bound": "hbm" if t_hbm >= t_tc else "tensor", "floor_ms": floor,
                         "weight_bytes": info["weight_bytes"], "flops": fl, "frac": floor / p50, "peak_source": src}}


def bench_clip_step(B=64, dev=0, steps=50, warmup=5):
    """One config-5 frame step of B batched 39M clips: device-resident inputs,
    one graph replay per step (CUDA events on the engine's stream), then one
    eager frame with per-launch device times (serialised, so shares only)."""
    import torch
    from chestnut_b200 import DeviceBuffer, Engine
    eng = Engine("39m", device=dev, batch=B, seed=0, carry_hidden=True)
    stream = torch.cuda.ExternalStream(eng.stream_handle(), device=dev)
    rng = np.random.default_rng(5)
    w = rng.integers(0, 256, (B, 2, 6, 128, 256), dtype=np.uint8)
    pk = np.zeros((B, 524), np.float32)
    pk[:, 8] = 1.0
    dW, dP = DeviceBuffer(w.nbytes, dev).upload(w), DeviceBuffer(pk.nbytes, dev).upload(pk)
    for _ in range(warmup):
        eng.run_frame_device(dW.ptr, dP.ptr)
    eng.sync()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(steps):
        eng.run_frame_device(dW.ptr, dP.ptr)
    b.record(stream)
    eng.sync()
    torch.cuda.synchronize(dev)
    ms = a.elapsed_time(b) / steps
    prof = eng.profile_frame(w, pk)
    eng.close()
    tot = sum(t for _, t in prof)
    kinds = {}
    for name, t in prof:
        k = name.split(":")[0]
        kinds[k] = kinds.get(k, 0.0) + t
    return {"kernel": f"config-5 frame step, {B} batched 39M clips", "ms_per_step": ms, "frames_per_s": B / ms * 1e3,
            "launches": len(prof),
            "eager_launch_list": [{"name": n, "us": round(t * 1e3, 1), "share": round(t / tot, 4)} for n, t in prof],
            "by_kind_share": {k: round(v / tot, 4) for k, v in sorted(kinds.items(), key=lambda x: -x[1])}}


def cpu_kernel_baselines():
    """Configs 1 and 2 on the host cores through the C restatement (oracle/cref.c,
    OpenMP, every thread), and config 3 through the numpy oracle frame."""
    from oracle import build as ob
    thr = ob.nthreads()
    out = {}
    rs = np.random.default_rng(0)
    A = (rs.standard_normal((768, 6144)) / 6144 ** 0.5).astype(np.float16)
    B = (rs.standard_normal((6144, 256)) / 6144 ** 0.5).astype(np.float16)
    C = np.zeros((768, 256), np.float32)
    t = time.perf_counter()
    ob.gemm_chain(A, B, C, 0, thr)
    s = time.perf_counter() - t
    out["config1_gemm"] = {"us_per_call": s * 1e6, "cores": thr, "kind": "port",
                           "sample": "one full 768x256x6144 call, per-output f32 fma chain over K (the FFMA "
                                     "consumer's order), C restatement, OpenMP"}
    rows, L = 384, 12288 * 32
    x = (rs.random((rows, L), np.float32) * 2 - 1).astype(np.float16)
    w = (rs.random(L, np.float32) * 2 - 1).astype(np.float16)
    ob.reduce_rows(x[:8], w, thr)
    t = time.perf_counter()
    ob.reduce_rows(x, w, thr)
    s = time.perf_counter() - t
    out["config2_reduce"] = {"us_per_call": s * 1e6 * 3072 / rows, "cores": thr, "kind": "port",
                             "sample": f"{rows} of the 3072 rows (x {rows * L * 2 / 1e6:.0f} MB), scaled to the "
                                       "full call; C restatement, f32 accumulate in index order, OpenMP"}
    from oracle import model as om
    clip = om.Clip("39m", 0)
    w8, pk = frame_inputs(np.random.default_rng(7), 1, 1)
    clip.run_frame(w8[0, 0], pk[0, 0])
    ts = []
    start = time.perf_counter()
    while time.perf_counter() - start < 6.0 and len(ts) < 40:
        t = time.perf_counter()
        o = clip.run_frame(w8[0, 0], pk[0, 0])
        ts.append(time.perf_counter() - t)
        pk[0, 0, 12:] = o[2811:]
    out["config3_frame_39m"] = {"ms_per_frame_p50": 1e3 * statistics.median(ts), "cores": os.cpu_count(),
                                "kind": "port", "sample": f"{len(ts)} recurrent frames of the synthetic 39M model, "
                                                          "numpy/BLAS oracle"}
    return out


def kernel_legs(dev, cpu=True):
    k = {"config1_gemm": bench_gemm(), "config2_reduce": bench_reduce(), "config3_frame_39m": bench_frame("39m", dev),
         "frame_warp": bench_warp()}
    k["config3_frame_39m"]["vs_published_2080_ms"] = PUBLISHED_39M_MS
    if cpu:
        for name, cb in cpu_kernel_baselines().items():
            k[name]["cpu_baseline"] = cb
    return k


# ------------------------------------------------------------------ main legs
def run_ours(args, rank, world, local_rank):
    import torch
    from chestnut_b200 import Engine, DeviceBuffer
    from chestnut_b200._lib import lib

    dev = local_rank
    torch.cuda.set_device(dev)
    dist = None
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", dev))

    def barrier():
        if dist:
            dist.barrier()

    B = args.batch
    eng = Engine(args.model, device=dev, batch=B, seed=args.seed, carry_hidden=True)
    stream = torch.cuda.ExternalStream(eng.stream_handle(), device=dev)
    n_launch = eng.info()["n_kernels"]
    eng_info = eng.info()
    rng = np.random.default_rng(1000 + rank)
    nfr = 8
    w, pk = frame_inputs(rng, nfr, B)
    # device-resident inputs for the `value` leg
    dW = [DeviceBuffer(w[i].nbytes, dev).upload(w[i]) for i in range(nfr)]
    dP = [DeviceBuffer(pk[i].nbytes, dev).upload(pk[i]) for i in range(nfr)]
    for i in range(args.warmup):
        eng.run_frame_device(dW[i % nfr].ptr, dP[i % nfr].ptr)
    eng.sync()

    clk = Clocks(dev)
    clk.__enter__()
    # ---- value + latency: device-resident inputs, one graph replay per frame
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize(dev)
    eng.sync()
    t0.record(stream)
    for i in range(args.steps):
        evs[i][0].record(stream)
        eng.run_frame_device(dW[i % nfr].ptr, dP[i % nfr].ptr)
        evs[i][1].record(stream)
    t1.record(stream)
    eng.sync()
    torch.cuda.synchronize(dev)
    barrier()
    total_ms = t0.elapsed_time(t1)
    lat = sorted(a.elapsed_time(b) for a, b in evs)

    # ---- config 4's latency definition: 1,200 recurrent frames
    n12 = args.latency_frames
    ev12 = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n12)]
    for i in range(n12):
        ev12[i][0].record(stream)
        eng.run_frame_device(dW[i % nfr].ptr, dP[i % nfr].ptr)
        ev12[i][1].record(stream)
    eng.sync()
    torch.cuda.synchronize(dev)
    lat12 = sorted(a.elapsed_time(b) for a, b in ev12)

    # ---- dominant kernel timed inside the graph: the persistent transformer
    # trunk (single-clip frames) or, with per-layer kernels, the fc2 GEMMs
    trunk = any(k["name"] == "transformer_trunk" for k in eng.kernel_list())
    eng.set_timed_class("transformer_trunk" if trunk else ".fc2")
    kms = []
    for i in range(args.steps):
        eng.run_frame_device(dW[i % nfr].ptr, dP[i % nfr].ptr)
        eng.sync()
        kms += eng.timed_class_ms()
    eng.set_timed_class("")
    # the persistent conv stem, timed the same way
    stem_ms = None
    if any(k["name"] == "conv_stem" for k in eng.kernel_list()):
        eng.set_timed_class("conv_stem")
        sms = []
        for i in range(args.steps):
            eng.run_frame_device(dW[i % nfr].ptr, dP[i % nfr].ptr)
            eng.sync()
            sms += eng.timed_class_ms()
        eng.set_timed_class("")
        stem_ms = statistics.median(sms) if sms else None

    # ---- e2e through the public run_frame with pinned host buffers
    hw = ctypes.c_void_p()
    hp = ctypes.c_void_p()
    ho = ctypes.c_void_p()
    lib().cn_host_alloc_pinned(ctypes.byref(hw), w[0].nbytes * nfr)
    lib().cn_host_alloc_pinned(ctypes.byref(hp), pk[0].nbytes * nfr)
    lib().cn_host_alloc_pinned(ctypes.byref(ho), B * N_OUT * 4)
    ctypes.memmove(hw.value, w.ctypes.data, w.nbytes)
    ctypes.memmove(hp.value, pk.ctypes.data, pk.nbytes)
    out_np = np.frombuffer((ctypes.c_float * (B * N_OUT)).from_address(ho.value), np.float32)
    barrier()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        j = i % nfr
        lib().cn_run_frame(eng._h, hw.value + j * w[0].nbytes, hp.value + j * pk[0].nbytes, ho.value)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    e2e_ms = e0.elapsed_time(e1)
    digest = float(np.abs(out_np).sum())

    eng.close()

    # ---- config 5: clip throughput of the 39M model, a rank's clips batched per launch
    clip = clip_throughput(args, rank, world, dev, dist, barrier) if args.clips > 0 else None
    clk.__exit__()

    # ---- kernel-level legs (configs 1-3), one GPU only
    kern = kernel_legs(dev, cpu=not args.no_cpu_baseline) if world == 1 and not args.no_kernels else None

    # ---- max over ranks, gather clip digests (bench bookkeeping, not the product path)
    vals = torch.tensor([total_ms, e2e_ms, digest, clip["ms"] if clip else 0.0], dtype=torch.float64,
                        device=f"cuda:{dev}")
    if dist:
        allv = [torch.zeros_like(vals) for _ in range(world)]
        dist.all_gather(allv, vals)
        allv = torch.stack(allv).cpu().numpy()
    else:
        allv = vals.cpu().numpy()[None]
    for p in (hw, hp, ho):
        lib().cn_host_free_pinned(p)
    if rank != 0:
        if dist:
            dist.barrier()
            dist.destroy_process_group()
        return None
    max_ms = float(allv[:, 0].max())
    max_e2e = float(allv[:, 1].max())
    frames = args.steps * B * world
    hbm, tf, src = peaks()
    stem, d, mlp, layers = MODEL_DIMS[args.model]
    rows = 88 * B
    if trunk:
        kname = "transformer_trunk (persistent: all layers, weight streaming)"
        kbytes = trunk_bytes(d, mlp, rows, layers)
    else:
        kname = "gemm_tc (fc2: MLP down-projection, weight streaming)"
        kbytes = mlp * d * 2 + rows * mlp * 2 + rows * d * 4 * 2 + d * 4
    k_avg = statistics.mean(kms) if kms else float("nan")
    info = eng_info
    achieved = kbytes / (k_avg * 1e-3) / 1e9
    floor_ms = info["weight_bytes"] / (hbm * 1e9) * 1e3
    line = {
        "metric": METRIC,
        "value": frames / (max_ms * 1e-3),
        "unit": "frames/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": max_ms / args.steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": (frames / (max_ms * 1e-3)) / (1000.0 / PUBLISHED_MS),
        "dtype": "f16",
        "data": "synthetic (seeded u8 frames, one-hot desire/traffic convention, hash-RNG He-init weights)",
        "config": {"workload": f"config 4: synthetic {args.model} big-driving frame, batch {B} per clip, one clip per GPU"
                               " (clip sharding per config 5), 1 CUDA graph per frame",
                   "model": args.model, "batch_per_gpu": B, "tokens": 88, "params": info["n_params"],
                   "weight_bytes": info["weight_bytes"], "parallelism": f"clip-sharded x{world}, no per-frame collective",
                   "l2": "weights (%.2f GB) streamed every frame exceed the 126 MB L2" % (info["weight_bytes"] / 1e9)},
        "latency_ms": {"p50": lat[len(lat) // 2], "p90": pct(lat, 0.9), "p99": pct(lat, 0.99),
                       "mean": statistics.mean(lat)},
        "latency_1200": {"frames": n12, "p50_ms": pct(lat12, 0.5), "p90_ms": pct(lat12, 0.9),
                         "p99_ms": pct(lat12, 0.99), "max_ms": lat12[-1],
                         "note": "recurrent frames, hidden state carried on the device, one graph replay each"},
        "e2e": {"value": frames / (max_e2e * 1e-3), "unit": "frames/s", "ms_per_frame": max_e2e / args.steps,
                "h2d_bytes_per_step": B * (FRAME + 524 * 4) * world,
                "d2h_bytes_per_step": B * N_OUT * 4 * world},
        "gpu_launches": n_launch * args.steps,
        "launches_per_frame": n_launch,
        "roofline": {"kernel": kname, "bound": "hbm",
                     "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "peak_source": src, "algorithmic_bytes_per_launch": kbytes, "avg_launch_ms": k_avg,
                     "traffic": ncu_traffic(args.model) if trunk else None},
        "frame_roofline": {"bound": "hbm", "weight_bytes": info["weight_bytes"], "floor_ms": floor_ms,
                           "frac": floor_ms / lat[len(lat) // 2]},
        "stem": ({"kernel": "conv_stem (persistent: 5 conv stages, cond and token embeddings)",
                  "ms_per_launch_median": stem_ms, "weight_bytes": stem_weight_bytes(args.model),
                  "note": "a dependency chain of 10 GEMM phases, latency-bound (profiles/stem_1b.md)"}
                 if stem_ms is not None else None),
        "clocks": clk.summary(),
        "clip_digests": allv[:, 2].tolist(),
    }
    if clip:
        cms = float(allv[:, 3].max())
        fps = args.clips * args.clip_frames / (cms * 1e-3)
        fl = frame_flops("39m")
        w39 = clip["weight_bytes"]
        per_launch_ms = max(w39 / (hbm * 1e9), clip["batch"] * fl / (tf * 1e12)) * 1e3
        roof_fps = world * clip["batch"] / (per_launch_ms * 1e-3)
        line["clip_throughput"] = {
            "workload": f"config 5: {args.clips} synthetic 39M clips x {args.clip_frames} frames, {clip['batch']} clips "
                        f"per graph launch, round-robin over {world} GPU(s), per-clip results gathered once at "
                        "clip end", "value": fps, "unit": "frames/s", "ms": cms, "scaling": "strong",
            "path": "public C ABI (cn_stage_input / cn_run_staged_async / cn_wait_output: frame f+1 uploaded and "
                    "queued while the host reads frame f), frames and outputs in pinned host memory, H2D + D2H "
                    "every frame, hidden state carried on the device",
            "gather": clip["gather"],
            "roofline": {"bound": "tensor", "per_launch_floor_ms": per_launch_ms, "frames_per_s_floor": roof_fps,
                         "frac": fps / roof_fps, "flops_per_frame": fl, "weight_bytes": w39, "peak_source": src},
            "gathered_checksum": clip["checksum"]}
    if kern:
        line["kernels"] = kern
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(args.model, budget_s=args.cpu_budget)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return line


def clip_throughput(args, rank, world, dev, dist, barrier):
    """Config 5: this rank's share of the clips, `--clip-batch` per launch
    (default: all of the rank's clips, at most 64), frames through run_frame."""
    import torch
    from chestnut_b200 import Engine, PinnedArray, clips
    from chestnut_b200._lib import lib

    mine = clips.assign(args.clips, world, rank)
    B = args.clip_batch if args.clip_batch > 0 else max(1, min(64, len(mine)))
    # the hidden state is carried on the device (bit for bit the host carry), so
    # the runner queues frame f+1 before it reads frame f's output
    eng = Engine("39m", device=dev, batch=B, seed=args.seed, carry_hidden=True)
    stream = torch.cuda.ExternalStream(eng.stream_handle(), device=dev)
    # clip c, frame f reads pool frame (c + f) % 4 with clip-specific desire: a pure
    # function of (clip, frame), so the gathered results agree for any GPU count
    # (bit for bit at equal clips per launch; the batched GEMMs tile by M, so
    # other batch sizes differ in the f32 summation order only).  The batches
    # are staged once in pinned host memory, as a camera pipeline hands the
    # engine its frames.
    rng = np.random.default_rng(77)
    pool = rng.integers(0, 256, (4, 2, 6, 128, 256), dtype=np.uint8)
    groups = clips.batches(mine, B)
    nb = len(groups) * 4
    pin = ctypes.c_void_p()
    lib().cn_host_alloc_pinned(ctypes.byref(pin), max(1, nb * B * FRAME))
    staged = {}
    for gi, group in enumerate(groups):
        for f4 in range(4):
            k = gi * 4 + f4
            w = np.frombuffer((ctypes.c_uint8 * (len(group) * FRAME)).from_address(pin.value + k * B * FRAME),
                              np.uint8).reshape(len(group), 2, 6, 128, 256)
            w[:] = np.stack([pool[(c + f4) % 4] for c in group])
            pk = np.zeros((len(group), 524), np.float32)
            for i, c in enumerate(group):
                pk[i, c % 8] = 1.0
                pk[i, 8 + c % 2] = 1.0
            staged[(tuple(group), f4)] = (w, pk)

    def batch_source(group, f):
        w, pk = staged[(tuple(group), f % 4)]
        return w, pk.copy()

    def factory(n):
        return eng if n == B else Engine("39m", device=dev, batch=n, seed=args.seed, carry_hidden=True)

    pinned = []

    def alloc(shape, dtype):
        pinned.append(PinnedArray(shape, dtype))
        return pinned[-1].array

    clips.run_rank_pipelined(factory, groups[0], 3, B, batch_source, alloc)  # warm-up
    eng.reset()
    barrier()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    res = clips.run_rank_pipelined(factory, mine, args.clip_frames, B, batch_source, alloc)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1)
    weight_bytes = eng.info()["weight_bytes"]
    eng.close()
    lib().cn_host_free_pinned(pin)
    for p in pinned:
        p.free()
    # the clip-end gather: NCCL driven from C++ (libcncomm.so); the bench's own
    # process group only hands the rendezvous id to every rank
    transport = None
    if dist:
        uid = [clips.NcclGather.new_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        transport = clips.NcclGather(rank, world, dev, uid[0], timeout_s=60.0)
    t = time.perf_counter()
    sums, _ = clips.gather(res, args.clips, args.clip_frames, N_OUT, transport)
    gms = (time.perf_counter() - t) * 1e3
    if transport:
        transport.close()
    return {"ms": ms, "batch": B, "checksum": float(np.abs(sums).sum()), "weight_bytes": weight_bytes,
            "gather": {"ms": gms, "bytes_per_rank": args.clips * (args.clip_frames + N_OUT) * 8,
                       "transport": "ncclAllGather from C++ (libcncomm.so)" if transport else "single process"}}


def cpu_baseline(model, budget_s=25.0, max_frames=None, warmup=0):
    """Time the oracle frame (reference semantics, numpy/BLAS) on the host cores,
    after `warmup` untimed frames."""
    from oracle import model as om
    t = time.perf_counter()
    clip = om.Clip(model, 0)
    setup = time.perf_counter() - t
    rng = np.random.default_rng(7)
    w, pk = frame_inputs(rng, 1, 1)
    for _ in range(warmup):
        out = clip.run_frame(w[0, 0], pk[0, 0])
        pk[0, 0, 12:] = out[2811:]
    ts = []
    start = time.perf_counter()
    while True:
        t = time.perf_counter()
        out = clip.run_frame(w[0, 0], pk[0, 0])
        ts.append(time.perf_counter() - t)
        pk[0, 0, 12:] = out[2811:]
        if time.perf_counter() - start > budget_s or (max_frames and len(ts) >= max_frames) or len(ts) >= 50:
            break
    cores = os.cpu_count()
    return {"value": 1.0 / statistics.median(ts), "unit": "frames/s", "ms_per_frame_p50": 1e3 * statistics.median(ts),
            "cores": cores, "kind": "port",
            "sample": f"{len(ts)} recurrent frames of the synthetic {model} model, batch 1, numpy/BLAS on {cores} "
                      f"threads (weights generated untimed in {setup:.1f}s); restatement, not tinygrad"}


def run_reference(args, rank):
    if rank != 0:
        return None
    warm = min(args.warmup, 3)  # an oracle frame of the 1B model takes seconds
    cb = cpu_baseline(args.model, budget_s=args.cpu_budget, max_frames=max(2, args.steps), warmup=warm)
    return {"metric": METRIC, "impl": "reference", "value": cb["value"], "unit": "frames/s", "n_gpus": args.gpus,
            "steps": int(cb["sample"].split()[0]), "warmup": warm, "ms_per_step": cb["ms_per_frame_p50"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": cb["value"] / (1000.0 / PUBLISHED_MS),
            "dtype": "f32 (f16-rounded activations)", "data": "synthetic",
            "config": {"workload": f"config 4: synthetic {args.model} frame, batch 1, CPU oracle", "model": args.model},
            "cpu_baseline": cb,
            "e2e": {"value": cb["value"], "unit": "frames/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--model", default="1b", choices=["1b", "39m"])
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--cpu-budget", type=float, default=25.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-kernels", action="store_true", help="skip the kernel-level legs (configs 1-3)")
    ap.add_argument("--latency-frames", type=int, default=1200, help="recurrent frames of the latency_1200 leg")
    ap.add_argument("--clips", type=int, default=64, help="config-5 clips (0 skips the clip-throughput leg)")
    ap.add_argument("--clip-frames", type=int, default=1200, help="frames per clip in the clip-throughput leg")
    ap.add_argument("--clip-batch", type=int, default=0,
                    help="clips per launch in the clip-throughput leg (0: all of a rank's clips, at most 64)")
    ap.add_argument("--kernel", choices=["gemm", "reduce", "frame39m", "warp", "clips39m"],
                    help="run one kernel-level leg alone and print its JSON")
    ap.add_argument("--bn", type=int, default=0)
    ap.add_argument("--splits", type=int, default=0)
    ap.add_argument("--reps", type=int, default=0)
    ap.add_argument("--reduce-rows", type=int, default=3072, help="rows of the --kernel reduce case")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.kernel:
        import torch
        torch.cuda.set_device(local_rank)
        if args.kernel == "gemm":
            line = bench_gemm(args.reps or 50, args.bn, args.splits)
        elif args.kernel == "reduce":
            line = bench_reduce(args.reps or 10, rows=args.reduce_rows)
        elif args.kernel == "warp":
            line = bench_warp(args.reps or 64)
        elif args.kernel == "clips39m":
            line = bench_clip_step(args.clip_batch or 64, local_rank)
        else:
            line = bench_frame("39m", local_rank)
    elif args.impl == "reference":
        line = run_reference(args, rank)
    else:
        line = run_ours(args, rank, world, local_rank)
    if line is not None:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
