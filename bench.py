"""Benchmark: synthetic 1B big-driving frame on the B200 engine.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (clip-sharded per config 5): every rank drives
its own recurrent clip of the 1B synthetic model at batch 1, one CUDA-graph
replay per frame.  A step = one frame of every clip.  `value` = frames of all
ranks / max-over-ranks device time (inputs resident in HBM); `latency_ms`
holds the per-frame p50/p90/p99 (graph launch -> outputs ready on device);
`e2e` = the same frames through the public run_frame call with pinned host
buffers (H2D of warped+packed and D2H of the output inside the timed region).
No collective runs per frame; each rank's clip digest is all-gathered over
NCCL once at the end.

--impl reference times the reference-semantics CPU implementation of the same
frame (the numpy oracle restatement: the reference's own tinygrad CPU
backend is not importable here) on all host threads, rank 0 only.
"""
import argparse
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
MEASURED = os.path.join(ROOT, "MEASURED_PEAKS.json")


def peaks():
    try:
        with open(MEASURED) as f:
            p = json.load(f)
        return p["hbm_gbs"], p["bf16_tflops"], "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


class Clocks:
    """nvidia-smi sampler for the timed region."""

    def __init__(self, index):
        self.index = index
        self.p = None
        self.path = None

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        self.path = f"/tmp/cn_clocks_{os.getpid()}.csv"
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}",
                                       "--format=csv,noheader,nounits", "-lms", "200"],
                                      stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        if self.p:
            self.p.terminate()
            self.p.wait()

    def summary(self):
        try:
            rows = [r.split(",") for r in open(self.path).read().strip().splitlines()]
            sm = [float(r[1]) for r in rows]
            mx = float(rows[0][2])
            names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
            reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].strip() == "Active"})
            return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": reasons, "samples": len(sm)}
        except Exception as ex:  # pragma: no cover
            return {"error": str(ex)}


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
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "profiles", "trunk_%s_ncu.json" % model)
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


def run_ours(args, rank, world, local_rank):
    import torch
    from chestnut_b200 import Engine, DeviceBuffer

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

    # ---- value + latency: device-resident inputs, one graph replay per frame
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize(dev)
    eng.sync()
    with Clocks(dev) as clk:
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

    # ---- e2e through the public run_frame with pinned host buffers
    import ctypes
    from chestnut_b200._lib import lib
    hw = ctypes.c_void_p()
    hp = ctypes.c_void_p()
    ho = ctypes.c_void_p()
    lib().cn_host_alloc_pinned(ctypes.byref(hw), w[0].nbytes * nfr)
    lib().cn_host_alloc_pinned(ctypes.byref(hp), pk[0].nbytes * nfr)
    lib().cn_host_alloc_pinned(ctypes.byref(ho), B * 3323 * 4)
    ctypes.memmove(hw.value, w.ctypes.data, w.nbytes)
    ctypes.memmove(hp.value, pk.ctypes.data, pk.nbytes)
    out_np = np.frombuffer((ctypes.c_float * (B * 3323)).from_address(ho.value), np.float32)
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

    # ---- config 5: clip throughput of the 39M model, 8 clips per launch
    clip = clip_throughput(args, rank, world, dev, dist, barrier) if args.clips > 0 else None

    # ---- max over ranks, gather clip digests (the only collective)
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
    d = 2048 if args.model == "1b" else 512
    mlp = 4 * d
    rows = 88 * B
    layers = 20 if args.model == "1b" else 4
    if trunk:
        kname = "transformer_trunk (persistent: all layers, weight streaming)"
        kbytes = trunk_bytes(d, mlp, rows, layers)
    else:
        kname = "gemm_tc (fc2: MLP down-projection, weight streaming)"
        kbytes = mlp * d * 2 + rows * mlp * 2 + rows * d * 4 * 2 + d * 4
    k_avg = statistics.mean(kms) if kms else float("nan")
    info = eng_info
    achieved = kbytes / (k_avg * 1e-3) / 1e9
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
        "latency_ms": {"p50": lat[len(lat) // 2], "p90": lat[int(len(lat) * 0.9)], "p99": lat[min(len(lat) - 1, int(len(lat) * 0.99))],
                       "mean": statistics.mean(lat)},
        "e2e": {"value": frames / (max_e2e * 1e-3), "unit": "frames/s", "ms_per_frame": max_e2e / args.steps,
                "h2d_bytes_per_step": B * (2 * 6 * 128 * 256 + 524 * 4) * world,
                "d2h_bytes_per_step": B * 3323 * 4 * world},
        "gpu_launches": n_launch * args.steps,
        "launches_per_frame": n_launch,
        "roofline": {"kernel": kname, "bound": "hbm",
                     "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "peak_source": src, "algorithmic_bytes_per_launch": kbytes, "avg_launch_ms": k_avg,
                     "traffic": ncu_traffic(args.model) if trunk else None},
        "frame_roofline": {"bound": "hbm", "weight_bytes": info["weight_bytes"],
                           "floor_ms": info["weight_bytes"] / (hbm * 1e9) * 1e3,
                           "frac": (info["weight_bytes"] / (hbm * 1e9) * 1e3) / lat[len(lat) // 2]},
        "clocks": clk.summary(),
        "clip_digests": allv[:, 2].tolist(),
    }
    if clip:
        cms = float(allv[:, 3].max())
        line["clip_throughput"] = {
            "workload": f"config 5: {args.clips} synthetic 39M clips x {args.clip_frames} frames, {clip['batch']} clips "
                        f"per graph launch, round-robin over {world} GPU(s), per-clip results all-gathered once at "
                        "clip end", "value": args.clips * args.clip_frames / (cms * 1e-3), "unit": "frames/s",
            "ms": cms, "scaling": "strong", "path": "public run_frame with host buffers (H2D + D2H per frame)",
            "gathered_checksum": clip["checksum"]}
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(args.model, budget_s=args.cpu_budget)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return line


def clip_throughput(args, rank, world, dev, dist, barrier):
    """Config 5: this rank's share of the clips, 8 per launch, frames through run_frame."""
    import torch
    from chestnut_b200 import Engine, clips

    B = 8
    mine = clips.assign(args.clips, world, rank)
    eng = Engine("39m", device=dev, batch=B, seed=args.seed)
    stream = torch.cuda.ExternalStream(eng.stream_handle(), device=dev)
    # clip c, frame f reads pool frame (c + f) % 4 with clip-specific desire: a pure
    # function of (clip, frame), so the gathered results match for any GPU count
    rng = np.random.default_rng(77)
    pool = rng.integers(0, 256, (4, 2, 6, 128, 256), dtype=np.uint8)
    staged = {}
    for group in clips.batches(mine, B):
        for f4 in range(4):
            w = np.stack([pool[(c + f4) % 4] for c in group])
            pk = np.zeros((len(group), 524), np.float32)
            for i, c in enumerate(group):
                pk[i, c % 8] = 1.0
                pk[i, 8 + c % 2] = 1.0
            staged[(tuple(group), f4)] = (w, pk)

    def batch_source(group, f):
        w, pk = staged[(tuple(group), f % 4)]
        return w, pk.copy()

    def factory(n):
        return eng if n == B else Engine("39m", device=dev, batch=n, seed=args.seed)

    clips.run_rank(factory, None, clips.batches(mine, B)[0], 3, B, batch_source)  # warm-up
    eng.reset()
    barrier()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    res = clips.run_rank(factory, None, mine, args.clip_frames, B, batch_source)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1)
    sums, _ = clips.gather(res, args.clips, args.clip_frames, 3323, dist, device=f"cuda:{dev}")
    eng.close()
    return {"ms": ms, "batch": B, "checksum": float(np.abs(sums).sum())}


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
    ap.add_argument("--clips", type=int, default=64, help="config-5 clips (0 skips the clip-throughput leg)")
    ap.add_argument("--clip-frames", type=int, default=30, help="frames per clip in the clip-throughput leg")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        line = run_reference(args, rank)
    else:
        line = run_ours(args, rank, world, local_rank)
    if line is not None:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
