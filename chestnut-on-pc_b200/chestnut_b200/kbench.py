"""Kernel-level benchmarks for BASELINE configs 1 and 2.

    python -m chestnut_b200.kbench gemm   [--bn B --splits S --reps N]
    python -m chestnut_b200.kbench reduce [--cpr C --reps N]
    python -m chestnut_b200.kbench warp   [--reps N]

The B200 counterpart of the reference's single-kernel A/B benches
(``bench_r62.py`` for r_6_2_32_4_2_2_2_4_4_384, ``bench_alu.py`` for
r_32_32_3_12288_32): seeded inputs of the BASELINE shapes, the kernel launched
through the C ABI on the caller's stream, CUDA-event timing on that stream,
and a one-line JSON report with the roofline fraction.

* gemm: C f32[768x256] += A f16[768x6144] x B f16[6144x256] (B as [K][N], the
  BASELINE layout), A, B ~ N(0,1)/sqrt(6144).  Back-to-back launches captured
  in a CUDA graph (launch latency exceeds the kernel), operands L2-warm: the
  tensor roofline is the one that bounds it (2.416 GFLOP per call).
* reduce: out f32[3072] = x f16[3072x393216] . w f16[393216], U(-1,1).  The L2
  is flushed between launches (x is 2.4 GB anyway): HBM roofline, 2,416,717,824
  algorithmic bytes per call.
torch is used here only for device buffers, the flush and events.
"""
import argparse
import json
import os

import numpy as np


def _peaks():
    here = os.path.dirname(os.path.abspath(__file__))
    for path in (os.path.join(here, "..", "..", "MEASURED_PEAKS.json"),):
        try:
            with open(path) as f:
                p = json.load(f)
            return p["hbm_gbs"], p["bf16_tflops"], "measured"
        except Exception:
            pass
    return 6650.0, 1590.0, "fallback"


def bench_gemm(bn=0, splits=0, reps=50, b_kmajor=0):
    import torch
    from . import kernels
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
    hbm, tf, src = _peaks()
    ach = flops / (us * 1e-6) / 1e12
    return {"kernel": "gemm_tc (config 1)", "shape": [M, N, K], "b_layout": "[N][K]" if b_kmajor else "[K][N]",
            "bn": bn, "splits": splits, "us_per_call": us, "tflops": ach,
            "roofline": {"bound": "tensor", "achieved": ach, "peak": tf, "unit": "TFLOP/s", "frac": ach / tf,
                         "peak_source": src},
            "hbm_view": {"algorithmic_bytes": M * K * 2 + K * N * 2 + M * N * 4 * 2,
                         "frac_of_hbm": (M * K * 2 + K * N * 2 + M * N * 8) / (us * 1e-6) / 1e9 / hbm}}


def bench_reduce(cpr=0, reps=10):
    import torch
    from . import kernels
    rows, L = 32 * 32 * 3, 12288 * 32
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
    hbm, tf, src = _peaks()
    ach = byts / (us * 1e-6) / 1e9
    return {"kernel": "row_dot (config 2)", "shape": [rows, L], "chunks_per_row": cpr, "us_per_call": us,
            "roofline": {"bound": "hbm", "achieved": ach, "peak": hbm, "unit": "GB/s", "frac": ach / hbm,
                         "peak_source": src, "algorithmic_bytes": byts}}


def bench_warp(reps=64, pairs=32):
    """Frame preparation (cn_warp_frames): road + wide NV12 frames of a 1928 x 1208
    camera (stride 2048) -> u8[2,6,128,256].  Back-to-back calls in a graph over
    `pairs` distinct frame pairs (7.5 MB each, more than the L2 in total), so the
    sampled source bytes come from HBM.  Algorithmic bytes per call: the output
    (393,216 B) plus one source byte per output byte."""
    import torch
    from . import kernels
    width, height, stride, yh, uvh = 1928, 1208, 2048, 1216, 608
    fbytes = stride * (yh + uvh)
    g = torch.Generator(device="cuda").manual_seed(0)
    frames = torch.randint(0, 256, (pairs, 2, fbytes), device="cuda", generator=g, dtype=torch.uint8)
    out = torch.empty(2 * 6 * 128 * 256, device="cuda", dtype=torch.uint8)
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
    byts = 2 * 2 * 6 * 128 * 256
    hbm, tf, src = _peaks()
    ach = byts / (us * 1e-6) / 1e9
    return {"kernel": "warp_nv12 (frame preparation, 2 cameras)", "camera": [width, height, stride], "model": [512, 256],
            "us_per_call": us, "frame_pairs_per_s": 1e6 / us,
            "roofline": {"bound": "hbm", "achieved": ach, "peak": hbm, "unit": "GB/s", "frac": ach / hbm,
                         "peak_source": src, "algorithmic_bytes": byts}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("which", choices=["gemm", "reduce", "warp"])
    ap.add_argument("--bn", type=int, default=0)
    ap.add_argument("--splits", type=int, default=0)
    ap.add_argument("--cpr", type=int, default=0)
    ap.add_argument("--reps", type=int, default=0)
    ap.add_argument("--b-kmajor", type=int, default=0)
    a = ap.parse_args()
    if a.which == "gemm":
        r = bench_gemm(a.bn, a.splits, a.reps or 50, a.b_kmajor)
    elif a.which == "warp":
        r = bench_warp(a.reps or 64)
    else:
        r = bench_reduce(a.cpr, a.reps or 10)
    print(json.dumps(r))


if __name__ == "__main__":
    main()
