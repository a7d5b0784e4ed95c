"""Kernel micro-benchmarks (device time with CUDA events, DRAM-cold: weights rotate through a
set larger than the 126 MB L2).  Usage:

    python -m vllm_sly_radiance_b200.benchmarks.kernels gemm [--m 1,8,64,4096]
    python -m vllm_sly_radiance_b200.benchmarks.kernels attn
    python -m vllm_sly_radiance_b200.benchmarks.kernels gdn

Prints one JSON line per case with time, achieved bandwidth / FLOP rate and the fraction of the
measured peaks in MEASURED_PEAKS.json (fallback 6.65 TB/s, 1.59 PFLOP/s).
Reference analogue: sly/mxfp4/bench_{decode,prefill}_cells.py (DRAM-cold weight rotation)."""
from __future__ import annotations

import argparse
import json
import os

import torch

from ..ops import kernels as K
from ..quant.mxfp4 import MXFP4Weight


def peaks():
    p = os.path.join(os.path.dirname(__file__), "..", "..", "MEASURED_PEAKS.json")
    try:
        d = json.load(open(p))
        return d["hbm_gbs"] * 1e9, d["bf16_tflops"] * 1e12, "measured"
    except Exception:
        return 6.65e12, 1.59e15, "fallback"


ITERS = 50


def timeit(fn, iters=None, warmup=5):
    iters = iters or ITERS
    for _ in range(warmup):
        fn(0)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for i in range(iters):
        fn(i)
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters * 1e-3


def bench_gemm(ms, shapes):
    bw, fl, src = peaks()
    for (N, Kd, name) in shapes:
        nrot = max(2, int(300e6 // (N * Kd // 2)) + 1)       # > 2x L2 of weights
        ws = [MXFP4Weight.from_float(torch.randn(N, Kd, device="cuda") * 0.02) for _ in range(nrot)]
        for M in ms:
            x = torch.randn(M, Kd, device="cuda").to(torch.bfloat16)
            q, s = K.quant_fp8(x)
            out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")

            def fn(i):
                w = ws[i % nrot]
                K.mxfp4_gemm(q, s, w.packed, w.sf, w.scales, N, out=out)
            t = timeit(fn)
            byts = N * Kd // 2 + N * Kd // 32 + M * Kd + M * N * 2
            flops = 2.0 * M * N * Kd
            print(json.dumps({"kernel": "mxfp4_gemm", "shape": name, "M": M, "N": N, "K": Kd,
                              "us": round(t * 1e6, 2), "GBps": round(byts / t / 1e9, 1),
                              "TFLOPs": round(flops / t / 1e12, 1),
                              "frac_hbm": round(byts / t / bw, 3),
                              "frac_bf16_peak": round(flops / t / fl, 3), "peaks": src}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("what", choices=["gemm"])
    ap.add_argument("--m", default="1,8,16,64,256,1024,4096")
    ap.add_argument("--shape", default="", help="comma list of shape names (default: all)")
    ap.add_argument("--iters", type=int, default=50)
    a = ap.parse_args()
    global ITERS
    ITERS = a.iters
    ms = [int(v) for v in a.m.split(",")]
    shapes = [(16480, 5120, "gdn_in_proj"), (5120, 6144, "out_proj"), (17408, 5120, "gate_up"),
              (5120, 8704, "down"), (14336, 5120, "attn_qkv"), (248320, 5120, "lm_head")]
    if a.shape:
        keep = set(a.shape.split(","))
        shapes = [sh for sh in shapes if sh[2] in keep]
    if a.what == "gemm":
        bench_gemm(ms, shapes)


if __name__ == "__main__":
    main()
