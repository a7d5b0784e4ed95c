"""Kernel micro-benchmarks (device time with CUDA events, DRAM-cold: weights rotate through a
set larger than the 126 MB L2).  Usage:

    python -m vllm_sly_radiance_b200.benchmarks.kernels gemm [--m 1,8,64,4096]
    python -m vllm_sly_radiance_b200.benchmarks.kernels attn [--ctx 1500,4096 --splits 1,17]
    python -m vllm_sly_radiance_b200.benchmarks.kernels w4a16 [--m 1,8 --shape lm_head,62080x5120]
    python -m vllm_sly_radiance_b200.benchmarks.kernels gdn_prefill [--ctx 1500,4096]

Prints one JSON line per case with time, achieved bandwidth / FLOP rate and the fraction of the
measured peaks in MEASURED_PEAKS.json (fallback 6.65 TB/s, 1.59 PFLOP/s).  The W4A8 GEMMs run
tcgen05.mma.kind::mxf8f6f4 (e2m1 x e4m3 with UE8M0 block scales), which issues at the fp8 tensor
rate -- twice the bf16 rate -- so their compute fraction divides by 2x the measured bf16 GEMM.
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
    """Seconds per call on the device.  The calls are captured into one CUDA graph and replayed,
    so host launch overhead (which exceeds a short kernel's duration) is not measured; falls
    back to an eager loop if capture fails."""
    iters = iters or ITERS
    for i in range(warmup):
        fn(i)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    try:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for i in range(iters):
                fn(i)
        g.replay()
        torch.cuda.synchronize()
        s.record()
        g.replay()
        e.record()
        torch.cuda.synchronize()
        return s.elapsed_time(e) / iters * 1e-3
    except Exception:
        torch.cuda.synchronize()
    s.record()
    for i in range(iters):
        fn(i)
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters * 1e-3


def bench_gemm(ms, shapes):
    bw, fl, src = peaks()
    fp8_peak = 2 * fl          # kind::mxf8f6f4 issues at the fp8 rate
    for (N, Kd, name) in shapes:
        nrot = max(2, int(300e6 // (N * Kd // 2)) + 1)       # > 2x L2 of weights
        ws = [MXFP4Weight.from_float(torch.randn(N, Kd, device="cuda") * 0.02) for _ in range(nrot)]
        for M in ms:
            x = torch.randn(M, Kd, device="cuda").to(torch.bfloat16)
            q, s = K.quant_fp8(x)
            out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
            variants = [("mxfp4_gemm", lambda w: K.mxfp4_gemm(q, s, w.packed, w.sf, w.scales, N,
                                                               out=out))]
            if M <= K.GEMV_MAX_ROWS:
                variants.append(("mxfp4_gemv", lambda w: K.mxfp4_gemv(q, s, w, out)))
            for kname, call in variants:
                def fn(i, call=call):
                    call(ws[i % nrot])
                t = timeit(fn)
                byts = N * Kd // 2 + N * Kd // 32 + M * Kd + M * N * 2
                flops = 2.0 * M * N * Kd
                print(json.dumps({"kernel": kname, "shape": name, "M": M, "N": N, "K": Kd,
                                  "us": round(t * 1e6, 2), "GBps": round(byts / t / 1e9, 1),
                                  "TFLOPs": round(flops / t / 1e12, 1),
                                  "frac_hbm": round(byts / t / bw, 3),
                                  "frac_fp8_tensor_peak": round(flops / t / fp8_peak, 3),
                                  "peaks": src + " (fp8 tensor = 2x measured bf16)"}), flush=True)


class _AttnMeta:
    pass


def _attn_meta(ctx_lens, bs, Hq, Hkv, splits, dev):
    """Decode batch: one query token per sequence, contiguous random page tables."""
    B = len(ctx_lens)
    m = _AttnMeta()
    seq = [c + 1 for c in ctx_lens]
    nb = max((s + bs - 1) // bs for s in seq)
    perm = torch.randperm(B * nb, device="cpu").to(torch.int32)
    m.block_tables = perm.view(B, nb).to(dev)
    m.seq_lens = torch.tensor(seq, dtype=torch.int32, device=dev)
    m.query_start_loc = torch.arange(B + 1, dtype=torch.int32, device=dev)
    m.tile_seq = torch.arange(B, dtype=torch.int32, device=dev)
    m.tile_row0 = torch.zeros(B, dtype=torch.int32, device=dev)
    m.num_tokens = m.num_seqs = B
    m.num_splits = splits
    m.scratch_o = lambda s_, T, H, D: torch.empty(s_, T, H, D, device=dev)
    m.scratch_ml = lambda s_, T, H: torch.empty(s_, T, H, 2, device=dev)
    return m, B * nb


def _kv4_random(nblocks, Hkv, bs, D):
    """A random int4 (KV4) cache: 4-bit codes, then an fp16 (scale, zero) pair per 16 elements."""
    t = torch.randint(0, 256, (nblocks, Hkv, bs, D // 2 + D // 4), dtype=torch.uint8, device="cuda")
    sz = torch.tensor([0.05, -0.4], dtype=torch.float16, device="cuda").view(torch.uint8)
    t[..., D // 2:] = sz.repeat(D // 16)
    return t


def bench_attn(ctxs, splits_list, batch, kv: str = "fp8"):
    """Decode attention, Qwen3.8-27B head layout (24 q / 4 kv heads, D=256), fp8 or int4 KV."""
    bw, _, src = peaks()
    Hq, Hkv, D, bs = 24, 4, 256, 64
    row_bytes = D if kv == "fp8" else D // 2 + D // 4
    for ctx in ctxs:
        for sp in splits_list:
            for dec in (True, False):
                meta, nblocks = _attn_meta([ctx] * batch, bs, Hq, Hkv, sp, "cuda")
                if kv == "fp8":
                    kc = (torch.randn(nblocks, Hkv, bs, D, device="cuda") * 0.5).to(torch.float8_e4m3fn)
                    vc = torch.randn(nblocks, Hkv, bs, D, device="cuda").to(torch.float8_e4m3fn)
                else:
                    kc, vc = _kv4_random(nblocks, Hkv, bs, D), _kv4_random(nblocks, Hkv, bs, D)
                q = torch.randn(batch, Hq, D, device="cuda").to(torch.bfloat16)
                K._ATTN_DECODE = dec

                def fn(i):
                    K.paged_attention(q, kc, vc, meta, D ** -0.5)
                t = timeit(fn)
                byts = batch * (ctx + 1) * Hkv * row_bytes * 2
                print(json.dumps({"kernel": "paged_attention", "variant": "decode" if dec else "general",
                                  "kv": kv, "batch": batch, "ctx": ctx, "splits": sp,
                                  "us": round(t * 1e6, 2), "GBps": round(byts / t / 1e9, 1),
                                  "frac_hbm": round(byts / t / bw, 3), "peaks": src}), flush=True)
    K._ATTN_DECODE = True


def _int4_random(N, Kd, rows=16384):
    """A random int4 weight built on the host in row blocks (small device footprint)."""
    from ..quant.int4 import Int4Weight
    parts = [Int4Weight.from_float(torch.randn(min(rows, N - r), Kd) * 0.02)
             for r in range(0, N, rows)]
    return Int4Weight(torch.cat([p.packed for p in parts]), torch.cat([p.scales for p in parts]),
                      torch.cat([p.zeros for p in parts]), N, Kd).to("cuda")


def bench_w4a16(ms, shapes):
    """W4A16 int4 (g128) linear, DRAM-cold weight rotation."""
    from ..quant.int4 import w4a16_linear
    bw, fl, src = peaks()
    for (N, Kd, name) in shapes:
        per = N * Kd // 2 + N * (Kd // 128) * 4
        nrot = max(2, int(300e6 // per) + 1)
        ws = [_int4_random(N, Kd) for _ in range(nrot)]
        torch.cuda.empty_cache()
        for M in ms:
            x = torch.randn(M, Kd, device="cuda").to(torch.bfloat16)

            def fn(i):
                w4a16_linear(x, ws[i % nrot])
            t = timeit(fn)
            byts = per + M * Kd * 2 + M * N * 2
            print(json.dumps({"kernel": "w4a16", "shape": name, "M": M, "N": N, "K": Kd,
                              "us": round(t * 1e6, 2), "GBps": round(byts / t / 1e9, 1),
                              "frac_hbm": round(byts / t / bw, 3), "peaks": src}), flush=True)


def bench_gemm_finish(ms, shapes):
    """Decode GEMM whose last CTA runs the next linear's producer (finisher) against the GEMM
    followed by the stand-alone producer kernel."""
    bw, _, src = peaks()
    for (N, Kd, name) in shapes:
        nrot = max(2, int(300e6 // (N * Kd // 2)) + 1)
        ws = [MXFP4Weight.from_float(torch.randn(N, Kd, device="cuda") * 0.02) for _ in range(nrot)]
        mode = K.FIN_SILU if name.startswith("gate_up") else K.FIN_NORM
        for M in ms:
            x = torch.randn(M, Kd, device="cuda").to(torch.bfloat16)
            q, s = K.quant_fp8(x)
            res = torch.randn(M, N, device="cuda").to(torch.bfloat16)
            lw = torch.zeros(N, device="cuda", dtype=torch.bfloat16)
            ro = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)

            def fused(i):
                w = ws[i % nrot]
                if mode == K.FIN_NORM:
                    K.mxfp4_gemm_finish(q, s, w, mode, res, lw, ro, 1e-6)
                else:
                    K.mxfp4_gemm_finish(q, s, w, mode)

            def separate(i):
                w = ws[i % nrot]
                y = K.mxfp4_gemm(q, s, w.packed, w.sf, w.scales, N)
                if mode == K.FIN_NORM:
                    K.add_rms_quant(y, res, lw, 1e-6)
                else:
                    K.silu_mul_quant(y)
            for kname, fn in (("gemm+finisher", fused), ("gemm, producer", separate)):
                t = timeit(fn)
                byts = N * Kd // 2 + N * Kd // 32
                print(json.dumps({"kernel": kname, "shape": name, "M": M, "us": round(t * 1e6, 2),
                                  "frac_hbm": round(byts / t / bw, 3), "peaks": src}), flush=True)


def bench_fmha(q_len, ctxs):
    """Causal prefill attention (27B layout: 24 q / 4 kv heads, D = 256, fp8 pages of 64): the
    tcgen05 kernel and the mma.sync tile kernel, TFLOP/s of the causal work."""
    _, fl, src = peaks()
    Hq, Hkv, D, bs = 24, 4, 256, 64
    for ctx in ctxs:
        L = ctx + q_len
        nb = (L + bs - 1) // bs
        m = _AttnMeta()
        m.block_tables = torch.randperm(nb, dtype=torch.int32).view(1, nb).cuda()
        m.seq_lens = torch.tensor([L], dtype=torch.int32, device="cuda")
        m.query_start_loc = torch.tensor([0, q_len], dtype=torch.int32, device="cuda")
        R = q_len * (Hq // Hkv)
        m.tile_seq = torch.zeros((R + 63) // 64, dtype=torch.int32, device="cuda")
        m.tile_row0 = torch.arange(0, R, 64, dtype=torch.int32, device="cuda")
        m.num_tokens, m.num_seqs, m.num_splits = q_len, 1, 1
        m.scratch_o = lambda s_, T, H, D_: torch.empty(s_, T, H, D_, device="cuda")
        m.scratch_ml = lambda s_, T, H: torch.empty(s_, T, H, 2, device="cuda")
        kc = (torch.randn(nb, Hkv, bs, D, device="cuda") * 0.5).to(torch.float8_e4m3fn)
        vc = torch.randn(nb, Hkv, bs, D, device="cuda").to(torch.float8_e4m3fn)
        q = torch.randn(q_len, Hq, D, device="cuda").to(torch.float8_e4m3fn).to(torch.bfloat16)
        # causal work: each query row sees ctx + its position + 1 keys
        flops = 4.0 * Hq * D * (q_len * ctx + q_len * (q_len + 1) / 2)
        for name, on in (("fmha_tcgen05", True), ("paged_attn_mma_sync", False)):
            K._FMHA = on

            def fn(i):
                K.paged_attention(q, kc, vc, m, D ** -0.5)
            t = timeit(fn, iters=10)
            print(json.dumps({"kernel": name, "q_len": q_len, "ctx": ctx, "us": round(t * 1e6, 1),
                              "TFLOPs": round(flops / t / 1e12, 1),
                              "frac_fp8_tensor_peak": round(flops / t / (2 * fl), 3),
                              "peaks": src + " (fp8 tensor = 2x measured bf16)"}), flush=True)
        K._FMHA = True


def bench_gdn_decode(batches):
    """One-token GDN decode step of the 27B layout (16 k / 48 v heads, dk = dv = 128, fp32 state):
    conv update + norms + gates + delta rule (+ gated norm + e4m3 for the fused-quant variant);
    the state (64 KB per head) is read and written once."""
    bw, _, src = peaks()
    Hk, Hv, D = 16, 48, 128
    key_dim, vdim = Hk * D, Hv * D
    C = 2 * key_dim + vdim
    for B in batches:
        nrot = 8
        states = [torch.randn(B + 1, Hv, D, D, device="cuda") * 0.05 for _ in range(nrot)]
        conv = torch.randn(B + 1, C, 3, device="cuda").to(torch.bfloat16)
        x = torch.randn(B, C + vdim + 2 * Hv + 8, device="cuda").to(torch.bfloat16)
        conv_w = torch.randn(C, 4, device="cuda").to(torch.bfloat16)
        A_log = torch.zeros(Hv, device="cuda")
        dt = torch.zeros(Hv, device="cuda")
        nw = torch.ones(D, device="cuda", dtype=torch.bfloat16)
        m = _AttnMeta()
        m.state_slots = torch.arange(1, B + 1, dtype=torch.int32, device="cuda")
        m.has_initial = torch.ones(B, dtype=torch.int32, device="cuda")
        m.num_seqs = m.num_tokens = B
        byts = B * Hv * D * D * 4 * 2
        for name in ("gdn_decode_fused", "gdn_decode_fused_quant"):
            def fn(i, name=name):
                st = states[i % nrot]
                if name == "gdn_decode_fused":
                    K.gdn_decode_fused(x, C + vdim, conv_w, conv, st, A_log, dt, m, Hk, D ** -0.5, split=1)
                else:
                    K.gdn_decode_fused_quant(x, C + vdim, C, conv_w, conv, st, A_log, dt, m, Hk,
                                             D ** -0.5, nw, 1e-6)
            t = timeit(fn)
            print(json.dumps({"kernel": name, "B": B, "us": round(t * 1e6, 2),
                              "state_GBps": round(byts / t / 1e9, 1),
                              "frac_hbm": round(byts / t / bw, 3), "peaks": src}), flush=True)


def bench_gdn_prefill(lens, head_counts):
    """Prefill chunk scan of one GDN layer (dk = dv = 128, fp32 state, one sequence): the
    one-kernel form against the two-phase form (chunk-parallel solve + state scan), at the
    per-rank head counts of TP 1 / 2 / 4 / 8 (48 / 24 / 12 / 6 value heads, ratio 3)."""
    for Hv in head_counts:
        Hk = max(1, Hv // 3)
        D = 128
        for L in lens:
            y = (torch.randn(L, 2 * Hk * D + Hv * D, device="cuda") * 0.1).to(torch.bfloat16)
            ba = torch.randn(L, 2 * Hv, device="cuda").to(torch.bfloat16)
            A_log = torch.zeros(Hv, device="cuda")
            dt = torch.zeros(Hv, device="cuda")
            st = torch.zeros(2, Hv, D, D, device="cuda")
            m = _AttnMeta()
            m.query_start_loc = torch.tensor([0, L], dtype=torch.int32, device="cuda")
            m.state_slots = torch.tensor([1], dtype=torch.int32, device="cuda")
            m.has_initial = torch.zeros(1, dtype=torch.int32, device="cuda")
            m.num_seqs, m.num_tokens = 1, L
            m.commit_len = None
            out = {}
            for form in (False, True):
                K._GDN_TWO_PHASE = form
                out[form] = timeit(lambda i: K.gdn_recurrent(y, ba, A_log, dt, st, m, Hk, D ** -0.5))
            K._GDN_TWO_PHASE = True
            flops = 2 * L * Hv * D * D * 6          # ~6 [token x D x D] products per token
            print(json.dumps({"kernel": "gdn_chunk_prefill", "L": L, "Hv": Hv,
                              "one_kernel_us": round(out[False] * 1e6, 1),
                              "two_phase_us": round(out[True] * 1e6, 1),
                              "speedup": round(out[False] / out[True], 2),
                              "two_phase_tflops": round(flops / out[True] / 1e12, 1)}), flush=True)


def bench_topk(batches):
    for B in batches:
        x = torch.randn(B, 248320, device="cuda").to(torch.bfloat16)
        temp = torch.full((B,), 0.7, device="cuda")
        tk = torch.full((B,), 20, dtype=torch.int32, device="cuda")
        tp = torch.full((B,), 0.95, device="cuda")
        sd = torch.arange(B, dtype=torch.int64, device="cuda")
        t = timeit(lambda i: K.topk_sample(x, temp, tk, tp, None, sd, i))
        t2 = timeit(lambda i: torch.topk(x.float(), 64, dim=-1))
        print(json.dumps({"kernel": "topk_window+draw", "B": B, "us": round(t * 1e6, 2),
                          "torch_topk_us": round(t2 * 1e6, 2)}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("what", choices=["gemm", "attn", "w4a16", "gemm_fin", "fmha", "topk", "gdn",
                                          "gdn_prefill"])
    ap.add_argument("--q-len", type=int, default=2048)
    ap.add_argument("--ctx", default="1500,4096,16384")
    ap.add_argument("--splits", default="1,4,8,17,32")
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--kv", default="fp8", choices=["fp8", "int4"])
    ap.add_argument("--m", default="1,8,16,64,256,1024,4096")
    ap.add_argument("--shape", default="",
                    help="comma list of shape names or NxK (default: all named shapes)")
    ap.add_argument("--iters", type=int, default=50)
    a = ap.parse_args()
    global ITERS
    ITERS = a.iters
    ms = [int(v) for v in a.m.split(",")]
    shapes = [(16480, 5120, "gdn_in_proj"), (5120, 6144, "out_proj"), (17408, 5120, "gate_up"),
              (5120, 8704, "down"), (14336, 5120, "attn_qkv"), (248320, 5120, "lm_head")]
    if a.shape:
        keep = a.shape.split(",")
        # a name from the table, or an explicit NxK
        shapes = [sh for sh in shapes if sh[2] in keep] + [
            (int(k.split("x")[0]), int(k.split("x")[1]), k) for k in keep if "x" in k]
    if a.what == "gemm":
        bench_gemm(ms, shapes)
    elif a.what == "w4a16":
        bench_w4a16([m for m in ms if m <= 8] or [1], shapes)
    elif a.what == "attn":
        bench_attn([int(v) for v in a.ctx.split(",")], [int(v) for v in a.splits.split(",")],
                   a.batch, a.kv)
    elif a.what == "gemm_fin":
        bench_gemm_finish([m for m in ms if m <= 16] or [1],
                          [sh for sh in shapes if sh[2] in ("out_proj", "gate_up", "down")] or shapes)
    elif a.what == "fmha":
        bench_fmha(a.q_len, [int(v) for v in a.ctx.split(",")])
    elif a.what == "topk":
        bench_topk([int(v) for v in a.m.split(",")])
    elif a.what == "gdn":
        bench_gdn_decode([int(v) for v in a.m.split(",")])
    elif a.what == "gdn_prefill":
        bench_gdn_prefill([int(v) for v in a.ctx.split(",")], [48, 24, 12, 6])


if __name__ == "__main__":
    main()
