"""Expert-parallel MoE layer benchmark (config 5 shapes: hidden 2048, 256 experts, top-8, expert
intermediate 512): one routed-expert call per iteration (dispatch, grouped W4A8 gate_up and down,
combine) with the all_to_all transport and with the NVLink peer-memory transport.

    python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 \\
        -m vllm_sly_radiance_b200.benchmarks.ep --tokens 64

Device time with CUDA events around `iters` back-to-back calls after `warmup` calls, max over
ranks.  Prints one JSON line per transport (rank 0).
"""
from __future__ import annotations

import argparse
import json
import os
from datetime import timedelta

import torch


def main():
    import torch.distributed as dist
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=64, help="tokens per rank per call")
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    a = ap.parse_args()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120))
    from ..config import moe_hybrid
    from ..models.hybrid import TPInfo
    from ..models.moe import MoEBlock
    from ..models.weights import RandomWeights
    from ..ops import kernels as K
    from ..parallel.ep import make_ep_group
    cfg = moe_hybrid()
    dev = torch.device("cuda", local)
    res = {}
    for backend in ("a2a", "p2p"):
        ep = make_ep_group(rank, world, backend)
        if backend == "p2p":
            ep.transport.maxt = max(a.tokens, 64)
        blk = MoEBlock(cfg, TPInfo(), "mxfp4", RandomWeights(cfg, 0, dev), "layers.0.", ep=ep)
        blk.to(dev)
        g = torch.Generator(device=dev)
        g.manual_seed(rank)
        x = torch.randn(a.tokens, cfg.hidden_size, generator=g, device=dev).to(torch.bfloat16)
        q, s = K.quant_fp8(x)
        ids, w = blk.route(x)
        for _ in range(a.warmup):
            ep.transport.dispatch_combine(blk, x, (q, s), ids, w)
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(a.iters):
            ep.transport.dispatch_combine(blk, x, (q, s), ids, w)
        e1.record()
        torch.cuda.synchronize()
        us = torch.tensor([e0.elapsed_time(e1) * 1e3 / a.iters], device=dev)
        dist.all_reduce(us, op=dist.ReduceOp.MAX)
        K.check_status(dev)
        res[backend] = float(us)
        if backend == "p2p":
            dist.barrier()
            ep.transport.close()
        del blk
    if rank == 0:
        H, Kk = cfg.hidden_size, cfg.num_experts_per_tok
        # rows that leave this rank: dispatch (e4m3 row + 8 bytes) and combine (bf16 row)
        remote = a.tokens * Kk * (world - 1) / world
        nv_bytes = remote * (H + 8) + remote * 2 * H
        for backend, us in res.items():
            print(json.dumps({"bench": "ep_moe_layer", "transport": backend, "world": world,
                              "tokens_per_rank": a.tokens, "experts": cfg.num_experts,
                              "top_k": Kk, "hidden": H, "us_per_call": round(us, 2),
                              "nvlink_bytes_per_rank": int(nv_bytes),
                              "nvlink_floor_us": round(nv_bytes / 770e9 * 1e6, 2)}), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
