"""Command line:  python -m vllm_sly_radiance_b200 serve --model qwen38_27b [--tensor-parallel-size N]

Flags mirror the vLLM ones the reference launches with (``serve-mxfp4.sh:1326-1337``); each
EngineConfig field is also settable by a RADIANCE_<FIELD> environment variable.  With
--tensor-parallel-size N > 1 the command re-executes itself under torch.distributed.run (one
process per GPU, NCCL), rank 0 serving HTTP."""
from __future__ import annotations

import argparse
import dataclasses
import datetime
import logging
import os
import sys

from ..config import EngineConfig


def _parser():
    ap = argparse.ArgumentParser(prog="vllm_sly_radiance_b200")
    sub = ap.add_subparsers(dest="cmd", required=True)
    s = sub.add_parser("serve", help="OpenAI-compatible server")
    s.add_argument("model_pos", nargs="?", default=None)
    s.add_argument("--host", default="0.0.0.0")
    s.add_argument("--port", type=int, default=8000)
    s.add_argument("--served-model-name", default=None)
    s.add_argument("--tokenizer", default=None)
    s.add_argument("--reasoning-parser", default=None)
    s.add_argument("--tool-call-parser", default=None)
    s.add_argument("--enable-auto-tool-choice", action="store_true")
    s.add_argument("--speculative-method", default=None)
    s.add_argument("--data-parallel-size", type=int, default=1,
                   help="independent engine replicas, one GPU each, behind this server")
    for f in dataclasses.fields(EngineConfig):
        flag = "--" + f.name.replace("_", "-")
        if flag in ("--speculative-method",):
            continue
        if f.type in (bool, "bool"):
            s.add_argument(flag, dest=f.name, action=argparse.BooleanOptionalAction, default=None)
        else:
            s.add_argument(flag, dest=f.name, default=None)
    d = sub.add_parser("gpus", help="detect usable GPUs, pick the TP size, show the KV pin")
    d.add_argument("--model", default="qwen38_27b")
    d.add_argument("--min-gpu-mib", type=int, default=8192)
    c = sub.add_parser("calibrate-kv", help="measure the largest KV pool that survives a "
                                            "chunk-sized prefill + decode and save it")
    c.add_argument("--model", default="qwen38_27b")
    c.add_argument("--max-num-seqs", type=int, default=8)
    c.add_argument("--max-num-batched-tokens", type=int, default=4096)
    c.add_argument("--max-model-len", type=int, default=65536)
    c.add_argument("--dry-run", action="store_true")
    g = sub.add_parser("generate", help="one-shot offline generation")
    g.add_argument("--model", default="tiny_hybrid")
    g.add_argument("--prompt", default="Hello")
    g.add_argument("--max-tokens", type=int, default=32)
    g.add_argument("--temperature", type=float, default=0.0)
    g.add_argument("--device", default="cuda")
    return ap


def _engine_config(ns) -> EngineConfig:
    kw = {}
    for f in dataclasses.fields(EngineConfig):
        v = getattr(ns, f.name, None)
        if v is None:
            continue
        cur = f.default
        if isinstance(cur, bool):
            kw[f.name] = bool(v)
        elif isinstance(cur, int) and not isinstance(cur, bool):
            kw[f.name] = int(v)
        elif isinstance(cur, float):
            kw[f.name] = float(v)
        else:
            kw[f.name] = v
    if getattr(ns, "model_pos", None):
        kw["model"] = ns.model_pos
    if getattr(ns, "speculative_method", None):
        kw["speculative_method"] = ns.speculative_method
    return EngineConfig(**kw)


def serve(ns):
    import torch
    cfg = _engine_config(ns)
    tp = cfg.tensor_parallel_size
    if tp > 1 and "RANK" not in os.environ:
        cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={tp}",
               "--master-addr", "127.0.0.1", "--master-port", os.environ.get("RADIANCE_PORT", "29511"),
               "-m", "vllm_sly_radiance_b200"] + sys.argv[1:]
        os.execvp(cmd[0], cmd)
    from ..engine.llm_engine import LLMEngine
    from ..models.hybrid import TPInfo
    tpi = TPInfo()
    bcast = None
    if tp > 1:
        import torch.distributed as dist
        rank = int(os.environ["RANK"])
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600))
        from ..parallel.comm import make_tp_info
        from ..parallel.spmd import RequestBroadcaster, follower_loop
        tpi = make_tp_info(rank, tp, cfg.comm_backend)
        cpu = dist.new_group(backend="gloo")
        bcast = RequestBroadcaster(rank, cpu)
        engine = LLMEngine(cfg, tp=tpi, tokenizer_path=ns.tokenizer)
        if rank != 0:
            follower_loop(engine, bcast)
            return
    elif getattr(ns, "data_parallel_size", 1) > 1:
        from .dp import DataParallelEngine
        engine = DataParallelEngine(cfg, ns.data_parallel_size, tokenizer_path=ns.tokenizer)
    else:
        engine = LLMEngine(cfg, tokenizer_path=ns.tokenizer)
    import uvicorn
    from .openai_server import build_app
    app = build_app(engine, ns.served_model_name or cfg.model, ns.reasoning_parser,
                    ns.tool_call_parser, bcast)
    uvicorn.run(app, host=ns.host, port=ns.port, log_level="info")


def generate(ns):
    from ..engine.llm import LLM
    from ..engine.request import SamplingParams
    llm = LLM(ns.model, device=ns.device)
    out = llm.generate([ns.prompt], SamplingParams(temperature=ns.temperature, max_tokens=ns.max_tokens))
    print(out[0].outputs[0].text)


def gpus(ns):
    import json
    from ..config import get_model_config
    from .hw import detect_gpus
    print(json.dumps(detect_gpus(get_model_config(ns.model), min_mib=ns.min_gpu_mib), indent=1))


def calibrate(ns):
    from .hw import calibrate_kv, search_blocks
    cfg = EngineConfig(model=ns.model, max_num_seqs=ns.max_num_seqs,
                       max_num_batched_tokens=ns.max_num_batched_tokens,
                       max_model_len=ns.max_model_len)
    if ns.dry_run:
        print(f"would search num_kv_blocks for {cfg.model} at max_num_seqs={cfg.max_num_seqs}, "
              f"chunk={cfg.max_num_batched_tokens}: engine start + one chunk prefill + decode per try")
        return
    print(f"num_kv_blocks = {calibrate_kv(cfg)}")


def main(argv=None):
    logging.basicConfig(level=logging.INFO, format="[radiance] %(message)s")
    ns = _parser().parse_args(argv)
    if ns.cmd == "serve":
        serve(ns)
    elif ns.cmd == "generate":
        generate(ns)
    elif ns.cmd == "gpus":
        gpus(ns)
    elif ns.cmd == "calibrate-kv":
        calibrate(ns)


if __name__ == "__main__":
    main()
