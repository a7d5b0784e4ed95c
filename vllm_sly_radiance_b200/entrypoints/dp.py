"""Data parallelism: independent engine replicas, one process (and one GPU) each, behind one
engine-shaped front end.

``DataParallelEngine`` offers what the server's engine loop and ``LLMEngine.generate`` use --
``add_request``, ``abort_request``, ``has_unfinished_requests``, ``step``, ``config``,
``metrics`` -- and routes each new request to the replica with the fewest requests in flight.
A replica runs the full engine (scheduler, KV cache, CUDA graphs) on its own device and streams
its ``RequestOutput`` objects back; the front end never touches a GPU.  Replicas may themselves be
tensor-parallel groups only through the SPMD launcher (one process per rank); this module covers
the one-GPU-per-replica case the reference serves with ``--data-parallel-size`` (vLLM's DP
front end, ``README.md`` launch flags).
"""
from __future__ import annotations

import dataclasses
import itertools
import multiprocessing as mp
import queue
import time
from typing import Optional

from ..config import EngineConfig
from ..engine.request import RequestOutput, SamplingParams


def _replica_main(idx: int, cfg: EngineConfig, cmd_q, out_q):
    """Replica process: an engine on its own device; commands in, outputs out."""
    import torch
    from ..engine.llm_engine import LLMEngine
    if cfg.device.startswith("cuda"):
        torch.cuda.set_device(idx if cfg.device == "cuda" else torch.device(cfg.device).index)
    try:
        eng = LLMEngine(cfg)
    except Exception as e:            # report the failure instead of hanging the front end
        out_q.put(("dead", idx, repr(e)))
        return
    out_q.put(("ready", idx, None))
    running = True
    while running:
        cmds = []
        try:
            if not eng.has_unfinished_requests():
                cmds.append(cmd_q.get(timeout=0.05))
            while True:
                cmds.append(cmd_q.get_nowait())
        except queue.Empty:
            pass
        for c in cmds:
            if c[0] == "stop":
                running = False
            elif c[0] == "add":
                try:
                    eng.add_request(c[1], c[2], c[3])
                except Exception as e:
                    out_q.put(("error", c[3], repr(e)))
            elif c[0] == "abort":
                eng.abort_request(c[1])
        if running and eng.has_unfinished_requests():
            try:
                outs = eng.step()
            except Exception as e:
                out_q.put(("step_error", idx, repr(e)))
                continue
            if outs:
                out_q.put(("out", idx, outs))


class _DPMetrics:
    def __init__(self, owner: "DataParallelEngine"):
        self.owner = owner

    def prometheus(self, model_name: str) -> str:
        lines = ["# TYPE vllm:num_requests_running gauge"]
        for i, n in enumerate(self.owner.inflight):
            lines.append(f'vllm:num_requests_running{{model_name="{model_name}",replica="{i}"}} {n}')
        lines.append("# TYPE vllm:generation_tokens_total counter")
        lines.append(f'vllm:generation_tokens_total{{model_name="{model_name}"}} '
                     f"{self.owner.generated_tokens}")
        return "\n".join(lines) + "\n"


class DataParallelEngine:
    def __init__(self, config: EngineConfig, num_replicas: int, devices: Optional[list] = None,
                 start_timeout: float = 600.0, tokenizer_path: Optional[str] = None):
        if num_replicas < 1:
            raise ValueError("data-parallel size must be >= 1")
        from ..engine.tokenizer import get_tokenizer
        self.config = config
        # the front end's own tokenizer (chat templates); the replicas detokenize their outputs
        self.tokenizer = get_tokenizer(tokenizer_path, config.model_config().vocab_size)
        self.n = num_replicas
        ctx = mp.get_context("spawn")
        self.out_q = ctx.Queue()
        self.cmd_qs = [ctx.Queue() for _ in range(num_replicas)]
        self.procs = []
        for i in range(num_replicas):
            dev = devices[i] if devices else (f"cuda:{i}" if config.device.startswith("cuda")
                                              else config.device)
            cfg_i = dataclasses.replace(config, device=dev)
            p = ctx.Process(target=_replica_main, args=(i, cfg_i, self.cmd_qs[i], self.out_q),
                            daemon=True)
            p.start()
            self.procs.append(p)
        self.owner: dict = {}            # request id -> replica
        self.inflight = [0] * num_replicas
        self.generated_tokens = 0
        self.metrics = _DPMetrics(self)
        self._ids = itertools.count()
        self._pending: list = []
        ready, t0 = 0, time.time()
        while ready < num_replicas:
            left = start_timeout - (time.time() - t0)
            if left <= 0:
                self.shutdown()
                raise TimeoutError("data-parallel replicas did not start")
            kind, idx, info = self.out_q.get(timeout=left)
            if kind == "dead":
                self.shutdown()
                raise RuntimeError(f"replica {idx} failed to start: {info}")
            if kind == "ready":
                ready += 1
            else:
                self._pending.append((kind, idx, info))

    # ---- engine-shaped API ----
    def add_request(self, prompt, params: Optional[SamplingParams] = None,
                    request_id: Optional[str] = None) -> str:
        rid = request_id if request_id is not None else f"dp-{next(self._ids)}"
        r = min(range(self.n), key=lambda i: (self.inflight[i], i))
        self.owner[rid] = r
        self.inflight[r] += 1
        self.cmd_qs[r].put(("add", prompt, params or SamplingParams(), rid))
        return rid

    def abort_request(self, request_id: str) -> None:
        r = self.owner.pop(request_id, None)
        if r is not None:
            self.inflight[r] -= 1
            self.cmd_qs[r].put(("abort", request_id))

    def has_unfinished_requests(self) -> bool:
        return bool(self.owner)

    def step(self, timeout: float = 0.05) -> list[RequestOutput]:
        """Outputs the replicas produced since the last call (waits up to `timeout` for one)."""
        msgs = self._pending
        self._pending = []
        try:
            if not msgs:
                msgs.append(self.out_q.get(timeout=timeout))
            while True:
                msgs.append(self.out_q.get_nowait())
        except queue.Empty:
            pass
        outs = []
        for kind, idx, info in msgs:
            if kind == "out":
                for o in info:
                    if o.request_id not in self.owner:
                        continue                       # aborted meanwhile
                    if o.finished:
                        r = self.owner.pop(o.request_id)
                        self.inflight[r] -= 1
                        self.generated_tokens += sum(len(c.token_ids) for c in o.outputs)
                    outs.append(o)
            elif kind == "error":                      # a request the replica rejected
                r = self.owner.pop(idx, None)
                if r is not None:
                    self.inflight[r] -= 1
                raise ValueError(f"request {idx}: {info}")
            elif kind == "step_error":
                raise RuntimeError(f"replica {idx} step failed: {info}")
        return outs

    def generate(self, prompts, params=None) -> list[RequestOutput]:
        if isinstance(params, SamplingParams) or params is None:
            params = [params or SamplingParams()] * len(prompts)
        order = [self.add_request(p, sp) for p, sp in zip(prompts, params)]
        final = {}
        while self.has_unfinished_requests():
            for o in self.step(timeout=1.0):
                if o.finished:
                    final[o.request_id] = o
        return [final[r] for r in order]

    def shutdown(self) -> None:
        for q in self.cmd_qs:
            try:
                q.put(("stop",))
            except Exception:
                pass
        for p in self.procs:
            p.join(timeout=30)
            if p.is_alive():
                p.terminate()
        self.procs = []

    def __del__(self):
        if getattr(self, "procs", None):
            self.shutdown()
