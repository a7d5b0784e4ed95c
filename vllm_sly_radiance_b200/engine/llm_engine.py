"""LLMEngine: scheduler + KV/state cache manager + model runner (+ speculative decoding).

API (vLLM-compatible subset): ``add_request``, ``abort_request``, ``step`` ->
``list[RequestOutput]``, ``has_unfinished_requests``.  With tensor parallelism every rank runs
the same engine on the same request stream (SPMD); rank 0 returns outputs.
"""
from __future__ import annotations

import logging
import time
from typing import Optional, Union

import torch

from ..config import EngineConfig, ModelConfig
from ..models.hybrid import HybridModel, TPInfo
from ..ops import kernels as K
from ..utils.metrics import EngineMetrics
from .kv_cache import KVCacheManager
from .model_runner import ModelRunner
from .request import CompletionOutput, Request, RequestOutput, SamplingParams
from .scheduler import Scheduler
from .tokenizer import IncrementalDetokenizer, get_tokenizer

log = logging.getLogger("radiance.engine")


class EngineStepError(RuntimeError):
    """A step could not complete (e.g. a collective failed because a peer rank left); every open
    request was aborted."""


class LLMEngine:
    def __init__(self, config: EngineConfig, model: Optional[HybridModel] = None,
                 tokenizer=None, tp: Optional[TPInfo] = None, tokenizer_path: Optional[str] = None):
        self.config = config
        self.device = torch.device(config.device if (config.device != "cuda" or torch.cuda.is_available()) else "cpu")
        mcfg: ModelConfig = config.model_config()
        self.model_config = mcfg
        self.tp = tp or TPInfo()
        t0 = time.time()
        if model is None:
            quant = config.quantization if config.gemm_backend == "native" else "fp8"
            if quant == "nvfp4":
                quant = "mxfp4"
            model = HybridModel(mcfg, quant=quant, device=self.device, seed=config.seed, tp=self.tp,
                                lm_head_quant=config.lm_head_quant,
                                embed_quant=config.embed_quant)
        self.model = model
        self.load_time = time.time() - t0
        self.tokenizer = tokenizer or get_tokenizer(tokenizer_path, mcfg.vocab_size)
        self.eos_token_id = getattr(self.tokenizer, "eos_token_id", None)
        # ---- cache sizing ----
        bs = config.block_size
        num_slots = config.max_num_seqs + 2
        pin = None
        if not config.num_kv_blocks and self.device.type == "cuda":
            # a pool size measured on this device by `calibrate-kv`, when one exists
            from ..entrypoints.hw import lookup_pin
            pin = lookup_pin(torch.cuda.get_device_name(self.device), config.model,
                             config.tensor_parallel_size, config.max_num_seqs,
                             config.max_num_batched_tokens)
        if config.num_kv_blocks:
            num_blocks = config.num_kv_blocks
        elif pin:
            num_blocks = pin
        elif self.device.type == "cuda":
            torch.cuda.synchronize()
            free, total = torch.cuda.mem_get_info(self.device)
            per_block = max(1, model.cache_bytes_per_block(bs, config.kv_cache_dtype))
            n_snap_b = config.prefix_snapshot_slots if config.enable_prefix_caching else 0
            state = model.state_bytes_per_slot(config.ssm_state_dtype) * (num_slots + n_snap_b)
            activ = 4 << 30   # activations / graphs headroom
            budget = int(free - (1 - config.gpu_memory_utilization) * total) - state - activ
            need = (config.max_model_len + bs - 1) // bs * config.max_num_seqs + 1
            num_blocks = max(8, min(budget // per_block, need * 4))
        else:
            num_blocks = (config.max_model_len + bs - 1) // bs * config.max_num_seqs + 1
        self.num_blocks = int(num_blocks)
        n_snap = config.prefix_snapshot_slots if config.enable_prefix_caching else 0
        if n_snap and config.speculative_method == "dflash2":
            raise ValueError("prefix caching with the DFlash2 drafter is not supported: a cached "
                             "prefix would skip the target forward that feeds the drafter context")
        self.caches = model.make_caches(self.num_blocks, bs, num_slots + n_snap,
                                        config.kv_cache_dtype, config.ssm_state_dtype)
        self.kv = KVCacheManager(self.num_blocks, bs, num_slots, config.enable_prefix_caching,
                                 num_snapshots=n_snap,
                                 snapshot_interval=config.prefix_snapshot_interval)
        if config.enable_prefix_caching and (config.kv_offload_gb > 0 or config.kv_offload_disk_dir):
            from .kv_offload import OffloadManager
            self.kv.offload = OffloadManager(
                self.caches, int(config.kv_offload_gb * (1 << 30)), config.kv_offload_disk_dir,
                int(config.kv_offload_disk_gb * (1 << 30)), config.kv_offload_policy,
                state_fraction=config.kv_offload_state_fraction)
        k = config.num_speculative_tokens if config.speculative_method else 0
        self.scheduler = Scheduler(self.kv, config.max_num_seqs, config.max_num_batched_tokens,
                                   config.max_model_len, num_spec_tokens=k)
        self.runner = ModelRunner(model, self.caches, max_num_seqs=config.max_num_seqs,
                                  max_num_tokens=config.max_num_batched_tokens,
                                  max_model_len=config.max_model_len, device=self.device,
                                  enable_graphs=config.enable_cuda_graphs,
                                  graph_max_bs=config.cuda_graph_max_bs, num_spec_tokens=k)
        if config.capture_graphs_at_start and self.device.type == "cuda":
            t1 = time.time()
            self.runner.capture_all()
            log.info("captured %d decode graphs in %.1fs", len(self.runner.graphs), time.time() - t1)
        self.spec = None
        if config.speculative_method:
            from ..spec_decode.proposer import build_proposer
            self.spec = build_proposer(config, self)
        self.requests: dict[str, Request] = {}
        self.detok: dict[str, IncrementalDetokenizer] = {}
        self.metrics = EngineMetrics()
        from ..utils.step_trace import StepTrace
        self.trace = StepTrace(device=self.device)     # RADIANCE_STEP_TRACE=N
        self.faults = 0
        self.kv_tokens_capacity = self.num_blocks * bs
        log.info("engine ready: %d KV blocks (%d tokens), %d state slots, load %.1fs",
                 self.num_blocks, self.kv_tokens_capacity, num_slots, self.load_time)

    # ------------------------------------------------------------------------------------------
    def add_request(self, prompt: Union[str, list[int]], params: Optional[SamplingParams] = None,
                    request_id: Optional[str] = None) -> str:
        params = params or SamplingParams()
        ids = self.tokenizer.encode(prompt) if isinstance(prompt, str) else list(prompt)
        req = Request(ids, params, request_id, eos_token_id=self.eos_token_id)
        self.scheduler.add(req)
        self.requests[req.request_id] = req
        self.detok[req.request_id] = IncrementalDetokenizer(self.tokenizer, params.stop)
        self.metrics.on_arrival()
        return req.request_id

    def abort_request(self, request_id: str) -> bool:
        ok = self.scheduler.abort(request_id)
        self.requests.pop(request_id, None)
        self.detok.pop(request_id, None)
        return ok

    def has_unfinished_requests(self) -> bool:
        return self.scheduler.has_unfinished()

    # ------------------------------------------------------------------------------------------
    def step(self) -> list[RequestOutput]:
        t0 = time.perf_counter()
        tr = self.trace.begin()
        sched = self.scheduler.schedule()
        self.trace.mark(tr, "t_sched")
        if self.kv.offload is not None:
            self.kv.flush_offload()    # write-backs of blocks evicted by this schedule
        if sched.is_empty:
            return []
        for s in sched.seqs:         # prefix-cache hits resume from a GDN state snapshot
            if s.req.restore_snapshot is not None:
                self.model.copy_state(self.caches, s.req.restore_snapshot, s.req.state_slot)
                self.kv.release_restore(s.req)     # the copy is on the stream: slot reusable
        try:
            if self.spec is not None:
                result = self.spec.execute(sched)
            else:
                result = self.runner.execute(sched)
            code = self.runner.read_status()
            if K._CANARY:
                K.check_canaries()          # debug mode: no kernel wrote past its workspace
        except Exception as e:
            # a failed collective (a peer rank that left or timed out) or any other step error:
            # the step's outputs are lost, so no open request can continue
            n = self._abort_all()
            log.error("step failed (%r): %d open requests failed", e, n)
            raise EngineStepError(f"engine step failed: {e!r}") from e
        if code:
            self._fail_open_requests(code)
        self.trace.mark(tr, "t_exec")
        finished = self.scheduler.update(sched, result.sampled)
        if self.kv.num_snapshots:
            for s in sched.seqs:
                if not s.is_decode and s.req.state_slot is not None:
                    sid = self.kv.take_snapshot(s.req)
                    if sid is not None:
                        self.model.copy_state(self.caches, s.req.state_slot, sid)
        self.metrics.on_step(sched, result, time.perf_counter() - t0, self.kv.usage,
                             len(self.scheduler.running), len(self.scheduler.waiting))
        outs = []
        fin_ids = {r.request_id for r in finished}
        for s in sched.seqs:
            req = s.req
            rid = req.request_id
            if rid not in result.sampled and rid not in fin_ids:
                continue
            det = self.detok.get(rid)
            if det is not None:
                det.update(req.output_token_ids)
                if det.stopped and not req.status.finished:
                    self.scheduler.abort(rid)
                    from .request import RequestStatus
                    req.status = RequestStatus.FINISHED_STOPPED
                    fin_ids.add(rid)
            done = req.status.finished
            text = det.text if det else ""
            outs.append(RequestOutput(
                request_id=rid, prompt_token_ids=req.prompt_token_ids,
                outputs=[CompletionOutput(0, text, list(req.output_token_ids),
                                          req.status.value if done else None)],
                finished=done,
                metrics=dict(arrival=req.arrival_time, first_token=req.first_token_time,
                             finish=req.finish_time, num_preemptions=req.num_preemptions)))
            if done:
                self.metrics.on_finish(req)
                self.requests.pop(rid, None)
                self.detok.pop(rid, None)
        self.trace.end(tr, result.num_tokens)
        return outs

    def _fail_open_requests(self, code: int):
        """A kernel of this step recorded an error (a bounded wait expired or a bad index was
        refused): its outputs are not valid.  Every open request is aborted and the step raises;
        the OpenAI server turns this into an error for each client and reports itself unhealthy."""
        from ..ops.kernels import KernelFaultError, reset_status
        reset_status(self.device)
        n = self._abort_all()
        log.error("kernel fault (status %d): %d open requests failed", code, n)
        self.faults += 1
        raise KernelFaultError(code)

    def _abort_all(self) -> int:
        ids = list(self.requests)
        for rid in ids:
            self.abort_request(rid)
        return len(ids)

    def generate(self, prompts, params=None) -> list[RequestOutput]:
        if isinstance(params, SamplingParams) or params is None:
            params = [params or SamplingParams()] * len(prompts)
        order = [self.add_request(p, sp) for p, sp in zip(prompts, params)]
        final = {}
        while self.has_unfinished_requests():
            for o in self.step():
                if o.finished:
                    final[o.request_id] = o
        return [final[r] for r in order]
