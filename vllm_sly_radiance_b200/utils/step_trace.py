"""Per-step timing trace without a profiler: RADIANCE_STEP_TRACE=N logs a summary every N engine
steps (0 = off; nothing is timed).  Numbers per step, medians over the window:

  schedule   host time in the scheduler (continuous batching, KV / state allocation)
  execute    host time from the step's first launch to its result on the host: input build,
             graph replay or eager launches, and the wait for the sampled ids
  gpu        device time of the step's work on the launching stream (CUDA events)
  host_gap   execute - gpu: the part of the step the device spends waiting on the host
  update     host time to advance requests (stop checks, detokenisation, outputs)
  interval   time between consecutive step ends (the effective step time)

Reference behaviour: patch_step_trace.py (exec_model / sample_tok / rpc_wait / out_wait / out_iv
of the vLLM worker, CUDA events + perf_counter, summary every N steps on rank 0)."""
from __future__ import annotations

import logging
import os
import statistics
import time
from typing import Optional

import torch

log = logging.getLogger("radiance.steptrace")


class StepTrace:
    def __init__(self, every: Optional[int] = None, device=None):
        self.every = int(os.environ.get("RADIANCE_STEP_TRACE", "0") or 0) if every is None else every
        self.cuda = device is not None and torch.device(device).type == "cuda"
        self.rows: list = []
        self.pending: list = []
        self.last_end: Optional[float] = None
        self.summaries: list = []

    @property
    def enabled(self) -> bool:
        return self.every > 0

    def begin(self):
        if not self.enabled:
            return None
        rec = {"t0": time.perf_counter()}
        if self.cuda:
            rec["ev0"] = torch.cuda.Event(enable_timing=True)
            rec["ev0"].record()
        return rec

    def mark(self, rec, name: str):
        if rec is not None:
            rec[name] = time.perf_counter()

    def end(self, rec, num_tokens: int = 0):
        if rec is None:
            return
        rec["t_end"] = time.perf_counter()
        rec["tokens"] = num_tokens
        if self.cuda:
            rec["ev1"] = torch.cuda.Event(enable_timing=True)
            rec["ev1"].record()
        if self.last_end is not None:
            rec["interval"] = rec["t_end"] - self.last_end
        self.last_end = rec["t_end"]
        self.pending.append(rec)
        if len(self.pending) >= self.every:
            self._flush()

    def _flush(self):
        rows = []
        for r in self.pending:
            row = {"schedule": r.get("t_sched", r["t0"]) - r["t0"],
                   "execute": r.get("t_exec", r["t_end"]) - r.get("t_sched", r["t0"]),
                   "update": r["t_end"] - r.get("t_exec", r["t_end"]),
                   "tokens": r["tokens"]}
            if "interval" in r:
                row["interval"] = r["interval"]
            if self.cuda:
                r["ev1"].synchronize()
                row["gpu"] = r["ev0"].elapsed_time(r["ev1"]) / 1e3
                row["host_gap"] = max(0.0, row["execute"] - row["gpu"])
            rows.append(row)
        self.pending = []
        summ = {k: statistics.median(r[k] for r in rows if k in r) * 1e3
                for k in ("schedule", "execute", "gpu", "host_gap", "update", "interval")
                if any(k in r for r in rows)}
        summ["steps"] = len(rows)
        summ["tokens_per_step"] = statistics.mean(r["tokens"] for r in rows)
        self.summaries.append(summ)
        log.info("step trace (median ms over %d steps): %s", len(rows),
                 " ".join(f"{k}={v:.3f}" for k, v in summ.items() if k not in ("steps",)))
