"""Continuous-batching scheduler with chunked prefill (vLLM V1 semantics).

Each step gets a token budget (``max_num_batched_tokens``) and a sequence cap
(``max_num_seqs``).  Running requests are served first: a decoding request takes 1 token
(1 + k with speculative decoding, k per request under adaptive width), a request still in its
prompt takes the next prompt chunk.  Leftover budget admits waiting requests (FCFS), whose
prompt is chunked to fit.  When the KV pool is exhausted the most recently admitted running
request is preempted (recompute: its blocks and state slot are freed and it re-enters the
waiting queue at the front).  The step's batch is ordered decodes first, then prefill chunks.
Reference: vLLM V1 scheduler as configured by the reference (``serve-mxfp4.sh:1326-1337``:
``--max-num-seqs 8 --max-num-batched-tokens 4096``, chunked prefill on).
"""
from __future__ import annotations

from collections import deque
from dataclasses import dataclass, field
from typing import Optional

from .kv_cache import KVCacheManager
from .request import Request, RequestStatus


@dataclass
class ScheduledSeq:
    req: Request
    num_new_tokens: int          # tokens fed this step (prompt chunk, 1 decode token, or 1+k)
    is_decode: bool
    draft_tokens: list = field(default_factory=list)   # speculative tokens appended after the last

    @property
    def samples(self) -> bool:
        """Whether this step produces a sampled token for the request (prompt fully consumed)."""
        return self.req.num_computed_tokens + self.num_new_tokens >= self.req.num_tokens


@dataclass
class SchedulerOutput:
    seqs: list
    num_tokens: int
    preempted: list
    finished_ids: list

    @property
    def num_decodes(self) -> int:
        return sum(1 for s in self.seqs if s.is_decode)

    @property
    def is_empty(self) -> bool:
        return not self.seqs


class Scheduler:
    def __init__(self, kv: KVCacheManager, max_num_seqs: int, max_num_batched_tokens: int,
                 max_model_len: int, num_spec_tokens: int = 0):
        self.kv = kv
        self.max_num_seqs = max_num_seqs
        self.max_tokens = max_num_batched_tokens
        self.max_model_len = max_model_len
        self.num_spec_tokens = num_spec_tokens
        self.waiting: deque[Request] = deque()
        self.running: list[Request] = []
        self.finished_ids: list[str] = []
        self.num_preemptions = 0

    # ---- queue management ----
    def add(self, req: Request):
        if req.num_prompt_tokens == 0:
            raise ValueError("empty prompt")
        if req.num_prompt_tokens >= self.max_model_len:
            raise ValueError(f"prompt of {req.num_prompt_tokens} tokens exceeds max_model_len "
                             f"{self.max_model_len}")
        self.waiting.append(req)

    def abort(self, request_id: str) -> bool:
        for q in (self.running, self.waiting):
            for r in list(q):
                if r.request_id == request_id:
                    q.remove(r)
                    self.kv.free(r)
                    r.status = RequestStatus.FINISHED_ABORTED
                    self.finished_ids.append(r.request_id)
                    return True
        return False

    def has_unfinished(self) -> bool:
        return bool(self.waiting or self.running)

    # ---- scheduling ----
    def _preempt(self, victim: Request):
        self.running.remove(victim)
        self.kv.free(victim)
        victim.status = RequestStatus.PREEMPTED
        victim.num_computed_tokens = 0
        victim.num_preemptions += 1
        self.num_preemptions += 1
        self.waiting.appendleft(victim)

    def schedule(self) -> SchedulerOutput:
        budget = self.max_tokens
        seqs: list[ScheduledSeq] = []
        preempted: list[Request] = []
        scheduled = set()

        # 1) running requests, in admission order
        i = 0
        while i < len(self.running) and budget > 0:
            req = self.running[i]
            remaining = req.num_tokens - req.num_computed_tokens
            decoding = remaining == 1
            if decoding:
                k = self.num_spec_tokens if req.spec_width is None else req.spec_width
                k = min(k, len(req.draft_token_ids))
                n = 1 + k
                if n > budget:
                    k = max(0, budget - 1)
                    n = 1 + k
            else:
                n = self._chunk(req, min(remaining, budget))
                k = 0
            # make room (preempting from the back if needed)
            while not self.kv.allocate(req, req.num_computed_tokens + n):
                victim = self.running[-1]
                if victim is req:
                    break
                self._preempt(victim)
                preempted.append(victim)
            if req not in self.running:        # req preempted itself (pool too small)
                continue
            if len(req.block_ids) * self.kv.block_size < req.num_computed_tokens + n:
                self._preempt(req)
                preempted.append(req)
                continue
            seqs.append(ScheduledSeq(req, n, decoding, list(req.draft_token_ids[:k]) if decoding else []))
            scheduled.add(req.request_id)
            budget -= n
            i += 1

        # 2) admit waiting requests
        while self.waiting and budget > 0 and len(self.running) < self.max_num_seqs:
            req = self.waiting[0]
            if req.num_computed_tokens == 0 and not req.block_ids:
                cached = self.kv.match_prefix(req)
                if cached:
                    self.kv.adopt_prefix(req, cached)
                    req.num_computed_tokens = cached
            remaining = req.num_tokens - req.num_computed_tokens
            n = self._chunk(req, min(remaining, budget))
            if not self.kv.allocate(req, req.num_computed_tokens + n):
                break
            self.waiting.popleft()
            req.status = RequestStatus.RUNNING
            self.running.append(req)
            seqs.append(ScheduledSeq(req, n, False))
            budget -= n

        # decodes first, then prefill chunks
        seqs.sort(key=lambda s: 0 if s.is_decode else 1)
        fin = self.finished_ids
        self.finished_ids = []
        return SchedulerOutput(seqs, self.max_tokens - budget, preempted, fin)

    def _chunk(self, req: Request, n: int) -> int:
        """With GDN state snapshots on, a prefill chunk that would cross the request's snapshot
        boundary ends exactly there, so the state at that boundary can be copied out."""
        B = self.kv.snapshot_boundary(req)
        c = req.num_computed_tokens
        if B > 0 and c < B < c + n:
            return B - c
        return n

    def update(self, out: SchedulerOutput, sampled: dict, accepted: Optional[dict] = None) -> list:
        """Advance request state after a step.  `sampled[req_id]` = list of new token ids
        (1 token, or accepted drafts + bonus with speculation).  Returns finished requests."""
        finished = []
        for s in out.seqs:
            req = s.req
            if req.status.finished:
                continue
            toks = sampled.get(req.request_id)
            if s.is_decode:
                # the fed token + accepted drafts are now in the cache
                n_acc = len(toks) - 1 if toks else 0
                req.num_computed_tokens += 1 + n_acc
            else:
                req.num_computed_tokens += s.num_new_tokens
                self.kv.register_blocks(req)
            if toks:
                for t in toks:
                    req.append_token(t)
                    if req.check_stop(self.max_model_len):
                        break
            if req.status.finished:
                self.running.remove(req)
                self.kv.free(req)
                finished.append(req)
        return finished
