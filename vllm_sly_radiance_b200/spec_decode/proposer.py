"""Speculative decoding: draft proposers and the verify / accept / commit step.

Step with speculation (reference: vLLM V2 runner + DFlash2 speculator, dflash2/speculator.py):
  1. every decoding request feeds [last token, d_1..d_k] (its drafts from the previous step),
  2. one target forward over all rows; the GDN layers run the block without touching their state
     and keep their inputs (the reference writes one state snapshot per candidate instead, which
     costs k state writes per layer per step),
  3. target windows at every position -> rejection sampling (stock / Cactus / NSD, greedy),
  4. commit: the accepted prefix (1 + accepted) is applied to the GDN conv/SSM state from the
     saved inputs; attention KV of rejected positions is simply overwritten later,
  5. the proposer drafts the next k tokens for every running request.

Proposers:
  * ``lookup``  prompt-lookup: the tokens that followed the longest earlier occurrence of the
                request's suffix (``sly/radiance_lookup_draft.py``: suffix up to 24 tokens over the
                whole history, point-mass drafts, lossless).
  * ``dflash2`` the DFlash2 block drafter (``models/dflash2.py``).
  * ``mtp``     the target's multi-token-prediction head chained k times (``models/mtp.py``).
Adaptive verify width (``spec_decode/adaptive.py``, opt-in ``adaptive_width``) truncates each
request's drafts to the width that maximises expected tokens per unit of step time.

  * ``forced``  benchmark mode: drafts from the lookup proposer (or repeats), acceptance forced
                by a fixed schedule (mean 5.5 of 7) so verify throughput is measurable with random
                weights.
"""
from __future__ import annotations

import time
from typing import Optional

import numpy as np
import torch

from ..engine.model_runner import StepResult
from ..engine.sampler import SamplingTensors, apply_penalties, row_seed, sample
from ..engine.scheduler import SchedulerOutput
from .adaptive import AdaptiveWidth
from .rejection import AcceptRule, ForcedAcceptance, rejection_sample


class LookupProposer:
    """n-gram prompt lookup over each request's full token history.  On CUDA the scan runs in
    ``lookup_kernel`` (csrc/spec_decode.cu) over device-resident histories, one row per GDN state
    slot; only the tokens added since the previous step are uploaded."""

    def __init__(self, k: int, max_ngram: int = 24, min_ngram: int = 2, device=None,
                 num_rows: int = 0, max_len: int = 0):
        self.k = k
        self.max_ngram = max_ngram
        self.min_ngram = min_ngram
        self.dev = None
        if device is not None and torch.device(device).type == "cuda" and num_rows and max_len:
            self.dev = torch.device(device)
            self.hist = torch.zeros(num_rows, max_len, dtype=torch.int32, device=self.dev)
            self.row_owner: dict = {}          # row -> (request_id, tokens uploaded)

    def propose_gpu(self, reqs_tokens: list) -> list[list[int]]:
        """reqs_tokens: [(request, full token history)]; the request's state slot picks its row."""
        from ..ops._ext import ext
        rows, lens = [], []
        for req, toks in reqs_tokens:
            row = req.state_slot
            owner = self.row_owner.get(row)
            start = owner[1] if owner is not None and owner[0] == req.request_id else 0
            n = min(len(toks), self.hist.shape[1])
            if n > start:
                self.hist[row, start:n].copy_(torch.tensor(toks[start:n], dtype=torch.int32),
                                              non_blocking=False)
            self.row_owner[row] = (req.request_id, n)
            rows.append(row)
            lens.append(n)
        B = len(rows)
        rows_t = torch.tensor(rows, dtype=torch.int32).to(self.dev)
        lens_t = torch.tensor(lens, dtype=torch.int32).to(self.dev)
        out = torch.empty(B, self.k, dtype=torch.int32, device=self.dev)
        n_out = torch.empty(B, dtype=torch.int32, device=self.dev)
        ext().lookup_draft(self.hist, rows_t, lens_t, self.k, self.max_ngram, self.min_ngram,
                           out, n_out)
        o, n = out.cpu().tolist(), n_out.cpu().tolist()
        return [o[b][:n[b]] for b in range(B)]

    def propose_one(self, toks: list[int]) -> list[int]:
        n_tok = len(toks)
        a = np.asarray(toks, dtype=np.int64)
        for n in range(min(self.max_ngram, n_tok - 1), self.min_ngram - 1, -1):
            suf = a[n_tok - n:]
            # most recent earlier occurrence of the suffix
            win = np.lib.stride_tricks.sliding_window_view(a[:n_tok - 1], n)
            hits = np.nonzero((win == suf).all(1))[0]
            hits = hits[hits + n < n_tok]
            if len(hits):
                st = int(hits[-1]) + n
                d = toks[st:st + self.k]
                if d:
                    return d
        return []

    def propose(self, reqs) -> list[list[int]]:
        return [self.propose_one(r.all_token_ids) for r in reqs]


class SpecRunner:
    def __init__(self, engine, method: str, k: int, rule: AcceptRule,
                 forced: Optional[ForcedAcceptance] = None, drafter=None,
                 adaptive: Optional[AdaptiveWidth] = None):
        self.engine = engine
        self.runner = engine.runner
        self.model = engine.model
        self.k = k
        self.method = method
        self.rule = rule
        self.forced = forced
        self.drafter = drafter
        r = engine.runner
        self.lookup = LookupProposer(k, device=r.device, num_rows=engine.kv.slots.num_slots,
                                     max_len=r.max_blocks * r.bs)
        self.gen = None
        self.stats = dict(steps=0, drafts=0, draft_tokens=0, accepted=0)
        self.adaptive = adaptive

    # ------------------------------------------------------------------------------------------
    def execute(self, sched: SchedulerOutput) -> StepResult:
        r = self.runner
        dev = r.device
        verify = [s for s in sched.seqs if s.is_decode and s.draft_tokens]
        if not verify and self.drafter is None:
            res = r.execute(sched)
            self._propose(sched, res.sampled)
            return res
        r.step_count += 1
        t_step = time.perf_counter()
        meta, ids, sample_idx, sample_cnt = r.prepare(sched)
        commit = [0 if (s.is_decode and s.draft_tokens) else s.num_new_tokens for s in sched.seqs]
        meta.commit_len = torch.tensor(commit, dtype=torch.int32).to(dev, non_blocking=True)
        saved: list = []
        aux = [] if self.drafter is not None else None
        hidden = self.model.forward(ids, meta, r.caches, gdn_save=saved,
                                    aux_layers=self.drafter.aux_layers if self.drafter else None,
                                    aux_out=aux)
        if not sample_idx:
            # only intermediate prefill chunks this step (their state was written by the
            # forward itself): nothing to sample, verify or commit
            if self.drafter is not None:
                self.drafter.observe(sched, meta, aux, {}, sample_cnt, hidden=hidden)
            return StepResult({}, num_tokens=meta.num_tokens)
        sidx = torch.tensor(sample_idx, dtype=torch.long).to(dev, non_blocking=True)
        logits = self.model.logits(hidden[sidx])
        rows = []
        for s, c in zip(sched.seqs, sample_cnt):
            rows.extend([s.req] * c)
        st = SamplingTensors.from_requests(rows, dev)
        toks, probs, wids = sample(apply_penalties(logits, rows), st, 0, want_probs=True)
        if probs is None:       # greedy-only batch: build one-hot windows from the argmax
            vals, wids = torch.topk(logits.float(), 1, dim=-1)
            probs = torch.ones_like(vals)
        toks_h = toks.cpu().tolist()
        sampled = {}
        # group verify rows by draft length
        j = 0
        row_of = {}
        for s, c in zip(sched.seqs, sample_cnt):
            row_of[s.req.request_id] = (j, c)
            j += c
        commit_len = [-1] * len(sched.seqs)
        by_k: dict = {}
        for bi, s in enumerate(sched.seqs):
            if s.is_decode and s.draft_tokens:
                by_k.setdefault(len(s.draft_tokens), []).append((bi, s))
            elif sample_cnt[bi]:
                j0, _ = row_of[s.req.request_id]
                sampled[s.req.request_id] = [toks_h[j0]]
        n_acc_all = []
        for k, group in by_k.items():
            Bk = len(group)
            rsel = torch.tensor([row_of[s.req.request_id][0] + p for _, s in group for p in range(k + 1)],
                                device=dev)
            W = wids.shape[-1]
            t_ids = wids[rsel].view(Bk, k + 1, W)
            t_pr = probs[rsel].view(Bk, k + 1, W)
            draft = torch.tensor([s.draft_tokens for _, s in group], dtype=torch.long, device=dev)
            greedy = torch.tensor([s.req.params.greedy for _, s in group], device=dev)
            seq_lens = torch.tensor([s.req.num_tokens for _, s in group], device=dev)
            d_ids = d_pr = None
            if self.drafter is not None:
                d_ids, d_pr = self.drafter.draft_windows([s.req for _, s in group], k, dev)
            forced = self.forced.next(Bk, dev) if self.forced is not None else None
            seeds = torch.tensor([row_seed(s.req, 7919) for _, s in group], dtype=torch.int64)
            out, n_acc = rejection_sample(draft, t_ids, t_pr, d_ids, d_pr, greedy, self.rule,
                                          seq_lens, forced=forced, seeds=seeds)
            out_h, n_h = out.cpu().tolist(), n_acc.cpu().tolist()
            for (bi, s), o, n in zip(group, out_h, n_h):
                sampled[s.req.request_id] = [t for t in o[:n + 1]]
                commit_len[bi] = 1 + n
                n_acc_all.append(n)
                if self.adaptive is not None:
                    self.adaptive.observe(s.req.request_id, k, n)
        # commit the accepted prefixes to the GDN state
        cl = torch.tensor(commit_len, dtype=torch.int32).to(dev, non_blocking=True)
        meta.commit_len = None
        self.model.commit_gdn(meta, r.caches, saved, cl)
        if self.adaptive is not None and verify:
            # the step already synchronised on the sampled tokens: wall time ~ device time
            self.adaptive.record_step(meta.num_tokens, (time.perf_counter() - t_step) * 1e3)
        self.stats["steps"] += 1
        self.stats["drafts"] += len(verify)
        self.stats["draft_tokens"] += sum(len(s.draft_tokens) for s in verify)
        self.stats["accepted"] += sum(n_acc_all)
        self.engine.metrics.on_spec(len(verify), sum(len(s.draft_tokens) for s in verify),
                                    n_acc_all, self.k)
        if self.drafter is not None:
            self.drafter.observe(sched, meta, aux, sampled, sample_cnt, hidden=hidden)
        self._propose(sched, sampled)
        return StepResult(sampled, num_tokens=meta.num_tokens)

    def _propose(self, sched: SchedulerOutput, sampled: dict):
        """Draft the next block for every request that will be decoding next step."""
        reqs = []
        for s in sched.seqs:
            toks = sampled.get(s.req.request_id)
            if toks:
                reqs.append((s.req, toks))
        if not reqs:
            return
        if self.drafter is not None:
            drafts = self.drafter.propose([r for r, _ in reqs], [t for _, t in reqs])
        else:
            # history as it will be after the scheduler appends the new tokens
            if self.lookup.dev is not None:
                drafts = self.lookup.propose_gpu([(r, r.all_token_ids + t) for r, t in reqs])
            else:
                drafts = [self.lookup.propose_one(r.all_token_ids + t) for r, t in reqs]
            if self.forced is not None:
                drafts = [(d + [t[-1]] * self.k)[:self.k] for d, (r, t) in zip(drafts, reqs)]
        if self.adaptive is not None:
            widths = self.adaptive.choose([r.request_id for r, _ in reqs],
                                          [min(len(d), self.k) for d in drafts])
            drafts = [d[:w] for d, w in zip(drafts, widths)]
        for (req, _), d in zip(reqs, drafts):
            req.draft_token_ids = list(d[:self.k])


def build_proposer(config, engine) -> SpecRunner:
    k = config.num_speculative_tokens
    rule = AcceptRule.from_env(config.acceptance_rule)
    forced = ForcedAcceptance(k) if config.forced_acceptance else None
    drafter = None
    if config.speculative_method == "dflash2":
        from ..models.dflash2 import DFlash2Drafter
        drafter = DFlash2Drafter.for_engine(engine, k)
    elif config.speculative_method == "mtp":
        from ..models.mtp import MTPDrafter
        drafter = MTPDrafter.for_engine(engine, k)
    elif config.speculative_method not in ("lookup", "forced"):
        raise ValueError(f"unknown speculative method {config.speculative_method!r}")
    adaptive = AdaptiveWidth.from_env(k) if config.adaptive_width else None
    return SpecRunner(engine, config.speculative_method, k, rule, forced, drafter, adaptive)
