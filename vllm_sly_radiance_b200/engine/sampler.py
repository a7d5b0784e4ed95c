"""Sampling: greedy, temperature / top-k / top-p / min-p, penalties.

Rows are sampled from a top-64 window of the logits (the reference's composite top-k/top-p,
``radiance_topk.py:1-59``: exact whenever the nucleus fits in the window, which holds for the
production settings top_k=20, top_p=0.95).  Greedy-only batches use the argmax kernel."""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch

from ..ops import kernels as K

WINDOW = 64


@dataclass
class SamplingTensors:
    temperature: torch.Tensor   # [B] f32
    top_k: torch.Tensor         # [B] i32
    top_p: torch.Tensor         # [B] f32
    min_p: torch.Tensor         # [B] f32
    seeds: torch.Tensor         # [B] i64
    all_greedy: bool
    any_min_p: bool

    @staticmethod
    def from_requests(reqs, device, pin: bool = False) -> "SamplingTensors":
        B = len(reqs)
        t = torch.tensor([r.params.temperature for r in reqs], dtype=torch.float32)
        k = torch.tensor([r.params.top_k for r in reqs], dtype=torch.int32)
        p = torch.tensor([r.params.top_p for r in reqs], dtype=torch.float32)
        mp = torch.tensor([r.params.min_p for r in reqs], dtype=torch.float32)
        # per-row Philox stream: request seed folded with the request's own token position, so a
        # seeded request reproduces regardless of what else shares its batch
        sd = torch.tensor([row_seed(r) for r in reqs], dtype=torch.int64)
        greedy = all(r.params.greedy for r in reqs)
        return SamplingTensors(t.to(device), k.to(device), p.to(device), mp.to(device),
                               sd.to(device), greedy, bool((mp > 0).any()))


def row_seed(req, offset: int = 0) -> int:
    return (req.seed * 1000003 + len(req.output_token_ids) + offset) & 0x7FFFFFFFFFFF


def apply_penalties(logits: torch.Tensor, reqs) -> torch.Tensor:
    """Presence / frequency / repetition penalties over each request's generated tokens."""
    if not any(r.params.presence_penalty or r.params.frequency_penalty or
               r.params.repetition_penalty != 1.0 for r in reqs):
        return logits
    logits = logits.float().clone()
    for i, r in enumerate(reqs):
        p = r.params
        if not r.output_token_ids:
            continue
        ids = torch.tensor(r.output_token_ids, device=logits.device, dtype=torch.long)
        cnt = torch.bincount(ids, minlength=logits.shape[1]).to(logits.dtype)
        if p.repetition_penalty != 1.0:
            seen = torch.zeros_like(cnt, dtype=torch.bool)
            seen[torch.tensor(r.all_token_ids, device=logits.device, dtype=torch.long)] = True
            row = logits[i]
            row = torch.where(seen & (row > 0), row / p.repetition_penalty, row)
            row = torch.where(seen & (row <= 0), row * p.repetition_penalty, row)
            logits[i] = row
        logits[i] -= p.frequency_penalty * cnt + p.presence_penalty * (cnt > 0).to(logits.dtype)
    return logits


def sample(logits: torch.Tensor, st: SamplingTensors, step: int, want_probs: bool = False):
    """-> (token ids [B] int64, window probs [B, WINDOW] or None, window ids or None)."""
    if st.all_greedy and not want_probs:
        return K.argmax(logits), None, None
    V = logits.shape[1]
    w = min(WINDOW, V)
    vals, ids = torch.topk(logits.float(), w, dim=-1)
    toks, probs = K.sample_from_topk(vals, ids, st.temperature, st.top_k, st.top_p,
                                     st.min_p if st.any_min_p else None, st.seeds, step,
                                     want_probs=want_probs)
    return toks, probs, ids
