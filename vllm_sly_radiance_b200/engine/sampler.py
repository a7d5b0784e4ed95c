"""Sampling: greedy, temperature / top-k / top-p / min-p, penalties.

Routing follows the reference's composite top-k/top-p sampler (``radiance_topk.py:1-59``): a batch
whose every sampled row has 0 < top_k <= 64 (known on the host) draws from a top-64 window of the
logits, found and sampled in one CUDA launch -- exact, because each row's top-k set lies inside the
window.  A batch with any sampled row whose top_k is disabled (<= 0) or above 64 takes the
full-vocabulary path: the rows are sorted and drawn over the whole vocabulary, so top-p / min-p cut
the true distribution.  Greedy-only batches use the argmax kernel."""
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
    full_vocab: bool = False    # some sampled row has top_k disabled or above the window

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
                               sd.to(device), greedy, bool((mp > 0).any()),
                               needs_full_vocab(reqs))


def needs_full_vocab(reqs) -> bool:
    """True when a sampled row's top-k set does not fit the top-64 window."""
    return any(not r.params.greedy and (r.params.top_k <= 0 or r.params.top_k > WINDOW)
               for r in reqs)


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
    min_p = st.min_p if st.any_min_p else None
    if st.full_vocab and not want_probs:
        # exact over the whole vocabulary: sorted rows, drawn by the same per-row kernel
        vals, ids = torch.sort(logits.float(), dim=-1, descending=True)
        toks, _ = K.sample_from_topk(vals, ids, st.temperature, st.top_k, st.top_p, min_p,
                                     st.seeds, step)
        return toks, None, None
    # window path (speculative verify always reads the window: its rejection test works on the
    # top-64 candidates of each position)
    toks, probs, ids = K.topk_sample(logits, st.temperature, st.top_k, st.top_p, min_p, st.seeds,
                                     step, want_probs=want_probs)
    return toks, probs, ids
