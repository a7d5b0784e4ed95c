"""Speculative-decoding acceptance (rejection sampling) with the reference's acceptance rules.

Reference: vLLM's rejection sampler plus ``sly/patch_cactus.py`` / ``sly/patch_nsd.py``
(README.md:452-578).  Notation: for draft position i the target distribution is p_i (after
temperature / top-k / top-p), the draft distribution is q_i, the drafted token is d_i.

  stock (Leviathan)  accept d_i with probability min(1, p_i(d_i) / q_i(d_i))
  Cactus (delta)     raise the target probability to
                       h = clamp(p + sqrt(2 * delta_eff * p * (1 - p)), 0, 1),
                       capped at 1 - r * (1 - p) when cap_r > 0; accept with min(1, h / q).
                     delta_eff fades linearly from delta at `fade_start` sequence tokens to 0 at
                     `fade_end` (fade_end <= fade_start: hard cut at fade_start; 0: no fade).
                     Escape mixture: with probability eps the stock test runs instead (same u).
  NSD (theta)        accept when the stock test passes OR the target mass of tokens with a
                     strictly higher target probability than d_i is <= theta.
  on rejection       emit a sample of norm(max(0, p_i - q_i)); stop.
  all accepted       emit a bonus sample of p_k.
  greedy rows        accept iff d_i == argmax p_i; emit argmax p_i at the first mismatch.

Distributions are passed as windows: (ids [.., W], probs [.., W]) — the sampler's top-64 target
window and the drafter's candidate set — so nothing of vocabulary size is materialised.
"""
from __future__ import annotations

import math
import os
from dataclasses import dataclass
from typing import Optional

import torch


@dataclass
class AcceptRule:
    kind: str = "leviathan"           # leviathan | cactus | nsd
    delta: float = 0.5
    fade_start: int = 4096
    fade_end: int = 16384
    cap_r: float = 0.5
    escape: float = 0.0
    theta: float = 0.95

    def __post_init__(self):
        if self.kind not in ("leviathan", "cactus", "nsd"):
            raise ValueError(self.kind)
        if not (0.0 <= self.cap_r <= 1.0):
            raise ValueError("cactus cap_r must be in [0, 1]")
        if not (0.0 <= self.escape <= 1.0):
            raise ValueError("cactus escape must be in [0, 1]")
        if self.kind == "nsd" and not (0.0 <= self.theta < 1.0):
            raise ValueError("nsd theta must be in [0, 1)")

    @staticmethod
    def from_env(kind: str) -> "AcceptRule":
        import os
        g = os.environ.get
        return AcceptRule(kind=kind, delta=float(g("RADIANCE_CACTUS_DELTA", 0.5)),
                          fade_start=int(g("RADIANCE_CACTUS_FADE_START", 4096)),
                          fade_end=int(g("RADIANCE_CACTUS_FADE_END", 16384)),
                          cap_r=float(g("RADIANCE_CACTUS_CAP_R", 0.5)),
                          escape=float(g("RADIANCE_CACTUS_ESCAPE", 0.0)),
                          theta=float(g("RADIANCE_NSD_THETA", 0.95)))

    def delta_eff(self, seq_len: torch.Tensor) -> torch.Tensor:
        d = torch.full_like(seq_len, self.delta, dtype=torch.float32)
        if self.fade_end == 0:
            return d
        if self.fade_end <= self.fade_start:
            return torch.where(seq_len >= self.fade_start, torch.zeros_like(d), d)
        f = ((self.fade_end - seq_len.float()) / (self.fade_end - self.fade_start)).clamp(0, 1)
        return d * f


def _lookup(ids: torch.Tensor, probs: torch.Tensor, tok: torch.Tensor) -> torch.Tensor:
    """probs[..., j] where ids[..., j] == tok (0 when absent)."""
    m = ids == tok.unsqueeze(-1)
    return (probs * m).sum(-1)


def _sample_window(ids, probs, u):
    """Inverse-CDF draw from an (unnormalised) window with uniforms u [B]."""
    p = probs.clamp(min=0)
    z = p.sum(-1, keepdim=True).clamp(min=1e-30)
    c = torch.cumsum(p / z, -1)
    j = torch.searchsorted(c, u.unsqueeze(-1).clamp(max=1 - 1e-7)).clamp(max=ids.shape[-1] - 1)
    return ids.gather(-1, j).squeeze(-1)


_KIND = {"leviathan": 0, "cactus": 1, "nsd": 2}
_USE_CUDA = os.environ.get("RADIANCE_CUDA_REJECTION", "1") != "0"


def rejection_sample(draft: torch.Tensor, t_ids: torch.Tensor, t_probs: torch.Tensor,
                     d_ids: Optional[torch.Tensor], d_probs: Optional[torch.Tensor],
                     greedy: torch.Tensor, rule: AcceptRule, seq_lens: torch.Tensor,
                     gen: Optional[torch.Generator] = None,
                     forced: Optional[torch.Tensor] = None,
                     seeds: Optional[torch.Tensor] = None):
    """See the module docstring.  CUDA tensors run the one-warp-per-request kernel
    (``csrc/spec_decode.cu``) with a Philox stream per row keyed by `seeds` [B] (drawn from `gen`
    or torch's generator when absent); CPU tensors run the reference torch version below."""
    if draft.is_cuda and _USE_CUDA and t_ids.shape[-1] <= 64 and \
            (d_ids is None or d_ids.shape[-1] <= 64):
        from ..ops._ext import ext
        B, k = draft.shape
        dev = draft.device
        if seeds is None:
            seeds = torch.randint(0, 2 ** 62, (B,), generator=gen,
                                  device="cpu" if gen is None or gen.device.type == "cpu"
                                  else dev).to(dev)
        out = torch.empty(B, k + 1, dtype=torch.long, device=dev)
        n_acc = torch.empty(B, dtype=torch.long, device=dev)
        e = torch.empty(0, device=dev)
        ext().rejection_sample(draft.long().contiguous(), t_ids.long().contiguous(),
                               t_probs.float().contiguous(),
                               d_ids.long().contiguous() if d_ids is not None else e.long(),
                               d_probs.float().contiguous() if d_probs is not None else e,
                               greedy.bool().contiguous(), seq_lens.to(dev).long().contiguous(),
                               forced.to(dev).long().contiguous() if forced is not None else e.long(),
                               seeds.to(dev).long().contiguous(), _KIND[rule.kind], rule.delta,
                               rule.fade_start, rule.fade_end, rule.cap_r, rule.escape,
                               rule.theta, out, n_acc)
        return out, n_acc
    return _rejection_sample_torch(draft, t_ids, t_probs, d_ids, d_probs, greedy, rule, seq_lens,
                                   gen, forced)


def _rejection_sample_torch(draft: torch.Tensor, t_ids: torch.Tensor, t_probs: torch.Tensor,
                            d_ids: Optional[torch.Tensor], d_probs: Optional[torch.Tensor],
                            greedy: torch.Tensor, rule: AcceptRule, seq_lens: torch.Tensor,
                            gen: Optional[torch.Generator] = None,
                            forced: Optional[torch.Tensor] = None):
    """Per request b with k drafts:
      draft [B,k] drafted ids; t_ids/t_probs [B,k+1,W] target windows (probs sum to 1, sorted
      descending); d_ids/d_probs [B,k,Kd] draft windows (None -> point mass on the draft token,
      e.g. greedy / prompt-lookup drafters); greedy [B] bool; seq_lens [B] tokens before the block.
      forced [B] int (benchmark schedule): accept exactly that many drafts.
    Returns (out_tokens [B, k+1] (-1 padded), num_accepted [B])."""
    B, k = draft.shape
    dev = draft.device
    out = torch.full((B, k + 1), -1, dtype=torch.long, device=dev)
    alive = torch.ones(B, dtype=torch.bool, device=dev)
    n_acc = torch.zeros(B, dtype=torch.long, device=dev)
    rnd = lambda *s: torch.rand(*s, generator=gen, device="cpu" if gen is not None and
                                gen.device.type == "cpu" else dev).to(dev)
    u_acc = rnd(B, k)
    u_res = rnd(B, k + 1)
    u_esc = rnd(B, k)
    dlt = rule.delta_eff(seq_lens.to(dev)) if rule.kind == "cactus" else None
    for i in range(k + 1):
        if not bool(alive.any()):
            break
        p_ids, p_pr = t_ids[:, i], t_probs[:, i]
        top = p_ids[:, 0]
        if i == k:                                   # bonus position
            tok = torch.where(greedy, top, _sample_window(p_ids, p_pr, u_res[:, i]))
            out[:, i] = torch.where(alive, tok, out[:, i])
            break
        d = draft[:, i]
        if forced is not None:
            acc = i < forced
        else:
            pt = _lookup(p_ids, p_pr, d)
            qd = _lookup(d_ids[:, i], d_probs[:, i], d) if d_ids is not None else torch.ones_like(pt)
            qd = qd.clamp(min=1e-20)
            stock = u_acc[:, i] < torch.clamp(pt / qd, max=1.0)
            if rule.kind == "cactus":
                h = (pt + torch.sqrt((2 * dlt * pt * (1 - pt)).clamp(min=0))).clamp(0, 1)
                if rule.cap_r > 0:
                    h = torch.minimum(h, 1 - rule.cap_r * (1 - pt))
                cac = u_acc[:, i] < torch.clamp(h / qd, max=1.0)
                acc = torch.where(u_esc[:, i] < rule.escape, stock, cac) if rule.escape > 0 else cac
            elif rule.kind == "nsd":
                higher = (p_pr * (p_pr > pt.unsqueeze(-1))).sum(-1)
                acc = stock | ((pt > 0) & (higher <= rule.theta))
            else:
                acc = stock
            acc = torch.where(greedy, d == top, acc)
        acc = acc & alive
        out[:, i] = torch.where(acc, d, out[:, i])
        n_acc = n_acc + acc.long()
        rej = alive & ~acc
        if bool(rej.any()):
            if forced is not None:
                res_tok = top
            else:
                qx = torch.zeros_like(p_pr)
                if d_ids is not None:
                    eq = p_ids.unsqueeze(-1) == d_ids[:, i].unsqueeze(-2)      # [B,W,Kd]
                    qx = (eq * d_probs[:, i].unsqueeze(-2)).sum(-1)
                else:
                    qx = (p_ids == d.unsqueeze(-1)).float()
                resid = (p_pr - qx).clamp(min=0)
                empty = resid.sum(-1) <= 0
                resid = torch.where(empty.unsqueeze(-1), p_pr, resid)
                res_tok = _sample_window(p_ids, resid, u_res[:, i])
            res_tok = torch.where(greedy, top, res_tok)
            out[:, i] = torch.where(rej, res_tok, out[:, i])
        alive = alive & acc
    return out, n_acc


class ForcedAcceptance:
    """Benchmark acceptance-length schedule (random weights accept ~nothing): a fixed cycle of
    accepted-draft counts in [0, k] with the configured mean (default mean 5.5 of k = 7)."""

    def __init__(self, k: int = 7, pattern: Optional[list] = None):
        self.k = k
        self.pattern = pattern or [7, 4, 6, 5, 7, 3, 6, 6]    # mean 5.5
        self.i = 0

    def next(self, B: int, device) -> torch.Tensor:
        vals = [min(self.k, self.pattern[(self.i + b) % len(self.pattern)]) for b in range(B)]
        self.i += 1
        return torch.tensor(vals, dtype=torch.long, device=device)
