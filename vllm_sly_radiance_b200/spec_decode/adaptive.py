"""Adaptive verify width: per-request draft length chosen every step.

Behaviour of the reference (``sly/radiance_adaptive_width.py:1-45,106-295``): each request may be
verified with a width k_i from a small set ({1, 3, 5, 7}); the widths maximise the expected
tokens emitted per unit of step time,

    maximise  sum_i E_i(k_i) / T(M),    M = sum_i (1 + k_i) verify rows (rounded up to 8),

with E_i(k) = 1 + a_i + ... + a_i^k the expected tokens of a request whose drafts are accepted
independently with probability a_i (accepted prefix plus the bonus / correction token), and a
linear step-cost model T(M) = t0 + t1 * M.  a_i is a censored-geometric estimate from the
request's own history: every verify contributes its accepted count (successes) and one failure
if it stopped before the end of its drafts.

B200 specifics: the cost model is not the reference's R9700 constants; it starts from
(t0, t1) given by the config / environment and is refitted online by least squares from the
measured verify step times, once two distinct M have been seen.
"""
from __future__ import annotations

import os
from dataclasses import dataclass, field


@dataclass
class _ReqStats:
    successes: float = 0.0
    failures: float = 0.0


@dataclass
class AdaptiveWidth:
    widths: tuple = (1, 3, 5, 7)
    t0_ms: float = 4.6
    t1_ms: float = 0.03
    prior_alpha: float = 0.5
    prior_weight: float = 4.0
    row_multiple: int = 8
    max_samples: int = 256
    stats: dict = field(default_factory=dict)
    samples: list = field(default_factory=list)

    @staticmethod
    def from_env(k_max: int) -> "AdaptiveWidth":
        ws = tuple(w for w in (1, 3, 5, 7) if w <= k_max) or (k_max,)
        return AdaptiveWidth(widths=ws,
                             t0_ms=float(os.environ.get("RADIANCE_AW_T0_MS", "4.6")),
                             t1_ms=float(os.environ.get("RADIANCE_AW_T1_MS", "0.03")))

    # ---------------------------------------------------------------- acceptance estimates
    def alpha(self, rid) -> float:
        st = self.stats.get(rid)
        s = st.successes if st else 0.0
        f = st.failures if st else 0.0
        m = self.prior_weight
        return (s + self.prior_alpha * m) / (s + f + m)

    def observe(self, rid, k: int, accepted: int):
        st = self.stats.setdefault(rid, _ReqStats())
        st.successes += accepted
        if accepted < k:
            st.failures += 1.0

    def forget(self, rid):
        self.stats.pop(rid, None)

    # ---------------------------------------------------------------- cost model
    def cost(self, rows: int) -> float:
        m = self.row_multiple
        rows = (rows + m - 1) // m * m
        return self.t0_ms + self.t1_ms * rows

    def record_step(self, rows: int, ms: float):
        """A measured verify step (rows, wall ms); refits (t0, t1) by least squares."""
        self.samples.append((rows, ms))
        if len(self.samples) > self.max_samples:
            self.samples = self.samples[-self.max_samples:]
        xs = [r for r, _ in self.samples]
        if len(set(xs)) < 2:
            return
        n = len(xs)
        mx = sum(xs) / n
        my = sum(t for _, t in self.samples) / n
        sxx = sum((x - mx) ** 2 for x in xs)
        sxy = sum((x - mx) * (t - my) for x, t in self.samples)
        t1 = max(sxy / sxx, 1e-6)
        t0 = max(my - t1 * mx, 1e-3)
        self.t0_ms, self.t1_ms = t0, t1

    # ---------------------------------------------------------------- width choice
    @staticmethod
    def expected_tokens(a: float, k: int) -> float:
        if a >= 1.0:
            return k + 1.0
        return (1.0 - a ** (k + 1)) / (1.0 - a)

    def choose(self, rids: list, k_avail: list) -> list:
        """Width per request (<= its available drafts); coordinate ascent on the objective."""
        n = len(rids)
        if n == 0:
            return []
        if len(self.stats) > 4 * n + 1024:       # drop requests that left the batch long ago
            keep = set(rids)
            self.stats = {r: v for r, v in self.stats.items() if r in keep}
        al = [self.alpha(r) for r in rids]
        opts = [[w for w in self.widths if w <= ka] or [min(ka, self.widths[0])] for ka in k_avail]
        idx = [0] * n
        cur = [opts[i][0] for i in range(n)]

        def objective(ws):
            tok = sum(self.expected_tokens(al[i], ws[i]) for i in range(n))
            return tok / self.cost(sum(1 + w for w in ws))

        best = objective(cur)
        while True:
            cand = None
            for i in range(n):
                if idx[i] + 1 < len(opts[i]):
                    trial = list(cur)
                    trial[i] = opts[i][idx[i] + 1]
                    v = objective(trial)
                    if v > best + 1e-12 and (cand is None or v > cand[0]):
                        cand = (v, i)
            if cand is None:
                return cur
            best, i = cand
            idx[i] += 1
            cur[i] = opts[i][idx[i]]
