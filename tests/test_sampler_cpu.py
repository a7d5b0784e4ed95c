"""Sampler routing: rows whose top-k set fits the top-64 window draw from the window; rows with
top_k disabled (or above 64) draw over the whole vocabulary, so the empirical distribution matches
softmax over the full row (reference behaviour: radiance_topk.py:1-59 takes the window only when
every row's top_k is known to fit)."""
import torch

from vllm_sly_radiance_b200.engine.request import Request, SamplingParams
from vllm_sly_radiance_b200.engine.sampler import SamplingTensors, needs_full_vocab, sample


def _reqs(n, **kw):
    return [Request([1, 2, 3], SamplingParams(seed=i, **kw)) for i in range(n)]


def test_routing_flags():
    assert not needs_full_vocab(_reqs(2, temperature=0.7, top_k=20))
    assert needs_full_vocab(_reqs(2, temperature=0.7, top_k=0))
    assert needs_full_vocab(_reqs(2, temperature=0.7, top_k=65))
    assert not needs_full_vocab(_reqs(2, temperature=0.0, top_k=0))      # greedy rows


def test_full_vocab_distribution_matches_softmax():
    """top_k = 0, top_p = 1: tokens far outside the top 64 are drawn at their softmax rate."""
    V, N = 160, 6000
    g = torch.Generator().manual_seed(0)
    row = torch.randn(V, generator=g) * 0.5           # flat: most mass outside the top 64
    reqs = _reqs(N, temperature=1.0, top_k=0, top_p=1.0)
    st = SamplingTensors.from_requests(reqs, "cpu")
    assert st.full_vocab
    toks, _, _ = sample(row[None].expand(N, V).contiguous(), st, 0)
    emp = torch.bincount(toks, minlength=V).double() / N
    want = torch.softmax(row.double(), 0)
    tv = 0.5 * float((emp - want).abs().sum())
    assert tv < 0.08, tv
    order = torch.argsort(row, descending=True)
    outside = float(emp[order[64:]].sum())
    assert abs(outside - float(want[order[64:]].sum())) < 0.03, outside


def test_window_path_respects_top_k():
    V, N = 160, 400
    row = torch.linspace(1.0, 0.0, V)
    st = SamplingTensors.from_requests(_reqs(N, temperature=1.0, top_k=5, top_p=1.0), "cpu")
    assert not st.full_vocab
    toks, _, _ = sample(row[None].expand(N, V).contiguous(), st, 0)
    assert int(toks.max()) <= 4 and len(set(toks.tolist())) == 5
