"""Acceptance rules: the stock rule reproduces the target distribution exactly; Cactus with
delta 0 is the stock rule; Cactus / NSD only accept more; greedy and forced schedules."""
import torch

from vllm_sly_radiance_b200.spec_decode.rejection import (AcceptRule, ForcedAcceptance,
                                                          rejection_sample)


def _setup(B, p, q):
    V = len(p)
    ids = torch.arange(V).expand(B, V)
    t_ids = torch.stack([ids, ids], 1)                        # [B, 2, V]
    t_pr = torch.tensor(p).expand(B, 2, V).clone()
    d_ids = ids.unsqueeze(1)                                  # [B, 1, V]
    d_pr = torch.tensor(q).expand(B, 1, V).clone()
    g = torch.Generator().manual_seed(0)
    draft = torch.multinomial(torch.tensor(q).expand(B, V), 1, generator=g)
    return t_ids, t_pr, d_ids, d_pr, draft


def test_stock_rule_preserves_target_distribution():
    B = 200000
    p = [0.5, 0.3, 0.15, 0.05]
    q = [0.1, 0.2, 0.3, 0.4]
    t_ids, t_pr, d_ids, d_pr, draft = _setup(B, p, q)
    out, n = rejection_sample(draft, t_ids, t_pr, d_ids, d_pr, torch.zeros(B, dtype=torch.bool),
                              AcceptRule("leviathan"), torch.zeros(B, dtype=torch.long),
                              gen=torch.Generator().manual_seed(1))
    freq = torch.bincount(out[:, 0], minlength=4).float() / B
    assert torch.allclose(freq, torch.tensor(p), atol=0.006), freq
    # acceptance rate = sum_x min(p, q)
    assert abs(float(n.float().mean()) - sum(min(a, b) for a, b in zip(p, q))) < 0.006


def test_cactus_delta0_is_stock_and_cactus_accepts_more():
    B = 50000
    p = [0.5, 0.3, 0.15, 0.05]
    q = [0.1, 0.2, 0.3, 0.4]
    t_ids, t_pr, d_ids, d_pr, draft = _setup(B, p, q)
    args = (draft, t_ids, t_pr, d_ids, d_pr, torch.zeros(B, dtype=torch.bool))
    sl = torch.zeros(B, dtype=torch.long)
    o1, n1 = rejection_sample(*args, AcceptRule("leviathan"), sl, gen=torch.Generator().manual_seed(2))
    o2, n2 = rejection_sample(*args, AcceptRule("cactus", delta=0.0), sl, gen=torch.Generator().manual_seed(2))
    assert torch.equal(o1, o2) and torch.equal(n1, n2)
    o3, n3 = rejection_sample(*args, AcceptRule("cactus", delta=0.5), sl, gen=torch.Generator().manual_seed(2))
    assert n3.float().mean() > n1.float().mean()
    # the fade: at seq len >= fade_end cactus is the stock rule again
    o4, n4 = rejection_sample(*args, AcceptRule("cactus", delta=0.5), torch.full((B,), 20000),
                              gen=torch.Generator().manual_seed(2))
    assert torch.equal(n4, n1)
    o5, n5 = rejection_sample(*args, AcceptRule("nsd", theta=0.5), sl, gen=torch.Generator().manual_seed(2))
    assert n5.float().mean() >= n1.float().mean()


def test_greedy_and_forced():
    B, V, k = 3, 10, 3
    logits = torch.randn(B, k + 1, V)
    pr = torch.softmax(logits, -1)
    vals, ids = torch.sort(pr, -1, descending=True)
    top = ids[..., 0]
    draft = top[:, :k].clone()
    draft[1, 1] = (draft[1, 1] + 1) % V          # request 1 diverges at position 1
    out, n = rejection_sample(draft, ids, vals, None, None, torch.ones(B, dtype=torch.bool),
                              AcceptRule(), torch.zeros(B, dtype=torch.long))
    assert n.tolist() == [3, 1, 3]
    assert out[0].tolist() == top[0].tolist()
    assert out[1, :2].tolist() == [int(top[1, 0]), int(top[1, 1])] and out[1, 2] == -1
    f = ForcedAcceptance(k=3, pattern=[2])
    out, n = rejection_sample(draft, ids, vals, None, None, torch.ones(B, dtype=torch.bool),
                              AcceptRule(), torch.zeros(B, dtype=torch.long), forced=f.next(B, "cpu"))
    assert n.tolist() == [2, 2, 2]
    assert ForcedAcceptance().pattern and abs(sum(ForcedAcceptance().pattern) / 8 - 5.5) < 1e-9


def test_rule_validation():
    import pytest
    with pytest.raises(ValueError):
        AcceptRule("cactus", cap_r=1.5)
    with pytest.raises(ValueError):
        AcceptRule("nsd", theta=1.0)
