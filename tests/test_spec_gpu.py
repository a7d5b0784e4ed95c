"""CUDA speculative-decoding kernels (csrc/spec_decode.cu) against the torch reference:
rejection sampling (exact for greedy / forced rows, statistically for sampled rows) and the
prompt-lookup scan (exact)."""
import pytest
import torch

from vllm_sly_radiance_b200.spec_decode import rejection as R
from vllm_sly_radiance_b200.spec_decode.proposer import LookupProposer

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _windows(B, k, W, gen, peak=3.0):
    logits = torch.randn(B, k + 1, 4096, generator=gen) * peak
    p = torch.softmax(logits, -1)
    vals, ids = torch.topk(p, W, -1)
    vals = vals / vals.sum(-1, keepdim=True)
    return ids, vals


def test_rejection_greedy_and_forced_exact():
    g = torch.Generator().manual_seed(0)
    B, k, W = 64, 7, 64
    ids, pr = _windows(B, k, W, g)
    draft = torch.where(torch.rand(B, k, generator=g) < 0.6, ids[:, :k, 0],
                        torch.randint(0, 4096, (B, k), generator=g))
    greedy = torch.ones(B, dtype=torch.bool)
    sl = torch.full((B,), 100)
    rule = R.AcceptRule("leviathan")
    want = R._rejection_sample_torch(draft, ids, pr, None, None, greedy, rule, sl)
    got = R.rejection_sample(draft.to(DEV), ids.to(DEV), pr.to(DEV), None, None, greedy.to(DEV),
                             rule, sl)
    assert torch.equal(got[0].cpu(), want[0]) and torch.equal(got[1].cpu(), want[1])
    forced = torch.randint(0, k + 1, (B,), generator=g)
    want = R._rejection_sample_torch(draft, ids, pr, None, None, ~greedy, rule, sl, forced=forced)
    got = R.rejection_sample(draft.to(DEV), ids.to(DEV), pr.to(DEV), None, None,
                             (~greedy).to(DEV), rule, sl, forced=forced)
    # accepted drafts and the rejection token (argmax under the forced schedule) are exact; a
    # row that accepts all k drafts samples its bonus token (different random streams)
    assert torch.equal(got[1].cpu(), want[1])
    assert torch.equal(got[0].cpu()[:, :k], want[0][:, :k])
    short = forced < k
    assert torch.equal(got[0].cpu()[short, k], want[0][short, k])


@pytest.mark.parametrize("kind", ["leviathan", "cactus", "nsd"])
def test_rejection_acceptance_rates(kind):
    """Point-mass drafts on a fixed token: the kernel's acceptance frequency matches the rule's
    probability, and rejected rows resample from p without the drafted token."""
    g = torch.Generator().manual_seed(1)
    B, k, W = 20000, 1, 64
    ids1, pr1 = _windows(1, k, W, g, peak=1.0)
    ids = ids1.expand(B, -1, -1).contiguous()
    pr = pr1.expand(B, -1, -1).contiguous()
    d_tok = ids1[0, 0, 3]                       # the 4th most likely token
    draft = torch.full((B, k), int(d_tok))
    pt = float(pr1[0, 0, 3])
    rule = R.AcceptRule(kind, delta=0.5, fade_start=4096, fade_end=16384, cap_r=0.5, theta=0.3)
    sl = torch.full((B,), 100)
    if kind == "leviathan":
        want = pt
    elif kind == "cactus":
        h = min(max(pt + (2 * 0.5 * pt * (1 - pt)) ** 0.5, 0.0), 1.0)
        want = min(h, 1 - 0.5 * (1 - pt))
    else:
        higher = float(pr1[0, 0, :3].sum())
        want = 1.0 if higher <= 0.3 else pt
    seeds = torch.arange(B, dtype=torch.int64) * 7 + 1
    out, n = R.rejection_sample(draft.to(DEV), ids.to(DEV), pr.to(DEV), None, None,
                                torch.zeros(B, dtype=torch.bool, device=DEV), rule, sl,
                                seeds=seeds)
    freq = float(n.float().mean())
    assert abs(freq - want) < 0.02, (kind, freq, want)
    rej = out[:, 0][n.cpu() == 0].cpu()
    if rej.numel() > 500:
        assert not bool((rej == d_tok).any())
        # the most likely token is resampled with its renormalised residual probability
        p_top = float(pr1[0, 0, 0]) / (1 - pt)
        assert abs(float((rej == ids1[0, 0, 0]).float().mean()) - p_top) < 0.05


def test_rejection_draft_windows_leviathan():
    """Draft distributions given as windows: acceptance = min(1, p/q) per draft."""
    g = torch.Generator().manual_seed(2)
    B, k, W, Kd = 20000, 1, 64, 8
    ids1, pr1 = _windows(1, k, W, g, peak=1.0)
    d_ids = ids1[:, :k, :Kd].clone()
    d_pr = torch.softmax(torch.randn(1, k, Kd, generator=g), -1)
    j = 2
    d_tok = d_ids[0, 0, j]
    p = float(pr1[0, 0, j])
    q = float(d_pr[0, 0, j])
    rule = R.AcceptRule("leviathan")
    out, n = R.rejection_sample(
        torch.full((B, k), int(d_tok), device=DEV), ids1.expand(B, -1, -1).contiguous().to(DEV),
        pr1.expand(B, -1, -1).contiguous().to(DEV), d_ids.expand(B, -1, -1).contiguous().to(DEV),
        d_pr.expand(B, -1, -1).contiguous().to(DEV), torch.zeros(B, dtype=torch.bool, device=DEV),
        rule, torch.full((B,), 10), seeds=torch.arange(B, dtype=torch.int64))
    assert abs(float(n.float().mean()) - min(1.0, p / q)) < 0.02


def test_lookup_kernel_matches_numpy():
    g = torch.Generator().manual_seed(3)
    lp_cpu = LookupProposer(7)
    lp = LookupProposer(7, device=DEV, num_rows=8, max_len=2048)

    class _Req:
        def __init__(self, rid, slot):
            self.request_id, self.state_slot = rid, slot
    reqs = []
    for b in range(6):
        base = torch.randint(0, 50, (40,), generator=g).tolist()
        hist = base + torch.randint(0, 50, (200,), generator=g).tolist() + base[:int(5 + b * 5)]
        if b == 5:
            hist = torch.randint(1000, 2000, (30,), generator=g).tolist()    # no repeat
        reqs.append((_Req(f"r{b}", b + 1), hist))
    got = lp.propose_gpu(reqs)
    want = [lp_cpu.propose_one(h) for _, h in reqs]
    assert got == want
    # incremental upload: extend histories and propose again
    reqs2 = [(r, h + h[:3]) for r, h in reqs]
    assert lp.propose_gpu(reqs2) == [lp_cpu.propose_one(h) for _, h in reqs2]


def test_dflash_walk_kernel_matches_torch():
    """DFlash2 path walk kernel vs the torch walk: identical drafts and one-hot windows at T = 0;
    at T > 0 the windows equal softmax(score / T) along the sampled path, and Gumbel-max draws
    follow those probabilities."""
    from vllm_sly_radiance_b200.models.dflash2 import selector_walk_torch
    from vllm_sly_radiance_b200.ops import kernels as K
    from vllm_sly_radiance_b200.ops._ext import ext
    from vllm_sly_radiance_b200.ops.kernels import status_word
    g = torch.Generator().manual_seed(11)
    B, k, Kc, r, V = 37, 7, 8, 64, 5000
    unary = (torch.randn(B, k, Kc, generator=g) * 2).to(DEV)
    # distinct candidates per position (slot frequencies below are token frequencies)
    cand = (torch.arange(Kc) * (V // Kc) +
            torch.randint(0, V // Kc, (B, k, Kc), generator=g)).to(DEV)
    anchors = torch.randint(0, V, (B,), generator=g).to(DEV)
    hp = torch.randn(B, k, r, generator=g).to(DEV)
    pred = (torch.randn(V, r, generator=g) * 0.3).to(torch.bfloat16).to(DEV)
    succ = (torch.randn(V, r, generator=g) * 0.3).to(torch.bfloat16).to(DEV)
    st = status_word(torch.device(DEV))

    def run(temps, seeds):
        n = temps.numel()
        d = torch.empty(n, k, dtype=torch.int64, device=DEV)
        wp = torch.empty(n, k, Kc, dtype=torch.float32, device=DEV)
        ext().dflash_walk(unary[:n].contiguous(), cand[:n].contiguous(), anchors[:n].contiguous(),
                          hp[:n].contiguous(), pred, succ, temps, seeds, d, wp, st)
        return d, wp
    t0 = torch.zeros(B, device=DEV)
    d, wp = run(t0, torch.arange(B, dtype=torch.int64, device=DEV))
    dt, wt = selector_walk_torch(unary, cand, anchors, hp, pred, succ, t0)
    assert torch.equal(d, dt) and torch.equal(wp, wt)
    # T > 0: windows along the kernel's own path equal the torch softmax on that path
    t1 = torch.full((B,), 0.7, device=DEV)
    d, wp = run(t1, torch.arange(B, dtype=torch.int64, device=DEV) + 5)
    prev = anchors.clone()
    for i in range(k):
        sc = unary[:, i] + ((pred[prev].float() * hp[:, i]).unsqueeze(1) *
                            succ[cand[:, i]].float()).sum(-1)
        want = torch.softmax(sc / 0.7, -1)
        assert torch.allclose(wp[:, i], want, atol=1e-4), i
        assert bool((cand[:, i] == d[:, i:i + 1]).any(-1).all())
        prev = d[:, i]
    # Gumbel-max frequencies at position 0 of one request repeated under many seeds
    n = 20000
    one = lambda x: x[:1].expand(n, *x.shape[1:]).contiguous()
    dd = torch.empty(n, k, dtype=torch.int64, device=DEV)
    ww = torch.empty(n, k, Kc, dtype=torch.float32, device=DEV)
    ext().dflash_walk(one(unary), one(cand), one(anchors), one(hp), pred, succ,
                      torch.full((n,), 0.7, device=DEV),
                      torch.arange(n, dtype=torch.int64, device=DEV) * 3 + 1, dd, ww, st)
    K.check_status(torch.device(DEV))
    freq = torch.stack([(dd[:, 0] == cand[0, 0, c]).float().mean() for c in range(Kc)])
    assert float((freq - ww[0, 0]).abs().max()) < 0.02, (freq, ww[0, 0])


def test_mtp_drafter_engine_gpu():
    """The MTP drafter through the CUDA engine.  With bf16 weights and a bf16 KV cache the batched
    verify forward rounds exactly like the one-row decode forward, so greedy speculative output
    equals plain decoding token for token.  (With e4m3 activations or an fp8 KV cache the verify
    and decode kernels round differently and a near-tie of this random model may flip; that
    case only has to run.)"""
    from vllm_sly_radiance_b200.config import EngineConfig
    from vllm_sly_radiance_b200.engine.llm_engine import LLMEngine
    from vllm_sly_radiance_b200.engine.request import SamplingParams

    def eng(spec, quant="bf16", kv="bf16"):
        return LLMEngine(EngineConfig(model="tiny_hybrid", device="cuda", max_model_len=1024,
                                      max_num_seqs=4, max_num_batched_tokens=64,
                                      num_kv_blocks=64, speculative_method=spec,
                                      num_speculative_tokens=4, enable_cuda_graphs=False,
                                      quantization=quant, kv_cache_dtype=kv))
    prompt = list(range(100, 240))
    sp = SamplingParams(temperature=0, max_tokens=16, ignore_eos=True)
    base = eng(None).generate([prompt], sp)[0].outputs[0].token_ids
    e = eng("mtp")
    assert e.generate([prompt], sp)[0].outputs[0].token_ids == base
    assert e.spec.stats["draft_tokens"] > 0
    e8 = eng("mtp", "mxfp4", "fp8")
    sp2 = SamplingParams(temperature=0.8, top_p=0.95, max_tokens=8, seed=3, ignore_eos=True)
    assert len(e8.generate([prompt, prompt[:40]], sp2)[1].outputs[0].token_ids) == 8


@pytest.mark.parametrize("T,H,G,taps,block", [(8, 256, 16, 4, 8), (40, 5120, 320, 4, 8),
                                               (21, 512, 32, 3, 7)])
def test_dflash_grouped_conv_kernel(T, H, G, taps, block):
    """The drafter's block-causal grouped conv kernel against its torch form (fp32 oracle)."""
    from vllm_sly_radiance_b200.models.dflash2 import grouped_conv
    g = torch.Generator().manual_seed(T + H)
    h = torch.randn(T, H, generator=g).to(torch.bfloat16)
    co = torch.randn(T, 2 * taps * G, generator=g).to(torch.bfloat16)
    delta = co.view(T, 2, taps, G)[:, 1]
    base = (torch.randn(taps, H, generator=g) * 0.1).to(torch.bfloat16)
    want = grouped_conv(h, delta, base, block, G, taps).float()
    got = grouped_conv(h.cuda(), co.cuda().view(T, 2, taps, G)[:, 1], base.cuda(), block, G,
                       taps).float().cpu()
    assert torch.allclose(got, want, atol=2e-2, rtol=1e-2), float((got - want).abs().max())
