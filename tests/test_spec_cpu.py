"""Speculative decoding on the CPU tiny model: greedy verify with lookup drafts is lossless (same
tokens as plain decoding), the GDN commit restores exactly the accepted prefix, forced schedule."""
import torch

from vllm_sly_radiance_b200.config import EngineConfig
from vllm_sly_radiance_b200.engine.llm_engine import LLMEngine
from vllm_sly_radiance_b200.engine.request import SamplingParams
from vllm_sly_radiance_b200.spec_decode.proposer import LookupProposer


def _engine(spec=None, forced=None):
    cfg = EngineConfig(model="tiny_hybrid", device="cpu", max_model_len=1024, max_num_seqs=4,
                       max_num_batched_tokens=256, num_kv_blocks=64, speculative_method=spec,
                       num_speculative_tokens=4, forced_acceptance=forced)
    return LLMEngine(cfg)


def test_lookup_proposer():
    lp = LookupProposer(k=3)
    assert lp.propose_one([1, 2, 3, 4, 5, 9, 1, 2, 3]) == [4, 5, 9]
    assert lp.propose_one([5, 6, 7]) == []


def test_greedy_spec_is_lossless():
    """Drafts that are partly right (the true greedy continuation with every third token wrong):
    the verified output must equal plain greedy decoding token for token."""
    prompt = [11, 12, 13, 14, 15] * 8 + [11, 12]
    sp = SamplingParams(temperature=0, max_tokens=24, ignore_eos=True)
    base = _engine().generate([prompt], sp)[0].outputs[0].token_ids
    eng = _engine("lookup")

    def oracle(sched, sampled):
        for s in sched.seqs:
            t = sampled.get(s.req.request_id)
            if not t:
                continue
            n = len(s.req.output_token_ids) + len(t)
            d = list(base[n:n + 4])
            for i in range(len(d)):
                if (n + i) % 3 == 2:
                    d[i] = (d[i] + 1) % 4096
            s.req.draft_token_ids = d
    eng.spec._propose = oracle
    spec = eng.generate([prompt], sp)[0].outputs[0].token_ids
    assert spec == base
    st = eng.spec.stats
    assert st["draft_tokens"] > 0 and 0 < st["accepted"] < st["draft_tokens"]


def test_forced_acceptance_counts():
    eng = _engine("forced", forced="uniform")
    sp = SamplingParams(temperature=0, max_tokens=30, ignore_eos=True)
    out = eng.generate([list(range(20, 60))], sp)[0]
    assert len(out.outputs[0].token_ids) == 30
    st = eng.spec.stats
    assert st["steps"] > 0 and st["accepted"] / max(1, st["drafts"]) > 2.0


def test_dflash2_drafter_runs_and_is_lossless_greedy():
    """The DFlash2 drafter path (context K/V from target aux states, block forward, selector walk)
    runs end to end; greedy verification keeps the output identical to plain decoding."""
    prompt = list(range(100, 140))
    sp = SamplingParams(temperature=0, max_tokens=12, ignore_eos=True)
    base = _engine().generate([prompt], sp)[0].outputs[0].token_ids
    eng = _engine("dflash2")
    out = eng.generate([prompt], sp)[0].outputs[0].token_ids
    assert out == base
    assert eng.spec.stats["draft_tokens"] > 0
    sp2 = SamplingParams(temperature=0.8, top_p=0.95, top_k=20, max_tokens=10, seed=1, ignore_eos=True)
    assert len(eng.generate([prompt], sp2)[0].outputs[0].token_ids) == 10
