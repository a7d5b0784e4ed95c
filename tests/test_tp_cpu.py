"""Tensor parallelism on CPU ranks (gloo, world size 2): the sharded tiny model (column-parallel
in_proj / qkv / gate_up, row-parallel out / o / down + all-reduce, vocab-parallel lm_head +
all-gather) reproduces the single-rank logits; the SPMD request broadcast keeps ranks in step."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from vllm_sly_radiance_b200.config import EngineConfig, tiny_hybrid
from vllm_sly_radiance_b200.engine.llm_engine import LLMEngine
from vllm_sly_radiance_b200.engine.request import SamplingParams
from vllm_sly_radiance_b200.models.hybrid import HybridModel, TPInfo


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _logits(model, prompt):
    cfg = EngineConfig(model="tiny_hybrid", device="cpu", max_model_len=512, max_num_seqs=2,
                       max_num_batched_tokens=256, num_kv_blocks=32, quantization="bf16")
    eng = LLMEngine(cfg, model=model)
    eng.add_request(prompt, SamplingParams(temperature=0, max_tokens=3), "r")
    sched = eng.scheduler.schedule()
    res = eng.runner.execute(sched, want_logits=True)
    eng.scheduler.update(sched, res.sampled)
    out = eng.generate([prompt], SamplingParams(temperature=0, max_tokens=4, ignore_eos=True))
    return res.logits.float(), out[0].outputs[0].token_ids


def _worker(rank, world, port, prompt, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.manual_seed(0)

    def ar(x):
        dist.all_reduce(x)
        return x

    def ag(x):
        parts = [torch.empty_like(x) for _ in range(world)]
        dist.all_gather(parts, x.contiguous())
        return torch.cat(parts, -1)
    tp = TPInfo(rank, world, ar, ag)
    m = HybridModel(tiny_hybrid(), quant="bf16", device="cpu", seed=0, tp=tp)
    lg, toks = _logits(m, prompt)
    if rank == 0:
        q.put((lg, toks))
    dist.barrier()
    dist.destroy_process_group()


def test_tp2_matches_tp1():
    prompt = list(range(30, 90))
    ref_lg, ref_toks = _logits(HybridModel(tiny_hybrid(), quant="bf16", device="cpu", seed=0), prompt)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, prompt, q)) for r in range(2)]
    for p in procs:
        p.start()
    lg, toks = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    rel = float((lg - ref_lg).norm() / ref_lg.norm())
    assert rel < 2e-2, rel
    # bf16 partial sums reduce in a different order across ranks: near-tied argmaxes of a random
    # model may flip after a few steps, so only the first greedy tokens must agree
    assert toks[:2] == ref_toks[:2]


def test_tp3_geometry_of_target():
    """The 27B target widened for TP = 3: GQA 6 and the GDN value/key ratio 3 are kept."""
    from vllm_sly_radiance_b200.config import qwen38_27b
    from vllm_sly_radiance_b200.parallel.tp_pad import needs_padding, padded_config
    c = qwen38_27b(17408)
    p = padded_config(c, 3)
    assert (p.num_q_heads, p.num_kv_heads, p.gdn_num_k_heads, p.gdn_num_v_heads) == (36, 6, 18, 54)
    assert p.intermediate_size == 17472 and p.vocab_size == 248448 and p.real_vocab_size == 248320
    assert p.logical_vocab_size == 248320
    for tp in (1, 2, 4, 8):
        assert not needs_padding(c, tp)


@pytest.mark.parametrize("quant", ["bf16", "mxfp4"])
def test_padded_geometry_is_exact_on_one_rank(quant):
    """Dummy heads / channels / vocabulary rows compute exact zeros: the model widened for TP = 3
    but run on one rank gives the unpadded model's logits (up to the bf16 rounding of the
    row-parallel GEMMs, whose longer K is blocked differently by the host BLAS)."""
    prompt = list(range(30, 90))
    ref_lg, _ = _logits(HybridModel(tiny_hybrid(), quant=quant, device="cpu", seed=0), prompt)
    m = HybridModel(tiny_hybrid(), quant=quant, device="cpu", seed=0, tp_pad=3)
    assert m.cfg.num_kv_heads == 3 and m.cfg.gdn_num_k_heads == 6 and m.cfg.vocab_size == 4224
    lg, _ = _logits(m, prompt)
    assert lg.shape == ref_lg.shape
    rel = float((lg - ref_lg).norm() / ref_lg.norm())
    assert rel < 1e-2, rel
    # the dummy rows and columns themselves are exactly zero
    gdn = m.layers[0].mixer
    assert float(gdn.A_log[4:].abs().sum()) == 0.0 and gdn.conv_w.shape[0] == 2 * 6 * 64 + 6 * 64


def test_tp3_matches_tp1():
    """Three gloo ranks over the padded geometry (kv heads 2 -> 3, GDN heads 4 -> 6, vocab 4096
    -> 4224): the last rank holds every dummy, the gathered logits match one rank."""
    prompt = list(range(30, 90))
    ref_lg, ref_toks = _logits(HybridModel(tiny_hybrid(), quant="bf16", device="cpu", seed=0), prompt)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 3, port, prompt, q)) for r in range(3)]
    for p in procs:
        p.start()
    lg, toks = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert lg.shape == ref_lg.shape
    rel = float((lg - ref_lg).norm() / ref_lg.norm())
    # three bf16 partial sums per row-parallel output, reduced in another order than one rank's
    assert rel < 3e-2, rel
    assert toks[:2] == ref_toks[:2]
