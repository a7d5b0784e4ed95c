"""MoE block (routing, shared expert, expert dispatch) on CPU: the tiny MoE hybrid runs through
the engine; the routed output equals a dense per-token evaluation; work-table construction."""
import torch

from vllm_sly_radiance_b200.config import EngineConfig, tiny_moe
from vllm_sly_radiance_b200.engine.llm_engine import LLMEngine
from vllm_sly_radiance_b200.engine.request import SamplingParams
from vllm_sly_radiance_b200.models.hybrid import HybridModel
from vllm_sly_radiance_b200.ops.kernels import moe_work_items


def test_moe_model_generates():
    cfg = EngineConfig(model="tiny_moe", device="cpu", max_model_len=512, max_num_seqs=2,
                       max_num_batched_tokens=128, num_kv_blocks=32)
    out = LLMEngine(cfg).generate([list(range(10, 50))], SamplingParams(temperature=0, max_tokens=4))
    assert len(out[0].outputs[0].token_ids) == 4


def test_moe_routed_matches_dense():
    torch.manual_seed(0)
    m = HybridModel(tiny_moe(), quant="bf16", device="cpu", seed=0)
    blk = m.layers[0].mlp
    x = (torch.randn(6, 256) * 0.5).to(torch.bfloat16)
    ids, w = blk.route(x)
    assert torch.allclose(w.sum(-1), torch.ones(6))
    got = blk.local_experts(x, (None, None), ids, w).float()
    want = torch.zeros(6, 256)
    for t in range(6):
        for j in range(ids.shape[1]):
            e = int(ids[t, j])
            gu = x[t].float() @ blk.dense_gu[e].float().t()
            I = gu.shape[0] // 2
            a = (torch.nn.functional.silu(gu[:I]) * gu[I:]).to(torch.bfloat16).float()
            want[t] += float(w[t, j]) * (a @ blk.dense_dn[e].float().t())
    assert torch.allclose(got, want, atol=2e-2, rtol=2e-2)


def test_work_items():
    counts = torch.tensor([0, 5, 17, 1, 0, 16])
    it = moe_work_items(counts, 16, 10).tolist()
    real = [r for r in it if r[2] > 0]
    assert real == [[1, 0, 5], [2, 5, 16], [2, 21, 1], [3, 22, 1], [5, 23, 16]]
    assert all(r[2] == 0 for r in it[len(real):])


def _ep_logits(model, prompt):
    cfg = EngineConfig(model="tiny_moe", device="cpu", max_model_len=512, max_num_seqs=2,
                       max_num_batched_tokens=256, num_kv_blocks=32, quantization=model.quant,
                       enable_cuda_graphs=False)
    eng = LLMEngine(cfg, model=model)
    eng.add_request(prompt, SamplingParams(temperature=0, max_tokens=1), "r")
    sched = eng.scheduler.schedule()
    res = eng.runner.execute(sched, want_logits=True)
    eng.scheduler.update(sched, res.sampled)
    toks = eng.generate([prompt], SamplingParams(temperature=0, max_tokens=3, ignore_eos=True))
    return res.logits.float(), toks[0].outputs[0].token_ids


def _ep_worker(rank, world, port, quant, prompts, q):
    import os
    import torch.distributed as dist
    from vllm_sly_radiance_b200.parallel.ep import make_ep_group
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    ep = make_ep_group(rank, world, "a2a")
    m = HybridModel(tiny_moe(), quant=quant, device="cpu", seed=0, ep=ep)
    assert m.layers[0].mlp.e_local == 16 // world
    lg, toks = _ep_logits(m, prompts[rank])
    q.put((rank, lg, toks, ep.transport.calls))
    dist.barrier()
    dist.destroy_process_group()


import pytest  # noqa: E402


@pytest.mark.parametrize("quant", ["bf16", "mxfp4"])
def test_expert_parallel_dispatch_combine_matches_single_rank(quant):
    """Data-parallel attention + expert-parallel MoE over two gloo ranks: each rank serves its
    own prompt, owns 8 of the 16 experts and exchanges rows with all_to_all; every rank's logits
    and greedy tokens equal the single-process model's on that prompt."""
    import socket
    import torch.multiprocessing as mp
    prompts = [list(range(20, 70)), list(range(300, 350))]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    procs = [ctx.Process(target=_ep_worker, args=(r, 2, port, quant, prompts, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(2)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, lg, toks, calls in res:
        assert calls > 0
        ref_lg, ref_toks = _ep_logits(HybridModel(tiny_moe(), quant=quant, device="cpu", seed=0),
                                      prompts[rank])
        rel = float((lg - ref_lg).norm() / ref_lg.norm())
        assert rel < 2e-2, (rank, rel)
        assert toks[:2] == ref_toks[:2], (rank, toks, ref_toks)


def test_ep_transport_splits_a_large_step_into_rounds():
    """Tokens beyond the NVLink transport's per-call capacity run as several rounds of at most
    `maxt` tokens, in order; every rank runs the same round count (world 1 here)."""
    from vllm_sly_radiance_b200.parallel.ep_p2p import P2PTransport
    tr = P2PTransport(0, 1, maxt=4)
    tr.begin_step(10)
    assert tr.rounds == 3
    seen = []

    def fake_call(blk, q, s, ids, w):
        seen.append(q.shape[0])
        return q.float().clone()
    tr._call = fake_call

    class Blk:
        w_gate_up = object()
    q = torch.arange(10, dtype=torch.float32).view(10, 1)
    out = tr.dispatch_combine(Blk(), None, (q, torch.ones(10)), torch.zeros(10, 2, dtype=torch.long),
                              torch.ones(10, 2))
    assert seen == [4, 4, 2] and torch.equal(out, q)
    tr.begin_step(3)
    assert tr.rounds == 1
