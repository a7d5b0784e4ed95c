"""Failure detection without a GPU fault (host-side injection).

* A kernel error code in the device status word (a bounded wait that expired) makes the engine
  abort every open request and raise; the OpenAI server returns an error to each client and
  reports itself unhealthy.
* A tensor-parallel rank that leaves between steps: the other rank's next collective fails
  (gloo, short process-group timeout) and its engine aborts the open requests and raises.
Reference: the silent bounded spin of r4d_extras_rx10.patch:232-240 is what this replaces."""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
from fastapi.testclient import TestClient

from vllm_sly_radiance_b200.config import EngineConfig, tiny_hybrid
from vllm_sly_radiance_b200.engine.llm_engine import EngineStepError, LLMEngine
from vllm_sly_radiance_b200.engine.request import SamplingParams
from vllm_sly_radiance_b200.entrypoints.openai_server import build_app
from vllm_sly_radiance_b200.models.hybrid import HybridModel, TPInfo
from vllm_sly_radiance_b200.ops.kernels import KernelFaultError


def _engine(**kw):
    return LLMEngine(EngineConfig(model="tiny_hybrid", device="cpu", max_model_len=512,
                                  max_num_seqs=4, max_num_batched_tokens=128, num_kv_blocks=64,
                                  **kw))


def test_status_word_error_fails_open_requests():
    eng = _engine()
    eng.add_request([5, 6, 7, 8], SamplingParams(temperature=0, max_tokens=8), "a")
    eng.add_request([9, 10, 11], SamplingParams(temperature=0, max_tokens=8), "b")
    eng.step()
    codes = iter([2])
    eng.runner.read_status = lambda: next(codes, 0)      # a peer wait expired in this step
    with pytest.raises(KernelFaultError) as ei:
        eng.step()
    assert ei.value.code == 2
    assert not eng.has_unfinished_requests() and not eng.requests
    assert eng.faults == 1
    # the engine keeps serving new requests afterwards
    out = eng.generate([[1, 2, 3]], SamplingParams(temperature=0, max_tokens=2, ignore_eos=True))
    assert len(out[0].outputs[0].token_ids) == 2


def test_server_reports_kernel_fault():
    eng = _engine()
    state = {"fail": True}

    def read_status():
        if state["fail"]:
            state["fail"] = False
            return 1
        return 0
    eng.runner.read_status = read_status
    app = build_app(eng, "tiny")
    with TestClient(app) as c:
        assert c.get("/health").status_code == 200
        r = c.post("/v1/completions", json={"prompt": "hello", "max_tokens": 4, "temperature": 0})
        assert r.status_code >= 500, r.text
        assert "mbarrier wait timed out" in r.text
        assert c.get("/health").status_code == 503


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_leaves(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))

    def ar(x):
        dist.all_reduce(x)
        return x

    def ag(x):
        parts = [torch.empty_like(x) for _ in range(world)]
        dist.all_gather(parts, x.contiguous())
        return torch.cat(parts, -1)
    tp = TPInfo(rank, world, ar, ag)
    m = HybridModel(tiny_hybrid(), quant="bf16", device="cpu", seed=0, tp=tp)
    cfg = EngineConfig(model="tiny_hybrid", device="cpu", max_model_len=512, max_num_seqs=2,
                       max_num_batched_tokens=256, num_kv_blocks=32, quantization="bf16")
    eng = LLMEngine(cfg, model=m, tp=tp)
    eng.add_request([3, 4, 5, 6], SamplingParams(temperature=0, max_tokens=16), "r")
    eng.step()                          # both ranks: prefill
    eng.step()                          # both ranks: one decode step
    if rank == 1:
        os._exit(0)                     # leaves between steps, with nothing in flight
    try:
        eng.step()
        q.put("no error")
    except EngineStepError as e:
        q.put(("raised", eng.has_unfinished_requests(), len(eng.requests)))


def test_peer_rank_leaving_fails_the_step():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_rank_leaves, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = q.get(timeout=120)
    for p in ps:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert res == ("raised", False, 0), res


def test_workspace_canary_catches_an_overrun(monkeypatch):
    """Debug mode: a write past a workspace's end lands in its canary tail and the check names
    the workspace; untouched canaries pass."""
    from vllm_sly_radiance_b200.ops import kernels as K
    monkeypatch.setattr(K, "_CANARY", True)
    monkeypatch.setattr(K, "_CANARIES", [])
    monkeypatch.setattr(K, "_WS", {})
    ws = K.workspace("cpu", "probe", 100)
    K.check_canaries()
    name, base, n = K._CANARIES[0]
    assert name == "probe" and ws.numel() == n and base.numel() == n + K.CANARY_WORDS
    base[n + 3] = 7                      # an "overrun" by a kernel writing past ws
    with pytest.raises(RuntimeError, match="workspace 'probe' overrun: canary word 3"):
        K.check_canaries()
