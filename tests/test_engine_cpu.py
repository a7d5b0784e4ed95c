"""CPU tests of the model math and engine: GDN recurrent vs chunked oracle, chunked prefill vs
one-shot prefill, scheduler behaviour, the tiny config's KL(bf16 || MXFP4 W4A8)."""
import math

import pytest
import torch

from vllm_sly_radiance_b200.config import EngineConfig, tiny_hybrid
from vllm_sly_radiance_b200.engine.kv_cache import KVCacheManager
from vllm_sly_radiance_b200.engine.llm_engine import LLMEngine
from vllm_sly_radiance_b200.engine.request import Request, SamplingParams
from vllm_sly_radiance_b200.engine.scheduler import Scheduler
from vllm_sly_radiance_b200.models.hybrid import HybridModel
from vllm_sly_radiance_b200.ops import reference as ref


def test_gdn_chunked_equals_recurrent():
    torch.manual_seed(0)
    L, Hk, Hv, dk, dv = 150, 2, 4, 16, 8
    q = ref.l2norm(torch.randn(L, Hk, dk).double()).float()
    k = ref.l2norm(torch.randn(L, Hk, dk).double()).float()
    v = torch.randn(L, Hv, dv)
    g = -torch.rand(L, Hv) * 0.1
    beta = torch.rand(L, Hv)
    s0 = torch.randn(Hv, dv, dk) * 0.5
    o1, s1 = ref.gdn_recurrent(q, k, v, g, beta, s0, dk ** -0.5)
    o2, s2 = ref.gdn_chunked(q, k, v, g, beta, s0, dk ** -0.5)
    assert torch.allclose(o1, o2, atol=1e-4, rtol=1e-3)
    assert torch.allclose(s1, s2, atol=1e-4, rtol=1e-3)


def _engine(chunk, quant="mxfp4", graphs=False):
    cfg = EngineConfig(model="tiny_hybrid", device="cpu", max_model_len=1024, max_num_seqs=4,
                       max_num_batched_tokens=chunk, enable_cuda_graphs=graphs, num_kv_blocks=64,
                       quantization=quant)
    return LLMEngine(cfg)


def _prefill_logits(eng, prompt):
    eng.add_request(prompt, SamplingParams(temperature=0, max_tokens=1), "r")
    while True:
        sched = eng.scheduler.schedule()
        res = eng.runner.execute(sched, want_logits=True)
        eng.scheduler.update(sched, res.sampled)
        if res.sampled:
            return res.logits.float()


def test_chunked_prefill_matches_single_chunk():
    prompt = list(range(5, 5 + 200))
    a = _prefill_logits(_engine(4096), prompt)
    b = _prefill_logits(_engine(48), prompt)       # 5 chunks, 48 not a page multiple
    rel = float((a - b).abs().max() / a.abs().max())
    assert rel < 2e-2, rel


def test_decode_matches_recompute():
    """Greedy decode with cached state/KV produces the tokens a full recompute would."""
    eng = _engine(4096)
    prompt = list(range(40, 80))
    out = eng.generate([prompt], SamplingParams(temperature=0, max_tokens=4, ignore_eos=True))[0]
    toks = out.outputs[0].token_ids
    # recompute the last step from scratch with prompt + first 3 generated tokens
    eng2 = _engine(4096)
    lg = _prefill_logits(eng2, prompt + toks[:3])
    assert int(lg.argmax(-1)[0]) == toks[3]


def test_kl_quantized_vs_bf16_tiny():
    """BASELINE config 1 check: KL(bf16 || MXFP4 W4A8 + fp8 KV) on a 128-token prompt."""
    torch.manual_seed(0)
    prompt = torch.randint(3, 4096, (128,)).tolist()
    lq = _prefill_logits(_engine(4096, "mxfp4"), prompt)
    lb = _prefill_logits(_engine(4096, "bf16"), prompt)
    p = torch.log_softmax(lb, -1)
    q = torch.log_softmax(lq, -1)
    kl = float((p.exp() * (p - q)).sum(-1).mean())
    assert kl < 0.05, kl


def test_mxfp6_mxfp8_models_close_to_bf16():
    """The wider MX element types run the same engine path.  e2m3 and e4m3 both carry three
    mantissa bits (against e2m1's one), so both land well below MXFP4's KL to the bf16 model; the
    remaining gap is the e4m3 activations and KV they share."""
    torch.manual_seed(0)
    prompt = torch.randint(3, 4096, (96,)).tolist()
    lb = torch.log_softmax(_prefill_logits(_engine(4096, "bf16"), prompt), -1)
    kls = {}
    for quant in ("mxfp4", "mxfp6", "mxfp8"):
        eng = _engine(4096, quant)
        fmts = {lin.w.fmt for lin in _linears(eng.model)}
        assert fmts == {{"mxfp4": "e2m1", "mxfp6": "e2m3", "mxfp8": "e4m3"}[quant]}, fmts
        lq = torch.log_softmax(_prefill_logits(eng, prompt), -1)
        kls[quant] = float((lb.exp() * (lb - lq)).sum(-1).mean())
    assert kls["mxfp4"] < 0.05 and max(kls["mxfp6"], kls["mxfp8"]) < kls["mxfp4"] / 3, kls


def _linears(model):
    from vllm_sly_radiance_b200.models.layers import Linear
    out, seen = [], set()

    def walk(o, depth=0):
        if id(o) in seen or depth > 4:
            return
        seen.add(id(o))
        if isinstance(o, Linear):
            if o.quant == "mxfp4":
                out.append(o)
            return
        if isinstance(o, (list, tuple)):
            for v in o:
                walk(v, depth + 1)
        elif hasattr(o, "__dict__"):
            for v in vars(o).values():
                walk(v, depth + 1)
    walk(model)
    return out


def test_int4_model_and_int4_lm_head_close_to_bf16():
    """W4A16 INT4 linears (and an int4 lm_head on the MXFP4 model) stay close to the bf16 model."""
    torch.manual_seed(0)
    prompt = torch.randint(3, 4096, (96,)).tolist()
    lb = _prefill_logits(_engine(4096, "bf16"), prompt)
    li = _prefill_logits(_engine(4096, "int4"), prompt)
    cfg = EngineConfig(model="tiny_hybrid", device="cpu", max_model_len=1024, max_num_seqs=4,
                       max_num_batched_tokens=4096, enable_cuda_graphs=False, num_kv_blocks=64,
                       quantization="mxfp4", lm_head_quant="int4")
    eng = LLMEngine(cfg)
    assert eng.model.lm_head.quant == "int4"
    lh = _prefill_logits(eng, prompt)
    p = torch.log_softmax(lb, -1)
    for lq in (li, lh):
        q = torch.log_softmax(lq, -1)
        kl = float((p.exp() * (p - q)).sum(-1).mean())
        assert kl < 0.05, kl


def test_scheduler_chunking_and_preemption():
    kv = KVCacheManager(num_blocks=8, block_size=16, num_slots=4)
    sch = Scheduler(kv, max_num_seqs=3, max_num_batched_tokens=64, max_model_len=512)
    reqs = [Request(list(range(60)), SamplingParams(max_tokens=50)) for _ in range(3)]
    for r in reqs:
        sch.add(r)
    out = sch.schedule()
    assert [s.num_new_tokens for s in out.seqs] == [60, 4]
    sampled = {s.req.request_id: [7] for s in out.seqs if s.samples}
    sch.update(out, sampled)
    assert reqs[0].num_computed_tokens == 60 and len(reqs[0].output_token_ids) == 1
    # keep decoding until the 7 usable blocks run out -> preemption of the newest request
    preempted = 0
    for _ in range(80):
        out = sch.schedule()
        if out.is_empty:
            break
        preempted += len(out.preempted)
        sampled = {s.req.request_id: [7] for s in out.seqs if s.samples}
        sch.update(out, sampled)
    assert preempted > 0
    assert all(r.status.finished or r in sch.running or r in sch.waiting for r in reqs)


def test_engine_generate_stop_and_abort():
    eng = _engine(64)
    rid = eng.add_request(list(range(30)), SamplingParams(temperature=0, max_tokens=100))
    eng.step()
    assert eng.abort_request(rid)
    assert not eng.has_unfinished_requests()
    outs = eng.generate([list(range(20))], SamplingParams(temperature=0, max_tokens=3))
    assert len(outs[0].outputs[0].token_ids) == 3 and outs[0].outputs[0].finish_reason == "length"


def test_kv4_cache_engine_and_capacity():
    """4-bit KV cache (int4 + fp16 scale/zero per 16 elements, 16-token pages): the engine runs,
    logits stay close to the fp8-KV engine, and a page holds more tokens per byte."""
    from vllm_sly_radiance_b200.models.hybrid import HybridModel
    from vllm_sly_radiance_b200.config import tiny_hybrid
    prompt = list(range(5, 105))

    def run(kv):
        cfg = EngineConfig(model="tiny_hybrid", device="cpu", max_model_len=1024, max_num_seqs=4,
                           max_num_batched_tokens=48, num_kv_blocks=64, kv_cache_dtype=kv,
                           quantization="bf16")
        eng = LLMEngine(cfg)
        return _prefill_logits(eng, prompt), eng
    a, e4 = run("int4")
    b, e8 = run("bf16")
    assert e4.config.block_size == 16
    rel = float((a - b).norm() / b.norm())
    assert rel < 0.1, rel
    m = e4.model
    per_tok4 = m.cache_bytes_per_block(16, "int4") / 16
    per_tok8 = m.cache_bytes_per_block(64, "fp8") / 64
    assert per_tok4 < per_tok8


def _prefix_engine(prefix, interval=0):
    cfg = EngineConfig(model="tiny_hybrid", device="cpu", max_model_len=1024, max_num_seqs=4,
                       max_num_batched_tokens=4096, enable_cuda_graphs=False,
                       num_kv_blocks=64, block_size=16, enable_prefix_caching=prefix,
                       prefix_snapshot_slots=4, prefix_snapshot_interval=interval)
    return LLMEngine(cfg)


def _first_step_logits(eng, prompt):
    """Logits of the first sampled position; also the prompt tokens skipped by the cache."""
    eng.add_request(prompt, SamplingParams(temperature=0, max_tokens=1), "r2")
    skipped = None
    while True:
        sched = eng.scheduler.schedule()
        if skipped is None:
            skipped = sched.seqs[0].req.num_computed_tokens
        for s in sched.seqs:
            if s.req.restore_snapshot is not None:
                eng.model.copy_state(eng.caches, s.req.restore_snapshot, s.req.state_slot)
                eng.kv.release_restore(s.req)
        res = eng.runner.execute(sched, want_logits=True)
        eng.scheduler.update(sched, res.sampled)
        if res.sampled:
            return res.logits.float(), skipped


@pytest.mark.parametrize("interval,second_len,skip", [(0, None, 144), (64, 140, 128)])
def test_prefix_caching_restores_gdn_state(interval, second_len, skip):
    """A prompt sharing a cached prefix skips those tokens (attention blocks + the GDN state
    snapshot at a block boundary) and produces the logits of a full recompute: a multi-turn
    continuation (snapshot at the previous prompt's last boundary) and a shared leading part
    (snapshots every `interval` tokens)."""
    base = torch.randint(3, 4096, (150,), generator=torch.Generator().manual_seed(3)).tolist()
    second = (base + [11, 12, 13, 14, 15]) if second_len is None else \
        (base[:second_len] + [11, 12, 13, 14, 15])
    eng = _prefix_engine(True, interval)
    eng.generate([base], SamplingParams(temperature=0, max_tokens=2, ignore_eos=True))
    assert eng.kv.snap_by_hash, "no GDN snapshot taken"
    got, skipped = _first_step_logits(eng, second)
    assert skipped == skip, skipped
    want = _prefill_logits(_prefix_engine(False), second)
    rel = float((got - want).abs().max() / want.abs().max())
    assert rel < 2e-2, rel
    assert eng.kv.hits >= 1


def _offload_engine(host_gb, disk_dir=None, disk_gb=0.0, policy="lru", frac=0.5):
    cfg = EngineConfig(model="tiny_hybrid", device="cpu", max_model_len=1024, max_num_seqs=2,
                       max_num_batched_tokens=4096, enable_cuda_graphs=False,
                       num_kv_blocks=22, block_size=16, enable_prefix_caching=True,
                       prefix_snapshot_slots=1, kv_offload_gb=host_gb,
                       kv_offload_disk_dir=disk_dir, kv_offload_disk_gb=disk_gb,
                       kv_offload_policy=policy, kv_offload_state_fraction=frac)
    return LLMEngine(cfg)


@pytest.mark.parametrize("tier", ["host_lru", "host_arc", "disk"])
def test_kv_offload_tiers_restore_evicted_prefix(tier, tmp_path):
    """A prefix whose KV blocks and GDN snapshot were evicted from the GPU cache (a second long
    prompt takes all 21 blocks and the single snapshot slot) comes back from the host RAM tier
    (LRU / ARC) or, with a tiny RAM tier, partly from the disk tier: the tokens are skipped and
    the logits equal a full recompute."""
    g = torch.Generator().manual_seed(4)
    a = torch.randint(3, 4096, (150,), generator=g).tolist()
    b = torch.randint(3, 4096, (320,), generator=g).tolist()
    if tier == "disk":
        eng = _offload_engine(0.00025, str(tmp_path / "kv"), 0.01, frac=0.9)
    else:
        eng = _offload_engine(0.002, policy=tier.split("_")[1])
    eng.generate([a], SamplingParams(temperature=0, max_tokens=2, ignore_eos=True))
    eng.generate([b], SamplingParams(temperature=0, max_tokens=2, ignore_eos=True))
    st = eng.kv.offload.stats
    assert st["kv"]["saved"] >= 9 and st["state"]["saved"] >= 1, st
    if tier == "disk":
        assert st["kv"]["spilled"] > 0 and st["kv"]["disk_items"] > 0, st
    second = a + [11, 12, 13, 14, 15]
    got, skipped = _first_step_logits(eng, second)
    assert skipped == 144, skipped
    assert eng.kv.offload_hits == 1
    st = eng.kv.offload.stats
    assert st["kv"]["loaded_host"] + st["kv"]["loaded_disk"] >= 9, st
    if tier == "disk":
        assert st["kv"]["loaded_disk"] > 0, st
    want = _prefill_logits(_prefix_engine(False), second)
    rel = float((got - want).abs().max() / want.abs().max())
    assert rel < 2e-2, rel


def test_arc_policy_prefers_frequent_items():
    """ARC keeps an item hit twice (T2) over a scan of one-time items that LRU would keep."""
    from vllm_sly_radiance_b200.engine.kv_offload import ARCPolicy, LRUPolicy
    for cls, survives in ((ARCPolicy, True), (LRUPolicy, False)):
        p = cls(4)
        resident = set()
        for k in ("hot", "a", "b"):
            for v in p.insert(k):
                resident.discard(v)
            resident.add(k)
        p.hit("hot")
        for k in ("s1", "s2", "s3", "s4"):
            for v in p.insert(k):
                resident.discard(v)
            resident.add(k)
        assert ("hot" in p) == survives, cls
        assert len(p) <= 4 and resident == {k for k in resident if k in p}


def _snap_manager(num_blocks=64):
    return KVCacheManager(num_blocks, 16, 4, enable_prefix_caching=True, num_snapshots=1)


def _cache_prefix(kv, tokens):
    """Publish `tokens`' full blocks and a GDN snapshot at its last block boundary (what a
    finished prefill leaves behind)."""
    r = Request(tokens, SamplingParams(temperature=0, max_tokens=1))
    assert kv.allocate(r, len(tokens))
    r.num_computed_tokens = (len(tokens) - 1) // 16 * 16
    sid = kv.take_snapshot(r)
    assert sid is not None
    r.num_computed_tokens = len(tokens)
    kv.register_blocks(r)
    kv.free(r)
    return sid


def test_pending_snapshot_restore_is_pinned():
    """A waiting request whose admission failed after a prefix hit keeps its snapshot slot: other
    prefills that reserve snapshots meanwhile cannot recycle it (one snapshot slot)."""
    kv = _snap_manager()
    a = list(range(100, 150))
    sid = _cache_prefix(kv, a)
    b = Request(a + [7, 8, 9], SamplingParams(temperature=0, max_tokens=1))
    assert kv.match_prefix(b) == 48 and b.restore_snapshot == sid
    kv.adopt_prefix(b, 48)
    # another prompt reaches its snapshot point while b still waits: no slot may be taken
    c = Request(list(range(300, 340)), SamplingParams(temperature=0, max_tokens=1))
    assert kv.allocate(c, 40)
    c.num_computed_tokens = 32
    assert kv.take_snapshot(c) is None
    assert kv.snap_lru[sid] == kv._hashes(a[:48])[-1]      # b's snapshot untouched
    # the restore copy is issued: the slot becomes reusable
    kv.release_restore(b)
    assert kv.take_snapshot(c) == sid


def test_aborted_restore_unpins_snapshot():
    kv = _snap_manager()
    a = list(range(100, 150))
    sid = _cache_prefix(kv, a)
    b = Request(a + [7], SamplingParams(temperature=0, max_tokens=1))
    assert kv.match_prefix(b) == 48
    kv.adopt_prefix(b, 48)
    assert kv.snap_pins == {sid: 1}
    kv.free(b)                               # abort / preemption path
    assert kv.snap_pins == {} and b.restore_snapshot is None


class _FakeTier:
    """Offload stand-in: holds one GDN snapshot (hash `h`) and any KV blocks."""

    def __init__(self, h):
        self.h = h
        self.restored = 0

    def has_block(self, h):
        return False

    def has_state(self, h):
        return h == self.h

    def restore_state(self, h, reserve):
        sid = reserve()
        assert sid is not None
        self.restored += 1
        return sid

    def save_state(self, h, sid):
        pass


def test_tier_restore_skips_when_every_snapshot_slot_is_pinned():
    """A tier snapshot is only brought back when a snapshot slot can be reserved without
    recycling one that a pending restore pins (two requests in the same schedule)."""
    kv = _snap_manager()
    a = list(range(100, 150))
    sid = _cache_prefix(kv, a)
    b = Request(a + [1], SamplingParams(temperature=0, max_tokens=1))
    assert kv.match_prefix(b) == 48                # pins the only slot
    other = list(range(500, 550))
    r = Request(other, SamplingParams(temperature=0, max_tokens=1))
    assert kv.allocate(r, 50)
    r.num_computed_tokens = 50
    kv.register_blocks(r)
    kv.free(r)
    tier = _FakeTier(kv._hashes(other[:48])[-1])
    kv.offload = tier
    kv.flush_offload = lambda: None
    c = Request(other + [2], SamplingParams(temperature=0, max_tokens=1))
    assert kv.match_prefix(c) == 0 and tier.restored == 0 and c.restore_snapshot is None
    assert kv.snap_lru[sid] == kv._hashes(a[:48])[-1]
    kv.release_restore(b)
    assert kv.match_prefix(c) == 48 and tier.restored == 1 and c.restore_snapshot == sid


def test_step_trace_summaries():
    """RADIANCE_STEP_TRACE=N: a summary every N steps with the per-phase medians."""
    eng = _engine(4096)
    from vllm_sly_radiance_b200.utils.step_trace import StepTrace
    eng.trace = StepTrace(every=3, device="cpu")
    eng.generate([list(range(10, 40))], SamplingParams(temperature=0, max_tokens=7, ignore_eos=True))
    assert len(eng.trace.summaries) == 2
    s = eng.trace.summaries[0]
    assert s["steps"] == 3 and s["execute"] > 0 and "interval" in s


def test_workspace_growth_keeps_old_buffers_alive():
    """An outgrown kernel workspace stays allocated: CUDA graphs captured with it still address
    its counters."""
    from vllm_sly_radiance_b200.ops import kernels as K
    a = K.workspace("cpu", "test_grow", 10)
    b = K.workspace("cpu", "test_grow", 1 << 17)
    assert b.numel() >= 1 << 17 and b.data_ptr() != a.data_ptr()
    assert any(t is a for t in K._WS_RETIRED)
    assert K.workspace("cpu", "test_grow", 5) is b
