"""Engine on the GPU: the tiny hybrid model through the CUDA kernels vs the CPU oracle."""
import pytest
import torch

from vllm_sly_radiance_b200.config import EngineConfig, tiny_hybrid
from vllm_sly_radiance_b200.engine.llm_engine import LLMEngine
from vllm_sly_radiance_b200.engine.request import SamplingParams
from vllm_sly_radiance_b200.models.hybrid import HybridModel

pytestmark = pytest.mark.gpu


def _engine(device, graphs=False, chunk=64, quant="mxfp4", kv="fp8"):
    cfg = EngineConfig(model="tiny_hybrid", device=device, max_model_len=1024, max_num_seqs=4,
                       max_num_batched_tokens=chunk, enable_cuda_graphs=graphs, num_kv_blocks=64,
                       kv_cache_dtype=kv)
    # weights drawn on the CPU generator so both devices hold the same model
    model = HybridModel(tiny_hybrid(), quant=quant, device=device, seed=0, init_device="cpu")
    return LLMEngine(cfg, model=model)


@pytest.mark.parametrize("quant,kv,tol", [("bf16", "bf16", 2e-2), ("mxfp4", "fp8", 0.15)])
def test_prefill_logits_match_cpu_oracle(quant, kv, tol):
    """GPU kernels (attention, GDN, producers; GEMMs for mxfp4) vs the CPU oracle over a
    3-chunk prefill.  The W4A8 arm quantizes every activation to e4m3: the random tiny model
    amplifies single-code rounding flips (a 0.2 % input perturbation moves its logits ~12 %),
    so that arm only bounds the drift."""
    prompt = list(range(7, 7 + 150))
    outs = {}
    for dev in ("cpu", "cuda"):
        eng = _engine(dev, quant=quant, kv=kv)
        eng.add_request(prompt, SamplingParams(temperature=0, max_tokens=1), "r")
        sched = eng.scheduler.schedule()
        res = None
        while True:
            res = eng.runner.execute(sched, want_logits=True)
            eng.scheduler.update(sched, res.sampled)
            if res.sampled:
                break
            sched = eng.scheduler.schedule()
        outs[dev] = res.logits.float().cpu()
    a, b = outs["cuda"], outs["cpu"]
    # fp8 activation codes can flip at rounding boundaries between the kernels and the oracle;
    # compare in norm and by the greedy token
    rel = float((a - b).norm() / b.norm())
    assert rel < tol, rel


def test_greedy_decode_graph_matches_eager():
    prompts = [list(range(10, 60)), list(range(300, 420)), list(range(1000, 1003))]
    res = {}
    for graphs in (False, True):
        eng = _engine("cuda", graphs=graphs)
        outs = eng.generate(prompts, SamplingParams(temperature=0, max_tokens=12, ignore_eos=True))
        res[graphs] = [o.outputs[0].token_ids for o in outs]
    assert res[False] == res[True]


def test_sampling_runs_and_is_seeded():
    eng = _engine("cuda", graphs=True)
    sp = SamplingParams(temperature=0.7, top_p=0.95, top_k=20, max_tokens=10, seed=5, ignore_eos=True)
    a = eng.generate([list(range(50, 90))], sp)[0].outputs[0].token_ids
    b = eng.generate([list(range(50, 90))], sp)[0].outputs[0].token_ids
    assert len(a) == 10 and a == b


def test_kv_offload_host_tier_on_gpu():
    """Evicted prefix blocks and the GDN snapshot round-trip through pinned host memory (device
    gather kernel + one copy per item) and the resumed prefill equals a recompute."""
    from vllm_sly_radiance_b200.engine.request import SamplingParams as SP

    def eng_(offload):
        cfg = EngineConfig(model="tiny_hybrid", device="cuda", max_model_len=1024, max_num_seqs=2,
                           max_num_batched_tokens=4096, enable_cuda_graphs=False,
                           num_kv_blocks=22, block_size=16, enable_prefix_caching=offload,
                           prefix_snapshot_slots=1, kv_offload_gb=0.002 if offload else 0.0,
                           quantization="bf16", kv_cache_dtype="bf16")
        return LLMEngine(cfg)
    g = torch.Generator().manual_seed(4)
    a = torch.randint(3, 4096, (150,), generator=g).tolist()
    b = torch.randint(3, 4096, (320,), generator=g).tolist()
    eng = eng_(True)
    assert eng.kv.offload.kv.vec and eng.kv.offload.state.vec     # the kernel path
    eng.generate([a], SP(temperature=0, max_tokens=2, ignore_eos=True))
    eng.generate([b], SP(temperature=0, max_tokens=2, ignore_eos=True))
    out = eng.generate([a + [11, 12, 13]], SP(temperature=0, max_tokens=6, ignore_eos=True))
    assert eng.kv.offload_hits == 1
    assert eng.kv.offload.stats["kv"]["loaded_host"] >= 9
    ref = eng_(False).generate([a + [11, 12, 13]], SP(temperature=0, max_tokens=6,
                                                       ignore_eos=True))
    assert out[0].outputs[0].token_ids == ref[0].outputs[0].token_ids
