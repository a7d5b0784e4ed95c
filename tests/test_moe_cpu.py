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
