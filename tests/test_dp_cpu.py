"""Data parallelism on CPU: two engine replicas in their own processes behind the front end give
the same greedy tokens as one engine, and requests spread over both replicas."""
import pytest
import torch

from vllm_sly_radiance_b200.config import EngineConfig
from vllm_sly_radiance_b200.engine.llm_engine import LLMEngine
from vllm_sly_radiance_b200.engine.request import SamplingParams
from vllm_sly_radiance_b200.entrypoints.dp import DataParallelEngine


def _cfg():
    return EngineConfig(model="tiny_hybrid", device="cpu", max_model_len=512, max_num_seqs=4,
                        max_num_batched_tokens=256, num_kv_blocks=64, enable_cuda_graphs=False)


@pytest.mark.timeout(600)
def test_two_replicas_match_one_engine():
    prompts = [list(range(5 + i, 40 + 3 * i)) for i in range(4)]
    sp = SamplingParams(temperature=0, max_tokens=5, ignore_eos=True)
    want = [o.outputs[0].token_ids for o in LLMEngine(_cfg()).generate(prompts, sp)]
    dp = DataParallelEngine(_cfg(), 2)
    try:
        rids = [dp.add_request(p, sp) for p in prompts]
        assert sorted(dp.owner[r] for r in rids) == [0, 0, 1, 1]
        final = {}
        while dp.has_unfinished_requests():
            for o in dp.step(timeout=1.0):
                if o.finished:
                    final[o.request_id] = o
        assert [final[r].outputs[0].token_ids for r in rids] == want
        assert dp.generated_tokens == 4 * 5
        assert "replica=\"1\"" in dp.metrics.prometheus("m")
        # abort: the request leaves the front end at once and its replica drops it
        r = dp.add_request(prompts[0], SamplingParams(temperature=0, max_tokens=200, ignore_eos=True))
        dp.abort_request(r)
        assert not dp.has_unfinished_requests()
    finally:
        dp.shutdown()
