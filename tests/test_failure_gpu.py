"""Bounded device waits on one GPU: a push all-reduce receiver whose peer never pushes returns
after the run-time wait limit (1 ms) with the peer-timeout code in the status word -- no hang, the
context stays usable -- and the engine on that device then fails its open requests and raises."""
import time

import pytest
import torch

from vllm_sly_radiance_b200.ops import kernels as K
from vllm_sly_radiance_b200.ops._ext import ext

pytestmark = pytest.mark.gpu


def _expire_peer_wait(dev):
    """Receiver of a 2-rank push all-reduce with both 'ranks' on this GPU and nobody pushing."""
    H, M = 256, 1
    nbytes = ext().push_buffer_bytes(2, M, H)
    bufs = [torch.zeros(nbytes, dtype=torch.uint8, device=dev) for _ in range(2)]
    half_words = 2 * M * (H // 2)
    out = torch.empty(M, H, dtype=torch.bfloat16, device=dev)
    e = torch.empty(0, device=dev)
    ext().push_allreduce_recv([b.data_ptr() for b in bufs], 0, M, H, half_words, out, e, e, 0.0,
                              e, e, e, 1, K.status_word(dev))
    return bufs, out


def test_peer_wait_expires_with_status():
    dev = torch.device("cuda", 0)
    K.reset_status(dev)
    K.set_wait_limits(dev, mbar_us=0, peer_us=1000)
    try:
        t0 = time.perf_counter()
        _expire_peer_wait(dev)
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        assert dt < 2.0, dt                        # 1 ms limit, not the 5 s default
        with pytest.raises(K.KernelFaultError) as ei:
            K.check_status(dev)
        assert ei.value.code == 2
        assert int(K.status_word(dev)[0]) == 0     # reset, limits kept
        assert int(K.status_word(dev)[3]) == 1000
        x = torch.ones(4, device=dev)              # the context is still usable
        assert float((x * 2).sum()) == 8.0
    finally:
        K.set_wait_limits(dev, 0, 0)
        K.reset_status(dev)


def test_engine_raises_on_device_timeout():
    from vllm_sly_radiance_b200.config import EngineConfig
    from vllm_sly_radiance_b200.engine.llm_engine import LLMEngine
    from vllm_sly_radiance_b200.engine.request import SamplingParams
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(0)
    eng = LLMEngine(EngineConfig(model="tiny_hybrid", device="cuda", max_model_len=512,
                                 max_num_seqs=2, max_num_batched_tokens=256, num_kv_blocks=32,
                                 enable_cuda_graphs=True))
    eng.add_request(list(range(10, 40)), SamplingParams(temperature=0, max_tokens=8), "a")
    eng.step()
    K.set_wait_limits(dev, mbar_us=0, peer_us=1000)
    try:
        _expire_peer_wait(dev)          # on the engine's stream, before its next step
        with pytest.raises(K.KernelFaultError):
            eng.step()
        assert not eng.has_unfinished_requests()
        assert int(K.status_word(dev)[0]) == 0
    finally:
        K.set_wait_limits(dev, 0, 0)
    out = eng.generate([list(range(5, 20))], SamplingParams(temperature=0, max_tokens=3,
                                                            ignore_eos=True))
    assert len(out[0].outputs[0].token_ids) == 3
