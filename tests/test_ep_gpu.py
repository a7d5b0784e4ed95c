"""Expert-parallel MoE dispatch / combine over NVLink peer memory (``csrc/ep.cu``) against the
torch.distributed all_to_all transport, on two GPUs (skipped with fewer): each rank routes its own
tokens, different counts per rank, several calls in a row (sequence numbers advance)."""
import os
import socket
from datetime import timedelta

import pytest
import torch

pytestmark = pytest.mark.gpu


def _worker(rank, world, port, q):
    import torch.distributed as dist
    from vllm_sly_radiance_b200.config import tiny_moe
    from vllm_sly_radiance_b200.models.hybrid import HybridModel
    from vllm_sly_radiance_b200.ops import kernels as K
    from vllm_sly_radiance_b200.parallel.ep import make_ep_group
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        a2a = make_ep_group(rank, world, "a2a")
        p2p = make_ep_group(rank, world, "p2p")
        m = HybridModel(tiny_moe(), quant="mxfp4", device="cuda", seed=0, ep=a2a)
        errs = []
        for it, T in enumerate([5 + rank * 3, 33, 1, 64 - rank * 20, 17]):
            g = torch.Generator().manual_seed(100 * it + rank)
            x = (torch.randn(T, 256, generator=g) * 0.5).to(torch.bfloat16).cuda()
            for layer in (0, 1):
                blk = m.layers[layer].mlp
                qq, ss = K.quant_fp8(x)
                ids, w = blk.route(x)
                want = a2a.transport.dispatch_combine(blk, x, (qq, ss), ids, w)
                got = p2p.transport.dispatch_combine(blk, x, (qq, ss), ids, w)
                torch.cuda.synchronize()
                st = int(K.status_word(torch.device("cuda", rank))[0])
                if st:
                    print(f"rank {rank} call {len(errs)} T={T} status {st}: "
                          f"{p2p.transport.header()}", flush=True)
                err = float((got.float() - want.float()).abs().max() /
                            want.float().abs().max().clamp(min=1e-6))
                errs.append(err)
        K.check_status(torch.device("cuda", rank))
        q.put((rank, errs, p2p.transport.calls))
        torch.cuda.synchronize()
        dist.barrier()
        p2p.transport.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_ep_p2p_matches_all_to_all():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=240) for _ in range(2)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, errs, calls in res:
        assert calls == 10
        assert max(errs) < 1e-2, (rank, errs)


def test_ep_p2p_single_rank_protocol():
    """The whole dispatch / work-table / grouped GEMM / combine protocol on one rank (every flag
    it waits for was released by its own earlier kernel) against the local expert path."""
    from vllm_sly_radiance_b200.config import tiny_moe
    from vllm_sly_radiance_b200.models.hybrid import HybridModel
    from vllm_sly_radiance_b200.ops import kernels as K
    from vllm_sly_radiance_b200.parallel.ep import EPGroup
    from vllm_sly_radiance_b200.parallel.ep_p2p import P2PTransport
    tr = P2PTransport(0, 1)
    m = HybridModel(tiny_moe(), quant="mxfp4", device="cuda", seed=0, ep=EPGroup(0, 1, tr))
    dev = torch.device("cuda")
    for it, T in enumerate([5, 33, 1, 64, 17, 2]):
        g = torch.Generator().manual_seed(it)
        x = (torch.randn(T, 256, generator=g) * 0.5).to(torch.bfloat16).to(dev)
        blk = m.layers[it % 2].mlp
        qq, ss = K.quant_fp8(x)
        ids, w = blk.route(x)
        got = tr.dispatch_combine(blk, x, (qq, ss), ids, w)
        want = blk.local_experts(x, (qq, ss), ids, w)
        torch.cuda.synchronize()
        st = int(K.status_word(dev)[0])
        assert st == 0, (it, st, tr.header())
        err = float((got.float() - want.float()).abs().max() /
                    want.float().abs().max().clamp(min=1e-6))
        assert err < 1e-2, (it, err)
    assert tr.header()["epoch"] == 6
