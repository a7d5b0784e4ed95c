"""Expert parallelism with data-parallel attention: dispatch / combine of MoE rows.

Each rank of the EP group serves its own requests (attention and GDN layers unsharded) and owns
E / size routed experts.  In every MoE layer a rank sends each (token, top-k slot) row to the rank
owning the selected expert (dispatch), the owners run their experts as one grouped W4A8 GEMM
pair, and the outputs return to the token's rank, where the routing weights sum them (combine).
Every rank calls every MoE layer, with its own (possibly different) token count.

Transports:
  * ``AllToAllTransport`` - torch.distributed all_to_all (gloo on CPU, NCCL on GPU): the
    reference behaviour of vLLM's all2all managers, and the baseline;
  * ``P2PTransport`` (``csrc/ep.cu``) - rows written straight into the owner's receive buffer
    over NVLink peer memory by one kernel, counts and completion signalled with release/acquire
    flags, combine rows written back into the source's combine buffer and reduced there.

Reference behaviour: the reference serves MoE targets TP-sharded through vLLM fused_moe
(``moe-configs/E=256,...``); the EP path is the north star's fused dispatch/combine.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch


@dataclass
class EPGroup:
    rank: int
    size: int
    transport: object


class AllToAllTransport:
    """Dispatch / combine over ``torch.distributed.all_to_all_single``.

    Rows travel as bytes: e4m3 activation row + fp32 scale + int32 local expert id (W4A8 experts),
    or the bf16 row + int32 local expert id (bf16 experts)."""

    def __init__(self, rank: int, world: int, group=None):
        self.rank, self.world, self.group = rank, world, group
        self.calls = 0

    def _a2a(self, x: torch.Tensor, send: list, recv: list) -> torch.Tensor:
        import torch.distributed as dist
        out = x.new_empty((sum(recv),) + tuple(x.shape[1:]))
        dist.all_to_all_single(out, x.contiguous(), recv, send, group=self.group)
        return out

    def dispatch_combine(self, blk, xb, qs, ids, w):
        import torch.distributed as dist
        self.calls += 1
        T, K = ids.shape
        H, El = blk.H, blk.e_local
        dev = xb.device
        flat_e = ids.reshape(-1)
        dest = torch.div(flat_e, El, rounding_mode="floor")
        order = torch.argsort(dest, stable=True)
        rows_t = torch.arange(T, device=dev).repeat_interleave(K)[order]
        le = (flat_e[order] - dest[order] * El).to(torch.int32)
        send_counts = torch.bincount(dest, minlength=self.world).to(torch.int64)
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        send = send_counts.tolist()
        recv = recv_counts.tolist()
        q, s = qs
        w8 = q is not None
        if w8:
            payload = torch.cat([q[rows_t].view(torch.uint8),
                                 s[rows_t].float().view(torch.uint8).view(-1, 4),
                                 le.view(torch.uint8).view(-1, 4)], 1)
        else:
            payload = torch.cat([xb[rows_t].view(torch.uint8).view(-1, 2 * H),
                                 le.view(torch.uint8).view(-1, 4)], 1)
        got = self._a2a(payload, send, recv)
        r_le = got[:, -4:].contiguous().view(torch.int32).view(-1).long()
        if w8:
            r_q = got[:, :H].contiguous().view(torch.float8_e4m3fn)
            r_s = got[:, H:H + 4].contiguous().view(torch.float32).view(-1)
            r_x = None
        else:
            r_q = r_s = None
            r_x = got[:, :2 * H].contiguous().view(torch.bfloat16)
        y = blk.expert_rows(r_q, r_s, r_x, r_le)
        back = self._a2a(y, recv, send)
        out = torch.zeros(T, H, dtype=torch.float32, device=dev)
        out.index_add_(0, rows_t, back.float() * w.reshape(-1)[order][:, None].float())
        return out.to(torch.bfloat16)


def make_ep_group(rank: int, world: int, backend: str = "a2a", group=None) -> EPGroup:
    """backend: ``a2a`` (torch.distributed all_to_all) or ``p2p`` (this library's NVLink
    kernels; CUDA only)."""
    if backend == "p2p":
        from .ep_p2p import P2PTransport
        return EPGroup(rank, world, P2PTransport(rank, world, group))
    return EPGroup(rank, world, AllToAllTransport(rank, world, group))
