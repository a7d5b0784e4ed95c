"""Tensor-parallel communication.

Backends:
  * ``nccl``  - torch.distributed all-reduce / all-gather (the in-tree baseline build).
  * ``fused`` - this library's NVLink kernels (symmetric-memory all-reduce, fused into the
                row-parallel GEMM epilogue where available); falls back to NCCL per call only
                for shapes the fused path does not cover (reported by ``stats``).
Reference: RadianceAllreduce over P2P IPC scratch with NCCL fallback outside its size bands
(``radiance_allreduce.py:65-358``)."""
from __future__ import annotations

import torch

from ..models.hybrid import TPInfo


def make_tp_info(rank: int, world: int, backend: str = "nccl", group=None) -> TPInfo:
    import torch.distributed as dist

    def all_reduce(x: torch.Tensor) -> torch.Tensor:
        dist.all_reduce(x, group=group)
        return x

    def all_gather_last(x: torch.Tensor) -> torch.Tensor:
        parts = [torch.empty_like(x) for _ in range(world)]
        dist.all_gather(parts, x.contiguous(), group=group)
        return torch.cat(parts, dim=-1)

    tp = TPInfo(rank, world, all_reduce, all_gather_last)
    if backend == "fused" and torch.cuda.is_available():
        try:
            from .symm import FusedComm
            fc = FusedComm.create(rank, world, group)
            if fc is not None:
                tp.all_reduce = fc.all_reduce
                tp.all_reduce_add_rms_quant = fc.all_reduce_add_rms_quant
                tp.fused = fc
        except ImportError:
            pass
    return tp
