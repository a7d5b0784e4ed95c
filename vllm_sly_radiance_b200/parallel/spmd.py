"""SPMD request broadcast for tensor-parallel serving.

Every TP rank runs an identical engine (same scheduler decisions, same sampling seeds, identical
gathered logits), so the only cross-rank traffic outside the model is the request stream: rank 0
(the HTTP server) broadcasts each step's new/aborted requests over a CPU (gloo) group before the
step.  Reference analogue: vLLM's scheduler-output broadcast to TP workers over a shared-memory
queue (``radiance_allreduce.py:151-152`` uses the same CPU group for its handle exchange)."""
from __future__ import annotations

import torch.distributed as dist


class RequestBroadcaster:
    def __init__(self, rank: int, group=None):
        self.rank = rank
        self.group = group

    def broadcast(self, cmds: list) -> list:
        obj = [cmds if self.rank == 0 else None]
        dist.broadcast_object_list(obj, src=0, group=self.group)
        return obj[0]


def follower_loop(engine, broadcaster: RequestBroadcaster):
    """Ranks > 0: apply rank 0's commands and step in lockstep (no HTTP)."""
    while True:
        cmds = broadcaster.broadcast([])
        stop = False
        for c in cmds:
            if c[0] == "add":
                engine.add_request(c[1], c[2], c[3])
            elif c[0] == "abort":
                engine.abort_request(c[1])
            elif c[0] == "shutdown":
                stop = True
        if stop:
            return
        if engine.has_unfinished_requests():
            engine.step()
