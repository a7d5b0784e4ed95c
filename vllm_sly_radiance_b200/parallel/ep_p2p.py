"""NVLink peer-memory transport for expert-parallel MoE (``csrc/ep.cu``).

One IPC-mapped buffer per rank holds the receive rows of every source (e4m3 rows, fp32 scales,
(token, slot) meta), the per-expert counts and completion flags, and this rank's combine buffer.
Per MoE call: ``ep_dispatch`` (rows straight into the owners' grouped-GEMM input layout),
``ep_items`` (wait for every source, work table over the receive rows in place), the two grouped
W4A8 GEMMs with SiLU*mul + e4m3 between them on the covered rows only, and ``ep_combine``
(outputs back into each source's combine buffer; weighted top-k sum there).  No host
synchronisation: the sizes the host sees are capacities (``maxt`` tokens per rank per call).
"""
from __future__ import annotations

import torch

from ..ops._ext import ext
from ..ops.kernels import status_word


class P2PTransport:
    def __init__(self, rank: int, world: int, group=None, maxt: int = 256, bn: int = 16):
        self.rank, self.world, self.group = rank, world, group
        self.maxt, self.bn = maxt, bn
        self.rounds = 1          # transport rounds per MoE call this step (begin_step)
        self.buf = None
        self.calls = 0
        self.opened = []

    def _setup(self, H: int, K: int, El: int, device):
        """Allocate and IPC-map the buffers (collective: every rank's first call)."""
        import torch.distributed as dist
        self.H, self.K, self.El = H, K, El
        self.maxr = self.maxt * K
        nbytes = ext().ep_buffer_bytes(self.world, self.maxr, H, K, self.maxt)
        self.buf = torch.zeros(nbytes, dtype=torch.uint8, device=device)
        handles = [None] * self.world
        if self.world > 1:
            h = ext().ipc_handle(self.buf)
            dist.all_gather_object(handles, h.numpy().tobytes(), group=self.group)
        self.peers = []
        for r in range(self.world):
            if r == self.rank:
                self.peers.append(self.buf.data_ptr())
            else:
                p = ext().ipc_open(torch.frombuffer(bytearray(handles[r]), dtype=torch.uint8))
                self.peers.append(p)
                self.opened.append(p)
        q_off, s_off, _, _ = ext().ep_offsets(self.world, self.maxr, H, K, self.maxt)
        R = self.world * self.maxr
        self.R = R
        self.recv_q = self.buf[q_off:q_off + R * H].view(torch.float8_e4m3fn).view(R, H)
        self.recv_s = self.buf[s_off:s_off + R * 4].view(torch.float32)
        self.max_items = R // self.bn + self.world * El + 1
        self.items = torch.zeros(self.max_items, 3, dtype=torch.int32, device=device)
        torch.cuda.synchronize(device)
        if self.world > 1:
            dist.barrier(group=self.group)

    def begin_step(self, T: int) -> None:
        """Per forward step, before the first MoE layer: every rank learns the largest token count
        of the group (one small collective), so all ranks run the same number of transport
        rounds of at most ``maxt`` tokens each (a prefill chunk larger than the capacity runs as
        several rounds; ranks with fewer tokens send empty slices)."""
        if self.world <= 1:
            self.rounds = max(1, -(-T // self.maxt))
            return
        import torch.distributed as dist
        t = torch.tensor([T], dtype=torch.int64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)
        self.rounds = max(1, -(-int(t.item()) // self.maxt))

    def dispatch_combine(self, blk, xb, qs, ids, w):
        q, s = qs
        if q is None or blk.w_gate_up is None:
            raise RuntimeError("the NVLink EP transport needs W4A8 (mxfp4) experts")
        T, K = ids.shape
        if self.rounds > 1:
            if T > self.rounds * self.maxt:
                raise RuntimeError(f"{T} tokens exceed {self.rounds} rounds of {self.maxt}")
            outs = []
            for r in range(self.rounds):
                a, b = min(T, r * self.maxt), min(T, (r + 1) * self.maxt)
                outs.append(self._call(blk, q[a:b], s[a:b], ids[a:b], w[a:b]))
            return torch.cat(outs, 0)
        if T > self.maxt:
            raise RuntimeError(f"{T} tokens exceed the EP transport capacity {self.maxt} per call")
        return self._call(blk, q, s, ids, w)

    def _call(self, blk, q, s, ids, w):
        T, K = ids.shape
        dev = q.device
        if self.buf is None:
            self._setup(blk.H, K, blk.e_local, dev)
        self.calls += 1
        st = status_word(dev)
        I, H = blk.I, blk.H
        ext().ep_dispatch(self.peers, self.rank, self.maxr, self.El, self.maxt, q, s,
                          ids.to(torch.int32).contiguous(), st)
        ext().ep_items(self.peers, self.rank, self.maxr, H, K, self.El, self.maxt, self.bn,
                       self.items, st)
        gu = torch.empty(self.R, 2 * I, dtype=torch.bfloat16, device=dev)
        ext().mxfp4_grouped_gemm(self.recv_q, self.recv_s, blk.w_gate_up.packed, blk.w_gate_up.sf,
                                 gu, self.items, self.bn, 2 * I, st)
        aq = torch.empty(self.R, I, dtype=torch.float8_e4m3fn, device=dev)
        asc = torch.empty(self.R, dtype=torch.float32, device=dev)
        ext().ep_silu_items(gu, self.items, self.bn, aq, asc)
        y = torch.empty(self.R, H, dtype=torch.bfloat16, device=dev)
        ext().mxfp4_grouped_gemm(aq, asc, blk.w_down.packed, blk.w_down.sf, y, self.items,
                                 self.bn, H, st)
        out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
        ext().ep_combine(self.peers, self.rank, self.maxr, self.El, self.maxt, y,
                         w.float().contiguous(), out, st)
        return out

    def header(self) -> dict:
        """Protocol words of this rank's buffer (sequence number, flags, counts) for diagnostics."""
        w = self.buf[:2048].view(torch.int32).cpu()
        return {"epoch": int(w[0]), "arrive": w[16:19].tolist(),
                "disp_done": w[64:64 + self.world].tolist(),
                "comb_done": w[80:80 + self.world].tolist(),
                "nrows": w[96:96 + self.world].tolist(),
                "counts": w[256:256 + self.world * self.El].tolist()}

    def close(self):
        for p in self.opened:
            ext().ipc_close(p)
        self.opened = []
