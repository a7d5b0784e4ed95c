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

    def dispatch_combine(self, blk, xb, qs, ids, w):
        q, s = qs
        if q is None or blk.w_gate_up is None:
            raise RuntimeError("the NVLink EP transport needs W4A8 (mxfp4) experts")
        T, K = ids.shape
        if T > self.maxt:
            raise RuntimeError(f"{T} tokens exceed the EP transport capacity {self.maxt} per call")
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
