"""Symmetric peer memory for the NVLink collectives (``csrc/comm.cu``).

Each rank allocates device buffers (sequence header + two parity data halves), exports CUDA
IPC handles, and opens every peer's handle (exchange over the process group as a CPU
all_gather_object, like the reference's handle exchange ``radiance_allreduce.py:139-160``).
Only plain peer loads/stores touch these buffers."""
from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Optional

import torch

from ..ops._ext import ext
from ..ops.kernels import _empty, status_word

PUSH_MAX_ROWS = 64           # decode / verify batches use the GEMM-fused path
PUSH_MAX_HIDDEN = 10240


@dataclass
class PushedPartial:
    """Stand-in for the output of a row-parallel GEMM whose tiles were pushed from its epilogue:
    into every rank's receive buffer (kind "ll", decode: ``mxfp4_gemm_push``) or into the owners'
    reduce-scatter slots of the two-shot all-reduce (kind "rs", prefill: ``mxfp4_gemm_rs``).  The
    all-reduce call that consumes it only runs the remaining half."""
    M: int
    H: int
    expected: int
    device: torch.device
    kind: str = "ll"

    @property
    def shape(self):
        return (self.M, self.H)


TS_MIN_ROWS = 257           # prefill-sized all-reduces: two-shot NVLink (comm_ts.cu)
TS_MAX_ROWS = 4096          # the scheduler's chunk (max_num_batched_tokens) bounds a prefill step
TS_MAX_HIDDEN = 8192


class FusedComm:
    def __init__(self, rank: int, world: int, group, slot_bytes: int = 32 << 20,
                 ts_rows: int = TS_MAX_ROWS, ts_hidden: int = TS_MAX_HIDDEN):
        import torch.distributed as dist
        self.rank, self.world = rank, world
        self.slot_bytes = slot_bytes
        hdr = ext().symm_header_bytes()
        self.buf = torch.zeros(hdr + 2 * slot_bytes, dtype=torch.uint8, device="cuda")
        self.opened = []
        self.ptrs = self._exchange(self.buf, group)
        # receive buffers of the GEMM-fused all-reduce (row-parallel GEMM pushes its tiles)
        self.push_enabled = os.environ.get("RADIANCE_GEMM_PUSH", "1") != "0"
        self.push_ptrs = None
        if self.push_enabled:
            nbytes = ext().push_buffer_bytes(world, PUSH_MAX_ROWS, PUSH_MAX_HIDDEN)
            self.push_half_words = world * PUSH_MAX_ROWS * (PUSH_MAX_HIDDEN // 2)
            self.push_buf = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
            self.push_ptrs = self._exchange(self.push_buf, group)
        # two-shot all-reduce (reduce-scatter + all-gather pushes) for prefill chunks, with the
        # row-parallel GEMM pushing its rows to their owners from its epilogue: opt-in
        # (RADIANCE_TS=1).  Measured on 2 B200s (27B hybrid, TP2 prefill): 30.8k tok/s at 1.5k
        # tokens and 34.0k at 11.8k with it, 39.7k and 43.2k with NCCL's all-reduce for chunks
        # over 256 rows, so prefill-sized rows go to NCCL by default.  Decode rows keep the
        # GEMM-fused push (246 vs 155 tok/s against NCCL).
        self.ts_enabled = os.environ.get("RADIANCE_TS", "0") == "1"
        self.ts_ptrs = None
        if self.ts_enabled:
            self.ts_bytes = ext().ts_buffer_bytes(ts_rows, ts_hidden)
            self.ts_buf = torch.zeros(self.ts_bytes, dtype=torch.uint8, device="cuda")
            self.ts_ptrs = self._exchange(self.ts_buf, group)
        self.ts_calls = 0
        dist.barrier(group=group)
        self.calls = 0
        self.fallbacks = 0
        self.pushes = 0

    def _exchange(self, buf: torch.Tensor, group) -> list:
        """IPC-map every rank's `buf`; returns the device pointers, own one at `rank`."""
        import torch.distributed as dist
        h = ext().ipc_handle(buf)
        handles = [None] * self.world
        dist.all_gather_object(handles, h.numpy().tobytes(), group=group)
        ptrs = []
        for r in range(self.world):
            if r == self.rank:
                ptrs.append(buf.data_ptr())
            else:
                p = ext().ipc_open(torch.frombuffer(bytearray(handles[r]), dtype=torch.uint8))
                ptrs.append(p)
                self.opened.append(p)
        return ptrs

    # ---- GEMM-fused all-reduce ----
    def ts_fits(self, M: int, H: int) -> bool:
        return (self.ts_ptrs is not None and H % 8 == 0 and H <= 10240
                and ext().ts_buffer_bytes(M, H) <= self.ts_bytes)

    def can_push(self, M: int, N: int) -> bool:
        if M > PUSH_MAX_ROWS:
            return M >= TS_MIN_ROWS and self.ts_fits(M, N)
        return (self.push_ptrs is not None and 0 < M <= PUSH_MAX_ROWS and N % 8 == 0
                and N <= PUSH_MAX_HIDDEN)

    def gemm_push(self, q, s, w) -> PushedPartial:
        """Row-parallel W4A8 GEMM whose output tiles go straight into every rank's receive
        buffer (decode) or into the owners' reduce-scatter slots (prefill); the following
        all-reduce call runs the rest."""
        M = q.shape[0]
        if M > PUSH_MAX_ROWS:
            per = ext().ts_rows_per_rank(M, self.world)
            exp = ext().mxfp4_gemm_rs(q, s, w.packed, w.sf, self.ts_ptrs, self.rank, per,
                                      status_word(q.device))
            self.pushes += 1
            return PushedPartial(M, w.N, int(exp), q.device, "rs")
        from ..models.layers import GEMV_ON
        from ..ops import kernels as K
        if GEMV_ON and q.shape[0] <= K.GEMV_MAX_ROWS:
            exp = K.mxfp4_gemv_push(q, s, w, self.push_ptrs, self.rank, self.push_half_words)
        else:
            exp = ext().mxfp4_gemm_push(q, s, w.packed, w.sf, self.push_ptrs, self.rank,
                                        self.push_half_words, status_word(q.device))
        self.pushes += 1
        return PushedPartial(q.shape[0], w.N, int(exp), q.device)

    def _recv(self, x: PushedPartial, out, residual, weight, eps, res_out, q, s):
        e = _empty(x.device)
        ext().push_allreduce_recv(self.push_ptrs, self.rank, x.M, x.H, self.push_half_words,
                                  out if out is not None else e,
                                  residual if residual is not None else e,
                                  weight if weight is not None else e, eps,
                                  res_out if res_out is not None else e,
                                  q if q is not None else e, s if s is not None else e,
                                  min(64, x.M), status_word(x.device))

    @staticmethod
    def create(rank, world, group) -> Optional["FusedComm"]:
        if world < 2 or world > 8:
            return None
        return FusedComm(rank, world, group)

    def fits(self, x: torch.Tensor) -> bool:
        # every rank's rows land in each buffer as 8-byte words carrying two bf16
        return x.dim() == 2 and x.dtype == torch.bfloat16 and x.shape[1] % 8 == 0 and \
            x.shape[1] <= 10240 and self.world * x.numel() * 4 <= self.slot_bytes and \
            x.is_contiguous()

    def _ts(self, x, M, H, out, residual, weight, eps, res_out, q, s):
        """Two-shot all-reduce of x (a bf16 partial, or a PushedPartial of kind "rs")."""
        e = _empty(out.device if out is not None else q.device)
        pushed = isinstance(x, PushedPartial)
        self.ts_calls += 1
        ext().ts_allreduce(self.ts_ptrs, self.rank, M, H, self.ts_bytes, e if pushed else x,
                           pushed, x.expected if pushed else 0,
                           out if out is not None else e, residual if residual is not None else e,
                           weight if weight is not None else e, eps,
                           res_out if res_out is not None else e, q if q is not None else e,
                           s if s is not None else e,
                           status_word(out.device if out is not None else q.device))

    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        if isinstance(x, PushedPartial):
            out = torch.empty(x.M, x.H, dtype=torch.bfloat16, device=x.device)
            if x.kind == "rs":
                self._ts(x, x.M, x.H, out, None, None, 0.0, None, None, None)
            else:
                self._recv(x, out, None, None, 0.0, None, None, None)
            return out
        if (x.dim() == 2 and x.shape[0] >= TS_MIN_ROWS and x.dtype == torch.bfloat16
                and x.is_contiguous() and self.ts_fits(x.shape[0], x.shape[1])):
            out = torch.empty_like(x)
            self._ts(x, x.shape[0], x.shape[1], out, None, None, 0.0, None, None, None)
            return out
        if not self.fits(x) or x.shape[0] > 256:
            import torch.distributed as dist
            self.fallbacks += 1
            dist.all_reduce(x)
            return x
        self.calls += 1
        out = torch.empty_like(x)
        e = _empty(x.device)
        ext().allreduce_oneshot(self.ptrs, self.rank, x, self.slot_bytes, out, e, e, 0.0, e, e, e,
                                min(64, x.shape[0]), status_word(x.device))
        return out

    def all_reduce_add_rms_quant(self, x, residual, weight, eps):
        """Fused: all-reduce(x) + residual -> residual_out; Gemma RMSNorm + e4m3 quant."""
        M, H = x.shape
        if isinstance(x, PushedPartial):
            q = torch.empty(M, H, dtype=torch.float8_e4m3fn, device=x.device)
            s = torch.empty(M, dtype=torch.float32, device=x.device)
            r = torch.empty(M, H, dtype=torch.bfloat16, device=x.device)
            if x.kind == "rs":
                self._ts(x, M, H, None, residual, weight, eps, r, q, s)
            else:
                self._recv(x, None, residual, weight, eps, r, q, s)
            return q, s, r
        if (M >= TS_MIN_ROWS and x.dtype == torch.bfloat16 and x.is_contiguous()
                and self.ts_fits(M, H)):
            q = torch.empty(M, H, dtype=torch.float8_e4m3fn, device=x.device)
            s = torch.empty(M, dtype=torch.float32, device=x.device)
            r = torch.empty_like(x)
            self._ts(x, M, H, None, residual, weight, eps, r, q, s)
            return q, s, r
        if not self.fits(x) or M > 256:
            from ..ops import kernels as K
            return K.add_rms_quant(self.all_reduce(x), residual, weight, eps)
        q = torch.empty(M, H, dtype=torch.float8_e4m3fn, device=x.device)
        s = torch.empty(M, dtype=torch.float32, device=x.device)
        r = torch.empty_like(x)
        e = _empty(x.device)
        ext().allreduce_oneshot(self.ptrs, self.rank, x, self.slot_bytes, e, residual, weight, eps,
                                r, q, s, min(64, M), status_word(x.device))
        return q, s, r

    def close(self):
        for p in self.opened:
            ext().ipc_close(p)
        self.opened = []
