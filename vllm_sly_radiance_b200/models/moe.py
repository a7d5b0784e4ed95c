"""Mixture-of-experts block (256 routed experts, softmax top-8 with
renormalised weights, one shared expert behind a sigmoid gate; Qwen3-Next MoE semantics, served
TP-sharded by the reference through vLLM fused_moe, ``moe-configs/E=256,...``).

Routed experts run as ONE grouped W4A8 launch per projection: tokens are dispatched into an
expert-sorted buffer, a work table lists (expert, row tile) pairs, and the tcgen05 grouped GEMM
(``mxfp4_grouped_gemm`` in ``csrc/mxfp4_gemm.cu``) reads each expert's MXFP4 weights from one
stacked tensor.

Expert parallelism: the tensor-parallel ranks already hold every token of the step (attention is
head-sharded), so each of the `size` ranks owns E/size experts and a 1/size slice of the shared
expert, evaluates them for all tokens, and its output is a partial sum.  Dispatch is then a local
selection and the combine is the all-reduce the model runs after every MLP, which on NVLink is
the fused all-reduce + residual add + RMSNorm + e4m3 kernel (``csrc/comm.cu``).
"""
from __future__ import annotations

from typing import Optional

import torch

from ..config import ModelConfig
from ..ops import kernels as K
from ..quant.mxfp4 import MXFP4Weight, cat_rows
from .layers import Linear


class MoEBlock:
    def __init__(self, cfg: ModelConfig, tp, quant: str, W, prefix: str, ep=None):
        H = cfg.hidden_size
        E = cfg.num_experts
        I = cfg.moe_intermediate_size
        self.cfg = cfg
        self.E, self.H, self.I = E, H, I
        self.top_k = cfg.num_experts_per_tok
        self.quant = quant
        # experts owned by this rank: expert parallel over the tensor-parallel group (tokens
        # replicated, partial sums all-reduced), or over a data-parallel group `ep` (tokens
        # local to each rank, rows exchanged by the EP transport's dispatch / combine)
        self.ep = ep.transport if ep is not None else None
        size = ep.size if ep is not None else (tp.size if tp is not None else 1)
        rank = ep.rank if ep is not None else (tp.rank if tp is not None else 0)
        assert E % size == 0, (E, size)
        self.e0, self.e_local = rank * (E // size), E // size
        router = W.tensor(prefix + "router", (E, H), "linear_bf16") if hasattr(W, "tensor") else None
        self.router = router.to(torch.bfloat16).contiguous()
        gu, dn = [], []
        for e in range(self.e0, self.e0 + self.e_local):
            gu.append(W.linear(prefix + f"experts.{e}.gate_up", 2 * I, H))
            dn.append(W.linear(prefix + f"experts.{e}.down", H, I))
        if quant == "mxfp4":
            to_mx = lambda w: w if isinstance(w, MXFP4Weight) else MXFP4Weight.from_float(w)
            self.w_gate_up = cat_rows([to_mx(w) for w in gu])      # [E_local*2I, H/2] stacked
            self.w_down = cat_rows([to_mx(w) for w in dn])         # [E_local*H, I/2]
            self.dense_gu = self.dense_dn = None
        else:
            deq = lambda w: (w.dequantize() if isinstance(w, MXFP4Weight) else w).to(torch.bfloat16)
            self.dense_gu = torch.stack([deq(w) for w in gu])      # [E_local, 2I, H]
            self.dense_dn = torch.stack([deq(w) for w in dn])      # [E_local, H, I]
            self.w_gate_up = self.w_down = None
        del gu, dn
        Is = cfg.shared_expert_intermediate_size
        from .hybrid import _cat_sections, make_linear
        from .weights import slice_cols
        wsg = W.linear(prefix + "shared.gate_up", 2 * Is, H)
        self.shared_gate_up = make_linear(_cat_sections(wsg, [Is, Is], tp), quant, "sh_gate_up")
        wsd = W.linear(prefix + "shared.down", H, Is)
        s0, per = tp.shard(Is)
        self.shared_down = make_linear(slice_cols(wsd, s0, per), quant, "sh_down")
        self.shared_gate = W.tensor(prefix + "shared_gate", (1, H), "linear_bf16").to(torch.bfloat16)

    def to(self, device):
        for k, v in list(vars(self).items()):
            if isinstance(v, torch.Tensor):
                setattr(self, k, v.to(device))
            elif isinstance(v, MXFP4Weight):
                setattr(self, k, v.to(device))
            elif isinstance(v, Linear):
                v.to(device)
        return self

    # ------------------------------------------------------------------------------------------
    def route(self, x_bf16: torch.Tensor):
        """softmax over all experts, top-k, renormalised weights -> (ids [T,k], weights [T,k])."""
        logits = x_bf16.float() @ self.router.float().t()
        p = torch.softmax(logits, -1)
        w, ids = torch.topk(p, self.top_k, dim=-1)
        w = w / w.sum(-1, keepdim=True)
        return ids, w

    def forward(self, x):
        """x: (q, scale) from the fused producer or bf16 [T, H] -> bf16 [T, H]."""
        if isinstance(x, tuple):
            q, s = x
            xb = (q.float() * s[:, None]).to(torch.bfloat16)
        else:
            xb = x
            q, s = K.quant_fp8(x) if self.quant == "mxfp4" else (None, None)
        T = xb.shape[0]
        ids, w = self.route(xb)
        routed = self._experts(xb, (q, s), ids, w)
        sh = self.shared_down(K.silu_mul_quant(self.shared_gate_up((q, s) if q is not None else xb))
                              if self.quant == "mxfp4" else K.silu_mul(self.shared_gate_up(xb)))
        gate = torch.sigmoid(xb.float() @ self.shared_gate.float().t())
        return (routed.float() + gate * sh.float()).to(torch.bfloat16)

    def _experts(self, xb, qs, ids, w):
        if self.ep is not None:
            return self.ep.dispatch_combine(self, xb, qs, ids, w)
        return self.local_experts(xb, qs, ids, w)

    def expert_rows(self, q, s, xb, le):
        """Unweighted outputs of this rank's experts for rows routed to them: row i goes through
        local expert le[i] (any order; rows of one expert are grouped internally)."""
        n = le.shape[0]
        dev = le.device
        if n == 0:
            return torch.zeros(0, self.H, dtype=torch.bfloat16, device=dev)
        order = torch.argsort(le, stable=True)
        counts = torch.bincount(le, minlength=self.e_local)
        y = torch.empty(n, self.H, dtype=torch.bfloat16, device=dev)
        if self.w_gate_up is not None and le.is_cuda:
            y[order] = K.moe_grouped_mlp(q[order], s[order], counts, self.w_gate_up, self.w_down,
                                         self.I, self.H)
            return y
        starts = torch.cumsum(counts, 0) - counts
        for e in range(self.e_local):
            c = int(counts[e])
            if c == 0:
                continue
            idx = order[int(starts[e]):int(starts[e]) + c]
            if self.w_gate_up is not None:
                gsl = slice(e * 2 * self.I, (e + 1) * 2 * self.I)
                dsl = slice(e * self.H, (e + 1) * self.H)
                gu = K.mxfp4_gemm(q[idx], s[idx], self.w_gate_up.packed[gsl], None,
                                  self.w_gate_up.scales[gsl], 2 * self.I, fmt=self.w_gate_up.fmt)
                a = K.silu_mul_quant(gu)
                y[idx] = K.mxfp4_gemm(a[0], a[1], self.w_down.packed[dsl], None,
                                      self.w_down.scales[dsl], self.H, fmt=self.w_down.fmt)
            else:
                gu = xb[idx].float() @ self.dense_gu[e].float().t()
                a = K.silu_mul(gu.to(torch.bfloat16)).float()
                y[idx] = (a @ self.dense_dn[e].float().t()).to(torch.bfloat16)
        return y

    def local_experts(self, xb, qs, ids, w):
        """Experts [e0, e0+e_local) applied to every (token, slot) routed to them; the other
        slots contribute zero (they belong to another rank's experts)."""
        T, k = ids.shape
        dev = xb.device
        flat_e = ids.reshape(-1) - self.e0
        flat_t = torch.arange(T, device=dev).repeat_interleave(k)
        flat_w = w.reshape(-1)
        own = (flat_e >= 0) & (flat_e < self.e_local)
        if self.w_gate_up is not None and xb.is_cuda:
            # fixed shapes, no host sync (CUDA-graph safe): foreign slots sort to the end and
            # are not covered by any work item
            key = torch.where(own, flat_e, torch.full_like(flat_e, self.e_local))
            order = torch.argsort(key, stable=True)
            st = flat_t[order]
            sw = torch.where(own[order], flat_w[order], torch.zeros_like(flat_w))
            # scatter-add, not bincount: bincount reads its maximum back to the host, which a
            # CUDA-graph capture of the decode step cannot contain
            counts = torch.zeros(self.e_local + 1, dtype=torch.long, device=dev).scatter_add_(
                0, key, torch.ones_like(key))[:self.e_local]
            q, s = qs
            y = K.moe_grouped_mlp(q[st], s[st], counts, self.w_gate_up, self.w_down, self.I, self.H)
            out = torch.zeros(T, self.H, dtype=torch.float32, device=dev)
            out.index_add_(0, st, y.float() * sw[:, None])
            return out.to(torch.bfloat16)
        out = torch.zeros(T, self.H, dtype=torch.float32, device=dev)
        flat_e, flat_t, flat_w = flat_e[own], flat_t[own], flat_w[own]
        if flat_e.numel() == 0:
            return out.to(torch.bfloat16)
        order = torch.argsort(flat_e, stable=True)
        se, st, sw = flat_e[order], flat_t[order], flat_w[order]
        counts = torch.bincount(se, minlength=self.e_local)
        y = torch.empty(se.shape[0], self.H, dtype=torch.float32, device=dev)
        starts = torch.cumsum(counts, 0) - counts
        for e in range(self.e_local):
            c = int(counts[e])
            if c == 0:
                continue
            r0 = int(starts[e])
            rows = xb[st[r0:r0 + c]]
            if self.w_gate_up is not None:     # CPU W4A8 oracle
                qq, ss = qs[0][st[r0:r0 + c]], qs[1][st[r0:r0 + c]]
                gsl = slice(e * 2 * self.I, (e + 1) * 2 * self.I)
                dsl = slice(e * self.H, (e + 1) * self.H)
                gu = K.mxfp4_gemm(qq, ss, self.w_gate_up.packed[gsl], None,
                                  self.w_gate_up.scales[gsl], 2 * self.I, fmt=self.w_gate_up.fmt)
                a = K.silu_mul_quant(gu)
                y[r0:r0 + c] = K.mxfp4_gemm(a[0], a[1], self.w_down.packed[dsl], None,
                                            self.w_down.scales[dsl], self.H, fmt=self.w_down.fmt).float()
            else:
                gu = rows.float() @ self.dense_gu[e].float().t()
                a = K.silu_mul(gu.to(torch.bfloat16)).float()
                y[r0:r0 + c] = a @ self.dense_dn[e].float().t()
        out.index_add_(0, st, y.float() * sw[:, None])
        return out.to(torch.bfloat16)
