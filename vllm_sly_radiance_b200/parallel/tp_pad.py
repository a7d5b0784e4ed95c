"""Tensor parallelism at a degree that does not divide the checkpoint geometry.

The Qwen3.8-27B target has 24 q / 4 kv attention heads, 16 GDN key / 48 GDN value heads, a
17408-wide MLP and a 248320-entry vocabulary; none of 4, 16 or 248320 divides by 3, so TP = 3
needs a wider geometry.  It is widened Megatron-style: every sharded section gets zero-weight
dummy heads / channels appended at its end, so contiguous sharding leaves ranks 0..tp-2 all real
and puts the dummies on the last rank, where they compute exact zeros:

* a zero q/k/v attention head gives RMSNorm(0) = 0, RoPE(0) = 0, uniform softmax over a zero V,
  so a zero output, and its output gate multiplies zero; the o_proj columns of dummy heads are
  zero as well;
* a zero GDN head keeps a zero state (k = v = 0), its L2 norms have an epsilon, A_log = 0 is a
  finite decay, and the out_proj columns are zero;
* dummy MLP channels give silu(0) * 0 = 0 and meet zero down_proj columns;
* dummy vocabulary rows are cut from the gathered logits (``ModelConfig.real_vocab_size``).

The GQA ratio (q heads per kv head) and the GDN value/key head ratio are part of the trained
weights, so padding widens kv heads and GDN key heads and derives q / value heads from them.

Reference behaviour: ``radiance_tp3pad.py:1-60`` (geometry and zero-output argument),
``:236`` (fill rules), ``:270`` (config widening), ``:376`` (weight padding around the loader).
Here the widening is a ``ModelConfig`` transform plus a weight-source wrapper that the layer
constructors read through, so random-init and checkpoint weights take the same path.
"""
from __future__ import annotations

import dataclasses
import math

import torch

from ..config import ModelConfig
from ..models.weights import WeightT, cat_rows, slice_rows
from ..quant.mxfp4 import MXFP4Weight

MLP_ALIGN = 64      # per-rank MLP width stays a multiple of 64 (vector widths, MX scale groups)
VOCAB_ALIGN = 64    # per-rank vocabulary shard stays a multiple of 64


def _up(n: int, m: int) -> int:
    return (n + m - 1) // m * m


def needs_padding(cfg: ModelConfig, tp: int) -> bool:
    return padded_config(cfg, tp) != cfg


def padded_config(cfg: ModelConfig, tp: int) -> ModelConfig:
    """The smallest widening of ``cfg`` that every tensor-parallel shard of size ``tp`` divides.

    kv heads that ``tp`` divides, or that divide ``tp`` (replicated kv heads), stay as they are."""
    if tp <= 1:
        return cfg
    ch = {}
    Hq, Hkv = cfg.num_q_heads, cfg.num_kv_heads
    if Hkv % tp != 0 and tp % Hkv != 0:
        gqa = Hq // Hkv
        ch["num_kv_heads"] = _up(Hkv, tp)
        ch["num_q_heads"] = ch["num_kv_heads"] * gqa
    elif Hq % tp != 0:
        raise ValueError(f"q heads {Hq} do not divide by tp={tp} (kv heads {Hkv})")
    Hk, Hv = cfg.gdn_num_k_heads, cfg.gdn_num_v_heads
    if Hk % tp != 0:
        ratio = Hv // Hk
        ch["gdn_num_k_heads"] = _up(Hk, tp)
        ch["gdn_num_v_heads"] = ch["gdn_num_k_heads"] * ratio
    if not cfg.is_moe:
        I = cfg.intermediate_size
        if I % tp != 0 or (I // tp) % MLP_ALIGN != 0:
            ch["intermediate_size"] = _up(I, tp * MLP_ALIGN)
    elif cfg.moe_intermediate_size % tp or cfg.shared_expert_intermediate_size % tp:
        raise ValueError("MoE expert widths that do not divide by tp are not padded")
    V = cfg.vocab_size
    if V % tp != 0:
        ch["vocab_size"] = _up(V, tp * VOCAB_ALIGN)
        ch["real_vocab_size"] = cfg.logical_vocab_size
    return dataclasses.replace(cfg, **ch) if ch else cfg


def _zero_rows(like: WeightT, n: int, K: int) -> WeightT:
    if isinstance(like, MXFP4Weight):
        return MXFP4Weight.zeros(n, K, like.fmt, like.packed.device)
    return torch.zeros(n, K, dtype=like.dtype, device=like.device)


def _pad_sections_rows(w: WeightT, real: list[int], padded: list[int]) -> WeightT:
    """Rows of a merged weight made of sections: each section gets zero rows appended."""
    parts, off = [], 0
    K = w.K if isinstance(w, MXFP4Weight) else w.shape[1]
    for n, m in zip(real, padded):
        parts.append(slice_rows(w, off, n))
        if m > n:
            parts.append(_zero_rows(w, m - n, K))
        off += n
    return cat_rows(parts) if len(parts) > 1 else parts[0]


def _pad_cols(w: WeightT, K_new: int) -> WeightT:
    """Zero input features appended (dummy heads / channels of a row-parallel linear).  The MXFP4
    scale of a zero block is 2^0 (any finite scale gives zero; 0xFF would be NaN)."""
    if isinstance(w, MXFP4Weight):
        return w.pad_cols(K_new)
    if K_new == w.shape[1]:
        return w
    return torch.cat([w, torch.zeros(w.shape[0], K_new - w.shape[1], dtype=w.dtype,
                                     device=w.device)], 1)


def _pad_vec(t: torch.Tensor, sections_real: list[int], sections_pad: list[int]) -> torch.Tensor:
    """Dim-0 sections of a tensor (conv weights, per-head gate parameters) padded with zeros."""
    parts, off = [], 0
    for n, m in zip(sections_real, sections_pad):
        parts.append(t[off:off + n])
        if m > n:
            parts.append(torch.zeros((m - n,) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device))
        off += n
    return torch.cat(parts, 0)


class PaddedWeights:
    """Weight source in the padded geometry over a source in the real one.

    The layer constructors ask for tensors by name with padded shapes; this wrapper asks the inner
    source for the real shape and appends the zero sections.  Names follow the model's own
    (``layers.{i}.{in_proj,conv_w,A_log,dt_bias,out_proj,qkv,o_proj,gate_up,down}``, ``embed``,
    ``lm_head``); expert weights and everything unsharded pass through."""

    def __init__(self, inner, real: ModelConfig, padded: ModelConfig):
        self.inner, self.r, self.p = inner, real, padded
        self.cfg = padded
        self.device = getattr(inner, "device", None)

    def has(self, name: str) -> bool:
        return self.inner.has(name)

    @staticmethod
    def _gdn_in(c: ModelConfig) -> list[int]:
        return [c.gdn_key_dim, c.gdn_key_dim, c.gdn_value_dim, c.gdn_value_dim,
                c.gdn_num_v_heads, c.gdn_num_v_heads]

    @staticmethod
    def _qkv(c: ModelConfig) -> list[int]:
        qd = c.num_q_heads * c.head_dim * (2 if c.attn_output_gate else 1)
        return [qd, c.num_kv_heads * c.head_dim, c.num_kv_heads * c.head_dim]

    def linear(self, name: str, N: int, K: int) -> WeightT:
        r, p = self.r, self.p
        leaf = name.rsplit(".", 1)[-1]
        if ".experts." in name or ".shared." in name:
            return self.inner.linear(name, N, K)
        if leaf == "in_proj":
            w = self.inner.linear(name, r.gdn_in_proj_dim, K)
            return _pad_sections_rows(w, self._gdn_in(r), self._gdn_in(p))
        if leaf == "qkv":
            w = self.inner.linear(name, r.qkv_proj_dim, K)
            return _pad_sections_rows(w, self._qkv(r), self._qkv(p))
        if leaf == "gate_up":
            I, Ip = r.intermediate_size, p.intermediate_size
            return _pad_sections_rows(self.inner.linear(name, 2 * I, K), [I, I], [Ip, Ip])
        if leaf == "out_proj":
            return _pad_cols(self.inner.linear(name, N, r.gdn_value_dim), K)
        if leaf == "o_proj":
            return _pad_cols(self.inner.linear(name, N, r.num_q_heads * r.head_dim), K)
        if leaf == "down":
            return _pad_cols(self.inner.linear(name, N, r.intermediate_size), K)
        if leaf == "lm_head":
            w = self.inner.linear(name, r.vocab_size, K)
            return _pad_sections_rows(w, [r.vocab_size], [p.vocab_size])
        return self.inner.linear(name, N, K)

    def tensor(self, name: str, shape, kind: str = "norm") -> torch.Tensor:
        r, p = self.r, self.p
        leaf = name.rsplit(".", 1)[-1]
        if leaf == "conv_w":
            t = self.inner.tensor(name, (r.gdn_conv_dim, shape[1]), kind)
            return _pad_vec(t, [r.gdn_key_dim, r.gdn_key_dim, r.gdn_value_dim],
                            [p.gdn_key_dim, p.gdn_key_dim, p.gdn_value_dim])
        if leaf in ("A_log", "dt_bias"):
            t = self.inner.tensor(name, (r.gdn_num_v_heads,), kind)
            return _pad_vec(t, [r.gdn_num_v_heads], [p.gdn_num_v_heads])
        if leaf == "embed":
            t = self.inner.tensor(name, (r.vocab_size, shape[1]), kind)
            return _pad_vec(t, [r.vocab_size], [p.vocab_size])
        return self.inner.tensor(name, shape, kind)


def pad_summary(real: ModelConfig, padded: ModelConfig, tp: int) -> dict:
    """Geometry table (real -> padded, per rank) for logs."""
    keys = ["num_q_heads", "num_kv_heads", "gdn_num_k_heads", "gdn_num_v_heads",
            "intermediate_size", "vocab_size"]
    out = {}
    for k in keys:
        a, b = getattr(real, k), getattr(padded, k)
        out[k] = (a, b, b // tp if b % tp == 0 else math.nan)
    return out
