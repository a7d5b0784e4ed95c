"""Weight providers: random init (benchmarks, tests) or checkpoints (``quant/loaders.py``).

The model asks for tensors by canonical name, always in this engine's layout (full, unsharded):

  embed [V,H]  lm_head [V,H]  final_norm [H]
  layers.{i}.ln1 / ln2 [H]
  GDN  : in_proj [2kd+2vd+2Hv, H] as [q|k|v|z|b|a],  conv_w [2kd+vd, W],  A_log [Hv],
         dt_bias [Hv],  norm_w [dv],  out_proj [H, vd]
  ATTN : qkv [Hq*2hd + 2Hkv*hd, H] as [q0,gate0,q1,gate1,...|k|v],  q_norm/k_norm [hd],
         o_proj [H, Hq*hd]
  MLP  : gate_up [2I, H] as [gate|up],  down [H, I]
  MoE  : router [E, H],  experts.{e}.gate_up / down,  shared.gate_up / down,  shared_gate [1, H]

Linear weights come back either as float tensors (quantized by the model at load) or as
``MXFP4Weight`` (pre-quantized checkpoints)."""
from __future__ import annotations

from typing import Optional, Union

import zlib

import torch

from ..config import ModelConfig
from ..quant.mxfp4 import MXFP4Weight

WeightT = Union[torch.Tensor, MXFP4Weight]


class RandomWeights:
    """N(0, init_std) linears, small-noise norms, GDN gate parameters in their usual ranges.

    Every tensor is drawn from its own generator seeded by (seed, name), so a tensor's values do
    not depend on which other tensors a rank asks for (an expert-parallel rank draws only its own
    experts and still holds exactly the single-process model's values for them)."""

    def __init__(self, cfg: ModelConfig, seed: int, device):
        self.cfg = cfg
        self.device = torch.device(device)
        self.seed = seed

    def _gen(self, name: str) -> torch.Generator:
        g = torch.Generator(device=self.device)
        g.manual_seed((self.seed * 1000003 + zlib.crc32(name.encode())) & 0x7FFFFFFFFFFFFFFF)
        return g

    def linear(self, name: str, N: int, K: int) -> WeightT:
        return torch.randn(N, K, generator=self._gen(name), device=self.device) * self.cfg.init_std

    def tensor(self, name: str, shape, kind: str = "norm") -> torch.Tensor:
        g, d = self._gen(name), self.device
        if kind == "norm":             # Gemma (1+w) norms
            return (0.02 * torch.randn(*shape, generator=g, device=d)).to(torch.bfloat16)
        if kind == "norm_plain":       # plain-weight norm (GDN gated norm)
            return (1 + 0.02 * torch.randn(*shape, generator=g, device=d)).to(torch.bfloat16)
        if kind == "conv":
            return (torch.rand(*shape, generator=g, device=d) - 0.5).to(torch.bfloat16)
        if kind == "A_log":
            return torch.log(torch.rand(*shape, generator=g, device=d) * 15 + 1).float()
        if kind == "dt_bias":
            return (0.1 * torch.randn(*shape, generator=g, device=d)).float()
        if kind == "embed":
            return (torch.randn(*shape, generator=g, device=d) * self.cfg.init_std).to(torch.bfloat16)
        if kind == "codebook":
            return (torch.randn(*shape, generator=g, device=d) * 0.1).to(torch.bfloat16)
        if kind == "linear_bf16":
            return (torch.randn(*shape, generator=g, device=d) * self.cfg.init_std).to(torch.bfloat16)
        raise ValueError(kind)

    def has(self, name: str) -> bool:
        return True


# quantization names of the block-scaled (tcgen05 kind::mxf8f6f4) weight formats
MX_QUANTS = {"mxfp4": "e2m1", "mxfp6": "e2m3", "mxfp8": "e4m3"}


class MXCastWeights:
    """Weight source that returns every linear in one MX element type: float linears are
    quantised to it, MX linears of another type are re-quantised (an MXFP4 checkpoint served as
    MXFP8 keeps its values: e2m1 x 2^s is exact in e4m3 x 2^s').  ``skip`` names linears left as
    they are (an lm_head with its own format)."""

    def __init__(self, inner, fmt: str, skip=()):
        self.inner, self.fmt, self.skip = inner, fmt, set(skip)
        self.cfg = inner.cfg
        self.device = getattr(inner, "device", None)

    def linear(self, name: str, N: int, K: int) -> WeightT:
        w = self.inner.linear(name, N, K)
        if name in self.skip or K % 32:
            return w
        if isinstance(w, MXFP4Weight):
            if w.fmt == self.fmt:
                return w
            w = w.dequantize()
        elif not isinstance(w, torch.Tensor):
            return w                                   # other packed formats (int4) as stored
        return MXFP4Weight.from_float(w.float(), self.fmt)

    def __getattr__(self, item):
        return getattr(self.inner, item)


def _is_q(w) -> bool:
    from ..quant.int4 import Int4Weight
    return isinstance(w, (MXFP4Weight, Int4Weight))


def slice_rows(w: WeightT, start: int, length: int) -> WeightT:
    if _is_q(w):
        return w.narrow_rows(start, length)
    return w[start:start + length]


def slice_cols(w: WeightT, start: int, length: int) -> WeightT:
    if _is_q(w):
        return w.narrow_cols(start, length)
    return w[:, start:start + length].contiguous()


def pad_rows(w: WeightT, multiple: int) -> WeightT:
    """Append zero output rows so the row count is a multiple of `multiple` (keeps the row stride
    of the layer's output 16-byte aligned for the vectorised consumers)."""
    n = w.N if _is_q(w) else w.shape[0]
    pad = (-n) % multiple
    if pad == 0:
        return w
    from ..quant.int4 import Int4Weight
    if isinstance(w, Int4Weight):
        z = Int4Weight.from_float(torch.zeros(pad, w.K))
        return cat_rows([w, z])
    if isinstance(w, MXFP4Weight):
        z = MXFP4Weight.zeros(pad, w.K, w.fmt, w.packed.device)
        return cat_rows([w, z])
    return torch.cat([w, torch.zeros(pad, w.shape[1], dtype=w.dtype, device=w.device)], 0)


def cat_rows(ws: list) -> WeightT:
    from ..quant.int4 import Int4Weight
    if isinstance(ws[0], MXFP4Weight):
        from ..quant.mxfp4 import cat_rows as cr
        return cr(ws)
    if isinstance(ws[0], Int4Weight):
        from ..quant.int4 import cat_rows as ci
        return ci(ws)
    return torch.cat(ws, 0)
