"""Checkpoint loading (safetensors, sharded), mapped onto the engine's canonical weight layout.

Supported per-linear formats (auto-detected from the tensor names next to each weight):
  * bf16 / fp16 / fp32                 ``{p}.weight``                      -> quantized at load
  * MXFP4, compressed-tensors          ``{p}.weight_packed`` u8 [N,K/2] + ``{p}.weight_scale`` u8 [N,K/32]
  * MXFP4, Quark                       ``{p}.weight`` u8 [N,K/2] + ``{p}.weight_scale`` u8 [N,K/32]
  * MXFP6 (E2M3)                      ``weight_packed`` u8 [N,3K/4] (four 6-bit codes per three
                                       bytes, code i at bits 6i of the little-endian 24-bit word)
                                       + ``weight_scale`` u8 [N,K/32] -> MXFP6 as stored
  * BCQ4 (block-clustered tables)      ``weight_packed`` u8 [N,K/2] + ``weight_scale`` u8 table ids
                                       [N,K/32] + ``weight_row_exp`` u8 [N], with a [256, 8] table
                                       file (``bcq_tables.pt``): w = sign * T[id][mag] *
                                       2^(row_exp - 127) -> MXFP8 exactly (each table entry is an
                                       e4m3 value, the row exponent is the block scale); with a
                                       Hadamard-128 checkpoint (weights stored as W R) the rotation
                                       is undone at load (W = W' R^T) and W requantised to MXFP8
  * fp8 block W8A8                     ``weight`` e4m3 [N,K] + ``weight_scale_inv`` fp32
                                       [N/128,K/128] -> dequantised (served as MXFP8 with
                                       ``quantization=mxfp8``)
  * NVFP4 (compressed-tensors/modelopt) ``weight_packed`` + e4m3 ``weight_scale`` [N,K/16] +
                                       ``weight_global_scale`` (divisor) or ``weight_scale_2``
                                       (multiplier) -> requantized to MXFP4 (``radiance_nvfp4.py``
                                       'ocp' exponent mode)
  * INT4 W4A16 g128 (compressed-tensors pack-quantized) ``weight_packed`` i32 [N,K/8] +
                                       ``weight_scale`` [N,K/g] (+ ``weight_zero_point``)
                                       -> kept as int4 for ``quantization=int4`` (the W4A16
                                       kernel), else dequantized (then MXFP4 for W4A8)
  * INT4 GPTQ / AutoRound layout       ``qweight`` i32 [K/8,N] (8 k per word), ``scales``
                                       [K/g,N], ``qzeros`` i32 [K/g,N/8] (8 n per word; stored
                                       zero - 1 unless the config says ``gptq_v2`` /
                                       ``auto_round`` exact zeros) -> the same int4 path

Qwen3-Next naming (HF) and the layout transforms (reference loader behaviour:
``sly/mxfp4/radiance_mxfp4.py:1006-1120``, GDN in_proj merge ``radiance_gdnmerge.py:30-35``):
  * GDN ``in_proj_qkvz`` is grouped per key head ([q_g, k_g, v_g*, z_g*]) and ``in_proj_ba`` per
    key head ([b_g*, a_g*]); both are permuted into the merged [q|k|v|z|b|a] order.
  * attention ``q_proj`` (query+gate interleaved per head), ``k_proj``, ``v_proj`` -> ``qkv``.
  * ``gate_proj`` + ``up_proj`` -> ``gate_up``.
Shards are read tensor by tensor (peak host memory = one tensor, not one shard;
``docs/TECHNICAL.md:773-825``).
"""
from __future__ import annotations

import glob
import json
import os
from typing import Optional

import torch

from ..config import ModelConfig
from .formats import (MX_BITS, int4_g128_dequantize, mxfp4_quantize, nvfp4_to_mxfp4,
                      unpack_nibbles)
from .mxfp4 import MXFP4Weight


def hadamard_rotation(n: int = 128) -> torch.Tensor:
    """R = H_n diag(s) / sqrt(n): Sylvester Hadamard matrix with column signs s drawn as
    ``torch.rand(n) < 0.5 -> -1`` from a seed-0 generator -- the rotation the reference's
    Hadamard-128 checkpoints were written with (``sly/mxfp4/radiance_mxfp4.py:254-272``).
    Orthogonal: R R^T = I."""
    g = torch.Generator().manual_seed(0)
    sgn = torch.where(torch.rand(n, generator=g, dtype=torch.float32) < 0.5, -1.0, 1.0)
    H = torch.ones(1, 1)
    while H.shape[0] < n:
        H = torch.cat([torch.cat([H, H], 1), torch.cat([H, -H], 1)])
    return H * (sgn / n ** 0.5)


def bcq_dequantize(packed: torch.Tensor, ids: torch.Tensor, row_exp: torch.Tensor,
                   table: torch.Tensor) -> torch.Tensor:
    """BCQ4 -> fp32 [N, K]: w = sign * T[id[n, k/32]][code & 7] * 2^(row_exp[n] - 127), code =
    nibble (low nibble = even k), sign = code bit 3 (``ci/check_bcq_all_paths.py:52-58``)."""
    nib = unpack_nibbles(packed).long()
    t = ids.long().repeat_interleave(32, 1)
    mag = table.float()[t, nib & 7]
    return torch.where(nib >= 8, -mag, mag) * torch.exp2(row_exp.float() - 127.0)[:, None]


def bcq_to_mxfp8(packed: torch.Tensor, ids: torch.Tensor, row_exp: torch.Tensor,
                 table: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """BCQ4 -> MXFP8 (e4m3 codes [N, K], UE8M0 scales [N, K/32]) with no rounding: each element
    is a table entry (e4m3-exact) and the block scale is the row's exponent."""
    nib = unpack_nibbles(packed).long()
    t = ids.long().repeat_interleave(32, 1)
    tb = table.float().to(torch.float8_e4m3fn).view(torch.uint8)
    code = tb[t, nib & 7] | ((nib >= 8) & (tb[t, nib & 7] != 0)).to(torch.uint8) << 7
    scales = row_exp.to(torch.uint8)[:, None].expand(-1, ids.shape[1]).contiguous()
    return code.contiguous(), scales


class CheckpointWeights:
    def __init__(self, path: str, cfg: ModelConfig, device="cpu", prefix: str = "model."):
        from safetensors import safe_open
        self.cfg = cfg
        self.device = torch.device(device)
        self.keep_int4 = False         # True: int4 pack-quantized linears load as Int4Weight
        # GPTQ v1 stores zero points minus one; gptq_v2 / auto_round store them exactly
        self.gptq_zero_offset = 1
        files = sorted(glob.glob(os.path.join(path, "*.safetensors")))
        if not files:
            raise FileNotFoundError(f"no .safetensors files under {path}")
        self.index: dict[str, str] = {}
        self._open = {}
        for f in files:
            h = safe_open(f, framework="pt", device="cpu")
            self._open[f] = h
            for k in h.keys():
                self.index[k] = f
        self.prefix = prefix if any(k.startswith(prefix) for k in self.index) else ""
        qc = os.path.join(path, "config.json")
        self.hf_config = json.load(open(qc)) if os.path.exists(qc) else {}
        qcfg = self.hf_config.get("quantization_config", {}) or {}
        # BCQ4 tables ([256, 8] e4m3-exact magnitudes) and the Hadamard-128 flag
        self.bcq_table = None
        for tf in ("bcq_tables.pt", "mcb_tables.pt"):
            if os.path.exists(os.path.join(path, tf)):
                t = torch.load(os.path.join(path, tf), map_location="cpu").float()
                if tuple(t.shape) != (256, 8) or bool((t < 0).any()) or not torch.equal(
                        t.to(torch.float8_e4m3fn).float(), t):
                    raise ValueError(f"{tf}: want [256, 8] e4m3-exact magnitudes")
                self.bcq_table = t
                break
        self.hadamard = int(qcfg.get("hadamard", qcfg.get("radiance_hadamard", 0)) or 0)
        if self.hadamard not in (0, 128):
            raise ValueError(f"hadamard block {self.hadamard}: 0 or 128")
        self.fp8_block = tuple(qcfg.get("weight_block_size", (128, 128)) or (128, 128))
        fmt = str(qcfg.get("checkpoint_format", qcfg.get("packing_format", ""))).lower()
        if fmt in ("gptq_v2", "auto_round", "auto_round:gptq_v2") or \
                str(qcfg.get("quant_method", "")).lower() == "auto-round" and "v1" not in fmt:
            self.gptq_zero_offset = 0

    # ---- raw access ----
    def has(self, key: str) -> bool:
        return key in self.index

    def raw(self, key: str) -> torch.Tensor:
        return self._open[self.index[key]].get_tensor(key)

    def _hf(self, name: str) -> str:
        return self.prefix + name

    def _gptq_int4(self, p: str):
        """GPTQ / AutoRound packing -> canonical int4 (packed [N,K/2], scales, zeros)."""
        from .formats import pack_nibbles
        qw = self.raw(p + ".qweight").contiguous()          # [K/8, N] int32
        sc = self.raw(p + ".scales")                          # [K/g, N]
        K8, N = qw.shape
        K = K8 * 8
        shifts = torch.arange(8, dtype=torch.int32) * 4
        q = ((qw.unsqueeze(1) >> shifts.view(1, 8, 1)) & 0xF).reshape(K, N).t().contiguous()
        G = sc.shape[0]
        if self.has(p + ".qzeros"):
            qz = self.raw(p + ".qzeros").contiguous()         # [K/g, N/8] int32
            z = ((qz.unsqueeze(2) >> shifts.view(1, 1, 8)) & 0xF).reshape(G, -1)[:, :N]
            z = (z + self.gptq_zero_offset) & 0xF       # v1 stores (zero - 1) mod 16
        else:
            z = torch.full((G, N), 8, dtype=torch.int32)
        g = K // G
        packed = pack_nibbles(q.to(torch.uint8))
        zeros = z.t().contiguous().to(torch.uint8)
        scales = sc.t().contiguous().half()
        return packed, scales, zeros, N, K, g

    def _linear_any(self, hf_name: str):
        """Read one HF linear in whatever format it is stored: float tensor, MXFP4Weight or (for
        ``quantization=int4``) Int4Weight."""
        p = hf_name
        if self.has(p + ".qweight"):
            packed, scales, zeros, N, K, g = self._gptq_int4(p)
            if self.keep_int4 and g == 128:
                from .int4 import Int4Weight
                return Int4Weight(packed, scales, zeros, N, K)
            return int4_g128_dequantize(packed, scales.float(), zeros, g)
        if self.has(p + ".weight_packed") or (self.has(p + ".weight") and self.has(p + ".weight_scale")
                                              and self.raw(p + ".weight").dtype == torch.uint8):
            packed = self.raw(p + ".weight_packed") if self.has(p + ".weight_packed") else self.raw(p + ".weight")
            scale = self.raw(p + ".weight_scale")
            if packed.dtype == torch.int32:                     # int4 pack-quantized (8 per int32)
                N = packed.shape[0]
                b = packed.contiguous().view(torch.uint8).view(N, -1)
                K = b.shape[1] * 2
                g = K // scale.shape[1]
                if self.has(p + ".weight_zero_point"):
                    zp = self.raw(p + ".weight_zero_point")
                    zp = zp.view(torch.uint8) if zp.dtype == torch.int32 else zp
                    zp = unpack_nibbles(zp.view(N, -1))[:, :K // g] if zp.dtype == torch.uint8 and zp.shape[1] * 2 == K // g else zp
                else:
                    zp = torch.full((N, K // g), 8, dtype=torch.uint8)
                if self.keep_int4 and g == 128:
                    # served int4 (W4A16 kernel): keep the codes, scales and zero points as stored
                    from .int4 import Int4Weight
                    return Int4Weight(b.contiguous(), scale.half().contiguous(),
                                      zp.to(torch.uint8).contiguous(), N, K)
                w = int4_g128_dequantize(b, scale.float(), zp.to(torch.uint8), g)
                return w
            if scale.dtype == torch.uint8 and self.has(p + ".weight_row_exp"):    # BCQ4
                if self.bcq_table is None:
                    raise ValueError(f"{p}: BCQ4 weights need bcq_tables.pt next to the checkpoint")
                row_exp = self.raw(p + ".weight_row_exp").view(-1)
                if self.hadamard:
                    w = bcq_dequantize(packed, scale, row_exp, self.bcq_table)
                    N, K = w.shape
                    R = hadamard_rotation(self.hadamard)
                    w = (w.view(N, K // self.hadamard, self.hadamard) @ R.t()).view(N, K)
                    return MXFP4Weight.from_float(w, "e4m3")
                code, sc = bcq_to_mxfp8(packed, scale, row_exp, self.bcq_table)
                return MXFP4Weight.from_packed(code, sc, fmt="e4m3")
            if scale.dtype == torch.uint8:                      # MXFP4 / MXFP6 (UE8M0 per 32)
                K = scale.shape[1] * 32
                fmt = {K // 2: "e2m1", 3 * K // 4: "e2m3", K: "e4m3"}.get(packed.shape[1])
                if fmt is None:
                    raise ValueError(f"{p}: packed width {packed.shape[1]} is no MX type of K={K}")
                return MXFP4Weight.from_packed(packed.contiguous(), scale.contiguous(), fmt=fmt)
            if scale.dtype == torch.float8_e4m3fn:             # NVFP4
                if self.has(p + ".weight_global_scale"):
                    gs = 1.0 / self.raw(p + ".weight_global_scale").float()
                elif self.has(p + ".weight_scale_2"):
                    gs = self.raw(p + ".weight_scale_2").float()
                else:
                    gs = torch.tensor(1.0)
                mp, ms = nvfp4_to_mxfp4(packed.contiguous(), scale, gs.reshape(()))
                return MXFP4Weight.from_packed(mp, ms)
            raise ValueError(f"unsupported quantized format for {p}: scale dtype {scale.dtype}")
        w = self.raw(p + ".weight")
        if w.dtype == torch.float8_e4m3fn and self.has(p + ".weight_scale") and \
                self.raw(p + ".weight_scale").dtype == torch.uint8:
            # MXFP8: e4m3 elements with UE8M0 per-32 scales, served as stored
            return MXFP4Weight.from_packed(w.view(torch.uint8).contiguous(),
                                           self.raw(p + ".weight_scale").contiguous(), fmt="e4m3")
        if w.dtype == torch.float8_e4m3fn and self.has(p + ".weight_scale_inv"):
            # fp8 block W8A8: one fp32 scale per (bn x bk) block
            si = self.raw(p + ".weight_scale_inv").float()
            bn, bk = self.fp8_block
            N, K = w.shape
            s = si.repeat_interleave(bn, 0)[:N].repeat_interleave(bk, 1)[:, :K]
            return w.float() * s
        return w.float()

    # ---- provider interface ----
    def linear(self, name: str, N: int, K: int):
        cfg = self.cfg
        parts = name.split(".")
        if name == "lm_head":
            return self._linear_any("lm_head")
        i = int(parts[1])
        leaf = parts[2]
        L = f"layers.{i}."
        if leaf == "in_proj":
            qkvz = self._linear_any(self._hf(L + "linear_attn.in_proj_qkvz"))
            ba = self._linear_any(self._hf(L + "linear_attn.in_proj_ba"))
            return _merge_gdn_in_proj(qkvz, ba, cfg)
        if leaf == "out_proj":
            return self._linear_any(self._hf(L + "linear_attn.out_proj"))
        if leaf == "qkv":
            qs = [self._linear_any(self._hf(L + f"self_attn.{n}_proj")) for n in ("q", "k", "v")]
            return _cat(qs)
        if leaf == "o_proj":
            return self._linear_any(self._hf(L + "self_attn.o_proj"))
        if leaf == "gate_up":
            return _cat([self._linear_any(self._hf(L + "mlp.gate_proj")),
                         self._linear_any(self._hf(L + "mlp.up_proj"))])
        if leaf == "down":
            return self._linear_any(self._hf(L + "mlp.down_proj"))
        if leaf == "experts":
            e = int(parts[3])
            kind = parts[4]
            base = L + f"mlp.experts.{e}."
            if kind == "gate_up":
                return _cat([self._linear_any(self._hf(base + "gate_proj")),
                             self._linear_any(self._hf(base + "up_proj"))])
            return self._linear_any(self._hf(base + "down_proj"))
        if leaf == "shared":
            base = L + "mlp.shared_expert."
            if parts[3] == "gate_up":
                return _cat([self._linear_any(self._hf(base + "gate_proj")),
                             self._linear_any(self._hf(base + "up_proj"))])
            return self._linear_any(self._hf(base + "down_proj"))
        raise KeyError(name)

    def tensor(self, name: str, shape, kind: str = "norm") -> torch.Tensor:
        parts = name.split(".")
        if name == "embed":
            return self.raw(self._hf("embed_tokens.weight")).to(torch.bfloat16)
        if name == "final_norm":
            return self.raw(self._hf("norm.weight")).to(torch.bfloat16)
        i = int(parts[1])
        leaf = parts[2]
        L = f"layers.{i}."
        m = {"ln1": "input_layernorm.weight", "ln2": "post_attention_layernorm.weight",
             "q_norm": "self_attn.q_norm.weight", "k_norm": "self_attn.k_norm.weight",
             "A_log": "linear_attn.A_log", "dt_bias": "linear_attn.dt_bias",
             "norm_w": "linear_attn.norm.weight", "router": "mlp.gate.weight",
             "shared_gate": "mlp.shared_expert_gate.weight"}
        if leaf == "conv_w":
            w = self.raw(self._hf(L + "linear_attn.conv1d.weight"))
            return w.reshape(w.shape[0], -1).to(torch.bfloat16)
        t = self.raw(self._hf(L + m[leaf]))
        if leaf in ("A_log", "dt_bias", "router", "shared_gate"):
            return t.float()
        return t.to(torch.bfloat16)


def _cat(ws):
    from .int4 import Int4Weight
    if any(isinstance(w, MXFP4Weight) for w in ws):
        from .mxfp4 import cat_rows
        # parts stored in different MX types (or one left in float) meet in the widest type
        fmt = max((w.fmt for w in ws if isinstance(w, MXFP4Weight)), key=lambda f: MX_BITS[f])
        ws = [w if isinstance(w, MXFP4Weight) and w.fmt == fmt else
              MXFP4Weight.from_float(w.dequantize() if isinstance(w, MXFP4Weight) else w.float(), fmt)
              for w in ws]
        return cat_rows(ws)
    if isinstance(ws[0], Int4Weight):
        from .int4 import cat_rows as ci
        return ci(ws)
    if any(isinstance(w, Int4Weight) for w in ws):      # mixed (an unquantized part)
        ws = [w.dequantize() if isinstance(w, Int4Weight) else w for w in ws]
    return torch.cat(ws, 0)


def _rows(w, idx: torch.Tensor):
    from .int4 import Int4Weight
    if isinstance(w, MXFP4Weight):
        return MXFP4Weight.from_packed(w.packed[idx], w.scales[idx], w.K, w.fmt)
    if isinstance(w, Int4Weight):
        return w.index_rows(idx)
    return w[idx]


def gdn_in_proj_permutation(cfg: ModelConfig) -> tuple[torch.Tensor, torch.Tensor]:
    """Row indices taking HF's per-key-head grouped [q_g,k_g,v_g,z_g] (qkvz) and [b_g,a_g] (ba)
    layouts to the merged canonical [q|k|v|z] and [b|a] orders."""
    Hk, Hv = cfg.gdn_num_k_heads, cfg.gdn_num_v_heads
    dk, dv = cfg.gdn_head_k_dim, cfg.gdn_head_v_dim
    rep = Hv // Hk
    gsz = 2 * dk + 2 * rep * dv
    q, k, v, z = [], [], [], []
    for g in range(Hk):
        base = g * gsz
        q += range(base, base + dk)
        k += range(base + dk, base + 2 * dk)
        v += range(base + 2 * dk, base + 2 * dk + rep * dv)
        z += range(base + 2 * dk + rep * dv, base + gsz)
    qkvz = torch.tensor(q + k + v + z, dtype=torch.long)
    b, a = [], []
    for g in range(Hk):
        b += range(g * 2 * rep, g * 2 * rep + rep)
        a += range(g * 2 * rep + rep, (g + 1) * 2 * rep)
    return qkvz, torch.tensor(b + a, dtype=torch.long)


def _merge_gdn_in_proj(qkvz, ba, cfg: ModelConfig):
    from .int4 import Int4Weight
    pq, pb = gdn_in_proj_permutation(cfg)
    if isinstance(qkvz, Int4Weight) and not isinstance(ba, Int4Weight):
        ba = Int4Weight.from_float(ba.float() if not isinstance(ba, MXFP4Weight)
                                   else ba.dequantize())
    if isinstance(qkvz, MXFP4Weight) != isinstance(ba, MXFP4Weight) and \
            not isinstance(qkvz, Int4Weight):
        # ba is often left unquantized in MXFP4 checkpoints: quantize it to match
        if isinstance(qkvz, MXFP4Weight):
            ba = MXFP4Weight.from_float(ba, qkvz.fmt)
        else:
            qkvz = MXFP4Weight.from_float(qkvz, ba.fmt)
    return _cat([_rows(qkvz, pq), _rows(ba, pb)])


def load_model(path: str, cfg: Optional[ModelConfig] = None, quant: str = "mxfp4", device="cuda",
               tp=None):
    """Build a HybridModel from a checkpoint directory."""
    from ..config import get_model_config
    from ..models.hybrid import HybridModel
    cfg = cfg or get_model_config(path)
    W = CheckpointWeights(path, cfg)
    W.keep_int4 = quant == "int4"
    return HybridModel(cfg, quant=quant, device=device, tp=tp, weights=W, init_device="cpu")
