"""Gated-delta-net hybrid decoder (Qwen3-Next / Qwen3.8 family).

Layer i is full attention iff (i+1) % full_attn_interval == 0, else a gated delta net (GDN)
linear-attention layer; every layer has a SwiGLU MLP (or an MoE block).  Reference model code:
the vLLM Qwen3-Next files the reference patches (``sly/tests/fixtures/qwen3_next_v0.34.0.py.txt``,
decoder-layer fused norm ``:113-156``) and the GDN layer (``radiance_gdn.py``).

Forward over a flat varlen batch (prefill chunks and decode tokens mixed).  With MXFP4 weights
every linear runs W4A8: the fused producers turn the residual stream into (e4m3, scale) rows:

  add_rms_quant -> in_proj | qkv        (GDN | attention)
  GDN : conv(+SiLU, q/k L2) -> delta rule -> gated norm + quant -> out_proj
  ATTN: qk-norm + RoPE + KV write -> paged attention -> sigmoid gate + quant -> o_proj
  add_rms_quant -> gate_up -> silu_mul_quant -> down

Tensor parallelism: heads / intermediate are sharded per rank (column-parallel in_proj, qkv,
gate_up; row-parallel out_proj, o_proj, down followed by an all-reduce), vocab-parallel lm_head.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Callable, Optional

import os

import torch

from ..config import ModelConfig
from ..ops import kernels as K
from ..quant.formats import kv4_row_bytes
from ..quant.mxfp4 import MXFP4Weight
from .layers import FUSE_MAX_ROWS, Linear, NormAct, SiluAct, rope_cache
from .weights import RandomWeights, cat_rows, pad_rows, slice_cols, slice_rows


# ---------------------------------------------------------------------------------------------
# per-step metadata
# ---------------------------------------------------------------------------------------------
_FUSE_PRODUCERS = os.environ.get("RADIANCE_FUSE_PRODUCERS", "0") == "1"   # measured slower at M = 1
# NVTX ranges per decoder layer (and the final norm) for timeline profilers
_NVTX = os.environ.get("RADIANCE_NVTX", "0") == "1"

@dataclass
class StepMeta:
    """Device tensors describing one forward step (built by the model runner)."""
    num_seqs: int
    num_tokens: int
    query_start_loc: torch.Tensor      # [B+1] int32
    seq_lens: torch.Tensor             # [B] int32 (context incl. this step's tokens)
    has_initial: torch.Tensor          # [B] int32 (sequence has cached state/KV before this step)
    state_slots: torch.Tensor          # [B] int32 GDN state slot
    block_tables: torch.Tensor         # [B, max_blocks] int32
    slot_mapping: torch.Tensor         # [T] int64 KV slot of each token
    positions: torch.Tensor            # [T] int32
    token_seq: torch.Tensor            # [T] int32 sequence index of each token
    tile_seq: torch.Tensor             # [tiles] int32 attention row-tile -> sequence
    tile_row0: torch.Tensor            # [tiles] int32 first row of the tile
    num_splits: int = 1
    commit_len: Optional[torch.Tensor] = None   # spec-decode: tokens of each seq to commit to state
    gdn_write_out: bool = True
    _scratch: dict = field(default_factory=dict)

    def scratch_o(self, s, T, H, D):
        key = ("o", s, T, H, D)
        t = self._scratch.get(key)
        if t is None:
            t = torch.empty(s, T, H, D, dtype=torch.float32, device=self.query_start_loc.device)
            self._scratch[key] = t
        return t

    def scratch_ml(self, s, T, H):
        key = ("ml", s, T, H)
        t = self._scratch.get(key)
        if t is None:
            t = torch.empty(s, T, H, 2, dtype=torch.float32, device=self.query_start_loc.device)
            self._scratch[key] = t
        return t


@dataclass
class ModelCaches:
    k: list          # per attention layer [blocks, Hkv_local, block_size, hd]
    v: list
    conv: list       # per GDN layer [slots, conv_dim_local, W-1] bf16
    ssm: list        # per GDN layer [slots, Hv_local, dv, dk]
    block_size: int

    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for ts in (self.k, self.v, self.conv, self.ssm)
                   for t in ts)


# ---------------------------------------------------------------------------------------------
# tensor-parallel helpers
# ---------------------------------------------------------------------------------------------
@dataclass
class TPInfo:
    rank: int = 0
    size: int = 1
    all_reduce: Optional[Callable[[torch.Tensor], torch.Tensor]] = None
    all_gather_last: Optional[Callable[[torch.Tensor], torch.Tensor]] = None
    # fused all-reduce + residual add + RMSNorm + e4m3 quant (NVLink kernel); None = unfused
    all_reduce_add_rms_quant: Optional[Callable] = None

    def shard(self, n: int) -> tuple[int, int]:
        assert n % self.size == 0, (n, self.size)
        per = n // self.size
        return self.rank * per, per


def _cat_sections(w, sections: list[int], tp: TPInfo):
    """Column-parallel slice of a merged weight made of `sections` along dim 0."""
    parts, off = [], 0
    for n in sections:
        s0, per = tp.shard(n)
        parts.append(slice_rows(w, off + s0, per))
        off += n
    return cat_rows(parts) if len(parts) > 1 else parts[0]


def make_linear(w, quant: str, name: str) -> Linear:
    from ..quant.int4 import Int4Weight
    if isinstance(w, MXFP4Weight):
        if quant != "mxfp4":
            return Linear(w.dequantize().to(torch.bfloat16), quant, name)
        return Linear.from_mxfp4(w, name)
    if isinstance(w, Int4Weight):
        if quant == "int4":
            return Linear.from_int4(w, name)        # checkpoint codes kept as stored
        return Linear(w.dequantize(), quant, name)
    return Linear(w, quant, name)


# ---------------------------------------------------------------------------------------------
# layers
# ---------------------------------------------------------------------------------------------
class GDNMixer:
    def __init__(self, cfg: ModelConfig, tp: TPInfo, quant: str, W, prefix: str):
        self.cfg = cfg
        self.tp = tp
        H = cfg.hidden_size
        self.Hk = cfg.gdn_num_k_heads // tp.size
        self.Hv = cfg.gdn_num_v_heads // tp.size
        self.dk, self.dv = cfg.gdn_head_k_dim, cfg.gdn_head_v_dim
        self.key_dim = self.Hk * self.dk
        self.value_dim = self.Hv * self.dv
        self.conv_dim = 2 * self.key_dim + self.value_dim
        kd, vd, hv = cfg.gdn_key_dim, cfg.gdn_value_dim, cfg.gdn_num_v_heads
        w_in = W.linear(prefix + "in_proj", cfg.gdn_in_proj_dim, H)
        # [q|k|v|z|b|a] of this rank, padded to a multiple of 8 outputs: the consumers read z with
        # 16-byte vectors, so the output row stride must stay 16-byte aligned at every TP size
        self.in_proj = make_linear(pad_rows(_cat_sections(w_in, [kd, kd, vd, vd, hv, hv], tp), 8),
                                   quant, "in_proj")
        del w_in
        conv = W.tensor(prefix + "conv_w", (cfg.gdn_conv_dim, cfg.gdn_conv_kernel), "conv")
        self.conv_w = _cat_sections(conv, [kd, kd, vd], tp).to(torch.bfloat16).contiguous()
        h0, _ = tp.shard(hv)
        self.A_log = W.tensor(prefix + "A_log", (hv,), "A_log").float()[h0:h0 + self.Hv].contiguous()
        self.dt_bias = W.tensor(prefix + "dt_bias", (hv,), "dt_bias").float()[h0:h0 + self.Hv].contiguous()
        self.norm_w = W.tensor(prefix + "norm_w", (self.dv,), "norm_plain").to(torch.bfloat16)
        w_out = W.linear(prefix + "out_proj", H, vd)
        s0, per = tp.shard(vd)
        self.out_proj = make_linear(slice_cols(w_out, s0, per), quant, "out_proj")
        del w_out
        self.quant = quant
        self.scale = self.dk ** -0.5

    def forward(self, x, meta: StepMeta, conv_state, ssm_state, save=None, fin=None):
        """fin = (residual, norm weight, eps): the out_proj GEMM also runs the post-mixer
        residual add + RMSNorm + e4m3 and returns (q, scale, new residual) instead of h."""
        cfg = self.cfg
        proj = self.in_proj(x)                                    # [T, in_proj_local]
        cd, vd = self.conv_dim, self.value_dim
        xc = proj[:, :cd]
        z = proj[:, cd:cd + vd]
        ba = proj[:, cd + vd:cd + vd + 2 * self.Hv]
        fused_state = meta.commit_len is None and meta.num_tokens == meta.num_seqs
        if (fused_state and save is None and proj.is_cuda and K._GDN_DECODE_FUSED
                and self.dk == 128 and self.dv == 128 and conv_state.shape[2] == 3):
            if self.quant == "mxfp4" and K._GDN_DECODE_FUSED_QUANT:
                # decode: the whole GDN step and the out_proj producer (gated norm + e4m3) in
                # one launch
                act = K.gdn_decode_fused_quant(proj, cd + vd, cd, self.conv_w, conv_state,
                                               ssm_state, self.A_log, self.dt_bias, meta, self.Hk,
                                               self.scale, self.norm_w, cfg.rms_norm_eps)
                if fin is not None and self.out_proj.can_finish(act):
                    return self.out_proj.call_finish(act, K.FIN_NORM, *fin)
                return self.out_proj(act)
            # decode: the whole GDN step (conv, norms, gates, delta rule) in one launch
            o = K.gdn_decode_fused(proj, cd + vd, self.conv_w, conv_state, ssm_state, self.A_log,
                                   self.dt_bias, meta, self.Hk, self.scale)
        else:
            y = K.gdn_conv(xc, self.conv_w, conv_state, meta, self.key_dim, self.dk,
                           update_state=fused_state)
            if not fused_state:
                K.gdn_conv_state_update(xc, conv_state, meta, meta.commit_len)
            o = K.gdn_recurrent(y, ba, self.A_log, self.dt_bias, ssm_state, meta, self.Hk,
                                self.scale, commit_len=meta.commit_len)
            if save is not None:    # speculative verify: keep inputs for the commit pass
                save.append((proj, y))
        if self.quant in ("bf16", "int4"):
            h = self.out_proj(K.gdn_gated_norm(o, z, self.norm_w, cfg.rms_norm_eps, self.dv))
        else:
            act = K.gdn_norm_quant(o, z, self.norm_w, cfg.rms_norm_eps, self.dv)
            if fin is not None and self.out_proj.can_finish(act):
                return self.out_proj.call_finish(act, K.FIN_NORM, *fin)
            h = self.out_proj(act)
        return h

    def commit(self, saved, meta: StepMeta, conv_state, ssm_state, commit_len):
        """Apply the first commit_len[b] tokens of a verified block to the conv / SSM state."""
        proj, y = saved
        cd, vd = self.conv_dim, self.value_dim
        K.gdn_conv_state_update(proj[:, :cd], conv_state, meta, commit_len)
        K.gdn_recurrent(y, proj[:, cd + vd:cd + vd + 2 * self.Hv], self.A_log, self.dt_bias, ssm_state, meta, self.Hk,
                        self.scale, commit_len=commit_len, write_out=False)


class AttentionMixer:
    def __init__(self, cfg: ModelConfig, tp: TPInfo, quant: str, W, prefix: str):
        self.cfg = cfg
        self.tp = tp
        H = cfg.hidden_size
        hd = cfg.head_dim
        self.hd = hd
        self.Hq = cfg.num_q_heads // tp.size
        # kv heads: sharded when divisible, else replicated (each rank keeps its group's head)
        if cfg.num_kv_heads % tp.size == 0:
            self.Hkv = cfg.num_kv_heads // tp.size
            kv_sel = [tp.rank * self.Hkv + i for i in range(self.Hkv)]
        else:
            assert tp.size % cfg.num_kv_heads == 0
            self.Hkv = 1
            kv_sel = [tp.rank * cfg.num_kv_heads // tp.size]
        gated = cfg.attn_output_gate
        qd = cfg.num_q_heads * hd * (2 if gated else 1)
        w = W.linear(prefix + "qkv", cfg.qkv_proj_dim, H)
        s0, per = tp.shard(qd)
        kvd = cfg.num_kv_heads * hd
        rows = [slice_rows(w, s0, per)]
        rows += [slice_rows(w, qd + h * hd, hd) for h in kv_sel]
        rows += [slice_rows(w, qd + kvd + h * hd, hd) for h in kv_sel]
        self.qkv = make_linear(cat_rows(rows), quant, "qkv")
        del w, rows
        self.q_norm = W.tensor(prefix + "q_norm", (hd,), "norm")
        self.k_norm = W.tensor(prefix + "k_norm", (hd,), "norm")
        w_o = W.linear(prefix + "o_proj", H, cfg.num_q_heads * hd)
        s0, per = tp.shard(cfg.num_q_heads * hd)
        self.o_proj = make_linear(slice_cols(w_o, s0, per), quant, "o_proj")
        del w_o
        self.quant = quant
        self.gated = gated
        self.scale = hd ** -0.5
        self.cos_sin = None

    def forward(self, x, meta: StepMeta, k_cache, v_cache, fin=None):
        """fin: as GDNMixer.forward (o_proj runs the post-mixer norm as its finisher)."""
        cfg = self.cfg
        hd = self.hd
        qkv = self.qkv(x)
        T = qkv.shape[0]
        q = K.qkv_prologue(qkv, meta.positions, self.q_norm, self.k_norm, self.cos_sin, k_cache,
                           v_cache, meta.slot_mapping, num_q_heads=self.Hq,
                           num_kv_heads=self.Hkv, head_dim=hd, rotary_dim=cfg.rotary_dim,
                           theta=cfg.rope_theta, eps=cfg.rms_norm_eps, gated=self.gated,
                           block_size=k_cache.shape[2])
        if (self.gated and self.quant == "mxfp4" and
                K.attention_decode_gated_ok(q, k_cache, meta)):
            # decode: the sigmoid gate and the e4m3 quantisation run inside the attention launch
            act = K.paged_attention_gated(q, k_cache, v_cache, meta, self.scale, qkv[:, hd:],
                                          2 * hd)
            if fin is not None and self.o_proj.can_finish(act):
                return self.o_proj.call_finish(act, K.FIN_NORM, *fin)
            return self.o_proj(act)
        a = K.paged_attention(q, k_cache, v_cache, meta, self.scale).view(T, -1)
        if self.quant in ("bf16", "int4"):
            return self.o_proj(K.gate_mul(a, qkv[:, hd:], hd, 2 * hd) if self.gated else a)
        act = K.gate_mul_quant(a, qkv[:, hd:], hd, 2 * hd) if self.gated else K.quant_fp8(a)
        if fin is not None and self.o_proj.can_finish(act):
            return self.o_proj.call_finish(act, K.FIN_NORM, *fin)
        return self.o_proj(act)


class MLP:
    def __init__(self, cfg: ModelConfig, tp: TPInfo, quant: str, W, prefix: str,
                 inter: Optional[int] = None):
        H = cfg.hidden_size
        I = inter or cfg.intermediate_size
        w = W.linear(prefix + "gate_up", 2 * I, H)
        self.gate_up = make_linear(_cat_sections(w, [I, I], tp), quant, "gate_up")
        del w
        w = W.linear(prefix + "down", H, I)
        s0, per = tp.shard(I)
        self.down = make_linear(slice_cols(w, s0, per), quant, "down")
        del w
        self.quant = quant

    def forward(self, x, fin=None):
        """fin = (residual, next norm weight, eps): the down GEMM also produces the next layer's
        input (q, scale, new residual).  Decode-sized W4A8 inputs run SiLU * mul + e4m3 as the
        gate_up GEMM's finisher."""
        if self.gate_up.can_finish(x):
            act = self.gate_up.call_finish(x, K.FIN_SILU)
            if fin is not None and self.down.can_finish(act):
                return self.down.call_finish(act, K.FIN_NORM, *fin)
            return self.down(act)
        gu = self.gate_up(x)
        if self.quant in ("bf16", "int4"):
            return self.down(K.silu_mul(gu))
        if self.quant == "mxfp4" and gu.is_cuda and gu.shape[0] <= FUSE_MAX_ROWS and _FUSE_PRODUCERS:
            return self.down(SiluAct(gu))       # SiLU * mul + e4m3 inside the down GEMM
        return self.down(K.silu_mul_quant(gu))


class DecoderLayer:
    def __init__(self, cfg, idx, tp, quant, W, ep=None):
        self.idx = idx
        p = f"layers.{idx}."
        self.is_attn = cfg.is_attention_layer(idx)
        self.ln1 = W.tensor(p + "ln1", (cfg.hidden_size,), "norm")
        self.ln2 = W.tensor(p + "ln2", (cfg.hidden_size,), "norm")
        if self.is_attn:
            self.mixer = AttentionMixer(cfg, tp, quant, W, p)
        else:
            self.mixer = GDNMixer(cfg, tp, quant, W, p)
        if cfg.is_moe:
            from .moe import MoEBlock
            self.mlp = MoEBlock(cfg, tp, quant, W, p, ep=ep)
        else:
            self.mlp = MLP(cfg, tp, quant, W, p)


class HybridModel:
    """Random-init (or loaded) hybrid model.  Weights are created per layer on `device` and
    quantized to MXFP4 at load when quant == 'mxfp4'."""

    def __init__(self, cfg: ModelConfig, quant: str = "mxfp4", device="cpu", seed: int = 0,
                 tp: Optional[TPInfo] = None, init_device=None, weights=None,
                 lm_head_quant: Optional[str] = None, tp_pad: Optional[int] = None,
                 ep=None, embed_quant: Optional[str] = None):
        # MXFP6 / MXFP8 run the MXFP4 code path with another element type in the weights: every
        # linear arrives from the weight source already in that type
        from .weights import MX_QUANTS, MXCastWeights
        self.mx_fmt = MX_QUANTS.get(quant)
        if quant in ("mxfp6", "mxfp8"):
            quant = "mxfp4"
        self.quant = quant
        self.device = torch.device(device)
        self.tp = tp or TPInfo()
        init_dev = torch.device(init_device) if init_device is not None else self.device
        W = weights if weights is not None else RandomWeights(cfg, seed, init_dev)
        # a TP degree that does not divide the geometry (TP = 3): zero-weight dummy heads and
        # channels widen it (``tp_pad`` forces the widening of that degree at any TP size)
        from ..parallel.tp_pad import PaddedWeights, padded_config
        pcfg = padded_config(cfg, tp_pad or self.tp.size)
        if pcfg != cfg:
            W = PaddedWeights(W, cfg, pcfg)
            cfg = pcfg
        if self.mx_fmt not in (None, "e2m1"):
            W = MXCastWeights(W, self.mx_fmt, skip=("lm_head",) if lm_head_quant else ())
        self.cfg = cfg
        H, V = cfg.hidden_size, cfg.vocab_size
        self.embed = W.tensor("embed", (V, H), "embed").to(torch.bfloat16)
        # embedding table format: bf16, or int8 / int4 codes dequantised by the lookup kernel
        self.embed_quant = embed_quant
        # ep: data-parallel attention with expert-parallel MoE layers (parallel/ep.py)
        self.ep = ep
        self.layers = [DecoderLayer(cfg, i, self.tp, quant, W, ep=ep)
                       for i in range(cfg.num_layers)]
        self.final_norm = W.tensor("final_norm", (H,), "norm")
        # vocab-parallel lm_head
        w = W.linear("lm_head", V, H) if not cfg.tie_word_embeddings else self.embed.float()
        if self.mx_fmt not in (None, "e2m1") and not lm_head_quant and isinstance(w, torch.Tensor):
            w = MXFP4Weight.from_float(w.float(), self.mx_fmt)
        s0, per = self.tp.shard(V)
        self.vocab_start = s0
        # lm_head format: the model's by default; "int4" = W4A16 g128 with MSE clip search (the
        # reference's int4 lm_head: a quarter of the bf16 bytes on the decode critical path)
        self.lm_head = make_linear(slice_rows(w, s0, per), lm_head_quant or quant, "lm_head")
        del w
        if embed_quant in ("int8", "int4"):
            from ..quant.embed import QuantEmbedding
            self.embed = QuantEmbedding.from_float(self.embed, 8 if embed_quant == "int8" else 4)
        elif embed_quant not in (None, "bf16"):
            raise ValueError(f"embed_quant: int8, int4 or bf16, got {embed_quant}")
        if init_dev != self.device or getattr(W, "device", self.device) != self.device:
            self.to(self.device)
        self._init_rope()
        self._attach_push()

    def _attach_push(self):
        """TP > 1 with the NVLink communicator: the row-parallel linears (GDN out_proj,
        attention o_proj, dense MLP down) push their output tiles to every rank from the GEMM
        epilogue; the model's all-reduce call then only runs the receiving half."""
        comm = getattr(self.tp, "fused", None)
        if comm is None or self.quant != "mxfp4" or not getattr(comm, "push_enabled", False):
            return
        for layer in self.layers:
            lin = layer.mixer.out_proj if not layer.is_attn else layer.mixer.o_proj
            lin.push = comm
            if isinstance(layer.mlp, MLP):
                layer.mlp.down.push = comm

    def _init_rope(self):
        cfg = self.cfg
        for layer in self.layers:
            if layer.is_attn:
                if self.device.type == "cuda":
                    layer.mixer.cos_sin = rope_cache(cfg.max_position_embeddings, cfg.rotary_dim,
                                                     cfg.rope_theta, self.device)

    def to(self, device):
        device = torch.device(device)

        def mv(obj):
            for k, v in list(vars(obj).items()):
                if isinstance(v, torch.Tensor):
                    setattr(obj, k, v.to(device))
                elif isinstance(v, Linear):
                    v.to(device)
        self.embed = self.embed.to(device)
        self.final_norm = self.final_norm.to(device)
        self.lm_head.to(device)
        for layer in self.layers:
            mv(layer)
            mv(layer.mixer)
            mv(layer.mlp)
            if hasattr(layer.mlp, "to"):
                layer.mlp.to(device)
        self.device = device
        return self

    # ---- caches ----
    def make_caches(self, num_blocks: int, block_size: int, num_slots: int,
                    kv_dtype: str = "fp8", ssm_dtype: str = "float32") -> ModelCaches:
        cfg = self.cfg
        kdt = {"fp8": torch.float8_e4m3fn, "bf16": torch.bfloat16, "int4": torch.uint8}[kv_dtype]
        sdt = {"float32": torch.float32, "bfloat16": torch.bfloat16}[ssm_dtype]
        ks, vs, convs, ssms = [], [], [], []
        for layer in self.layers:
            m = layer.mixer
            if layer.is_attn:
                # zero-filled: stale pages never hold NaN bit patterns
                row = kv4_row_bytes(m.hd) if kv_dtype == "int4" else m.hd
                ks.append(torch.zeros(num_blocks, m.Hkv, block_size, row, dtype=kdt, device=self.device))
                vs.append(torch.zeros(num_blocks, m.Hkv, block_size, row, dtype=kdt, device=self.device))
            else:
                convs.append(torch.zeros(num_slots, m.conv_dim, cfg.gdn_conv_kernel - 1,
                                         dtype=torch.bfloat16, device=self.device))
                ssms.append(torch.zeros(num_slots, m.Hv, m.dv, m.dk, dtype=sdt, device=self.device))
        return ModelCaches(ks, vs, convs, ssms, block_size)

    @staticmethod
    def copy_state(caches: ModelCaches, src: int, dst: int):
        """Copy every GDN layer's conv + SSM state from slot `src` to slot `dst`."""
        for c in caches.conv:
            c[dst].copy_(c[src])
        for t in caches.ssm:
            t[dst].copy_(t[src])

    def cache_bytes_per_block(self, block_size: int, kv_dtype: str = "fp8") -> int:
        n = 0
        for layer in self.layers:
            if layer.is_attn:
                hd = layer.mixer.hd
                row = {"fp8": hd, "bf16": 2 * hd, "int4": kv4_row_bytes(hd)}[kv_dtype]
                n += 2 * layer.mixer.Hkv * block_size * row
        return n

    def state_bytes_per_slot(self, ssm_dtype: str = "float32") -> int:
        es = 4 if ssm_dtype == "float32" else 2
        n = 0
        for layer in self.layers:
            if not layer.is_attn:
                m = layer.mixer
                n += m.conv_dim * (self.cfg.gdn_conv_kernel - 1) * 2 + m.Hv * m.dv * m.dk * es
        return n

    # ---- forward ----
    def _reduce(self, h):
        if self.tp.size > 1:
            return self.tp.all_reduce(h)
        return h

    def forward(self, input_ids: torch.Tensor, meta: StepMeta, caches: ModelCaches,
                aux_layers: Optional[list] = None, aux_out: Optional[list] = None,
                gdn_save: Optional[list] = None) -> torch.Tensor:
        """Returns final-normed hidden states [T, H] bf16.  When `aux_layers` is given, the
        residual stream after each listed layer is appended to `aux_out` (drafter conditioning)."""
        cfg = self.cfg
        eps = cfg.rms_norm_eps
        if self.ep is not None and hasattr(self.ep.transport, "begin_step"):
            self.ep.transport.begin_step(int(input_ids.shape[0]))   # EP rounds for this step
        x = self.embed[input_ids.long()]
        residual = None
        h = x
        ai = gi = 0
        quant = self.quant in ("mxfp4", "fp8")     # e4m3 activations (int4 / bf16: bf16 ones)
        fused_ar = self.tp.size > 1 and quant and self.tp.all_reduce_add_rms_quant is not None
        # decode-sized steps: residual add + RMSNorm + e4m3 run inside the next GEMM
        fuse_prod = (self.quant == "mxfp4" and input_ids.is_cuda and _FUSE_PRODUCERS
                     and input_ids.shape[0] <= FUSE_MAX_ROWS)
        pending = None          # (q, s) produced by a fused all-reduce epilogue for the next norm
        # decode-sized W4A8 steps at TP1: the post-mixer and next-layer norms run as finishers of
        # the out_proj / o_proj and down GEMMs (no producer launches between the linears)
        fin_norm = (self.quant == "mxfp4" and input_ids.is_cuda and self.tp.size == 1
                    and not fuse_prod and input_ids.shape[0] <= K.GEMV_MAX_ROWS)
        for li, layer in enumerate(self.layers):
            if _NVTX:
                if li:
                    torch.cuda.nvtx.range_pop()
                torch.cuda.nvtx.range_push(f"layer {li} {'attn' if layer.is_attn else 'gdn'}")
            nxt = self.layers[li + 1] if li + 1 < len(self.layers) else None
            if pending is not None:
                a_in = pending
                pending = None
            elif fuse_prod:
                res_new = torch.empty_like(h)
                a_in = NormAct(h, residual, layer.ln1, eps, res_new)
                residual = res_new
            elif quant:
                a_in = K.add_rms_quant(h, residual, layer.ln1, eps)
                residual = a_in[2]
                a_in = (a_in[0], a_in[1])
            else:
                a_in, residual = K.add_rms_norm(h, residual, layer.ln1, eps)
            mfin = (residual, layer.ln2, eps) if fin_norm else None
            if layer.is_attn:
                h = layer.mixer.forward(a_in, meta, caches.k[ai], caches.v[ai], fin=mfin)
                ai += 1
            else:
                h = layer.mixer.forward(a_in, meta, caches.conv[gi], caches.ssm[gi], save=gdn_save,
                                        fin=mfin)
                gi += 1
            dense = isinstance(layer.mlp, MLP)
            if isinstance(h, tuple):        # the out GEMM's finisher: (q, s, new residual)
                q, s, residual = h
                # the down GEMM's finisher adds the MLP output to this (new) residual
                dfin = (residual, nxt.ln1, eps) if fin_norm and nxt is not None and dense else None
                h = layer.mlp.forward((q, s), fin=dfin) if dense else layer.mlp.forward((q, s))
            elif fused_ar:
                q, s, residual = self.tp.all_reduce_add_rms_quant(h, residual, layer.ln2, eps)
                h = layer.mlp.forward((q, s))
            else:
                h = self._reduce(h)
                if fuse_prod and isinstance(layer.mlp, MLP):
                    res_new = torch.empty_like(h)
                    h = layer.mlp.forward(NormAct(h, residual, layer.ln2, eps, res_new))
                    residual = res_new
                elif quant:
                    q, s, residual = K.add_rms_quant(h, residual, layer.ln2, eps)
                    h = layer.mlp.forward((q, s))
                else:
                    n, residual = K.add_rms_norm(h, residual, layer.ln2, eps)
                    h = layer.mlp.forward(n)
            if isinstance(h, tuple):        # the down GEMM's finisher: the next layer's input
                q, s, residual = h
                pending = (q, s)
                h = None
                if aux_layers is not None and li in aux_layers:
                    aux_out.append(residual)          # bf16(h + residual), as computed below
                continue
            if fused_ar and nxt is not None and aux_layers is None:
                q, s, residual = self.tp.all_reduce_add_rms_quant(h, residual, nxt.ln1, eps)
                pending = (q, s)
                h = None
            else:
                h = self._reduce(h)
            if aux_layers is not None and li in aux_layers:
                aux_out.append((h.float() + residual.float()).to(torch.bfloat16))
        if _NVTX and self.layers:
            torch.cuda.nvtx.range_pop()
        out, _ = K.add_rms_norm(h, residual, self.final_norm, eps, want_residual=False)
        return out

    def commit_gdn(self, meta: StepMeta, caches: ModelCaches, saved: list,
                   commit_len: torch.Tensor):
        """Speculative verify: apply the accepted prefix (commit_len[b] tokens, -1 = skip row) of
        each sequence to the GDN conv / SSM state, from the inputs saved during the verify pass."""
        gi = 0
        for layer in self.layers:
            if not layer.is_attn:
                layer.mixer.commit(saved[gi], meta, caches.conv[gi], caches.ssm[gi], commit_len)
                gi += 1

    def logits(self, hidden: torch.Tensor) -> torch.Tensor:
        """[n, H] -> [n, V] bf16 (vocab-parallel shards gathered when TP > 1)."""
        lg = self.lm_head(hidden)
        if self.tp.size > 1:
            lg = self.tp.all_gather_last(lg)
        if self.cfg.real_vocab_size:
            lg = lg[..., :self.cfg.real_vocab_size].contiguous()    # drop padding rows
        return lg

    def weight_bytes(self) -> int:
        n = (self.embed.nbytes if hasattr(self.embed, "nbytes") and not isinstance(self.embed, torch.Tensor)
             else self.embed.numel() * 2) + self.lm_head.nbytes
        for layer in self.layers:
            for obj in (layer.mixer, layer.mlp):
                for v in vars(obj).values():
                    if isinstance(v, Linear):
                        n += v.nbytes
        return n
