"""DFlash2 block drafter (speculative decoding), re-implemented from the reference's behaviour
(``dflash2/qwen3_dflash2.py:26-307``, ``dflash2/speculator.py:109-215``):

  * conditioning: the target's residual stream at `num_aux_layers` evenly spaced layers is
    concatenated per token and projected by ``fc`` (num_aux*H_t -> H_d).  The projected context
    is turned into attention K/V for every drafter layer once per token and stored in the
    drafter's paged KV cache (the reference's "context K/V in one GEMM",
    ``patch_dflash_fused_kv_fp8.py``).
  * block: one forward over [anchor token, mask x k] at positions P..P+k; attention is
    non-causal inside the block and sees the context through a sliding window (2048).
  * every layer is wrapped by grouped depthwise convolutions over block positions
    (``DFlashGroupedConv``): per-position coefficients = base kernel + kernel_projection(h),
    applied before attention / MLP (side 0) and after them (side 1).
  * candidates: the target's lm_head scores the k draft positions, top-K candidates per
    position; a low-rank selector scores predecessor->successor edges
    (``unary + <pred[prev] * proj(h), succ[cand]>``) and a path walk picks one candidate per
    step (greedy, or Gumbel-noised argmax at the request temperature).  The realised scores give
    the draft distribution the rejection sampler checks (fp32 window, everything else -inf).
  * embeddings and lm_head are shared with the target; drafter linears are MXFP4 W4A8.
"""
from __future__ import annotations

import math
from typing import Optional

import os

import torch
import torch.nn.functional as F

from ..config import DrafterConfig, ModelConfig
from ..ops import kernels as K
from .hybrid import StepMeta
from .layers import Linear, rope_cache


class _DrafterLayer:
    def __init__(self, dc: DrafterConfig, gen, device, quant):
        H, hd = dc.hidden_size, dc.head_dim
        std = 0.02
        rnd = lambda *s: torch.randn(*s, generator=gen, device=device) * std
        self.ln1 = torch.zeros(H, dtype=torch.bfloat16, device=device)
        self.ln2 = torch.zeros(H, dtype=torch.bfloat16, device=device)
        self.qkv = Linear(rnd(dc.num_q_heads * hd + 2 * dc.num_kv_heads * hd, H), quant, "d_qkv")
        self.o = Linear(rnd(H, dc.num_q_heads * hd), quant, "d_o")
        self.q_norm = torch.zeros(hd, dtype=torch.bfloat16, device=device)
        self.k_norm = torch.zeros(hd, dtype=torch.bfloat16, device=device)
        self.gate_up = Linear(rnd(2 * dc.intermediate_size, H), quant, "d_gate_up")
        self.down = Linear(rnd(H, dc.intermediate_size), quant, "d_down")
        G = H // dc.conv_group_size
        self.G = G
        # grouped conv: base kernels [2 sides, taps, H] and kernel_projection H -> 2*taps*G,
        # one pair for attention and one for the MLP
        self.attn_base = (torch.randn(2, dc.conv_taps, H, generator=gen, device=device) * 0.1).to(torch.bfloat16)
        self.mlp_base = (torch.randn(2, dc.conv_taps, H, generator=gen, device=device) * 0.1).to(torch.bfloat16)
        self.attn_kproj = Linear(rnd(2 * dc.conv_taps * G, H).contiguous(), "bf16", "d_attn_kproj")
        self.mlp_kproj = Linear(rnd(2 * dc.conv_taps * G, H).contiguous(), "bf16", "d_mlp_kproj")


def selector_walk_torch(unary, cand, anchors, hp, pred_cb, succ_cb, temps):
    """Candidate path walk (torch ops): unary [B,k,Kc], cand [B,k,Kc], anchors [B], hp [B,k,r],
    codebooks [V,r], temps [B] -> drafts [B,k], window probs [B,k,Kc].  Edge scores
    unary + <pred[prev] * hp, succ[cand]> with prev the token chosen one position earlier (the
    anchor first); Gumbel-noised argmax of score / T at T > 0, argmax at T = 0."""
    B, k, Kc = unary.shape
    dev = unary.device
    prev_ids = torch.cat([anchors.view(B, 1, 1).expand(B, 1, Kc), cand[:, :-1]], dim=1)
    pred = pred_cb[prev_ids].float()                                    # [B,k,Kp,r]
    succ = succ_cb[cand].float()                                        # [B,k,Kc,r]
    scores = unary.unsqueeze(2) + torch.einsum("bkpr,bkcr->bkpc", pred * hp.unsqueeze(2), succ)
    temps = temps.view(B, 1)
    prev = torch.zeros(B, dtype=torch.long, device=dev)
    drafts, win_p = [], []
    for i in range(k):
        s = scores[torch.arange(B, device=dev), i, prev]               # [B, Kc]
        t = temps.clamp(min=1e-6)
        probs = torch.softmax(s / t, -1)
        g = -torch.log(-torch.log(torch.rand(B, Kc, device=dev).clamp(1e-9, 1 - 1e-9)))
        noisy = torch.where(temps > 0, s / t + g, s)
        ch = noisy.argmax(-1)
        greedy_p = F.one_hot(s.argmax(-1), Kc).float()
        win_p.append(torch.where(temps > 0, probs, greedy_p))
        drafts.append(cand[torch.arange(B, device=dev), i, ch])
        prev = ch
    return torch.stack(drafts, 1), torch.stack(win_p, 1)


def grouped_conv(h: torch.Tensor, delta: torch.Tensor, base: torch.Tensor, block: int,
                 G: int, taps: int) -> torch.Tensor:
    """h [T, H] (T = n_blocks * block, block-major); delta [T, taps, G]; base [taps, H].
    out[t] = sum_{tap <= pos(t)} (base[tap] + delta[t, tap, group]) * h[t - tap].  CUDA rows run
    as one kernel (``csrc/spec_decode.cu`` dflash_conv_kernel); this torch form is its oracle."""
    if h.is_cuda:
        from ..ops._ext import ext
        out = torch.empty(h.shape, dtype=torch.bfloat16, device=h.device)
        ext().dflash_conv(h.contiguous(), delta, base.contiguous(), G, block, out)
        return out
    T, H = h.shape
    gs = H // G
    hb = h.float().view(T, G, gs)
    coef = base.float().view(1, taps, G, gs) + delta.float().unsqueeze(-1)
    pos = torch.arange(T, device=h.device) % block
    out = coef[:, 0] * hb
    for tap in range(1, taps):
        sh = F.pad(hb[:-tap], (0, 0, 0, 0, tap, 0))
        out = out + coef[:, tap] * sh * (pos >= tap).view(-1, 1, 1).float()
    return out.view(T, H).to(torch.bfloat16)


class DFlash2Drafter:
    def __init__(self, dc: DrafterConfig, target, k: int, device, block_size: int,
                 num_blocks: int, seed: int = 1, quant: str = "mxfp4"):
        self.dc = dc
        self.target = target
        self.k = k
        self.device = torch.device(device)
        gen = torch.Generator(device=self.device)
        gen.manual_seed(seed)
        tcfg: ModelConfig = target.cfg
        L = tcfg.num_layers
        na = dc.num_aux_layers
        # evenly spaced target layers (their residual stream after the layer)
        self.aux_layers = [min(L - 1, round((i + 1) * L / (na + 1))) for i in range(na)]
        H = dc.hidden_size
        self.fc = Linear(torch.randn(H, na * tcfg.hidden_size, generator=gen, device=self.device) * 0.02,
                         quant, "d_fc")
        self.layers = [_DrafterLayer(dc, gen, self.device, quant) for _ in range(dc.num_layers)]
        self.final_norm = torch.zeros(H, dtype=torch.bfloat16, device=self.device)
        self.mask_embed = (torch.randn(tcfg.hidden_size, generator=gen, device=self.device) * 0.02).to(torch.bfloat16)
        self.pred_codebook = (torch.randn(tcfg.vocab_size, dc.selector_rank, generator=gen, device=self.device) * 0.1).to(torch.bfloat16)
        self.succ_codebook = (torch.randn(tcfg.vocab_size, dc.selector_rank, generator=gen, device=self.device) * 0.1).to(torch.bfloat16)
        self.hidden_proj = Linear(torch.randn(dc.selector_rank, H, generator=gen, device=self.device) * 0.02, "bf16", "d_sel")
        if H != tcfg.hidden_size:
            raise ValueError("drafter hidden size must equal the target's (shared embed / lm_head)")
        kdt = torch.float8_e4m3fn
        self.kc = [torch.zeros(num_blocks, dc.num_kv_heads, block_size, dc.head_dim, dtype=kdt, device=self.device)
                   for _ in range(dc.num_layers)]
        self.vc = [torch.zeros_like(t) for t in self.kc]
        self.block_size = block_size
        self.rope = rope_cache(tcfg.max_position_embeddings, dc.head_dim, dc.rope_theta, self.device) \
            if self.device.type == "cuda" else None
        self.last = {}          # request id -> (candidate ids [k,Kc], draft probs [k,Kc])
        self.kv = None          # engine KV manager (set by for_engine)
        # prefill window skip (RADIANCE_DFLASH_PREFILL_WINDOW_SKIP, on by default): every drafter
        # layer attends through the sliding window only, so prompt rows more than window + margin
        # before the prompt's end get no fc / context K/V.  margin >= 2 KV blocks keeps the block
        # holding the last skipped position wholly below the first block a draft can touch.
        # Reference: sly/radiance_dflash_skip.py:1-60 (there per step: whole chunks are skipped).
        self.window_skip = os.environ.get("RADIANCE_DFLASH_PREFILL_WINDOW_SKIP", "1") == "1"
        self.skip_margin = max(int(os.environ.get("RADIANCE_DFLASH_PREFILL_WINDOW_SKIP_MARGIN",
                                                  "512")), 2 * block_size)
        self.skipped_rows = 0

    @staticmethod
    def for_engine(engine, k: int) -> "DFlash2Drafter":
        tcfg = engine.model_config
        if tcfg.hidden_size <= 512:
            dc = DrafterConfig.tiny()
            dc.hidden_size = tcfg.hidden_size
        else:
            dc = DrafterConfig()
        dc.block_size = k + 1
        d = DFlash2Drafter(dc, engine.model, k, engine.device, engine.config.block_size,
                           engine.num_blocks)
        d.kv = engine.kv
        return d

    def _prefill_skip_span(self) -> int:
        """Prompt rows closer than this to the prompt's end keep their context K/V (0 = the
        skip is off)."""
        if not self.window_skip or not self.dc.window:
            return 0
        return self.dc.window + self.skip_margin

    # ------------------------------------------------------------------------------------------
    def _kv_write(self, li, h_norm, positions, slot_mapping):
        """K/V of `h_norm` rows into drafter layer li's cache; returns the rotated queries."""
        dc = self.dc
        lay = self.layers[li]
        qkv = lay.qkv(h_norm)
        return K.qkv_prologue(qkv, positions, lay.q_norm, lay.k_norm, self.rope, self.kc[li],
                              self.vc[li], slot_mapping, num_q_heads=dc.num_q_heads,
                              num_kv_heads=dc.num_kv_heads, head_dim=dc.head_dim,
                              rotary_dim=dc.head_dim, theta=dc.rope_theta, eps=dc.rms_norm_eps,
                              gated=False, block_size=self.block_size)

    def observe(self, sched, meta: StepMeta, aux: list, sampled: dict, sample_cnt, hidden=None):
        """Write context K/V for the tokens the target just committed (prefill chunks and the
        accepted prefix of verified blocks), from the target's aux-layer hidden states."""
        if not aux:
            return
        rows, pos, slots = [], [], []
        qsl = meta.query_start_loc.cpu().tolist()
        pos_h = meta.positions.cpu().tolist()
        skip_below = self._prefill_skip_span()
        for bi, s in enumerate(sched.seqs):
            n = s.num_new_tokens
            if s.is_decode and s.draft_tokens:
                toks = sampled.get(s.req.request_id, [])
                n = max(1, len(toks))          # the fed token + accepted drafts
            # prefill window skip: prompt positions the sliding-window drafter will never attend
            # to (more than window + margin before the prompt's end) need no context K/V
            lo = s.req.num_prompt_tokens - skip_below if (skip_below and not s.is_decode) else None
            for t in range(qsl[bi], qsl[bi] + min(n, qsl[bi + 1] - qsl[bi])):
                if lo is not None and pos_h[t] < lo:
                    self.skipped_rows += 1
                    continue
                rows.append(t)
        if not rows:
            return
        idx = torch.tensor(rows, device=self.device)
        ctx = torch.cat([a[idx] for a in aux], dim=1)
        h = self.fc(ctx)
        positions = meta.positions[idx]
        slot_mapping = meta.slot_mapping[idx]
        for li in range(len(self.layers)):
            self._kv_write(li, h, positions, slot_mapping)

    def propose(self, reqs, new_tokens) -> list[list[int]]:
        """One block forward per request: [anchor, mask*k] at positions P..P+k."""
        dc, k = self.dc, self.k
        B = len(reqs)
        blk = k + 1
        dev = self.device
        anchors = [t[-1] for t in new_tokens]
        P = [r.num_tokens + len(t) - 1 for r, t in zip(reqs, new_tokens)]   # anchor position
        emb = self.target.embed[torch.tensor(anchors, device=dev)]
        x = self.mask_embed.unsqueeze(0).repeat(B * blk, 1)
        x.view(B, blk, -1)[:, 0] = emb
        positions = torch.tensor([p + j for p in P for j in range(blk)], dtype=torch.int32, device=dev)
        bs = self.block_size
        slots, bts, seqlens = [], [], []
        maxb = 0
        for r, p in zip(reqs, P):
            need = (p + blk + bs - 1) // bs
            if self.kv is not None and len(r.block_ids) < need:
                self.kv.allocate(r, p + blk)   # the next verify step needs these pages anyway
            blocks = list(r.block_ids)
            while len(blocks) < need:          # pool exhausted: unwritten dummy page
                blocks.append(0)
            bts.append(blocks)
            maxb = max(maxb, len(blocks))
            for j in range(blk):
                q = p + j
                slots.append(blocks[q // bs] * bs + q % bs if (q // bs) < len(r.block_ids) else -1)
            seqlens.append(p + blk)
        bt = torch.zeros(B, maxb, dtype=torch.int32)
        for i, b in enumerate(bts):
            bt[i, :len(b)] = torch.tensor(b, dtype=torch.int32)
        G = dc.num_q_heads // dc.num_kv_heads
        tiles_s, tiles_r = [], []
        for b in range(B):
            for r0 in range(0, blk * G, 64):
                tiles_s.append(b)
                tiles_r.append(r0)
        i32 = lambda v: torch.tensor(v, dtype=torch.int32, device=dev)
        meta = StepMeta(num_seqs=B, num_tokens=B * blk,
                        query_start_loc=i32([b * blk for b in range(B + 1)]),
                        seq_lens=i32(seqlens), has_initial=i32([1] * B), state_slots=i32([0] * B),
                        block_tables=bt.to(dev), slot_mapping=torch.tensor(slots, dtype=torch.int64, device=dev),
                        positions=positions, token_seq=i32([b for b in range(B) for _ in range(blk)]),
                        tile_seq=i32(tiles_s), tile_row0=i32(tiles_r), num_splits=1)
        h = x
        res = None
        for li, lay in enumerate(self.layers):
            n, res = K.add_rms_norm(h, res, lay.ln1, dc.rms_norm_eps)
            co = lay.attn_kproj(n).view(B * blk, 2, dc.conv_taps, lay.G)
            n = grouped_conv(n, co[:, 0], lay.attn_base[0], blk, lay.G, dc.conv_taps)
            q = self._kv_write(li, n, positions, meta.slot_mapping)
            a = K.paged_attention(q, self.kc[li], self.vc[li], meta, dc.head_dim ** -0.5,
                                  causal=False, window=dc.window).view(B * blk, -1)
            a = lay.o(a)
            a = grouped_conv(a, co[:, 1], lay.attn_base[1], blk, lay.G, dc.conv_taps)
            n, res = K.add_rms_norm(a, res, lay.ln2, dc.rms_norm_eps)
            co = lay.mlp_kproj(n).view(B * blk, 2, dc.conv_taps, lay.G)
            n = grouped_conv(n, co[:, 0], lay.mlp_base[0], blk, lay.G, dc.conv_taps)
            gu = lay.gate_up(n)
            m = lay.down(K.silu_mul_quant(gu))
            h = grouped_conv(m, co[:, 1], lay.mlp_base[1], blk, lay.G, dc.conv_taps)
        hf, _ = K.add_rms_norm(h, res, self.final_norm, dc.rms_norm_eps, want_residual=False)
        hd = hf.view(B, blk, -1)[:, 1:].reshape(B * k, -1)             # draft positions
        logits = self.target.logits(hd)                                 # shared lm_head
        Kc = dc.top_k_candidates
        if logits.is_cuda and Kc <= K.TOPK_WINDOW:
            # the sampler's top-64 window kernel (sorted, ties to the lowest id) over the vocab
            unary, cand = K.topk_window(logits)
            unary, cand = unary[:, :Kc].contiguous(), cand[:, :Kc].contiguous()
        else:
            unary, cand = torch.topk(logits.float(), Kc, dim=-1)        # [B*k, Kc]
        unary, cand = unary.view(B, k, Kc), cand.view(B, k, Kc)
        hp = self.hidden_proj(hd).float().view(B, k, -1)                # [B,k,r]
        temps = torch.tensor([r.params.temperature for r in reqs], device=dev).view(B)
        if dev.type == "cuda" and Kc <= 32:
            D, Wp = self.walk_cuda(unary, cand, anchors, hp, temps, reqs)
        else:
            D, Wp = selector_walk_torch(unary, cand, torch.tensor(anchors, device=dev), hp,
                                        self.pred_codebook, self.succ_codebook, temps)
        out = D.cpu().tolist()
        for b, r in enumerate(reqs):
            self.last[r.request_id] = (cand[b], Wp[b])
        return out

    def walk_cuda(self, unary, cand, anchors, hp, temps, reqs):
        """The path walk as one kernel (``csrc/spec_decode.cu`` walk_kernel): scores along the
        chosen path only, Gumbel-max at T > 0, window probabilities for the rejection test."""
        from ..engine.sampler import row_seed
        from ..ops._ext import ext
        from ..ops.kernels import status_word
        B, k, Kc = unary.shape
        dev = unary.device
        drafts = torch.empty(B, k, dtype=torch.int64, device=dev)
        winp = torch.empty(B, k, Kc, dtype=torch.float32, device=dev)
        seeds = torch.tensor([row_seed(r, 104729) for r in reqs], dtype=torch.int64).to(dev)
        anc = torch.as_tensor(anchors, dtype=torch.int64).to(dev)
        ext().dflash_walk(unary.float().contiguous(), cand.contiguous(), anc, hp.contiguous(),
                          self.pred_codebook.contiguous(), self.succ_codebook.contiguous(),
                          temps.float().contiguous(), seeds, drafts, winp, status_word(dev))
        return drafts, winp

    def draft_windows(self, reqs, k, dev):
        ids = torch.stack([self.last[r.request_id][0][:k] for r in reqs])
        pr = torch.stack([self.last[r.request_id][1][:k] for r in reqs])
        return ids, pr
