"""Pure-PyTorch reference implementations of every engine op (the CPU oracle).

Each function here defines the exact semantics the CUDA kernels in ``csrc/`` implement; the
GPU numerics tests compare kernel output against these in fp32.  The model runs on CPU with
these ops, and the same functions are the fp32 references of the kernel
tests.  None of them is reached from a CUDA tensor in the engine: ``ops/*.py`` dispatch CUDA
tensors to the compiled extension and fail loudly if it is missing.
"""
from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn.functional as F

from ..quant.formats import (FP8_MAX, FP8_SCALE_FLOOR, fp8_e4m3, kv4_dequantize, kv4_quantize,
                             mx_dequantize, per_token_fp8)


# ---------------------------------------------------------------------------------------------
# norms and fused producers (reference: sly/mxfp4/radiance_mxfp4_fp8.hip:1715-1730, 1941, 2079)
# ---------------------------------------------------------------------------------------------
def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float, gemma: bool = True) -> torch.Tensor:
    xf = x.float()
    n = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    w = weight.float() + 1.0 if gemma else weight.float()
    return (n * w).to(torch.bfloat16)


def add_rms_norm(x, residual, weight, eps):
    """Returns (normed bf16, residual_out bf16); the fp32 sum feeds both outputs."""
    s = x.float() + (residual.float() if residual is not None else 0.0)
    res_o = s.to(torch.bfloat16)
    n = s * torch.rsqrt(s.pow(2).mean(-1, keepdim=True) + eps) * (weight.float() + 1.0)
    return n.to(torch.bfloat16), res_o


def quant_fp8_rows(n_bf16: torch.Tensor):
    """Per-token e4m3 quant of a bf16 tensor: amax over the bf16-rounded row."""
    nf = n_bf16.float()
    amax = nf.abs().amax(-1)
    scale = torch.clamp(amax / FP8_MAX, min=FP8_SCALE_FLOOR)
    q = fp8_e4m3(nf / scale.unsqueeze(-1))
    return q, scale


def add_rms_quant(x, residual, weight, eps):
    """Fused residual add + Gemma RMSNorm + per-token e4m3 quant -> (q, scale, residual_out)."""
    n, res_o = add_rms_norm(x, residual, weight, eps)
    q, s = quant_fp8_rows(n)
    return q, s, res_o


def silu_mul(gate_up: torch.Tensor) -> torch.Tensor:
    I = gate_up.shape[-1] // 2
    g = gate_up[..., :I].float()
    u = gate_up[..., I:].float()
    return (F.silu(g) * u).to(torch.bfloat16)


def silu_mul_quant(gate_up: torch.Tensor):
    return quant_fp8_rows(silu_mul(gate_up))


def gdn_gated_norm(o: torch.Tensor, z: torch.Tensor, weight: torch.Tensor, eps: float,
                   head_dim: int) -> torch.Tensor:
    """Per-head RMSNorm with a plain weight, gated by silu(z): ((x*rsqrt)*w)*silu(z) -> bf16."""
    T = o.shape[0]
    of = o.float().view(T, -1, head_dim)
    zf = z.float().view(T, -1, head_dim)
    n = of * torch.rsqrt(of.pow(2).mean(-1, keepdim=True) + eps) * weight.float()
    n = n.to(torch.bfloat16).float() * F.silu(zf)
    return n.view(T, -1).to(torch.bfloat16)


def gdn_norm_quant(o, z, weight, eps, head_dim):
    return quant_fp8_rows(gdn_gated_norm(o, z, weight, eps, head_dim))


def gate_mul(attn_out: torch.Tensor, gate: torch.Tensor) -> torch.Tensor:
    return (attn_out.float() * torch.sigmoid(gate.float())).to(torch.bfloat16)


def gate_mul_quant(attn_out, gate):
    return quant_fp8_rows(gate_mul(attn_out, gate))


# ---------------------------------------------------------------------------------------------
# linears
# ---------------------------------------------------------------------------------------------
def mxfp4_linear(q: torch.Tensor, scale: torch.Tensor, w_packed: torch.Tensor,
                 w_scales: torch.Tensor, bias: Optional[torch.Tensor] = None,
                 fmt: str = "e2m1") -> torch.Tensor:
    """C[M,N] = a_scale[m] * sum_k e4m3(q[m,k]) * w(w[n,k]) * 2^(ws[n,k/32]-127), fp32
    accumulate; w = e2m1 (MXFP4), e2m3 (MXFP6) or e4m3 (MXFP8) codes."""
    w = mx_dequantize(w_packed, w_scales, fmt)                  # [N, Kp] fp32 exact
    w = w[:, :q.shape[1]]                                       # zero-padded K tail
    c = (q.float() @ w.t()) * scale.float().unsqueeze(-1)
    if bias is not None:
        c = c + bias.float()
    return c.to(torch.bfloat16)


# ---------------------------------------------------------------------------------------------
# rotary embedding (neox style over the first rotary_dim dims)
# ---------------------------------------------------------------------------------------------
def rope_cos_sin(positions: torch.Tensor, rotary_dim: int, theta: float):
    inv = 1.0 / (theta ** (torch.arange(0, rotary_dim, 2, dtype=torch.float64) / rotary_dim))
    ang = positions.double().unsqueeze(-1) * inv.to(positions.device)
    return torch.cos(ang).float(), torch.sin(ang).float()


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, rotary_dim: int):
    """x [T, H, D] fp32; rotate-half on x[..., :rotary_dim]."""
    half = rotary_dim // 2
    x1 = x[..., :half]
    x2 = x[..., half:rotary_dim]
    c = cos.unsqueeze(1)
    s = sin.unsqueeze(1)
    r1 = x1 * c - x2 * s
    r2 = x2 * c + x1 * s
    return torch.cat([r1, r2, x[..., rotary_dim:]], dim=-1)


def qkv_prologue(qkv: torch.Tensor, positions: torch.Tensor, q_norm_w, k_norm_w, *,
                 num_q_heads: int, num_kv_heads: int, head_dim: int, rotary_dim: int,
                 theta: float, eps: float, gated: bool = True):
    """Split merged qkv, Gemma-RMSNorm q and k per head, apply RoPE.
    Returns q [T,Hq,D] bf16, k [T,Hkv,D] bf16, v [T,Hkv,D] bf16, gate [T,Hq*D] bf16 (or None)."""
    T = qkv.shape[0]
    qd = num_q_heads * head_dim * (2 if gated else 1)
    kd = num_kv_heads * head_dim
    qg = qkv[:, :qd].view(T, num_q_heads, -1)
    q = qg[..., :head_dim]
    gate = qg[..., head_dim:].reshape(T, -1) if gated else None
    k = qkv[:, qd:qd + kd].view(T, num_kv_heads, head_dim)
    v = qkv[:, qd + kd:qd + 2 * kd].view(T, num_kv_heads, head_dim)
    qn = rms_norm(q, q_norm_w, eps).float()
    kn = rms_norm(k, k_norm_w, eps).float()
    cos, sin = rope_cos_sin(positions, rotary_dim, theta)
    qn = apply_rope(qn, cos, sin, rotary_dim).to(torch.bfloat16)
    kn = apply_rope(kn, cos, sin, rotary_dim).to(torch.bfloat16)
    return qn, kn, v.to(torch.bfloat16), (gate.to(torch.bfloat16) if gated else None)


# ---------------------------------------------------------------------------------------------
# paged KV cache + attention
# ---------------------------------------------------------------------------------------------
def kv_cache_write(k, v, k_cache, v_cache, slot_mapping, block_size: int):
    """k,v [T,Hkv,D]; caches [num_blocks, Hkv, block_size, D] (fp8 e4m3 or bf16) or 4-bit rows
    [num_blocks, Hkv, block_size, D/2 + D/4] (uint8)."""
    keep = slot_mapping >= 0
    k, v, slot_mapping = k[keep], v[keep], slot_mapping[keep]
    blk = slot_mapping // block_size
    off = slot_mapping % block_size
    if k_cache.dtype == torch.uint8:
        kq, vq = kv4_quantize(k.to(torch.bfloat16).float()), kv4_quantize(v.float())
    elif k_cache.dtype == torch.float8_e4m3fn:
        kq, vq = fp8_e4m3(k.float()), fp8_e4m3(v.float())
    else:
        kq, vq = k.to(k_cache.dtype), v.to(v_cache.dtype)
    k_cache[blk, :, off] = kq
    v_cache[blk, :, off] = vq


def gather_kv(cache, block_table, length: int, block_size: int, head_dim: int = 0):
    nb = (length + block_size - 1) // block_size
    blocks = cache[block_table[:nb].long()]                      # [nb, H, bs, D]
    x = blocks.permute(0, 2, 1, 3).reshape(nb * block_size, cache.shape[1], cache.shape[3])
    if cache.dtype == torch.uint8:
        return kv4_dequantize(x[:length], head_dim)
    return x[:length].float()


def paged_attention(q, k_cache, v_cache, block_tables, seq_lens, query_start_loc, block_size,
                    scale: float, causal: bool = True, window: int = 0) -> torch.Tensor:
    """Varlen paged attention.  q [T,Hq,D] (query tokens are the last q_len positions of each
    sequence); seq_lens[b] = total context incl. the query tokens.  Returns bf16 [T,Hq,D].
    Query values are rounded to e4m3 when the cache is fp8 (the kernels run QK^T in fp8)."""
    T, Hq, D = q.shape
    Hkv = k_cache.shape[1]
    group = Hq // Hkv
    block_size = k_cache.shape[2]
    out = torch.zeros(T, Hq, D, dtype=torch.float32, device=q.device)
    qf = q.float()
    if k_cache.dtype == torch.float8_e4m3fn:
        qf = fp8_e4m3(qf).float()
    B = seq_lens.shape[0]
    for b in range(B):
        s0, s1 = int(query_start_loc[b]), int(query_start_loc[b + 1])
        ql = s1 - s0
        if ql == 0:
            continue
        L = int(seq_lens[b])
        K = gather_kv(k_cache, block_tables[b], L, block_size, D)   # [L,Hkv,D]
        V = gather_kv(v_cache, block_tables[b], L, block_size, D)
        Kr = K.repeat_interleave(group, dim=1)                    # [L,Hq,D]
        Vr = V.repeat_interleave(group, dim=1)
        qq = qf[s0:s1]                                            # [ql,Hq,D]
        sc = torch.einsum("qhd,khd->hqk", qq, Kr) * scale
        qpos = torch.arange(L - ql, L, device=q.device)
        kpos = torch.arange(L, device=q.device)
        mask = torch.ones(ql, L, dtype=torch.bool, device=q.device)
        if causal:
            mask &= kpos[None, :] <= qpos[:, None]
        if window > 0:
            mask &= kpos[None, :] > qpos[:, None] - window
        sc = sc.masked_fill(~mask[None], float("-inf"))
        p = torch.softmax(sc, dim=-1)
        out[s0:s1] = torch.einsum("hqk,khd->qhd", p, Vr)
    return out.to(torch.bfloat16)


# ---------------------------------------------------------------------------------------------
# gated delta net (reference formulas: sly/gdn/chunk_scan_ref.py:48-110)
# ---------------------------------------------------------------------------------------------
def causal_conv1d(x: torch.Tensor, weight: torch.Tensor, conv_state: Optional[torch.Tensor]):
    """Depthwise causal conv + SiLU over one sequence.  x [L, C]; weight [C, W];
    conv_state [C, W-1] = the previous W-1 inputs (oldest first).  Returns (y [L,C], new_state)."""
    L, C = x.shape
    W = weight.shape[1]
    prev = conv_state.float() if conv_state is not None else torch.zeros(C, W - 1, device=x.device)
    xx = torch.cat([prev.t(), x.float()], dim=0)                   # [W-1+L, C]
    y = torch.zeros(L, C, device=x.device)
    for j in range(W):
        y += xx[j:j + L] * weight[:, j].float()
    new_state = xx[-(W - 1):].t().contiguous()
    return F.silu(y), new_state


def l2norm(x: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    xf = x.float()
    return xf * torch.rsqrt((xf * xf).sum(-1, keepdim=True) + eps)


def gdn_gates(a: torch.Tensor, b: torch.Tensor, A_log: torch.Tensor, dt_bias: torch.Tensor):
    """g (log decay) = -exp(A_log) * softplus(a + dt_bias); beta = sigmoid(b)."""
    g = -torch.exp(A_log.float()) * F.softplus(a.float() + dt_bias.float())
    beta = torch.sigmoid(b.float())
    return g, beta


def gdn_recurrent(q, k, v, g, beta, state, scale):
    """Token-by-token gated delta rule for one sequence.
    q,k [L,Hk,dk] (already l2-normed); v [L,Hv,dv]; g,beta [L,Hv]; state [Hv,dv,dk] fp32.
    S <- e^g S; S <- S + beta (v - S k) k^T; o = scale S q.   Returns (o [L,Hv,dv], state)."""
    L, Hv, dv = v.shape
    Hk = q.shape[1]
    rep = Hv // Hk
    S = state.float().clone()
    o = torch.zeros(L, Hv, dv, device=v.device)
    for t in range(L):
        kt = k[t].float().repeat_interleave(rep, 0)               # [Hv, dk]
        qt = q[t].float().repeat_interleave(rep, 0)
        S = S * torch.exp(g[t].float())[:, None, None]
        kv = torch.einsum("hvk,hk->hv", S, kt)
        d = beta[t].float()[:, None] * (v[t].float() - kv)
        S = S + d[:, :, None] * kt[:, None, :]
        o[t] = scale * torch.einsum("hvk,hk->hv", S, qt)
    return o, S


def gdn_chunked(q, k, v, g, beta, state, scale, chunk: int = 64):
    """Chunked (WY) form of ``gdn_recurrent`` for one sequence, exact decay (no midpoint split).
    Same inputs/outputs; this is the math the prefill kernels implement."""
    L, Hv, dv = v.shape
    Hk = q.shape[1]
    rep = Hv // Hk
    S = state.float().clone()                                      # [Hv, dv, dk]
    o = torch.zeros(L, Hv, dv, device=v.device)
    qf = q.float().repeat_interleave(rep, 1)                       # [L,Hv,dk]
    kf = k.float().repeat_interleave(rep, 1)
    vf = v.float()
    for c0 in range(0, L, chunk):
        c1 = min(c0 + chunk, L)
        m = c1 - c0
        gc = torch.cumsum(g[c0:c1].float(), 0)                     # [m,Hv]
        bc = beta[c0:c1].float()
        for h in range(Hv):
            kk, qq, vv = kf[c0:c1, h], qf[c0:c1, h], vf[c0:c1, h]
            gg = gc[:, h]
            D = torch.exp((gg[:, None] - gg[None, :]).tril())
            Lm = torch.tril(bc[:, h, None] * (kk @ kk.t()) * D, -1)
            Ainv = torch.linalg.inv(torch.eye(m, device=v.device) + Lm)
            ge = torch.exp(gg)
            Wv = bc[:, h, None] * (vv - ge[:, None] * (kk @ S[h].t()))
            u = Ainv @ Wv                                          # [m, dv]
            o[c0:c1, h] = scale * (ge[:, None] * (qq @ S[h].t())) + \
                scale * (torch.tril(qq @ kk.t()) * D) @ u
            S[h] = torch.exp(gg[-1]) * S[h] + (torch.exp(gg[-1] - gg)[:, None] * u).t() @ kk
    return o, S


# ---------------------------------------------------------------------------------------------
# sampling
# ---------------------------------------------------------------------------------------------
def apply_top_k_top_p(logits: torch.Tensor, top_k: torch.Tensor, top_p: torch.Tensor,
                      min_p: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Mask logits [B,V] outside top-k / nucleus top-p (per row; k<=0 or p>=1 disables)."""
    B, V = logits.shape
    out = logits.clone().float()
    srt, idx = torch.sort(out, dim=-1, descending=True)
    ranks = torch.arange(V, device=logits.device).unsqueeze(0)
    k = top_k.long().clone()
    k = torch.where(k <= 0, torch.full_like(k, V), k).clamp(max=V)
    keep = ranks < k.unsqueeze(1)
    probs = torch.softmax(srt.masked_fill(~keep, float("-inf")), dim=-1)
    cum = torch.cumsum(probs, dim=-1)
    keep &= (cum - probs) < top_p.float().unsqueeze(1)
    if min_p is not None:
        keep &= probs >= (min_p.float().unsqueeze(1) * probs[:, :1])
    keep[:, 0] = True
    masked = srt.masked_fill(~keep, float("-inf"))
    out.scatter_(1, idx, masked)
    return out
