"""Engine ops.  CUDA tensors run the sm_100a kernels of ``csrc/``; CPU tensors run the PyTorch
oracle of ``ops/reference.py`` (the CPU model of the tiny config and the fp32 references of the
kernel tests).  There is no CUDA->PyTorch fallback: a missing kernel library raises."""
from __future__ import annotations

from typing import Optional

import os

import torch

from . import reference as ref
from ._ext import ext

_EMPTY: dict = {}


def _empty(device) -> torch.Tensor:
    t = _EMPTY.get(device)
    if t is None:
        t = torch.empty(0, device=device)
        _EMPTY[device] = t
    return t


_STATUS: dict = {}

# error codes of the device status word (csrc/common.cuh StatusCode)
STATUS_NAMES = {1: "mbarrier wait timed out", 2: "peer wait timed out",
                3: "index out of bounds", 4: "tensor-memory allocation failed"}


class KernelFaultError(RuntimeError):
    """A kernel recorded an error in the device status word (a bounded wait that expired, or a
    bad index it refused to use).  The kernel returned normally; its outputs are not valid."""

    def __init__(self, code: int):
        self.code = code
        super().__init__(f"kernel reported error {code}: {STATUS_NAMES.get(code, 'unknown')}")


def status_word(device) -> torch.Tensor:
    """Per-device int32[4] status word: [0] error code the kernels write (0 = ok), [2] / [3] the
    mbarrier / peer-flag wait limits in microseconds (0 = the compiled-in 200 ms / 5 s)."""
    device = torch.device(device)
    if device.type == "cuda" and device.index is None:
        device = torch.device("cuda", torch.cuda.current_device())
    t = _STATUS.get(device)
    if t is None:
        t = torch.zeros(4, dtype=torch.int32, device=device)
        _STATUS[device] = t
    return t


def set_wait_limits(device, mbar_us: int = 0, peer_us: int = 0):
    """Time limits of the kernels' bounded waits on `device` (0 = default).  Ordered on the
    current stream, so kernels launched after it see the new limits."""
    t = status_word(device)
    t[2] = int(mbar_us)
    t[3] = int(peer_us)


def reset_status(device):
    status_word(device)[:2].zero_()


def check_status(device, reset: bool = True) -> int:
    """Host check of the device error word (syncs).  Raises KernelFaultError on a recorded
    error; the wait limits are kept."""
    t = status_word(device)
    code = int(t[0].item())
    if code != 0:
        if reset:
            reset_status(device)
        raise KernelFaultError(code)
    return code


_WS: dict = {}
_WS_RETIRED: list = []
# Debug mode (RADIANCE_CANARY=1): every workspace carries a tail of canary words that no kernel
# may write; the engine checks them after each step (check_canaries) and names an overrun.
_CANARY = os.environ.get("RADIANCE_CANARY", "0") == "1"
CANARY_WORDS = 1024
CANARY_VALUE = 0x5A5A5A5A
_CANARIES: list = []


def workspace(device, name: str, numel: int) -> torch.Tensor:
    """Zero-initialised int32 workspace shared by launches of one kernel family (counters in it
    are self-resetting).  Grown on demand outside CUDA-graph capture.  A workspace that is
    outgrown is kept alive, never freed: CUDA graphs captured earlier still address it, and its
    counters must not land in memory the allocator has handed to another tensor."""
    device = torch.device(device)
    if device.type == "cuda" and device.index is None:
        device = torch.device("cuda", torch.cuda.current_device())
    key = (str(device), name)
    t = _WS.get(key)
    if t is None or t.numel() < numel:
        if t is not None:
            _WS_RETIRED.append(t)
        n = max(numel, 1 << 16, 2 * t.numel() if t is not None else 0)
        if _CANARY:
            base = torch.zeros(n + CANARY_WORDS, dtype=torch.int32, device=device)
            base[n:] = CANARY_VALUE
            _CANARIES.append((name, base, n))
            t = base[:n]
        else:
            t = torch.zeros(n, dtype=torch.int32, device=device)
        _WS[key] = t
    return t


def check_canaries() -> None:
    """Debug mode: raise if any workspace's canary tail was written (syncs)."""
    for name, base, n in _CANARIES:
        tail = base[n:]
        if not bool((tail == CANARY_VALUE).all()):
            first = int((tail != CANARY_VALUE).nonzero()[0])
            raise RuntimeError(f"workspace '{name}' overrun: canary word {first} past its "
                               f"{n} words was written")


def _none(t, device):
    return t if t is not None else _empty(device)


# ---------------------------------------------------------------------------------------------
# producers
# ---------------------------------------------------------------------------------------------
def add_rms_quant(x: torch.Tensor, residual: Optional[torch.Tensor], weight: torch.Tensor,
                  eps: float, res_out: Optional[torch.Tensor] = None):
    """-> (q e4m3 [M,H], scale fp32 [M], residual_out bf16 [M,H])."""
    if not x.is_cuda:
        return ref.add_rms_quant(x, residual, weight, eps)
    M, H = x.shape
    q = torch.empty(M, H, dtype=torch.float8_e4m3fn, device=x.device)
    s = torch.empty(M, dtype=torch.float32, device=x.device)
    if res_out is None:
        res_out = torch.empty(M, H, dtype=torch.bfloat16, device=x.device)
    e = _empty(x.device)
    ext().add_rms_quant(x, _none(residual, x.device), weight, res_out, q, s, e, eps)
    return q, s, res_out


def add_rms_norm(x: torch.Tensor, residual: Optional[torch.Tensor], weight: torch.Tensor,
                 eps: float, want_residual: bool = True):
    """-> (normed bf16, residual_out bf16 or None)."""
    if not x.is_cuda:
        n, r = ref.add_rms_norm(x, residual, weight, eps)
        return n, r
    M, H = x.shape
    n = torch.empty(M, H, dtype=torch.bfloat16, device=x.device)
    r = torch.empty(M, H, dtype=torch.bfloat16, device=x.device) if want_residual else None
    e = _empty(x.device)
    ext().add_rms_quant(x, _none(residual, x.device), weight, _none(r, x.device), e, e, n, eps)
    return n, r


def silu_mul_quant(gate_up: torch.Tensor):
    if not gate_up.is_cuda:
        return ref.silu_mul_quant(gate_up)
    M, I2 = gate_up.shape
    q = torch.empty(M, I2 // 2, dtype=torch.float8_e4m3fn, device=gate_up.device)
    s = torch.empty(M, dtype=torch.float32, device=gate_up.device)
    ext().silu_mul_quant(gate_up, q, s)
    return q, s


def silu_mul(gate_up: torch.Tensor) -> torch.Tensor:
    """bf16 silu(gate)*up (unquantized reference model path only; the W4A8 hot path uses
    silu_mul_quant)."""
    if not gate_up.is_cuda:
        return ref.silu_mul(gate_up)
    I = gate_up.shape[1] // 2
    g = gate_up[:, :I].float()
    return (g * torch.sigmoid(g) * gate_up[:, I:].float()).to(torch.bfloat16)


def gdn_norm_quant(o: torch.Tensor, z: torch.Tensor, weight: torch.Tensor, eps: float,
                   head_dim: int):
    if not o.is_cuda:
        return ref.gdn_norm_quant(o, z, weight, eps, head_dim)
    M, D = o.shape
    q = torch.empty(M, D, dtype=torch.float8_e4m3fn, device=o.device)
    s = torch.empty(M, dtype=torch.float32, device=o.device)
    ext().gdn_norm_quant(o, z, weight, head_dim, eps, q, s, _empty(o.device))
    return q, s


def gdn_gated_norm(o, z, weight, eps, head_dim):
    if not o.is_cuda:
        return ref.gdn_gated_norm(o, z, weight, eps, head_dim)
    M, D = o.shape
    n = torch.empty(M, D, dtype=torch.bfloat16, device=o.device)
    e = _empty(o.device)
    ext().gdn_norm_quant(o, z, weight, head_dim, eps, e, e, n)
    return n


def gate_mul_quant(a: torch.Tensor, gate: torch.Tensor, head_dim: int, gate_head_stride: int):
    """a [M, H*hd]; gate = a strided view whose head h starts at column h*gate_head_stride."""
    if not a.is_cuda:
        M = a.shape[0]
        H = a.shape[1] // head_dim
        g = torch.stack([gate[:, h * gate_head_stride:h * gate_head_stride + head_dim]
                         for h in range(H)], 1).reshape(M, -1)
        return ref.gate_mul_quant(a, g)
    M, D = a.shape
    q = torch.empty(M, D, dtype=torch.float8_e4m3fn, device=a.device)
    s = torch.empty(M, dtype=torch.float32, device=a.device)
    ext().gate_mul_quant(a, gate, head_dim, gate_head_stride, q, s, _empty(a.device))
    return q, s


def gate_mul(a, gate, head_dim, gate_head_stride):
    if not a.is_cuda:
        M = a.shape[0]
        H = a.shape[1] // head_dim
        g = torch.stack([gate[:, h * gate_head_stride:h * gate_head_stride + head_dim]
                         for h in range(H)], 1).reshape(M, -1)
        return ref.gate_mul(a, g)
    M, D = a.shape
    n = torch.empty(M, D, dtype=torch.bfloat16, device=a.device)
    e = _empty(a.device)
    ext().gate_mul_quant(a, gate, head_dim, gate_head_stride, e, e, n)
    return n


def quant_fp8(x: torch.Tensor):
    if not x.is_cuda:
        return ref.quant_fp8_rows(x)
    M, D = x.shape
    q = torch.empty(M, D, dtype=torch.float8_e4m3fn, device=x.device)
    s = torch.empty(M, dtype=torch.float32, device=x.device)
    ext().quant_fp8_rows(x, q, s)
    return q, s


# ---------------------------------------------------------------------------------------------
# linears
# ---------------------------------------------------------------------------------------------
def mxfp4_gemm(q: torch.Tensor, scale: torch.Tensor, packed: torch.Tensor, sf: torch.Tensor,
               scales_plain: torch.Tensor, N: int, out: Optional[torch.Tensor] = None,
               splits: int = 0, fmt: str = "e2m1") -> torch.Tensor:
    """Block-scaled W(4|6|8)A8 GEMM; the CUDA kernel reads the weight type from the packed row
    width, fmt names it for the CPU path."""
    if not q.is_cuda:
        return ref.mxfp4_linear(q, scale, packed, scales_plain, fmt=fmt)
    M = q.shape[0]
    if out is None:
        out = torch.empty(M, N, dtype=torch.bfloat16, device=q.device)
    ext().mxfp4_gemm(q, scale, packed, sf, out, splits, status_word(q.device))
    return out


# persistent stream-K decode GEMM: one CTA per SM by default (RADIANCE_GEMV_CTAS_PER_SM)
GEMV_MAX_ROWS = 16
_GEMV_CPS = int(os.environ.get("RADIANCE_GEMV_CTAS_PER_SM", "1"))
FIN_NONE, FIN_NORM, FIN_SILU = 0, 1, 2


def _gemv_ws(device):
    return workspace(device, "gemv", 8192 + 2 * 160 * max(1, _GEMV_CPS) * 16 * 128)


def mxfp4_gemv(q, scale, w, out=None, fin: int = FIN_NONE, res=None, norm_w=None, res_out=None,
               eps: float = 1e-6):
    """Decode W4A8 GEMM (1..16 rows, CUDA) -> out [M, N] bf16; with fin = FIN_NORM / FIN_SILU
    the CTA that completes the last tile also produces the next linear's (e4m3, scale) rows:
    residual add + RMSNorm(1 + w) (new residual into res_out) or SiLU(g) * u.  Returns out, or
    (out, q, scale) with a finisher."""
    M = q.shape[0]
    dev = q.device
    if out is None:
        out = torch.empty(M, w.N, dtype=torch.bfloat16, device=dev)
    e = _empty(dev)
    if fin == FIN_NONE:
        ext().mxfp4_gemv(q, scale, w.packed, w.sf, out, _gemv_ws(dev), _GEMV_CPS, 0, e, e, e, e, e,
                         0.0, status_word(dev))
        return out
    H = w.N if fin == FIN_NORM else w.N // 2
    fq = torch.empty(M, H, dtype=torch.float8_e4m3fn, device=dev)
    fs = torch.empty(M, dtype=torch.float32, device=dev)
    ext().mxfp4_gemv(q, scale, w.packed, w.sf, out, _gemv_ws(dev), _GEMV_CPS, fin,
                     _none(res, dev), _none(norm_w, dev), _none(res_out, dev), fq, fs, eps,
                     status_word(dev))
    return out, fq, fs


def mxfp4_gemm_finish(q, scale, w, fin: int, res=None, norm_w=None, res_out=None,
                      eps: float = 1e-6):
    """Decode W4A8 GEMM (1..16 rows, CUDA) whose last CTA also produces the next linear's
    (e4m3, scale) rows -- FIN_NORM: residual add + RMSNorm(1 + w), new residual into res_out;
    FIN_SILU: SiLU(g) * u of the output [g | u].  -> (out, q, scale)."""
    M = q.shape[0]
    dev = q.device
    out = torch.empty(M, w.N, dtype=torch.bfloat16, device=dev)
    H = w.N if fin == FIN_NORM else w.N // 2
    fq = torch.empty(M, H, dtype=torch.float8_e4m3fn, device=dev)
    fs = torch.empty(M, dtype=torch.float32, device=dev)
    ext().mxfp4_gemm_fin(q, scale, w.packed, w.sf, out, fin, _none(res, dev), _none(norm_w, dev),
                         _none(res_out, dev), fq, fs, eps, workspace(dev, "gemm_fin", 1),
                         status_word(dev))
    return out, fq, fs


def mxfp4_gemv_push(q, scale, w, peers, rank: int, half_words: int) -> int:
    return ext().mxfp4_gemv_push(q, scale, w.packed, w.sf, _gemv_ws(q.device), _GEMV_CPS, peers,
                                 rank, half_words, status_word(q.device))


def mxfp4_gemm_act(mode: int, x, res, w_norm, res_out, eps: float, w, out):
    """Decode GEMM with the producer fused in (CUDA only): mode 1 = add + RMSNorm + e4m3 of
    x (+ res), new residual -> res_out; mode 2 = SiLU(g) * u + e4m3 of x = [g | u]."""
    e = _empty(x.device)
    ext().mxfp4_gemm_act(mode, x, res if res is not None else e,
                         w_norm if w_norm is not None else e, res_out if res_out is not None else e,
                         eps, w.packed, w.sf, out, status_word(x.device))
    return out


def moe_work_items(counts: torch.Tensor, bn: int, max_items: int) -> torch.Tensor:
    """(expert, first row, rows) per row tile of the expert-sorted buffer, padded with empty
    items to a fixed length (device ops only: no host sync, CUDA-graph safe)."""
    tiles = (counts + bn - 1) // bn
    starts = torch.cumsum(counts, 0) - counts
    tcum = torch.cumsum(tiles, 0)
    i = torch.arange(max_items, device=counts.device)
    e = torch.searchsorted(tcum, i, right=True).clamp(max=counts.shape[0] - 1)
    j = i - (tcum[e] - tiles[e])
    rows = torch.clamp(counts[e] - j * bn, min=0, max=bn)
    rows = torch.where(i < tcum[-1], rows, torch.zeros_like(rows))
    return torch.stack([e, starts[e] + j * bn, rows], 1).to(torch.int32).contiguous()


def moe_grouped_gemm(q, s, w, n_per_group: int, counts: torch.Tensor) -> torch.Tensor:
    """Expert-sorted rows (q, s) x stacked expert MXFP4 weights -> [R, n_per_group] bf16."""
    R = q.shape[0]
    E = counts.shape[0]
    avg = max(1, R // max(1, counts.numel()))
    bn = 16 if avg <= 16 else 32 if avg <= 32 else 64 if avg <= 64 else 128 if avg <= 128 else 256
    max_items = (R + bn - 1) // bn + E
    items = moe_work_items(counts, bn, max_items)
    out = torch.zeros(R, n_per_group, dtype=torch.bfloat16, device=q.device)   # uncovered rows = 0
    ext().mxfp4_grouped_gemm(q, s, w.packed, w.sf, out, items, bn, n_per_group,
                             status_word(q.device))
    return out


def moe_grouped_mlp(q, s, counts, w_gate_up, w_down, I: int, H: int) -> torch.Tensor:
    gu = moe_grouped_gemm(q, s, w_gate_up, 2 * I, counts)
    a = silu_mul_quant(gu)
    return moe_grouped_gemm(a[0], a[1], w_down, H, counts)


# ---------------------------------------------------------------------------------------------
# attention
# ---------------------------------------------------------------------------------------------
def qkv_prologue(qkv, positions, q_norm_w, k_norm_w, cos_sin, k_cache, v_cache, slot_mapping, *,
                 num_q_heads, num_kv_heads, head_dim, rotary_dim, theta, eps, gated, block_size):
    """-> q [T,Hq,D] bf16 (e4m3-rounded when the cache is fp8); k/v written into the caches."""
    T = qkv.shape[0]
    qd = num_q_heads * head_dim * (2 if gated else 1)
    kd = num_kv_heads * head_dim
    if not qkv.is_cuda:
        q, k, v, _ = ref.qkv_prologue(qkv, positions, q_norm_w, k_norm_w,
                                      num_q_heads=num_q_heads, num_kv_heads=num_kv_heads,
                                      head_dim=head_dim, rotary_dim=rotary_dim, theta=theta,
                                      eps=eps, gated=gated)
        ref.kv_cache_write(k, v, k_cache, v_cache, slot_mapping, block_size)
        if k_cache.dtype == torch.float8_e4m3fn:
            q = ref.fp8_e4m3(q.float()).to(torch.bfloat16)
        return q
    q = torch.empty(T, num_q_heads, head_dim, dtype=torch.bfloat16, device=qkv.device)
    ext().qkv_prologue(qkv, head_dim * (2 if gated else 1), qd, qd + kd, positions, q_norm_w,
                       k_norm_w, cos_sin, rotary_dim, num_q_heads, num_kv_heads, eps, q, k_cache,
                       v_cache, slot_mapping)
    return q


_ATTN_DECODE = os.environ.get("RADIANCE_ATTN_DECODE", "1") != "0"
# chunked prefill over the fp8 cache on the tcgen05 attention kernel (csrc/fmha.cu)
_FMHA = os.environ.get("RADIANCE_FMHA", "1") != "0"


def attention_decode_gated_ok(q, k_cache, meta) -> bool:
    """The decode kernel can run the o_proj producer (sigmoid gate + e4m3) itself."""
    T, Hq, D = q.shape
    return (q.is_cuda and _ATTN_DECODE and _ATTN_GATE_FUSED and meta.num_tokens == meta.num_seqs
            and Hq // k_cache.shape[1] <= 16 and Hq * D * 4 <= 144 * D * 2)


def paged_attention_gated(q, k_cache, v_cache, meta, scale: float, gate, gate_head_stride: int):
    """Decode attention (one query token per sequence) with the o_proj producer in the same
    launch: y = bf16(o * sigmoid(gate)) of each token row, quantised to (e4m3, scale)."""
    T, Hq, D = q.shape
    dev = q.device
    out = torch.empty(T, Hq, D, dtype=torch.bfloat16, device=dev)
    gq = torch.empty(T, Hq * D, dtype=torch.float8_e4m3fn, device=dev)
    gs = torch.empty(T, dtype=torch.float32, device=dev)
    _paged_attention_launch(q, k_cache, v_cache, meta, scale, True, 0, out, True,
                            (gate, gate_head_stride, workspace(dev, "attn_gate", max(4096, T)),
                             gq, gs))
    return gq, gs


def _paged_attention_launch(q, k_cache, v_cache, meta, scale, causal, window, out, decode,
                            gated=None):
    T, Hq, D = q.shape
    splits = meta.num_splits if decode else min(meta.num_splits, 32)
    if splits > 1:
        part_o = meta.scratch_o(splits, T, Hq, D)
        part_ml = meta.scratch_ml(splits, T, Hq)
    else:
        part_o = part_ml = _empty(q.device)
    e = _empty(q.device)
    g, ghs, cnt, gq, gs = gated if gated is not None else (e, 0, e, e, e)
    ext().paged_attention(q, k_cache, v_cache, meta.block_tables, meta.seq_lens,
                          meta.query_start_loc, meta.tile_seq, meta.tile_row0, scale, causal,
                          window, splits, part_o, part_ml, out,
                          workspace(q.device, "attn", meta.tile_seq.shape[0] * k_cache.shape[1]),
                          decode, g, ghs, cnt, gq, gs)


def paged_attention(q, k_cache, v_cache, meta, scale: float, causal: bool = True,
                    window: int = 0, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Varlen paged attention over the batch described by ``meta`` (an AttnMeta)."""
    if not q.is_cuda:
        return ref.paged_attention(q, k_cache, v_cache, meta.block_tables, meta.seq_lens,
                                   meta.query_start_loc, k_cache.shape[2], scale, causal, window)
    T, Hq, D = q.shape
    if out is None:
        out = torch.empty(T, Hq, D, dtype=torch.bfloat16, device=q.device)
    # one query token per sequence and at most 16 query heads per kv head: the decode kernel
    # (keys split across warps) replaces the 64-row tile kernel
    decode = (meta.num_tokens == meta.num_seqs and Hq // k_cache.shape[1] <= 16
              and _ATTN_DECODE)
    if (not decode and _FMHA and causal and window == 0 and meta.num_splits == 1 and D == 256
            and ((k_cache.shape[2] == 64 and k_cache.dtype == torch.float8_e4m3fn)
                 or k_cache.dtype == torch.uint8)):
        # prefill on tcgen05 (e4m3 QK / PV legs, TMEM accumulators, TMA-fed pages)
        kc, vc, bt = k_cache, v_cache, meta.block_tables
        if k_cache.dtype == torch.uint8:
            # 4-bit cache (any page size): the keys this chunk reaches, dequantised once into
            # 64-key e4m3 pages renumbered per sequence
            B, nb = bt.shape
            Hkv = k_cache.shape[1]
            p64 = (nb * k_cache.shape[2] + 63) // 64
            page = Hkv * 64 * D
            npg = B * p64
            ws = workspace(q.device, "kv4_e4m3", (2 * npg * page + 255) // 256 * 64 + npg + 64)
            raw = ws.view(torch.uint8)
            kc = raw[:npg * page].view(torch.float8_e4m3fn).view(npg, Hkv, 64, D)
            vc = raw[npg * page:2 * npg * page].view(torch.float8_e4m3fn).view(npg, Hkv, 64, D)
            off = (2 * npg * page + 255) // 256 * 64          # int32 words, 256-byte aligned
            bt = ws[off:off + npg].view(B, p64)
            ext().kv4_to_e4m3_pages(k_cache, v_cache, meta.block_tables, meta.seq_lens, kc, vc, bt)
        ext().fmha_prefill(q, kc, vc, bt, meta.seq_lens, meta.query_start_loc, meta.tile_seq,
                           meta.tile_row0, scale, out, status_word(q.device))
        return out
    # the decode kernel merges up to 128 KV splits in-kernel, the tile kernel up to 32
    _paged_attention_launch(q, k_cache, v_cache, meta, scale, causal, window, out, decode)
    return out


# ---------------------------------------------------------------------------------------------
# gated delta net
# ---------------------------------------------------------------------------------------------
def gdn_conv(x, conv_w, conv_state, meta, qk_dim: int, head_dim: int, eps: float = 1e-6,
             update_state: bool = False):
    """x [T, conv_dim] (pre-conv q|k|v) -> y [T, conv_dim] bf16 (SiLU, q/k L2-normed).
    update_state (only valid when every sequence feeds exactly one token) also shifts the conv
    state in place; otherwise gdn_conv_state_update does it in a second launch."""
    T, C = x.shape[0], conv_w.shape[0]
    if not x.is_cuda:
        y = torch.empty(T, C, dtype=torch.bfloat16)
        qsl = meta.query_start_loc
        for b in range(meta.num_seqs):
            s0, s1 = int(qsl[b]), int(qsl[b + 1])
            if s1 == s0:
                continue
            st = conv_state[int(meta.state_slots[b])] if int(meta.has_initial[b]) else None
            yy, _ = ref.causal_conv1d(x[s0:s1, :C], conv_w, st)
            yy = yy.clone()
            nk = qk_dim // head_dim
            for hh in range(2 * nk):
                sl = slice(hh * head_dim, (hh + 1) * head_dim)
                yy[:, sl] = ref.l2norm(yy[:, sl])
            y[s0:s1] = yy.to(torch.bfloat16)
        if update_state:
            gdn_conv_state_update(x, conv_state, meta)
        return y
    y = torch.empty(T, C, dtype=torch.bfloat16, device=x.device)
    # the kernel L2-normalises the first `2 * qk_dim` channels (q and k heads)
    ext().gdn_conv(x, conv_w, conv_state, meta.query_start_loc, meta.state_slots,
                   meta.has_initial, meta.token_seq, 2 * qk_dim, head_dim, y, eps, update_state)
    return y


def gdn_conv_state_update(x, conv_state, meta, commit_len: Optional[torch.Tensor] = None):
    C = conv_state.shape[1]
    if not x.is_cuda:
        qsl = meta.query_start_loc
        for b in range(meta.num_seqs):
            s0, s1 = int(qsl[b]), int(qsl[b + 1])
            n = int(commit_len[b]) if commit_len is not None else s1 - s0
            if n < 0:
                continue
            slot = int(meta.state_slots[b])
            st = conv_state[slot].float() if int(meta.has_initial[b]) else \
                torch.zeros(C, conv_state.shape[2])
            xx = torch.cat([st.t(), x[s0:s0 + n, :C].float()], 0)
            conv_state[slot] = xx[-conv_state.shape[2]:].t().to(conv_state.dtype)
        return
    ext().gdn_conv_state_update(x, conv_state, meta.query_start_loc, meta.state_slots,
                                meta.has_initial, _none(commit_len, x.device))


def gdn_decode_fused(proj, ba_off: int, conv_w, conv_state, ssm_state, A_log, dt_bias, meta,
                     num_k_heads: int, scale: float, eps: float = 1e-6,
                     split: int = 0) -> torch.Tensor:
    """One token per sequence (CUDA): conv update + SiLU + q/k L2 norm + gates + delta rule in
    one launch.  proj = in_proj output rows; returns o [B, Hv * dv] bf16; states updated.
    split: CTAs per head (1, 2, 4; 0 = the library default)."""
    B = meta.num_seqs
    _, Hv, DV, _ = ssm_state.shape
    out = torch.empty(B, Hv * DV, dtype=torch.bfloat16, device=proj.device)
    e = _empty(proj.device)
    ext().gdn_decode_fused(proj, ba_off, conv_w, conv_state, A_log, dt_bias, ssm_state,
                           meta.state_slots, meta.has_initial, num_k_heads, scale, eps, out,
                           split, 0, e, 0.0, e, e, e, e)
    return out


def gdn_decode_fused_quant(proj, ba_off: int, z_off: int, conv_w, conv_state, ssm_state, A_log,
                           dt_bias, meta, num_k_heads: int, scale: float, norm_w, norm_eps: float,
                           eps: float = 1e-6):
    """gdn_decode_fused with the out_proj producer in the same launch: the gated RMSNorm of each
    head (z at column z_off of proj) and the per-token e4m3 quantisation -> (q, scale)."""
    B = meta.num_seqs
    _, Hv, DV, _ = ssm_state.shape
    dev = proj.device
    nout = torch.empty(B, Hv * DV, dtype=torch.bfloat16, device=dev)
    q = torch.empty(B, Hv * DV, dtype=torch.float8_e4m3fn, device=dev)
    qs = torch.empty(B, dtype=torch.float32, device=dev)
    ws = workspace(dev, "gdn_fq", 4096 + B * Hv)
    ext().gdn_decode_fused(proj, ba_off, conv_w, conv_state, A_log, dt_bias, ssm_state,
                           meta.state_slots, meta.has_initial, num_k_heads, scale, eps,
                           _empty(dev), 1, z_off, norm_w, norm_eps, nout, ws, q, qs)
    return q, qs


_GDN_CHUNKED = os.environ.get("RADIANCE_GDN_CHUNKED", "1") != "0"
_GDN_CHUNK_SPLIT = int(os.environ.get("RADIANCE_GDN_CHUNK_SPLIT", "0"))   # 0: by batch size
_GDN_TWO_PHASE = os.environ.get("RADIANCE_GDN_TWO_PHASE", "1") != "0"
_GDN_DECODE_FUSED = os.environ.get("RADIANCE_GDN_DECODE_FUSED", "1") != "0"
# the o_proj producer inside decode attention: opt-in, it measured slower than attention followed
# by gate_mul_quant (the gate runs after two levels of last-CTA serialisation: splits, kv heads)
_ATTN_GATE_FUSED = os.environ.get("RADIANCE_ATTN_GATE_FUSED", "0") == "1"
# the out_proj producer (gated norm + e4m3) inside the fused decode step
_GDN_DECODE_FUSED_QUANT = os.environ.get("RADIANCE_GDN_DECODE_FUSED_QUANT", "1") != "0"


def gdn_recurrent(y, ba, A_log, dt_bias, ssm_state, meta, num_k_heads: int, scale: float,
                  out: Optional[torch.Tensor] = None, commit_len=None, write_out: bool = True):
    """Delta rule over the batch; ssm_state [S, Hv, dv, dk] updated in place (after the first
    commit_len[b] tokens when given).  Returns o [T, Hv*dv] bf16."""
    T = y.shape[0]
    S_, Hv, DV, DK = ssm_state.shape
    if out is None:
        out = torch.empty(T, Hv * DV, dtype=torch.bfloat16, device=y.device)
    if not y.is_cuda:
        key_dim = num_k_heads * DK
        qsl = meta.query_start_loc
        for b in range(meta.num_seqs):
            s0, s1 = int(qsl[b]), int(qsl[b + 1])
            if s1 == s0:
                continue
            slot = int(meta.state_slots[b])
            st = ssm_state[slot].float() if int(meta.has_initial[b]) else torch.zeros(Hv, DV, DK)
            q = y[s0:s1, :key_dim].float().view(-1, num_k_heads, DK)
            k = y[s0:s1, key_dim:2 * key_dim].float().view(-1, num_k_heads, DK)
            v = y[s0:s1, 2 * key_dim:2 * key_dim + Hv * DV].float().view(-1, Hv, DV)
            g, beta = ref.gdn_gates(ba[s0:s1, Hv:2 * Hv], ba[s0:s1, :Hv], A_log, dt_bias)
            n = int(commit_len[b]) if commit_len is not None else s1 - s0
            if n < 0:
                continue
            o, _ = ref.gdn_recurrent(q, k, v, g, beta, st, scale)
            _, st_c = ref.gdn_recurrent(q[:n], k[:n], v[:n], g[:n], beta[:n], st, scale)
            ssm_state[slot] = st_c.to(ssm_state.dtype)
            if write_out:
                out[s0:s1] = o.reshape(s1 - s0, -1).to(torch.bfloat16)
        return out
    if (commit_len is None and write_out and _GDN_CHUNKED and DK == 128 and DV == 128
            and meta.num_tokens > meta.num_seqs):
        # prefill rows in the batch: the 64-token chunk scan on the tensor cores -- by default in
        # two phases (every chunk's triangular solve in parallel, then the state scan split over
        # value columns)
        if _GDN_TWO_PHASE:
            T, B = y.shape[0], meta.state_slots.shape[0]
            ws = workspace(y.device, "gdn2", ext().gdn_chunked2_ws_bytes(T, B, Hv) // 4 + 4)
            ext().gdn_chunked2(y, ba, A_log, dt_bias, ssm_state, meta.query_start_loc,
                               meta.state_slots, meta.has_initial, num_k_heads, scale, out, ws,
                               _GDN_CHUNK_SPLIT if _GDN_CHUNK_SPLIT in (2, 4, 8) else 0)
        else:
            ext().gdn_chunked(y, ba, A_log, dt_bias, ssm_state, meta.query_start_loc,
                              meta.state_slots, meta.has_initial, num_k_heads, scale, out,
                              _GDN_CHUNK_SPLIT)
        return out
    ext().gdn_recurrent(y, ba, A_log, dt_bias, ssm_state, meta.query_start_loc, meta.state_slots,
                        meta.has_initial, _none(commit_len, y.device), num_k_heads, scale, out,
                        write_out)
    return out


# ---------------------------------------------------------------------------------------------
# sampling
# ---------------------------------------------------------------------------------------------
def argmax(logits: torch.Tensor) -> torch.Tensor:
    if not logits.is_cuda:
        return logits.float().argmax(-1)
    ids = torch.empty(logits.shape[0], dtype=torch.int64, device=logits.device)
    ext().argmax_rows(logits, ids, _empty(logits.device), workspace(logits.device, "argmax",
                                                                     4096 + logits.shape[0] * 128))
    return ids


def sample_from_topk(vals, ids, temperature, top_k, top_p, min_p, seeds, step: int,
                     want_probs: bool = False):
    """vals/ids [B, K] sorted descending -> (token ids [B], probs over the window or None).
    K may be the whole vocabulary (a sorted row): the full-vocabulary sampling path."""
    B, K = vals.shape
    out = torch.empty(B, dtype=torch.int64, device=vals.device)
    probs = torch.empty(B, K, dtype=torch.float32, device=vals.device) if want_probs else None
    if not vals.is_cuda:
        return _sample_rows_cpu(vals, ids, temperature, top_k, top_p, min_p, seeds, step,
                                want_probs)
    ext().sample_from_topk(vals.float().contiguous(), ids.contiguous(), temperature, top_k,
                           top_p, _none(min_p, vals.device), seeds, step, out,
                           _empty(vals.device), _none(probs, vals.device))
    return out, probs


def _sample_rows_cpu(vals, ids, temperature, top_k, top_p, min_p, seeds, step, want_probs):
    B, K = vals.shape
    gen = torch.Generator()
    res = []
    pr = []
    for b in range(B):
        T = float(temperature[b])
        if T <= 0:
            res.append(int(ids[b, 0]))
            pr.append(torch.nn.functional.one_hot(torch.tensor(0), K).float())
            continue
        lg = vals[b].float() / T
        masked = ref.apply_top_k_top_p(lg[None], top_k[b:b + 1], top_p[b:b + 1],
                                       None if min_p is None else min_p[b:b + 1])[0]
        p = torch.softmax(masked, -1)
        gen.manual_seed(int(seeds[b]) * 1000003 + step)
        res.append(int(ids[b, torch.multinomial(p, 1, generator=gen)]))
        pr.append(p)
    out = torch.tensor(res, dtype=torch.int64)
    return out, (torch.stack(pr) if want_probs else None)


TOPK_WINDOW = 64


def topk_window(logits: torch.Tensor):
    """Top-64 window of each row: (values [B, 64] fp32 descending, ids [B, 64] int64).  Ties
    resolve to the lowest column."""
    B, V = logits.shape
    if not logits.is_cuda:
        vals, ids = torch.topk(logits.float(), min(TOPK_WINDOW, V), dim=-1)
        return vals, ids
    vals = torch.empty(B, TOPK_WINDOW, dtype=torch.float32, device=logits.device)
    ids = torch.empty(B, TOPK_WINDOW, dtype=torch.int64, device=logits.device)
    e = _empty(logits.device)
    ext().topk_window(logits, vals, ids, _topk_ws(logits), e, e, e, e, e, 0, e, e)
    return vals, ids


def _topk_ws(logits):
    B, V = logits.shape
    nch = (V + 4095) // 4096
    return workspace(logits.device, "topk", 4096 + B * nch * TOPK_WINDOW * 2)


def topk_sample(logits, temperature, top_k, top_p, min_p, seeds, step: int,
                want_probs: bool = False):
    """One launch: the top-64 window of each row and the row's draw from it (temperature, top-k
    <= 64, top-p, min-p; Philox stream per (seed, step)).  -> (tokens [B], window probs or None,
    window ids [B, 64])."""
    B, V = logits.shape
    if not logits.is_cuda:
        vals, ids = topk_window(logits)
        toks, probs = sample_from_topk(vals, ids, temperature, top_k, top_p, min_p, seeds, step,
                                       want_probs)
        return toks, probs, ids
    dev = logits.device
    ids = torch.empty(B, TOPK_WINDOW, dtype=torch.int64, device=dev)
    toks = torch.empty(B, dtype=torch.int64, device=dev)
    probs = torch.empty(B, TOPK_WINDOW, dtype=torch.float32, device=dev) if want_probs else None
    ext().topk_window(logits, _empty(dev), ids, _topk_ws(logits), temperature, top_k, top_p,
                      _none(min_p, dev), seeds, step, toks, _none(probs, dev))
    return toks, probs, ids
