"""Number formats used by the engine, as exact torch (CPU or GPU) codecs.

* MXFP4 (OCP MX v1.0): E2M1 elements, one UE8M0 scale per 32 consecutive K elements.
  Scale rule: byte = clamp(floor(log2(amax)) - 2 + 127, 0, 254), byte 0 for an all-zero block
  (reference: ``sly/kvq/reference.py:23-33``).  Elements round to nearest, ties to even code,
  saturating at 6.  Packing: low nibble = even K index (``sly/mxfp4/radiance_mxfp4_fp8.hip:18-23``).
* fp8 E4M3 per-token activations: scale = max(amax/448, 1/(448*512)),
  q = e4m3_rne(clamp(x/scale, +-448))  (``sly/mxfp4/radiance_mxfp4_fp8.hip:1715-1730``).
* NVFP4: E2M1 + E4M3 scale per 16 + fp32 global scale, requantized to MXFP4 at load
  (``radiance_nvfp4.py:114-189``).
* INT4 g128 (W4A16): symmetric or asymmetric group-128 integer weights.
"""
from __future__ import annotations

import torch

E2M1_VALUES = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=torch.float32)
E2M1_LUT = torch.cat([E2M1_VALUES, -E2M1_VALUES])          # code 0..15, bit 3 = sign
FP8_MAX = 448.0
FP8_SCALE_FLOOR = 1.0 / (448.0 * 512.0)
MX_BLOCK = 32


# ---------------------------------------------------------------------------------------------
# E2M1
# ---------------------------------------------------------------------------------------------
def e2m1_encode(x: torch.Tensor) -> torch.Tensor:
    """float -> 4-bit code (uint8 0..15), round-to-nearest-even on the E2M1 grid, saturating."""
    a = x.abs().float()
    # midpoints between consecutive magnitudes: 0.25 0.75 1.25 1.75 2.5 3.5 5
    # ties go to the even code (codes 0,2,4,6 have an even mantissa bit)
    mags = E2M1_VALUES.to(x.device)
    mids = (mags[:-1] + mags[1:]) / 2
    idx = torch.bucketize(a, mids, right=False)              # a <= mid -> lower index
    # exact tie: bucketize(right=False) puts a==mid in the lower bucket; move to the even code
    tie = (a.unsqueeze(-1) == mids).any(-1)
    lower = torch.bucketize(a, mids, right=False)
    even_up = (lower % 2 == 1)                                # lower code odd -> upper is even
    idx = torch.where(tie & even_up, lower + 1, idx)
    idx = idx.clamp(max=7).to(torch.uint8)
    sign = (x < 0) & (idx > 0)
    return idx | (sign.to(torch.uint8) << 3)


def e2m1_decode(code: torch.Tensor) -> torch.Tensor:
    return E2M1_LUT.to(code.device)[code.long()]


def pack_nibbles(codes: torch.Tensor) -> torch.Tensor:
    """[..., K] uint8 codes -> [..., K/2] bytes, low nibble = even index."""
    lo = codes[..., 0::2]
    hi = codes[..., 1::2]
    return (lo | (hi << 4)).to(torch.uint8)


def unpack_nibbles(packed: torch.Tensor) -> torch.Tensor:
    lo = packed & 0xF
    hi = packed >> 4
    return torch.stack([lo, hi], dim=-1).flatten(-2)


# ---------------------------------------------------------------------------------------------
# UE8M0 / MXFP4
# ---------------------------------------------------------------------------------------------
def ue8m0_ocp(amax: torch.Tensor) -> torch.Tensor:
    """OCP shared-scale byte per block: floor(log2 amax) - 2 (E2M1 emax), biased by 127."""
    a = amax.double()
    _, e = torch.frexp(a)                                      # a = m*2^e, m in [0.5,1)
    s = (e.long() - 1 - 2 + 127).clamp(0, 254)
    s = torch.where(a == 0, torch.zeros_like(s), s)
    return s.to(torch.uint8)


def ue8m0_to_float(b: torch.Tensor) -> torch.Tensor:
    return torch.exp2(b.float() - 127.0)


def mxfp4_quantize(w: torch.Tensor):
    """w [N, K] (K % 32 == 0) -> (packed uint8 [N, K/2], scales uint8 [N, K/32])."""
    N, K = w.shape
    assert K % MX_BLOCK == 0, K
    wb = w.float().view(N, K // MX_BLOCK, MX_BLOCK)
    sb = ue8m0_ocp(wb.abs().amax(-1))
    scale = ue8m0_to_float(sb).unsqueeze(-1)
    codes = e2m1_encode(wb / scale).view(N, K)
    return pack_nibbles(codes), sb


def mxfp4_dequantize(packed: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    N = packed.shape[0]
    K = packed.shape[1] * 2
    vals = e2m1_decode(unpack_nibbles(packed)).view(N, K // MX_BLOCK, MX_BLOCK)
    return (vals * ue8m0_to_float(scales).unsqueeze(-1)).view(N, K)


# ---------------------------------------------------------------------------------------------
# MXFP6 (E2M3) and MXFP8 (E4M3) weights: the other element types of tcgen05 kind::mxf8f6f4
# ---------------------------------------------------------------------------------------------
# E2M3: sign bit 5, 2 exponent bits (bias 1), 3 mantissa bits; magnitudes k/8 for k < 8, then
# (8 + m)/8 * 2^(e-1): 1 .. 7.5.  OCP shared scale: floor(log2 amax) - 2 (emax 2), as E2M1.
E2M3_VALUES = torch.tensor([i / 8 for i in range(8)] + [(8 + m) / 8 * 2.0 ** (e - 1)
                                                        for e in (1, 2, 3) for m in range(8)])


def e2m3_encode(x: torch.Tensor) -> torch.Tensor:
    """float -> 6-bit code (uint8 0..63), round to nearest on the E2M3 grid (ties to the even
    code), saturating at 7.5."""
    a = x.abs().float().clamp(max=7.5)
    mags = E2M3_VALUES.to(x.device)
    mids = (mags[:-1] + mags[1:]) / 2
    lower = torch.bucketize(a, mids, right=False)
    tie = (a.unsqueeze(-1) == mids).any(-1)
    idx = torch.where(tie & (lower % 2 == 1), lower + 1, lower).clamp(max=31).to(torch.uint8)
    sign = (x < 0) & (idx > 0)
    return idx | (sign.to(torch.uint8) << 5)


def e2m3_decode(code: torch.Tensor) -> torch.Tensor:
    c = code.long()
    mag = E2M3_VALUES.to(code.device)[c & 31]
    return torch.where((c & 32) != 0, -mag, mag)


def pack_6bit(codes: torch.Tensor) -> torch.Tensor:
    """[..., K] 6-bit codes (K % 4 == 0) -> [..., 3K/4] bytes: four codes per three bytes, code i
    of a group at bits [6i, 6i + 6) of the little-endian 24-bit word (the reference's MXFP6
    checkpoint packing, and 16 codes per 12 bytes as TMA's 16U6 type reads them)."""
    c = codes.to(torch.int32).view(*codes.shape[:-1], -1, 4)
    w = c[..., 0] | (c[..., 1] << 6) | (c[..., 2] << 12) | (c[..., 3] << 18)
    b = torch.stack([w & 255, (w >> 8) & 255, (w >> 16) & 255], -1)
    return b.to(torch.uint8).view(*codes.shape[:-1], -1)


def unpack_6bit(packed: torch.Tensor) -> torch.Tensor:
    t = packed.to(torch.int32).view(*packed.shape[:-1], -1, 3)
    w = t[..., 0] | (t[..., 1] << 8) | (t[..., 2] << 16)
    return torch.stack([(w >> (6 * i)) & 63 for i in range(4)], -1).view(
        *packed.shape[:-1], -1).to(torch.uint8)


def ue8m0_for(amax: torch.Tensor, emax: int) -> torch.Tensor:
    """OCP shared-scale byte: floor(log2 amax) - emax of the element type, biased by 127."""
    a = amax.double()
    _, e = torch.frexp(a)
    s = (e.long() - 1 - emax + 127).clamp(0, 254)
    return torch.where(a == 0, torch.zeros_like(s), s).to(torch.uint8)


def ue8m0_ceil(amax: torch.Tensor, vmax: float) -> torch.Tensor:
    """Smallest power-of-two scale with amax / scale <= vmax (no element saturates), biased."""
    x = amax.double() / vmax
    m, e = torch.frexp(x)                       # x = m * 2^e, m in [0.5, 1)
    s = (e.long() - (m == 0.5).long() + 127).clamp(0, 254)
    return torch.where(amax == 0, torch.zeros_like(s), s).to(torch.uint8)


def mx_quantize(w: torch.Tensor, fmt: str):
    """w [N, K] -> (packed, UE8M0 scales [N, K/32]) for fmt e2m1 (MXFP4, [N, K/2]), e2m3 (MXFP6,
    [N, 3K/4]) or e4m3 (MXFP8, [N, K] bytes).  e2m1 / e2m3 take the OCP scale floor(log2 amax) -
    emax (the block maximum may round down to the largest code); e4m3 takes the smallest scale
    that does not saturate, since the OCP rule would clip up to 12 % off a block's largest
    values there (amax / scale reaches 511 against a largest code of 448)."""
    if fmt == "e2m1":
        return mxfp4_quantize(w)
    N, K = w.shape
    assert K % MX_BLOCK == 0, K
    wb = w.float().view(N, K // MX_BLOCK, MX_BLOCK)
    amax = wb.abs().amax(-1)
    sb = ue8m0_for(amax, 2) if fmt == "e2m3" else ue8m0_ceil(amax, 448.0)
    x = (wb / ue8m0_to_float(sb).unsqueeze(-1)).view(N, K)
    if fmt == "e2m3":
        return pack_6bit(e2m3_encode(x)), sb
    if fmt == "e4m3":
        return fp8_e4m3(x).view(torch.uint8), sb
    raise ValueError(fmt)


def mx_dequantize(packed: torch.Tensor, scales: torch.Tensor, fmt: str) -> torch.Tensor:
    if fmt == "e2m1":
        return mxfp4_dequantize(packed, scales)
    N = packed.shape[0]
    if fmt == "e2m3":
        vals = e2m3_decode(unpack_6bit(packed))
    else:
        vals = packed.view(torch.float8_e4m3fn).float()
    K = vals.shape[1]
    return (vals.view(N, K // MX_BLOCK, MX_BLOCK) * ue8m0_to_float(scales).unsqueeze(-1)).view(N, K)


MX_BITS = {"e2m1": 4, "e2m3": 6, "e4m3": 8}


# ---------------------------------------------------------------------------------------------
# fp8 e4m3 per-token activations
# ---------------------------------------------------------------------------------------------
def fp8_e4m3(x: torch.Tensor) -> torch.Tensor:
    """RNE to e4m3fn with saturation at +-448 (torch's cast is non-saturating)."""
    return x.float().clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn)


def per_token_fp8(x: torch.Tensor):
    """x [M, K] -> (q fp8 [M, K], scale fp32 [M]).  amax is taken over the bf16-rounded row."""
    xf = x.to(torch.bfloat16).float()
    amax = xf.abs().amax(-1)
    scale = torch.clamp(amax / FP8_MAX, min=FP8_SCALE_FLOOR)
    q = fp8_e4m3(xf / scale.unsqueeze(-1))
    return q, scale


def per_token_fp8_dequant(q: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    return q.float() * scale.unsqueeze(-1)


# ---------------------------------------------------------------------------------------------
# NVFP4 -> MXFP4 requantization
# ---------------------------------------------------------------------------------------------
def nvfp4_quantize(w: torch.Tensor):
    """Reference NVFP4 encoder (for tests / synthetic checkpoints): e2m1 + e4m3 scale per 16
    + fp32 global scale.  Returns (packed [N,K/2], block_scales e4m3 [N,K/16], global fp32)."""
    N, K = w.shape
    wb = w.float().view(N, K // 16, 16)
    amax = wb.abs().amax(-1)
    gscale = (w.float().abs().max() / (6.0 * 448.0)).clamp(min=1e-12)
    bs = fp8_e4m3(amax / 6.0 / gscale)
    eff = bs.float() * gscale
    eff = torch.where(eff == 0, torch.ones_like(eff), eff)
    codes = e2m1_encode(wb / eff.unsqueeze(-1)).view(N, K)
    return pack_nibbles(codes), bs, gscale.float()


def nvfp4_dequantize(packed, block_scales, gscale):
    N = packed.shape[0]
    K = packed.shape[1] * 2
    vals = e2m1_decode(unpack_nibbles(packed)).view(N, K // 16, 16)
    return (vals * (block_scales.float() * gscale).unsqueeze(-1)).view(N, K)


def nvfp4_to_mxfp4(packed, block_scales, gscale):
    """Requantize an NVFP4 tensor into MXFP4 (the reference's 'ocp' exponent mode:
    dequantize to fp32, then OCP MXFP4 quantization per 32)."""
    return mxfp4_quantize(nvfp4_dequantize(packed, block_scales, gscale))


# ---------------------------------------------------------------------------------------------
# INT4 group-128 (W4A16)
# ---------------------------------------------------------------------------------------------
def int4_g128_quantize(w: torch.Tensor, group: int = 128, symmetric: bool = False):
    """w [N,K] -> (packed uint8 [N,K/2] low nibble even, scales fp16 [N,K/g], zeros uint8 [N,K/g])."""
    N, K = w.shape
    wg = w.float().view(N, K // group, group)
    if symmetric:
        amax = wg.abs().amax(-1).clamp(min=1e-8)
        scale = amax / 7.0
        zero = torch.full_like(scale, 8.0)
    else:
        lo = wg.amin(-1)
        hi = wg.amax(-1)
        scale = ((hi - lo) / 15.0).clamp(min=1e-8)
        zero = torch.round(-lo / scale).clamp(0, 15)
    q = torch.round(wg / scale.unsqueeze(-1) + zero.unsqueeze(-1)).clamp(0, 15).to(torch.uint8)
    return pack_nibbles(q.view(N, K)), scale.half(), zero.to(torch.uint8)


def int4_g128_dequantize(packed, scales, zeros, group: int = 128):
    N = packed.shape[0]
    K = packed.shape[1] * 2
    q = unpack_nibbles(packed).float().view(N, K // group, group)
    return ((q - zeros.float().unsqueeze(-1)) * scales.float().unsqueeze(-1)).view(N, K)


# ---------------------------------------------------------------------------------------------
# tcgen05 scale-factor tile layout
# ---------------------------------------------------------------------------------------------
def sf_tile_layout(scales: torch.Tensor) -> torch.Tensor:
    """[N, K/32] UE8M0 bytes -> the block-scaled MMA scale-factor tile layout.

    The tensor core reads per-32 scales from tensor memory in 128-row x 4-block atoms
    (512 bytes): byte (n % 32) * 16 + ((n % 128) // 32) * 4 + (kb % 4) of atom
    (n // 128, kb // 4), atoms ordered with the K atom index fastest.  Rows are padded to a
    multiple of 128 (pad bytes 127 = 1.0) and K blocks to a multiple of 4.  One atom is one
    TMA-free 512-byte bulk copy per 128x128 weight tile, so the weight loader writes this
    layout once at load time (the analogue of the reference's PSW repack, ``psw_fold_ws``)."""
    N, KB = scales.shape
    Np = (N + 127) // 128 * 128
    KBp = (KB + 3) // 4 * 4
    s = torch.full((Np, KBp), 127, dtype=torch.uint8, device=scales.device)
    s[:N, :KB] = scales
    # [Np/128, 4(m/32), 32(m%32), KBp/4, 4(kb%4)] -> [Np/128, KBp/4, 32, 4, 4]
    s = s.view(Np // 128, 4, 32, KBp // 4, 4).permute(0, 3, 2, 1, 4).contiguous()
    return s.view(-1)


def sf_tile_layout_inverse(tiled: torch.Tensor, N: int, KB: int) -> torch.Tensor:
    Np = (N + 127) // 128 * 128
    KBp = (KB + 3) // 4 * 4
    s = tiled.view(Np // 128, KBp // 4, 32, 4, 4).permute(0, 3, 2, 1, 4).contiguous()
    return s.view(Np, KBp)[:N, :KB]


# ---------------------------------------------------------------------------------------------
# 4-bit KV cache (int4, fp16 scale + zero per 16 elements per head)
# ---------------------------------------------------------------------------------------------
KV4_GROUP = 16


def kv4_row_bytes(head_dim: int) -> int:
    """Bytes of one (token, kv-head) row: head_dim/2 nibble bytes + (scale, zero) fp16 pairs."""
    return head_dim // 2 + (head_dim // KV4_GROUP) * 4


def kv4_quantize(x: torch.Tensor) -> torch.Tensor:
    """x [..., D] -> uint8 rows [..., kv4_row_bytes(D)]: asymmetric 4-bit per 16-element group,
    zero = group min, scale = (max - min) / 15 (1 when flat), both stored as fp16."""
    D = x.shape[-1]
    g = x.float().reshape(*x.shape[:-1], D // KV4_GROUP, KV4_GROUP)
    lo = g.amin(-1)
    hi = g.amax(-1)
    scale = ((hi - lo) / 15.0)
    scale = torch.where(scale > 0, scale, torch.ones_like(scale)).half()
    lo16 = lo.half()
    q = torch.round((g - lo16.float().unsqueeze(-1)) / scale.float().unsqueeze(-1)).clamp(0, 15)
    q = q.to(torch.uint8).reshape(*x.shape[:-1], D)
    packed = pack_nibbles(q)
    meta = torch.stack([scale, lo16], -1).reshape(*x.shape[:-1], -1).contiguous().view(torch.uint8)
    return torch.cat([packed, meta], -1)


def kv4_dequantize(rows: torch.Tensor, D: int) -> torch.Tensor:
    data = rows[..., :D // 2]
    meta = rows[..., D // 2:].contiguous().view(torch.float16).reshape(*rows.shape[:-1], D // KV4_GROUP, 2)
    q = unpack_nibbles(data).float().reshape(*rows.shape[:-1], D // KV4_GROUP, KV4_GROUP)
    return (q * meta[..., 0:1].float() + meta[..., 1:2].float()).reshape(*rows.shape[:-1], D)
