"""INT4 (W4A16) weight container: g128 asymmetric int4 with fp16 scales and uint8 zero points.

Canonical layout: ``packed`` uint8 [N, K/2] (low nibble = even k), ``scales`` fp16 [N, K/128],
``zeros`` uint8 [N, K/128]; w[n, k] = (q - zero) * scale.  This is the compressed-tensors
``pack-quantized`` int4 format after unpacking its int32 words, the format of the reference's INT4
targets, DFlash2 drafter weights and int4 lm_head (``sly/patch_w4a16_tiles.py``,
``sly/mxfp4/radiance_lmhead_int4.py:92-349``).  On the GPU the weight is re-laid once into
tensor-core fragment order (``mma_tile``, consumed by ``csrc/w4a16.cu``).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch

from .formats import int4_g128_dequantize, int4_g128_quantize, pack_nibbles, unpack_nibbles

GROUP = 128


def mma_tile(packed: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor):
    """Canonical [N, K/2] / [N, K/128] int4 -> the tensor-core fragment layout of the CUDA kernels.

    Rows are padded to a multiple of 16 (zero scale).  Weights: uint8 [Np, K/2] holding, for each
    16-row tile T and 64-column block kb, 32 lanes x 4 steps of one 32-bit word, in which nibble
    i = h + 2c + 4p is w[16T + 8h + g, 64kb + 16t + 4s + 2c + p] for lane = 4g + t and step s.
    That word, split by (shift, mask, or 0x4300), is the lane's mma.m16n8k16 A fragment of step
    s (k permuted consistently with the activation fragment, which the dot product allows).
    Scales/zeros: int32 [Np/16, K/128, 8, 2]: word 0 = fp16x2 (s[g], s[g+8]), word 1 =
    bf16x2 bits (128 + z[g], 128 + z[g+8])."""
    N, K2 = packed.shape
    K = K2 * 2
    Np = (N + 15) // 16 * 16
    q = unpack_nibbles(packed)
    sc = scales.half()
    z = zeros.to(torch.int32)
    if Np != N:
        q = torch.cat([q, q.new_zeros(Np - N, K)])
        sc = torch.cat([sc, sc.new_zeros(Np - N, sc.shape[1])])
        z = torch.cat([z, z.new_zeros(Np - N, z.shape[1])])
    T, KB, NG = Np // 16, K // 64, K // GROUP
    qt = q.view(T, 2, 8, KB, 4, 4, 2, 2).permute(0, 3, 2, 4, 5, 7, 6, 1).reshape(Np, K)
    wt = pack_nibbles(qt).contiguous()
    s2 = sc.view(T, 2, 8, NG).permute(0, 3, 2, 1).contiguous()            # [T, NG, 8, 2] fp16
    z2 = (z + 0x4300).view(T, 2, 8, NG).permute(0, 3, 2, 1)
    sw = s2.view(torch.int16).to(torch.int32) & 0xFFFF
    zw = z2[..., 0] | (z2[..., 1] << 16)
    sz = torch.stack([sw[..., 0] | (sw[..., 1] << 16), zw], -1).contiguous()
    return wt, sz


def mma_untile(wt: torch.Tensor, sz: torch.Tensor, N: int, K: int):
    """Inverse of ``mma_tile`` (canonical packed, scales, zeros)."""
    Np = wt.shape[0]
    T, KB, NG = Np // 16, K // 64, K // GROUP
    qt = unpack_nibbles(wt).view(T, KB, 8, 4, 4, 2, 2, 2)
    q = qt.permute(0, 7, 2, 1, 3, 4, 6, 5).reshape(Np, K)[:N]
    sw = sz[..., 0]
    s2 = torch.stack([sw & 0xFFFF, (sw >> 16) & 0xFFFF], -1).to(torch.int16).view(torch.float16)
    scales = s2.permute(0, 3, 2, 1).reshape(Np, NG)[:N]
    zw = sz[..., 1]
    z2 = torch.stack([zw & 0xFFFF, (zw >> 16) & 0xFFFF], -1) - 0x4300
    zeros = z2.permute(0, 3, 2, 1).reshape(Np, NG)[:N].to(torch.uint8)
    return pack_nibbles(q), scales.contiguous(), zeros.contiguous()


@dataclass
class Int4Weight:
    """On a CUDA device the weight lives in the fragment layout of ``mma_tile`` (``packed`` =
    tiled nibbles, ``sz`` = tiled scales and zeros; ``scales``/``zeros`` are None); on the host it
    is canonical."""
    packed: torch.Tensor                  # uint8 [N, K/2] (canonical) or [Np, K/2] (tiled)
    scales: Optional[torch.Tensor]        # fp16 [N, K/128] (canonical only)
    zeros: Optional[torch.Tensor]         # uint8 [N, K/128] (canonical only)
    N: int
    K: int
    sz: Optional[torch.Tensor] = None     # int32 [Np/16, K/128, 8, 2] (tiled only)

    @property
    def tiled(self) -> bool:
        return self.sz is not None

    @staticmethod
    def from_float(w: torch.Tensor, clip_search: bool = False) -> "Int4Weight":
        """Quantise [N, K] (K % 128 == 0).  With clip_search, each group's range is shrunk by the
        factor (1.0, 0.95, ..., 0.75) that minimises its squared reconstruction error, as the
        reference's int4 lm_head builder does (MSE clip search).  A CUDA input gives a tiled
        weight."""
        N, K = w.shape
        if K % GROUP != 0:
            raise ValueError(f"INT4 g128 needs K % 128 == 0 (got {K})")
        if not clip_search:
            p, s, z = int4_g128_quantize(w)
            return Int4Weight(p.contiguous(), s.contiguous(), z.contiguous(), N, K)._placed()
        wg = w.float().view(N, K // GROUP, GROUP)
        best = None
        for f in (1.0, 0.95, 0.9, 0.85, 0.8, 0.75):
            lo = wg.amin(-1) * f
            hi = wg.amax(-1) * f
            scale = ((hi - lo) / 15.0).clamp(min=1e-8)
            zero = torch.round(-lo / scale).clamp(0, 15)
            q = torch.round(wg / scale[..., None] + zero[..., None]).clamp(0, 15)
            err = (((q - zero[..., None]) * scale[..., None] - wg) ** 2).sum(-1)
            if best is None:
                best = (err, q, scale, zero)
            else:
                m = err < best[0]
                best = (torch.where(m, err, best[0]), torch.where(m[..., None], q, best[1]),
                        torch.where(m, scale, best[2]), torch.where(m, zero, best[3]))
        _, q, scale, zero = best
        packed = pack_nibbles(q.to(torch.uint8).view(N, K))
        return Int4Weight(packed.contiguous(), scale.half().contiguous(),
                          zero.to(torch.uint8).contiguous(), N, K)._placed()

    def _placed(self) -> "Int4Weight":
        if self.packed.is_cuda and not self.tiled:
            wt, sz = mma_tile(self.packed, self.scales, self.zeros)
            return Int4Weight(wt, None, None, self.N, self.K, sz)
        return self

    def canonical(self):
        """(packed, scales, zeros) in the canonical layout."""
        if self.tiled:
            return mma_untile(self.packed, self.sz, self.N, self.K)
        return self.packed, self.scales, self.zeros

    def dequantize(self) -> torch.Tensor:
        return int4_g128_dequantize(*self.canonical(), GROUP)

    def to(self, device) -> "Int4Weight":
        p, s, z = self.canonical()
        return Int4Weight(p.to(device), s.to(device), z.to(device), self.N, self.K)._placed()

    # ---- sharding / merging on the canonical codes (checkpoint weights stay int4) ----
    def narrow_rows(self, start: int, length: int) -> "Int4Weight":
        p, s, z = self.canonical()
        return Int4Weight(p[start:start + length].contiguous(), s[start:start + length].contiguous(),
                          z[start:start + length].contiguous(), length, self.K)

    def narrow_cols(self, start: int, length: int) -> "Int4Weight":
        """K slice (row-parallel shard); start / length multiples of the 128-column group."""
        assert start % GROUP == 0 and length % GROUP == 0 and start + length <= self.K
        p, s, z = self.canonical()
        g0, ng = start // GROUP, length // GROUP
        return Int4Weight(p[:, start // 2:(start + length) // 2].contiguous(),
                          s[:, g0:g0 + ng].contiguous(), z[:, g0:g0 + ng].contiguous(),
                          self.N, length)

    def index_rows(self, idx: torch.Tensor) -> "Int4Weight":
        p, s, z = self.canonical()
        return Int4Weight(p[idx].contiguous(), s[idx].contiguous(), z[idx].contiguous(),
                          int(idx.numel()), self.K)

    @property
    def nbytes(self) -> int:
        if self.tiled:
            return self.packed.numel() + self.sz.numel() * 4
        return self.packed.numel() + self.scales.numel() * 2 + self.zeros.numel()


def cat_rows(ws: list) -> Int4Weight:
    """Merged linear (qkv, gate_up): concatenate along N."""
    assert all(w.K == ws[0].K for w in ws)
    parts = [w.canonical() for w in ws]
    return Int4Weight(torch.cat([p for p, _, _ in parts]), torch.cat([s for _, s, _ in parts]),
                      torch.cat([z for _, _, z in parts]), sum(w.N for w in ws), ws[0].K)


def w4a16_linear(x: torch.Tensor, w: Int4Weight, row_block: int = 16384) -> torch.Tensor:
    """y = x w^T for bf16 x [M, K].  CUDA: the int4 tensor-core GEMV kernel for M <= 8, else row
    blocks of the weight expanded to bf16 and multiplied by the library GEMM; CPU: fp32
    reference."""
    if not x.is_cuda:
        return (x.float() @ w.dequantize().t()).to(torch.bfloat16)
    from ..ops._ext import ext
    from ..ops.kernels import status_word
    M = x.shape[0]
    x = x.to(torch.bfloat16).contiguous()
    out = torch.empty(M, w.N, dtype=torch.bfloat16, device=x.device)
    if M <= 8:
        ext().w4a16_gemv(x, w.packed, w.sz, out, status_word(x.device))
        return out
    rb = min(row_block, (w.N + 15) // 16 * 16)
    tmp = torch.empty(rb, w.K, dtype=torch.bfloat16, device=x.device)
    for n0 in range(0, w.N, rb):
        n = min(rb, w.N - n0)
        ext().w4a16_dequant(w.packed, w.sz, n0, tmp[:n])
        torch.matmul(x, tmp[:n].t(), out=out[:, n0:n0 + n])
    return out
