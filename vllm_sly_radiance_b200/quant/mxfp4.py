"""MX weight container (MXFP4 / MXFP6 / MXFP8) for the block-scaled linears.

Layout contract (what the tcgen05 block-scaled GEMM consumes):
  * ``packed``  uint8, row-major, one of
      - ``e2m1`` (MXFP4): [N, K/2], low nibble = even K index (TMA type 16U4_ALIGN16B);
      - ``e2m3`` (MXFP6): [N, 3K/4], four 6-bit codes per three bytes, code i of a group at
        bits [6i, 6i + 6) of the little-endian 24-bit word (TMA type 16U6_ALIGN16B);
      - ``e4m3`` (MXFP8): [N, K] fp8 bytes (TMA type UINT8).
    TMA expands each 16-value group to 16 bytes in shared memory (the padded form the f8f6f4
    MMA reads), so there is no repack of the payload for any of them.
  * ``sf``      uint8, scale factors in the 128-row x 4-block atom order of
    ``formats.sf_tile_layout`` (one 512-byte bulk copy per 128x128 weight tile).
  * ``scales``  uint8 [N, K/32] plain UE8M0 bytes, kept for loaders / references.

The reference's load-time transforms (scale transpose, row reference exponent, WPERM fragment
permute, PSW preshuffle: ``sly/mxfp4/radiance_mxfp4.py:1039-1175``) collapse into this single
scale relayout because the B200 tensor core applies the per-32 scales natively.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch

from .formats import MX_BITS, mx_dequantize, mx_quantize, sf_tile_layout


KPAD = 128   # the GEMM's K tile: stored weights are zero-padded to a multiple of it


def col_bytes(k: int, fmt: str) -> int:
    """Bytes that k input features (a multiple of 32) take in a packed row of format fmt."""
    return k * MX_BITS[fmt] // 8


@dataclass
class MXFP4Weight:
    packed: torch.Tensor          # uint8 [N, Kp * bits / 8], Kp = K rounded up to KPAD (zero tail)
    scales: torch.Tensor          # uint8 [N, Kp/32]
    sf: torch.Tensor              # uint8 tiled scale factors
    N: int
    K: int                        # logical input features (a multiple of 32)
    fmt: str = "e2m1"             # element type: e2m1 (MXFP4), e2m3 (MXFP6), e4m3 (MXFP8)

    @staticmethod
    def from_float(w: torch.Tensor, fmt: str = "e2m1") -> "MXFP4Weight":
        N, K = w.shape
        if K % 32 != 0:
            raise ValueError(f"MX linear needs K % 32 == 0 (got K={K})")
        packed, scales = mx_quantize(w, fmt)
        return MXFP4Weight.from_packed(packed, scales, fmt=fmt)

    @staticmethod
    def from_packed(packed: torch.Tensor, scales: torch.Tensor, K: Optional[int] = None,
                    fmt: str = "e2m1") -> "MXFP4Weight":
        """packed [N, Kc * bits / 8] / scales [N, Kc/32] with Kc >= K; columns beyond K must be
        zero.  A tail that does not fill a whole K tile is zero-padded here (a row-parallel shard
        such as 8704 / 8 = 1088 input features), so the GEMM only ever reads whole tiles of
        weights.  Code 0 is +0 in all three element types."""
        N, Kb = packed.shape
        Kc = Kb * 8 // MX_BITS[fmt]
        K = Kc if K is None else K
        assert scales.shape == (N, Kc // 32) and K <= Kc and K % 32 == 0, (scales.shape, N, K, Kc)
        Kp = (K + KPAD - 1) // KPAD * KPAD
        if Kc != Kp:
            pk = torch.zeros(N, col_bytes(Kp, fmt), dtype=torch.uint8, device=packed.device)
            sc = torch.full((N, Kp // 32), 127, dtype=torch.uint8, device=scales.device)
            pk[:, :col_bytes(K, fmt)] = packed[:, :col_bytes(K, fmt)]
            sc[:, :K // 32] = scales[:, :K // 32]
            packed, scales = pk, sc
        return MXFP4Weight(packed.contiguous(), scales.contiguous(),
                           sf_tile_layout(scales), N, K, fmt)

    @staticmethod
    def zeros(n: int, K: int, fmt: str = "e2m1", device=None) -> "MXFP4Weight":
        """n rows of zero weights (padding rows of a TP shard); the zero block's scale is 2^0."""
        return MXFP4Weight.from_packed(
            torch.zeros(n, col_bytes(K, fmt), dtype=torch.uint8, device=device),
            torch.full((n, K // 32), 127, dtype=torch.uint8, device=device), K, fmt)

    @property
    def K_padded(self) -> int:
        return self.packed.shape[1] * 8 // MX_BITS[self.fmt]

    def dequantize(self) -> torch.Tensor:
        return mx_dequantize(self.packed[:, :col_bytes(self.K, self.fmt)],
                             self.scales[:, :self.K // 32], self.fmt)

    def to(self, device) -> "MXFP4Weight":
        return MXFP4Weight(self.packed.to(device), self.scales.to(device), self.sf.to(device),
                           self.N, self.K, self.fmt)

    def narrow_rows(self, start: int, length: int) -> "MXFP4Weight":
        """Row slice (output-feature shard for column-parallel TP)."""
        return MXFP4Weight.from_packed(self.packed[start:start + length],
                                       self.scales[start:start + length], self.K, self.fmt)

    def narrow_cols(self, start: int, length: int) -> "MXFP4Weight":
        """K slice (input-feature shard for row-parallel TP); start/length multiples of 32."""
        assert start % 32 == 0 and length % 32 == 0 and start + length <= self.K
        b0, b1 = col_bytes(start, self.fmt), col_bytes(start + length, self.fmt)
        return MXFP4Weight.from_packed(self.packed[:, b0:b1],
                                       self.scales[:, start // 32:(start + length) // 32],
                                       fmt=self.fmt)

    def pad_cols(self, K_new: int) -> "MXFP4Weight":
        """Zero input features appended (dummy heads / channels of a row-parallel linear)."""
        if K_new == self.K:
            return self
        assert K_new > self.K and (K_new - self.K) % 32 == 0
        dev = self.packed.device
        pk = torch.cat([self.packed[:, :col_bytes(self.K, self.fmt)],
                        torch.zeros(self.N, col_bytes(K_new - self.K, self.fmt), dtype=torch.uint8,
                                    device=dev)], 1)
        sc = torch.cat([self.scales[:, :self.K // 32],
                        torch.full((self.N, (K_new - self.K) // 32), 127, dtype=torch.uint8,
                                   device=dev)], 1)
        return MXFP4Weight.from_packed(pk, sc, K_new, self.fmt)

    @property
    def nbytes(self) -> int:
        return self.packed.numel() + self.sf.numel()


MXWeight = MXFP4Weight


def cat_rows(ws: list[MXFP4Weight]) -> MXFP4Weight:
    """Merged linear (qkvz+ba, gate_up): concatenate along N."""
    assert all(w.K == ws[0].K and w.fmt == ws[0].fmt for w in ws)
    return MXFP4Weight.from_packed(torch.cat([w.packed for w in ws], 0),
                                   torch.cat([w.scales for w in ws], 0), ws[0].K, ws[0].fmt)
