"""MXFP4 weight container for the W4A8 linears.

Layout contract (what the tcgen05 block-scaled GEMM consumes):
  * ``packed``  uint8 [N, K/2], row-major, low nibble = even K index.  The GEMM loads it with a
    TMA map of type 16U4_ALIGN16B, which expands each 16-value group to 16 bytes in shared
    memory (the padded e2m1 form the f8f6f4 MMA reads), so there is no repack of the payload.
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

from .formats import (mxfp4_dequantize, mxfp4_quantize, sf_tile_layout)


KPAD = 128   # the GEMM's K tile: stored weights are zero-padded to a multiple of it


@dataclass
class MXFP4Weight:
    packed: torch.Tensor          # uint8 [N, Kp/2], Kp = K rounded up to KPAD (zero tail)
    scales: torch.Tensor          # uint8 [N, Kp/32]
    sf: torch.Tensor              # uint8 tiled scale factors
    N: int
    K: int                        # logical input features (a multiple of 32)

    @staticmethod
    def from_float(w: torch.Tensor) -> "MXFP4Weight":
        N, K = w.shape
        if K % 32 != 0:
            raise ValueError(f"MXFP4 linear needs K % 32 == 0 (got K={K})")
        packed, scales = mxfp4_quantize(w)
        return MXFP4Weight.from_packed(packed, scales)

    @staticmethod
    def from_packed(packed: torch.Tensor, scales: torch.Tensor, K: Optional[int] = None) -> "MXFP4Weight":
        """packed [N, Kc/2] / scales [N, Kc/32] with Kc >= K; columns beyond K must be zero.
        A tail that does not fill a whole K tile is zero-padded here (a row-parallel shard such as
        8704 / 8 = 1088 input features), so the GEMM only ever reads whole tiles of weights."""
        N, K2 = packed.shape
        Kc = K2 * 2
        K = Kc if K is None else K
        assert scales.shape == (N, Kc // 32) and K <= Kc and K % 32 == 0, (scales.shape, N, K, Kc)
        Kp = (K + KPAD - 1) // KPAD * KPAD
        if Kc != Kp:
            pk = torch.zeros(N, Kp // 2, dtype=torch.uint8, device=packed.device)
            sc = torch.full((N, Kp // 32), 127, dtype=torch.uint8, device=scales.device)
            pk[:, :K // 2] = packed[:, :K // 2]
            sc[:, :K // 32] = scales[:, :K // 32]
            packed, scales = pk, sc
        return MXFP4Weight(packed.contiguous(), scales.contiguous(),
                           sf_tile_layout(scales), N, K)

    @property
    def K_padded(self) -> int:
        return self.packed.shape[1] * 2

    def dequantize(self) -> torch.Tensor:
        return mxfp4_dequantize(self.packed[:, :self.K // 2], self.scales[:, :self.K // 32])

    def to(self, device) -> "MXFP4Weight":
        return MXFP4Weight(self.packed.to(device), self.scales.to(device), self.sf.to(device),
                           self.N, self.K)

    def narrow_rows(self, start: int, length: int) -> "MXFP4Weight":
        """Row slice (output-feature shard for column-parallel TP)."""
        return MXFP4Weight.from_packed(self.packed[start:start + length],
                                       self.scales[start:start + length], self.K)

    def narrow_cols(self, start: int, length: int) -> "MXFP4Weight":
        """K slice (input-feature shard for row-parallel TP); start/length multiples of 32."""
        assert start % 32 == 0 and length % 32 == 0 and start + length <= self.K
        return MXFP4Weight.from_packed(self.packed[:, start // 2:(start + length) // 2],
                                       self.scales[:, start // 32:(start + length) // 32])

    @property
    def nbytes(self) -> int:
        return self.packed.numel() + self.sf.numel()


def cat_rows(ws: list[MXFP4Weight]) -> MXFP4Weight:
    """Merged linear (qkvz+ba, gate_up): concatenate along N."""
    assert all(w.K == ws[0].K for w in ws)
    return MXFP4Weight.from_packed(torch.cat([w.packed for w in ws], 0),
                                   torch.cat([w.scales for w in ws], 0), ws[0].K)
