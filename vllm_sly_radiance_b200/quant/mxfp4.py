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


@dataclass
class MXFP4Weight:
    packed: torch.Tensor          # uint8 [N, K/2]
    scales: torch.Tensor          # uint8 [N, K/32]
    sf: torch.Tensor              # uint8 tiled scale factors
    N: int
    K: int

    @staticmethod
    def from_float(w: torch.Tensor) -> "MXFP4Weight":
        N, K = w.shape
        if K % 128 != 0:
            raise ValueError(f"MXFP4 linear needs K % 128 == 0 (got K={K}); pad at load")
        packed, scales = mxfp4_quantize(w)
        return MXFP4Weight.from_packed(packed, scales)

    @staticmethod
    def from_packed(packed: torch.Tensor, scales: torch.Tensor) -> "MXFP4Weight":
        N, K2 = packed.shape
        K = K2 * 2
        assert scales.shape == (N, K // 32), (scales.shape, N, K)
        return MXFP4Weight(packed.contiguous(), scales.contiguous(),
                           sf_tile_layout(scales), N, K)

    def dequantize(self) -> torch.Tensor:
        return mxfp4_dequantize(self.packed, self.scales)

    def to(self, device) -> "MXFP4Weight":
        return MXFP4Weight(self.packed.to(device), self.scales.to(device), self.sf.to(device),
                           self.N, self.K)

    def narrow_rows(self, start: int, length: int) -> "MXFP4Weight":
        """Row slice (output-feature shard for column-parallel TP)."""
        return MXFP4Weight.from_packed(self.packed[start:start + length],
                                       self.scales[start:start + length])

    def narrow_cols(self, start: int, length: int) -> "MXFP4Weight":
        """K slice (input-feature shard for row-parallel TP); start/length multiples of 128."""
        assert start % 128 == 0 and length % 128 == 0
        return MXFP4Weight.from_packed(self.packed[:, start // 2:(start + length) // 2],
                                       self.scales[:, start // 32:(start + length) // 32])

    @property
    def nbytes(self) -> int:
        return self.packed.numel() + self.sf.numel()


def cat_rows(ws: list[MXFP4Weight]) -> MXFP4Weight:
    """Merged linear (qkvz+ba, gate_up): concatenate along N."""
    return MXFP4Weight.from_packed(torch.cat([w.packed for w in ws], 0),
                                   torch.cat([w.scales for w in ws], 0))
