"""Quantised token-embedding table: int8 with one fp32 scale per row, or int4 codes (two per byte,
low nibble = even column, value = code - 8) with one bf16 scale per 128 columns.

Reference behaviour: ``sly/mxfp4/radiance_embed_int8.py:47-114`` (RADIANCE_EMBED_INT8 /
RADIANCE_EMBED_BITS: quantise embed_tokens at load, dequantise on lookup; 2.54 GB of bf16 for the
248k x 5120 table becomes 1.27 GB at int8 or 0.66 GB at int4).  Quantisation rounds to nearest
with a per-row (int8, /127) or per-group (int4, /7, clamp [-8, 7]) absmax scale, built in row
chunks so the fp32 transient stays small; the CUDA lookup is ``csrc/embed.cu``."""
from __future__ import annotations

import torch

CHUNK_ROWS = 8192
GROUP = 128


class QuantEmbedding:
    def __init__(self, codes: torch.Tensor, scales: torch.Tensor, bits: int, hidden: int):
        self.codes, self.scales, self.bits, self.hidden = codes, scales, bits, hidden

    @staticmethod
    def from_float(w: torch.Tensor, bits: int) -> "QuantEmbedding":
        if bits not in (4, 8):
            raise ValueError(f"embedding bits must be 4 or 8, got {bits}")
        V, H = w.shape
        if bits == 8:
            codes = torch.empty(V, H, dtype=torch.int8, device=w.device)
            scales = torch.empty(V, dtype=torch.float32, device=w.device)
            for i in range(0, V, CHUNK_ROWS):
                blk = w[i:i + CHUNK_ROWS].float()
                s = blk.abs().amax(1).clamp_min(1e-8) / 127.0
                codes[i:i + CHUNK_ROWS] = torch.round(blk / s[:, None]).clamp_(-127, 127).to(torch.int8)
                scales[i:i + CHUNK_ROWS] = s
        else:
            if H % GROUP:
                raise ValueError(f"hidden {H} is not a multiple of {GROUP}")
            codes = torch.empty(V, H // 2, dtype=torch.uint8, device=w.device)
            scales = torch.empty(V, H // GROUP, dtype=torch.bfloat16, device=w.device)
            for i in range(0, V, CHUNK_ROWS):
                blk = w[i:i + CHUNK_ROWS].float().view(-1, H // GROUP, GROUP)
                s = (blk.abs().amax(2, keepdim=True).clamp_min(1e-8) / 7.0).to(torch.bfloat16)
                nib = (torch.round(blk / s.float()).clamp_(-8, 7) + 8).to(torch.uint8).view(-1, H)
                codes[i:i + CHUNK_ROWS] = nib[:, 0::2] | (nib[:, 1::2] << 4)
                scales[i:i + CHUNK_ROWS] = s.view(-1, H // GROUP)
        return QuantEmbedding(codes, scales, bits, H)

    def to(self, device) -> "QuantEmbedding":
        self.codes = self.codes.to(device)
        self.scales = self.scales.to(device)
        return self

    @property
    def nbytes(self) -> int:
        return self.codes.numel() * self.codes.element_size() + \
            self.scales.numel() * self.scales.element_size()

    def dequantize_rows(self, ids: torch.Tensor) -> torch.Tensor:
        """PyTorch oracle of the lookup (CPU path)."""
        rows = self.codes[ids]
        if self.bits == 8:
            return (rows.float() * self.scales[ids][:, None]).to(torch.bfloat16)
        nib = torch.stack(((rows & 0xF).to(torch.int16), (rows >> 4).to(torch.int16)), -1)
        nib = nib.view(-1, self.hidden // GROUP, GROUP).float() - 8
        return (nib * self.scales[ids].float()[:, :, None]).view(-1, self.hidden).to(torch.bfloat16)

    def __getitem__(self, ids: torch.Tensor) -> torch.Tensor:
        ids = ids.reshape(-1).long()
        if not self.codes.is_cuda:
            return self.dequantize_rows(ids)
        from ..ops._ext import ext
        out = torch.empty(ids.shape[0], self.hidden, dtype=torch.bfloat16, device=ids.device)
        ext().embed_gather(self.codes, self.scales, ids.contiguous(), self.bits, out)
        return out
