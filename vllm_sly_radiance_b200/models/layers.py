"""Model building blocks: linears (MXFP4 W4A8, INT4 W4A16, bf16, fp8 baseline), RoPE tables, norms.

A linear consumes either a bf16 activation or a pre-quantized ``(q_e4m3, scale)`` pair produced
by a fused producer kernel (the reference's tuple input contract,
``sly/mxfp4/radiance_mxfp4.py:1186-1193``)."""
from __future__ import annotations

import math
from typing import Optional, Union

import torch

from ..ops import kernels as K
from ..quant.mxfp4 import MXFP4Weight

Act = Union[torch.Tensor, tuple, "NormAct", "SiluAct"]


class NormAct:
    """Activation given as its producer: residual add + RMSNorm(1 + w) of `h` (+ `res`), quantised
    to e4m3 inside the decode GEMM.  `res_out` receives the new residual stream."""
    __slots__ = ("h", "res", "w", "eps", "res_out")

    def __init__(self, h, res, w, eps, res_out):
        self.h, self.res, self.w, self.eps, self.res_out = h, res, w, eps, res_out


class SiluAct:
    """Activation given as its producer: SiLU(g) * u of `gu` = [g | u], quantised in the GEMM."""
    __slots__ = ("gu",)

    def __init__(self, gu):
        self.gu = gu


FUSE_MAX_ROWS = 1          # fused producers: single-row decode (the rows are held in registers)
FUSE_MAX_K = 9216

import os as _os

# decode batches (<= 16 rows): RADIANCE_FINISH=1 lets the GEMM's last CTA produce the next
# linear's e4m3 rows in the same launch.  Opt-in: on the 27B decode step it measured 198 against
# 227 tok/s, since one CTA finishing a whole row (5-9 us) sits serially at each GEMM's tail where
# the stand-alone producer overlapped under programmatic dependent launch.  RADIANCE_GEMV=1
# selects the persistent stream-K decode GEMM (one CTA per SM) instead of the split-K cluster
# GEMM: it measured slower (fewer weight bytes in flight per SM), so it is opt-in too.
GEMV_ON = _os.environ.get("RADIANCE_GEMV", "0") == "1"
FINISH_ON = _os.environ.get("RADIANCE_FINISH", "0") == "1"


def rope_cache(max_pos: int, rotary_dim: int, theta: float, device) -> torch.Tensor:
    """[max_pos, rotary_dim] fp32: cos in [:rot/2], sin in [rot/2:], computed in fp64."""
    inv = 1.0 / (theta ** (torch.arange(0, rotary_dim, 2, dtype=torch.float64) / rotary_dim))
    ang = torch.arange(max_pos, dtype=torch.float64)[:, None] * inv[None]
    return torch.cat([torch.cos(ang), torch.sin(ang)], 1).float().to(device)


class Linear:
    """y = x W^T with W [N, K] stored as an MX block-scaled type (MXFP4 / MXFP6 / MXFP8 weights
    with e4m3 activations), bf16, or per-channel fp8 (the cuBLAS baseline build)."""

    def __init__(self, weight: torch.Tensor, quant: str = "mxfp4", name: str = ""):
        self.name = name
        self.quant = quant
        self.N, self.K = weight.shape
        if quant in ("mxfp4", "mxfp6", "mxfp8"):
            # one code path for the three block-scaled element types (e2m1 / e2m3 / e4m3)
            self.w = MXFP4Weight.from_float(weight, {"mxfp4": "e2m1", "mxfp6": "e2m3",
                                                     "mxfp8": "e4m3"}[quant])
            self.quant = "mxfp4"
        elif quant == "bf16":
            self.w = weight.to(torch.bfloat16).contiguous()
        elif quant == "int4":
            from ..quant.int4 import Int4Weight
            self.w = Int4Weight.from_float(weight, clip_search=True)
        elif quant == "fp8":
            amax = weight.float().abs().amax(1).clamp(min=1e-8)
            self.w_scale = (amax / 448.0).float()
            self.w = (weight.float() / self.w_scale[:, None]).clamp(-448, 448).to(
                torch.float8_e4m3fn).contiguous()
        else:
            raise ValueError(quant)

    @staticmethod
    def from_mxfp4(w: MXFP4Weight, name: str = "") -> "Linear":
        lin = Linear.__new__(Linear)
        lin.name, lin.quant, lin.N, lin.K, lin.w = name, "mxfp4", w.N, w.K, w
        return lin

    @staticmethod
    def from_int4(w, name: str = "") -> "Linear":
        lin = Linear.__new__(Linear)
        lin.name, lin.quant, lin.N, lin.K, lin.w = name, "int4", w.N, w.K, w
        return lin

    def to(self, device) -> "Linear":
        if self.quant in ("mxfp4", "int4"):
            self.w = self.w.to(device)
        else:
            self.w = self.w.to(device)
            if self.quant == "fp8":
                self.w_scale = self.w_scale.to(device)
        return self

    def _fused(self, x, out):
        """The decode GEMM with its producer inside (one launch instead of two)."""
        if isinstance(x, NormAct):
            M = x.h.shape[0]
            ok = (self.quant == "mxfp4" and x.h.is_cuda and M <= FUSE_MAX_ROWS and self.push is None
                  and self.K <= FUSE_MAX_K)
            if not ok:
                q, s_, r = K.add_rms_quant(x.h, x.res, x.w, x.eps)
                x.res_out.copy_(r)
                return self((q, s_), out)
            if out is None:
                out = torch.empty(M, self.N, dtype=torch.bfloat16, device=x.h.device)
            K.mxfp4_gemm_act(1, x.h, x.res, x.w, x.res_out, x.eps, self.w, out)
            return out
        M = x.gu.shape[0]
        ok = (self.quant == "mxfp4" and x.gu.is_cuda and M <= FUSE_MAX_ROWS and self.push is None
              and self.K <= FUSE_MAX_K)
        if not ok:
            act = K.silu_mul_quant(x.gu) if self.quant != "bf16" else K.silu_mul(x.gu)
            return self(act, out)
        if out is None:
            out = torch.empty(M, self.N, dtype=torch.bfloat16, device=x.gu.device)
        K.mxfp4_gemm_act(2, x.gu, None, None, None, 0.0, self.w, out)
        return out

    @property
    def nbytes(self) -> int:
        if self.quant in ("mxfp4", "int4"):
            return self.w.nbytes
        return self.w.numel() * self.w.element_size()

    # row-parallel linears of a TP>1 model get the NVLink communicator here: for decode-sized
    # batches their GEMM pushes its output tiles to every rank (fused GEMM -> all-reduce)
    push = None

    def can_finish(self, x) -> bool:
        """A decode-sized (e4m3, scale) input this MXFP4 linear can run with a fused finisher."""
        return (FINISH_ON and self.quant == "mxfp4" and isinstance(x, tuple)
                and x[0].is_cuda and 0 < x[0].shape[0] <= K.GEMV_MAX_ROWS and self.push is None)

    def call_finish(self, x, mode: int, res=None, norm_w=None, eps: float = 0.0):
        """y = x W^T followed, in the same launch, by the producer of the next linear:
        FIN_NORM -> (q, scale, new residual = bf16(y + res)) of RMSNorm(1 + norm_w);
        FIN_SILU -> (q, scale) of SiLU(g) * u with y = [g | u].  CPU / ineligible inputs run the
        same ops unfused."""
        if not self.can_finish(x):
            y = self(x)
            if mode == K.FIN_NORM:
                return K.add_rms_quant(y, res, norm_w, eps)
            return K.silu_mul_quant(y)
        q, s = x
        if mode == K.FIN_NORM:
            res_new = torch.empty(q.shape[0], self.N, dtype=torch.bfloat16, device=q.device)
            if GEMV_ON and self.w.fmt == "e2m1":
                _, fq, fs = K.mxfp4_gemv(q, s, self.w, None, K.FIN_NORM, res, norm_w, res_new, eps)
            else:
                _, fq, fs = K.mxfp4_gemm_finish(q, s, self.w, K.FIN_NORM, res, norm_w, res_new, eps)
            return fq, fs, res_new
        if GEMV_ON and self.w.fmt == "e2m1":
            _, fq, fs = K.mxfp4_gemv(q, s, self.w, None, K.FIN_SILU)
        else:
            _, fq, fs = K.mxfp4_gemm_finish(q, s, self.w, K.FIN_SILU)
        return fq, fs

    def __call__(self, x: Act, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        if isinstance(x, (NormAct, SiluAct)):
            return self._fused(x, out)
        if self.quant == "mxfp4":
            if isinstance(x, tuple):
                q, s = x
            else:
                q, s = K.quant_fp8(x)
            if self.push is not None and out is None and q.is_cuda and \
                    self.push.can_push(q.shape[0], self.N):
                return self.push.gemm_push(q, s, self.w)
            if GEMV_ON and self.w.fmt == "e2m1" and q.is_cuda and 0 < q.shape[0] <= K.GEMV_MAX_ROWS:
                return K.mxfp4_gemv(q, s, self.w, out)
            return K.mxfp4_gemm(q, s, self.w.packed, self.w.sf, self.w.scales, self.N, out=out,
                                fmt=self.w.fmt)
        if self.quant == "fp8":
            if isinstance(x, tuple):
                q, s = x
            else:
                q, s = K.quant_fp8(x)
            if q.is_cuda:
                y = torch._scaled_mm(q, self.w.t(), scale_a=s[:, None].float(),
                                     scale_b=self.w_scale[None, :].float(), out_dtype=torch.bfloat16)
            else:
                y = ((q.float() * s[:, None]) @ (self.w.float() * self.w_scale[:, None]).t()).to(
                    torch.bfloat16)
            if out is not None:
                out.copy_(y)
                return out
            return y
        if self.quant == "int4":
            from ..quant.int4 import w4a16_linear
            if isinstance(x, tuple):
                q, s = x
                x = (q.float() * s[:, None]).to(torch.bfloat16)
            y = w4a16_linear(x, self.w)
            if out is not None:
                out.copy_(y)
                return out
            return y
        # bf16
        if isinstance(x, tuple):
            q, s = x
            x = (q.float() * s[:, None]).to(torch.bfloat16)
        if x.is_cuda:
            y = torch.matmul(x, self.w.t())
        else:
            y = (x.float() @ self.w.float().t()).to(torch.bfloat16)
        if out is not None:
            out.copy_(y)
            return out
        return y
