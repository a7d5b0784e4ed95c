"""Numerics of every sm_100a kernel against the PyTorch fp32 reference of the same op."""
import math

import pytest
import torch

from vllm_sly_radiance_b200.ops import kernels as K
from vllm_sly_radiance_b200.ops import reference as ref
from vllm_sly_radiance_b200.quant.mxfp4 import MXFP4Weight

pytestmark = pytest.mark.gpu
DEV = "cuda"


def fp8_close(q, s, qw, sw):
    """Dequantized e4m3 rows agree up to one e4m3 step (bf16 rounding of the producer input
    can flip a code when the kernel's rsqrt/exp differ from torch's in the last bit)."""
    dq = q.cpu().float() * s.cpu().float()[:, None]
    dw = qw.cpu().float() * sw.cpu().float()[:, None]
    tol = 0.07 * dw.abs() + 1e-3 * dw.abs().max()
    bad = ((dq - dw).abs() > tol).float().mean()
    return float(bad) < 1e-3


def rel_err(a, b):
    a = a.float().cpu()
    b = b.float().cpu()
    return float((a - b).abs().max() / b.abs().max().clamp(min=1e-6))


@pytest.mark.parametrize("M,N,Kd,splits", [
    (1, 256, 256, 0), (5, 384, 512, 0), (16, 256, 1024, 4), (37, 200, 768, 0),
    (64, 512, 512, 2), (128, 256, 256, 0), (300, 512, 1024, 0), (1, 5120, 8704, 0),
    (8, 16480, 5120, 0), (520, 640, 2048, 1),
    # K tail (a row-parallel shard of 8704 / 8 = 1088 features): zero-padded weight tiles
    (1, 5120, 1088, 0), (40, 2176, 1088, 0), (3, 384, 1088, 2)])
def test_mxfp4_gemm(M, N, Kd, splits):
    g = torch.Generator().manual_seed(M * 7 + N)
    w = torch.randn(N, Kd, generator=g) * 0.02
    x = torch.randn(M, Kd, generator=g)
    wq = MXFP4Weight.from_float(w)
    q, s = ref.quant_fp8_rows(x.to(torch.bfloat16))
    want = ref.mxfp4_linear(q, s, wq.packed, wq.scales)
    wg = wq.to(DEV)
    got = K.mxfp4_gemm(q.to(DEV), s.to(DEV), wg.packed, wg.sf, wg.scales, N, splits=splits)
    torch.cuda.synchronize()
    K.check_status(got.device)
    assert rel_err(got, want) < 1e-2, rel_err(got, want)


@pytest.mark.parametrize("M,N,Kd,fmt", [
    (512, 256, 256, "e2m1"), (1031, 640, 1088, "e2m1"), (4096, 5120, 1088, "e2m1"),
    (777, 2176, 5120, "e2m1"), (2048, 384, 512, "e4m3"), (600, 1000, 768, "e2m3")])
def test_mxfp4_gemm_cta_pair(M, N, Kd, fmt):
    """Prefill GEMM on CTA pairs (tcgen05 cta_group::2, persistent, M >= 512) against the fp32
    product and against the one-CTA kernel (forced by an explicit split count)."""
    g = torch.Generator().manual_seed(M + N + Kd)
    w = torch.randn(N, Kd, generator=g) * 0.02
    x = torch.randn(M, Kd, generator=g)
    wq = MXFP4Weight.from_float(w, fmt)
    q, s = ref.quant_fp8_rows(x.to(torch.bfloat16))
    want = ref.mxfp4_linear(q, s, wq.packed, wq.scales, fmt=fmt)
    wg = wq.to(DEV)
    for rep in range(2):
        got = K.mxfp4_gemm(q.to(DEV), s.to(DEV), wg.packed, wg.sf, wg.scales, N)
        one = K.mxfp4_gemm(q.to(DEV), s.to(DEV), wg.packed, wg.sf, wg.scales, N, splits=1)
        torch.cuda.synchronize()
        K.check_status(got.device)
        assert rel_err(got, want) < 1e-2, (rep, rel_err(got, want))
        assert rel_err(got, one) < 5e-3, (rep, rel_err(got, one))


@pytest.mark.parametrize("fmt", ["e2m3", "e4m3"])
@pytest.mark.parametrize("M,N,Kd,splits", [
    (1, 256, 256, 0), (5, 384, 512, 0), (16, 256, 1024, 4), (37, 200, 768, 0),
    (128, 256, 256, 0), (300, 512, 1024, 0), (1, 5120, 8704, 0), (3, 384, 1088, 2),
    (40, 2176, 1088, 0)])
def test_mx_gemm_formats(fmt, M, N, Kd, splits):
    """MXFP6 (e2m3, TMA 16U6) and MXFP8 (e4m3) weights through the same block-scaled kernel."""
    g = torch.Generator().manual_seed(M * 7 + N + len(fmt))
    w = torch.randn(N, Kd, generator=g) * 0.02
    x = torch.randn(M, Kd, generator=g)
    wq = MXFP4Weight.from_float(w, fmt)
    q, s = ref.quant_fp8_rows(x.to(torch.bfloat16))
    want = ref.mxfp4_linear(q, s, wq.packed, wq.scales, fmt=fmt)
    wg = wq.to(DEV)
    got = K.mxfp4_gemm(q.to(DEV), s.to(DEV), wg.packed, wg.sf, wg.scales, N, splits=splits)
    torch.cuda.synchronize()
    K.check_status(got.device)
    assert rel_err(got, want) < 1e-2, rel_err(got, want)


@pytest.mark.parametrize("fmt", ["e2m3", "e4m3"])
def test_mx_formats_fused_and_grouped(fmt):
    """The decode producer-fused GEMM, the finisher GEMM and the grouped (MoE) GEMM accept the
    wider element types too."""
    from vllm_sly_radiance_b200.quant.mxfp4 import cat_rows
    g = torch.Generator().manual_seed(21)
    N, Kd = 2176, 1088
    wq = MXFP4Weight.from_float(torch.randn(N, Kd, generator=g) * 0.02, fmt).to(DEV)
    h = torch.randn(1, Kd, generator=g).to(torch.bfloat16).to(DEV)
    lw = (0.1 * torch.randn(Kd, generator=g)).to(torch.bfloat16).to(DEV)
    q, s, r = K.add_rms_quant(h, None, lw, 1e-6)
    want = ref.mxfp4_linear(q.cpu(), s.cpu(), wq.packed.cpu(), wq.scales.cpu(), fmt=fmt)
    out = torch.empty(1, N, dtype=torch.bfloat16, device=DEV)
    K.mxfp4_gemm_act(1, h, None, lw, None, 1e-6, wq, out)
    torch.cuda.synchronize()
    K.check_status(out.device)
    assert rel_err(out, want) < 1e-2, rel_err(out, want)
    # finisher: SiLU * mul + e4m3 of the GEMM's own output rows
    got, fq, fs = K.mxfp4_gemm_finish(q, s, wq, K.FIN_SILU)
    torch.cuda.synchronize()
    assert rel_err(got, want) < 1e-2
    wq2, ws2 = K.silu_mul_quant(got)
    assert fp8_close(fq, fs, wq2, ws2)
    # grouped
    E, Ng, Kg = 4, 256, 512
    ws = [MXFP4Weight.from_float(torch.randn(Ng, Kg, generator=g) * 0.02, fmt) for _ in range(E)]
    counts = torch.tensor([3, 0, 40, 1])
    x = torch.randn(int(counts.sum()), Kg, generator=g).to(torch.bfloat16)
    q, s = ref.quant_fp8_rows(x)
    want, r0 = torch.empty(x.shape[0], Ng), 0
    for e in range(E):
        c = int(counts[e])
        if c:
            want[r0:r0 + c] = ref.mxfp4_linear(q[r0:r0 + c], s[r0:r0 + c], ws[e].packed,
                                               ws[e].scales, fmt=fmt).float()
        r0 += c
    got = K.moe_grouped_gemm(q.to(DEV), s.to(DEV), cat_rows(ws).to(DEV), Ng, counts.to(DEV))
    torch.cuda.synchronize()
    K.check_status(got.device)
    assert rel_err(got, want) < 1e-2, rel_err(got, want)


@pytest.mark.parametrize("mode,M,N,Kd,with_res", [
    (1, 1, 16480, 5120, True), (1, 1, 2176, 1088, False), (1, 1, 5120, 256, True),
    (2, 1, 5120, 8704, False), (2, 1, 384, 1088, False), (2, 1, 256, 768, False)])
def test_mxfp4_gemm_fused_producer(mode, M, N, Kd, with_res):
    """Decode GEMM with the producer inside (add + RMSNorm + e4m3, or SiLU * mul + e4m3)
    against the stand-alone producer kernel followed by the plain GEMM."""
    g = torch.Generator().manual_seed(M * 11 + N + mode)
    wq = MXFP4Weight.from_float(torch.randn(N, Kd, generator=g) * 0.02).to(DEV)
    out = torch.empty(M, N, dtype=torch.bfloat16, device=DEV)
    if mode == 1:
        h = torch.randn(M, Kd, generator=g).to(torch.bfloat16).to(DEV)
        res = torch.randn(M, Kd, generator=g).to(torch.bfloat16).to(DEV) if with_res else None
        lw = (0.1 * torch.randn(Kd, generator=g)).to(torch.bfloat16).to(DEV)
        q, s, r = K.add_rms_quant(h, res, lw, 1e-6)
        want = K.mxfp4_gemm(q, s, wq.packed, wq.sf, wq.scales, N)
        ro = torch.empty(M, Kd, dtype=torch.bfloat16, device=DEV)
        K.mxfp4_gemm_act(1, h, res, lw, ro, 1e-6, wq, out)
        torch.cuda.synchronize()
        assert torch.equal(ro, r)
    else:
        gu = (torch.randn(M, 2 * Kd, generator=g) * 2).to(torch.bfloat16).to(DEV)
        q, s = K.silu_mul_quant(gu)
        want = K.mxfp4_gemm(q, s, wq.packed, wq.sf, wq.scales, N)
        K.mxfp4_gemm_act(2, gu, None, None, None, 0.0, wq, out)
        torch.cuda.synchronize()
    K.check_status(out.device)
    assert rel_err(out, want) < 1e-2, rel_err(out, want)


@pytest.mark.parametrize("M,N,Kd", [(1, 256, 256), (1, 5120, 6144), (3, 16480, 5120),
                                     (16, 5120, 8704), (1, 5120, 1088), (8, 2176, 1088),
                                     (1, 248320, 5120), (5, 200, 768), (2, 96, 128)])
def test_mxfp4_gemv(M, N, Kd):
    """Persistent stream-K decode GEMM against the fp32 product: tiles whose K range spans
    several CTAs are reduced in-kernel; two launches in a row check the counter resets."""
    g = torch.Generator().manual_seed(M * 13 + N + Kd)
    wq = MXFP4Weight.from_float(torch.randn(N, Kd, generator=g) * 0.02)
    wg = wq.to(DEV)
    for rep in range(2):
        x = torch.randn(M, Kd, generator=g)
        q, s = ref.quant_fp8_rows(x.to(torch.bfloat16))
        want = ref.mxfp4_linear(q, s, wq.packed, wq.scales)
        got = K.mxfp4_gemv(q.to(DEV), s.to(DEV), wg)
        torch.cuda.synchronize()
        K.check_status(got.device)
        assert rel_err(got, want) < 1e-2, (rep, rel_err(got, want))


@pytest.mark.parametrize("impl", ["cluster", "gemv"])
@pytest.mark.parametrize("mode,M,N,Kd,with_res", [
    (1, 1, 5120, 6144, True), (1, 4, 5120, 8704, True), (1, 1, 2048, 1088, False),
    (2, 1, 17408, 5120, False), (2, 3, 4352, 5120, False), (2, 16, 768, 256, False)])
def test_mxfp4_gemv_finisher(mode, M, N, Kd, with_res, impl):
    """The finisher run by the last CTA (residual add + RMSNorm + e4m3, or SiLU * mul + e4m3), in
    the split-K cluster decode GEMM and in the persistent stream-K one, equals the stand-alone
    producer applied to the GEMM output."""
    g = torch.Generator().manual_seed(M * 5 + N + mode)
    wq = MXFP4Weight.from_float(torch.randn(N, Kd, generator=g) * 0.02).to(DEV)
    x = torch.randn(M, Kd, generator=g).to(torch.bfloat16).to(DEV)
    q, s = K.quant_fp8(x)
    for rep in range(2):
        if mode == 1:
            res = torch.randn(M, N, generator=g).to(torch.bfloat16).to(DEV) if with_res else None
            lw = (0.1 * torch.randn(N, generator=g)).to(torch.bfloat16).to(DEV)
            ro = torch.empty(M, N, dtype=torch.bfloat16, device=DEV)
            if impl == "gemv":
                out, fq, fs = K.mxfp4_gemv(q, s, wq, None, K.FIN_NORM, res, lw, ro, 1e-6)
            else:
                out, fq, fs = K.mxfp4_gemm_finish(q, s, wq, K.FIN_NORM, res, lw, ro, 1e-6)
            wq_, ws_, wr = K.add_rms_quant(out, res, lw, 1e-6)
            torch.cuda.synchronize()
            assert torch.equal(ro, wr)
        else:
            if impl == "gemv":
                out, fq, fs = K.mxfp4_gemv(q, s, wq, None, K.FIN_SILU)
            else:
                out, fq, fs = K.mxfp4_gemm_finish(q, s, wq, K.FIN_SILU)
            wq_, ws_ = K.silu_mul_quant(out)
            torch.cuda.synchronize()
        K.check_status(out.device)
        torch.testing.assert_close(fs, ws_, rtol=1e-5, atol=0)
        assert fp8_close(fq, fs, wq_, ws_)
        want = K.mxfp4_gemm(q, s, wq.packed, wq.sf, wq.scales, N)
        assert rel_err(out, want) < 1e-2


@pytest.mark.parametrize("M,N,Kd", [(1, 248320 // 8, 5120), (3, 5120, 8704), (8, 1000, 1024),
                                     (40, 2176, 1024), (2, 96, 128), (12, 1000, 256),
                                     (5, 17408, 5120)])
def test_w4a16_linear(M, N, Kd):
    """INT4 g128 W4A16: the tensor-core GEMV (M <= 8) and the dequantise + GEMM path against the
    fp32 product with the dequantised weight."""
    from vllm_sly_radiance_b200.quant.int4 import Int4Weight, w4a16_linear
    g = torch.Generator().manual_seed(M + N)
    w = Int4Weight.from_float(torch.randn(N, Kd, generator=g) * 0.02)
    x = torch.randn(M, Kd, generator=g).to(torch.bfloat16)
    want = x.float() @ w.dequantize().t()
    wd = w.to(DEV)
    assert wd.tiled
    got = w4a16_linear(x.to(DEV), wd)
    torch.cuda.synchronize()
    K.check_status(got.device)
    assert rel_err(got, want) < 1e-2, rel_err(got, want)


def test_mxfp4_gemm_repeat_no_stale_state():
    """Back-to-back launches without a sync between them (split-K reduction must not leak)."""
    g = torch.Generator().manual_seed(3)
    N, Kd = 1024, 4096
    wq = MXFP4Weight.from_float(torch.randn(N, Kd, generator=g) * 0.02)
    wg = wq.to(DEV)
    outs, wants = [], []
    for i in range(4):
        x = torch.randn(3, Kd, generator=g)
        q, s = ref.quant_fp8_rows(x.to(torch.bfloat16))
        wants.append(ref.mxfp4_linear(q, s, wq.packed, wq.scales))
        outs.append(K.mxfp4_gemm(q.to(DEV), s.to(DEV), wg.packed, wg.sf, wg.scales, N))
    torch.cuda.synchronize()
    for o, w_ in zip(outs, wants):
        assert rel_err(o, w_) < 1e-2


@pytest.mark.parametrize("M,H,with_res", [(1, 5120, True), (7, 256, False), (33, 2048, True)])
def test_add_rms_quant(M, H, with_res):
    g = torch.Generator().manual_seed(M + H)
    x = torch.randn(M, H, generator=g).to(torch.bfloat16)
    r = torch.randn(M, H, generator=g).to(torch.bfloat16) if with_res else None
    w = (torch.randn(H, generator=g) * 0.1).to(torch.bfloat16)
    qw, sw, rw = ref.add_rms_quant(x, r, w, 1e-6)
    q, s, ro = K.add_rms_quant(x.to(DEV), None if r is None else r.to(DEV), w.to(DEV), 1e-6)
    torch.cuda.synchronize()
    assert torch.equal(ro.cpu(), rw)
    torch.testing.assert_close(s.cpu(), sw, rtol=1e-5, atol=0)
    assert fp8_close(q, s, qw, sw)


def test_silu_mul_and_gdn_norm_and_gate():
    g = torch.Generator().manual_seed(1)
    gu = torch.randn(9, 2 * 1024, generator=g).to(torch.bfloat16)
    qw, sw = ref.silu_mul_quant(gu)
    q, s = K.silu_mul_quant(gu.to(DEV))
    assert fp8_close(q, s, qw, sw)
    o = torch.randn(5, 4 * 128, generator=g).to(torch.bfloat16)
    zbuf = torch.randn(5, 3 * 4 * 128, generator=g).to(torch.bfloat16)
    z = zbuf[:, 512:1024]
    w = (1 + 0.1 * torch.randn(128, generator=g)).to(torch.bfloat16)
    qw, sw = ref.gdn_norm_quant(o, z, w, 1e-6, 128)
    q, s = K.gdn_norm_quant(o.to(DEV), zbuf.to(DEV)[:, 512:1024], w.to(DEV), 1e-6, 128)
    assert fp8_close(q, s, qw, sw)
    a = torch.randn(6, 3 * 64, generator=g).to(torch.bfloat16)
    qkv = torch.randn(6, 3 * 128, generator=g).to(torch.bfloat16)
    qw, sw = K.gate_mul_quant(a, qkv[:, 64:], 64, 128)
    q, s = K.gate_mul_quant(a.to(DEV), qkv.to(DEV)[:, 64:], 64, 128)
    assert fp8_close(q, s, qw, sw)


class _Meta:
    pass


def _attn_meta(q_lens, ctx_lens, block_size, Hq, Hkv, num_splits, dev):
    B = len(q_lens)
    m = _Meta()
    qsl = [0]
    for ql in q_lens:
        qsl.append(qsl[-1] + ql)
    seq_lens = [c + q for c, q in zip(ctx_lens, q_lens)]
    max_blocks = max((s + block_size - 1) // block_size for s in seq_lens)
    bt = torch.zeros(B, max_blocks, dtype=torch.int32)
    nxt = 0
    perm = torch.randperm(B * max_blocks, generator=torch.Generator().manual_seed(0))
    for b in range(B):
        for j in range(max_blocks):
            bt[b, j] = int(perm[nxt])
            nxt += 1
    G = Hq // Hkv
    ts, tr = [], []
    for b in range(B):
        R = q_lens[b] * G
        for r0 in range(0, R, 64):
            ts.append(b)
            tr.append(r0)
    m.query_start_loc = torch.tensor(qsl, dtype=torch.int32, device=dev)
    m.seq_lens = torch.tensor(seq_lens, dtype=torch.int32, device=dev)
    m.block_tables = bt.to(dev)
    m.num_tokens, m.num_seqs = sum(q_lens), B
    m.tile_seq = torch.tensor(ts, dtype=torch.int32, device=dev)
    m.tile_row0 = torch.tensor(tr, dtype=torch.int32, device=dev)
    m.num_splits = num_splits
    m.scratch_o = lambda s, T, H, D: torch.empty(s, T, H, D, device=dev)
    m.scratch_ml = lambda s, T, H: torch.empty(s, T, H, 2, device=dev)
    return m, B * max_blocks


@pytest.mark.parametrize("D,Hq,Hkv,q_lens,ctx_lens,splits,fp8", [
    (256, 24, 4, [1, 1, 1], [100, 1500, 63], 1, True),
    (256, 24, 4, [1, 1], [3000, 700], 8, True),
    (256, 24, 4, [8, 8], [500, 1200], 4, True),
    (256, 24, 4, [200, 70], [0, 130], 1, True),
    (64, 4, 2, [33, 1], [0, 90], 1, False),
    (64, 4, 2, [1, 1, 1, 1], [130, 62, 10, 0], 5, True),
    (64, 4, 2, [64, 22], [64, 128], 1, True),
    (64, 4, 2, [1, 1], [200, 70], 3, False),
    (128, 32, 8, [8], [250], 2, True)])
def test_paged_attention(D, Hq, Hkv, q_lens, ctx_lens, splits, fp8):
    torch.manual_seed(0)
    bs = 64
    meta, nblocks = _attn_meta(q_lens, ctx_lens, bs, Hq, Hkv, splits, DEV)
    cdt = torch.float8_e4m3fn if fp8 else torch.bfloat16
    kc = (torch.randn(nblocks, Hkv, bs, D) * 0.5).to(cdt)
    vc = torch.randn(nblocks, Hkv, bs, D).to(cdt)
    T = sum(q_lens)
    q = torch.randn(T, Hq, D).to(torch.bfloat16)
    if fp8:
        q = ref.fp8_e4m3(q.float()).to(torch.bfloat16)
    scale = D ** -0.5
    metac = _Meta()
    metac.block_tables = meta.block_tables.cpu()
    metac.seq_lens = meta.seq_lens.cpu()
    metac.query_start_loc = meta.query_start_loc.cpu()
    want = ref.paged_attention(q, kc, vc, metac.block_tables, metac.seq_lens,
                               metac.query_start_loc, bs, scale)
    got = K.paged_attention(q.to(DEV), kc.to(DEV), vc.to(DEV), meta, scale)
    torch.cuda.synchronize()
    assert rel_err(got, want) < 2e-2, rel_err(got, want)


@pytest.mark.parametrize("D,Hq,Hkv,ctx_lens,splits,fmt", [
    (256, 24, 4, [1500, 100, 0], 17, "fp8"), (256, 24, 4, [4000], 32, "fp8"),
    (256, 24, 4, [700, 63], 1, "bf16"), (256, 24, 4, [900, 65], 6, "int4"),
    (128, 32, 2, [300, 1], 3, "fp8"), (64, 4, 2, [130, 62, 10], 5, "int4"),
    (256, 6, 1, [2048], 8, "fp8"),
    (256, 24, 4, [16384, 3000], 96, "fp8"), (256, 24, 4, [8192], 128, "bf16")])   # > 32 splits
def test_paged_attention_decode_kernel(D, Hq, Hkv, ctx_lens, splits, fmt, monkeypatch):
    """The decode kernel (one token per sequence, keys split across warps) agrees with the
    general 64-row tile kernel and with the fp32 oracle, for every cache format."""
    from vllm_sly_radiance_b200.quant import formats as F
    torch.manual_seed(5)
    bs = 16 if fmt == "int4" else 64
    q_lens = [1] * len(ctx_lens)
    meta, nblocks = _attn_meta(q_lens, ctx_lens, bs, Hq, Hkv, splits, DEV)
    k = torch.randn(nblocks, Hkv, bs, D) * 0.5
    v = torch.randn(nblocks, Hkv, bs, D)
    q = torch.randn(len(ctx_lens), Hq, D).to(torch.bfloat16)
    if fmt == "fp8":
        kc, vc = k.to(torch.float8_e4m3fn), v.to(torch.float8_e4m3fn)
        q = ref.fp8_e4m3(q.float()).to(torch.bfloat16)
    elif fmt == "bf16":
        kc, vc = k.to(torch.bfloat16), v.to(torch.bfloat16)
    else:
        kc, vc = F.kv4_quantize(k), F.kv4_quantize(v)
    scale = D ** -0.5
    want = ref.paged_attention(q, kc, vc, meta.block_tables.cpu(), meta.seq_lens.cpu(),
                               meta.query_start_loc.cpu(), bs, scale)
    got = K.paged_attention(q.to(DEV), kc.to(DEV), vc.to(DEV), meta, scale)
    monkeypatch.setattr(K, "_ATTN_DECODE", False)
    general = K.paged_attention(q.to(DEV), kc.to(DEV), vc.to(DEV), meta, scale)
    torch.cuda.synchronize()
    assert rel_err(got, want) < 2e-2, rel_err(got, want)
    assert rel_err(got, general) < 1e-2, rel_err(got, general)


@pytest.mark.parametrize("kv", ["fp8", "int4", "int4_p64"])
@pytest.mark.parametrize("q_lens,ctx_lens", [([256], [0]), ([300, 77], [1000, 40]),
                                            ([130], [5000]), ([1024], [3000])])
def test_fmha_prefill_tcgen05(q_lens, ctx_lens, kv, monkeypatch):
    """Causal chunked-prefill attention on tcgen05 (e4m3 QK and P V legs, TMEM accumulators,
    TMA-fed fp8 pages) against the fp32 oracle and the mma.sync tile kernel, GQA 6, head 256.
    A 4-bit cache (the engine's 16-token pages, or 64-token ones) reaches the kernel through its
    keys dequantised into 64-key e4m3 pages."""
    from vllm_sly_radiance_b200.quant.formats import kv4_quantize
    torch.manual_seed(21)
    D, Hq, Hkv = 256, 24, 4
    bs = 16 if kv == "int4" else 64
    meta, nblocks = _attn_meta(q_lens, ctx_lens, bs, Hq, Hkv, 1, DEV)
    if kv == "fp8":
        k = (torch.randn(nblocks, Hkv, bs, D) * 0.5).to(torch.float8_e4m3fn)
        v = torch.randn(nblocks, Hkv, bs, D).to(torch.float8_e4m3fn)
    else:
        k = kv4_quantize(torch.randn(nblocks, Hkv, bs, D) * 0.5)
        v = kv4_quantize(torch.randn(nblocks, Hkv, bs, D))
    T = sum(q_lens)
    q = ref.fp8_e4m3(torch.randn(T, Hq, D)).to(torch.bfloat16)
    scale = D ** -0.5
    want = ref.paged_attention(q, k, v, meta.block_tables.cpu(), meta.seq_lens.cpu(),
                               meta.query_start_loc.cpu(), bs, scale)
    monkeypatch.setattr(K, "_FMHA", True)
    got = K.paged_attention(q.to(DEV), k.to(DEV), v.to(DEV), meta, scale)
    monkeypatch.setattr(K, "_FMHA", False)
    tile = K.paged_attention(q.to(DEV), k.to(DEV), v.to(DEV), meta, scale)
    torch.cuda.synchronize()
    K.check_status(got.device)
    assert rel_err(tile, want) < 2e-2
    # P and V on the e4m3 leg: a few percent of the row maximum (the 4-bit cache's dequantised
    # K / V take one more e4m3 rounding)
    assert rel_err(got, want) < (5e-2 if kv == "fp8" else 7e-2), rel_err(got, want)


@pytest.mark.parametrize("Hq,Hkv,ctx_lens,splits", [(24, 4, [1500], 8), (24, 4, [300, 2000, 64], 1),
                                                   (6, 1, [700, 4000], 5)])
def test_paged_attention_decode_gated(Hq, Hkv, ctx_lens, splits):
    """Decode attention with the o_proj producer inside (sigmoid gate + per-token e4m3 by the last
    kv-head CTA of each token) against attention followed by gate_mul_quant, twice in a row."""
    torch.manual_seed(9)
    D, bs = 256, 64
    q_lens = [1] * len(ctx_lens)
    meta, nblocks = _attn_meta(q_lens, ctx_lens, bs, Hq, Hkv, splits, DEV)
    kc = (torch.randn(nblocks, Hkv, bs, D) * 0.5).to(torch.float8_e4m3fn).to(DEV)
    vc = torch.randn(nblocks, Hkv, bs, D).to(torch.float8_e4m3fn).to(DEV)
    T = len(ctx_lens)
    for rep in range(2):
        q = ref.fp8_e4m3(torch.randn(T, Hq, D)).to(torch.bfloat16).to(DEV)
        qkv = torch.randn(T, Hq * 2 * D + 64).to(torch.bfloat16).to(DEV)
        gq, gs = K.paged_attention_gated(q, kc, vc, meta, D ** -0.5, qkv[:, D:], 2 * D)
        a = K.paged_attention(q, kc, vc, meta, D ** -0.5).view(T, -1)
        wq, ws_ = K.gate_mul_quant(a, qkv[:, D:], D, 2 * D)
        torch.cuda.synchronize()
        torch.testing.assert_close(gs, ws_, rtol=1e-6, atol=0)
        assert torch.equal(gq.view(torch.uint8), wq.view(torch.uint8)), rep


@pytest.mark.parametrize("two_phase", [False, True])
@pytest.mark.parametrize("lens,has_init,sdt,split", [
    ([1500], [0], torch.float32, 0), ([64, 1, 200, 7], [1, 1, 0, 1], torch.float32, 1),
    ([130, 65], [1, 0], torch.bfloat16, 2), ([300], [1], torch.float32, 4),
    ([4096], [1], torch.float32, 8), ([63, 129, 640], [0, 1, 1], torch.bfloat16, 0)])
def test_gdn_chunked_matches_recurrent(lens, has_init, sdt, split, two_phase, monkeypatch):
    """The 64-token chunk-scan kernels (tensor cores, bf16 operands, fp32 state; one kernel, or
    the chunk-parallel solve followed by the state scan) against the fp32 token-serial oracle and
    against the token-serial CUDA kernel: outputs and final states."""
    if (split == 8 and not two_phase) or (split == 1 and two_phase):
        pytest.skip("split not offered by this form")
    monkeypatch.setattr(K, "_GDN_TWO_PHASE", two_phase)
    torch.manual_seed(7)
    Hk, Hv, D = 4, 12, 128
    key_dim, vdim = Hk * D, Hv * D
    T = sum(lens)
    qk = torch.randn(T, 2 * Hk, D)
    qk = qk / qk.norm(dim=-1, keepdim=True)
    v = torch.randn(T, vdim) * 0.5
    y = torch.cat([qk.reshape(T, -1), v], 1).to(torch.bfloat16)
    ba = (torch.randn(T, 2 * Hv) * 1.5).to(torch.bfloat16)
    A_log = torch.log(torch.rand(Hv) * 8 + 0.5)
    dt_bias = torch.randn(Hv) * 0.3
    state0 = (torch.randn(len(lens) + 1, Hv, D, D) * 0.05).to(sdt)
    meta = _Meta()
    qsl = [0]
    for l in lens:
        qsl.append(qsl[-1] + l)
    meta.query_start_loc = torch.tensor(qsl, dtype=torch.int32, device=DEV)
    meta.state_slots = torch.arange(1, len(lens) + 1, dtype=torch.int32, device=DEV)
    meta.has_initial = torch.tensor(has_init, dtype=torch.int32, device=DEV)
    meta.num_seqs, meta.num_tokens = len(lens), T
    scale = D ** -0.5
    monkeypatch.setattr(K, "_GDN_CHUNK_SPLIT", split)
    st_chunk = state0.to(DEV).clone()
    got = K.gdn_recurrent(y.to(DEV), ba.to(DEV), A_log.to(DEV), dt_bias.to(DEV), st_chunk, meta,
                          Hk, scale)
    monkeypatch.setattr(K, "_GDN_CHUNKED", False)
    st_serial = state0.to(DEV).clone()
    serial = K.gdn_recurrent(y.to(DEV), ba.to(DEV), A_log.to(DEV), dt_bias.to(DEV), st_serial,
                             meta, Hk, scale)
    torch.cuda.synchronize()
    yf = y.float()
    for bi, (s0, s1) in enumerate(zip(qsl[:-1], qsl[1:])):
        q = yf[s0:s1, :key_dim].view(-1, Hk, D)
        k = yf[s0:s1, key_dim:2 * key_dim].view(-1, Hk, D)
        vv = yf[s0:s1, 2 * key_dim:].view(-1, Hv, D)
        g, beta = ref.gdn_gates(ba[s0:s1, Hv:], ba[s0:s1, :Hv], A_log, dt_bias)
        s_init = state0[bi + 1].float() if has_init[bi] else torch.zeros(Hv, D, D)
        o_ref, s_ref = ref.gdn_recurrent(q, k, vv, g, beta, s_init, scale)
        o_got = got[s0:s1].float().cpu().view(-1, Hv, D)
        assert rel_err(o_got, o_ref) < 3e-2, (bi, rel_err(o_got, o_ref))
        assert rel_err(st_chunk[bi + 1].float().cpu(), s_ref) < 3e-2, bi
        assert rel_err(o_got, serial[s0:s1].float().cpu().view(-1, Hv, D)) < 3e-2, bi


@pytest.mark.parametrize("split", [1, 2, 4])
@pytest.mark.parametrize("B,Hk,Hv,sdt,init", [(1, 4, 12, torch.float32, 1), (5, 2, 6, torch.float32, 1),
                                              (3, 4, 4, torch.bfloat16, 1), (2, 2, 6, torch.float32, 0)])
def test_gdn_decode_fused_matches_separate(B, Hk, Hv, sdt, init, split):
    """One-launch GDN decode step against conv (+ in-place state shift) followed by the
    token-serial recurrence: outputs, SSM states and conv states."""
    torch.manual_seed(11)
    D = 128
    key_dim, vdim = Hk * D, Hv * D
    C = 2 * key_dim + vdim
    ncol = C + vdim + 2 * Hv + 8
    x = (torch.randn(B, ncol) * 0.7).to(torch.bfloat16).to(DEV)
    conv_w = (0.4 * torch.randn(C, 4)).to(torch.bfloat16).to(DEV)
    conv0 = (0.5 * torch.randn(B + 1, C, 3)).to(torch.bfloat16).to(DEV)
    ssm0 = (torch.randn(B + 1, Hv, D, D) * 0.05).to(sdt).to(DEV)
    A_log = torch.log(torch.rand(Hv) * 8 + 0.5).to(DEV)
    dt_bias = (torch.randn(Hv) * 0.3).to(DEV)
    meta = _Meta()
    meta.query_start_loc = torch.arange(B + 1, dtype=torch.int32, device=DEV)
    meta.state_slots = torch.arange(1, B + 1, dtype=torch.int32, device=DEV)
    meta.has_initial = torch.full((B,), init, dtype=torch.int32, device=DEV)
    meta.token_seq = torch.arange(B, dtype=torch.int32, device=DEV)
    meta.num_seqs = meta.num_tokens = B
    meta.commit_len = None
    scale = D ** -0.5
    ba_off = C + vdim
    c1, s1 = conv0.clone(), ssm0.clone()
    got = K.gdn_decode_fused(x, ba_off, conv_w, c1, s1, A_log, dt_bias, meta, Hk, scale,
                             split=split)
    c2, s2 = conv0.clone(), ssm0.clone()
    y = K.gdn_conv(x[:, :C], conv_w, c2, meta, key_dim, D, update_state=True)
    want = K.gdn_recurrent(y, x[:, ba_off:ba_off + 2 * Hv], A_log, dt_bias, s2, meta, Hk, scale)
    torch.cuda.synchronize()
    assert rel_err(got, want) < 1e-2, rel_err(got, want)
    assert rel_err(s1.float(), s2.float()) < 1e-2
    assert torch.equal(c1, c2)


@pytest.mark.parametrize("B,Hk,Hv,sdt", [(1, 16, 48, torch.float32), (4, 4, 12, torch.float32),
                                         (3, 4, 4, torch.bfloat16)])
def test_gdn_decode_fused_quant(B, Hk, Hv, sdt):
    """The decode step with the out_proj producer inside (per-head gated RMSNorm in the head's
    CTA, per-row e4m3 by the last head CTA) against the step followed by gdn_norm_quant; two
    launches in a row (the per-row counters reset)."""
    torch.manual_seed(12)
    D = 128
    key_dim, vdim = Hk * D, Hv * D
    C = 2 * key_dim + vdim
    ncol = C + vdim + 2 * Hv + 8
    conv_w = (0.4 * torch.randn(C, 4)).to(torch.bfloat16).to(DEV)
    A_log = torch.log(torch.rand(Hv) * 8 + 0.5).to(DEV)
    dt_bias = (torch.randn(Hv) * 0.3).to(DEV)
    norm_w = (1 + 0.1 * torch.randn(D)).to(torch.bfloat16).to(DEV)
    meta = _Meta()
    meta.query_start_loc = torch.arange(B + 1, dtype=torch.int32, device=DEV)
    meta.state_slots = torch.arange(1, B + 1, dtype=torch.int32, device=DEV)
    meta.has_initial = torch.ones(B, dtype=torch.int32, device=DEV)
    meta.token_seq = torch.arange(B, dtype=torch.int32, device=DEV)
    meta.num_seqs = meta.num_tokens = B
    meta.commit_len = None
    scale = D ** -0.5
    ba_off = C + vdim
    conv0 = (0.5 * torch.randn(B + 1, C, 3)).to(torch.bfloat16).to(DEV)
    ssm0 = (torch.randn(B + 1, Hv, D, D) * 0.05).to(sdt).to(DEV)
    c1, s1, c2, s2 = conv0.clone(), ssm0.clone(), conv0.clone(), ssm0.clone()
    for rep in range(2):
        x = (torch.randn(B, ncol) * 0.7).to(torch.bfloat16).to(DEV)
        q, qs = K.gdn_decode_fused_quant(x, ba_off, C, conv_w, c1, s1, A_log, dt_bias, meta, Hk,
                                         scale, norm_w, 1e-6)
        o = K.gdn_decode_fused(x, ba_off, conv_w, c2, s2, A_log, dt_bias, meta, Hk, scale, split=1)
        wq, wqs = K.gdn_norm_quant(o, x[:, C:C + vdim], norm_w, 1e-6, D)
        torch.cuda.synchronize()
        assert torch.equal(c1, c2) and torch.equal(s1, s2), rep
        torch.testing.assert_close(qs, wqs, rtol=1e-5, atol=0)
        assert fp8_close(q, qs, wq, wqs), rep


def test_qkv_prologue():
    torch.manual_seed(1)
    T, Hq, Hkv, D, rot = 5, 4, 2, 256, 64
    bs = 64
    qkv = torch.randn(T, Hq * D * 2 + 2 * Hkv * D).to(torch.bfloat16)
    pos = torch.tensor([0, 1, 7, 300, 65000], dtype=torch.int32)
    qn = (0.1 * torch.randn(D)).to(torch.bfloat16)
    kn = (0.1 * torch.randn(D)).to(torch.bfloat16)
    slots = torch.tensor([3, 64, 65, 130, 200], dtype=torch.int64)
    kc = torch.zeros(4, Hkv, bs, D, dtype=torch.float8_e4m3fn)
    vc = torch.zeros_like(kc)
    kw = dict(num_q_heads=Hq, num_kv_heads=Hkv, head_dim=D, rotary_dim=rot, theta=1e7, eps=1e-6,
              gated=True, block_size=bs)
    qw = K.qkv_prologue(qkv, pos, qn, kn, None, kc, vc, slots, **kw)
    from vllm_sly_radiance_b200.models.layers import rope_cache
    cs = rope_cache(70000, rot, 1e7, DEV)
    kcg, vcg = torch.zeros_like(kc).to(DEV), torch.zeros_like(vc).to(DEV)
    qg = K.qkv_prologue(qkv.to(DEV), pos.to(DEV), qn.to(DEV), kn.to(DEV), cs, kcg, vcg,
                        slots.to(DEV), **kw)
    torch.cuda.synchronize()
    assert rel_err(qg, qw) < 2e-2
    assert rel_err(kcg.float(), kc.float()) < 2e-2
    assert torch.equal(vcg.cpu().float(), vc.float())


@pytest.mark.parametrize("Dh", [64, 128])
def test_gdn_conv_and_recurrent(Dh):
    """Varlen conv (head 64: per-token kernel; head 128: the token-tiled prefill kernel, whose
    8-token tiles here straddle sequence boundaries) and the recurrent rule against the oracle."""
    torch.manual_seed(2)
    Hk, Hv, W = 2, 4, 4
    key_dim, vdim = Hk * Dh, Hv * Dh
    C = 2 * key_dim + vdim
    q_lens = [1, 5, 70]
    has_init = [1, 1, 0]
    slots = [2, 0, 1]
    qsl = [0, 1, 6, 76]
    T = qsl[-1]
    x = torch.randn(T, C + vdim + 2 * Hv).to(torch.bfloat16)
    conv_w = (0.3 * torch.randn(C, W)).to(torch.bfloat16)
    conv_state = torch.randn(3, C, W - 1).to(torch.bfloat16)
    ssm = torch.randn(3, Hv, Dh, Dh) * 0.1
    A_log = torch.log(torch.rand(Hv) * 15 + 1)
    dt_bias = torch.randn(Hv) * 0.1
    m = _Meta()
    m.num_seqs = 3
    m.num_tokens = T
    m.query_start_loc = torch.tensor(qsl, dtype=torch.int32)
    m.state_slots = torch.tensor(slots, dtype=torch.int32)
    m.has_initial = torch.tensor(has_init, dtype=torch.int32)
    m.token_seq = torch.tensor(sum([[b] * l for b, l in enumerate(q_lens)], []), dtype=torch.int32)
    mg = _Meta()
    for k_ in ("query_start_loc", "state_slots", "has_initial", "token_seq"):
        setattr(mg, k_, getattr(m, k_).to(DEV))
    mg.num_seqs = 3
    mg.num_tokens = T
    y_w = K.gdn_conv(x[:, :C], conv_w, conv_state, m, key_dim, Dh)
    y_g = K.gdn_conv(x.to(DEV)[:, :C], conv_w.to(DEV), conv_state.to(DEV), mg, key_dim, Dh)
    torch.cuda.synchronize()
    assert rel_err(y_g, y_w) < 2e-2
    ba = x[:, C + vdim:]
    ssm_w = ssm.clone()
    o_w = K.gdn_recurrent(y_w, ba, A_log, dt_bias, ssm_w, m, Hk, Dh ** -0.5)
    ssm_g = ssm.clone().to(DEV)
    o_g = K.gdn_recurrent(y_w.to(DEV), ba.to(DEV), A_log.to(DEV), dt_bias.to(DEV), ssm_g, mg, Hk,
                          Dh ** -0.5)
    torch.cuda.synchronize()
    assert rel_err(o_g, o_w) < 2e-2
    # head 128 takes the chunked (tensor-core) scan: bf16 operands, a few 1e-3 of the state
    assert rel_err(ssm_g, ssm_w) < (1e-3 if Dh == 64 else 3e-2)
    cs_w = conv_state.clone()
    K.gdn_conv_state_update(x[:, :C], cs_w, m)
    cs_g = conv_state.clone().to(DEV)
    K.gdn_conv_state_update(x.to(DEV)[:, :C], cs_g, mg)
    torch.cuda.synchronize()
    assert torch.equal(cs_g.cpu(), cs_w)


def test_argmax_and_sampling():
    torch.manual_seed(3)
    x = torch.randn(5, 248320).to(torch.bfloat16)
    ids = K.argmax(x.to(DEV))
    assert torch.equal(ids.cpu(), x.float().argmax(-1))
    vals, idx = torch.topk(x.float(), 64, dim=-1)
    B = 5
    temp = torch.tensor([0.0, 0.7, 1.0, 0.7, 0.7])
    topk = torch.tensor([20, 20, 0, 1, 64], dtype=torch.int32)
    topp = torch.tensor([0.95, 0.95, 1.0, 0.9, 0.5])
    seeds = torch.arange(B, dtype=torch.int64)
    out, probs = K.sample_from_topk(vals.to(DEV), idx.to(DEV), temp.to(DEV), topk.to(DEV),
                                    topp.to(DEV), None, seeds.to(DEV), 0, want_probs=True)
    torch.cuda.synchronize()
    out = out.cpu()
    assert out[0] == idx[0, 0] and out[3] == idx[3, 0]
    for b in range(B):
        assert int(out[b]) in idx[b].tolist()
    # probabilities of the kept window sum to one for sampled rows
    for b in (1, 2, 4):
        assert abs(float(probs[b].sum()) - 1.0) < 1e-4


@pytest.mark.parametrize("B,V,dtype", [(1, 248320, torch.bfloat16), (5, 248320, torch.float32),
                                      (3, 4096, torch.bfloat16), (2, 5000, torch.float32)])
def test_topk_window_matches_sorted_prefix(B, V, dtype):
    """The top-64 window kernel equals the first 64 entries of a stable descending sort (ties
    at equal values keep the lowest column), on two launches in a row (counters reset)."""
    for rep in range(2):
        g = torch.Generator().manual_seed(B * 31 + V + rep)
        x = torch.randn(B, V, generator=g).to(dtype)       # bf16 rows hold many ties
        vals, ids = K.topk_window(x.to(DEV))
        torch.cuda.synchronize()
        nv, ni = torch.sort(-x.float(), dim=-1, stable=True)
        assert torch.equal(vals.cpu(), -nv[:, :64])
        assert torch.equal(ids.cpu(), ni[:, :64])


def test_topk_fused_draw_equals_window_draw():
    """The draw fused into the window kernel is the per-row window draw of sample_from_topk."""
    torch.manual_seed(5)
    B = 6
    x = torch.randn(B, 248320).to(torch.bfloat16).to(DEV)
    temp = torch.tensor([0.0, 0.7, 1.0, 0.7, 0.7, 1.3], device=DEV)
    topk = torch.tensor([20, 20, 64, 1, 64, 5], dtype=torch.int32, device=DEV)
    topp = torch.tensor([0.95, 0.95, 1.0, 0.9, 0.5, 0.8], device=DEV)
    minp = torch.tensor([0.0, 0.0, 0.05, 0.0, 0.0, 0.0], device=DEV)
    seeds = torch.arange(B, dtype=torch.int64, device=DEV) * 7
    for step in (0, 3):
        toks, probs, ids = K.topk_sample(x, temp, topk, topp, minp, seeds, step, want_probs=True)
        vals, ids2 = K.topk_window(x)
        want, wprobs = K.sample_from_topk(vals, ids2, temp, topk, topp, minp, seeds, step,
                                          want_probs=True)
        torch.cuda.synchronize()
        assert torch.equal(ids.cpu(), ids2.cpu())
        assert torch.equal(toks.cpu(), want.cpu())
        assert torch.allclose(probs.cpu(), wprobs.cpu(), atol=1e-6)
    assert int(toks[0]) == int(x[0].float().argmax())


def test_full_vocab_sampling_distribution():
    """top_k disabled: rows are drawn over the whole vocabulary (sorted row + the same draw);
    the empirical distribution matches softmax, mass beyond the top 64 included."""
    from vllm_sly_radiance_b200.engine.sampler import SamplingTensors, sample
    V, N = 4096, 8000
    g = torch.Generator().manual_seed(1)
    row = torch.randn(V, generator=g) * 0.2
    st = SamplingTensors(torch.ones(N, device=DEV), torch.zeros(N, dtype=torch.int32, device=DEV),
                         torch.ones(N, device=DEV), torch.zeros(N, device=DEV),
                         torch.arange(N, dtype=torch.int64, device=DEV) * 13 + 1, False, False, True)
    toks, _, _ = sample(row[None].expand(N, V).contiguous().to(DEV), st, 0)
    emp = torch.bincount(toks.cpu(), minlength=V).double() / N
    want = torch.softmax(row.double(), 0)
    order = torch.argsort(row, descending=True)
    assert abs(float(emp[order[64:]].sum()) - float(want[order[64:]].sum())) < 0.03
    # coarse bins of 64 ranks: per-bin mass within sampling noise
    eb = emp[order].view(64, 64).sum(1)
    wb = want[order].view(64, 64).sum(1)
    assert float((eb - wb).abs().max()) < 0.02


@pytest.mark.parametrize("D,Hq,Hkv,splits", [(64, 4, 2, 5), (256, 24, 4, 8)])
def test_paged_attention_split_repeated(D, Hq, Hkv, splits):
    """Back-to-back split-KV launches on the same metadata (as in CUDA-graph replays): the
    in-kernel merge counters reset and no partial of a previous launch leaks into the next."""
    torch.manual_seed(5)
    bs = 64
    q_lens, ctx = [1, 1, 1, 1], [121, 55, 10, 0]
    meta, nblocks = _attn_meta(q_lens, ctx, bs, Hq, Hkv, splits, DEV)
    kc = (torch.randn(nblocks, Hkv, bs, D) * 0.5).to(torch.float8_e4m3fn)
    vc = torch.randn(nblocks, Hkv, bs, D).to(torch.float8_e4m3fn)
    metac = _Meta()
    metac.block_tables = meta.block_tables.cpu()
    metac.seq_lens = meta.seq_lens.cpu()
    metac.query_start_loc = meta.query_start_loc.cpu()
    kg, vg = kc.to(DEV), vc.to(DEV)
    for it in range(4):
        q = ref.fp8_e4m3(torch.randn(4, Hq, D)).to(torch.bfloat16)
        want = ref.paged_attention(q, kc, vc, metac.block_tables, metac.seq_lens,
                                   metac.query_start_loc, bs, D ** -0.5)
        got = K.paged_attention(q.to(DEV), kg, vg, meta, D ** -0.5)
        torch.cuda.synchronize()
        assert rel_err(got, want) < 2e-2, (it, rel_err(got, want))


@pytest.mark.parametrize("R_per_expert", [1, 3, 40, 300])
def test_moe_grouped_gemm(R_per_expert):
    """Grouped tcgen05 GEMM over stacked expert weights vs per-expert fp32 references."""
    from vllm_sly_radiance_b200.quant.mxfp4 import MXFP4Weight, cat_rows
    torch.manual_seed(7)
    E, N, Kd = 6, 256, 512
    ws = [MXFP4Weight.from_float(torch.randn(N, Kd) * 0.02) for _ in range(E)]
    stacked = cat_rows(ws)
    counts = torch.tensor([R_per_expert, 0, 2 * R_per_expert, 1, R_per_expert, 0])
    R = int(counts.sum())
    x = torch.randn(R, Kd).to(torch.bfloat16)
    q, s = ref.quant_fp8_rows(x)
    want = torch.empty(R, N)
    r0 = 0
    for e in range(E):
        c = int(counts[e])
        if c:
            want[r0:r0 + c] = ref.mxfp4_linear(q[r0:r0 + c], s[r0:r0 + c], ws[e].packed, ws[e].scales).float()
        r0 += c
    sg = stacked.to(DEV)
    got = K.moe_grouped_gemm(q.to(DEV), s.to(DEV), sg, N, counts.to(DEV))
    torch.cuda.synchronize()
    K.check_status(got.device)
    assert rel_err(got, want) < 1e-2, rel_err(got, want)


def test_segment_copy_gather_scatter_roundtrip():
    """The offload copy engine: segments of items (block / slot indices) of several cache tensors
    pack into a contiguous staging buffer exactly, and unpack into other items exactly."""
    from vllm_sly_radiance_b200.ops._ext import ext
    g = torch.Generator().manual_seed(9)
    ts = [torch.randint(0, 255, (12, 2, 16, 64), generator=g, dtype=torch.uint8).to(DEV),
          torch.randn(12, 3, 40, generator=g).to(torch.bfloat16).to(DEV),
          torch.randn(12, 4, 8, 8, generator=g).to(DEV)]
    seg = [t[0].numel() * t.element_size() for t in ts]
    offs = [0, seg[0], seg[0] + seg[1]]
    item = sum(seg)
    table = torch.tensor([[t.data_ptr(), t.stride(0) * t.element_size(), b] for t, b in zip(ts, seg)],
                         dtype=torch.int64, device=DEV)
    offs_t = torch.tensor(offs, dtype=torch.int64, device=DEV)
    idx = torch.tensor([7, 2, 11], dtype=torch.int32, device=DEV)
    stage = torch.empty(3, item, dtype=torch.uint8, device=DEV)
    ext().segment_copy(table, offs_t, idx, stage, item, True)
    for k, i in enumerate([7, 2, 11]):
        for t, o, b in zip(ts, offs, seg):
            assert torch.equal(stage[k, o:o + b], t[i].reshape(-1).view(torch.uint8))
    ref = [t.clone() for t in ts]
    dst = torch.tensor([1, 5, 9], dtype=torch.int32, device=DEV)
    ext().segment_copy(table, offs_t, dst, stage, item, False)
    torch.cuda.synchronize()
    for t, r in zip(ts, ref):
        assert torch.equal(t[[1, 5, 9]], r[[7, 2, 11]])
        keep = [j for j in range(12) if j not in (1, 5, 9)]
        assert torch.equal(t[keep], r[keep])


@pytest.mark.parametrize("bits", [8, 4])
def test_embed_gather_quantised(bits):
    """int8 / int4-g128 embedding lookup kernel equals the PyTorch dequantisation of the rows."""
    from vllm_sly_radiance_b200.quant.embed import QuantEmbedding
    g = torch.Generator().manual_seed(bits)
    w = (torch.randn(1000, 5120, generator=g) * 0.03).to(torch.bfloat16)
    qe = QuantEmbedding.from_float(w, bits)
    ids = torch.tensor([3, 999, 0, 3, 512, 77], dtype=torch.int64)
    want = qe.dequantize_rows(ids)
    got = qe.to(DEV)[ids.to(DEV)]
    torch.cuda.synchronize()
    assert torch.equal(got.cpu(), want)
