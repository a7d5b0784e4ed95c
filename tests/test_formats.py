"""Number formats: E2M1 / UE8M0 / MXFP4, e4m3 per-token, NVFP4 requant, INT4, SF tile layout."""
import pytest
import torch

from vllm_sly_radiance_b200.ops import reference as ref
from vllm_sly_radiance_b200.quant import formats as F
from vllm_sly_radiance_b200.quant.mxfp4 import MXFP4Weight, cat_rows


def test_e2m1_roundtrip_and_ties():
    vals = torch.tensor([0, 0.5, 1, 1.5, 2, 3, 4, 6, -0.5, -6], dtype=torch.float32)
    assert torch.equal(F.e2m1_decode(F.e2m1_encode(vals)), vals)
    # ties go to the even code: 0.25->0, 0.75->1.0, 1.25->1.0, 1.75->2.0, 2.5->2, 3.5->4, 5->4
    ties = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0])
    assert F.e2m1_decode(F.e2m1_encode(ties)).tolist() == [0.0, 1.0, 1.0, 2.0, 2.0, 4.0, 4.0]
    assert F.e2m1_decode(F.e2m1_encode(torch.tensor([100.0, -7.0]))).tolist() == [6.0, -6.0]


def test_ue8m0_ocp_rule():
    # floor(log2 amax) - 2 + 127; zero block -> 0
    amax = torch.tensor([6.0, 1.0, 0.75, 0.0, 2 ** -130])
    b = F.ue8m0_ocp(amax)
    assert b.tolist() == [127, 125, 124, 0, 0]


def test_mxfp4_quant_error_and_packing():
    torch.manual_seed(0)
    w = torch.randn(64, 256)
    packed, scales = F.mxfp4_quantize(w)
    assert packed.shape == (64, 128) and scales.shape == (64, 8)
    dq = F.mxfp4_dequantize(packed, scales)
    rel = ((dq - w).norm() / w.norm()).item()
    assert rel < 0.15, rel
    # low nibble holds the even index
    codes = F.unpack_nibbles(packed)
    assert torch.equal(codes[:, 0], packed[:, 0] & 0xF)
    assert torch.equal(F.pack_nibbles(codes), packed)


def test_sf_tile_layout_roundtrip():
    s = torch.randint(0, 255, (300, 20), dtype=torch.uint8)
    t = F.sf_tile_layout(s)
    assert t.numel() == 384 * 20
    assert torch.equal(F.sf_tile_layout_inverse(t, 300, 20), s)
    # byte (n%32)*16 + ((n%128)//32)*4 + kb%4 of atom (n//128, kb//4)
    n, kb = 130, 9
    atoms_k = 20 // 4
    off = ((n // 128) * atoms_k + kb // 4) * 512 + (n % 32) * 16 + ((n % 128) // 32) * 4 + kb % 4
    assert int(t[off]) == int(s[n, kb])


def test_per_token_fp8():
    x = torch.randn(5, 64) * 10
    q, s = F.per_token_fp8(x)
    assert q.dtype == torch.float8_e4m3fn
    dq = F.per_token_fp8_dequant(q, s)
    assert ((dq - x.to(torch.bfloat16).float()).abs().max() / x.abs().max()) < 0.07
    z, sz = F.per_token_fp8(torch.zeros(2, 16))
    assert torch.all(sz == F.FP8_SCALE_FLOOR)


def test_nvfp4_requant_and_int4():
    torch.manual_seed(1)
    w = torch.randn(32, 128)
    p, bs, gs = F.nvfp4_quantize(w)
    mp, ms = F.nvfp4_to_mxfp4(p, bs, gs)
    dq = F.mxfp4_dequantize(mp, ms)
    assert ((dq - w).norm() / w.norm()) < 0.2
    p4, sc, zp = F.int4_g128_quantize(w)
    dq4 = F.int4_g128_dequantize(p4, sc, zp)
    assert ((dq4 - w).norm() / w.norm()) < 0.15


def test_mxfp4_weight_slicing():
    w = torch.randn(256, 512)
    mw = MXFP4Weight.from_float(w)
    a = mw.narrow_rows(0, 128)
    b = mw.narrow_rows(128, 128)
    cat = cat_rows([a, b])
    assert torch.equal(cat.packed, mw.packed) and torch.equal(cat.sf, mw.sf)
    c = mw.narrow_cols(256, 256)
    assert torch.equal(c.dequantize(), mw.dequantize()[:, 256:])


def test_mxfp4_weight_k_tail_padding():
    """K not a multiple of the 128-wide GEMM tile: the stored weight is zero-padded to whole
    tiles, the logical K is kept, and a linear over the padded weight equals the unpadded one."""
    g = torch.Generator().manual_seed(0)
    w = torch.randn(40, 8704, generator=g) * 0.02
    full = MXFP4Weight.from_float(w)
    shard = full.narrow_cols(1088 * 3, 1088)
    assert shard.K == 1088 and shard.K_padded == 1152
    assert torch.equal(shard.dequantize(), full.dequantize()[:, 1088 * 3:1088 * 4])
    assert int(shard.packed[:, 1088 // 2:].sum()) == 0
    x = torch.randn(3, 1088, generator=g)
    q, s = ref.quant_fp8_rows(x.to(torch.bfloat16))
    got = ref.mxfp4_linear(q, s, shard.packed, shard.scales).float()
    want = ((q.float() @ shard.dequantize().t()) * s[:, None]).to(torch.bfloat16).float()
    assert torch.equal(got, want)


def test_int4_weight_roundtrip_and_clip_search():
    """INT4 g128 container: dequantisation matches the format, the MSE clip search never loses to
    the plain min/max range, and the host W4A16 linear is x @ dequant(w)^T."""
    from vllm_sly_radiance_b200.quant.int4 import Int4Weight, w4a16_linear
    g = torch.Generator().manual_seed(5)
    w = torch.randn(64, 512, generator=g)
    w[3, 7] = 9.0                                            # an outlier group
    plain = Int4Weight.from_float(w)
    clipped = Int4Weight.from_float(w, clip_search=True)
    e_plain = float((plain.dequantize() - w).pow(2).sum())
    e_clip = float((clipped.dequantize() - w).pow(2).sum())
    assert e_clip <= e_plain + 1e-6 and e_clip / float(w.pow(2).sum()) < 0.02
    x = torch.randn(5, 512, generator=g).to(torch.bfloat16)
    y = w4a16_linear(x, clipped)
    want = (x.float() @ clipped.dequantize().t()).to(torch.bfloat16)
    assert torch.equal(y, want)
    assert clipped.nbytes == 64 * 256 + 64 * 4 * 3


def test_int4_fragment_tiling_roundtrip():
    """The tensor-core fragment layout of int4 weights is a pure permutation: nibble i = h + 2c + 4p
    of lane 4g + t, step s of tile T / block kb is w[16T + 8h + g, 64kb + 16t + 4s + 2c + p]."""
    from vllm_sly_radiance_b200.quant.formats import unpack_nibbles
    from vllm_sly_radiance_b200.quant.int4 import Int4Weight, mma_tile, mma_untile
    w = Int4Weight.from_float(torch.randn(40, 384))
    wt, sz = mma_tile(w.packed, w.scales, w.zeros)
    assert wt.shape == (48, 192) and sz.shape == (3, 3, 8, 2)
    p, s, z = mma_untile(wt, sz, 40, 384)
    assert torch.equal(p, w.packed) and torch.equal(s, w.scales) and torch.equal(z, w.zeros)
    q = unpack_nibbles(w.packed)
    words = wt.view(torch.int32).view(3, 6, 32, 4)
    g = torch.Generator().manual_seed(0)
    for _ in range(100):
        T, kb, lane, st, i = (int(torch.randint(0, n, (1,), generator=g)) for n in (2, 6, 32, 4, 8))
        h, c, pp = i & 1, (i >> 1) & 1, i >> 2
        v = (int(words[T, kb, lane, st]) >> (4 * i)) & 15
        assert v == int(q[16 * T + 8 * h + lane // 4, 64 * kb + 16 * (lane % 4) + 4 * st + 2 * c + pp])
    # scale/zero words: fp16 pair of rows (g, g + 8), bf16 bits of 128 + zero
    sw = int(sz[1, 2, 5, 0]) & 0xFFFF
    assert torch.tensor([sw], dtype=torch.int32).to(torch.int16).view(torch.float16) == w.scales[21, 2]
    assert ((int(sz[1, 2, 5, 1]) >> 16) & 0xFFFF) - 0x4300 == int(w.zeros[29, 2])


def test_quant_embedding_roundtrip():
    """int8 (per-row) and int4 (g128) embedding tables: the lookup dequantises to within half a
    quantisation step of the bf16 table (reference: radiance_embed_int8.py:47-114)."""
    from vllm_sly_radiance_b200.quant.embed import QuantEmbedding
    g = torch.Generator().manual_seed(0)
    w = (torch.randn(300, 256, generator=g) * 0.05).to(torch.bfloat16)
    ids = torch.tensor([0, 5, 299, 5, 17])
    for bits, tol in ((8, 1 / 127), (4, 1 / 7)):
        qe = QuantEmbedding.from_float(w, bits)
        got = qe[ids].float()
        want = w[ids].float()
        step = want.abs().amax(1, keepdim=True) * tol
        assert ((got - want).abs() <= 0.51 * step + 4e-3 * want.abs()).all(), bits
    assert QuantEmbedding.from_float(w, 4).nbytes < w.numel() * 2 // 3


# ---- MXFP6 (e2m3) / MXFP8 (e4m3) weights ----------------------------------------------------
def test_e2m3_grid_and_rounding():
    # every code decodes to the OCP E2M3 value (bias 1, subnormals k/8) and encodes back
    codes = torch.arange(64, dtype=torch.uint8)
    vals = F.e2m3_decode(codes)
    for c in range(64):
        sgn = -1.0 if c & 32 else 1.0
        e, m = (c >> 3) & 3, c & 7
        want = m / 8 if e == 0 else (1 + m / 8) * 2.0 ** (e - 1)
        assert float(vals[c]) == sgn * want, c
    nz = codes[(codes != 32)]                    # -0 encodes as +0
    assert torch.equal(F.e2m3_encode(F.e2m3_decode(nz)), nz)
    # saturation and ties to even code: 7.75 -> 7.5, 0.0625 (between 0 and 1/8) -> 0
    x = torch.tensor([100.0, -100.0, 7.75, 0.0625, 0.1875, 1.0625])
    got = F.e2m3_decode(F.e2m3_encode(x)).tolist()
    assert got == [7.5, -7.5, 7.5, 0.0, 0.25, 1.0]


def test_pack_6bit_layout():
    # four codes per three bytes, code i at bits [6i, 6i + 6) of the little-endian 24-bit word
    codes = torch.tensor([[1, 2, 3, 63]], dtype=torch.uint8)
    word = 1 | (2 << 6) | (3 << 12) | (63 << 18)
    assert F.pack_6bit(codes).tolist() == [[word & 255, (word >> 8) & 255, word >> 16]]
    c = torch.randint(0, 64, (5, 64), dtype=torch.uint8)
    assert torch.equal(F.unpack_6bit(F.pack_6bit(c)), c)


@pytest.mark.parametrize("fmt,bits,tol", [("e2m1", 4, 0.15), ("e2m3", 6, 0.05), ("e4m3", 8, 0.04)])
def test_mx_formats_quantize(fmt, bits, tol):
    g = torch.Generator().manual_seed(1)
    w = torch.randn(48, 320, generator=g)
    p, s = F.mx_quantize(w, fmt)
    assert p.shape == (48, 320 * bits // 8) and s.shape == (48, 10)
    dq = F.mx_dequantize(p, s, fmt)
    assert ((dq - w).norm() / w.norm()).item() < tol
    # the block maximum never saturates: amax / 2^(floor(log2 amax) - emax) < 2^(emax + 1)
    blk = w.view(48, 10, 32).abs().amax(-1)
    scale = F.ue8m0_to_float(s)
    limit = {"e2m1": 6.0, "e2m3": 7.5, "e4m3": 448.0}[fmt]
    assert bool(((blk / scale) < 2 * limit).all())


@pytest.mark.parametrize("fmt", ["e2m3", "e4m3"])
def test_mx_weight_container(fmt):
    from vllm_sly_radiance_b200.quant.mxfp4 import cat_rows
    g = torch.Generator().manual_seed(2)
    w = torch.randn(40, 8704, generator=g) * 0.02
    full = MXFP4Weight.from_float(w, fmt)
    assert full.fmt == fmt and full.K_padded == 8704
    shard = full.narrow_cols(1088 * 3, 1088)
    assert shard.fmt == fmt and shard.K == 1088 and shard.K_padded == 1152
    assert torch.equal(shard.dequantize(), full.dequantize()[:, 1088 * 3:1088 * 4])
    rows = full.narrow_rows(8, 16)
    assert torch.equal(rows.dequantize(), full.dequantize()[8:24])
    both = cat_rows([rows, full.narrow_rows(0, 8)])
    assert both.fmt == fmt and both.N == 24
    padded = shard.pad_cols(1152 + 32)
    assert torch.equal(padded.dequantize()[:, :1088], shard.dequantize())
    assert float(padded.dequantize()[:, 1088:].abs().sum()) == 0.0
    x = torch.randn(3, 1088, generator=g)
    q, s = ref.quant_fp8_rows(x.to(torch.bfloat16))
    got = ref.mxfp4_linear(q, s, shard.packed, shard.scales, fmt=fmt).float()
    want = ((q.float() @ shard.dequantize().t()) * s[:, None]).to(torch.bfloat16).float()
    assert torch.equal(got, want)


def test_mx_cast_weights_keeps_mxfp4_values():
    """An MXFP4 linear served as MXFP8 is exact (e2m1 x 2^s is representable in e4m3 x 2^s')."""
    from vllm_sly_radiance_b200.models.weights import MXCastWeights

    class Src:
        cfg = None

        def linear(self, name, N, K):
            return MXFP4Weight.from_float(torch.randn(N, K, generator=torch.Generator().manual_seed(3)))
    src = Src()
    w8 = MXCastWeights(src, "e4m3").linear("x", 16, 256)
    assert w8.fmt == "e4m3"
    assert torch.equal(w8.dequantize(), src.linear("x", 16, 256).dequantize())
    assert MXCastWeights(src, "e4m3", skip=("x",)).linear("x", 16, 256).fmt == "e2m1"
