"""Checkpoint loader: a synthetic Qwen3-Next-named safetensors checkpoint (bf16, MXFP4
compressed-tensors, NVFP4) loads into the same model the canonical weights define."""
import os

import pytest
import torch
from safetensors.torch import save_file

from vllm_sly_radiance_b200.config import tiny_hybrid
from vllm_sly_radiance_b200.models.hybrid import HybridModel
from vllm_sly_radiance_b200.models.weights import RandomWeights
from vllm_sly_radiance_b200.quant import formats as F
from vllm_sly_radiance_b200.quant.loaders import CheckpointWeights, gdn_in_proj_permutation


class Recorder(RandomWeights):
    """Random provider that remembers what it handed out (the canonical truth)."""

    def __init__(self, cfg):
        super().__init__(cfg, 0, "cpu")
        self.lin, self.ten = {}, {}

    def linear(self, name, N, K):
        w = super().linear(name, N, K).to(torch.bfloat16).float()   # bf16-representable truth
        self.lin[name] = w.clone()
        return w

    def tensor(self, name, shape, kind="norm"):
        t = super().tensor(name, shape, kind)
        self.ten[name] = t.clone()
        return t


def _write_hf(rec, cfg, path, fmt):
    sd = {}

    def put_linear(hf, w):
        if fmt == "bf16":
            sd[hf + ".weight"] = w.to(torch.bfloat16)
        elif fmt == "mxfp4":
            p, s = F.mxfp4_quantize(w)
            sd[hf + ".weight_packed"] = p
            sd[hf + ".weight_scale"] = s
        elif fmt == "mxfp6":
            p, s = F.mx_quantize(w, "e2m3")
            sd[hf + ".weight_packed"] = p
            sd[hf + ".weight_scale"] = s
        elif fmt == "int4":       # compressed-tensors pack-quantized, 8 nibbles per int32
            p, sc, zp = F.int4_g128_quantize(w)
            sd[hf + ".weight_packed"] = p.contiguous().view(torch.int32)
            sd[hf + ".weight_scale"] = sc
            sd[hf + ".weight_zero_point"] = zp
        elif fmt == "gptq":       # GPTQ v1 / AutoRound layout: K-packed qweight, N-packed qzeros
            p, sc, zp = F.int4_g128_quantize(w)
            N, K = w.shape
            q = F.unpack_nibbles(p).to(torch.int32).t().contiguous()            # [K, N]
            qw = torch.zeros(K // 8, N, dtype=torch.int32)
            for i in range(8):
                qw |= q[i::8] << (4 * i)
            zq = (zp.to(torch.int32) - 1).t().contiguous()                       # [K/g, N], zero-1
            qz = torch.zeros(zq.shape[0], (N + 7) // 8, dtype=torch.int32)
            for i in range(8):
                col = zq[:, i::8]
                qz[:, :col.shape[1]] |= (col & 0xF) << (4 * i)
            sd[hf + ".qweight"] = qw
            sd[hf + ".scales"] = sc.t().contiguous()
            sd[hf + ".qzeros"] = qz
        elif fmt == "nvfp4":
            p, bs, gs = F.nvfp4_quantize(w)
            sd[hf + ".weight_packed"] = p
            sd[hf + ".weight_scale"] = bs
            sd[hf + ".weight_global_scale"] = (1.0 / gs).reshape(1)

    sd["model.embed_tokens.weight"] = rec.ten["embed"]
    sd["model.norm.weight"] = rec.ten["final_norm"]
    put_linear("lm_head", rec.lin["lm_head"])
    pq, pb = gdn_in_proj_permutation(cfg)
    kd, vd, hv = cfg.gdn_key_dim, cfg.gdn_value_dim, cfg.gdn_num_v_heads
    for i in range(cfg.num_layers):
        L = f"model.layers.{i}."
        c = f"layers.{i}."
        sd[L + "input_layernorm.weight"] = rec.ten[c + "ln1"]
        sd[L + "post_attention_layernorm.weight"] = rec.ten[c + "ln2"]
        g = rec.lin[c + "gate_up"]
        I = g.shape[0] // 2
        put_linear(L + "mlp.gate_proj", g[:I])
        put_linear(L + "mlp.up_proj", g[I:])
        put_linear(L + "mlp.down_proj", rec.lin[c + "down"])
        if cfg.is_attention_layer(i):
            w = rec.lin[c + "qkv"]
            qd = cfg.num_q_heads * cfg.head_dim * 2
            kvd = cfg.num_kv_heads * cfg.head_dim
            put_linear(L + "self_attn.q_proj", w[:qd])
            put_linear(L + "self_attn.k_proj", w[qd:qd + kvd])
            put_linear(L + "self_attn.v_proj", w[qd + kvd:])
            put_linear(L + "self_attn.o_proj", rec.lin[c + "o_proj"])
            sd[L + "self_attn.q_norm.weight"] = rec.ten[c + "q_norm"]
            sd[L + "self_attn.k_norm.weight"] = rec.ten[c + "k_norm"]
        else:
            w = rec.lin[c + "in_proj"]
            n_qkvz = 2 * kd + 2 * vd
            hf_qkvz = torch.empty_like(w[:n_qkvz])
            hf_qkvz[pq] = w[:n_qkvz]
            hf_ba = torch.empty_like(w[n_qkvz:])
            hf_ba[pb] = w[n_qkvz:]
            put_linear(L + "linear_attn.in_proj_qkvz", hf_qkvz)
            sd[L + "linear_attn.in_proj_ba.weight"] = hf_ba.to(torch.bfloat16)   # left unquantized
            put_linear(L + "linear_attn.out_proj", rec.lin[c + "out_proj"])
            sd[L + "linear_attn.conv1d.weight"] = rec.ten[c + "conv_w"].unsqueeze(1)
            sd[L + "linear_attn.A_log"] = rec.ten[c + "A_log"]
            sd[L + "linear_attn.dt_bias"] = rec.ten[c + "dt_bias"]
            sd[L + "linear_attn.norm.weight"] = rec.ten[c + "norm_w"]
    os.makedirs(path, exist_ok=True)
    keys = sorted(sd)
    half = len(keys) // 2       # two shards
    save_file({k: sd[k].contiguous() for k in keys[:half]}, os.path.join(path, "model-00001.safetensors"))
    save_file({k: sd[k].contiguous() for k in keys[half:]}, os.path.join(path, "model-00002.safetensors"))


@pytest.mark.parametrize("fmt", ["bf16", "mxfp4", "nvfp4"])
def test_load_matches_canonical(tmp_path, fmt):
    cfg = tiny_hybrid()
    rec = Recorder(cfg)
    ref_model = HybridModel(cfg, quant="mxfp4", device="cpu", weights=rec)
    _write_hf(rec, cfg, str(tmp_path), fmt)
    W = CheckpointWeights(str(tmp_path), cfg)
    m = HybridModel(cfg, quant="mxfp4", device="cpu", weights=W)
    l0, l1 = ref_model.layers[0], m.layers[0]
    if fmt in ("bf16", "mxfp4"):
        # MXFP4 from bf16 or from the packed checkpoint: bit-identical codes
        assert torch.equal(l0.mixer.in_proj.w.packed, l1.mixer.in_proj.w.packed)
        assert torch.equal(ref_model.layers[3].mixer.qkv.w.packed, m.layers[3].mixer.qkv.w.packed)
    else:
        a = l0.mixer.in_proj.w.dequantize()
        b = l1.mixer.in_proj.w.dequantize()
        assert ((a - b).norm() / a.norm()) < 0.2
    assert torch.equal(l0.mixer.conv_w, l1.mixer.conv_w)
    assert torch.equal(m.embed, ref_model.embed)


def test_mxfp6_checkpoint_model(tmp_path):
    """A whole MXFP6 checkpoint (merged GDN in_proj with its float ba part, qkv, gate_up) loads
    into the codes an mxfp6 model quantises from the same weights."""
    cfg = tiny_hybrid()
    rec = Recorder(cfg)
    ref_model = HybridModel(cfg, quant="mxfp6", device="cpu", weights=rec)
    _write_hf(rec, cfg, str(tmp_path), "mxfp6")
    m = HybridModel(cfg, quant="mxfp6", device="cpu", weights=CheckpointWeights(str(tmp_path), cfg))
    for a, b in ((ref_model.layers[0].mixer.in_proj, m.layers[0].mixer.in_proj),
                 (ref_model.layers[3].mixer.qkv, m.layers[3].mixer.qkv),
                 (ref_model.layers[1].mlp.gate_up, m.layers[1].mlp.gate_up)):
        assert a.w.fmt == b.w.fmt == "e2m3"
        assert torch.equal(a.w.packed, b.w.packed)


@pytest.mark.parametrize("fmt", ["int4", "gptq"])
def test_int4_checkpoint_stays_int4(tmp_path, fmt):
    """An INT4 (W4A16 pack-quantized) checkpoint served with quantization=int4 keeps its codes:
    the merged / sharded linears hold exactly the stored nibbles, scales and zero points (no
    dequantise + requantise), and the model runs close to the bf16 model."""
    from vllm_sly_radiance_b200.quant.int4 import Int4Weight
    cfg = tiny_hybrid()
    rec = Recorder(cfg)
    ref_model = HybridModel(cfg, quant="bf16", device="cpu", weights=rec)
    _write_hf(rec, cfg, str(tmp_path), fmt)
    W = CheckpointWeights(str(tmp_path), cfg)
    W.keep_int4 = True
    m = HybridModel(cfg, quant="int4", device="cpu", weights=W)
    down = m.layers[0].mlp.down.w
    assert isinstance(down, Int4Weight)
    p, s, z = F.int4_g128_quantize(rec.lin["layers.0.down"])
    assert torch.equal(down.packed, p) and torch.equal(down.zeros, z)
    assert torch.equal(down.scales, s)
    assert isinstance(m.layers[0].mixer.in_proj.w, Int4Weight)
    assert isinstance(m.layers[3].mixer.qkv.w, Int4Weight)
    x = (torch.randn(3, cfg.hidden_size) * 0.5).to(torch.bfloat16)
    a = ref_model.layers[0].mlp.gate_up(x).float()
    b = m.layers[0].mlp.gate_up(x).float()
    assert float((a - b).norm() / a.norm()) < 0.15


# ---- single-linear checkpoints of the other stored formats ----------------------------------
def _one_linear(tmp_path, tensors, qcfg=None, table=None):
    import json
    from vllm_sly_radiance_b200.quant.loaders import CheckpointWeights
    save_file({k: v.contiguous() for k, v in tensors.items()}, os.path.join(tmp_path, "m.safetensors"))
    if qcfg is not None:
        json.dump({"quantization_config": qcfg}, open(os.path.join(tmp_path, "config.json"), "w"))
    if table is not None:
        torch.save(table, os.path.join(tmp_path, "bcq_tables.pt"))
    return CheckpointWeights(str(tmp_path), tiny_hybrid())


def _bcq_case(N=64, K=256, seed=0):
    g = torch.Generator().manual_seed(seed)
    table = torch.rand(256, 8, generator=g) * 6
    table[:, 0] = 0
    table = table.to(torch.float8_e4m3fn).float()                  # e4m3-exact magnitudes
    packed = torch.randint(0, 256, (N, K // 2), generator=g, dtype=torch.uint8)
    ids = torch.randint(0, 256, (N, K // 32), generator=g, dtype=torch.uint8)
    row_exp = torch.randint(115, 125, (N,), generator=g, dtype=torch.uint8)
    return table, packed, ids, row_exp


def test_mxfp6_checkpoint_loads_as_stored(tmp_path):
    w = torch.randn(64, 256) * 0.05
    p, s = F.mx_quantize(w, "e2m3")
    W = _one_linear(tmp_path, {"x.weight_packed": p, "x.weight_scale": s})
    got = W._linear_any("x")
    assert got.fmt == "e2m3" and torch.equal(got.packed, p) and got.K == 256
    assert torch.equal(got.dequantize(), F.mx_dequantize(p, s, "e2m3"))


def test_mxfp8_checkpoint_loads_as_stored(tmp_path):
    w = torch.randn(32, 128) * 0.05
    p, s = F.mx_quantize(w, "e4m3")
    W = _one_linear(tmp_path, {"x.weight": p.view(torch.float8_e4m3fn), "x.weight_scale": s})
    got = W._linear_any("x")
    assert got.fmt == "e4m3" and torch.equal(got.packed, p)


def test_bcq4_checkpoint_is_exact_in_mxfp8(tmp_path):
    """BCQ4: sign * table[id][mag] * 2^(row_exp - 127) -> MXFP8 with no rounding."""
    from vllm_sly_radiance_b200.quant.loaders import bcq_dequantize
    table, packed, ids, row_exp = _bcq_case()
    W = _one_linear(tmp_path, {"x.weight_packed": packed, "x.weight_scale": ids,
                               "x.weight_row_exp": row_exp}, table=table)
    got = W._linear_any("x")
    want = bcq_dequantize(packed, ids, row_exp, table)
    assert got.fmt == "e4m3"
    assert torch.equal(got.dequantize(), want)
    # independent decode of one element: row 3, column 37 (odd -> high nibble of byte 18)
    nib = int(packed[3, 18]) >> 4
    v = float(table[int(ids[3, 1]), nib & 7]) * 2.0 ** (int(row_exp[3]) - 127)
    assert float(want[3, 37]) == (-v if nib >= 8 else v)


def test_bcq4_hadamard_checkpoint_is_derotated(tmp_path):
    """Hadamard-128 BCQ4 (stored W' = W R): the loaded weight W' R^T serves y = x W^T, the same
    product the reference forms as (x R) W'^T with the rotation applied to activations."""
    from vllm_sly_radiance_b200.quant.loaders import bcq_dequantize, hadamard_rotation
    R = hadamard_rotation(128)
    assert torch.allclose(R @ R.t(), torch.eye(128), atol=1e-5)
    table, packed, ids, row_exp = _bcq_case(seed=1)
    W = _one_linear(tmp_path, {"x.weight_packed": packed, "x.weight_scale": ids,
                               "x.weight_row_exp": row_exp}, qcfg={"hadamard": 128}, table=table)
    got = W._linear_any("x")
    wr = bcq_dequantize(packed, ids, row_exp, table)                  # W' (rotated)
    x = torch.randn(5, 256)
    want = (x.view(5, 2, 128) @ R).view(5, 256) @ wr.t()
    y = x @ got.dequantize().t()
    assert float((y - want).norm() / want.norm()) < 0.03


def test_fp8_block_checkpoint_dequantizes(tmp_path):
    g = torch.Generator().manual_seed(4)
    q = (torch.randn(256, 384, generator=g) * 50).clamp(-448, 448).to(torch.float8_e4m3fn)
    si = torch.rand(2, 3, generator=g) + 0.01
    W = _one_linear(tmp_path, {"x.weight": q, "x.weight_scale_inv": si},
                    qcfg={"weight_block_size": [128, 128]})
    got = W._linear_any("x")
    assert torch.equal(got[130:, 260:], q.float()[130:, 260:] * si[1, 2])
    assert torch.equal(got[:128, :128], q.float()[:128, :128] * si[0, 0])
