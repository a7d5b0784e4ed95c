"""Model and engine configuration.

The model family is the gated-delta-net (GDN) hybrid decoder served by the reference
(Qwen3-Next / Qwen3.8 layout: 3 GDN layers then 1 full-attention layer, Gemma-style ``(1+w)``
RMSNorm, sigmoid-gated attention output, SwiGLU MLP).  Reference model facts:
``radiance_tp3pad.py:12-27`` (head counts), ``docs/PREFILL-4000.md:25-31`` (shapes),
``sly/mxfp4/radiance_fused_norm.py:6-12`` (Gemma norm).

Presets:
  * ``tiny_hybrid``   - 4-layer CPU oracle model (3 GDN + 1 GQA), hidden 256.
  * ``qwen38_27b``    - the 64-layer hybrid benchmarked at TP 1/2/4/8.
  * ``moe_hybrid``    - 40-layer hybrid with 256 routed experts (top-8) + 1 shared expert.
  * ``dflash2_drafter`` - the 5-layer block drafter used for speculative decoding.
"""
from __future__ import annotations

import dataclasses
import json
import os
from dataclasses import dataclass, field
from typing import Optional


@dataclass
class ModelConfig:
    name: str = "tiny_hybrid"
    vocab_size: int = 4096
    hidden_size: int = 256
    intermediate_size: int = 768
    num_layers: int = 4
    # full attention every `full_attn_interval` layers (layer i is attention iff (i+1) % interval == 0)
    full_attn_interval: int = 4
    # full attention
    num_q_heads: int = 4
    num_kv_heads: int = 2
    head_dim: int = 64
    rope_theta: float = 1.0e6
    partial_rotary_factor: float = 0.25
    attn_output_gate: bool = True
    # gated delta net
    gdn_num_k_heads: int = 4
    gdn_num_v_heads: int = 4
    gdn_head_k_dim: int = 64
    gdn_head_v_dim: int = 64
    gdn_conv_kernel: int = 4
    # MoE (0 experts = dense MLP)
    num_experts: int = 0
    num_experts_per_tok: int = 0
    moe_intermediate_size: int = 0
    shared_expert_intermediate_size: int = 0
    # misc
    rms_norm_eps: float = 1e-6
    max_position_embeddings: int = 262144
    init_std: float = 0.02
    tie_word_embeddings: bool = False
    # vocabulary rows beyond this are tensor-parallel padding (0 = no padding)
    real_vocab_size: int = 0

    # ---- derived -------------------------------------------------------------------------
    def is_attention_layer(self, i: int) -> bool:
        return (i + 1) % self.full_attn_interval == 0

    @property
    def attention_layers(self) -> list[int]:
        return [i for i in range(self.num_layers) if self.is_attention_layer(i)]

    @property
    def gdn_layers(self) -> list[int]:
        return [i for i in range(self.num_layers) if not self.is_attention_layer(i)]

    @property
    def rotary_dim(self) -> int:
        return int(self.head_dim * self.partial_rotary_factor)

    @property
    def gdn_key_dim(self) -> int:
        return self.gdn_num_k_heads * self.gdn_head_k_dim

    @property
    def gdn_value_dim(self) -> int:
        return self.gdn_num_v_heads * self.gdn_head_v_dim

    @property
    def gdn_conv_dim(self) -> int:
        return 2 * self.gdn_key_dim + self.gdn_value_dim

    @property
    def gdn_in_proj_dim(self) -> int:
        # merged in_proj: [q | k | v | z | b | a]  (the reference merges qkvz and ba after load,
        # radiance_gdnmerge.py:30-35; here it is one linear from the start)
        return 2 * self.gdn_key_dim + 2 * self.gdn_value_dim + 2 * self.gdn_num_v_heads

    @property
    def qkv_proj_dim(self) -> int:
        # [q+gate interleaved per head (2*hd each) | k | v]
        qd = self.num_q_heads * self.head_dim * (2 if self.attn_output_gate else 1)
        return qd + 2 * self.num_kv_heads * self.head_dim

    @property
    def logical_vocab_size(self) -> int:
        return self.real_vocab_size or self.vocab_size

    @property
    def is_moe(self) -> bool:
        return self.num_experts > 0

    def to_json(self) -> str:
        return json.dumps(dataclasses.asdict(self))

    @staticmethod
    def from_dict(d: dict) -> "ModelConfig":
        names = {f.name for f in dataclasses.fields(ModelConfig)}
        return ModelConfig(**{k: v for k, v in d.items() if k in names})

    def num_params(self) -> int:
        h = self.hidden_size
        n = self.vocab_size * h * (1 if self.tie_word_embeddings else 2)
        for i in range(self.num_layers):
            if self.is_attention_layer(i):
                n += h * self.qkv_proj_dim + self.num_q_heads * self.head_dim * h
            else:
                n += h * self.gdn_in_proj_dim + self.gdn_value_dim * h
                n += self.gdn_conv_dim * self.gdn_conv_kernel
            if self.is_moe:
                n += self.num_experts * 3 * h * self.moe_intermediate_size
                n += 3 * h * self.shared_expert_intermediate_size + h * self.num_experts
            else:
                n += 3 * h * self.intermediate_size
        return n


def tiny_hybrid() -> ModelConfig:
    """CPU oracle model: 4 layers (0-2 GDN 4 heads dk=dv=64, conv 4; 3 = GQA 4q/2kv hd 64)."""
    return ModelConfig(name="tiny_hybrid")


def qwen38_27b(intermediate_size: int = 8704) -> ModelConfig:
    """Qwen3.8-27B-shaped hybrid (64 layers, 3:1 GDN:attention, hidden 5120).

    The benchmark config sets the SwiGLU intermediate to 8704 (fused gate_up N=17408);
    the production checkpoint uses 17408 (fused 34816); both are supported."""
    return ModelConfig(
        name="qwen38_27b" if intermediate_size == 8704 else f"qwen38_27b_i{intermediate_size}",
        vocab_size=248320, hidden_size=5120, intermediate_size=intermediate_size,
        num_layers=64, full_attn_interval=4,
        num_q_heads=24, num_kv_heads=4, head_dim=256, rope_theta=1.0e7,
        partial_rotary_factor=0.25,
        gdn_num_k_heads=16, gdn_num_v_heads=48, gdn_head_k_dim=128, gdn_head_v_dim=128,
        gdn_conv_kernel=4)


def moe_hybrid() -> ModelConfig:
    """MoE hybrid: 40 layers 3:1, hidden 2048, attn 16q/2kv hd 256, 256 experts top-8 + 1 shared."""
    return ModelConfig(
        name="moe_hybrid", vocab_size=248320, hidden_size=2048, intermediate_size=0,
        num_layers=40, full_attn_interval=4, num_q_heads=16, num_kv_heads=2, head_dim=256,
        rope_theta=1.0e7, gdn_num_k_heads=16, gdn_num_v_heads=32, gdn_head_k_dim=128,
        gdn_head_v_dim=128, num_experts=256, num_experts_per_tok=8, moe_intermediate_size=512,
        shared_expert_intermediate_size=512)


def tiny_moe() -> ModelConfig:
    """Small MoE hybrid for CPU tests of routing / expert parallel logic."""
    return ModelConfig(
        name="tiny_moe", vocab_size=4096, hidden_size=256, intermediate_size=0, num_layers=4,
        num_q_heads=4, num_kv_heads=2, head_dim=64, gdn_num_k_heads=4, gdn_num_v_heads=4,
        gdn_head_k_dim=64, gdn_head_v_dim=64, num_experts=16, num_experts_per_tok=4,
        moe_intermediate_size=128, shared_expert_intermediate_size=128)


@dataclass
class DrafterConfig:
    """DFlash2 block drafter (``dflash2/qwen3_dflash2.py:26-307``): non-causal sliding-window
    attention layers wrapped by grouped depthwise convolutions, conditioned on target hidden
    states from ``num_aux_layers`` evenly spaced target layers, drafting ``block_size-1`` tokens."""
    num_layers: int = 5
    hidden_size: int = 5120
    num_q_heads: int = 32
    num_kv_heads: int = 8
    head_dim: int = 128
    intermediate_size: int = 17408
    block_size: int = 8            # 1 + k, k = 7
    window: int = 2048
    num_aux_layers: int = 5
    conv_taps: int = 4
    conv_group_size: int = 128
    selector_rank: int = 64
    top_k_candidates: int = 8
    rope_theta: float = 1.0e7
    rms_norm_eps: float = 1e-6

    @staticmethod
    def tiny() -> "DrafterConfig":
        return DrafterConfig(num_layers=2, hidden_size=256, num_q_heads=4, num_kv_heads=2,
                             head_dim=64, intermediate_size=512, window=64, num_aux_layers=2,
                             conv_group_size=64, selector_rank=16, top_k_candidates=4)


PRESETS = {
    "tiny_hybrid": tiny_hybrid,
    "qwen38_27b": qwen38_27b,
    "qwen38_27b_i17408": lambda: qwen38_27b(17408),
    "moe_hybrid": moe_hybrid,
    "tiny_moe": tiny_moe,
}


def get_model_config(name_or_path: str) -> ModelConfig:
    """Preset name, or a directory / json file with a config."""
    if name_or_path in PRESETS:
        return PRESETS[name_or_path]()
    p = name_or_path
    if os.path.isdir(p):
        p = os.path.join(p, "config.json")
    if os.path.isfile(p):
        with open(p) as f:
            d = json.load(f)
        return config_from_hf(d) if "model_type" in d else ModelConfig.from_dict(d)
    raise ValueError(f"unknown model {name_or_path!r}; presets: {sorted(PRESETS)}")


def config_from_hf(d: dict) -> ModelConfig:
    """Map a Qwen3-Next style HF config.json onto ModelConfig."""
    tc = d.get("text_config", d)
    interval = tc.get("full_attention_interval", 4)
    return ModelConfig(
        name=tc.get("model_type", "hf"),
        vocab_size=tc["vocab_size"], hidden_size=tc["hidden_size"],
        intermediate_size=tc.get("intermediate_size", 0), num_layers=tc["num_hidden_layers"],
        full_attn_interval=interval, num_q_heads=tc["num_attention_heads"],
        num_kv_heads=tc["num_key_value_heads"], head_dim=tc.get("head_dim", 256),
        rope_theta=tc.get("rope_theta", 1e7),
        partial_rotary_factor=tc.get("partial_rotary_factor", 0.25),
        gdn_num_k_heads=tc.get("linear_num_key_heads", 16),
        gdn_num_v_heads=tc.get("linear_num_value_heads", 32),
        gdn_head_k_dim=tc.get("linear_key_head_dim", 128),
        gdn_head_v_dim=tc.get("linear_value_head_dim", 128),
        gdn_conv_kernel=tc.get("linear_conv_kernel_dim", 4),
        num_experts=tc.get("num_experts", 0), num_experts_per_tok=tc.get("num_experts_per_tok", 0),
        moe_intermediate_size=tc.get("moe_intermediate_size", 0),
        shared_expert_intermediate_size=tc.get("shared_expert_intermediate_size", 0),
        rms_norm_eps=tc.get("rms_norm_eps", 1e-6),
        tie_word_embeddings=tc.get("tie_word_embeddings", False))


def _env(name: str, default, typ=str):
    v = os.environ.get(name)
    if v is None or v == "":
        return default
    if typ is bool:
        return v.lower() in ("1", "true", "yes", "on")
    return typ(v)


@dataclass
class EngineConfig:
    """Serving engine configuration (CLI flags, each overridable by a RADIANCE_* env var).

    Defaults mirror the reference's production launch (``README.md:236-270``):
    ``--max-num-seqs 8 --max-num-batched-tokens 4096`` chunked prefill, fp8 KV cache,
    FULL decode CUDA graphs for batch sizes up to 64."""
    model: str = "tiny_hybrid"
    tensor_parallel_size: int = 1
    expert_parallel: bool = False
    dtype: str = "bfloat16"
    quantization: str = "mxfp4"         # mxfp4 (W4A8) | mxfp6 (W6A8) | mxfp8 (W8A8) | bf16 |
    #                                     nvfp4 (requantized to mxfp4) | int4
    kv_cache_dtype: str = "fp8"         # fp8 | int4 (4-bit per-16 scale/zero) | bf16
    lm_head_quant: Optional[str] = None  # None (the model's) | int4 (W4A16 g128) | bf16 | mxfp4
    embed_quant: Optional[str] = None    # None (bf16) | int8 (per-row scale) | int4 (g128 scales)
    ssm_state_dtype: str = "float32"    # float32 | bfloat16
    block_size: int = 64                # KV page size in tokens
    max_model_len: int = 65536
    max_num_seqs: int = 8
    max_num_batched_tokens: int = 4096
    gpu_memory_utilization: float = 0.90
    num_kv_blocks: Optional[int] = None
    enable_cuda_graphs: bool = True
    cuda_graph_max_bs: int = 64
    capture_graphs_at_start: bool = True   # capture every decode bucket at engine start
    enable_prefix_caching: bool = False
    prefix_snapshot_slots: int = 16  # GDN state snapshots kept for cached prefixes
    prefix_snapshot_interval: int = 0  # also snapshot every N prompt tokens (0: last boundary only)
    # offload tiers under the GPU prefix cache (evicted KV blocks and GDN snapshots)
    kv_offload_gb: float = 0.0          # pinned host RAM tier (0 = off)
    kv_offload_disk_dir: Optional[str] = None
    kv_offload_disk_gb: float = 0.0     # disk tier below the RAM tier
    kv_offload_policy: str = "lru"      # lru | arc
    kv_offload_state_fraction: float = 0.5   # share of each tier for GDN state snapshots
    seed: int = 0
    # speculative decoding
    speculative_method: Optional[str] = None   # None | "dflash2" | "mtp" | "lookup" | "forced"
    num_speculative_tokens: int = 7
    adaptive_width: bool = False     # per-request verify width from acceptance + step-cost model
    acceptance_rule: str = "leviathan"          # leviathan | cactus | nsd
    forced_acceptance: Optional[str] = None     # benchmarking: "uniform07" forced schedule
    # comm
    comm_backend: str = "fused"                 # fused (own NVLink kernels) | nccl (baseline)
    gemm_backend: str = "native"                # native (own tcgen05) | cublas (baseline fp8)
    device: str = "cuda"

    def __post_init__(self):
        for f in dataclasses.fields(self):
            env = "RADIANCE_" + f.name.upper()
            if env in os.environ:
                cur = getattr(self, f.name)
                typ = type(cur) if cur is not None else str
                if typ is bool:
                    setattr(self, f.name, _env(env, cur, bool))
                else:
                    setattr(self, f.name, _env(env, cur, typ))
        if self.max_num_batched_tokens < self.max_num_seqs:
            raise ValueError("max_num_batched_tokens must be >= max_num_seqs")
        if self.kv_cache_dtype not in ("fp8", "int4", "bf16"):
            raise ValueError(f"kv_cache_dtype {self.kv_cache_dtype!r} not supported")
        if self.acceptance_rule not in ("leviathan", "cactus", "nsd"):
            raise ValueError(f"acceptance_rule {self.acceptance_rule!r} not supported")
        if self.kv_cache_dtype == "int4":
            # 4-bit KV pages hold 16 tokens (per-16-element fp16 scale/zero per head)
            self.block_size = 16

    def model_config(self) -> ModelConfig:
        return get_model_config(self.model)
