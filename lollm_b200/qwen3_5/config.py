"""Qwen3.5 text-stack configuration (the shape source for every kernel launch).

Mirrors the reference family's config object (`src/qwen3_5/config.py:15-101`): the same
field names, the same derived dimensions (`n_rep`, `rotary_dim`, `key_dim`, `value_dim`,
`conv_dim`, `v_per_k`), and `from_hf` reading the `text_config` sub-dict of an HF
`config.json`. Non-HF formats hard-fail exactly like `build_config`
(`src/qwen3_5/config.py:104-109`).

The module also carries the named benchmark shapes as HF-style raw dicts:
`TINY` (the CPU-parity config), `QWEN35_2B` (the 2B verify-step config) and `MICRO`
(a few-MB shape for golden fixtures and GPU parity tests).
"""

from __future__ import annotations

from dataclasses import dataclass, field


@dataclass
class Qwen3_5Config:
    vocab_size: int
    hidden_size: int
    intermediate_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    rms_norm_eps: float
    rope_theta: float
    partial_rotary_factor: float
    tie_word_embeddings: bool
    hidden_act: str
    layer_types: list
    full_attention_interval: int
    attn_output_gate: bool
    output_gate_type: str
    linear_num_key_heads: int
    linear_num_value_heads: int
    linear_key_head_dim: int
    linear_value_head_dim: int
    linear_conv_kernel_dim: int
    # sparse-MoE FFN fields (qwen3_5_moe shape); num_experts == 0 means a dense SwiGLU MLP
    num_experts: int = 0
    num_experts_per_tok: int = 0
    moe_intermediate_size: int = 0
    shared_expert_intermediate_size: int = 0
    norm_topk_prob: bool = True
    decoder_sparse_step: int = 1
    mlp_only_layers: list = field(default_factory=list)
    extra: dict = field(default_factory=dict)

    # derived dimensions (same definitions as src/qwen3_5/config.py:43-68)
    @property
    def n_rep(self) -> int:
        return self.num_attention_heads // self.num_key_value_heads

    @property
    def rotary_dim(self) -> int:
        return int(self.head_dim * self.partial_rotary_factor)

    @property
    def key_dim(self) -> int:
        return self.linear_key_head_dim * self.linear_num_key_heads

    @property
    def value_dim(self) -> int:
        return self.linear_value_head_dim * self.linear_num_value_heads

    @property
    def conv_dim(self) -> int:
        return 2 * self.key_dim + self.value_dim

    @property
    def v_per_k(self) -> int:
        return self.linear_num_value_heads // self.linear_num_key_heads

    def layer_type(self, i: int) -> str:
        return self.layer_types[i]

    @property
    def attn_layers(self) -> list:
        return [i for i, t in enumerate(self.layer_types) if t == "full_attention"]

    @property
    def gdn_layers(self) -> list:
        return [i for i, t in enumerate(self.layer_types) if t != "full_attention"]

    @property
    def is_moe(self) -> bool:
        return self.num_experts > 0

    def is_moe_layer(self, i: int) -> bool:
        """Sparse FFN on layer i unless it is forced dense — the HF rule of
        `Qwen3_5MoeConfig.is_moe_layer` (src/qwen3_5_moe/config.py:80-86). The MTP head's
        single block asks for layer 0 (src/qwen3_5_moe/mtp.py:34-36)."""
        if i in self.mlp_only_layers or self.num_experts <= 0:
            return False
        return (i + 1) % self.decoder_sparse_step == 0

    @classmethod
    def from_hf(cls, raw: dict) -> "Qwen3_5Config":
        t = raw.get("text_config", raw)
        hidden = t["hidden_size"]
        n_head = t["num_attention_heads"]
        rp = t.get("rope_parameters", {}) or {}
        n_experts = t.get("num_experts", t.get("n_routed_experts", 0))
        moe_inter = t.get("moe_intermediate_size", t.get("intermediate_size", 0))
        top_k = t.get("num_experts_per_tok", t.get("num_experts_per_token"))
        if n_experts > 0 and top_k is None:
            # the reference refuses to default the router width (src/qwen3_5_moe/config.py:100-113)
            raise KeyError("qwen3_5_moe config has no 'num_experts_per_tok' (router top-k width)")
        return cls(
            vocab_size=t["vocab_size"],
            hidden_size=hidden,
            intermediate_size=t.get("intermediate_size", moe_inter),
            num_hidden_layers=t["num_hidden_layers"],
            num_attention_heads=n_head,
            num_key_value_heads=t.get("num_key_value_heads", n_head),
            head_dim=t.get("head_dim", hidden // n_head),
            rms_norm_eps=t.get("rms_norm_eps", 1e-6),
            rope_theta=rp.get("rope_theta", t.get("rope_theta", 1e7)),
            partial_rotary_factor=rp.get("partial_rotary_factor",
                                         t.get("partial_rotary_factor", 1.0)),
            tie_word_embeddings=t.get("tie_word_embeddings",
                                      raw.get("tie_word_embeddings", False)),
            hidden_act=t.get("hidden_act", "silu"),
            layer_types=list(t["layer_types"]),
            full_attention_interval=t.get("full_attention_interval", 4),
            attn_output_gate=t.get("attn_output_gate", True),
            output_gate_type=t.get("output_gate_type", "sigmoid"),
            linear_num_key_heads=t["linear_num_key_heads"],
            linear_num_value_heads=t["linear_num_value_heads"],
            linear_key_head_dim=t["linear_key_head_dim"],
            linear_value_head_dim=t["linear_value_head_dim"],
            linear_conv_kernel_dim=t["linear_conv_kernel_dim"],
            num_experts=n_experts,
            num_experts_per_tok=top_k or 0,
            moe_intermediate_size=moe_inter if n_experts > 0 else 0,
            shared_expert_intermediate_size=t.get("shared_expert_intermediate_size", 0),
            norm_topk_prob=t.get("norm_topk_prob", True),
            decoder_sparse_step=t.get("decoder_sparse_step", 1),
            mlp_only_layers=list(t.get("mlp_only_layers", [])),
        )


def build_config(raw: dict, fmt: str) -> Qwen3_5Config:
    """Same contract as the reference's `build_config`: only HF safetensors configs."""
    if fmt != "hf":
        raise NotImplementedError(
            "qwen3_5: only safetensors (hf) supported; GGUF for Gated DeltaNet "
            "is not standardized")
    return Qwen3_5Config.from_hf(raw)


def _schedule(n_layers: int, interval: int = 4) -> list:
    return ["full_attention" if i % interval == interval - 1 else "linear_attention"
            for i in range(n_layers)]


def _raw(model_type="qwen3_5", **kw) -> dict:
    base = dict(rms_norm_eps=1e-6, rope_theta=1e7, partial_rotary_factor=0.25,
                tie_word_embeddings=True, hidden_act="silu", full_attention_interval=4,
                attn_output_gate=True, linear_conv_kernel_dim=4)
    base.update(kw)
    base["layer_types"] = _schedule(base["num_hidden_layers"])
    return {"model_type": model_type, "text_config": base}


# tiny, fp32 CPU-parity shape.
TINY = _raw(vocab_size=32768, hidden_size=512, intermediate_size=1536, num_hidden_layers=8,
            num_attention_heads=8, num_key_value_heads=2, head_dim=64,
            linear_num_key_heads=4, linear_num_value_heads=8, linear_key_head_dim=64,
            linear_value_head_dim=64)

# the 2B verify-step shape (bf16).
QWEN35_2B = _raw(vocab_size=151936, hidden_size=2048, intermediate_size=6144,
                 num_hidden_layers=24, num_attention_heads=16, num_key_value_heads=2,
                 head_dim=256, linear_num_key_heads=16, linear_num_value_heads=32,
                 linear_key_head_dim=128, linear_value_head_dim=128)

# A few-MB shape with every structural feature (GQA, v_per_k=2, partial RoPE, 2 attention
# layers) for golden fixtures and fast GPU parity tests.
MICRO = _raw(vocab_size=512, hidden_size=128, intermediate_size=256, num_hidden_layers=8,
             num_attention_heads=4, num_key_value_heads=2, head_dim=32,
             linear_num_key_heads=2, linear_num_value_heads=4, linear_key_head_dim=32,
             linear_value_head_dim=32)

# The same MICRO stack with a kernel-friendly 2B-like head geometry (hd 256 / dk 128),
# used to exercise the production tile shapes at a small hidden size.
MICRO_WIDE = _raw(vocab_size=1024, hidden_size=256, intermediate_size=512,
                  num_hidden_layers=4, num_attention_heads=4, num_key_value_heads=2,
                  head_dim=256, linear_num_key_heads=2, linear_num_value_heads=4,
                  linear_key_head_dim=128, linear_value_head_dim=128)

# the qwen3_5_moe shape (bf16): 48 layers, every FFN a sparse MoE block
# with 512 routed experts (top-10, width 512) plus one always-on shared expert of width 512.
QWEN35_MOE = _raw(model_type="qwen3_5_moe", vocab_size=151936, hidden_size=2048,
                  intermediate_size=512, num_hidden_layers=48, num_attention_heads=16,
                  num_key_value_heads=2, head_dim=256, linear_num_key_heads=16,
                  linear_num_value_heads=32, linear_key_head_dim=128, linear_value_head_dim=128,
                  num_experts=512, num_experts_per_tok=10, moe_intermediate_size=512,
                  shared_expert_intermediate_size=512, norm_topk_prob=True)

# MICRO with a sparse FFN: 8 experts (top-2, width 64) + a shared expert; layer 1 is forced
# dense through `mlp_only_layers` so both FFN kinds and the sparse stride rule are exercised.
MICRO_MOE = _raw(model_type="qwen3_5_moe", vocab_size=512, hidden_size=128,
                 intermediate_size=256, num_hidden_layers=8, num_attention_heads=4,
                 num_key_value_heads=2, head_dim=32, linear_num_key_heads=2,
                 linear_num_value_heads=4, linear_key_head_dim=32, linear_value_head_dim=32,
                 num_experts=8, num_experts_per_tok=2, moe_intermediate_size=64,
                 shared_expert_intermediate_size=64, norm_topk_prob=True, mlp_only_layers=[1])
