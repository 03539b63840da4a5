"""Weight names, seeded random init, and the load seam (checkpoint dict -> device layout).

Name map: the HF checkpoint keeps the text stack under `model.language_model.*`, `mtp.*` at
top level and `lm_head.weight` only when untied — the same seam as the reference's
`to_raw` (`src/qwen3_5/weights.py:27-37`) and `_mtp_raw` (`src/qwen3_5/mtp.py:165-168`).

`param_specs` lists every parameter in the order the reference modules register them
(`named_parameters()` of `Qwen3_5Model`, `src/qwen3_5/modeling_qwen3_5.py:64-73`, then of
`MTP`, `src/qwen3_5/mtp.py:44-54`), so a seeded stream of normals assigns the same value
to the same tensor whichever side builds the dict.

`random_init` is the benchmark/test weight source (no checkpoints offline): every tensor
~ N(0, 0.02). Two generators:
  * "numpy": PCG64 float32 standard normals — bit-identical on every host, used for the
    parity fixtures (the golden script and the GPU tests rebuild the same weights);
  * "torch": a seeded torch generator on the target device — fast for the 2B shape.

`load_checkpoint` is the strict, shape-checked load (`src/qwen3_5/weights.py:40-70`,
`src/qwen3_5/mtp.py:171-189`): a missing tensor or a shape mismatch raises RuntimeError.
"""

from __future__ import annotations

import numpy as np
import torch

from .config import Qwen3_5Config


def to_raw(canonical: str) -> str:
    if canonical.startswith("model."):
        return "model.language_model." + canonical[len("model."):]
    return canonical


def _attn_specs(cfg: Qwen3_5Config, pre: str):
    h, hd = cfg.hidden_size, cfg.head_dim
    return [
        (pre + "self_attn.q_proj.weight", (cfg.num_attention_heads * hd * 2, h)),
        (pre + "self_attn.k_proj.weight", (cfg.num_key_value_heads * hd, h)),
        (pre + "self_attn.v_proj.weight", (cfg.num_key_value_heads * hd, h)),
        (pre + "self_attn.o_proj.weight", (h, cfg.num_attention_heads * hd)),
        (pre + "self_attn.q_norm.weight", (hd,)),
        (pre + "self_attn.k_norm.weight", (hd,)),
    ]


def _gdn_specs(cfg: Qwen3_5Config, pre: str):
    h, nv = cfg.hidden_size, cfg.linear_num_value_heads
    p = pre + "linear_attn."
    return [
        # module-level parameters register before the child modules' parameters
        (p + "dt_bias", (nv,)),
        (p + "A_log", (nv,)),
        (p + "in_proj_qkv.weight", (cfg.conv_dim, h)),
        (p + "in_proj_z.weight", (cfg.value_dim, h)),
        (p + "in_proj_b.weight", (nv, h)),
        (p + "in_proj_a.weight", (nv, h)),
        (p + "conv1d.weight", (cfg.conv_dim, 1, cfg.linear_conv_kernel_dim)),
        (p + "norm.weight", (cfg.linear_value_head_dim,)),
        (p + "out_proj.weight", (h, cfg.value_dim)),
    ]


def _ffn_specs(cfg: Qwen3_5Config, pre: str, moe: bool):
    h = cfg.hidden_size
    if not moe:
        i = cfg.intermediate_size
        return [(pre + "mlp.gate_proj.weight", (i, h)),
                (pre + "mlp.up_proj.weight", (i, h)),
                (pre + "mlp.down_proj.weight", (h, i))]
    e, im, ish = cfg.num_experts, cfg.moe_intermediate_size, cfg.shared_expert_intermediate_size
    specs = [(pre + "mlp.gate.weight", (e, h)),
             (pre + "mlp.experts.gate_up_proj", (e, 2 * im, h)),
             (pre + "mlp.experts.down_proj", (e, h, im))]
    if ish > 0:
        specs += [(pre + "mlp.shared_expert.gate_proj.weight", (ish, h)),
                  (pre + "mlp.shared_expert.up_proj.weight", (ish, h)),
                  (pre + "mlp.shared_expert.down_proj.weight", (h, ish)),
                  (pre + "mlp.shared_expert_gate.weight", (1, h))]
    return specs


def _layer_specs(cfg: Qwen3_5Config, pre: str, layer_type: str, moe: bool):
    h = cfg.hidden_size
    mixer = _attn_specs(cfg, pre) if layer_type == "full_attention" else _gdn_specs(cfg, pre)
    return ([(pre + "input_layernorm.weight", (h,))] + mixer
            + [(pre + "post_attention_layernorm.weight", (h,))] + _ffn_specs(cfg, pre, moe))


def param_specs(cfg: Qwen3_5Config, with_mtp: bool = True):
    """[(canonical_name, shape)] in reference registration order (tied lm_head omitted)."""
    h = cfg.hidden_size
    specs = [("model.embed_tokens.weight", (cfg.vocab_size, h))]
    for i in range(cfg.num_hidden_layers):
        specs += _layer_specs(cfg, f"model.layers.{i}.", cfg.layer_type(i), cfg.is_moe_layer(i))
    specs.append(("model.norm.weight", (h,)))
    if not cfg.tie_word_embeddings:
        specs.append(("lm_head.weight", (cfg.vocab_size, h)))
    if with_mtp:
        specs += [("mtp.pre_fc_norm_embedding.weight", (h,)),
                  ("mtp.pre_fc_norm_hidden.weight", (h,)),
                  ("mtp.fc.weight", (h, 2 * h))]
        specs += _layer_specs(cfg, "mtp.layers.0.", "full_attention", cfg.is_moe_layer(0))
        specs.append(("mtp.norm.weight", (h,)))
    return specs


def random_init(cfg: Qwen3_5Config, seed: int, *, dtype=torch.float32, device="cpu",
                std: float = 0.02, with_mtp: bool = True, generator: str = "numpy") -> dict:
    """Seeded N(0, std) weights as an HF-named dict {raw_name: tensor}."""
    out = {}
    if generator == "numpy":
        rng = np.random.Generator(np.random.PCG64(seed))
        for name, shape in param_specs(cfg, with_mtp):
            a = rng.standard_normal(int(np.prod(shape)), dtype=np.float32) * np.float32(std)
            out[to_raw(name)] = torch.from_numpy(a.reshape(shape)).to(device=device, dtype=dtype)
    elif generator == "torch":
        g = torch.Generator(device=device)
        g.manual_seed(seed)
        for name, shape in param_specs(cfg, with_mtp):
            t = torch.empty(shape, device=device, dtype=dtype)
            t.normal_(0.0, std, generator=g)
            out[to_raw(name)] = t
    else:
        raise ValueError(f"unknown generator {generator!r}")
    return out


def load_checkpoint(cfg: Qwen3_5Config, weights: dict, *, with_mtp: bool = True,
                    device="cpu", dtype=None) -> dict:
    """Strict shape-checked load: {canonical_name: tensor on device}, lm_head re-tied."""
    params = {}
    for name, shape in param_specs(cfg, with_mtp):
        raw = to_raw(name)
        if raw not in weights:
            raise RuntimeError(f"qwen3_5: missing tensor for {name} (raw {raw})")
        t = weights[raw]
        if tuple(t.shape) != tuple(shape):
            raise RuntimeError(f"qwen3_5: shape mismatch {name}: {tuple(t.shape)} vs {shape}")
        if dtype is not None:
            t = t.to(dtype)
        params[name] = t.to(device)
    if cfg.tie_word_embeddings or "lm_head.weight" not in params:
        params["lm_head.weight"] = params["model.embed_tokens.weight"]
    return params
