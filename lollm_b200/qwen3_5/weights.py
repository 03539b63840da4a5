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


_M64 = (1 << 64) - 1


def _s64(v: int) -> int:
    """An unsigned 64-bit constant as the int64 torch stores (two's complement)."""
    v &= _M64
    return v - (1 << 64) if v >= (1 << 63) else v


def _shr(x: torch.Tensor, s: int) -> torch.Tensor:
    """Logical right shift of int64 lanes (torch's >> is arithmetic)."""
    return (x >> s) & ((1 << (64 - s)) - 1)


def counter_uniform(n: int, offset: int, seed: int, device, std: float = 0.02) -> torch.Tensor:
    """n float32 values uniform in [-a, a) with a = std·√3 (standard deviation `std`), value i
    from the splitmix64 hash of (seed, offset + i). Integer arithmetic only (int64 products
    wrap identically everywhere), so the values are bit-identical on any CPU and on the GPU,
    and any slice can be generated on its own."""
    i = torch.arange(offset, offset + n, dtype=torch.int64, device=device)
    x = i * _s64(0x9E3779B97F4A7C15) + _s64(seed * 0xD1B54A32D192ED03 + 0x632BE59BD9B4E019)
    x = (x ^ _shr(x, 30)) * _s64(0xBF58476D1CE4E5B9)
    x = (x ^ _shr(x, 27)) * _s64(0x94D049BB133111EB)
    x = x ^ _shr(x, 31)
    u = _shr(x, 40).to(torch.float32) * (1.0 / (1 << 24))          # 24 bits: exact in fp32
    a = torch.tensor(std * (3.0 ** 0.5), dtype=torch.float32, device=device)   # one fp32 rounding, same everywhere
    return (u * 2.0 - 1.0) * a


def counter_init(cfg: Qwen3_5Config, seed: int, *, dtype=torch.float32, device="cpu", std: float = 0.02,
                 with_mtp: bool = True, chunk: int = 1 << 26) -> dict:
    """Seeded weights from `counter_uniform` (uniform with standard deviation `std`) as an
    HF-named dict, every tensor the slice of one global counter stream in `param_specs` order.
    Bit-identical on CPU and GPU: fixtures for multi-GB shapes are made on the host by running
    the reference and rebuilt on the GPU in seconds."""
    out, off = {}, 0
    for name, shape in param_specs(cfg, with_mtp):
        n = int(np.prod(shape))
        t = torch.empty(n, dtype=dtype, device=device)
        for c0 in range(0, n, chunk):
            c1 = min(n, c0 + chunk)
            t[c0:c1] = counter_uniform(c1 - c0, off + c0, seed, device, std).to(dtype)
        out[to_raw(name)] = t.view(shape)
        off += n
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


# ─────────────────────────────────────── streaming load ───────────────────────────────────────

class StreamingParams:
    """{canonical name: tensor} that produces each tensor only when the model asks for it and
    keeps no reference afterwards, so building a model holds at most one source tensor beyond
    the model itself — the reference's meta-build-then-stream load (src/qwen3_5/weights.py:
    40-70, mtp.py:171-189), for sources that do not fit twice in memory (the 48-layer MoE shape
    is ~160 GB of bf16).

    `fetch(raw_name) -> tensor` supplies the HF-named tensor. Every tensor is shape-checked
    against `param_specs` when produced (RuntimeError on a mismatch or a missing name), then
    cast to `dtype` and moved to `device`. `tied` says whether lm_head shares the embedding
    (the model then reuses the embedding and never asks for lm_head).
    """

    def __init__(self, cfg: Qwen3_5Config, fetch, *, tied: bool, device=None, dtype=None,
                 with_mtp: bool = True):
        self.cfg, self._fetch, self.tied = cfg, fetch, bool(tied)
        self.device, self.dtype = device, dtype
        self._shapes = dict(param_specs(cfg, with_mtp))
        if not self.tied:
            self._shapes["lm_head.weight"] = (cfg.vocab_size, cfg.hidden_size)

    def __contains__(self, name):
        return name in self._shapes

    def keys(self):
        return self._shapes.keys()

    def __getitem__(self, name: str) -> torch.Tensor:
        if name == "lm_head.weight" and self.tied:
            raise RuntimeError("qwen3_5: lm_head is tied to the embedding; use the embedding tensor")
        if name not in self._shapes:
            raise RuntimeError(f"qwen3_5: no parameter named {name}")
        t = self._fetch(to_raw(name))
        if t is None:
            raise RuntimeError(f"qwen3_5: missing tensor for {name} (raw {to_raw(name)})")
        if tuple(t.shape) != tuple(self._shapes[name]):
            raise RuntimeError(f"qwen3_5: shape mismatch {name}: {tuple(t.shape)} vs {self._shapes[name]}")
        if self.dtype is not None or self.device is not None:
            t = t.to(device=self.device if self.device is not None else t.device,
                      dtype=self.dtype if self.dtype is not None else t.dtype)
        return t

    # ---------------------------------------------------------------- sources
    @classmethod
    def from_dict(cls, cfg, weights: dict, *, consume: bool = True, **kw):
        """An HF-named dict; with `consume` each tensor is popped as the model takes it (the
        caller's dict shrinks as the model grows, as the reference's load does)."""
        tied = cfg.tie_word_embeddings or "lm_head.weight" not in weights
        fetch = (lambda raw: weights.pop(raw, None)) if consume else (lambda raw: weights.get(raw))
        return cls(cfg, fetch, tied=tied, **kw)

    @classmethod
    def from_safetensors(cls, cfg, path: str, **kw):
        """A safetensors checkpoint: one file, or a directory holding `model.safetensors` or a
        sharded `model.safetensors.index.json`. Tensors are read one at a time."""
        import json
        import os
        from safetensors import safe_open
        if os.path.isdir(path):
            idx = os.path.join(path, "model.safetensors.index.json")
            if os.path.exists(idx):
                wmap = json.load(open(idx))["weight_map"]
                files = {raw: os.path.join(path, f) for raw, f in wmap.items()}
            else:
                path = os.path.join(path, "model.safetensors")
                files = None
        else:
            files = None
        if files is None:
            with safe_open(path, framework="pt", device="cpu") as f:
                files = {raw: path for raw in f.keys()}
        handles = {}

        def fetch(raw):
            fn = files.get(raw)
            if fn is None:
                return None
            if fn not in handles:
                handles[fn] = safe_open(fn, framework="pt", device="cpu")
            return handles[fn].get_tensor(raw)

        tied = cfg.tie_word_embeddings or "lm_head.weight" not in files
        return cls(cfg, fetch, tied=tied, **kw)

    @classmethod
    def random(cls, cfg, seed: int, *, device, dtype=torch.bfloat16, std: float = 0.02, **kw):
        """Seeded N(0, std) tensors generated on `device` when asked for: each name has its own
        generator seeded from (seed, the name's position in `param_specs`), so a tensor's values
        do not depend on the order the model asks for them."""
        order = {to_raw(n): i for i, (n, _) in enumerate(param_specs(cfg, True))}
        shapes = {to_raw(n): s for n, s in param_specs(cfg, True)}

        def fetch(raw):
            if raw not in shapes:
                return None
            g = torch.Generator(device=device)
            g.manual_seed(seed * 1_000_003 + order[raw])
            t = torch.empty(shapes[raw], device=device, dtype=dtype)
            return t.normal_(0.0, std, generator=g)

        return cls(cfg, fetch, tied=cfg.tie_word_embeddings, device=device, dtype=dtype, **kw)
