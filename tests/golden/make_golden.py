"""Generate the golden fixtures under tests/golden/ by running the REFERENCE implementation.

Run in a container where the reference checkout is importable:

    python tests/golden/make_golden.py --reference <path-to-lollm>/src

It imports the reference's own modules (`qwen3_5.blocks`, `qwen3_5.weights.load`,
`qwen3_5.mtp`, `generate`, `attention`), feeds them seeded inputs and the seeded weights of
`lollm_b200.qwen3_5.weights.random_init` (numpy PCG64: bit-identical on every host), and
stores inputs + outputs as safetensors. Nothing at test time reads the reference: the GPU
box only sees these files. Re-running the script reproduces them bit-for-bit.
"""

from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np
import torch
from safetensors.torch import save_file

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from lollm_b200.qwen3_5.config import MICRO, TINY, Qwen3_5Config  # noqa: E402
from lollm_b200.qwen3_5.weights import random_init  # noqa: E402

WEIGHT_SEED = 1234


def rng(seed):
    return np.random.Generator(np.random.PCG64(seed))


def randn(g, *shape, scale=1.0):
    return torch.from_numpy(g.standard_normal(int(np.prod(shape)), dtype=np.float32).reshape(shape) * np.float32(scale))


def ops_fixtures(ref):
    """Per-op goldens: each reference function on seeded inputs, fp32 and bf16."""
    blocks = ref["blocks"]
    attention = ref["attention"]
    g = rng(7)
    out = {}
    for dt_name, dt in (("f32", torch.float32), ("bf16", torch.bfloat16)):
        x = randn(g, 5, 64).to(dt)
        w = randn(g, 64, scale=0.1).to(dt)
        m = blocks.RMSNorm(64, 1e-6)
        m.weight.data = w.clone()
        out[f"rmsnorm.{dt_name}.x"], out[f"rmsnorm.{dt_name}.w"] = x, w
        out[f"rmsnorm.{dt_name}.y"] = m(x)

        x = randn(g, 6, 32).to(dt)
        z = randn(g, 6, 32).to(dt)
        w = (1.0 + randn(g, 32, scale=0.1)).to(dt)
        m = blocks.RMSNormGated(32, 1e-6).to(dt)
        m.weight.data = w.clone()
        out[f"rmsnorm_gated.{dt_name}.x"], out[f"rmsnorm_gated.{dt_name}.z"] = x, z
        out[f"rmsnorm_gated.{dt_name}.w"] = w
        out[f"rmsnorm_gated.{dt_name}.y"] = m(x, z)

        x = randn(g, 4, 3, 32).to(dt)
        out[f"l2norm.{dt_name}.x"], out[f"l2norm.{dt_name}.y"] = x, blocks.l2norm(x)

    # delta rules (fp32 state), with an initial state, l2norm inside the kernel
    for name, fn, T in (("recurrent", blocks.torch_recurrent_gated_delta_rule, 4),
                        ("chunked", blocks.torch_chunk_gated_delta_rule, 70)):
        B, H, d = 2, 3, 16
        q, k, v = randn(g, B, T, H, d), randn(g, B, T, H, d), randn(g, B, T, H, d)
        gg = -torch.nn.functional.softplus(randn(g, B, T, H)) * (1 + 3 * torch.rand(B, T, H, generator=torch.Generator().manual_seed(3)))
        beta = torch.sigmoid(randn(g, B, T, H))
        s0 = randn(g, B, H, d, d, scale=0.1)
        o, s = fn(q, k, v, gg, beta, initial_state=s0.clone(), use_qk_l2norm_in_kernel=True)
        for kname, t in (("q", q), ("k", k), ("v", v), ("g", gg), ("beta", beta), ("s0", s0),
                         ("out", o), ("state", s)):
            out[f"delta_{name}.{kname}"] = t

    # partial RoPE tables + rotation
    rope = blocks.RoPE(16, 1e7, "cpu")
    pos = torch.tensor([0, 1, 5, 1023, 4097, 32767])
    cos, sin = rope.cos_sin(pos, torch.float32)
    q = randn(g, 1, 2, 6, 64)
    k = randn(g, 1, 2, 6, 64)
    qr, kr = blocks.RoPE.apply(q, k, cos, sin)
    out.update({"rope.pos": pos, "rope.cos": cos, "rope.sin": sin, "rope.q": q, "rope.k": k,
                "rope.q_out": qr, "rope.k_out": kr})
    cosb, sinb = rope.cos_sin(pos, torch.bfloat16)
    out.update({"rope.cos_bf16": cosb, "rope.sin_bf16": sinb})

    # offset-causal attention (torch SDPA path), q_len 4 over 21 keys, plus decode
    for dt_name, dt in (("f32", torch.float32), ("bf16", torch.bfloat16)):
        q = randn(g, 2, 4, 4, 32).to(dt)
        k = randn(g, 2, 4, 21, 32).to(dt)
        v = randn(g, 2, 4, 21, 32).to(dt)
        out[f"attn.{dt_name}.q"], out[f"attn.{dt_name}.k"], out[f"attn.{dt_name}.v"] = q, k, v
        out[f"attn.{dt_name}.o"] = attention.torch_attention(q, k, v)
        out[f"attn.{dt_name}.o_decode"] = attention.torch_attention(q[:, :, -1:], k, v)
    return out


def sampler_fixtures(ref):
    """Capture the distribution the reference's sample_next draws from (torch.multinomial
    is intercepted and its probability vector recorded), plus greedy picks."""
    gen = ref["generate"]
    g = rng(11)
    out = {}
    cases = [(0.7, 20, 0.8, 1.1), (1.0, 0, 0.9, 1.0), (0.8, 50, 1.0, 1.0), (0.5, 0, 1.0, 1.05)]
    captured = []
    orig = torch.multinomial

    def grab(p, n):
        captured.append(p.detach().clone())
        return orig(p, n)

    prev = [3, 17, 17, 200, 511]
    logits_all = randn(g, len(cases), 512, scale=2.0)
    gen.torch.multinomial = grab
    try:
        for i, (t, tk, tp, rp) in enumerate(cases):
            gen.sample_next(logits_all[i].clone(), t, tk, tp, rp, prev)
    finally:
        gen.torch.multinomial = orig
    out["sampler.logits"] = logits_all
    out["sampler.params"] = torch.tensor(cases, dtype=torch.float64)
    out["sampler.prev"] = torch.tensor(prev)
    out["sampler.probs"] = torch.stack(captured)
    greedy = [gen.sample_next(logits_all[i].clone(), 0.0, 0, 1.0, rp, prev) for i, (_, _, _, rp) in enumerate(cases)]
    out["sampler.greedy"] = torch.tensor(greedy)
    return out


def build_ref_model(ref, raw_cfg, dtype, seed=WEIGHT_SEED):
    cfg = Qwen3_5Config.from_hf(raw_cfg)
    w = random_init(cfg, seed, dtype=torch.float32, generator="numpy")
    model = ref["weights"].load(raw_cfg, dict(w), "hf", device="cpu", dtype=dtype)
    mtp = ref["mtp"].load_mtp(model, dict(w), "hf", device="cpu", dtype=dtype)
    return cfg, model, mtp


def micro_fixtures(ref, dt_name, dtype):
    """MICRO model: prefill, a T=4 verify on the cache, a T=1 decode, the cache contents,
    and MTP outputs — everything through the reference's own modules."""
    cfg, model, mtp = build_ref_model(ref, MICRO, dtype)
    g = rng(21)
    B, P = 2, 10
    ids = torch.from_numpy(g.integers(0, cfg.vocab_size, size=(B, P))).long()
    out = {"ids": ids}
    logits, past, hidden = model(ids, return_hidden=True)
    out["prefill.logits"], out["prefill.hidden"] = logits, hidden
    ver = torch.from_numpy(g.integers(0, cfg.vocab_size, size=(B, 4))).long()
    out["verify.ids"] = ver
    logits, past, hidden = model(ver, past, return_hidden=True)
    out["verify.logits"], out["verify.hidden"] = logits, hidden
    dec = torch.from_numpy(g.integers(0, cfg.vocab_size, size=(B, 1))).long()
    out["decode.ids"] = dec
    logits, past, hidden = model(dec, past, return_hidden=True)
    out["decode.logits"], out["decode.hidden"] = logits, hidden
    for i, s in enumerate(past.layers):
        if cfg.layer_type(i) == "full_attention":
            out[f"cache.{i}.k"], out[f"cache.{i}.v"] = s[0], s[1]
        else:
            out[f"cache.{i}.conv"], out[f"cache.{i}.rec"] = s[0], s[1]
    # MTP: speculate over the prompt, and one depth-1 draft from the last hidden
    out["mtp.speculate"] = ref["mtp"].speculate(model, mtp, ids)
    emb = model.model.embed_tokens(dec)
    h1 = mtp(hidden[:, -1:], emb)
    out["mtp.draft_hidden"] = hidden[:, -1:]
    out["mtp.draft_out"] = h1
    out["mtp.draft_logits"] = model.lm_head(h1)
    return {f"micro.{dt_name}.{k}": v for k, v in out.items()}


def tiny_fixtures(ref, n_new=64, prompt_len=128):
    """greedy generate() and generate_mtp() (k=1) token streams, plus
    the last-position prefill logits."""
    cfg, model, mtp = build_ref_model(ref, TINY, torch.float32)
    g = rng(31)
    prompt = g.integers(0, cfg.vocab_size, size=prompt_len).tolist()
    decode = lambda toks: "".join(chr(0x1000 + t) for t in toks)   # one char per token
    kw = dict(max_new_tokens=n_new, temperature=0.0, top_k=0, top_p=1.0, repetition_penalty=1.0)
    greedy = "".join(ref["generate"].generate(model, prompt, decode, [], "cpu", **kw))
    calls = []
    orig_forward = model.forward

    def counting_forward(input_ids, past=None, return_hidden=False):
        calls.append(int(input_ids.shape[1]))
        return orig_forward(input_ids, past, return_hidden)

    model.forward = counting_forward
    spec = "".join(ref["mtp"].generate_mtp(model, mtp, prompt, decode, [], "cpu", **kw))
    model.forward = orig_forward
    ids = torch.tensor([prompt])
    logits, _, hidden = model(ids, return_hidden=True)
    return {
        "tiny.prompt": torch.tensor(prompt),
        "tiny.greedy": torch.tensor([ord(c) - 0x1000 for c in greedy]),
        "tiny.spec_k1": torch.tensor([ord(c) - 0x1000 for c in spec]),
        "tiny.spec_k1_forward_lens": torch.tensor(calls),
        "tiny.prefill_last_logits": logits[0, -1],
        "tiny.prefill_last_hidden": hidden[0, -1],
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path to the reference's src/ directory")
    ap.add_argument("--skip-tiny", action="store_true")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    import attention  # noqa: F401
    import generate
    from qwen3_5 import blocks, mtp, weights
    ref = {"blocks": blocks, "attention": attention, "generate": generate, "weights": weights, "mtp": mtp}
    torch.set_grad_enabled(False)

    tensors = {}
    tensors.update(ops_fixtures(ref))
    tensors.update(sampler_fixtures(ref))
    tensors.update(micro_fixtures(ref, "f32", torch.float32))
    tensors.update(micro_fixtures(ref, "bf16", torch.bfloat16))
    if not args.skip_tiny:
        tensors.update(tiny_fixtures(ref))
    tensors = {k: v.contiguous().clone() for k, v in tensors.items()}
    save_file(tensors, os.path.join(HERE, "golden.safetensors"))
    meta = {"weight_seed": WEIGHT_SEED, "weight_generator": "numpy-pcg64 N(0,0.02) float32",
            "configs": {"micro": MICRO, "tiny": TINY}, "torch": torch.__version__,
            "n_tensors": len(tensors)}
    with open(os.path.join(HERE, "golden_meta.json"), "w") as f:
        json.dump(meta, f, indent=1)
    print(f"wrote {len(tensors)} tensors")


if __name__ == "__main__":
    main()
