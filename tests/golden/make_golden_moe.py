"""Generate tests/golden/golden_moe.safetensors by running the REFERENCE's qwen3_5_moe family.

Run in a container where the reference checkout is importable:

    python tests/golden/make_golden_moe.py --reference <path-to-lollm>/src

It imports the reference's own `qwen3_5_moe` modules (`blocks.SparseMoeBlock`,
`weights.load`, `mtp.load_mtp` / `speculate` / `generate_mtp`) and the shared `generate`
loop, feeds them seeded inputs and the seeded weights of
`lollm_b200.qwen3_5.weights.random_init` (numpy PCG64: bit-identical on every host), and
stores inputs + outputs. Nothing at test time reads the reference. Re-running the script
reproduces the file bit-for-bit.

Contents:
  moe.<case>.w.*      the block's fp32 weights (the bf16 case casts them);
  moe.<case>.<dt>.*   one SparseMoeBlock (blocks.py:399-421) on seeded tokens: the input,
                      every weight, the router logits and the output, for three cases
                      (shared expert + renormalised top-k; no shared expert; top-k without
                      renormalisation), fp32 and bf16;
  micro_moe.<dt>.*    the MICRO_MOE model (every FFN sparse except the forced-dense layer 1):
                      prefill / verify / decode logits and hidden states, plus the MTP head;
  micro_moe.greedy / .spec_k1   fp32 generate() and generate_mtp() (k=1) token streams
                      (temperature 0 with repetition penalty 4).
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

from lollm_b200.qwen3_5.config import MICRO_MOE, Qwen3_5Config  # noqa: E402
from lollm_b200.qwen3_5.weights import random_init  # noqa: E402

WEIGHT_SEED = 1234

# (name, hidden, experts, top_k, inter, shared_inter, norm_topk_prob, tokens)
MOE_CASES = [
    ("shared", 128, 16, 4, 64, 64, True, 40),
    ("noshared", 128, 16, 4, 64, 0, True, 24),
    ("nonorm", 64, 8, 3, 32, 32, False, 17),
]


def rng(seed):
    return np.random.Generator(np.random.PCG64(seed))


def randn(g, *shape, scale=1.0):
    return torch.from_numpy(g.standard_normal(int(np.prod(shape)), dtype=np.float32).reshape(shape)
                            * np.float32(scale))


def moe_block_fixtures(ref):
    blocks = ref["blocks"]
    out = {}
    g = rng(41)
    for name, h, e, k, im, ish, norm, n in MOE_CASES:
        raw = dict(MICRO_MOE["text_config"])
        raw.update(hidden_size=h, num_experts=e, num_experts_per_tok=k, moe_intermediate_size=im,
                   shared_expert_intermediate_size=ish, norm_topk_prob=norm)
        cfg = ref["config"].Qwen3_5MoeConfig.from_hf({"text_config": raw})
        x32 = randn(g, n, h)
        w32 = {"gate.weight": randn(g, e, h, scale=0.05),
               "experts.gate_up_proj": randn(g, e, 2 * im, h, scale=0.05),
               "experts.down_proj": randn(g, e, h, im, scale=0.05)}
        if ish > 0:
            w32.update({"shared_expert.gate_proj.weight": randn(g, ish, h, scale=0.05),
                        "shared_expert.up_proj.weight": randn(g, ish, h, scale=0.05),
                        "shared_expert.down_proj.weight": randn(g, h, ish, scale=0.05),
                        "shared_expert_gate.weight": randn(g, 1, h, scale=0.05)})
        for dt_name, dt in (("f32", torch.float32), ("bf16", torch.bfloat16)):
            m = blocks.SparseMoeBlock(cfg).to(dt)
            sd = {kk: v.to(dt) for kk, v in w32.items()}
            m.load_state_dict(sd, strict=True)
            x = x32.to(dt)
            p = f"moe.{name}.{dt_name}."
            out[p + "x"] = x
            if dt == torch.float32:   # the bf16 case uses these cast to bf16
                for kk, v in sd.items():
                    out[f"moe.{name}.w." + kk] = v
            out[p + "router_logits"] = m.gate(x)
            out[p + "y"] = m(x[None])[0]
    return out


def build_ref_model(ref, raw_cfg, dtype, seed=WEIGHT_SEED):
    cfg = Qwen3_5Config.from_hf(raw_cfg)
    w = random_init(cfg, seed, dtype=torch.float32, generator="numpy")
    model = ref["weights"].load(raw_cfg, dict(w), "hf", device="cpu", dtype=dtype)
    mtp = ref["mtp"].load_mtp(model, dict(w), "hf", device="cpu", dtype=dtype)
    return cfg, model, mtp


def micro_moe_fixtures(ref, dt_name, dtype):
    cfg, model, mtp = build_ref_model(ref, MICRO_MOE, dtype)
    g = rng(51)
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
    out["mtp.speculate"] = ref["mtp"].speculate(model, mtp, ids)
    emb = model.model.embed_tokens(dec)
    h1 = mtp(hidden[:, -1:], emb)
    out["mtp.draft_hidden"] = hidden[:, -1:]
    out["mtp.draft_out"] = h1
    out["mtp.draft_logits"] = model.lm_head(h1)
    return {f"micro_moe.{dt_name}.{k}": v for k, v in out.items()}


def micro_moe_streams(ref, n_new=24, prompt_len=16):
    cfg, model, mtp = build_ref_model(ref, MICRO_MOE, torch.float32)
    g = rng(61)
    prompt = g.integers(0, cfg.vocab_size, size=prompt_len).tolist()
    decode = lambda toks: "".join(chr(0x1000 + t) for t in toks)   # one char per token
    # greedy with a repetition penalty: random-init weights otherwise repeat one token
    kw = dict(max_new_tokens=n_new, temperature=0.0, top_k=0, top_p=1.0, repetition_penalty=4.0)
    greedy = "".join(ref["generate"].generate(model, prompt, decode, [], "cpu", **kw))
    spec = "".join(ref["mtp"].generate_mtp(model, mtp, prompt, decode, [], "cpu", **kw))
    return {"micro_moe.prompt": torch.tensor(prompt),
            "micro_moe.greedy": torch.tensor([ord(c) - 0x1000 for c in greedy]),
            "micro_moe.spec_k1": torch.tensor([ord(c) - 0x1000 for c in spec])}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path to the reference's src/ directory")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    import generate
    from qwen3_5_moe import blocks, config, mtp, weights
    ref = {"blocks": blocks, "config": config, "generate": generate, "weights": weights, "mtp": mtp}
    torch.set_grad_enabled(False)

    tensors = {}
    tensors.update(moe_block_fixtures(ref))
    tensors.update(micro_moe_fixtures(ref, "f32", torch.float32))
    tensors.update(micro_moe_fixtures(ref, "bf16", torch.bfloat16))
    tensors.update(micro_moe_streams(ref))
    tensors = {k: v.contiguous().clone() for k, v in tensors.items()}
    save_file(tensors, os.path.join(HERE, "golden_moe.safetensors"))
    meta = {"weight_seed": WEIGHT_SEED, "weight_generator": "numpy-pcg64 N(0,0.02) float32",
            "configs": {"micro_moe": MICRO_MOE}, "moe_cases": MOE_CASES,
            "torch": torch.__version__, "n_tensors": len(tensors)}
    with open(os.path.join(HERE, "golden_moe_meta.json"), "w") as f:
        json.dump(meta, f, indent=1)
    print(f"wrote {len(tensors)} tensors")


if __name__ == "__main__":
    main()
