"""Generate tests/golden/golden_moe_cfg5.safetensors by running the REFERENCE's qwen3_5_moe
family at the per-layer shapes of BASELINE configs[4] (hidden 2048, 512 experts top-10 of
width 512 + a shared expert, GDN 16/32 heads of 128, attention 16/2 heads of 256, vocab
151936) with 2 layers (a GDN layer and an attention layer) and the MTP head, in fp32.

fp32, not bf16: with 512 experts the 10th and 11th router logits of a token are ~1 % of the
logit scale apart, within one or two bf16 rounding steps for about half of the tokens, so in
bf16 any last-bit difference upstream can change the routing of most tokens (the bf16 MoE
block is checked per token, with such near-ties flagged, by the other fixtures). In fp32 the
routing is unambiguous and the whole stack can be compared at its real shapes.

    python tests/golden/make_golden_moe_cfg5.py --reference <path-to-lollm>/src

Weights: `counter_init(seed 4321)` in fp32: uniform with standard deviation 0.02 from an
integer counter hash, bit-identical on every host and on the GPU, where the test rebuilds
the ~21 GB in seconds (a sequential numpy stream takes minutes at this size).
The logits rows are 151936 wide, so the file keeps per row: the argmax, the 32 largest
values with their indices, and the values at 1024 fixed vocabulary positions; plus every
router's logits (the tests flag routing near-ties from them). Contents, for B=2:
  prefill (12 prompt tokens), a speculative-width verify (T=4), a decode (T=1) and the MTP
  head's depth-1 draft from the decode's hidden state.
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

from lollm_b200.qwen3_5.config import QWEN35_MOE, Qwen3_5Config  # noqa: E402
from lollm_b200.qwen3_5.weights import counter_init  # noqa: E402

WEIGHT_SEED = 4321
LAYERS = 2
TOPN = 32
N_SAMPLE = 1024


def cfg5_reduced():
    raw = json.loads(json.dumps(QWEN35_MOE))
    raw["text_config"]["num_hidden_layers"] = LAYERS
    raw["text_config"]["layer_types"] = ["linear_attention", "full_attention"]
    return raw


def sample_columns(vocab):
    g = np.random.Generator(np.random.PCG64(99))
    return torch.from_numpy(np.sort(g.choice(vocab, size=N_SAMPLE, replace=False))).long()


def summarize(name, logits, cols):
    """argmax, top-32 (values, indices) and the values at `cols` of every row."""
    lf = logits.float()
    top = lf.topk(TOPN, dim=-1)
    return {f"{name}.argmax": lf.argmax(-1), f"{name}.top_v": top.values.to(logits.dtype),
            f"{name}.top_i": top.indices, f"{name}.cols": logits[..., cols]}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path to the reference's src/ directory")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    from qwen3_5_moe import mtp as rmtp
    from qwen3_5_moe import weights as rweights
    torch.set_grad_enabled(False)
    raw = cfg5_reduced()
    cfg = Qwen3_5Config.from_hf(raw)
    w = counter_init(cfg, WEIGHT_SEED, dtype=torch.float32)
    model = rweights.load(raw, dict(w), "hf", device="cpu", dtype=torch.float32)
    mtp = rmtp.load_mtp(model, dict(w), "hf", device="cpu", dtype=torch.float32)
    del w
    # record every router's logits, in call order
    routers = []
    for mod in list(model.modules()) + list(mtp.modules()):
        if type(mod).__name__ == "SparseMoeBlock":
            mod.gate.register_forward_hook(lambda m, i, o: routers.append(o.detach().clone()))
    cols = sample_columns(cfg.vocab_size)
    g = np.random.Generator(np.random.PCG64(71))
    B, P = 2, 12
    ids = torch.from_numpy(g.integers(0, cfg.vocab_size, size=(B, P))).long()
    ver = torch.from_numpy(g.integers(0, cfg.vocab_size, size=(B, 4))).long()
    dec = torch.from_numpy(g.integers(0, cfg.vocab_size, size=(B, 1))).long()
    out = {"ids": ids, "verify.ids": ver, "decode.ids": dec, "cols": cols}
    stages = []
    logits, past, hidden = model(ids, return_hidden=True)
    out.update(summarize("prefill", logits, cols)); stages.append(("prefill", len(routers)))
    logits, past, hidden = model(ver, past, return_hidden=True)
    out.update(summarize("verify", logits, cols)); stages.append(("verify", len(routers)))
    logits, past, hidden = model(dec, past, return_hidden=True)
    out.update(summarize("decode", logits, cols)); stages.append(("decode", len(routers)))
    out["decode.hidden"] = hidden
    emb = model.model.embed_tokens(dec)
    h1 = mtp(hidden[:, -1:], emb)
    out.update(summarize("draft", model.lm_head(h1), cols)); stages.append(("draft", len(routers)))
    for i, r in enumerate(routers):
        out[f"router.{i}"] = r
    out = {k: v.contiguous().clone() for k, v in out.items()}
    save_file(out, os.path.join(HERE, "golden_moe_cfg5.safetensors"))
    meta = {"weight_seed": WEIGHT_SEED, "weight_generator": "counter_init: splitmix64 counter hash, uniform, std 0.02, float32",
            "config": raw, "router_calls_after_stage": stages, "topn": TOPN, "n_sample_cols": N_SAMPLE,
            "torch": torch.__version__, "n_tensors": len(out)}
    with open(os.path.join(HERE, "golden_moe_cfg5_meta.json"), "w") as f:
        json.dump(meta, f, indent=1)
    print(f"wrote {len(out)} tensors")


if __name__ == "__main__":
    main()
