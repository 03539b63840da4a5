"""Pin the CPU oracle's sparse-MoE FFN and the MoE-family model against goldens produced by
the reference's own qwen3_5_moe modules (CPU only).

Fixtures: tests/golden/golden_moe.safetensors, written by tests/golden/make_golden_moe.py.
"""

import os

import pytest
import torch

from oracle import loops as L
from oracle import qwen35 as Q
from lollm_b200.qwen3_5.config import MICRO_MOE, Qwen3_5Config
from lollm_b200.qwen3_5.weights import load_checkpoint, random_init

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
WEIGHT_SEED = 1234
# (name, hidden, experts, top_k, inter, shared_inter, norm_topk_prob, tokens) — as generated
MOE_CASES = [
    ("shared", 128, 16, 4, 64, 64, True, 40),
    ("noshared", 128, 16, 4, 64, 0, True, 24),
    ("nonorm", 64, 8, 3, 32, 32, False, 17),
]


@pytest.fixture(scope="module")
def golden_moe():
    from safetensors.torch import load_file
    return load_file(os.path.join(ROOT, "tests", "golden", "golden_moe.safetensors"))


def moe_case(G, name, dt):
    """(cfg, params {"mlp.*": tensor}, x, router logits, y) of one generated block case."""
    _, h, e, k, im, ish, norm, _ = next(c for c in MOE_CASES if c[0] == name)
    raw = dict(MICRO_MOE["text_config"])
    raw.update(hidden_size=h, num_experts=e, num_experts_per_tok=k, moe_intermediate_size=im,
               shared_expert_intermediate_size=ish, norm_topk_prob=norm)
    cfg = Qwen3_5Config.from_hf({"text_config": raw})
    dtype = torch.float32 if dt == "f32" else torch.bfloat16
    pre = f"moe.{name}.w."
    P = {"mlp." + kk[len(pre):]: v.to(dtype) for kk, v in G.items() if kk.startswith(pre)}
    p = f"moe.{name}.{dt}."
    return cfg, P, G[p + "x"], G[p + "router_logits"], G[p + "y"]


def close(a, b, rtol, atol):
    torch.testing.assert_close(a.float(), b.float(), rtol=rtol, atol=atol)


@pytest.mark.parametrize("dt", ["f32", "bf16"])
@pytest.mark.parametrize("name", [c[0] for c in MOE_CASES])
def test_moe_block(golden_moe, name, dt):
    cfg, P, x, logits, y = moe_case(golden_moe, name, dt)
    # the same torch ops in the same order as SparseMoeBlock.forward: bit-identical
    close(Q.linear(x, P["mlp.gate.weight"]), logits, rtol=0, atol=0)
    close(Q.moe_ffn(P, "mlp.", cfg, x), y, rtol=0, atol=0)


def _micro_moe(dtype):
    cfg = Qwen3_5Config.from_hf(MICRO_MOE)
    P = load_checkpoint(cfg, random_init(cfg, WEIGHT_SEED, generator="numpy"), dtype=dtype)
    return cfg, P


def test_micro_moe_config_rules():
    cfg = Qwen3_5Config.from_hf(MICRO_MOE)
    assert [cfg.is_moe_layer(i) for i in range(cfg.num_hidden_layers)] == [
        True, False, True, True, True, True, True, True]
    raw = {"text_config": dict(MICRO_MOE["text_config"])}
    del raw["text_config"]["num_experts_per_tok"]
    with pytest.raises(KeyError):
        Qwen3_5Config.from_hf(raw)


def routed_forward(P, cfg, ids, cache, stale):
    """Oracle forward that also returns the rows to compare: not a routing near-tie in this
    call and not in a sequence (`stale`, updated in place) flagged by an earlier call."""
    Q.ROUTER_MARGINS = []
    try:
        logits, cache, hidden = Q.model_forward(P, cfg, ids, cache)
        flag = Q.near_tie_rows(Q.ROUTER_MARGINS, *ids.shape)
    finally:
        Q.ROUTER_MARGINS = None
    flag |= stale[:, None]
    stale |= flag.any(dim=1)
    return logits, cache, hidden, ~flag


@pytest.mark.parametrize("dt", ["f32", "bf16"])
def test_micro_moe_model(golden_moe, dt):
    """In bf16 a token whose k-th and (k+1)-th router logits are within two rounding steps
    is a flagged near-tie: the reference's chunked GDN and this oracle round differently in
    the last bit, which can swap one expert. Flagged rows (and the rest of their sequence)
    are excluded and counted; fp32 has none."""
    G = {k[len(f"micro_moe.{dt}."):]: v for k, v in golden_moe.items() if k.startswith(f"micro_moe.{dt}.")}
    cfg, P = _micro_moe(torch.float32 if dt == "f32" else torch.bfloat16)
    tol = dict(rtol=1e-4, atol=1e-5) if dt == "f32" else dict(rtol=2e-2, atol=2e-2)
    stale = torch.zeros(G["ids"].shape[0], dtype=torch.bool)
    n_cmp = 0
    logits, cache, hidden, ok = routed_forward(P, cfg, G["ids"], None, stale)
    close(logits[ok], G["prefill.logits"][ok], **tol)
    close(hidden[ok], G["prefill.hidden"][ok], **tol)
    n_cmp += int(ok.sum())
    for name in ("verify", "decode"):
        logits, cache, hidden, ok = routed_forward(P, cfg, G[f"{name}.ids"], cache, stale)
        close(logits[ok], G[f"{name}.logits"][ok], **tol)
        n_cmp += int(ok.sum())
    assert n_cmp >= (26 if dt == "f32" else 12), n_cmp
    post, _ = Q.mtp_forward(P, cfg, G["mtp.draft_hidden"], torch.nn.functional.embedding(
        G["decode.ids"], P["model.embed_tokens.weight"]))
    close(post, G["mtp.draft_out"], **tol)
    close(Q.lm_head(P, post), G["mtp.draft_logits"], **tol)
    _, _, hid = Q.model_forward(P, cfg, G["ids"])
    emb = torch.nn.functional.embedding(G["ids"], P["model.embed_tokens.weight"])
    post, _ = Q.mtp_forward(P, cfg, hid[:, :-1], emb[:, 1:])
    close(Q.lm_head(P, post), G["mtp.speculate"], **tol)


def test_micro_moe_penalised_greedy_stream(golden_moe):
    """generate() at temperature 0 with repetition penalty 4 (fp32): the oracle's stream is
    the reference's; generate_mtp (k=1) produced the same stream."""
    cfg, P = _micro_moe(torch.float32)
    prompt = golden_moe["micro_moe.prompt"][None]
    want = golden_moe["micro_moe.greedy"].tolist()
    got = L.greedy_generate(P, cfg, prompt, len(want), repetition_penalty=4.0)[0].tolist()
    assert got == want
    assert golden_moe["micro_moe.spec_k1"].tolist() == want
