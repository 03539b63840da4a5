"""Pin the CPU oracle against goldens produced by the reference itself (CPU only).

Fixtures: tests/golden/golden.safetensors, written by tests/golden/make_golden.py from the
reference's own functions on seeded inputs and seeded weights.
"""

import numpy as np
import pytest
import torch

from oracle import loops as L
from oracle import qwen35 as Q
from oracle import sampling as S
from lollm_b200.qwen3_5.config import MICRO, TINY, Qwen3_5Config
from lollm_b200.qwen3_5.weights import load_checkpoint, random_init

WEIGHT_SEED = 1234


def close(a, b, rtol, atol):
    torch.testing.assert_close(a.float(), b.float(), rtol=rtol, atol=atol)


@pytest.mark.parametrize("dt", ["f32", "bf16"])
def test_norms(golden, dt):
    G = golden
    tol = dict(rtol=1e-6, atol=1e-6) if dt == "f32" else dict(rtol=0, atol=0)
    close(Q.rms_norm(G[f"rmsnorm.{dt}.x"], G[f"rmsnorm.{dt}.w"], 1e-6), G[f"rmsnorm.{dt}.y"], **tol)
    close(Q.rms_norm_gated(G[f"rmsnorm_gated.{dt}.x"], G[f"rmsnorm_gated.{dt}.z"],
                           G[f"rmsnorm_gated.{dt}.w"], 1e-6), G[f"rmsnorm_gated.{dt}.y"], **tol)
    close(Q.l2_normalize(G[f"l2norm.{dt}.x"]), G[f"l2norm.{dt}.y"], **tol)


@pytest.mark.parametrize("name", ["recurrent", "chunked"])
@pytest.mark.parametrize("algo", ["recurrent", "chunked"])
def test_delta_rule(golden, name, algo):
    G = golden
    p = f"delta_{name}."
    q, k = Q.l2_normalize(G[p + "q"]), Q.l2_normalize(G[p + "k"])
    fn = Q.delta_rule_recurrent if algo == "recurrent" else Q.delta_rule_chunked
    out, st = fn(q, k, G[p + "v"], G[p + "g"], G[p + "beta"], G[p + "s0"])
    close(out, G[p + "out"], rtol=1e-4, atol=2e-5)
    close(st, G[p + "state"], rtol=1e-4, atol=2e-5)


def test_rope(golden):
    G = golden
    cos, sin = Q.rope_cos_sin(G["rope.pos"], 16, 1e7, torch.float32)
    assert torch.equal(cos, G["rope.cos"]) and torch.equal(sin, G["rope.sin"])
    cb, sb = Q.rope_cos_sin(G["rope.pos"], 16, 1e7, torch.bfloat16)
    assert torch.equal(cb, G["rope.cos_bf16"]) and torch.equal(sb, G["rope.sin_bf16"])
    close(Q.rope_rotate(G["rope.q"], cos, sin), G["rope.q_out"], rtol=1e-6, atol=1e-6)
    close(Q.rope_rotate(G["rope.k"], cos, sin), G["rope.k_out"], rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("dt", ["f32", "bf16"])
def test_attention(golden, dt):
    G = golden
    q, k, v = G[f"attn.{dt}.q"], G[f"attn.{dt}.k"], G[f"attn.{dt}.v"]
    tol = dict(rtol=1e-5, atol=1e-5) if dt == "f32" else dict(rtol=0, atol=1.6e-2)
    for b in range(q.shape[0]):
        close(Q.offset_causal_attention(q[b], k[b], v[b]), G[f"attn.{dt}.o"][b], **tol)
        close(Q.offset_causal_attention(q[b, :, -1:], k[b], v[b]), G[f"attn.{dt}.o_decode"][b], **tol)


def test_sampler_distribution(golden):
    G = golden
    prev = G["sampler.prev"].tolist()
    for i, (t, tk, tp, rp) in enumerate(G["sampler.params"].tolist()):
        p = S.filtered_probs(G["sampler.logits"][i], t, int(tk), tp, rp, prev)
        close(p, G["sampler.probs"][i], rtol=1e-5, atol=1e-7)
        assert ((p > 0) == (G["sampler.probs"][i] > 0)).all()
        assert S.sample_next(G["sampler.logits"][i], 0.0, 0, 1.0, rp, prev) == int(G["sampler.greedy"][i])


def test_speculative_accept_reduces_to_greedy():
    g = torch.Generator().manual_seed(0)
    V, k = 50, 3
    for _ in range(20):
        logits = torch.randn(k + 1, V, generator=g)
        tgt = logits.argmax(-1)
        drafts = torch.where(torch.rand(k, generator=g) < 0.5, tgt[:k], torch.randint(0, V, (k,), generator=g))
        p = torch.nn.functional.one_hot(tgt, V).float()
        q = torch.nn.functional.one_hot(drafts, V).float()
        a1, t1 = S.greedy_accept(tgt, drafts)
        a2, t2, _ = S.speculative_accept(p, q, drafts, torch.rand(k, generator=g), torch.rand(1, generator=g)[0])
        assert (a1, t1) == (a2, t2)


def test_speculative_accept_is_lossless():
    """The output-token distribution of one speculative step equals p (Monte Carlo)."""
    g = np.random.Generator(np.random.PCG64(5))
    V = 6
    p = torch.tensor(g.dirichlet(np.ones(V)), dtype=torch.float64)[None].repeat(2, 1)
    q = torch.tensor(g.dirichlet(np.ones(V)), dtype=torch.float64)[None]
    counts = np.zeros(V)
    n = 20000
    for _ in range(n):
        d = S.inverse_cdf(q[0], g.random())
        a, t, _ = S.speculative_accept(p, q, [d], [g.random()], g.random())
        counts[d if a == 1 else t] += 1
    assert np.abs(counts / n - p[0].numpy()).max() < 0.015


def _micro(dtype):
    cfg = Qwen3_5Config.from_hf(MICRO)
    P = load_checkpoint(cfg, random_init(cfg, WEIGHT_SEED, generator="numpy"), dtype=dtype)
    return cfg, P


@pytest.mark.parametrize("dt", ["f32", "bf16"])
def test_micro_model(golden, dt):
    G = {k[len(f"micro.{dt}."):]: v for k, v in golden.items() if k.startswith(f"micro.{dt}.")}
    cfg, P = _micro(torch.float32 if dt == "f32" else torch.bfloat16)
    tol = dict(rtol=1e-4, atol=1e-5) if dt == "f32" else dict(rtol=2e-2, atol=2e-2)
    logits, cache, hidden = Q.model_forward(P, cfg, G["ids"])
    close(logits, G["prefill.logits"], **tol)
    close(hidden, G["prefill.hidden"], **tol)
    logits, cache, hidden = Q.model_forward(P, cfg, G["verify.ids"], cache)
    close(logits, G["verify.logits"], **tol)
    logits, cache, hidden = Q.model_forward(P, cfg, G["decode.ids"], cache)
    close(logits, G["decode.logits"], **tol)
    for i in cfg.attn_layers:
        for b in range(2):
            close(cache.kv[i][b][0], G[f"cache.{i}.k"][b], **tol)
            close(cache.kv[i][b][1], G[f"cache.{i}.v"][b], **tol)
    for i in cfg.gdn_layers:
        close(cache.gdn[i][0], G[f"cache.{i}.conv"], **tol)
        close(cache.gdn[i][1], G[f"cache.{i}.rec"], **tol)
    post, _ = Q.mtp_forward(P, cfg, G["mtp.draft_hidden"], torch.nn.functional.embedding(
        G["decode.ids"], P["model.embed_tokens.weight"]))
    close(post, G["mtp.draft_out"], **tol)
    close(Q.lm_head(P, post), G["mtp.draft_logits"], **tol)
    # speculate(): MTP over the whole prompt, hidden i paired with the embedding of token i+1
    _, _, hid = Q.model_forward(P, cfg, G["ids"])
    emb = torch.nn.functional.embedding(G["ids"], P["model.embed_tokens.weight"])
    post, _ = Q.mtp_forward(P, cfg, hid[:, :-1], emb[:, 1:])
    close(Q.lm_head(P, post), G["mtp.speculate"], **tol)


def test_micro_recurrent_matches_chunked(golden):
    """The recurrent-only scan (what the CUDA kernel computes) agrees with the reference's
    chunked dispatch on the whole model in fp32."""
    G = {k[len("micro.f32."):]: v for k, v in golden.items() if k.startswith("micro.f32.")}
    cfg, P = _micro(torch.float32)
    logits, cache, _ = Q.model_forward(P, cfg, G["ids"], scan="recurrent")
    close(logits, G["prefill.logits"], rtol=1e-4, atol=1e-5)
    logits, cache, _ = Q.model_forward(P, cfg, G["verify.ids"], cache, scan="recurrent")
    close(logits, G["verify.logits"], rtol=1e-4, atol=1e-5)


@pytest.mark.slow
def test_tiny_greedy_stream(golden):
    """BASELINE configs[0] shape: the oracle's greedy stream and its k=1 speculative stream
    both equal the reference's generate() stream (fp32)."""
    cfg = Qwen3_5Config.from_hf(TINY)
    P = load_checkpoint(cfg, random_init(cfg, WEIGHT_SEED, generator="numpy"))
    prompt = golden["tiny.prompt"][None]
    n = 16
    logits, _, hidden = Q.model_forward(P, cfg, prompt)
    close(logits[0, -1], golden["tiny.prefill_last_logits"], rtol=1e-4, atol=1e-5)
    got = L.greedy_generate(P, cfg, prompt, n)[0]
    assert got.tolist() == golden["tiny.greedy"][:n].tolist()
    spec, _ = L.spec_generate(P, cfg, prompt, n, k=1)
    assert spec[0] == golden["tiny.spec_k1"][:n].tolist()
