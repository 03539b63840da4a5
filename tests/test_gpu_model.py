"""Whole-step parity on the GPU: the qsp model path (C ABI) against the reference's own
outputs (golden fixtures) and the CPU oracle. fp32 logits within 1e-4 relative, bf16 within
2e-2 (tests/tolerance.py); greedy token streams token-identical; speculative streams equal the
greedy stream."""

import pytest
import torch

from oracle import loops as OL
from oracle import qwen35 as Q
from lollm_b200.qwen3_5.config import MICRO, TINY, Qwen3_5Config
from lollm_b200.qwen3_5.weights import load_checkpoint, random_init
from tolerance import assert_close_dt

pytestmark = pytest.mark.gpu
SEED = 1234


def build(raw, dtype, **kw):
    from lollm_b200 import qwen3_5 as fam
    cfg = Qwen3_5Config.from_hf(raw)
    w = random_init(cfg, SEED, generator="numpy")
    model = fam.load(raw, dict(w), dtype=dtype, **kw)
    mtp = fam.load_mtp(model, dict(w))
    return cfg, model, mtp, w


def close(got, want, dt):
    assert_close_dt(got, want, dt)


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_micro_forward_matches_reference(golden, dt):
    name = "f32" if dt == torch.float32 else "bf16"
    G = {k[len(f"micro.{name}."):]: v for k, v in golden.items() if k.startswith(f"micro.{name}.")}
    cfg, model, mtp, _ = build(MICRO, dt, max_positions=256)
    logits, past, hidden = model(G["ids"].cuda(), return_hidden=True)
    close(logits, G["prefill.logits"], dt)
    close(hidden, G["prefill.hidden"], dt)
    logits, past, hidden = model(G["verify.ids"].cuda(), past, return_hidden=True)
    close(logits, G["verify.logits"], dt)
    logits, past, hidden = model(G["decode.ids"].cuda(), past, return_hidden=True)
    close(logits, G["decode.logits"], dt)
    for i in cfg.gdn_layers:
        conv, rec = past.linear_state(i)
        close(conv, G[f"cache.{i}.conv"], dt)
        close(rec, G[f"cache.{i}.rec"], dt)
    for i in cfg.attn_layers:
        k, v = past.read_kv(i)
        close(k, G[f"cache.{i}.k"], dt)
        close(v, G[f"cache.{i}.v"], dt)
    assert past.seen_tokens == 15
    # MTP depth 1 from (hidden, token) — the reference head's logits
    ids = torch.zeros(2, 2, dtype=torch.int64, device="cuda")
    ids[:, 0] = G["decode.ids"][:, 0].cuda()
    h = G["mtp.draft_hidden"][:, 0].to(device="cuda", dtype=dt).contiguous()
    dl = mtp.draft(h, ids, 1)
    close(dl[:, 0], G["mtp.draft_logits"][:, 0], dt)
    assert torch.equal(ids[:, 1].cpu(), G["mtp.draft_logits"][:, 0].float().argmax(-1))


def test_micro_speculative_forward_and_rollback_match_oracle():
    """fp32: a speculative T=4 forward, ragged accept, then a decode — logits and the flushed
    GDN state match the oracle run on exactly the kept tokens."""
    dt = torch.float32
    cfg, model, mtp, w = build(MICRO, dt, max_positions=256)
    P = load_checkpoint(cfg, random_init(cfg, SEED, generator="numpy"))
    g = torch.Generator().manual_seed(3)
    B = 3
    prompt = torch.randint(0, cfg.vocab_size, (B, 7), generator=g)
    cache = model.new_cache(B, 64)
    model(prompt.cuda(), cache)
    _, oc, _ = Q.model_forward(P, cfg, prompt, scan="recurrent")
    ver = torch.randint(0, cfg.vocab_size, (B, 4), generator=g)
    logits, _ = model(ver.cuda(), cache, speculative=True)
    ol, _, _ = Q.model_forward(P, cfg, ver, oc.clone(), scan="recurrent")
    close(logits, ol, dt)
    keep = [1, 4, 2]
    cache.accept(torch.tensor([k - 1 for k in keep], dtype=torch.int32, device="cuda"))
    # oracle: per sequence, the kept prefix only
    from oracle.loops import _merge, _select
    subs = []
    for b in range(B):
        sub = _select(oc, b)
        _, sub, _ = Q.model_forward(P, cfg, ver[b:b + 1, :keep[b]], sub, scan="recurrent")
        subs.append(sub)
    oc = _merge(subs, cfg.num_hidden_layers)
    assert cache.seen_tokens == [7 + k for k in keep]
    dec = torch.randint(0, cfg.vocab_size, (B, 1), generator=g)
    logits, _ = model(dec.cuda(), cache)
    ol, oc, _ = Q.model_forward(P, cfg, dec, oc, scan="recurrent")
    close(logits, ol, dt)
    for i in cfg.gdn_layers:
        conv, rec = cache.linear_state(i)
        close(rec, oc.gdn[i][1], dt)
        close(conv, oc.gdn[i][0], dt)


@pytest.mark.parametrize("k", [1, 3])
def test_tiny_speculative_stream_equals_reference_greedy(golden, k):
    """BASELINE configs[0] (fp32): the speculative decoder's committed stream equals the
    reference's greedy generate() stream token for token."""
    from lollm_b200.qwen3_5 import SpecDecoder
    cfg, model, mtp, _ = build(TINY, torch.float32, max_positions=512)
    prompt = golden["tiny.prompt"][None].cuda()
    n = 64
    dec = SpecDecoder(model, mtp, 1, k, 128 + n + 2 * k + 4, out_capacity=n + k + 1)
    dec.prefill(prompt)
    while int(dec.n_out[0]) - dec.prompt_len < n:
        dec.step()
    got = dec.outputs()[0][:n]
    assert got == golden["tiny.greedy"][:n].tolist()


def test_tiny_prefill_logits_and_plain_greedy(golden):
    from lollm_b200.generate import generate
    cfg, model, mtp, _ = build(TINY, torch.float32, max_positions=512)
    prompt = golden["tiny.prompt"].tolist()
    logits, _ = model(torch.tensor([prompt]).cuda())
    close(logits[0, -1], golden["tiny.prefill_last_logits"], torch.float32)
    dec = lambda toks: "".join(chr(0x1000 + t) for t in toks)
    text = "".join(generate(model, prompt, dec, [], "cuda", max_new_tokens=24, temperature=0.0,
                            top_k=0, top_p=1.0, repetition_penalty=1.0))
    assert [ord(c) - 0x1000 for c in text] == golden["tiny.greedy"][:24].tolist()


def test_micro_batched_spec_matches_oracle_greedy():
    """Batch of 4 ragged-accepting sequences, k=3, graph-captured steps: each stream equals
    the oracle's greedy stream (fp32)."""
    from lollm_b200.qwen3_5 import SpecDecoder
    cfg, model, mtp, _ = build(MICRO, torch.float32, max_positions=256)
    P = load_checkpoint(cfg, random_init(cfg, SEED, generator="numpy"))
    g = torch.Generator().manual_seed(5)
    B, n = 4, 20
    prompt = torch.randint(0, cfg.vocab_size, (B, 9), generator=g)
    want = OL.greedy_generate(P, cfg, prompt, n, scan="recurrent")
    dec = SpecDecoder(model, mtp, B, 3, 9 + n + 12, out_capacity=n + 8)
    dec.prefill(prompt.cuda())
    while int(dec.n_out.min()) - dec.prompt_len < n:
        dec.step()
    assert [o[:n] for o in dec.outputs()] == want.tolist()
    # the same through a captured CUDA graph (one eager warm-up step, then replays)
    dec2 = SpecDecoder(model, mtp, B, 3, 9 + n + 12, out_capacity=n + 8)
    dec2.prefill(prompt.cuda())
    dec2.capture(warmup=1)
    while int(dec2.n_out.min()) - dec2.prompt_len < n:
        dec2.replay()
    assert [o[:n] for o in dec2.outputs()] == want.tolist()


def test_tiny_speculative_with_repetition_penalty_equals_plain_generate():
    """Greedy decoding with the reference's repetition penalty: the speculative decoder (k=3;
    penalty context = prompt + committed tokens + the step's tokens up to each position)
    commits exactly the stream of plain autoregressive generate() with the same penalty."""
    from lollm_b200.generate import generate
    from lollm_b200.qwen3_5 import SpecDecoder
    cfg, model, mtp, _ = build(TINY, torch.float32, max_positions=512)
    g = torch.Generator().manual_seed(3)
    prompt = torch.randint(0, cfg.vocab_size, (48,), generator=g).tolist()
    n, rp = 32, 1.3
    dec_txt = lambda toks: "".join(chr(0x1000 + t) for t in toks)
    text = "".join(generate(model, prompt, dec_txt, [], "cuda", max_new_tokens=n, temperature=0.0,
                            top_k=0, top_p=1.0, repetition_penalty=rp))
    want = [ord(c) - 0x1000 for c in text]
    dec = SpecDecoder(model, mtp, 1, 3, len(prompt) + n + 12, repetition_penalty=rp, out_capacity=n + 4)
    dec.prefill(torch.tensor([prompt]).cuda())
    while int(dec.n_out[0]) - dec.prompt_len < n:
        dec.step()
    assert dec.outputs()[0][:n] == want


def test_micro_filtered_stochastic_spec_runs_in_a_graph():
    """The reference generate_mtp's default sampling (T 0.7, top-k 20, top-p 0.8, penalty 1.1)
    through the lossless sampler, batched and captured in a CUDA graph: tokens are valid and
    every step commits 1..k+1 tokens per sequence."""
    from lollm_b200.qwen3_5 import SpecDecoder
    cfg, model, mtp, _ = build(MICRO, torch.bfloat16, max_positions=256)
    B, k = 3, 3
    g = torch.Generator(device="cuda").manual_seed(9)
    dec = SpecDecoder(model, mtp, B, k, 16 + 40 * (k + 1), temperature=0.7, top_k=20, top_p=0.8,
                      repetition_penalty=1.1, out_capacity=40 * (k + 1))
    dec.u = {"draft": torch.rand(B, k, device="cuda", generator=g), "accept": torch.rand(B, k, device="cuda", generator=g),
             "resample": torch.rand(B, device="cuda", generator=g)}
    dec.prefill(torch.randint(0, cfg.vocab_size, (B, 16), device="cuda"),
                u_first=torch.rand(B, device="cuda", generator=g))
    dec.capture(warmup=1)
    prev = dec.n_out.clone()
    for _ in range(10):
        for t in dec.u.values():
            t.copy_(torch.rand(t.shape, device="cuda", generator=g))
        dec.replay()
        d = (dec.n_out - prev).tolist()
        assert all(1 <= x <= k + 1 for x in d)
        prev = dec.n_out.clone()
    for toks in dec.outputs():
        assert all(0 <= t < cfg.vocab_size for t in toks)


def test_graft_entry_smoke():
    """The packaged smoke check (one forward against the oracle, then speculative steps whose
    committed stream must equal the oracle's greedy stream) runs as a test too."""
    import __graft_entry__
    __graft_entry__.smoke()
