"""Filtered sampling on the GPU (repetition penalty, temperature, top-k, top-p: sample_next,
src/generate.py:17-37) against the reference's own distributions captured in tests/golden,
and against the oracle restatement on larger rows; the filtered p/q speculative sampler
against oracle.sampling.speculative_accept on the filtered distributions.

A categorical draw is compared through the inverse CDF at the same uniform; uniforms that
fall within 1e-5 of a bucket edge are skipped (fp32 vs fp64 rounding may move them)."""

import pytest
import torch

from oracle import sampling as S

pytestmark = pytest.mark.gpu
DEV = "cuda"


def K():
    from lollm_b200 import kernels
    return kernels


def draw(logits, temperature, top_k, top_p, rep, hist_rows=None, step=None, step_base=0, rows_per_seq=1, u=None):
    """GPU filtered draw for every row; hist_rows: list (per sequence) of token lists."""
    k = K()
    rows, V = logits.shape
    hist = hist_n = None
    if hist_rows is not None:
        n = max(1, max(len(h) for h in hist_rows))
        hist = torch.full((len(hist_rows), n), -1, dtype=torch.int64)
        for b, h in enumerate(hist_rows):
            hist[b, :len(h)] = torch.tensor(h, dtype=torch.int64)
        hist = hist.to(DEV)
        hist_n = torch.tensor([len(h) for h in hist_rows], dtype=torch.int32, device=DEV)
    step_d = step.to(DEV).contiguous() if step is not None else None
    sp = k.sample_params(temperature, top_k, top_p, rep, hist=hist, hist_n=hist_n, step_ids=step_d,
                         step_base=step_base)
    ws = torch.empty(k.filter_workspace_bytes(rows, V), dtype=torch.uint8, device=DEV)
    out = torch.empty(rows, dtype=torch.int64, device=DEV)
    ud = None if u is None else torch.as_tensor(u, dtype=torch.float32).to(DEV)
    k.sample_filtered(logits.to(DEV).contiguous(), sp, ud, out, ws, rows_per_seq=rows_per_seq)
    return out.cpu().tolist()


def test_filtered_draws_match_reference_distributions(golden):
    """The four golden rows: the reference's filtered probabilities (captured from its own
    sample_next) at 24 uniforms each, and its greedy choice with the penalty."""
    G = golden
    prev = G["sampler.prev"].tolist()
    logits = G["sampler.logits"]
    us = [(i + 0.5) / 24 for i in range(24)]
    checked = 0
    for i, (t, tk, tp, rp) in enumerate(G["sampler.params"].tolist()):
        row = logits[i:i + 1].repeat(len(us), 1)
        got = draw(row, t, int(tk), tp, rp, hist_rows=[prev] * len(us), u=us)
        want_p = G["sampler.probs"][i]
        for u, g in zip(us, got):
            if S.cdf_margin(want_p, u) < 1e-5:
                continue
            assert g == S.inverse_cdf(want_p, u), (i, u)
            checked += 1
        greedy = draw(logits[i:i + 1], 0.0, 0, 1.0, rp, hist_rows=[prev])
        assert greedy[0] == int(G["sampler.greedy"][i])
    assert checked > 60


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("params", [(0.7, 20, 0.8, 1.1), (1.0, 0, 0.9, 1.0), (0.5, 50, 1.0, 1.0),
                                    (1.3, 0, 1.0, 1.3), (0.8, 1, 0.5, 1.0)])
def test_filtered_draws_match_oracle_large_vocab(dt, params):
    """Rows of a 2-sequence x 3-position step over V = 32768: each row's penalty context is the
    sequence's history plus the step tokens before its position."""
    t, tk, tp, rp = params
    g = torch.Generator().manual_seed(7)
    B, R, V = 2, 3, 32768
    logits = (torch.randn(B * R, V, generator=g) * 3).to(dt)
    hist = [torch.randint(0, V, (40,), generator=g).tolist(), torch.randint(0, 200, (25,), generator=g).tolist()]
    step = torch.randint(0, V, (B, R), generator=g)
    us = torch.rand(B * R, generator=g).tolist()
    got = draw(logits, t, tk, tp, rp, hist_rows=hist, step=step, step_base=1, rows_per_seq=R, u=us)
    for r in range(B * R):
        b, pos = divmod(r, R)
        ctx = hist[b] + step[b, :1 + pos].tolist()
        p = S.filtered_probs(logits[r], t, tk, tp, rp, ctx)
        if S.cdf_margin(p, us[r]) < 1e-5:
            continue
        assert got[r] == S.inverse_cdf(p, us[r]), (r, params)
        greedy = draw(logits[r:r + 1], 0.0, 0, 1.0, rp, hist_rows=[ctx])
        assert greedy[0] == S.sample_next(logits[r], 0.0, 0, 1.0, rp, ctx)


@pytest.mark.parametrize("temperature", [0.0, 0.8])
def test_filtered_speculative_sampler_matches_oracle(temperature):
    """p/q acceptance over the filtered target (B·(k+1) rows) and draft (B·k rows)
    distributions, penalty context = history + the step's tokens up to each position."""
    k = K()
    g = torch.Generator().manual_seed(11)
    B, kk, V = 4, 3, 4096
    tk, tp, rp = 40, 0.9, 1.2
    tl = torch.randn(B * (kk + 1), V, generator=g) * 2
    dlg = tl[[b * (kk + 1) + a for b in range(B) for a in range(kk)]] + 0.3 * torch.randn(B * kk, V, generator=g)
    hist = [torch.randint(0, V, (10 + b,), generator=g).tolist() for b in range(B)]
    pending = torch.randint(0, V, (B,), generator=g)
    drafts = torch.zeros(B, kk, dtype=torch.int64)
    for b in range(B):   # draft from the filtered q so some are accepted
        for a in range(kk):
            ctx = hist[b] + [int(pending[b])] + drafts[b, :a].tolist()
            q = S.filtered_probs(dlg[b * kk + a], max(temperature, 1.0), tk, tp, rp, ctx)
            drafts[b, a] = int(torch.multinomial(q, 1, generator=g))
    ids = torch.cat([pending[:, None], drafts], 1)
    ua = torch.rand(B, kk, generator=g)
    ur = torch.rand(B, generator=g)
    hist_t = torch.full((B, 16), -1, dtype=torch.int64)
    for b, h in enumerate(hist):
        hist_t[b, :len(h)] = torch.tensor(h)
    hist_n = torch.tensor([len(h) for h in hist], dtype=torch.int32)
    ids_d = ids.to(DEV).contiguous()
    hist_d, hist_n_d = hist_t.to(DEV), hist_n.to(DEV)
    sp = k.sample_params(temperature, tk, tp, rp, hist=hist_d, hist_n=hist_n_d, step_ids=ids_d, step_base=1)
    ws = torch.empty(k.filter_workspace_bytes(B * (2 * kk + 1), V), dtype=torch.uint8, device=DEV)
    acc = torch.zeros(B, dtype=torch.int32, device=DEV)
    nxt = torch.zeros(B, dtype=torch.int64, device=DEV)
    k.spec_sample_filtered(tl.to(DEV), dlg.to(DEV) if temperature > 0 else None, B, kk, sp, ids_d[:, 1:], kk + 1,
                           ua.to(DEV) if temperature > 0 else None, ur.to(DEV) if temperature > 0 else None,
                           acc, nxt, ws)
    acc, nxt = acc.cpu().tolist(), nxt.cpu().tolist()
    for b in range(B):
        ctxs = [hist[b] + ids[b, :1 + a].tolist() for a in range(kk + 1)]
        if temperature <= 0:
            am = [S.sample_next(tl[b * (kk + 1) + a], 0.0, 0, 1.0, rp, ctxs[a]) for a in range(kk + 1)]
            a_want = 0
            while a_want < kk and int(drafts[b, a_want]) == am[a_want]:
                a_want += 1
            assert acc[b] == a_want and nxt[b] == am[a_want], b
            continue
        p = torch.stack([S.filtered_probs(tl[b * (kk + 1) + a], temperature, tk, tp, rp, ctxs[a])
                         for a in range(kk + 1)])
        q = torch.stack([S.filtered_probs(dlg[b * kk + a], temperature, tk, tp, rp, ctxs[a]) for a in range(kk)])
        a_want, tok_want, margins = S.speculative_accept(p, q, drafts[b], ua[b], float(ur[b]))
        if min(margins) < 1e-5:
            continue   # a near-tie acceptance decision: fp32 rounding may flip it
        assert acc[b] == a_want, b
        w = torch.clamp(p[a_want] - q[a_want], min=0) if a_want < kk else p[kk]
        if S.cdf_margin(w, float(ur[b])) < 1e-5:
            continue
        assert nxt[b] == tok_want, b
