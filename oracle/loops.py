"""CPU restatement of the decode loops (test infrastructure only; see oracle/__init__.py).

* `greedy_generate`: `src/generate.py:41-62` at temperature 0, batched lock-step
  (equal-length prompts), no stop ids.
* `spec_generate`: `src/qwen3_5/mtp.py:92-162` generalised to a batch and to k drafts.
  The reference drafts one token; the k>1 chain is defined by this build (the reference
  does not define it): depth d feeds the MTP head the previous depth's PRE-norm MTP output
  as `hidden` and the previous depth's token as the next embedding, mirroring how the main
  model hands its pre-norm hidden to depth 1 (mtp.py:120,137). Verification feeds
  [pending, d_1..d_k] (T = k+1); acceptance is exact match at temperature 0 (the
  reference's rule) or the lossless p/q rule otherwise (`sampling.speculative_accept`).
  Rollback restores the pre-verify snapshot and re-runs the a+1 kept tokens, exactly the
  reference's recovery (mtp.py:141, 156-162).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from . import qwen35 as Q
from . import sampling as S


def prefill(P, cfg, prompts, scan="reference"):
    logits, cache, hidden = Q.model_forward(P, cfg, prompts, None, scan)
    return logits, cache, hidden


def greedy_generate(P, cfg, prompts, n_new, scan="reference", repetition_penalty=1.0):
    """Returns (B, n_new) generated ids at temperature 0. With a repetition penalty each
    pick is `sample_next`'s penalised argmax over the sequence's context so far
    (src/generate.py:17-27, 52-61)."""
    ctx = [row.tolist() for row in prompts]

    def pick(lg):
        if repetition_penalty == 1.0:
            return lg.float().argmax(-1)
        return torch.tensor([S.sample_next(lg[b].float(), 0.0, 0, 1.0, repetition_penalty, ctx[b])
                             for b in range(lg.shape[0])])

    logits, cache, _ = prefill(P, cfg, prompts, scan)
    nxt = pick(logits[:, -1])
    out = []
    for _ in range(n_new):
        out.append(nxt)
        for b in range(len(ctx)):
            ctx[b].append(int(nxt[b]))
        logits, cache, _ = Q.model_forward(P, cfg, nxt[:, None], cache, scan)
        nxt = pick(logits[:, -1])
    return torch.stack(out, dim=1)


def draft_chain(P, cfg, hidden_last, pending, k, temperature=0.0, u_draft=None,
                top_k=0, top_p=1.0):
    """k MTP drafts per sequence. hidden_last: (B,H) pre-norm main hidden; pending: (B,).
    Returns (drafts (B,k) int64, q (B,k,V) fp32 draft probabilities or None if greedy)."""
    B = pending.shape[0]
    h, tok = hidden_last[:, None], pending
    drafts, qs = [], []
    for d in range(k):
        emb = F.embedding(tok[:, None], P["model.embed_tokens.weight"])
        post, pre = Q.mtp_forward(P, cfg, h, emb)
        logits = Q.lm_head(P, post)[:, 0].float()
        if temperature <= 0:
            tok = logits.argmax(-1)
        else:
            q = S.filtered_probs(logits, temperature, top_k, top_p)
            qs.append(q)
            tok = torch.tensor([S.inverse_cdf(q[b], u_draft[b, d]) for b in range(B)])
        drafts.append(tok)
        h = pre
    return torch.stack(drafts, 1), (torch.stack(qs, 1) if qs else None)


def spec_step(P, cfg, cache, hidden_last, pending, k, temperature=0.0, uniforms=None,
              top_k=0, top_p=1.0, scan="reference"):
    """One speculative step for a batch. uniforms: dict with 'draft' (B,k), 'accept' (B,k),
    'resample' (B,) when temperature > 0. Returns (cache, hidden_last, pending,
    committed list-of-lists, n_accepted (B,), margins list-of-lists)."""
    B = pending.shape[0]
    drafts, q = draft_chain(P, cfg, hidden_last, pending, k, temperature,
                            None if uniforms is None else uniforms["draft"], top_k, top_p)
    ids = torch.cat([pending[:, None], drafts], dim=1)                 # (B, k+1)
    snap = cache.clone()
    logits, cache_v, hidden = Q.model_forward(P, cfg, ids, cache, scan)
    acc, nxt, margins = [], [], []
    for b in range(B):
        if temperature <= 0:
            a, t = S.greedy_accept(logits[b].float().argmax(-1), drafts[b])
            m = []
        else:
            p = S.filtered_probs(logits[b].float(), temperature, top_k, top_p)
            a, t, m = S.speculative_accept(p, q[b], drafts[b], uniforms["accept"][b],
                                           uniforms["resample"][b])
        acc.append(a)
        nxt.append(t)
        margins.append(m)
    committed = [ids[b, :acc[b] + 1].tolist() for b in range(B)]
    if all(a == k for a in acc):
        new_cache, new_hidden = cache_v, hidden[:, k]
    else:
        # restore + recompute exactly the kept tokens, one sequence at a time (ragged)
        new_cache = snap
        hs = []
        per_seq = []
        for b in range(B):
            sub = _select(snap, b)
            _, sub, hb = Q.model_forward(P, cfg, ids[b:b + 1, :acc[b] + 1], sub, scan)
            per_seq.append(sub)
            hs.append(hb[0, -1])
        new_cache = _merge(per_seq, cfg.num_hidden_layers)
        new_hidden = torch.stack(hs)
    return (new_cache, new_hidden, torch.tensor(nxt), committed,
            torch.tensor(acc), margins)


def _select(cache, b):
    c = Q.OracleCache(cache.n_layers)
    c.kv = {l: [(s[b][0].clone(), s[b][1].clone())] for l, s in cache.kv.items()}
    c.gdn = {l: (cv[b:b + 1].clone(), rc[b:b + 1].clone()) for l, (cv, rc) in cache.gdn.items()}
    c.lens = [cache.lens[b]]
    return c


def _merge(caches, n_layers):
    c = Q.OracleCache(n_layers)
    c.kv = {l: [cc.kv[l][0] for cc in caches] for l in caches[0].kv}
    c.gdn = {l: (torch.cat([cc.gdn[l][0] for cc in caches]), torch.cat([cc.gdn[l][1] for cc in caches]))
             for l in caches[0].gdn}
    c.lens = [cc.lens[0] for cc in caches]
    return c


def spec_generate(P, cfg, prompts, n_new, k, temperature=0.0, uniform_stream=None,
                  top_k=0, top_p=1.0, scan="reference"):
    """Batched speculative generation. Returns (list of per-seq generated ids (≥ n_new,
    truncated to n_new), per-step accepted counts). `uniform_stream(step)` → uniforms dict."""
    logits, cache, hidden = prefill(P, cfg, prompts, scan)
    B = prompts.shape[0]
    if temperature <= 0:
        pending = logits[:, -1].float().argmax(-1)
    else:
        u0 = uniform_stream(-1)["resample"]
        pend = [S.inverse_cdf(S.filtered_probs(logits[b, -1].float(), temperature, top_k, top_p), u0[b])
                for b in range(B)]
        pending = torch.tensor(pend)
    hidden_last = hidden[:, -1]
    out = [[] for _ in range(B)]
    accepts = []
    step = 0
    while min(len(o) for o in out) < n_new:
        u = None if temperature <= 0 else uniform_stream(step)
        cache, hidden_last, pending, committed, acc, _ = spec_step(
            P, cfg, cache, hidden_last, pending, k, temperature, u, top_k, top_p, scan)
        for b in range(B):
            out[b].extend(committed[b])
        accepts.append(acc)
        step += 1
    return [o[:n_new] for o in out], accepts
