"""CPU restatement of token selection (test infrastructure only; see oracle/__init__.py).

* `filtered_probs` / `sample_next`: the reference sampler `src/generate.py:17-37`
  (repetition penalty → greedy argmax, or temperature → top-k → top-p → categorical). The
  reference draws with `torch.multinomial`; the CUDA library draws by inverse CDF from a
  caller-supplied uniform, so this restatement exposes the *distribution* (pinned against
  the reference's own, captured in tests/golden) and an inverse-CDF draw.
* `speculative_accept`: the lossless speculative-sampling rule the reference does NOT have
  (its `generate_mtp` accepts by exact match, `src/qwen3_5/mtp.py:144-162`). Restated from
  the published algorithm (Leviathan, Kalman & Matias 2023, "Fast Inference from
  Transformers via Speculative Decoding", Alg. 1; Chen et al. 2023): draft i is accepted
  when u_i < p_i(d_i)/q_i(d_i); at the first rejection the replacement is drawn from
  norm(max(0, p_i − q_i)); after k acceptances a bonus token is drawn from p_{k+1}. With
  temperature 0 (one-hot p and q) it reduces to the reference's exact-match rule.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


def penalize(logits, repetition_penalty, prev_ids):
    """generate.py:18-22: divide positive / multiply negative logits of seen tokens."""
    if repetition_penalty == 1.0 or not prev_ids:
        return logits
    idx = torch.tensor(sorted(set(prev_ids)), dtype=torch.long)
    out = logits.clone()
    s = out[idx]
    out[idx] = torch.where(s > 0, s / repetition_penalty, s * repetition_penalty)
    return out


def filtered_logits(logits, temperature, top_k, top_p):
    """generate.py:25-36 without the draw: temperature, then top-k (ties with the k-th value
    survive), then top-p (keep the shortest sorted prefix whose mass reaches top_p,
    including the token that crosses it)."""
    x = (logits / temperature).float()     # the reference divides in the logits' dtype
    if top_k and top_k > 0:
        kth = torch.topk(x, top_k).values[..., -1:]
        x = x.masked_fill(x < kth, float("-inf"))
    if top_p and 0.0 < top_p < 1.0:
        sv, si = torch.sort(x, descending=True)
        cum = torch.cumsum(torch.softmax(sv, dim=-1), dim=-1)
        drop = torch.zeros_like(cum, dtype=torch.bool)
        drop[..., 1:] = cum[..., :-1] > top_p
        sv = sv.masked_fill(drop, float("-inf"))
        x = torch.empty_like(x).scatter_(-1, si, sv)
    return x


def filtered_probs(logits, temperature, top_k=0, top_p=1.0, repetition_penalty=1.0, prev_ids=None):
    """The categorical distribution `sample_next` draws from (temperature > 0)."""
    x = penalize(logits, repetition_penalty, prev_ids)
    return torch.softmax(filtered_logits(x, temperature, top_k, top_p), dim=-1)


def inverse_cdf(weights, u):
    """Smallest index j with cumsum(weights)[j] > u·Σweights (weights ≥ 0, not normalised).
    Summation is sequential fp64 so the CPU answer is the exact-arithmetic one up to
    fp64 rounding; `cdf_margin` reports how close u sat to a bucket edge."""
    w = weights.double()
    c = torch.cumsum(w, dim=0)
    tgt = float(u) * float(c[-1])
    j = int(torch.searchsorted(c, torch.tensor([tgt], dtype=torch.float64), right=True)[0])
    j = min(j, w.numel() - 1)
    while j > 0 and w[j] == 0:           # never land on a zero-mass bucket
        j -= 1
    return j


def cdf_margin(weights, u):
    w = weights.double()
    c = torch.cumsum(w, dim=0)
    tot = float(c[-1])
    if tot <= 0:
        return 0.0
    return float(torch.min(torch.abs(c / tot - float(u))))


def sample_next(logits, temperature, top_k=0, top_p=1.0, repetition_penalty=1.0,
                prev_ids=None, u=None):
    """generate.py:17-37 with the categorical draw done by inverse CDF at uniform `u`."""
    x = penalize(logits, repetition_penalty, prev_ids)
    if temperature <= 0.0:
        return int(torch.argmax(x))
    return inverse_cdf(torch.softmax(filtered_logits(x, temperature, top_k, top_p), dim=-1), u)


def speculative_accept(p, q, drafts, u_accept, u_resample):
    """One sequence. p: (k+1, V) target probabilities (row i scores the token after input i);
    q: (k, V) draft probabilities; drafts: k ints; u_accept: k uniforms; u_resample: one
    uniform. Returns (n_accepted, next_token, margins) where margins[i] = |u_i·q − p| for
    every decision made (for near-tie flagging)."""
    k = len(drafts)
    margins = []
    for i in range(k):
        d = int(drafts[i])
        pd, qd = float(p[i, d]), float(q[i, d])
        margins.append(abs(float(u_accept[i]) * qd - pd))
        if float(u_accept[i]) * qd < pd:
            continue
        resid = torch.clamp(p[i].double() - q[i].double(), min=0.0)
        if float(resid.sum()) <= 0.0:         # p == q exactly: fall back to p
            resid = p[i].double()
        return i, inverse_cdf(resid, u_resample), margins
    return k, inverse_cdf(p[k].double(), u_resample), margins


def greedy_accept(target_argmax, drafts):
    """Exact-match acceptance (mtp.py:144-162 generalised to k drafts): accept while
    draft i equals argmax of row i; the next token is argmax of the first unmatched row."""
    k = len(drafts)
    for i in range(k):
        if int(drafts[i]) != int(target_argmax[i]):
            return i, int(target_argmax[i])
    return k, int(target_argmax[k])
