"""The shared generation loop and sampler (src/generate.py:17-62) on the qsp kernels.

`generate` keeps the reference signature and output; the model is any family model with
`forward(ids, past) -> (logits, past)`, and the loop keeps its token state on the device
(`_TokenLoop`). `sample_next` keeps
the reference signature and semantics: repetition penalty over `prev_ids`, then argmax
(temperature <= 0) or temperature → top-k → top-p → a categorical draw, by inverse CDF at a
uniform from a seeded device generator (the reference uses torch.multinomial over the same
distribution). Without any filter the plain argmax / softmax kernels run.
"""

from __future__ import annotations

import torch

from . import kernels as K

_gen = {}


def _uniform(device, seed=0):
    if device not in _gen:
        g = torch.Generator(device=device)
        g.manual_seed(seed)
        _gen[device] = g
    return torch.rand(1, generator=_gen[device], device=device)


def sample_next(logits, temperature, top_k, top_p, repetition_penalty=1.0, prev_ids=None):
    row = logits.reshape(1, -1).contiguous()
    dev = row.device
    out = torch.empty(1, dtype=torch.int64, device=dev)
    filtered = ((repetition_penalty != 1.0 and prev_ids) or (top_k and top_k > 0)
                or (top_p is not None and 0.0 < top_p < 1.0))
    if not filtered:
        if temperature <= 0.0:
            K.argmax_rows(row, out)
        else:
            ws = torch.empty(16, dtype=torch.float32, device=dev)
            K.sample_rows(row, temperature, _uniform(dev), out, ws)
        return int(out.item())
    hist = hist_n = None
    if repetition_penalty != 1.0 and prev_ids:
        hist = torch.tensor([list(prev_ids)], dtype=torch.int64, device=dev)
        hist_n = torch.tensor([hist.shape[1]], dtype=torch.int32, device=dev)
    sp = K.sample_params(temperature, top_k, top_p, repetition_penalty, hist=hist, hist_n=hist_n)
    ws = torch.empty(K.filter_workspace_bytes(1, row.shape[1]), dtype=torch.uint8, device=dev)
    K.sample_filtered(row, sp, _uniform(dev) if temperature > 0 else None, out, ws)
    return int(out.item())


class _TokenLoop:
    """Device-resident state of one sequence's autoregressive loop: the next forward's (1, 1)
    input, the sequence's token history (prompt + generated, the repetition-penalty context)
    grown in place by `qsp_commit_tokens`, the sampler's filter parameters over that history,
    and a pinned host slot through which the host reads each token."""

    def __init__(self, prompt, max_new, vocab, device, temperature, top_k, top_p, repetition_penalty):
        dev = torch.device(device)
        n = len(prompt)
        self.temperature = float(temperature)
        self.tok = torch.zeros(1, 1, dtype=torch.int64, device=dev)
        self.hist = torch.zeros(1, n + max_new + 1, dtype=torch.int64, device=dev)
        self.hist[0, :n] = torch.tensor(prompt, dtype=torch.int64, device=dev)
        self.hist_n = torch.tensor([n], dtype=torch.int32, device=dev)
        self.keep0 = torch.zeros(1, dtype=torch.int32, device=dev)
        self.host = torch.empty(1, dtype=torch.int64, pin_memory=dev.type == "cuda")
        self.filtered = ((repetition_penalty != 1.0 and n > 0) or (top_k and top_k > 0)
                         or (top_p is not None and 0.0 < top_p < 1.0))
        if self.filtered:
            use_hist = repetition_penalty != 1.0
            self.params = K.sample_params(temperature, top_k, top_p, repetition_penalty,
                                          hist=self.hist if use_hist else None,
                                          hist_n=self.hist_n if use_hist else None)
            self.ws = torch.empty(K.filter_workspace_bytes(1, vocab), dtype=torch.uint8, device=dev)
        elif self.temperature > 0:
            self.ws = torch.empty(16, dtype=torch.float32, device=dev)

    def pick(self, row):
        """Sample the next token from a (1, V) logits row into `tok`, append it to the history,
        and return it on the host."""
        u = _uniform(row.device) if self.temperature > 0 else None
        flat = self.tok.view(1)
        if self.filtered:
            K.sample_filtered(row, self.params, u, flat, self.ws)
        elif u is None:
            K.argmax_rows(row, flat)
        else:
            K.sample_rows(row, self.temperature, u, flat, self.ws)
        # history[n] = tok, n += 1 (a keep-one commit whose next pending token is tok itself)
        K.commit_tokens(1, 1, flat, self.keep0, flat, self.hist, self.hist_n)
        self.host.copy_(flat, non_blocking=True)
        torch.cuda.current_stream(row.device).synchronize()
        return int(self.host[0])


@torch.no_grad()
def generate(model, ids, decode, stop_ids, device, *, max_new_tokens=128, temperature=0.7,
             top_k=20, top_p=0.8, repetition_penalty=1.1):
    """Drop-in for the reference's `generate` (src/generate.py:41-62): same signature, same
    defaults and the same output — prefill, then one token per forward until `stop_ids` or
    `max_new_tokens`, yielding the newly decoded text after each token (`decode(list[int])
    -> str`). The sampled token never leaves the device on its way into the next forward
    and the penalty context lives on the device; the host reads one token per step to
    decide on stopping and to decode."""
    prompt = list(ids)
    loop = _TokenLoop(prompt, max_new_tokens, model.cfg.vocab_size, device, temperature, top_k, top_p,
                      repetition_penalty)
    logits, past = model(torch.tensor([prompt], device=device))
    eos = set(stop_ids)
    out, shown = [], 0
    while len(out) < max_new_tokens:
        t = loop.pick(logits[0, -1:])
        if t in eos:
            return
        out.append(t)
        text = decode(out)
        if len(text) > shown:
            yield text[shown:]
            shown = len(text)
        if len(out) < max_new_tokens:
            logits, past = model(loop.tok, past)
