"""The shared generation loop and sampler (src/generate.py:17-62) on the qsp kernels.

`generate` keeps the reference signature and its prefill → decode → stop structure; the
model is any family model with `forward(ids, past) -> (logits, past)`. `sample_next` keeps
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


@torch.no_grad()
def generate(model, ids, decode, stop_ids, device, *, max_new_tokens=128, temperature=0.7,
             top_k=20, top_p=0.8, repetition_penalty=1.1):
    """`decode(list[int]) -> str`. Yields incremental text pieces (generate.py:41-62)."""
    input_ids = torch.tensor([ids], device=device)
    context = list(ids)
    eos = set(stop_ids)
    logits, past = model(input_ids)
    nxt = sample_next(logits[0, -1], temperature, top_k, top_p, repetition_penalty, context)
    generated, prev = [], ""
    for _ in range(max_new_tokens):
        if nxt in eos:
            break
        generated.append(nxt)
        context.append(nxt)
        text = decode(generated)
        if len(text) > len(prev):
            yield text[len(prev):]
            prev = text
        logits, past = model(torch.tensor([[nxt]], device=device), past)
        nxt = sample_next(logits[0, -1], temperature, top_k, top_p, repetition_penalty, context)
