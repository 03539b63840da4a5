"""The shared generation loop and sampler (src/generate.py:17-62) on the qsp kernels.

`generate` keeps the reference signature and its prefill → decode → stop structure; the
model is any family model with `forward(ids, past) -> (logits, past)`. `sample_next` keeps
the reference signature. Greedy (temperature <= 0, repetition penalty 1) runs the argmax
kernel; temperature > 0 draws by inverse CDF from softmax(logits/τ) with a uniform from a
seeded device generator. top-k, top-p and repetition penalty are rejected rather than
silently ignored (not built into the fused sampler).
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
    if repetition_penalty != 1.0 and prev_ids:
        raise NotImplementedError("sample_next: repetition_penalty is not supported by the qsp sampler")
    if (top_k and top_k > 0) or (top_p and 0.0 < top_p < 1.0):
        raise NotImplementedError("sample_next: top_k/top_p are not supported by the qsp sampler")
    row = logits.reshape(1, -1).contiguous()
    out = torch.empty(1, dtype=torch.int64, device=row.device)
    if temperature <= 0.0:
        K.argmax_rows(row, out)
    else:
        ws = torch.empty(16, dtype=torch.float32, device=row.device)
        K.sample_rows(row, temperature, _uniform(row.device), out, ws)
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
