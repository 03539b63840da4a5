"""MTP draft head and the batched speculative decoder.

MTP forward (src/qwen3_5/mtp.py:61-73):
    x = fc([RMSNorm_e(emb(tok)) ; RMSNorm_h(hidden)]) → one full-attention DecoderLayer with no
    cache → RMSNorm → shared lm_head.
With one position and no cache the attention softmax runs over a single key, so its output
is exactly v and the q/k projections, QK-norm and RoPE cannot affect the result; the head
therefore projects only the output-gate half of q_proj and v_proj
(`qsp_mtp_single_token_attn`). Same values, ~half the attention weight reads.

Draft chain for k > 1 (not defined by the reference, which drafts one token): depth d feeds
the head the PRE-norm output of depth d−1 as `hidden` and the token drafted at depth d−1 as
the next embedding, the same pairing the main model uses for depth 1 (mtp.py:120,137).

SpecDecoder is `generate_mtp` (mtp.py:92-162) generalised to a batch of independent
sequences and k drafts: draft k tokens → verify [pending, d1..dk] in one forward with the
GDN updates left pending → accept (exact match at temperature 0, the reference's rule; the
lossless p/q rule otherwise) → keep a prefix by index (no snapshot, no recompute) → emit
pending + accepted drafts. Everything stays on the device, so `step()` can be captured in a
CUDA graph and replayed with no host synchronisation.
"""

from __future__ import annotations

import torch

from .. import kernels as K
from .modeling_qwen3_5 import Qwen3_5Model
from .moe import SparseMoeBlock


class MTP:
    def __init__(self, model: Qwen3_5Model, params: dict):
        cfg, dt, dev = model.cfg, model.dtype, model.device
        self.model, self.cfg = model, cfg
        g = lambda n: params[n].to(device=dev, dtype=dt).contiguous()
        H, nh, nkv, hd = cfg.hidden_size, cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
        self.norm_e = g("mtp.pre_fc_norm_embedding.weight")
        self.norm_h = g("mtp.pre_fc_norm_hidden.weight")
        self.fc = g("mtp.fc.weight")
        p = "mtp.layers.0."
        self.in_norm = g(p + "input_layernorm.weight")
        self.post_norm = g(p + "post_attention_layernorm.weight")
        q = g(p + "self_attn.q_proj.weight").view(nh, 2, hd, H)
        self.w_gv = torch.cat([q[:, 1].reshape(nh * hd, H), g(p + "self_attn.v_proj.weight")]).contiguous()
        self.o_proj = g(p + "self_attn.o_proj.weight")
        # the MoE family's MTP block takes the FFN kind of layer 0 (qwen3_5_moe/mtp.py:34-36)
        self.moe = SparseMoeBlock(cfg, params, p, dtype=dt, device=dev) if cfg.is_moe_layer(0) else None
        if self.moe is None:
            self.w_gu = torch.cat([g(p + "mlp.gate_proj.weight"), g(p + "mlp.up_proj.weight")]).contiguous()
            self.down = g(p + "mlp.down_proj.weight")
        self.norm = g("mtp.norm.weight")
        self._ws = {}

    def workspace(self, B: int, k: int):
        if (B, k) not in self._ws:
            cfg, dt, dev = self.cfg, self.model.dtype, self.model.device
            H, nh, nkv, hd = cfg.hidden_size, cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
            e = lambda *s: torch.empty(*s, dtype=dt, device=dev)
            I = 1 if self.moe is not None else self.down.shape[1]
            self._ws[(B, k)] = dict(emb=e(B, H), cat=e(B, 2 * H), x=e(B, H), xn=e(B, H),
                                    gv=e(B, (nh + nkv) * hd), ao=e(B, nh * hd), gu=e(B, 2 * I),
                                    act=e(B, I), logits=e(B, k, cfg.vocab_size))
            if self.moe is not None:
                self._ws[(B, k)]["moe_ws"] = torch.empty(self.moe.workspace_bytes(B), dtype=torch.uint8, device=dev)
        return self._ws[(B, k)]

    @torch.no_grad()
    def draft(self, hidden_last: torch.Tensor, ids: torch.Tensor, k: int, temperature: float = 0.0,
              u_draft: torch.Tensor | None = None, filtered=None):
        """Fill ids[:, 1..k] with k drafted tokens, given ids[:, 0] (the pending token) and the
        main model's pre-norm hidden at the last kept position. Returns the [B, k, V] draft
        logits buffer (row d = the head's logits at depth d). `filtered(d, logits_d)`, when
        given, draws depth d's token with the sampling filters (stochastic drafts)."""
        cfg, m = self.cfg, self.model
        B = ids.shape[0]
        H, nh, nkv, hd = cfg.hidden_size, cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
        w = self.workspace(B, k)
        eps = cfg.rms_norm_eps
        h = hidden_last
        for d in range(k):
            K.embed(ids[:, d:], m.embed, w["emb"], ids_stride=k + 1, rows=B)
            K.rmsnorm(w["emb"], self.norm_e, w["cat"][:, :H], eps)
            K.rmsnorm(h, self.norm_h, w["cat"][:, H:], eps)
            K.gemm(w["cat"], self.fc, w["x"])
            K.rmsnorm(w["x"], self.in_norm, w["xn"], eps)
            K.gemm(w["xn"], self.w_gv, w["gv"])
            K.mtp_single_token_attn(w["gv"], hd, w["gv"][:, nh * hd:], w["ao"], nh, nkv, hd)
            K.gemm_residual_rmsnorm(w["ao"], self.o_proj, w["x"], self.post_norm, w["xn"], eps)
            # x stays the pre-norm output (next depth's hidden); xn = final norm for lm_head
            if self.moe is not None:
                self.moe(w["xn"], w["x"], self.norm, w["xn"], eps, B, w["moe_ws"])
            else:
                K.gemm_swiglu(w["xn"], self.w_gu, w["act"], w["gu"])
                K.gemm_residual_rmsnorm(w["act"], self.down, w["x"], self.norm, w["xn"], eps)
            lg = w["logits"][:, d]
            K.gemm(w["xn"], m.lm_head, lg)
            if temperature <= 0:
                K.argmax_rows(lg, ids[:, d + 1:], rows=B, out_stride=k + 1)
            elif filtered is not None:
                filtered(d, lg)
            else:
                K.sample_rows(lg, temperature, u_draft[:, d].contiguous() if u_draft.stride(0) != 1 else u_draft[:, d],
                              ids[:, d + 1:], self._sel_ws(B), rows=B, out_stride=k + 1)
            h = w["x"]
        return w["logits"]

    def _sel_ws(self, B):
        key = ("sel", B)
        if key not in self._ws:
            self._ws[key] = torch.empty(2 * B + 16, dtype=torch.float32, device=self.model.device)
        return self._ws[key]


class SpecDecoder:
    """Batched k-deep speculative decoding over independent sequences on one GPU."""

    def __init__(self, model: Qwen3_5Model, mtp: MTP, batch: int, k: int, max_len: int, *,
                 temperature: float = 0.0, top_k: int = 0, top_p: float = 1.0,
                 repetition_penalty: float = 1.0, out_capacity: int | None = None, **cache_kw):
        self.model, self.mtp, self.B, self.k = model, mtp, batch, k
        self.T = k + 1
        self.temperature = float(temperature)
        self.top_k, self.top_p, self.rep = int(top_k or 0), float(top_p if top_p is not None else 1.0), float(repetition_penalty)
        # sample_next's filters (generate.py:17-37): the penalty context of a scored position
        # is the sequence's prompt + committed tokens (`out`) plus the step's tokens before it
        self.filtered = self.rep != 1.0 or self.top_k > 0 or 0.0 < self.top_p < 1.0
        dev = model.device
        self.cache = model.new_cache(batch, max_len, max_spec_tokens=max(self.T, 2), **cache_kw)
        self.ids = torch.zeros(batch, self.T, dtype=torch.int64, device=dev)
        self.hidden_last = torch.zeros(batch, model.cfg.hidden_size, dtype=model.dtype, device=dev)
        self.accept_n = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.next_tok = torch.zeros(batch, dtype=torch.int64, device=dev)
        self.amax = torch.zeros(batch * self.T, dtype=torch.int64, device=dev)
        self.cap = out_capacity or max_len
        self.prompt_len = 0
        self.out = torch.zeros(batch, self.cap, dtype=torch.int64, device=dev)   # prompt + committed
        self.n_out = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.sel_ws = torch.empty(4 * batch * self.T + 64, dtype=torch.float32, device=dev)
        self.filt_ws = None
        if self.filtered:
            V = model.cfg.vocab_size
            self.filt_ws = torch.empty(K.filter_workspace_bytes(batch * (2 * k + 1), V), dtype=torch.uint8, device=dev)
        self.u = None            # uniforms for stochastic steps: dict of device tensors
        self.graph = None

    # ------------------------------------------------------------------ prefill
    @torch.no_grad()
    def prefill(self, prompts: torch.Tensor, chunk: int = 64, u_first: torch.Tensor | None = None):
        """Run the prompts (B, P) through the model in commit-all chunks; set the pending
        token (argmax, or a draw at u_first when temperature > 0) and the MTP hidden."""
        B, P = prompts.shape
        assert B == self.B
        prompts = prompts.to(self.model.device).contiguous()
        for s in range(0, P, chunk):
            lrow, hid = self.model.prefill_last(prompts[:, s:s + chunk], self.cache)
        # the output rows start with the prompt (the repetition-penalty context)
        self.prompt_len = P
        self.out = torch.zeros(B, P + self.cap, dtype=torch.int64, device=self.model.device)
        self.out[:, :P] = prompts
        self.n_out.fill_(P)
        if self.filtered:
            sp = self._params(None, 0)
            K.sample_filtered(lrow, sp, u_first, self.ids, self.filt_ws, rows=B, out_stride=self.T)
        elif self.temperature <= 0:
            K.argmax_rows(lrow, self.ids, rows=B, out_stride=self.T)
        else:
            K.sample_rows(lrow, self.temperature, u_first, self.ids, self.sel_ws, rows=B, out_stride=self.T)
        self.hidden_last.copy_(hid)

    def _params(self, step_ids, step_base):
        return K.sample_params(self.temperature, self.top_k, self.top_p, self.rep, hist=self.out,
                               hist_n=self.n_out, step_ids=step_ids, step_base=step_base)

    # ------------------------------------------------------------------ one step
    @torch.no_grad()
    def step(self):
        m, B, T, k = self.model, self.B, self.T, self.k
        stochastic = self.temperature > 0
        filt = None
        if self.filtered and stochastic:
            def filt(d, lg):   # depth d predicts token d+1 after [pending, d1..dd]
                K.sample_filtered(lg, self._params(self.ids, d + 1), self.u["draft"][:, d].contiguous(),
                                  self.ids[:, d + 1:], self.filt_ws, rows=B, out_stride=k + 1)
        dl = self.mtp.draft(self.hidden_last, self.ids, k, self.temperature,
                            self.u["draft"] if stochastic else None, filtered=filt)
        ws = m._forward_into(self.ids, self.cache, B, T, True)
        if self.filtered:
            K.spec_sample_filtered(ws.logits, dl.view(B * k, -1) if stochastic else None, B, k,
                                   self._params(self.ids, 1), self.ids[:, 1:], T,
                                   self.u["accept"] if stochastic else None,
                                   self.u["resample"] if stochastic else None,
                                   self.accept_n, self.next_tok, self.filt_ws)
        elif not stochastic:
            K.greedy_verify(ws.logits, B, T, self.ids[:, 1:], T, self.accept_n, self.next_tok, self.amax)
        else:
            K.spec_sample(ws.logits, dl.view(B * k, -1), B, k, self.temperature, self.ids[:, 1:], T,
                          self.u["accept"], self.u["resample"], self.accept_n, self.next_tok, self.sel_ws)
        self.cache.accept(self.accept_n)
        K.select_rows(ws.x, B, T, self.accept_n, self.hidden_last)
        K.commit_tokens(B, T, self.ids, self.accept_n, self.next_tok, self.out, self.n_out)

    def capture(self, warmup: int = 2):
        """Record step() into a CUDA graph (after `warmup` eager steps on a side stream)."""
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(warmup):
                self.step()
        torch.cuda.current_stream().wait_stream(s)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.step()
        return self.graph

    def replay(self):
        if self.graph is None:
            self.step()
        else:
            self.graph.replay()

    def outputs(self):
        """The committed tokens of every sequence (after its prompt)."""
        n = self.n_out.tolist()
        o = self.out.cpu()
        P = self.prompt_len
        return [o[b, P:min(n[b], P + self.cap)].tolist() for b in range(self.B)]


@torch.no_grad()
def generate_mtp(model: Qwen3_5Model, mtp: MTP, ids, decode, stop_ids, device=None, *,
                 max_new_tokens=128, temperature=0.7, top_k=20, top_p=0.8,
                 repetition_penalty=1.1, k: int = 1, seed: int = 0):
    """Drop-in for the reference generator (mtp.py:92-162), same defaults: yields text pieces
    of one sequence. Greedy (temperature <= 0) output equals `generate()` with the same
    repetition penalty. temperature > 0 uses the lossless p/q sampler over the filtered
    target and draft distributions (penalty → temperature → top-k → top-p, as sample_next),
    with uniforms from a seeded device generator."""
    eos = set(stop_ids)
    prompt = torch.tensor([list(ids)], dtype=torch.int64, device=model.device)
    dec = SpecDecoder(model, mtp, 1, k, prompt.shape[1] + max_new_tokens + k + 2,
                      temperature=temperature, top_k=top_k, top_p=top_p,
                      repetition_penalty=repetition_penalty, out_capacity=max_new_tokens + k + 1)
    gen = torch.Generator(device=model.device)
    gen.manual_seed(seed)
    rand = lambda *s: torch.rand(*s, generator=gen, device=model.device)
    if temperature > 0:
        dec.u = {"draft": rand(1, k), "accept": rand(1, k), "resample": rand(1)}
    dec.prefill(prompt, u_first=rand(1) if temperature > 0 else None)
    generated, prev, emitted = [], "", 0
    while emitted < max_new_tokens:
        if temperature > 0:
            for key, t in dec.u.items():
                t.copy_(rand(*t.shape))
        dec.step()
        toks = dec.outputs()[0]
        for t in toks[emitted:]:
            if t in eos or emitted >= max_new_tokens:
                return
            generated.append(t)
            emitted += 1
            text = decode(generated)
            if len(text) > len(prev):
                yield text[len(prev):]
                prev = text
