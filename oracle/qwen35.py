"""CPU restatement of the qwen3_5 decoder (test infrastructure only; see oracle/__init__.py).

Every op keeps the reference's rounding points so that, in bf16, it lands on the same
values the reference produces (the casts `.to(dtype)` below sit where the reference's do).
Weights come as a {canonical_name: tensor} dict (`lollm_b200.qwen3_5.weights.load_checkpoint`).

The cache here is deliberately simple — per-sequence Python lists — so that ragged lengths
(which the reference's scalar `seen_tokens`, `src/qwen3_5/kv.py:23`, cannot express) are
handled one sequence at a time. For equal lengths it is the reference cache's semantics.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F


# ─────────────────────────────── primitives ───────────────────────────────

def rms_norm(x, w, eps):
    """(1+w)·x̂ with the statistics in fp32 — src/qwen3_5/blocks.py:31-35."""
    dt = x.dtype
    xf = x.float()
    inv = torch.rsqrt(xf.square().mean(-1, keepdim=True) + eps)
    return ((xf * inv) * (w.float() + 1.0)).to(dt)


def rms_norm_gated(x, z, w, eps):
    """w·x̂ (x̂ cast back to the input dtype first) · silu(z in fp32) — blocks.py:46-51."""
    dt = x.dtype
    xf = x.float()
    xn = (xf * torch.rsqrt(xf.square().mean(-1, keepdim=True) + eps)).to(dt)
    return ((w * xn) * F.silu(z.float())).to(dt)


def l2_normalize(x, eps=1e-6):
    """x / sqrt(Σx² + eps) over the last dim, in the tensor's own dtype — blocks.py:54-56."""
    return x * torch.rsqrt(x.square().sum(-1, keepdim=True) + eps)


def linear(x, w):
    return F.linear(x, w)


def silu_mul(g, u):
    return F.silu(g) * u


# ───────────────────────────── delta rule (GDN) ─────────────────────────────

def delta_rule_recurrent(q, k, v, g, beta, state):
    """Token-by-token gated delta rule — blocks.py:116-144 (the exact definition).

    q,k,v: (B,T,H,d) already l2-normalised (q not yet scaled); g, beta: (B,T,H);
    state: (B,H,dk,dv) fp32 or None. Returns (out (B,T,H,dv) in q.dtype, state fp32).
    """
    dt = q.dtype
    qf, kf, vf = (t.float().transpose(1, 2) for t in (q, k, v))       # (B,H,T,d)
    gf, bf = g.float().transpose(1, 2), beta.float().transpose(1, 2)   # (B,H,T)
    B, H, T, dk = kf.shape
    dv = vf.shape[-1]
    qf = qf * (dk ** -0.5)
    S = (torch.zeros(B, H, dk, dv) if state is None else state.float().clone())
    outs = []
    for t in range(T):
        S = S * gf[:, :, t].exp()[..., None, None]
        pred = torch.einsum("bhkv,bhk->bhv", S, kf[:, :, t])
        delta = (vf[:, :, t] - pred) * bf[:, :, t][..., None]
        S = S + kf[:, :, t][..., :, None] * delta[..., None, :]
        outs.append(torch.einsum("bhkv,bhk->bhv", S, qf[:, :, t]))
    out = torch.stack(outs, dim=2).transpose(1, 2).contiguous().to(dt)
    return out, S


def delta_rule_chunked(q, k, v, g, beta, state, chunk=64):
    """Chunk-parallel form of the same recurrence — what the reference runs for T>1
    (blocks.py:59-113, dispatched at blocks.py:316-322).

    Derivation used here (own formulation, same math): inside a chunk with cumulative
    log-decay G_i, the per-position corrections δ_i = β_i(v_i − e^{G_i}S0ᵀk_i −
    Σ_{j<i} e^{G_i−G_j}(k_i·k_j)δ_j) solve a unit lower-triangular system; outputs are
    e^{G_i}S0ᵀq_i + Σ_{j≤i} e^{G_i−G_j}(q_i·k_j)δ_j and the carried state is
    e^{G_C}S0 + Σ_j e^{G_C−G_j} k_j δ_jᵀ. Zero-padding to the chunk size is unnecessary
    (padded positions would leave the state unchanged), so the last chunk is ragged.
    """
    dt = q.dtype
    qf, kf, vf = (t.float().transpose(1, 2) for t in (q, k, v))
    gf, bf = g.float().transpose(1, 2), beta.float().transpose(1, 2)
    B, H, T, dk = kf.shape
    dv = vf.shape[-1]
    qf = qf * (dk ** -0.5)
    S = (torch.zeros(B, H, dk, dv) if state is None else state.float().clone())
    outs = []
    for s in range(0, T, chunk):
        e = min(s + chunk, T)
        qc, kc, vc = qf[:, :, s:e], kf[:, :, s:e], vf[:, :, s:e]
        G = gf[:, :, s:e].cumsum(-1)                                   # (B,H,C)
        bc = bf[:, :, s:e]
        C = e - s
        rel = G[..., :, None] - G[..., None, :]                         # G_i − G_j
        lower = torch.tril(torch.ones(C, C, dtype=torch.bool), -1)
        lower_eq = torch.tril(torch.ones(C, C, dtype=torch.bool), 0)
        decay = torch.where(lower_eq, rel, torch.full_like(rel, -math.inf)).exp()
        kk = kc @ kc.transpose(-1, -2)
        Lmat = torch.where(lower, bc[..., :, None] * decay * kk, torch.zeros_like(kk))
        rhs = bc[..., None] * (vc - G.exp()[..., None] * (kc @ S))    # (B,H,C,dv)
        eye = torch.eye(C).expand_as(Lmat)
        delta = torch.linalg.solve_triangular(eye + Lmat, rhs, upper=False, unitriangular=True)
        qk = torch.where(lower_eq, (qc @ kc.transpose(-1, -2)) * decay, torch.zeros_like(kk))
        outs.append(G.exp()[..., None] * (qc @ S) + qk @ delta)
        tail = (G[..., -1:] - G).exp()                                  # e^{G_C − G_j}
        S = G[..., -1].exp()[..., None, None] * S + (kc * tail[..., None]).transpose(-1, -2) @ delta
    out = torch.cat(outs, dim=2).transpose(1, 2).contiguous().to(dt)
    return out, S


# ────────────────────────────── causal conv ──────────────────────────────

def causal_conv_silu(raw, conv_state, w):
    """Depthwise causal conv (kernel K, no bias) + SiLU over cat(q,k,v) channels —
    blocks.py:268-286. raw: (B,T,C); conv_state: (B,C,K-1) or None; w: (C,1,K).
    Returns (out (B,T,C), new_state (B,C,K-1)) where new_state = the last K-1 raw columns
    of [conv_state | raw] (zero-padded on the left if shorter)."""
    B, T, C = raw.shape
    K = w.shape[-1]
    x = raw.transpose(1, 2)                                             # (B,C,T)
    hist = torch.zeros(B, C, K - 1, dtype=raw.dtype) if conv_state is None else conv_state
    full = torch.cat([hist.to(raw.dtype), x], dim=-1)                   # (B,C,K-1+T)
    y = F.conv1d(full, w.to(raw.dtype), None, padding=0, groups=C)     # (B,C,T)
    out = F.silu(y).transpose(1, 2)
    return out, full[:, :, -(K - 1):].clone()


# ─────────────────────────────── partial RoPE ───────────────────────────────

def rope_inv_freq(rotary_dim, theta):
    """inv_freq_i = 1/θ^(2i/rd) in fp32 — blocks.py:166-168."""
    idx = torch.arange(0, rotary_dim, 2, dtype=torch.float32)
    return 1.0 / (theta ** (idx / rotary_dim))


def rope_cos_sin(positions, rotary_dim, theta, dtype):
    """cos/sin tables (T, rd) with the half-repeated frequency layout — blocks.py:170-173."""
    f = positions.float()[:, None] * rope_inv_freq(rotary_dim, theta)[None, :]
    f = torch.cat([f, f], dim=-1)
    return f.cos().to(dtype), f.sin().to(dtype)


def rope_rotate(x, cos, sin):
    """Rotate the first rd dims of x (…,T,hd) by rotate-half; pass the rest — blocks.py:175-183."""
    rd = cos.shape[-1]
    xr, xp = x[..., :rd], x[..., rd:]
    h = rd // 2
    rot = torch.cat([-xr[..., h:], xr[..., :h]], dim=-1)
    return torch.cat([xr * cos + rot * sin, xp], dim=-1)


# ─────────────────────────────── attention ───────────────────────────────

def offset_causal_attention(q, k, v, scale=None):
    """Softmax attention where query i (of T) sits at absolute position L−T+i and sees keys
    at positions ≤ that — attention.py:43-51 (SDPA scale hd^-0.5 by default).
    q: (H,T,hd); k,v: (H,L,hd), already GQA-expanded. Computed in fp32, cast back."""
    dt = q.dtype
    H, T, hd = q.shape
    L = k.shape[1]
    scale = hd ** -0.5 if scale is None else scale
    s = torch.einsum("htd,hld->htl", q.float(), k.float()) * scale
    qpos = torch.arange(L - T, L)[:, None]
    kpos = torch.arange(L)[None, :]
    s = s.masked_fill(kpos > qpos, -math.inf)
    p = torch.softmax(s, dim=-1)
    return torch.einsum("htl,hld->htd", p, v.float()).to(dt)


# ────────────────────────────────── cache ──────────────────────────────────

@dataclass
class OracleCache:
    """Per-layer state, per-sequence lengths. KV: layer -> [per-seq (K (n_kv,L,hd), V)];
    GDN: layer -> (conv (B,C,K-1), rec (B,Hv,dk,dv) fp32)."""
    n_layers: int
    kv: dict = field(default_factory=dict)
    gdn: dict = field(default_factory=dict)
    lens: list = None

    def clone(self):
        c = OracleCache(self.n_layers)
        c.kv = {l: [(k.clone(), v.clone()) for k, v in s] for l, s in self.kv.items()}
        c.gdn = {l: (a.clone(), b.clone()) for l, (a, b) in self.gdn.items()}
        c.lens = list(self.lens) if self.lens is not None else None
        return c

    def truncate(self, keep):
        """Per-sequence rollback to `keep[b]` tokens (KV only; GDN state is not invertible)."""
        for l, s in self.kv.items():
            self.kv[l] = [(k[:, :n].clone(), v[:, :n].clone()) for (k, v), n in zip(s, keep)]
        self.lens = list(keep)


# ────────────────────────────────── layers ──────────────────────────────────

def gdn_mixer(P, pre, cfg, x, state, scan="reference"):
    """Gated DeltaNet token mixer — blocks.py:288-329. x: (B,T,H) model dtype.
    state: (conv, rec) or None. Returns (out (B,T,H), (conv, rec))."""
    B, T, _ = x.shape
    nk, nv, dk, dv = (cfg.linear_num_key_heads, cfg.linear_num_value_heads,
                      cfg.linear_key_head_dim, cfg.linear_value_head_dim)
    qkv = linear(x, P[pre + "in_proj_qkv.weight"])
    z = linear(x, P[pre + "in_proj_z.weight"]).reshape(B, T, nv, dv)
    b = linear(x, P[pre + "in_proj_b.weight"])
    a = linear(x, P[pre + "in_proj_a.weight"])
    conv_state, rec = (None, None) if state is None else state
    act, new_conv = causal_conv_silu(qkv, conv_state, P[pre + "conv1d.weight"])
    q, k, v = act.split([cfg.key_dim, cfg.key_dim, cfg.value_dim], dim=-1)
    q = q.reshape(B, T, nk, dk).repeat_interleave(cfg.v_per_k, dim=2)
    k = k.reshape(B, T, nk, dk).repeat_interleave(cfg.v_per_k, dim=2)
    v = v.reshape(B, T, nv, dv)
    beta = b.sigmoid()
    g = -P[pre + "A_log"].float().exp() * F.softplus(a.float() + P[pre + "dt_bias"].float())
    q, k = l2_normalize(q), l2_normalize(k)
    use_recurrent = (scan == "recurrent") or (scan == "reference" and state is not None and T == 1)
    rule = delta_rule_recurrent if use_recurrent else delta_rule_chunked
    core, new_rec = rule(q, k, v, g, beta, rec)
    core = rms_norm_gated(core.reshape(-1, dv), z.reshape(-1, dv), P[pre + "norm.weight"],
                          cfg.rms_norm_eps).reshape(B, T, cfg.value_dim)
    return linear(core, P[pre + "out_proj.weight"]), (new_conv, new_rec)


def attn_project(P, pre, cfg, x):
    """q(+gate)/k/v projection, QK-norm — blocks.py:211-220. Returns q (B,nh,T,hd),
    gate (B,T,nh*hd), k, v (B,nkv,T,hd) before RoPE."""
    B, T, _ = x.shape
    nh, nkv, hd = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
    qg = linear(x, P[pre + "q_proj.weight"]).view(B, T, nh, 2 * hd)
    q, gate = qg[..., :hd], qg[..., hd:]
    gate = gate.reshape(B, T, nh * hd)
    q = rms_norm(q, P[pre + "q_norm.weight"], cfg.rms_norm_eps).transpose(1, 2)
    k = rms_norm(linear(x, P[pre + "k_proj.weight"]).view(B, T, nkv, hd),
                 P[pre + "k_norm.weight"], cfg.rms_norm_eps).transpose(1, 2)
    v = linear(x, P[pre + "v_proj.weight"]).view(B, T, nkv, hd).transpose(1, 2)
    return q, gate, k, v


def attn_mixer(P, pre, cfg, x, positions, kv_seqs):
    """Gated full attention with a per-sequence KV cache — blocks.py:211-236.
    positions: (B,T) absolute positions; kv_seqs: list of per-seq (K,V) or None.
    Returns (out (B,T,H), new kv_seqs)."""
    B, T, _ = x.shape
    nh, hd = cfg.num_attention_heads, cfg.head_dim
    q, gate, k, v = attn_project(P, pre, cfg, x)
    outs, new_kv = [], []
    for bi in range(B):
        cos, sin = rope_cos_sin(positions[bi], cfg.rotary_dim, cfg.rope_theta, x.dtype)
        qb, kb = rope_rotate(q[bi], cos, sin), rope_rotate(k[bi], cos, sin)
        vb = v[bi]
        if kv_seqs is not None and kv_seqs[bi] is not None:
            kb = torch.cat([kv_seqs[bi][0], kb], dim=1)
            vb = torch.cat([kv_seqs[bi][1], vb], dim=1)
        new_kv.append((kb, vb))
        ke = kb.repeat_interleave(cfg.n_rep, dim=0)
        ve = vb.repeat_interleave(cfg.n_rep, dim=0)
        outs.append(offset_causal_attention(qb, ke, ve))
    o = torch.stack(outs).transpose(1, 2).reshape(B, T, nh * hd)
    o = o * torch.sigmoid(gate)
    return linear(o, P[pre + "o_proj.weight"]), new_kv


def ffn(P, pre, cfg, x, moe=False):
    """SwiGLU MLP (blocks.py:332-342) or, on layers where `cfg.is_moe_layer` holds, the
    sparse MoE block (src/qwen3_5_moe/blocks.py:399-421)."""
    if not moe:
        return linear(silu_mul(linear(x, P[pre + "mlp.gate_proj.weight"]),
                               linear(x, P[pre + "mlp.up_proj.weight"])),
                      P[pre + "mlp.down_proj.weight"])
    return moe_ffn(P, pre + "mlp.", cfg, x)


# When a list, moe_ffn appends (prefix, margins) per call: margins[n] is the gap between
# token n's k-th and (k+1)-th router logits in units of the model dtype's rounding step at
# the k-th logit (inf in fp32). A bf16 gap of a step or two is a near-tie: rounding noise
# upstream (accumulation order of any earlier op) can swap which expert is selected, so
# tests flag those tokens instead of comparing them.
ROUTER_MARGINS = None


def router_margin_ulps(logits, k):
    """Gap between the k-th and (k+1)-th largest logit per row, in bf16 steps."""
    if logits.dtype != torch.bfloat16 or k >= logits.shape[-1]:
        return torch.full(logits.shape[:-1], float("inf"))
    s = logits.float().sort(-1, descending=True).values
    ulp = torch.exp2(torch.floor(torch.log2(s[..., k - 1].abs().clamp_min(1e-30))) - 7)
    return (s[..., k - 1] - s[..., k]) / ulp


def near_tie_rows(margin_log, B, T, thresh=2.0):
    """(B, T) bool: tokens of a (B, T) forward whose routing was a near-tie (margin below
    `thresh` bf16 steps) on any MoE layer of the logged call, with every later position of
    the same sequence (they attend to / scan over the flagged one)."""
    flag = torch.zeros(B, T, dtype=torch.bool)
    for pre, m in margin_log:
        if not pre.startswith("model."):
            continue
        flag |= (m.reshape(B, T) < thresh)
    return flag.int().cummax(dim=1).values.bool()


def moe_ffn(P, pre, cfg, x):
    """Router softmax (fp32) → top-k → renorm → Σ p·SwiGLU_e(x) + σ(gate_s x)·SwiGLU_s(x) —
    src/qwen3_5_moe/blocks.py:399-421, the same per-expert loop in ascending expert order
    (so the model-dtype accumulation of index_add_ rounds in the same order)."""
    shp = x.shape
    xt = x.reshape(-1, shp[-1])
    router = linear(xt, P[pre + "gate.weight"])
    if ROUTER_MARGINS is not None:
        ROUTER_MARGINS.append((pre, router_margin_ulps(router, cfg.num_experts_per_tok)))
    probs = F.softmax(router, dim=-1, dtype=torch.float32)
    w, idx = torch.topk(probs, cfg.num_experts_per_tok, dim=-1)
    if cfg.norm_topk_prob:
        w = w / w.sum(-1, keepdim=True)
    w = w.to(x.dtype)
    y = torch.zeros_like(xt)
    gu, dn = P[pre + "experts.gate_up_proj"], P[pre + "experts.down_proj"]
    im = cfg.moe_intermediate_size
    for e in torch.unique(idx).tolist():
        tok, slot = torch.where(idx == e)
        h = linear(xt[tok], gu[e])
        o = linear(silu_mul(h[:, :im], h[:, im:]), dn[e]) * w[tok, slot, None]
        y.index_add_(0, tok, o.to(y.dtype))
    if cfg.shared_expert_intermediate_size > 0:
        s = linear(silu_mul(linear(xt, P[pre + "shared_expert.gate_proj.weight"]),
                            linear(xt, P[pre + "shared_expert.up_proj.weight"])),
                   P[pre + "shared_expert.down_proj.weight"])
        y = y + torch.sigmoid(linear(xt, P[pre + "shared_expert_gate.weight"])) * s
    return y.reshape(shp)


# ─────────────────────────────────── model ───────────────────────────────────

def model_forward(P, cfg, ids, cache=None, scan="reference"):
    """Qwen3_5Model.forward — src/qwen3_5/modeling_qwen3_5.py:82-102 (and its MoE sibling
    src/qwen3_5_moe/modeling_qwen3_5_moe.py:81-102, whose layers pick the FFN per
    `is_moe_layer`, modeling_qwen3_5_moe.py:42-43), with per-sequence
    positions (lens[b] + t). ids: (B,T) int64. Returns (logits (B,T,V), cache, hidden)."""
    B, T = ids.shape
    if cache is None:
        cache = OracleCache(cfg.num_hidden_layers, lens=[0] * B)
    x = F.embedding(ids, P["model.embed_tokens.weight"])
    positions = torch.stack([torch.arange(n, n + T) for n in cache.lens])
    for i in range(cfg.num_hidden_layers):
        pre = f"model.layers.{i}."
        h = rms_norm(x, P[pre + "input_layernorm.weight"], cfg.rms_norm_eps)
        if cfg.layer_type(i) == "full_attention":
            h, cache.kv[i] = attn_mixer(P, pre + "self_attn.", cfg, h, positions, cache.kv.get(i))
        else:
            h, cache.gdn[i] = gdn_mixer(P, pre + "linear_attn.", cfg, h, cache.gdn.get(i), scan)
        x = x + h
        x = x + ffn(P, pre, cfg, rms_norm(x, P[pre + "post_attention_layernorm.weight"],
                                          cfg.rms_norm_eps), moe=cfg.is_moe_layer(i))
    cache.lens = [n + T for n in cache.lens]
    hidden = x
    logits = linear(rms_norm(hidden, P["model.norm.weight"], cfg.rms_norm_eps), P["lm_head.weight"])
    return logits, cache, hidden


def mtp_forward(P, cfg, hidden, next_emb):
    """MTP head — src/qwen3_5/mtp.py:61-73: x = fc([norm_e(emb); norm_h(hidden)]) → one
    full-attention DecoderLayer with no cache → final norm. Returns (post_norm, pre_norm),
    both (B,L,H). With no cache each position attends only to itself, so the attention
    output is exactly v and RoPE/QK-norm cancel; this restatement still runs them
    (positions 1..L as at mtp.py:66-67) to stay literal."""
    B, L, _ = hidden.shape
    x = linear(torch.cat([rms_norm(next_emb, P["mtp.pre_fc_norm_embedding.weight"], cfg.rms_norm_eps),
                          rms_norm(hidden, P["mtp.pre_fc_norm_hidden.weight"], cfg.rms_norm_eps)],
                         dim=-1), P["mtp.fc.weight"])
    pre = "mtp.layers.0."
    h = rms_norm(x, P[pre + "input_layernorm.weight"], cfg.rms_norm_eps)
    # one-shot attention over the L positions of this call (no cache): offset-causal with
    # total_k == T, i.e. plain causal (attention.py:51)
    positions = torch.arange(1, L + 1)[None].expand(B, L)
    h, _ = attn_mixer(P, pre + "self_attn.", cfg, h, positions, None)
    x = x + h
    x = x + ffn(P, pre, cfg, rms_norm(x, P[pre + "post_attention_layernorm.weight"], cfg.rms_norm_eps),
                moe=cfg.is_moe_layer(0))   # the MoE family's MTP block asks for layer 0
    return rms_norm(x, P["mtp.norm.weight"], cfg.rms_norm_eps), x


def lm_head(P, x):
    return linear(x, P["lm_head.weight"])
