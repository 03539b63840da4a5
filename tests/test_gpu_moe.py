"""Sparse-MoE FFN (qsp_moe_ffn) and the qwen3_5_moe model on the GPU against the reference's
goldens and the CPU oracle.

fp32 runs the CUDA-core expert path, bf16 the tcgen05 grouped expert GEMMs. Tolerances are
the suite's: fp32 1e-4 relative, bf16 2e-2. In bf16 a token whose k-th and (k+1)-th router
logits lie within two rounding steps is a flagged near-tie: the last-bit rounding of any
upstream op decides which expert wins, so those tokens are excluded and counted (fp32 has
none). Expert selection is otherwise identical: checked through the per-expert counts.
"""

import os

import pytest
import torch

from oracle import loops as OL
from oracle import qwen35 as Q
from lollm_b200.qwen3_5.config import MICRO_MOE, Qwen3_5Config
from lollm_b200.qwen3_5.weights import load_checkpoint, random_init
from tolerance import assert_close_dt

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SEED = 1234
MOE_CASES = [
    ("shared", 128, 16, 4, 64, 64, True, 40),
    ("noshared", 128, 16, 4, 64, 0, True, 24),
    ("nonorm", 64, 8, 3, 32, 32, False, 17),
]


@pytest.fixture(scope="module")
def golden_moe():
    from safetensors.torch import load_file
    return load_file(os.path.join(ROOT, "tests", "golden", "golden_moe.safetensors"))


def moe_cfg(h, e, k, im, ish, norm):
    raw = dict(MICRO_MOE["text_config"])
    raw.update(hidden_size=h, num_experts=e, num_experts_per_tok=k, moe_intermediate_size=im,
               shared_expert_intermediate_size=ish, norm_topk_prob=norm)
    return Qwen3_5Config.from_hf({"text_config": raw})


def run_block(cfg, P, xn, dt, x=None, norm_w=None, eps=1e-6):
    """GPU qsp_moe_ffn: returns (x after the residual add, y or None, expert counts)."""
    from lollm_b200.qwen3_5.moe import SparseMoeBlock
    blk = SparseMoeBlock(cfg, P, "", dtype=dt, device="cuda")
    m, H = xn.shape
    xg = (torch.zeros(m, H) if x is None else x).to(device="cuda", dtype=dt).contiguous()
    xng = xn.to(device="cuda", dtype=dt).contiguous()
    nw = None if norm_w is None else norm_w.to(device="cuda", dtype=dt)
    y = torch.empty_like(xg) if nw is not None else None
    ws = torch.empty(blk.workspace_bytes(m), dtype=torch.uint8, device="cuda")
    counts = torch.full((cfg.num_experts,), -1, dtype=torch.int32, device="cuda")
    blk(xng, xg, nw, y, eps, m, ws, expert_counts=counts)
    torch.cuda.synchronize()
    return xg.cpu(), (None if y is None else y.cpu()), counts.cpu()


def oracle_counts(cfg, P, xn):
    logits = Q.linear(xn, P["mlp.gate.weight"])
    probs = torch.softmax(logits.float(), -1)
    idx = torch.topk(probs, cfg.num_experts_per_tok, -1).indices
    return torch.bincount(idx.flatten(), minlength=cfg.num_experts).int()


def margins_ok(cfg, P, xn):
    return Q.router_margin_ulps(Q.linear(xn, P["mlp.gate.weight"]), cfg.num_experts_per_tok) >= 2.0


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("case", MOE_CASES, ids=[c[0] for c in MOE_CASES])
def test_moe_block_matches_reference(golden_moe, case, dt):
    name, h, e, k, im, ish, norm, n = case
    cfg = moe_cfg(h, e, k, im, ish, norm)
    tag = "f32" if dt == torch.float32 else "bf16"
    P = {"mlp." + kk[len(f"moe.{name}.w."):]: v.to(dt) for kk, v in golden_moe.items()
         if kk.startswith(f"moe.{name}.w.")}
    xn = golden_moe[f"moe.{name}.{tag}.x"]
    got, _, counts = run_block(cfg, P, xn, dt)
    want = golden_moe[f"moe.{name}.{tag}.y"]
    ok = margins_ok(cfg, P, xn)
    assert int(ok.sum()) >= n - 2
    assert_close_dt(got[ok].float(), want[ok].float(), dt)
    if bool(ok.all()):
        assert torch.equal(counts, oracle_counts(cfg, P, xn))


def random_block(h, e, k, im, ish, norm, m, dt, skew_expert=None, seed=0):
    g = torch.Generator().manual_seed(seed)
    r = lambda *s, sc=0.05: torch.randn(*s, generator=g) * sc
    P = {"mlp.gate.weight": r(e, h), "mlp.experts.gate_up_proj": r(e, 2 * im, h),
         "mlp.experts.down_proj": r(e, h, im)}
    if ish:
        P.update({"mlp.shared_expert.gate_proj.weight": r(ish, h), "mlp.shared_expert.up_proj.weight": r(ish, h),
                  "mlp.shared_expert.down_proj.weight": r(h, ish), "mlp.shared_expert_gate.weight": r(1, h)})
    xn = torch.randn(m, h, generator=g)
    if skew_expert is not None:
        # every token routes to this expert: its router row follows the tokens' mean direction
        d = xn.mean(0)
        xn = xn + 5.0 * d / d.norm()
        P["mlp.gate.weight"][skew_expert] = 3.0 * d / d.norm()
    P = {kk: v.to(dt) for kk, v in P.items()}
    return moe_cfg(h, e, k, im, ish, norm), P, xn.to(dt), torch.randn(m, h, generator=g).to(dt), \
        (torch.randn(h, generator=g) * 0.1).to(dt)


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("shape", [
    # (hidden, experts, top_k, inter, shared, norm, tokens, skewed expert)
    (256, 64, 8, 128, 128, True, 256, None),    # ~32 tokens per expert: one token tile each
    (256, 32, 4, 96, 64, True, 300, 5),         # expert 5 takes all 300 tokens: five 64-token tiles
    (128, 6, 6, 64, 0, False, 7, None),         # top_k = n_experts, no shared expert, no renorm
    (192, 12, 3, 40, 24, True, 1, None),        # one token; E + 1 not a multiple of 8; I % 64 != 0
])
def test_moe_block_fused_residual_norm_matches_oracle(shape, dt):
    h, e, k, im, ish, norm, m, skew = shape
    cfg, P, xn, x0, nw = random_block(h, e, k, im, ish, norm, m, dt, skew)
    eps = 1e-6
    got_x, got_y, counts = run_block(cfg, P, xn, dt, x=x0, norm_w=nw, eps=eps)
    moe = Q.moe_ffn(P, "mlp.", cfg, xn)
    want_x = x0 + moe
    want_y = Q.rms_norm(want_x, nw, eps)
    ok = margins_ok(cfg, P, xn)
    assert int(ok.sum()) >= int(0.85 * m)
    assert_close_dt(got_x[ok].float(), want_x[ok].float(), dt)
    assert_close_dt(got_y[ok].float(), want_y[ok].float(), dt)
    if bool(ok.all()):
        assert torch.equal(counts, oracle_counts(cfg, P, xn))
    if skew is not None:
        assert int(counts[skew]) == m


def test_moe_repeated_calls_are_deterministic():
    """The sorted position of a (token, expert) pair depends on atomic order; the results do
    not: two calls give bit-identical outputs (bf16, tensor-core path)."""
    cfg, P, xn, x0, nw = random_block(256, 64, 8, 128, 128, True, 256, torch.bfloat16, seed=4)
    a = run_block(cfg, P, xn, torch.bfloat16, x=x0, norm_w=nw)
    b = run_block(cfg, P, xn, torch.bfloat16, x=x0, norm_w=nw)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1]) and torch.equal(a[2], b[2])


def test_moe_rejects_bad_sizes():
    from lollm_b200 import _lib as L
    import ctypes
    d = L.MoeLayer()
    d.tokens, d.hidden, d.n_experts, d.top_k, d.inter, d.dtype = 4, 64, 8, 9, 32, L.QSP_BF16
    assert L.load().qsp_moe_ffn(ctypes.byref(d), None) == L.QSP_ERR_INVALID
    d.top_k, d.n_experts = 2, 2000
    assert L.load().qsp_moe_ffn(ctypes.byref(d), None) == L.QSP_ERR_INVALID


# ------------------------------------------------------------------ model level

def build(raw, dtype, **kw):
    from lollm_b200 import qwen3_5 as fam
    cfg = Qwen3_5Config.from_hf(raw)
    w = random_init(cfg, SEED, generator="numpy")
    model = fam.load(raw, dict(w), dtype=dtype, **kw)
    mtp = fam.load_mtp(model, dict(w))
    return cfg, model, mtp


def routed_oracle(P, cfg, ids, cache, stale):
    """Oracle forward; returns (rows to compare, cache): rows that were no routing near-tie
    in this call, in sequences (`stale`, updated in place) never flagged before."""
    Q.ROUTER_MARGINS = []
    try:
        _, cache, _ = Q.model_forward(P, cfg, ids, cache)
        flag = Q.near_tie_rows(Q.ROUTER_MARGINS, *ids.shape)
    finally:
        Q.ROUTER_MARGINS = None
    flag |= stale[:, None]
    stale |= flag.any(dim=1)
    return ~flag, cache


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_micro_moe_forward_matches_reference(golden_moe, dt):
    tag = "f32" if dt == torch.float32 else "bf16"
    G = {k[len(f"micro_moe.{tag}."):]: v for k, v in golden_moe.items() if k.startswith(f"micro_moe.{tag}.")}
    cfg, model, mtp = build(MICRO_MOE, dt, max_positions=256)
    P = load_checkpoint(cfg, random_init(cfg, SEED, generator="numpy"), dtype=dt)
    stale = torch.zeros(2, dtype=torch.bool)
    cache, oc, n_cmp = None, None, 0
    for name in ("prefill", "verify", "decode"):
        ids = G["ids" if name == "prefill" else f"{name}.ids"]
        if dt == torch.bfloat16:
            ok, oc = routed_oracle(P, cfg, ids, oc, stale)
        else:
            ok = torch.ones(ids.shape, dtype=torch.bool)
        logits, cache, hidden = model(ids.cuda(), cache, return_hidden=True)
        assert_close_dt(logits.cpu()[ok].float(), G[f"{name}.logits"][ok].float(), dt)
        n_cmp += int(ok.sum())
    assert n_cmp >= (30 if dt == torch.float32 else 12)
    ids = torch.zeros(2, 2, dtype=torch.int64, device="cuda")
    ids[:, 0] = G["decode.ids"][:, 0].cuda()
    h = G["mtp.draft_hidden"][:, 0].to(device="cuda", dtype=dt).contiguous()
    dl = mtp.draft(h, ids, 1)
    assert_close_dt(dl[:, 0].cpu().float(), G["mtp.draft_logits"][:, 0].float(), dt)


def test_micro_moe_all_experts_bf16_matches_oracle():
    """top_k = n_experts removes routing choice, so bf16 compares every row: prefill, a
    speculative verify with ragged accept and a decode, against the oracle."""
    raw = {"model_type": "qwen3_5_moe", "text_config": dict(MICRO_MOE["text_config"], num_experts=4,
                                                            num_experts_per_tok=4)}
    dt = torch.bfloat16
    cfg, model, mtp = build(raw, dt, max_positions=256)
    P = load_checkpoint(cfg, random_init(cfg, SEED, generator="numpy"), dtype=dt)
    g = torch.Generator().manual_seed(8)
    prompt = torch.randint(0, cfg.vocab_size, (3, 11), generator=g)
    cache = model.new_cache(3, 64)
    logits, _ = model(prompt.cuda(), cache)
    ol, oc, _ = Q.model_forward(P, cfg, prompt)
    assert_close_dt(logits.cpu().float(), ol.float(), dt)
    ver = torch.randint(0, cfg.vocab_size, (3, 4), generator=g)
    logits, _ = model(ver.cuda(), cache)
    ol, oc, _ = Q.model_forward(P, cfg, ver, oc)
    assert_close_dt(logits.cpu().float(), ol.float(), dt)


@pytest.mark.parametrize("k", [1, 3])
def test_micro_moe_penalised_spec_stream_equals_reference(golden_moe, k):
    """fp32, temperature 0 with repetition penalty 4: the speculative decoder (k drafts, the
    MTP block's FFN sparse too) commits the reference's generate() stream token for token."""
    from lollm_b200.qwen3_5 import generate_mtp
    cfg, model, mtp = build(MICRO_MOE, torch.float32, max_positions=256)
    prompt = golden_moe["micro_moe.prompt"].tolist()
    want = golden_moe["micro_moe.greedy"].tolist()
    dec = lambda toks: "".join(chr(0x1000 + t) for t in toks)
    text = "".join(generate_mtp(model, mtp, prompt, dec, [], max_new_tokens=len(want), temperature=0.0,
                                top_k=0, top_p=1.0, repetition_penalty=4.0, k=k))
    assert [ord(c) - 0x1000 for c in text] == want


def test_micro_moe_plain_generate_equals_reference(golden_moe):
    from lollm_b200.generate import generate
    cfg, model, mtp = build(MICRO_MOE, torch.float32, max_positions=256)
    prompt = golden_moe["micro_moe.prompt"].tolist()
    want = golden_moe["micro_moe.greedy"].tolist()
    dec = lambda toks: "".join(chr(0x1000 + t) for t in toks)
    text = "".join(generate(model, prompt, dec, [], "cuda", max_new_tokens=len(want), temperature=0.0,
                            top_k=0, top_p=1.0, repetition_penalty=4.0))
    assert [ord(c) - 0x1000 for c in text] == want
