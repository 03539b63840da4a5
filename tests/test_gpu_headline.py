"""Parity at the production configuration (BASELINE configs[1]-[3]): the kernels and launch
grids the benchmark times, checked against the CPU oracle.

* One speculative step of the full 24-layer 2B-shape model in bf16 at batch 64 with ragged
  contexts around 2048 (the bench's 296-CTA GDN grid over 64x32 heads, its attention split
  count and the vocabulary K-split tail at 151936). The oracle recomputes 8 of the 64
  sequences (they are independent): MTP draft logits at every depth; every mixer and FFN of
  the verify forward on the GPU's own inputs (bf16 rounding differences of one step per
  block add up over 24 layers to ~3 % of the largest logit at random init, so blocks are
  compared one at a time and the end-to-end drift only bounded); greedy acceptance of drafts
  planted to be accepted 0..3 times; the committed GDN states after the index rollback; and
  the decode after it, block by block from the kept-token state.
* The verify attention at configs[2] lengths (up to 32768 keys) at the bench's split count.
* The GDN update at configs[3] shape (64 sequences, 16 key / 32 value heads of 128) with a
  ragged rollback checked bit for bit against fresh forwards over the kept tokens.

bf16 tolerance: 2e-2 (`tolerance.assert_bf16_close`: relative to the tensor's largest magnitude
for every element, and elementwise 2e-2 atol + 2e-2 rtol for all but 0.1 % of them). A greedy pick is
only compared where the oracle's two best logits are more than 2 bf16 steps apart at that
value (a near-tie: a last-bit rounding difference anywhere upstream decides it); near-ties
are counted and the rest of that sequence's step is excluded.
"""

import math

import pytest
import torch

from oracle import loops as OL
from oracle import qwen35 as Q
from tolerance import assert_bf16_close

pytestmark = pytest.mark.gpu
DEV = "cuda"
BF = torch.bfloat16
SUBSET = [0, 9, 18, 27, 36, 45, 54, 63]


def near_tie(logits_row, thresh=2.0):
    """True when the best and second-best logits are within `thresh` bf16 steps."""
    s = logits_row.float().topk(2).values
    ulp = 2.0 ** (math.floor(math.log2(max(abs(float(s[0])), 1e-30))) - 7)
    return float(s[0] - s[1]) < thresh * ulp


@pytest.fixture(scope="module")
def two_b():
    from lollm_b200.qwen3_5 import MTP, Qwen3_5Model
    from lollm_b200.qwen3_5.config import QWEN35_2B, Qwen3_5Config
    from lollm_b200.qwen3_5.weights import load_checkpoint, random_init
    cfg = Qwen3_5Config.from_hf(QWEN35_2B)
    w = random_init(cfg, 7, dtype=BF, device=DEV, generator="torch")
    params = load_checkpoint(cfg, w, device=DEV)
    model = Qwen3_5Model(cfg, params, dtype=BF, device=DEV, max_positions=2400)
    mtp = MTP(model, params)
    host = {k: v.cpu() for k, v in params.items() if k != "lm_head.weight"}
    host["lm_head.weight"] = host["model.embed_tokens.weight"]
    del w, params
    torch.cuda.empty_cache()
    return cfg, model, mtp, host


def filled_cache(cfg, model, B, lens, seed):
    """A cache holding lens[b] positions per sequence: random post-RoPE K/V pages, random
    conv windows and fp32 recurrent states N(0, 0.1); and its oracle mirror for SUBSET."""
    g = torch.Generator().manual_seed(seed)
    cache = model.new_cache(B, 2304, max_spec_tokens=4)
    ps = cache.page_size
    for s in range(len(cfg.attn_layers)):
        for t in (cache.k_pages, cache.v_pages):
            t[s].copy_(torch.randn(t[s].shape, generator=g).to(BF))
    cache.state.copy_(torch.randn(cache.state.shape, generator=g) * 0.1)
    Kc = cfg.linear_conv_kernel_dim
    conv = torch.randn(cache.conv_hist.shape[0], B, Kc - 1, cfg.conv_dim, generator=g).to(BF)
    cache.conv_hist[:, 0, :, :Kc - 1].copy_(conv)
    cache.seq_lens.copy_(torch.tensor(lens, dtype=torch.int32))
    oc = Q.OracleCache(cfg.num_hidden_layers, lens=[lens[b] for b in SUBSET])
    for i in cfg.attn_layers:
        s = cache.attn_slot[i]
        per = []
        for b in SUBSET:
            n = lens[b]
            pages = cache.page_table[b, :math.ceil(n / ps)].long()
            kk = cache.k_pages[s, pages].permute(1, 0, 2, 3).reshape(cfg.num_key_value_heads, -1, cfg.head_dim)[:, :n]
            vv = cache.v_pages[s, pages].permute(1, 0, 2, 3).reshape(cfg.num_key_value_heads, -1, cfg.head_dim)[:, :n]
            per.append((kk.cpu(), vv.cpu()))
        oc.kv[i] = per
    idx = torch.tensor(SUBSET)
    for i in cfg.gdn_layers:
        s = cache.gdn_slot[i]
        oc.gdn[i] = (conv[s][idx].transpose(1, 2).contiguous(), cache.state[s][idx.to(DEV)].cpu())
    return cache, oc


def _teacher_forced(P, cfg, trace, rows, T, oc, what, keep=None):
    """Check one traced GPU forward block by block against the oracle fed the GPU's own
    inputs: layer i's mixer runs on the GPU's residual stream entering layer i, its FFN on the
    GPU's stream after the mixer, the logits on the GPU's final stream. Every block must then
    match to bf16 rounding, whatever the drift accumulated over the layers before it. `oc`
    (the oracle cache of the SUBSET, updated in place) supplies the K/V and GDN state the
    blocks start from; with `keep` the GDN states and K/V are left as after only the first
    keep[j] tokens of sequence j (the rollback). Returns the last stream (S, T, H)."""
    eps = cfg.rms_norm_eps
    S = len(rows)
    xs = [t.view(-1, T, t.shape[-1])[rows].cpu() for t in trace]
    positions = torch.stack([torch.arange(n, n + T) for n in oc.lens])
    for i in range(cfg.num_hidden_layers):
        pre = f"model.layers.{i}."
        x_in, x_mid, x_out = xs[2 * i], xs[2 * i + 1], xs[2 * i + 2]
        h = Q.rms_norm(x_in, P[pre + "input_layernorm.weight"], eps)
        if cfg.layer_type(i) == "full_attention":
            o, kv = Q.attn_mixer(P, pre + "self_attn.", cfg, h, positions, oc.kv.get(i))
            oc.kv[i] = kv if keep is None else [(k_[:, :n + keep[j]], v_[:, :n + keep[j]])
                                                for j, ((k_, v_), n) in enumerate(zip(kv, oc.lens))]
        else:
            o, st = Q.gdn_mixer(P, pre + "linear_attn.", cfg, h, oc.gdn.get(i))
            if keep is None:
                oc.gdn[i] = st
            else:   # the state after only the kept tokens of each sequence
                convs, recs = [], []
                for j in range(S):
                    _, (cv, rc) = Q.gdn_mixer(P, pre + "linear_attn.", cfg, h[j:j + 1, :keep[j]],
                                              (oc.gdn[i][0][j:j + 1], oc.gdn[i][1][j:j + 1]))
                    convs.append(cv)
                    recs.append(rc)
                oc.gdn[i] = (torch.cat(convs), torch.cat(recs))
        assert_bf16_close(x_mid, x_in + o, what=f"{what}: layer {i} mixer")
        f = Q.ffn(P, pre, cfg, Q.rms_norm(x_mid, P[pre + "post_attention_layernorm.weight"], eps))
        assert_bf16_close(x_out, x_mid + f, what=f"{what}: layer {i} FFN")
    oc.lens = [n + (T if keep is None else keep[j]) for j, n in enumerate(oc.lens)]
    return xs[-1]


def test_two_b_speculative_step_matches_oracle(two_b):
    """One speculative step of the production configuration, checked block by block (each
    mixer and FFN of all 24 layers on the GPU's own inputs, so bf16 rounding differences do
    not compound into the comparison), plus the end-to-end drift, the greedy acceptance of
    drafts planted to be accepted 0..3 times, the index rollback and the decode after it."""
    cfg, model, mtp, P = two_b
    from lollm_b200 import kernels as K
    B, k = 64, 3
    T = k + 1
    g = torch.Generator().manual_seed(11)
    lens = torch.randint(1900, 2201, (B,), generator=g).tolist()
    cache, oc = filled_cache(cfg, model, B, lens, seed=12)
    hidden_last = torch.randn(B, cfg.hidden_size, generator=g).to(BF)
    pending = torch.randint(0, cfg.vocab_size, (B,), generator=g)
    ids = torch.zeros(B, T, dtype=torch.int64, device=DEV)
    ids[:, 0] = pending.to(DEV)
    sub = torch.tensor(SUBSET)
    rows = sub.to(DEV)

    # ---- MTP drafts (depth 1..k): logits per depth, the oracle fed the GPU's drafted tokens
    dl = mtp.draft(hidden_last.to(DEV).contiguous(), ids, k).cpu()
    h, tok = hidden_last[sub][:, None], pending[sub]
    for d in range(k):
        emb = torch.nn.functional.embedding(tok[:, None], P["model.embed_tokens.weight"])
        post, pre = Q.mtp_forward(P, cfg, h, emb)
        want = Q.lm_head(P, post)[:, 0]
        assert_bf16_close(dl[sub, d], want, what=f"draft logits depth {d + 1}")
        got_tok = ids[rows, d + 1].cpu()
        for j, b in enumerate(SUBSET):
            if not near_tie(want[j]):
                assert int(got_tok[j]) == int(want[j].float().argmax()), f"draft depth {d + 1}, sequence {b}"
        h, tok = pre, got_tok

    # ---- plant drafts accepted a_b = 0..3 times: the target's own pick at the accepted
    #      positions (found by verify passes on copies of the cache; the kernels are
    #      deterministic, so the real pass repeats those picks), a different token after
    plan = [j % (k + 1) for j in range(B)]
    planv = torch.tensor(plan, device=DEV)
    for d in range(k):
        c2 = cache.clone()
        ws = model._forward_into(ids, c2, B, T, True)
        best = ws.logits.view(B, T, -1)[:, d].float().argmax(-1)
        ids[:, d + 1] = torch.where(planv > d, best, (best + 1) % cfg.vocab_size)
        del c2
        torch.cuda.empty_cache()

    # ---- the speculative verify forward, traced, checked block by block
    trace = []
    ws = model._forward_into(ids, cache, B, T, True, trace=trace)
    logits = ws.logits.view(B, T, -1)
    oc_v = oc.clone()
    x_last = _teacher_forced(P, cfg, trace, rows, T, oc_v, "verify")
    lg_tf = Q.lm_head(P, Q.rms_norm(x_last, P["model.norm.weight"], cfg.rms_norm_eps))
    assert_bf16_close(logits[rows], lg_tf, what="verify logits (final stream)")
    # end to end: the oracle's own 24 layers from the same cache. bf16 rounding differences
    # of one step per block accumulate over the residual stream (measured: ~3 % of the
    # largest logit after 24 layers at random init), so this bound only catches gross errors
    ol, _, _ = Q.model_forward(P, cfg, ids[rows].cpu(), oc.clone())
    drift = float((logits[rows].float().cpu() - ol.float()).abs().max() / ol.float().abs().max())
    assert drift < 0.1, f"end-to-end logits drift {drift:.3f} of the largest logit"

    # ---- greedy acceptance (exact match) and the next token
    accept_n = torch.zeros(B, dtype=torch.int32, device=DEV)
    next_tok = torch.zeros(B, dtype=torch.int64, device=DEV)
    amax = torch.zeros(B * T, dtype=torch.int64, device=DEV)
    K.greedy_verify(ws.logits, B, T, ids[:, 1:], T, accept_n, next_tok, amax)
    acc = accept_n.cpu()
    nxt = next_tok.cpu()
    assert acc.tolist() == plan, "accepted counts differ from the planted drafts"
    am = logits.float().argmax(-1).cpu()            # torch's argmax of the same logits
    assert torch.equal(am.flatten(), amax.cpu())
    assert nxt.tolist() == [int(am[b, plan[b]]) for b in range(B)]
    # and the reference's picks from the same final stream (off near-ties)
    for j, b in enumerate(SUBSET):
        for t in range(plan[b] + 1):
            if not near_tie(lg_tf[j, t]):
                assert int(am[b, t]) == int(lg_tf[j, t].float().argmax()), f"sequence {b} position {t}"

    # ---- rollback by index, then one decode step from the kept tokens
    cache.accept(accept_n)
    keep = (acc + 1).tolist()
    assert cache.seq_lens.cpu().tolist() == [lens[b] + keep[b] for b in range(B)]
    oc_r = oc.clone()
    _teacher_forced(P, cfg, trace, rows, T, oc_r, "verify (kept tokens)", keep=[keep[b] for b in SUBSET])
    # the committed GDN states (pending updates flushed) equal the kept-token states
    for i in cfg.gdn_layers:
        conv, rec = cache.linear_state(i)
        assert_bf16_close(rec[rows], oc_r.gdn[i][1], what=f"GDN state layer {i}")
        assert_bf16_close(conv[rows], oc_r.gdn[i][0], what=f"conv window layer {i}")
    trace2 = []
    ws2 = model._forward_into(nxt[:, None].to(DEV).contiguous(), cache, B, 1, False, trace=trace2)
    x2 = _teacher_forced(P, cfg, trace2, rows, 1, oc_r, "decode after rollback")
    lg2 = Q.lm_head(P, Q.rms_norm(x2, P["model.norm.weight"], cfg.rms_norm_eps))
    assert_bf16_close(ws2.logits.view(B, 1, -1)[rows], lg2, what="decode logits after rollback")
    assert int(cache.bad_index) == 0 and K.device_status() == 0
    print(f"end-to-end verify logits drift: {drift:.4f} of the largest logit")


@pytest.mark.parametrize("splits", [64, 32, 1])
def test_attention_at_configs2_lengths(splits):
    """16 q / 2 kv heads of 256, T=4, contexts spanning [1024, 32768], page size
    64 (the tensor-core kernel), at 64 splits, at the split count the model and the isolated
    bench take at a 32k capacity (32) and at the step's 2.3k capacity (1), against the
    oracle's offset-causal attention."""
    from test_gpu_kernels import _attn_case, _attn_reference
    from lollm_b200 import kernels as K
    lens = [1024, 32764, 5000, 17000, 2047, 30001, 1500, 9999, 24576, 12345, 4096, 31000]
    B, T, nh, nkv, hd, rd = len(lens), 4, 16, 2, 256, 64
    d, D, H = _attn_case(BF, B, T, nh, nkv, hd, rd, lens, page_size=64, splits=splits, seed=21)
    K.attn_prep(d)
    K.attn_verify(d)
    assert int(D["bad"]) == 0
    out = D["out"].cpu().view(B, T, nh * hd)
    for b in range(B):
        assert_bf16_close(out[b], _attn_reference(H, b, lens[b], T, nh, nkv, hd, 64)[0], what=f"sequence {b}")
    assert K.device_status() == 0


def test_gdn_configs3_ragged_rollback_is_bitwise():
    """64 sequences, 16 key / 32 value heads of 128, fp32 state N(0, 0.1), T=4
    speculative, then a rollback keeping 1..4 tokens per sequence. The next launch replays
    exactly the kept tokens; the flushed state and conv window equal, bit for bit, those of
    a fresh commit-all forward over the same tokens, and match the oracle within bf16
    tolerance."""
    from test_gpu_kernels import GdnCase, _gdn_flush
    from lollm_b200 import kernels as K
    B, Hk, Hv, d = 64, 16, 32, 128
    mk = lambda: GdnCase(BF, B=B, Hk=Hk, Hv=Hv, d=d, Ts=8, seed=31)
    c1 = mk()
    g = torch.Generator().manual_seed(32)
    s0 = torch.randn(B, Hv, d, d, generator=g) * 0.1
    c1.state.copy_(s0)
    proj = c1.random_proj(4)
    out = c1.run(proj, speculative=True)
    conv0 = torch.zeros(B, c1.C, c1.Kc - 1, dtype=BF)
    want, _, _ = c1.oracle(proj, conv0, s0)
    assert_bf16_close(out, want, what="GDN outputs")
    keep = torch.randint(1, 5, (B,), generator=g)
    K.cache_accept(B, 4, (keep - 1).int().to(DEV), c1.lens, c1.replay, c1.coff)
    _gdn_flush(c1)
    p1 = int(c1.parity.item())
    conv1 = c1.hist[p1, :, :c1.Kc - 1].clone()
    for n in range(1, 5):
        c2 = mk()
        c2.state.copy_(s0)
        c2.run(proj[:, :n].contiguous(), speculative=False)
        rows = (keep == n).nonzero()[:, 0].to(DEV)
        p2 = int(c2.parity.item())
        assert torch.equal(c1.state[rows], c2.state[rows]), f"state differs for kept {n}"
        assert torch.equal(conv1[rows], c2.hist[p2, :, :c2.Kc - 1][rows]), f"conv differs for kept {n}"
        del c2
    # oracle on the kept tokens of a few sequences
    for b in (0, 17, 40, 63):
        _, cv, rc = c1.oracle(proj[b:b + 1, :int(keep[b])], conv0[b:b + 1], s0[b:b + 1])
        assert_bf16_close(c1.state[b], rc[0], what=f"state of sequence {b}")
    assert K.device_status() == 0
