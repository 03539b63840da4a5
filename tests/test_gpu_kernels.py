"""Per-kernel parity of the CUDA path (through the C ABI) against the CPU oracle.

Tolerances: fp32 1e-4 relative, bf16 2e-2; index/rollback results
bit-exact.
"""

import math

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import qwen35 as Q
from oracle import sampling as S

pytestmark = pytest.mark.gpu

DEV = "cuda"
TOL = {torch.float32: dict(rtol=1e-4, atol=1e-5), torch.bfloat16: dict(rtol=2e-2, atol=2e-2)}
DTS = [torch.float32, torch.bfloat16]


def K():
    from lollm_b200 import kernels
    return kernels


def gen(seed):
    return torch.Generator().manual_seed(seed)


def rn(g, *s, scale=1.0, dtype=torch.float32):
    return (torch.randn(*s, generator=g) * scale).to(dtype)


def close(got, want, dtype):
    torch.testing.assert_close(got.float().cpu(), want.float().cpu(), **TOL[dtype])


@pytest.mark.parametrize("dt", DTS)
def test_rmsnorm_and_add(dt):
    g = gen(0)
    x, h, w = rn(g, 37, 200, dtype=dt), rn(g, 37, 200, dtype=dt), rn(g, 200, scale=0.1, dtype=dt)
    y = torch.empty_like(x, device=DEV)
    xd = x.to(DEV)
    K().rmsnorm(xd, w.to(DEV), y, 1e-6)
    close(y, Q.rms_norm(x, w, 1e-6), dt)
    K().add_rmsnorm(xd, h.to(DEV), w.to(DEV), y, 1e-6)
    xs = (x + h)
    assert torch.equal(xd.cpu(), xs)
    close(y, Q.rms_norm(xs, w, 1e-6), dt)


@pytest.mark.parametrize("dt", DTS)
@pytest.mark.parametrize("mnk", [(1, 64, 64), (7, 129, 100), (64, 384, 512), (256, 1000, 2048), (130, 256, 136),
                                 (256, 2048, 4096), (256, 12352, 2048), (64, 4608, 2048), (300, 256, 512),
                                 (1024, 384, 256), (16, 256, 64), (33, 200, 6144),
                                 # 149 weight tiles on 148 SMs: the last tile is split along K
                                 (64, 19000, 1024), (100, 19072, 520),
                                 # several rounds of tiles over the CTA pairs (the persistent pair
                                 # kernel), one with a partial last 16-column chunk
                                 (256, 40000, 512), (136, 19016, 256)])
def test_gemm(dt, mnk):
    m, n, k = mnk
    g = gen(1)
    a, w, c0 = rn(g, m, k, dtype=dt), rn(g, n, k, scale=0.05, dtype=dt), rn(g, m, n, dtype=dt)
    c = torch.empty(m, n, dtype=dt, device=DEV)
    K().gemm(a.to(DEV), w.to(DEV), c)
    ref = (a.double() @ w.double().T)
    # fp32: summation-order error grows like sqrt(k) (outputs here have O(1) magnitude)
    tol = dict(TOL[dt]) if dt == torch.bfloat16 else dict(rtol=1e-4, atol=1e-6 * math.sqrt(k))
    torch.testing.assert_close(c.float().cpu(), ref.to(dt).float(), **tol)
    cd = c0.to(DEV)
    K().gemm(a.to(DEV), w.to(DEV), cd, accumulate=True)
    torch.testing.assert_close(cd.float().cpu(), (c0.float() + ref.to(dt).float()).to(dt).float(), **tol)
    assert K().device_status() == 0


@pytest.mark.parametrize("m", [64, 200, 256])
def test_gemm_fused_epilogues(m):
    """The projections' fused tails in bf16 — residual add + next RMSNorm and SwiGLU — at the
    verify-step row counts (m = 200, 256 take the cluster split-K kernel, m = 64 the persistent
    one), against a float64 product with the same rounding points."""
    dt = torch.bfloat16
    g = gen(11)
    eps = 1e-6
    a, w = rn(g, m, 4096, dtype=dt), rn(g, 2048, 4096, scale=0.02, dtype=dt)
    x0, nw = rn(g, m, 2048, dtype=dt), rn(g, 2048, scale=0.1, dtype=dt)
    x, y = x0.to(DEV), torch.empty(m, 2048, dtype=dt, device=DEV)
    K().gemm_residual_rmsnorm(a.to(DEV), w.to(DEV), x, nw.to(DEV), y, eps)
    xr = (x0.float() + (a.double() @ w.double().T).to(dt).float()).to(dt)
    close(x, xr, dt)
    close(y, Q.rms_norm(xr, nw, eps), dt)
    inter = 1536
    a2, wgu = rn(g, m, 2048, dtype=dt), rn(g, 2 * inter, 2048, scale=0.02, dtype=dt)
    act = torch.empty(m, inter, dtype=dt, device=DEV)
    tmp = torch.empty(m, 2 * inter, dtype=dt, device=DEV)
    K().gemm_swiglu(a2.to(DEV), wgu.to(DEV), act, tmp)
    h = (a2.double() @ wgu.double().T).to(dt)
    close(act, Q.silu_mul(h[:, :inter], h[:, inter:]), dt)
    # the in_proj shape (12352 columns: a partial last tile) through plain qsp_gemm
    w3 = rn(g, 12352, 2048, scale=0.02, dtype=dt)
    c = torch.empty(m, 12352, dtype=dt, device=DEV)
    K().gemm(a2.to(DEV), w3.to(DEV), c)
    close(c, (a2.double() @ w3.double().T).to(dt), dt)
    assert K().device_status() == 0


@pytest.mark.parametrize("m", [136, 256])
def test_gemm_fused_epilogues_ragged(m):
    """Products whose column count is not a whole number of weight tiles and whose depth is not
    a whole number of 64-wide k-blocks, at verify row counts (the CTA-pair kernel writes only
    columns < n and rows < m; its last tile is partial)."""
    dt = torch.bfloat16
    g = gen(12)
    eps = 1e-6
    n, k = 2032, 1000
    a, w = rn(g, m, k, dtype=dt), rn(g, n, k, scale=0.03, dtype=dt)
    x0, nw = rn(g, m, n, dtype=dt), rn(g, n, scale=0.1, dtype=dt)
    x, y = x0.to(DEV), torch.empty(m, n, dtype=dt, device=DEV)
    K().gemm_residual_rmsnorm(a.to(DEV), w.to(DEV), x, nw.to(DEV), y, eps)
    xr = (x0.float() + (a.double() @ w.double().T).to(dt).float()).to(dt)
    close(x, xr, dt)
    close(y, Q.rms_norm(xr, nw, eps), dt)
    inter, k2 = 1000, 2056
    a2, wgu = rn(g, m, k2, dtype=dt), rn(g, 2 * inter, k2, scale=0.02, dtype=dt)
    act = torch.empty(m, inter, dtype=dt, device=DEV)
    tmp = torch.empty(m, 2 * inter, dtype=dt, device=DEV)
    K().gemm_swiglu(a2.to(DEV), wgu.to(DEV), act, tmp)
    h = (a2.double() @ wgu.double().T).to(dt)
    close(act, Q.silu_mul(h[:, :inter], h[:, inter:]), dt)
    for n3 in (1000, 4104):
        w3 = rn(g, n3, k2, scale=0.02, dtype=dt)
        c = torch.empty(m, n3, dtype=dt, device=DEV)
        K().gemm(a2.to(DEV), w3.to(DEV), c)
        close(c, (a2.double() @ w3.double().T).to(dt), dt)
    assert K().device_status() == 0


@pytest.mark.parametrize("dt", DTS)
def test_swiglu_embed_select(dt):
    g = gen(2)
    gu = rn(g, 9, 2 * 300, dtype=dt)
    y = torch.empty(9, 300, dtype=dt, device=DEV)
    K().swiglu(gu.to(DEV), y, 300)
    close(y, Q.silu_mul(gu[:, :300], gu[:, 300:]), dt)
    table = rn(g, 50, 64, dtype=dt)
    ids = torch.tensor([3, 0, 49, 7, 3], dtype=torch.int64)
    out = torch.empty(5, 64, dtype=dt, device=DEV)
    bad = torch.zeros(1, dtype=torch.int32, device=DEV)
    K().embed(ids.to(DEV), table.to(DEV), out, bad=bad)
    assert torch.equal(out.cpu(), table[ids]) and int(bad) == 0
    K().embed(torch.tensor([1, 50], device=DEV), table.to(DEV), out[:2], bad=bad)
    assert int(bad) == 1 and torch.all(out[1].cpu() == 0)
    # strided ids (the draft chain reads column d of a [B, k+1] id buffer)
    ids2 = torch.tensor([[1, 2, 3], [4, 5, 6]], device=DEV)
    K().embed(ids2[:, 1:], table.to(DEV), out[:2], ids_stride=3, rows=2)
    assert torch.equal(out[:2].cpu(), table[torch.tensor([2, 5])])
    src = rn(g, 4 * 3, 64, dtype=dt).to(DEV)
    idx = torch.tensor([2, 0, 1, 2], dtype=torch.int32, device=DEV)
    dst = torch.empty(4, 64, dtype=dt, device=DEV)
    K().select_rows(src, 4, 3, idx, dst)
    assert torch.equal(dst.cpu(), src.view(4, 3, 64)[torch.arange(4), idx.long().cpu()].cpu())


# ─────────────────────────────────────────── GDN ───────────────────────────────────────────

class GdnCase:
    """Random GDN layer weights + a device cache slot, with an oracle mirror of the state."""

    def __init__(self, dt, B=3, Hk=2, Hv=4, d=32, Kc=4, Ts=5, seed=3):
        from lollm_b200 import _lib as L
        self.dt, self.B, self.Hk, self.Hv, self.d, self.Kc, self.Ts = dt, B, Hk, Hv, d, Kc, Ts
        g = gen(seed)
        self.C = 2 * Hk * d + Hv * d
        self.Vd = Hv * d
        self.conv_w = rn(g, self.C, Kc, scale=0.3, dtype=dt)
        self.a_log = rn(g, Hv, scale=0.5, dtype=dt)
        self.dt_bias = rn(g, Hv, scale=0.5, dtype=dt)
        self.norm_w = (1 + rn(g, d, scale=0.1)).to(dt)
        self.g = g
        self.state = torch.zeros(B, Hv, d, d, device=DEV)
        self.hist = torch.zeros(2, B, Kc - 1 + Ts, self.C, dtype=dt, device=DEV)
        self.pending = torch.zeros(K().gdn_pending_bytes(B, Hk, Hv, d, d, Ts, dt), dtype=torch.uint8, device=DEV)
        self.replay = torch.zeros(B, dtype=torch.int32, device=DEV)
        self.coff = torch.zeros(B, dtype=torch.int32, device=DEV)
        self.parity = torch.zeros(1, dtype=torch.int32, device=DEV)
        self.lens = torch.zeros(B, dtype=torch.int32, device=DEV)
        self.dev_w = [t.to(DEV) for t in (self.conv_w, self.a_log, self.dt_bias, self.norm_w)]
        self.L = L

    def random_proj(self, T):
        return rn(self.g, self.B, T, self.C + self.Vd + 2 * self.Hv, dtype=self.dt)

    def run(self, proj, speculative):
        L = self.L
        B, T, _ = proj.shape
        pd = proj.reshape(B * T, -1).to(DEV).contiguous()
        out = torch.zeros(B * T, self.Vd, dtype=self.dt, device=DEV)
        desc = L.GdnLayer()
        desc.batch, desc.tokens, desc.n_k_heads, desc.n_v_heads = B, T, self.Hk, self.Hv
        desc.head_k = desc.head_v = self.d
        desc.conv_kernel, desc.max_spec_tokens, desc.speculative = self.Kc, self.Ts, int(speculative)
        desc.dtype, desc.eps = L.dtype_code(self.dt), 1e-6
        desc.proj, desc.ld_proj = pd.data_ptr(), pd.stride(0)
        desc.conv_w, desc.a_log, desc.dt_bias, desc.norm_w = [t.data_ptr() for t in self.dev_w]
        desc.state, desc.conv_hist, desc.pending = self.state.data_ptr(), self.hist.data_ptr(), self.pending.data_ptr()
        desc.replay_n, desc.conv_off, desc.parity = self.replay.data_ptr(), self.coff.data_ptr(), self.parity.data_ptr()
        desc.out, desc.ld_out = out.data_ptr(), out.stride(0)
        K().gdn_verify(desc)
        K().cache_finalize(B, T, speculative, self.lens, self.replay, self.coff, self.parity)
        return out.view(B, T, -1)

    def oracle(self, proj, conv_state, rec):
        """Oracle core output for raw projections (conv → split → gates → l2norm → delta rule
        → RMSNormGated), from (conv_state, rec) per sequence."""
        B, T, _ = proj.shape
        d, C, Vd, Hv, Hk = self.d, self.C, self.Vd, self.Hv, self.Hk
        qkv, z = proj[..., :C], proj[..., C:C + Vd]
        b, a = proj[..., C + Vd:C + Vd + Hv], proj[..., C + Vd + Hv:]
        act, new_conv = Q.causal_conv_silu(qkv, conv_state, self.conv_w[:, None, :])
        q, k, v = act.split([Hk * d, Hk * d, Vd], dim=-1)
        q = q.reshape(B, T, Hk, d).repeat_interleave(Hv // Hk, dim=2)
        k = k.reshape(B, T, Hk, d).repeat_interleave(Hv // Hk, dim=2)
        v = v.reshape(B, T, Hv, d)
        beta = b.sigmoid()
        gg = -self.a_log.float().exp() * F.softplus(a.float() + self.dt_bias.float())
        core, new_rec = Q.delta_rule_recurrent(Q.l2_normalize(q), Q.l2_normalize(k), v, gg, beta, rec)
        core = Q.rms_norm_gated(core.reshape(-1, d), z.reshape(-1, d), self.norm_w, 1e-6).reshape(B, T, Vd)
        return core, new_conv, new_rec


@pytest.mark.parametrize("dt", DTS)
@pytest.mark.parametrize("d", [32, 64, 128])
def test_gdn_commit_all_matches_oracle(dt, d):
    c = GdnCase(dt, d=d, seed=d)
    conv = torch.zeros(c.B, c.C, c.Kc - 1, dtype=dt)
    rec = torch.zeros(c.B, c.Hv, d, d)
    for T in (6, 1, 19, 3):
        proj = c.random_proj(T)
        got = c.run(proj, speculative=False)
        want, conv, rec = c.oracle(proj, conv, rec)
        close(got, want, dt)
        close(c.state, rec, dt)


def _gdn_flush(c):
    """Replay-only commit-all launch (T = 0): applies pending updates to the stored state."""
    from lollm_b200 import _lib as L
    dummy = torch.zeros(1, c.Vd, dtype=c.dt, device=DEV)
    d = L.GdnLayer()
    d.batch, d.tokens, d.n_k_heads, d.n_v_heads, d.head_k, d.head_v = c.B, 0, c.Hk, c.Hv, c.d, c.d
    d.conv_kernel, d.max_spec_tokens, d.speculative, d.dtype, d.eps = c.Kc, c.Ts, 0, L.dtype_code(c.dt), 1e-6
    d.proj, d.ld_proj = dummy.data_ptr(), c.C + c.Vd + 2 * c.Hv
    d.conv_w, d.a_log, d.dt_bias, d.norm_w = [t.data_ptr() for t in c.dev_w]
    d.state, d.conv_hist, d.pending = c.state.data_ptr(), c.hist.data_ptr(), c.pending.data_ptr()
    d.replay_n, d.conv_off, d.parity = c.replay.data_ptr(), c.coff.data_ptr(), c.parity.data_ptr()
    d.out, d.ld_out = dummy.data_ptr(), c.Vd
    K().gdn_verify(d)
    K().cache_finalize(c.B, 0, False, c.lens, c.replay, c.coff, c.parity)


@pytest.mark.parametrize("dt", DTS)
def test_gdn_speculative_steps_match_oracle(dt):
    """Speculative T=4 calls with ragged keep counts, each followed by accept(); outputs and
    the flushed state / conv window match the oracle run on exactly the kept tokens."""
    c = GdnCase(dt, B=4, d=64, seed=11)
    warm = c.random_proj(5)
    c.run(warm, False)
    _, conv_o, rec_o = c.oracle(warm, torch.zeros(c.B, c.C, c.Kc - 1, dtype=dt), torch.zeros(c.B, c.Hv, c.d, c.d))
    for keep in ([1, 2, 3, 4], [4, 1, 1, 2], [2, 4, 3, 1]):
        proj = c.random_proj(4)
        got = c.run(proj, speculative=True)
        want, _, _ = c.oracle(proj, conv_o, rec_o)
        close(got, want, dt)
        acc = torch.tensor([n - 1 for n in keep], dtype=torch.int32, device=DEV)
        K().cache_accept(c.B, 4, acc, c.lens, c.replay, c.coff)
        rec_new, conv_new = [], []
        for b in range(c.B):
            _, cv, rc = c.oracle(proj[b:b + 1, :keep[b]], conv_o[b:b + 1], rec_o[b:b + 1])
            rec_new.append(rc)
            conv_new.append(cv)
        rec_o, conv_o = torch.cat(rec_new), torch.cat(conv_new)
    _gdn_flush(c)
    close(c.state, rec_o, dt)
    p = int(c.parity.item())
    conv_dev = c.hist[p, :, :c.Kc - 1].transpose(1, 2).cpu()
    assert torch.equal(conv_dev, conv_o.to(dt))


@pytest.mark.parametrize("dt", DTS)
def test_gdn_replay_bitwise_equals_fresh_forward(dt):
    """Index rollback is bit-exact: spec(T=4) + accept(a) + next call  ≡  commit-all(a+1 tokens)."""
    for a in range(4):
        c1 = GdnCase(dt, B=2, d=128, seed=5)
        c2 = GdnCase(dt, B=2, d=128, seed=5)
        warm = c1.random_proj(3)
        c2.random_proj(3)
        c1.run(warm, False)
        c2.run(warm, False)
        proj = c1.random_proj(4)
        c2.random_proj(4)
        c1.run(proj, True)
        K().cache_accept(2, 4, torch.full((2,), a, dtype=torch.int32, device=DEV), c1.lens, c1.replay, c1.coff)
        c2.run(proj[:, :a + 1].contiguous(), False)
        nxt = c1.random_proj(2)
        c2.random_proj(2)
        o1 = c1.run(nxt, False)
        o2 = c2.run(nxt, False)
        assert torch.equal(c1.state, c2.state), f"state differs after rollback to {a}"
        assert torch.equal(o1, o2), f"outputs differ after rollback to {a}"


# ─────────────────────────────────────────── attention ───────────────────────────────────────────

def _attn_case(dt, B, T, nh, nkv, hd, rd, lens, page_size=16, seed=4, shuffle_pages=True, splits=3):
    from lollm_b200 import _lib as L
    from lollm_b200.qwen3_5.modeling_qwen3_5 import rope_table
    g = gen(seed)
    cap = max(lens) + T
    max_pages = math.ceil(cap / page_size) + 1
    num_pages = B * max_pages + 3
    perm = torch.randperm(num_pages, generator=g)[:B * max_pages] if shuffle_pages else torch.arange(B * max_pages)
    page_table = perm.view(B, max_pages).int()
    n_qkv = 2 * nh * hd + 2 * nkv * hd
    qkv = rn(g, B * T, n_qkv, dtype=dt)
    qn, kn = rn(g, hd, scale=0.1, dtype=dt), rn(g, hd, scale=0.1, dtype=dt)
    rows = cap + 8
    cos, sin = rope_table(rd, 1e7, rows, dt)
    # pre-existing cache contents (already-roped keys), random
    kp = rn(g, num_pages, nkv, page_size, hd, dtype=dt)
    vp = rn(g, num_pages, nkv, page_size, hd, dtype=dt)
    dev = lambda t: t.to(DEV).contiguous()
    D = dict(qkv=dev(qkv), qn=dev(qn), kn=dev(kn), cos=dev(cos), sin=dev(sin), kp=dev(kp), vp=dev(vp),
             pt=dev(page_table), lens=dev(torch.tensor(lens, dtype=torch.int32)))
    D["q_buf"] = torch.empty(B * T, nh * hd, dtype=dt, device=DEV)
    D["out"] = torch.empty(B * T, nh * hd, dtype=dt, device=DEV)
    from lollm_b200 import kernels
    D["partial"] = torch.empty(kernels.attn_workspace_bytes(B, T, nh, hd, splits) // 4, device=DEV)
    D["bad"] = torch.zeros(1, dtype=torch.int32, device=DEV)
    d = L.AttnLayer()
    d.batch, d.tokens, d.n_heads, d.n_kv_heads, d.head_dim, d.rotary_dim = B, T, nh, nkv, hd, rd
    d.page_size, d.max_pages, d.num_pages = page_size, max_pages, num_pages
    d.dtype, d.eps, d.scale = L.dtype_code(dt), 1e-6, hd ** -0.5
    d.qkv, d.ld_qkv = D["qkv"].data_ptr(), n_qkv
    d.q_norm_w, d.k_norm_w = D["qn"].data_ptr(), D["kn"].data_ptr()
    d.rope_cos, d.rope_sin, d.rope_rows = D["cos"].data_ptr(), D["sin"].data_ptr(), rows
    d.k_pages, d.v_pages = D["kp"].data_ptr(), D["vp"].data_ptr()
    d.page_table, d.seq_lens = D["pt"].data_ptr(), D["lens"].data_ptr()
    d.q_buf, d.out, d.ld_out = D["q_buf"].data_ptr(), D["out"].data_ptr(), nh * hd
    d.partial, d.num_splits, d.bad_index = D["partial"].data_ptr(), splits, D["bad"].data_ptr()
    return d, D, dict(qkv=qkv, qn=qn, kn=kn, kp=kp, vp=vp, pt=page_table, cos=cos, sin=sin)


def _attn_reference(H, b, n, T, nh, nkv, hd, ps):
    """Oracle gated attention output (T, nh*hd) of sequence b with n cached keys: QK-norm and
    RoPE of the new rows, the pages' old keys + the new ones, offset-causal softmax, σ(gate);
    also returns the roped new keys (nkv, T, hd)."""
    qkv = H["qkv"].view(-1, T, H["qkv"].shape[-1])
    pos = torch.arange(n, n + T)
    cos, sin = H["cos"][pos], H["sin"][pos]
    qg = qkv[b, :, :2 * nh * hd].view(T, nh, 2 * hd)
    q = Q.rms_norm(qg[..., :hd], H["qn"], 1e-6).transpose(0, 1)      # (nh, T, hd)
    gate = qg[..., hd:].reshape(T, nh * hd)
    k = Q.rms_norm(qkv[b, :, 2 * nh * hd:2 * nh * hd + nkv * hd].view(T, nkv, hd), H["kn"], 1e-6).transpose(0, 1)
    v = qkv[b, :, 2 * nh * hd + nkv * hd:].view(T, nkv, hd).transpose(0, 1)
    q, k = Q.rope_rotate(q, cos, sin), Q.rope_rotate(k, cos, sin)
    if n > 0:
        pages = H["pt"][b, :math.ceil(n / ps)].long()
        kold = H["kp"][pages].permute(1, 0, 2, 3).reshape(nkv, -1, hd)[:, :n]
        vold = H["vp"][pages].permute(1, 0, 2, 3).reshape(nkv, -1, hd)[:, :n]
        kf, vf = torch.cat([kold, k], 1), torch.cat([vold, v], 1)
    else:
        kf, vf = k, v
    o = Q.offset_causal_attention(q, kf.repeat_interleave(nh // nkv, 0), vf.repeat_interleave(nh // nkv, 0))
    return o.transpose(0, 1).reshape(T, nh * hd) * torch.sigmoid(gate), k


@pytest.mark.parametrize("dt", DTS)
@pytest.mark.parametrize("shape", [(2, 4, 4, 2, 32, 8, [5, 17], 16, 3), (3, 4, 16, 2, 256, 64, [40, 1, 77], 16, 3),
                                   (2, 1, 8, 2, 64, 16, [100, 3], 16, 3), (1, 9, 4, 1, 128, 32, [0], 16, 3),
                                   (3, 4, 16, 2, 256, 64, [700, 1500, 64], 64, 4),
                                   (2, 16, 4, 2, 64, 16, [300, 129], 64, 2),
                                   # one split: the tensor-core kernel merges its key halves itself
                                   (3, 4, 16, 2, 256, 64, [700, 1500, 64], 64, 1),
                                   (2, 16, 4, 2, 64, 16, [300, 129], 64, 1),
                                   (1, 9, 4, 1, 128, 32, [0], 64, 1),
                                   (2, 1, 8, 2, 64, 16, [100, 3], 64, 1)])
def test_attention_matches_oracle(dt, shape):
    B, T, nh, nkv, hd, rd, lens, ps, splits = shape
    d, D, H = _attn_case(dt, B, T, nh, nkv, hd, rd, lens, page_size=ps, splits=splits)
    K().attn_prep(d)
    K().attn_verify(d)
    assert int(D["bad"]) == 0
    ps = d.page_size
    out = D["out"].cpu().view(B, T, nh * hd)
    kp_dev = D["kp"].cpu()
    for b in range(B):
        n = lens[b]
        o, k = _attn_reference(H, b, n, T, nh, nkv, hd, ps)
        close(out[b], o, dt)
        # the appended keys/values sit in the pages at positions n..n+T-1
        for t in range(T):
            p = H["pt"][b, (n + t) // ps]
            close(kp_dev[p, :, (n + t) % ps], k[:, t], dt)


# ─────────────────────────────────────────── selection ───────────────────────────────────────────

@pytest.mark.parametrize("dt", DTS)
def test_argmax_first_index_and_greedy_verify(dt):
    g = gen(6)
    B, T, V = 5, 4, 3001
    logits = rn(g, B * T, V, dtype=dt)
    logits[3, 17] = logits[3, 2900] = 50.0            # tie → first index
    ld = logits.to(DEV)
    out = torch.empty(B * T, dtype=torch.int64, device=DEV)
    K().argmax_rows(ld, out)
    want = logits.float().argmax(-1)
    assert torch.equal(out.cpu(), want) and int(out[3]) == 17
    drafts = torch.randint(0, V, (B, T - 1), generator=g)
    for b in range(B):  # plant matching prefixes of length b % T
        for i in range(b % T):
            drafts[b, i] = want[b * T + i]
    ids = torch.cat([torch.zeros(B, 1, dtype=torch.int64), drafts], 1).to(DEV)
    acc = torch.empty(B, dtype=torch.int32, device=DEV)
    nxt = torch.empty(B, dtype=torch.int64, device=DEV)
    amax = torch.empty(B * T, dtype=torch.int64, device=DEV)
    K().greedy_verify(ld, B, T, ids[:, 1:], T, acc, nxt, amax)
    for b in range(B):
        a, t = S.greedy_accept(want[b * T:(b + 1) * T], drafts[b])
        assert int(acc[b]) == a and int(nxt[b]) == t


@pytest.mark.parametrize("rows", [1, 3, 64, 256])
def test_argmax_vocab_rows_split_over_clusters(rows):
    """Few rows of a 151936-entry vocabulary are split over 2-8 CTAs per row; the result is
    torch's first-maximum index, including ties planted across chunk boundaries."""
    g = gen(16 + rows)
    V = 151936
    logits = rn(g, rows, V, dtype=torch.bfloat16)
    for r in range(rows):
        a, b = sorted(torch.randint(0, V, (2,), generator=g).tolist())
        logits[r, a] = logits[r, b] = 30.0 + r % 3           # tie → the smaller index
    logits[0, V - 1] = 40.0                                   # maximum in the ragged last chunk
    ld = logits.to(DEV)
    out = torch.empty(rows, dtype=torch.int64, device=DEV)
    K().argmax_rows(ld, out)
    assert torch.equal(out.cpu(), logits.float().argmax(-1))


def test_spec_sample_matches_oracle_off_near_ties():
    g = gen(7)
    B, k, V, temp = 16, 3, 2000, 0.8
    tl = rn(g, B * (k + 1), V, scale=2.0)
    dl = rn(g, B * k, V, scale=2.0)
    # make drafts plausible under q: sample them from q with fixed uniforms
    q = torch.softmax(dl / temp, -1).view(B, k, V)
    p = torch.softmax(tl / temp, -1).view(B, k + 1, V)
    ud, ua, ur = torch.rand(B, k, generator=g), torch.rand(B, k, generator=g), torch.rand(B, generator=g)
    drafts = torch.tensor([[S.inverse_cdf(q[b, i], ud[b, i]) for i in range(k)] for b in range(B)])
    ids = torch.cat([torch.zeros(B, 1, dtype=torch.int64), drafts], 1).to(DEV)
    acc = torch.empty(B, dtype=torch.int32, device=DEV)
    nxt = torch.empty(B, dtype=torch.int64, device=DEV)
    ws = torch.empty(4 * B * (k + 1) + 64, device=DEV)
    K().spec_sample(tl.to(DEV), dl.to(DEV), B, k, temp, ids[:, 1:], k + 1, ua.to(DEV), ur.to(DEV), acc, nxt, ws)
    checked = 0
    for b in range(B):
        a, t, margins = S.speculative_accept(p[b], q[b], drafts[b], ua[b], ur[b])
        if min(margins, default=1.0) < 1e-5:
            continue   # flagged near-tie: fp32 rounding may flip the decision
        resid = torch.clamp(p[b, a].double() - (q[b, a].double() if a < k else 0), min=0) if a < k else p[b, a].double()
        if S.cdf_margin(resid, ur[b]) < 1e-5:
            continue
        assert int(acc[b]) == a and int(nxt[b]) == t, (b, a, t, int(acc[b]), int(nxt[b]))
        checked += 1
    assert checked >= B - 2


def test_sample_rows_inverse_cdf():
    g = gen(8)
    R, V, temp = 12, 5000, 0.7
    lg = rn(g, R, V, scale=3.0)
    u = torch.rand(R, generator=g)
    out = torch.empty(R, dtype=torch.int64, device=DEV)
    ws = torch.empty(2 * R + 16, device=DEV)
    K().sample_rows(lg.to(DEV), temp, u.to(DEV), out, ws)
    for r in range(R):
        p = torch.softmax(lg[r] / temp, -1)
        if S.cdf_margin(p, u[r]) < 1e-5:
            continue
        assert int(out[r]) == S.inverse_cdf(p, u[r])
