"""qsp_attn_verify_static (split-KV partials in the library's fixed per-device scratch region,
no device allocation in the call) gives the same output as qsp_attn_verify with a caller
workspace, on two calls in a row, and refuses shapes beyond the region.

Self-contained on purpose: it must pass alone in a fresh process as well as after every
other test (the file name sorts it last)."""

import ctypes as C
import math

import pytest
import torch

from lollm_b200 import _lib as L

pytestmark = pytest.mark.gpu

DEV = "cuda"
TOL = {torch.float32: dict(rtol=1e-4, atol=1e-5), torch.bfloat16: dict(rtol=2e-2, atol=2e-2)}


def _case(dt, B, T, nh, nkv, hd, rd, lens, page_size, splits, seed=11):
    from lollm_b200.qwen3_5.modeling_qwen3_5 import rope_table
    g = torch.Generator().manual_seed(seed)
    rn = lambda *s, scale=1.0: (torch.randn(*s, generator=g) * scale).to(dt).to(DEV).contiguous()
    cap = max(lens) + T
    max_pages = math.ceil(cap / page_size) + 1
    num_pages = B * max_pages + 2
    pt = torch.randperm(num_pages, generator=g)[:B * max_pages].view(B, max_pages).int().to(DEV)
    n_qkv = 2 * nh * hd + 2 * nkv * hd
    rows = cap + 8
    cos, sin = rope_table(rd, 1e7, rows, dt)
    D = dict(qkv=rn(B * T, n_qkv), qn=rn(hd, scale=0.1), kn=rn(hd, scale=0.1),
             cos=cos.to(DEV).contiguous(), sin=sin.to(DEV).contiguous(),
             kp=rn(num_pages, nkv, page_size, hd), vp=rn(num_pages, nkv, page_size, hd), pt=pt,
             lens=torch.tensor(lens, dtype=torch.int32, device=DEV),
             q_buf=torch.empty(B * T, nh * hd, dtype=dt, device=DEV),
             out=torch.empty(B * T, nh * hd, dtype=dt, device=DEV),
             bad=torch.zeros(1, dtype=torch.int32, device=DEV))
    D["partial"] = torch.empty(L.load().qsp_attn_workspace_bytes(B, T, nh, hd, splits) // 4, device=DEV)
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
    return d, D


def _stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("dt,shape", [
    # bf16 tensor-core path at the verify shape of the 2B model (16 q / 2 kv heads, hd 256)
    (torch.bfloat16, (3, 4, 16, 2, 256, 64, [700, 1500, 64], 64, 4)),
    # fp32 CUDA-core path, ragged lengths including an empty context
    (torch.float32, (2, 4, 8, 2, 64, 16, [0, 301], 16, 3)),
])
def test_static_scratch_matches_caller_workspace(dt, shape):
    B, T, nh, nkv, hd, rd, lens, ps, splits = shape
    d, D = _case(dt, B, T, nh, nkv, hd, rd, lens, ps, splits)
    L.call("qsp_attn_prep", C.byref(d), _stream())
    L.call("qsp_attn_verify", C.byref(d), _stream())
    want = D["out"].clone()
    d.partial = None                       # ignored by the static variant
    for _ in range(2):                     # two calls in a row reuse the same region
        D["out"].fill_(float("nan"))
        L.call("qsp_attn_verify_static", C.byref(d), _stream())
        torch.cuda.synchronize()
        torch.testing.assert_close(D["out"].float().cpu(), want.float().cpu(), **TOL[dt])
    assert int(D["bad"]) == 0


def test_static_scratch_rejects_oversized_shapes():
    B, T, nh, hd = 3, 4, 16, 256
    d, D = _case(torch.bfloat16, B, T, nh, 2, hd, 64, [100, 200, 300], 64, 4)
    lib = L.load()
    splits = L.QSP_ATTN_STATIC_SCRATCH_BYTES // lib.qsp_attn_workspace_bytes(B, T, nh, hd, 1) + 1
    d.num_splits = splits
    D["out"].fill_(7.0)
    rc = lib.qsp_attn_verify_static(C.byref(d), _stream())
    assert rc == L.QSP_ERR_INVALID
    assert b"static region" in lib.qsp_last_error()
    torch.cuda.synchronize()
    assert bool((D["out"] == 7.0).all()), "a refused call must launch nothing"
