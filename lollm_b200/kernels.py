"""Typed torch-tensor wrappers over the C ABI (include/qsp.h), launching on the current stream.

Tensors are torch-owned device memory; the wrappers check device, dtype and contiguity of
what they hand over and pass raw pointers. Nothing here computes on the CPU.
"""

from __future__ import annotations

import ctypes as C

import torch

from . import _lib as L


def _s():
    return L.stream_handle()


def _cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("qsp kernels take CUDA tensors only (no CPU fallback)")


def embed(ids: torch.Tensor, table: torch.Tensor, out: torch.Tensor, ids_stride: int = 1,
          rows: int | None = None, bad: torch.Tensor | None = None):
    _cuda(ids, table, out)
    assert ids.dtype == torch.int64
    n = ids.numel() // ids_stride if rows is None else rows
    L.call("qsp_embed", ids.data_ptr(), ids_stride, n, table.data_ptr(), table.shape[0],
           table.shape[1], out.data_ptr(), out.stride(0), L.ptr(bad), L.dtype_code(table.dtype), _s())


def rmsnorm(x, w, y, eps, rows=None):
    _cuda(x, w, y)
    n = x.shape[0] if rows is None else rows
    L.call("qsp_rmsnorm", x.data_ptr(), x.stride(0), w.data_ptr(), y.data_ptr(), y.stride(0), n,
           w.shape[0], eps, L.dtype_code(x.dtype), _s())


def add_rmsnorm(x, h, w, y, eps):
    _cuda(x, h, w, y)
    L.call("qsp_add_rmsnorm", x.data_ptr(), h.data_ptr(), w.data_ptr(), y.data_ptr(), x.shape[0],
           x.shape[1], eps, L.dtype_code(x.dtype), _s())


def swiglu(gu, y, inter, rows=None):
    _cuda(gu, y)
    n = gu.shape[0] if rows is None else rows
    L.call("qsp_swiglu", gu.data_ptr(), gu.stride(0), y.data_ptr(), y.stride(0), n, inter,
           L.dtype_code(gu.dtype), _s())


_gemm_ws = {}


def gemm_workspace(device) -> torch.Tensor:
    """One zero-initialised split-K workspace per device, shared by every GEMM launched on
    the (single) compute stream."""
    key = str(device)
    if key not in _gemm_ws:
        _gemm_ws[key] = torch.zeros(64 << 20, dtype=torch.uint8, device=device)
    return _gemm_ws[key]


def gemm(a, w, c, accumulate=False, m=None):
    """c[:m] (+)= a[:m] @ w.T (w is [n, k], nn.Linear layout)."""
    _cuda(a, w, c)
    if a.stride(-1) != 1 or w.stride(-1) != 1 or c.stride(-1) != 1:
        raise RuntimeError("gemm operands must be row-major with unit inner stride")
    mm = a.shape[0] if m is None else m
    n, k = w.shape
    ws = gemm_workspace(a.device)
    L.call("qsp_gemm", a.data_ptr(), a.stride(0), w.data_ptr(), w.stride(0), c.data_ptr(),
           c.stride(0), mm, n, k, L.dtype_code(a.dtype),
           L.QSP_GEMM_ACCUMULATE if accumulate else 0, ws.data_ptr(), ws.numel(), _s())


def gemm_residual_rmsnorm(a, w, x, norm_w, y, eps, m=None):
    """x[:m] += a[:m] @ w.T (bf16-rounded product), then y[:m] = RMSNorm(x[:m]) * (1 + norm_w)."""
    _cuda(a, w, x, norm_w, y)
    mm = a.shape[0] if m is None else m
    n, k = w.shape
    ws = gemm_workspace(a.device)
    L.call("qsp_gemm_residual_rmsnorm", a.data_ptr(), a.stride(0), w.data_ptr(), w.stride(0), x.data_ptr(),
           x.stride(0), norm_w.data_ptr(), y.data_ptr(), y.stride(0), mm, n, k, eps, L.dtype_code(a.dtype),
           ws.data_ptr(), ws.numel(), _s())


def gemm_swiglu(a, w_gu, act, gu_tmp, m=None):
    """act[:m] = silu(a @ w_gate.T) * (a @ w_up.T) with w_gu = [w_gate; w_up]."""
    _cuda(a, w_gu, act, gu_tmp)
    mm = a.shape[0] if m is None else m
    n2, k = w_gu.shape
    ws = gemm_workspace(a.device)
    L.call("qsp_gemm_swiglu", a.data_ptr(), a.stride(0), w_gu.data_ptr(), w_gu.stride(0), act.data_ptr(),
           act.stride(0), gu_tmp.data_ptr(), gu_tmp.stride(0), mm, n2 // 2, k, L.dtype_code(a.dtype),
           ws.data_ptr(), ws.numel(), _s())


def device_status(reset=True) -> int:
    import ctypes as C
    v = C.c_int32(0)
    L.call("qsp_device_status", C.byref(v), 1 if reset else 0)
    return int(v.value)


# device status codes (include/qsp.h)
DEV_BAD_ACCEPT, DEV_NAN_LOGITS, DEV_WAIT_PROBE = 401, 501, 901
DEVICE_CODES = {DEV_BAD_ACCEPT: "an accepted count outside [0, T-1] (clamped)",
                DEV_NAN_LOGITS: "a NaN logit in a sampled or argmax row",
                DEV_WAIT_PROBE: "the wait probe ran out (expected)"}


def wait_probe(polls: int, waited_ns: torch.Tensor | None = None):
    """Launch the bounded-wait probe: a wait that nothing ends, limited to `polls` polls; it
    records DEV_WAIT_PROBE in the device status and returns (test support)."""
    if waited_ns is not None:
        _cuda(waited_ns)
    L.call("qsp_wait_probe", int(polls), L.ptr(waited_ns), _s())


def gdn_verify(desc: L.GdnLayer):
    L.call("qsp_gdn_verify", C.byref(desc), _s())


def gdn_pending_bytes(batch, n_k_heads, n_v_heads, head_k, head_v, max_spec_tokens, dtype) -> int:
    """Bytes of one GDN layer's token ring (the `pending` buffer of qsp_gdn_verify)."""
    n = int(L.load().qsp_gdn_pending_bytes(batch, n_k_heads, n_v_heads, head_k, head_v, max_spec_tokens,
                                            L.dtype_code(dtype)))
    if n <= 0:
        raise RuntimeError("qsp_gdn_pending_bytes: invalid sizes")
    return n


def attn_prep(desc: L.AttnLayer):
    L.call("qsp_attn_prep", C.byref(desc), _s())


def attn_verify(desc: L.AttnLayer):
    L.call("qsp_attn_verify", C.byref(desc), _s())


def attn_workspace_bytes(batch, tokens, n_heads, head_dim, num_splits) -> int:
    return int(L.load().qsp_attn_workspace_bytes(batch, tokens, n_heads, head_dim, num_splits))


def mtp_single_token_attn(gate, gate_head_stride, v, out, n_heads, n_kv, hd, rows=None):
    _cuda(gate, v, out)
    n = out.shape[0] if rows is None else rows
    L.call("qsp_mtp_single_token_attn", gate.data_ptr(), gate.stride(0), gate_head_stride,
           v.data_ptr(), v.stride(0), out.data_ptr(), out.stride(0), n, n_heads, n_kv, hd,
           L.dtype_code(out.dtype), _s())


def select_rows(src, batch, tokens, index, dst):
    _cuda(src, index, dst)
    L.call("qsp_select_rows", src.data_ptr(), src.stride(0), batch, tokens, index.data_ptr(),
           dst.data_ptr(), dst.stride(0), dst.shape[1], L.dtype_code(src.dtype), _s())


def argmax_rows(logits, out, rows=None, out_stride=1, vocab=None):
    _cuda(logits, out)
    n = logits.shape[0] if rows is None else rows
    v = logits.shape[1] if vocab is None else vocab
    L.call("qsp_argmax_rows", logits.data_ptr(), logits.stride(0), n, v, out.data_ptr(),
           out_stride, L.dtype_code(logits.dtype), _s())


def greedy_verify(logits, batch, tokens, drafts, drafts_ld, accept_n, next_tok, argmax_out):
    _cuda(logits, accept_n, next_tok, argmax_out)
    L.call("qsp_greedy_verify", logits.data_ptr(), logits.stride(0), batch, tokens,
           logits.shape[1], L.ptr(drafts), drafts_ld, accept_n.data_ptr(), next_tok.data_ptr(),
           argmax_out.data_ptr(), None, L.dtype_code(logits.dtype), _s())


def spec_sample(target_logits, draft_logits, batch, k, temperature, drafts, drafts_ld,
                u_accept, u_resample, accept_n, next_tok, workspace):
    _cuda(target_logits, u_resample, accept_n, next_tok, workspace)
    L.call("qsp_spec_sample", target_logits.data_ptr(), target_logits.stride(0),
           L.ptr(draft_logits), 0 if draft_logits is None else draft_logits.stride(0), batch, k,
           target_logits.shape[1], float(temperature), L.ptr(drafts), drafts_ld, L.ptr(u_accept),
           u_resample.data_ptr(), accept_n.data_ptr(), next_tok.data_ptr(), workspace.data_ptr(),
           L.dtype_code(target_logits.dtype), _s())


def sample_rows(logits, temperature, u, out, workspace, rows=None, out_stride=1):
    _cuda(logits, out)
    n = logits.shape[0] if rows is None else rows
    L.call("qsp_sample_rows", logits.data_ptr(), logits.stride(0), n, logits.shape[1],
           float(temperature), L.ptr(u), out.data_ptr(), out_stride, L.ptr(workspace),
           L.dtype_code(logits.dtype), _s())


def select_workspace_bytes(rows, vocab) -> int:
    return int(L.load().qsp_select_workspace_bytes(rows, vocab))


def filter_workspace_bytes(rows, vocab) -> int:
    return int(L.load().qsp_filter_workspace_bytes(rows, vocab))


def sample_params(temperature=0.0, top_k=0, top_p=1.0, repetition_penalty=1.0, hist=None, hist_n=None,
                  step_ids=None, step_base=0) -> L.SampleParams:
    """qsp_sample_params for the filters of sample_next; hist [B, ·] / hist_n [B] is each
    sequence's token context, step_ids [B, ·] the tokens of the step being scored."""
    sp = L.SampleParams()
    sp.temperature, sp.top_k = float(temperature), int(top_k or 0)
    sp.top_p = float(top_p if top_p is not None else 1.0)
    sp.repetition_penalty = float(repetition_penalty)
    if hist is not None:
        _cuda(hist, hist_n)
        sp.hist, sp.hist_ld, sp.hist_n = hist.data_ptr(), hist.stride(0), hist_n.data_ptr()
    if step_ids is not None:
        _cuda(step_ids)
        sp.step_ids, sp.step_ld, sp.step_base = step_ids.data_ptr(), step_ids.stride(0), int(step_base)
    sp._keep = (hist, hist_n, step_ids)   # the struct holds raw pointers: keep the tensors alive
    return sp


def sample_filtered(logits, params: L.SampleParams, u, out, workspace, rows=None, rows_per_seq=1, out_stride=1):
    _cuda(logits, out, workspace)
    n = logits.shape[0] if rows is None else rows
    L.call("qsp_sample_filtered", logits.data_ptr(), logits.stride(0), n, rows_per_seq, logits.shape[1],
           C.byref(params), L.ptr(u), out.data_ptr(), out_stride, workspace.data_ptr(),
           workspace.numel() * workspace.element_size(), L.dtype_code(logits.dtype), _s())


def spec_sample_filtered(target_logits, draft_logits, batch, k, params: L.SampleParams, drafts, drafts_ld,
                         u_accept, u_resample, accept_n, next_tok, workspace):
    _cuda(target_logits, accept_n, next_tok, workspace)
    L.call("qsp_spec_sample_filtered", target_logits.data_ptr(), target_logits.stride(0), L.ptr(draft_logits),
           0 if draft_logits is None else draft_logits.stride(0), batch, k, target_logits.shape[1],
           C.byref(params), L.ptr(drafts), drafts_ld, L.ptr(u_accept), L.ptr(u_resample), accept_n.data_ptr(),
           next_tok.data_ptr(), workspace.data_ptr(), workspace.numel() * workspace.element_size(),
           L.dtype_code(target_logits.dtype), _s())


def cache_finalize(batch, tokens, speculative, seq_lens, replay_n, conv_off, parity):
    L.call("qsp_cache_finalize", batch, tokens, 1 if speculative else 0, seq_lens.data_ptr(),
           replay_n.data_ptr(), conv_off.data_ptr(), parity.data_ptr(), _s())


def cache_accept(batch, tokens, accept_n, seq_lens, replay_n, conv_off):
    L.call("qsp_cache_accept", batch, tokens, accept_n.data_ptr(), seq_lens.data_ptr(),
           replay_n.data_ptr(), conv_off.data_ptr(), _s())


def commit_tokens(batch, tokens, ids, accept_n, next_tok, out, n_out):
    L.call("qsp_commit_tokens", batch, tokens, ids.data_ptr(), accept_n.data_ptr(),
           next_tok.data_ptr(), out.data_ptr(), out.shape[1], n_out.data_ptr(), _s())
