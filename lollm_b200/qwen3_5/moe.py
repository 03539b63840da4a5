"""SparseMoeBlock — the qwen3_5_moe FFN on the qsp C ABI (`qsp_moe_ffn`).

Mirrors `SparseMoeBlock` / `FusedExperts` of the reference (src/qwen3_5_moe/blocks.py:347-421):
the routed experts stay fused exactly as the checkpoint stores them
(`experts.gate_up_proj` (E, 2·I, H), `experts.down_proj` (E, H, I)); the router, the shared
expert's gate (one row) and the shared expert's gate/up projections are stacked into one
weight `w_in` so a single GEMM reads the FFN input once for all of them (rows: router E,
shared gate 1, zero padding to a multiple of 8, shared gate_proj Is, shared up_proj Is).

Calling the block runs the whole FFN plus the residual add and the next RMSNorm that follow
it in the decoder layer (modeling_qwen3_5_moe.py:57-59), on the current stream, allocation
free (the caller passes a workspace of `workspace_bytes(tokens)` bytes).
"""

from __future__ import annotations

import ctypes as C

import torch

from .. import _lib as L
from .config import Qwen3_5Config


class SparseMoeBlock:
    def __init__(self, cfg: Qwen3_5Config, params: dict, pre: str, *, dtype, device):
        L.load()
        self.cfg, self.dtype, self.device = cfg, dtype, torch.device(device)
        E, H = cfg.num_experts, cfg.hidden_size
        self.E, self.H = E, H
        self.k, self.I, self.Is = cfg.num_experts_per_tok, cfg.moe_intermediate_size, cfg.shared_expert_intermediate_size
        g = lambda n: params[pre + n].to(device=self.device, dtype=dtype).contiguous()
        self.n_route = int(L.load().qsp_moe_router_rows(E, self.Is))
        w_in = torch.zeros(self.n_route + 2 * self.Is, H, dtype=dtype, device=self.device)
        w_in[:E] = g("mlp.gate.weight")
        if self.Is > 0:
            w_in[E] = g("mlp.shared_expert_gate.weight")[0]
            w_in[self.n_route:self.n_route + self.Is] = g("mlp.shared_expert.gate_proj.weight")
            w_in[self.n_route + self.Is:] = g("mlp.shared_expert.up_proj.weight")
            self.shared_down = g("mlp.shared_expert.down_proj.weight")
        else:
            self.shared_down = None
        self.w_in = w_in
        self.gate_up = g("mlp.experts.gate_up_proj")
        self.down = g("mlp.experts.down_proj")
        # when set (a device int32 [E] tensor), every call adds its per-expert token counts to it
        self.counts_probe = None

    def workspace_bytes(self, tokens: int) -> int:
        return int(L.load().qsp_moe_workspace_bytes(tokens, self.H, self.E, self.k, self.I, self.Is,
                                                     L.dtype_code(self.dtype)))

    def weight_bytes(self, expert_counts=None) -> int:
        """HBM bytes of the weights one call streams: every expert that received a token
        (all of them when `expert_counts` is None), the router/shared block."""
        per_expert = (self.gate_up[0].numel() + self.down[0].numel()) * self.gate_up.element_size()
        hit = self.E if expert_counts is None else int((expert_counts > 0).sum())
        dense = self.w_in.numel() + (0 if self.shared_down is None else self.shared_down.numel())
        return hit * per_expert + dense * self.w_in.element_size()

    def desc(self, xn, x, norm_w, y, eps, tokens, workspace, expert_counts=None) -> L.MoeLayer:
        for t in (xn, x, workspace):
            L.require_cuda(t, "SparseMoeBlock operand")
        d = L.MoeLayer()
        d.tokens, d.hidden, d.n_experts, d.top_k = tokens, self.H, self.E, self.k
        d.inter, d.shared_inter = self.I, self.Is
        d.norm_topk_prob = 1 if self.cfg.norm_topk_prob else 0
        d.dtype, d.eps = L.dtype_code(self.dtype), eps
        d.xn, d.ld_xn = xn.data_ptr(), xn.stride(0)
        d.w_in, d.gate_up, d.down = self.w_in.data_ptr(), self.gate_up.data_ptr(), self.down.data_ptr()
        d.shared_down = L.ptr(self.shared_down)
        d.x, d.ld_x = x.data_ptr(), x.stride(0)
        d.norm_w = L.ptr(norm_w)
        d.y, d.ld_y = (y.data_ptr(), y.stride(0)) if y is not None else (0, self.H)
        d.workspace, d.workspace_bytes = workspace.data_ptr(), workspace.numel() * workspace.element_size()
        d.expert_counts = L.ptr(expert_counts)
        return d

    def __call__(self, xn, x, norm_w, y, eps, tokens, workspace, expert_counts=None):
        """x[:tokens] += FFN(xn[:tokens]); y = RMSNorm(x)·(1+norm_w) when norm_w is given."""
        if expert_counts is None:
            expert_counts = self.counts_probe
        d = self.desc(xn, x, norm_w, y, eps, tokens, workspace, expert_counts)
        L.call("qsp_moe_ffn", C.byref(d), L.stream_handle())
