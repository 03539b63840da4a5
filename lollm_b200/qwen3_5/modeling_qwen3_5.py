"""Qwen3_5Model — the family forward, driven through the qsp C ABI on the GPU.

Contract of the reference (src/qwen3_5/modeling_qwen3_5.py:82-102):
    forward(input_ids, past=None, return_hidden=False) -> (logits, past[, hidden])
with `past` the family cache object and `hidden` the pre-final-norm residual stream the MTP
head consumes. Extensions, all keyword-only and off by default:
    speculative=True   leave this call's GDN updates pending so the caller can keep a prefix
                       of the T tokens by index (`past.accept(accept_n)`);
    copy_outputs=False return views of the internal activation buffers (the speculative
                       engine uses this; they are overwritten by the next call).

Per layer (modeling_qwen3_5.py:47-61), every box a C-ABI launch:
    [GDN: in_proj(qkv|z|b|a) GEMM → qsp_gdn_verify → out_proj GEMM + residual + RMSNorm]
  | [attn: q|k|v GEMM → qsp_attn_prep → qsp_attn_verify → o_proj GEMM + residual + RMSNorm]
    gate|up GEMM + SwiGLU → down GEMM + residual + next layer's input RMSNorm
  | (qwen3_5_moe layers where cfg.is_moe_layer(i), modeling_qwen3_5_moe.py:42-43)
    qsp_moe_ffn: router + experts + shared expert + residual + next RMSNorm
then the lm_head GEMM. Projections of one input are concatenated into one weight so each
reads the activation once; each residual add is fused with the RMSNorm that follows it.
"""

from __future__ import annotations

import math

import torch

from .. import kernels as K
from .. import _lib as L
from .config import Qwen3_5Config
from .kv import Qwen3_5Cache
from .moe import SparseMoeBlock


def rope_table(rotary_dim: int, theta: float, rows: int, dtype):
    """cos/sin (rows, rotary_dim) for positions 0..rows-1, built exactly as the reference's
    RoPE.cos_sin (blocks.py:166-173): fp32 inv_freq = 1/θ^(2i/rd), freqs = pos·inv_freq,
    duplicated halves, cos/sin in fp32, cast to the model dtype. Computed once on the host."""
    idx = torch.arange(0, rotary_dim, 2, dtype=torch.float32)
    inv = 1.0 / (theta ** (idx / rotary_dim))
    f = torch.arange(rows).float()[:, None] * inv[None, :]
    f = torch.cat([f, f], dim=-1)
    return f.cos().to(dtype), f.sin().to(dtype)


class _Workspace:
    """Activation buffers for one (batch, tokens) shape, reused across calls (and stable
    under CUDA-graph capture)."""

    def __init__(self, model: "Qwen3_5Model", B: int, T: int, num_splits: int):
        cfg, dt, dev = model.cfg, model.dtype, model.device
        M = B * T
        H = cfg.hidden_size
        n_in = cfg.conv_dim + cfg.value_dim + 2 * cfg.linear_num_value_heads
        n_qkv = 2 * cfg.num_attention_heads * cfg.head_dim + 2 * cfg.num_key_value_heads * cfg.head_dim
        e = lambda *s: torch.empty(*s, dtype=dt, device=dev)
        self.x = e(M, H)
        self.xn = e(M, H)
        self.proj = e(M, max(n_in, n_qkv))
        self.core = e(M, max(cfg.value_dim, cfg.num_attention_heads * cfg.head_dim))
        self.q_buf = e(M, cfg.num_attention_heads * cfg.head_dim)
        inter = cfg.intermediate_size
        self.gu = e(M, 2 * max(inter, 1))
        self.act = e(M, max(inter, 1))
        moe_ws = max([lw["moe"].workspace_bytes(M) for lw in model.layers if "moe" in lw] + [0])
        self.moe_ws = torch.empty(moe_ws, dtype=torch.uint8, device=dev) if moe_ws else None
        self._logits = None            # [M, vocab]: allocated on first use (a prompt prefill never needs it)
        self._M, self._V, self._e = M, cfg.vocab_size, e
        self.last_x = e(B, H)
        self.last_xn = e(B, H)
        self.last_logits = e(B, cfg.vocab_size)
        self.last_idx = torch.full((B,), T - 1, dtype=torch.int32, device=dev)
        self.num_splits = num_splits
        ws = K.attn_workspace_bytes(B, T, cfg.num_attention_heads, cfg.head_dim, num_splits)
        self.partial = torch.empty(max(ws // 4, 1), dtype=torch.float32, device=dev)

    @property
    def logits(self):
        if self._logits is None:
            self._logits = self._e(self._M, self._V)
        return self._logits


def attn_num_splits(capacity: int, n_seq_heads: int, sms: int = 148) -> int:
    """Key splits per (sequence, kv head) of the verify attention; the splits have a fixed
    length of capacity / splits keys, so short sequences of a ragged batch use fewer of them.
    Every work item (split × sequence × kv head) costs a fixed overhead, and one round of items
    over the SMs already balances the load when the sequences are about equally long, so a
    short context takes as many splits as fill the SMs once. Measured on B200 (64 sequences,
    2 kv heads, head dim 256, T = 4, L ~ U[2048, 2560]): 1 split 75.2 µs per call, 2 splits 81.5,
    3 splits 86.1, 5 splits 96.0. Long ragged contexts need more splits to balance: over
    configs[2]'s 1k–32k keys, 1024-key splits measured best (0.593 of measured HBM, against
    0.546 with 512 and 1536)."""
    by_len = 1 if capacity <= 4096 else math.ceil(capacity / 1024)
    by_fill = max(1, sms // max(n_seq_heads, 1))
    return max(1, min(max(by_len, by_fill), math.ceil(capacity / 32)))


class Qwen3_5Model:
    def __init__(self, cfg: Qwen3_5Config, params: dict, *, dtype=torch.bfloat16, device="cuda",
                 max_positions: int = 8192, page_size: int = 64, max_spec_tokens: int = 8):
        L.load()
        self.cfg, self.dtype, self.device = cfg, dtype, torch.device(device)
        if self.device.type != "cuda":
            raise RuntimeError("Qwen3_5Model runs on CUDA only (no CPU fallback)")
        self.page_size, self.max_spec_tokens = page_size, max_spec_tokens
        self.max_positions = max_positions
        dev = self.device
        g = lambda n: params[n].to(device=dev, dtype=dtype).contiguous()
        self.embed = g("model.embed_tokens.weight")
        tied = params.tied if hasattr(params, "tied") else \
            params["lm_head.weight"] is params["model.embed_tokens.weight"]
        self.lm_head = self.embed if tied else g("lm_head.weight")
        self.final_norm = g("model.norm.weight")
        self.layers = []
        for i in range(cfg.num_hidden_layers):
            p = f"model.layers.{i}."
            lw = {"type": cfg.layer_type(i), "in_norm": g(p + "input_layernorm.weight"),
                  "post_norm": g(p + "post_attention_layernorm.weight")}
            if cfg.is_moe_layer(i):
                lw["moe"] = SparseMoeBlock(cfg, params, p, dtype=dtype, device=dev)
            else:
                lw["w_gu"] = torch.cat([g(p + "mlp.gate_proj.weight"), g(p + "mlp.up_proj.weight")]).contiguous()
                lw["down"] = g(p + "mlp.down_proj.weight")
            if lw["type"] == "full_attention":
                a = p + "self_attn."
                lw["w_qkv"] = torch.cat([g(a + "q_proj.weight"), g(a + "k_proj.weight"),
                                         g(a + "v_proj.weight")]).contiguous()
                lw["q_norm"], lw["k_norm"] = g(a + "q_norm.weight"), g(a + "k_norm.weight")
                lw["o_proj"] = g(a + "o_proj.weight")
            else:
                a = p + "linear_attn."
                lw["w_in"] = torch.cat([g(a + "in_proj_qkv.weight"), g(a + "in_proj_z.weight"),
                                        g(a + "in_proj_b.weight"), g(a + "in_proj_a.weight")]).contiguous()
                lw["conv_w"] = g(a + "conv1d.weight").reshape(cfg.conv_dim, cfg.linear_conv_kernel_dim).contiguous()
                lw["a_log"], lw["dt_bias"] = g(a + "A_log"), g(a + "dt_bias")
                lw["norm_w"], lw["out_proj"] = g(a + "norm.weight"), g(a + "out_proj.weight")
            self.layers.append(lw)
        cos, sin = rope_table(cfg.rotary_dim, cfg.rope_theta, max_positions, dtype)
        self.rope_cos, self.rope_sin = cos.to(dev).contiguous(), sin.to(dev).contiguous()
        self._ws = {}

    # ------------------------------------------------------------------ helpers
    def new_cache(self, batch: int, max_len: int | None = None, **kw) -> Qwen3_5Cache:
        max_len = max_len or self.max_positions
        if max_len > self.max_positions:
            raise RuntimeError(f"max_len {max_len} exceeds the RoPE table ({self.max_positions})")
        return Qwen3_5Cache(self.cfg, batch, max_len, dtype=self.dtype, device=self.device,
                            page_size=kw.pop("page_size", self.page_size),
                            max_spec_tokens=kw.pop("max_spec_tokens", self.max_spec_tokens), **kw)

    def default_splits(self, B: int, cache: Qwen3_5Cache) -> int:
        """Key splits per (sequence, kv head) of the verify attention: `attn_num_splits`."""
        return attn_num_splits(cache.capacity, B * self.cfg.num_key_value_heads)

    def workspace(self, B: int, T: int, cache: Qwen3_5Cache) -> _Workspace:
        key = (B, T, cache.capacity)
        if key not in self._ws:
            self._ws[key] = _Workspace(self, B, T, self.default_splits(B, cache))
        return self._ws[key]

    def attn_desc(self, lw, cache: Qwen3_5Cache, slot: int, ws: _Workspace, B: int, T: int):
        cfg = self.cfg
        d = L.AttnLayer()
        d.batch, d.tokens = B, T
        d.n_heads, d.n_kv_heads, d.head_dim, d.rotary_dim = (cfg.num_attention_heads, cfg.num_key_value_heads,
                                                             cfg.head_dim, cfg.rotary_dim)
        d.page_size, d.max_pages, d.num_pages = cache.page_size, cache.max_pages, cache.num_pages
        d.dtype, d.eps, d.scale = L.dtype_code(self.dtype), cfg.rms_norm_eps, cfg.head_dim ** -0.5
        d.qkv, d.ld_qkv = ws.proj.data_ptr(), ws.proj.stride(0)
        d.q_norm_w, d.k_norm_w = lw["q_norm"].data_ptr(), lw["k_norm"].data_ptr()
        d.rope_cos, d.rope_sin, d.rope_rows = self.rope_cos.data_ptr(), self.rope_sin.data_ptr(), self.max_positions
        d.k_pages, d.v_pages = cache.k_pages[slot].data_ptr(), cache.v_pages[slot].data_ptr()
        d.page_table, d.seq_lens = cache.page_table.data_ptr(), cache.seq_lens.data_ptr()
        d.q_buf = ws.q_buf.data_ptr()
        d.out, d.ld_out = ws.core.data_ptr(), ws.core.stride(0)
        d.partial, d.num_splits = ws.partial.data_ptr(), ws.num_splits
        d.bad_index = cache.bad_index.data_ptr()
        return d

    # ------------------------------------------------------------------ forward
    @torch.no_grad()
    def forward(self, input_ids: torch.Tensor, past: Qwen3_5Cache | None = None,
                return_hidden: bool = False, *, speculative: bool = False,
                copy_outputs: bool = True):
        if input_ids.dim() != 2:
            raise RuntimeError("input_ids must be (batch, tokens)")
        B, T = input_ids.shape
        ids = input_ids.to(device=self.device, dtype=torch.int64).contiguous()
        cache = past if past is not None else self.new_cache(B)
        if cache.batch != B:
            raise RuntimeError(f"cache batch {cache.batch} != input batch {B}")
        if speculative and T > cache.max_spec_tokens:
            raise RuntimeError(f"speculative forward of {T} tokens > max_spec_tokens {cache.max_spec_tokens}")
        self._forward_into(ids, cache, B, T, speculative)
        ws = self.workspace(B, T, cache)
        logits = ws.logits.view(B, T, -1)
        hidden = ws.x.view(B, T, -1)
        if copy_outputs:
            logits, hidden = logits.clone(), hidden.clone()
        if return_hidden:
            return logits, cache, hidden
        return logits, cache

    __call__ = forward

    @torch.no_grad()
    def prefill_last(self, input_ids: torch.Tensor, past: Qwen3_5Cache):
        """Commit-all forward that computes logits only at each sequence's last position
        (what a prompt prefill needs). Returns views (logits (B, V), hidden (B, H))."""
        B, T = input_ids.shape
        ids = input_ids.to(device=self.device, dtype=torch.int64).contiguous()
        ws = self._forward_into(ids, past, B, T, False, last_only=True)
        return ws.last_logits, ws.last_x

    def _forward_into(self, ids, cache: Qwen3_5Cache, B: int, T: int, speculative: bool,
                      last_only: bool = False, trace: list | None = None):
        """The forward's launches into the workspace. `trace` (tests): a list that receives a
        copy of the residual stream after the embedding and after every mixer and FFN."""
        cfg = self.cfg
        ws = self.workspace(B, T, cache)
        M = B * T
        eps = cfg.rms_norm_eps
        K.embed(ids, self.embed, ws.x, rows=M, bad=cache.bad_index)
        K.rmsnorm(ws.x, self.layers[0]["in_norm"], ws.xn, eps, rows=M)
        if trace is not None:
            trace.append(ws.x[:M].clone())
        n_layers = len(self.layers)
        for i, lw in enumerate(self.layers):
            # ws.xn holds input_layernorm(x) of this layer (fused into the previous residual add)
            if lw["type"] == "full_attention":
                slot = cache.attn_slot[i]
                K.gemm(ws.xn, lw["w_qkv"], ws.proj, m=M)
                d = self.attn_desc(lw, cache, slot, ws, B, T)
                K.attn_prep(d)
                K.attn_verify(d)
                K.gemm_residual_rmsnorm(ws.core, lw["o_proj"], ws.x, lw["post_norm"], ws.xn, eps, m=M)
            else:
                slot = cache.gdn_slot[i]
                K.gemm(ws.xn, lw["w_in"], ws.proj, m=M)
                d = cache.gdn_desc(slot, ws.proj, ws.proj.stride(0), T, lw["conv_w"], lw["a_log"],
                                   lw["dt_bias"], lw["norm_w"], None, ws.core, speculative)
                K.gdn_verify(d)
                K.gemm_residual_rmsnorm(ws.core, lw["out_proj"], ws.x, lw["post_norm"], ws.xn, eps, m=M)
            if trace is not None:
                trace.append(ws.x[:M].clone())
            # residual add + the next norm: next layer's input_layernorm, or the final norm
            nxt = self.layers[i + 1]["in_norm"] if i + 1 < n_layers else (None if last_only else self.final_norm)
            if "moe" in lw:
                lw["moe"](ws.xn, ws.x, nxt, ws.xn, eps, M, ws.moe_ws)
            else:
                K.gemm_swiglu(ws.xn, lw["w_gu"], ws.act, ws.gu, m=M)
                if nxt is not None:
                    K.gemm_residual_rmsnorm(ws.act, lw["down"], ws.x, nxt, ws.xn, eps, m=M)
                else:
                    K.gemm(ws.act, lw["down"], ws.x, accumulate=True, m=M)
            if trace is not None:
                trace.append(ws.x[:M].clone())
        if last_only:
            K.select_rows(ws.x, B, T, ws.last_idx, ws.last_x)
            K.rmsnorm(ws.last_x, self.final_norm, ws.last_xn, eps, rows=B)
            K.gemm(ws.last_xn, self.lm_head, ws.last_logits, m=B)
        else:
            K.gemm(ws.xn, self.lm_head, ws.logits, m=M)
        K.cache_finalize(B, T, speculative, cache.seq_lens, cache.replay_n, cache.conv_off, cache.parity)
        cache.last_tokens, cache.last_speculative = T, speculative
        return ws
