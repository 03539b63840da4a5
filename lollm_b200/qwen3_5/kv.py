"""Qwen3_5Cache — the family cache, paged and batched, with index rollback.

Same method surface as the reference's cache (src/qwen3_5/kv.py:20-58): `append_kv`,
`read_kv`, `linear_state`, `set_linear_state`, `advance`, `clone`, `nbytes`, `seen_tokens`.
What changes is the storage (the reference's docstring anticipates exactly this swap,
kv.py:1-14 / modeling_qwen3_5.py:8-11):

* full-attention layers keep K/V in fixed-size pages, [num_pages, n_kv, page_size, hd] per
  layer, addressed through a per-sequence page table, instead of a tensor grown by
  `torch.cat` (kv.py:26-33);
* every sequence has its own length (`seq_lens`, device int32) instead of one scalar
  `seen_tokens` (kv.py:23), so a batch can be ragged;
* GDN layers keep the fp32 recurrent state [B, Hv, dk, dv] (the reference layout) plus a
  ping-pong conv-input history and a token ring of prepared per-token inputs (`pending`,
  sized by the library). A speculative forward leaves its T tokens pending; `accept(keep)` keeps a prefix by index and the next
  call replays exactly those tokens — no `clone()` snapshot and no recompute
  (mtp.py:141,156-162 is what this replaces). `flush()` materialises pending updates.

All bookkeeping lives on the device, so a speculative step never syncs with the host.
"""

from __future__ import annotations

import math

import torch

from .. import kernels as K
from .. import _lib as L
from .config import Qwen3_5Config


class Qwen3_5Cache:
    def __init__(self, cfg: Qwen3_5Config, batch: int, max_len: int, *, dtype, device,
                 page_size: int = 64, max_spec_tokens: int = 8, num_pages: int | None = None,
                 page_table: torch.Tensor | None = None):
        self.cfg, self.batch, self.dtype, self.device = cfg, batch, dtype, torch.device(device)
        self.page_size, self.max_spec_tokens = page_size, max_spec_tokens
        self.max_pages = math.ceil(max_len / page_size)
        self.capacity = self.max_pages * page_size
        self.attn_slot = {l: i for i, l in enumerate(cfg.attn_layers)}
        self.gdn_slot = {l: i for i, l in enumerate(cfg.gdn_layers)}
        n_attn, n_gdn = len(self.attn_slot), len(self.gdn_slot)
        nkv, hd = cfg.num_key_value_heads, cfg.head_dim
        self.num_pages = num_pages or batch * self.max_pages
        dev = self.device
        self.k_pages = torch.zeros(n_attn, self.num_pages, nkv, page_size, hd, dtype=dtype, device=dev)
        self.v_pages = torch.zeros_like(self.k_pages)
        if page_table is None:
            page_table = torch.arange(batch * self.max_pages, dtype=torch.int32).view(batch, self.max_pages)
        if tuple(page_table.shape) != (batch, self.max_pages):
            raise RuntimeError(f"page_table must be {(batch, self.max_pages)}")
        if int(page_table.max()) >= self.num_pages or int(page_table.min()) < 0:
            raise RuntimeError("page_table entries out of range of the page pool")
        self.page_table = page_table.to(device=dev, dtype=torch.int32).contiguous()
        self.seq_lens = torch.zeros(batch, dtype=torch.int32, device=dev)
        Hv, dk, dv = cfg.linear_num_value_heads, cfg.linear_key_head_dim, cfg.linear_value_head_dim
        Kc = cfg.linear_conv_kernel_dim
        self.state = torch.zeros(n_gdn, batch, Hv, dk, dv, dtype=torch.float32, device=dev)
        self.conv_hist = torch.zeros(n_gdn, 2, batch, Kc - 1 + max_spec_tokens, cfg.conv_dim,
                                     dtype=dtype, device=dev)
        ring = K.gdn_pending_bytes(batch, cfg.linear_num_key_heads, Hv, dk, dv, max_spec_tokens, dtype)
        self.pending = torch.zeros(n_gdn, ring, dtype=torch.uint8, device=dev)
        self.replay_n = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.conv_off = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.parity = torch.zeros(1, dtype=torch.int32, device=dev)
        self.bad_index = torch.zeros(1, dtype=torch.int32, device=dev)
        # last forward's token count and mode (host-side, for accept() / flush())
        self.last_tokens = 0
        self.last_speculative = False
        # placeholder weights for a replay-only GDN launch (flush): never read at T == 0
        self._dummy = torch.zeros(max(Hv, dv, cfg.conv_dim * Kc, 64), dtype=dtype, device=dev)

    # ------------------------------------------------------------------ reference surface
    @property
    def seen_tokens(self):
        """Positions consumed so far (kv.py:23): an int when the batch is aligned, else a list."""
        lens = self.seq_lens.tolist()
        return lens[0] if len(set(lens)) == 1 else lens

    def advance(self, n: int):
        """seen_tokens += n for every sequence (kv.py:46-47). The model's forward already
        advances through `qsp_cache_finalize`; this is for callers that append by hand."""
        self.seq_lens += n

    def append_kv(self, layer: int, k: torch.Tensor, v: torch.Tensor):
        """Write post-RoPE k, v (B, n_kv, t, hd) at each sequence's next positions and return
        the full (K, V) as read_kv does (kv.py:26-33). Compatibility path, not the hot path:
        the forward appends inside `qsp_attn_prep`."""
        s = self.attn_slot[layer]
        B, _, t, _ = k.shape
        lens = self.seq_lens.long()
        for j in range(t):
            pos = lens + j
            page = self.page_table.long().gather(1, (pos // self.page_size)[:, None])[:, 0]
            slot = pos % self.page_size
            self.k_pages[s, page, :, slot] = k[:, :, j].to(self.dtype)
            self.v_pages[s, page, :, slot] = v[:, :, j].to(self.dtype)
        self.seq_lens += t
        return self.read_kv(layer)

    def read_kv(self, layer: int):
        """(K, V) as (B, n_kv, L, hd) when all lengths are equal, else a list of per-sequence
        (n_kv, L_b, hd) pairs; None before anything was written (kv.py:35-36)."""
        s = self.attn_slot[layer]
        lens = self.seq_lens.tolist()
        if max(lens) == 0:
            return None
        per = []
        for b, n in enumerate(lens):
            npg = math.ceil(n / self.page_size)
            pages = self.page_table[b, :npg].long()
            kk = self.k_pages[s, pages].permute(1, 0, 2, 3).reshape(self.cfg.num_key_value_heads, -1, self.cfg.head_dim)[:, :n]
            vv = self.v_pages[s, pages].permute(1, 0, 2, 3).reshape(self.cfg.num_key_value_heads, -1, self.cfg.head_dim)[:, :n]
            per.append((kk, vv))
        if len(set(lens)) == 1:
            return torch.stack([p[0] for p in per]), torch.stack([p[1] for p in per])
        return per

    def linear_state(self, layer: int):
        """(conv_state (B, conv_dim, K-1), recurrent_state (B, Hv, dk, dv) fp32) of a GDN layer,
        with any pending speculative updates applied first (kv.py:39-40)."""
        self.flush()
        s = self.gdn_slot[layer]
        p = int(self.parity.item())
        Kc = self.cfg.linear_conv_kernel_dim
        conv = self.conv_hist[s, p, :, :Kc - 1].transpose(1, 2)
        return conv, self.state[s]

    def set_linear_state(self, layer: int, conv: torch.Tensor, rec: torch.Tensor):
        """Overwrite a GDN layer's state (kv.py:42-43); pending updates are flushed first."""
        self.flush()
        s = self.gdn_slot[layer]
        p = int(self.parity.item())
        Kc = self.cfg.linear_conv_kernel_dim
        self.conv_hist[s, p, :, :Kc - 1] = conv.transpose(1, 2).to(self.dtype)
        self.state[s].copy_(rec.float())

    def clone(self):
        """Deep copy (kv.py:49-54). The speculative loop does not need it (index rollback)."""
        new = object.__new__(Qwen3_5Cache)
        for k, v in self.__dict__.items():
            setattr(new, k, v.clone() if isinstance(v, torch.Tensor) else (dict(v) if isinstance(v, dict) else v))
        return new

    def nbytes(self) -> int:
        """Bytes held by the cache tensors (kv.py:56-58)."""
        return sum(t.numel() * t.element_size() for t in
                   (self.k_pages, self.v_pages, self.state, self.conv_hist, self.pending))

    def check(self):
        """Raise RuntimeError if a kernel flagged this cache or the device since the last check:
        a position outside its sequence's pages (the page pool or the capacity exhausted), an
        accepted count out of range, a NaN logit, or a bounded wait that ran out. Kernels
        record these on the device without stopping the stream; this call synchronises and
        turns them into the reference's hard failure (weights.py:57-62 style RuntimeError)."""
        bad = int(self.bad_index.item())
        code = K.device_status(reset=True)
        if bad:
            self.bad_index.zero_()
            raise RuntimeError("qsp cache: a token position fell outside its sequence's pages "
                               f"(capacity {self.capacity} positions per sequence, {self.num_pages} pages)")
        if code:
            raise RuntimeError(f"qsp device status {code}: {K.DEVICE_CODES.get(code, 'a bounded wait ran out')}")

    # ------------------------------------------------------------------ speculative support
    def accept(self, accept_n: torch.Tensor):
        """Keep accept_n[b] + 1 of the last speculative forward's tokens (device int32 [B])."""
        if not self.last_speculative:
            raise RuntimeError("accept() follows a speculative forward")
        K.cache_accept(self.batch, self.last_tokens, accept_n, self.seq_lens, self.replay_n, self.conv_off)

    def flush(self):
        """Apply pending GDN updates to the stored state (a replay-only launch per layer)."""
        if not self.last_speculative:
            return
        cfg = self.cfg
        d = self._dummy
        for s in range(len(self.gdn_slot)):
            desc = self.gdn_desc(s, None, 0, 0, d, d, d, d, d, None, speculative=False)
            K.gdn_verify(desc)
        K.cache_finalize(self.batch, 0, False, self.seq_lens, self.replay_n, self.conv_off, self.parity)
        self.last_speculative = False
        self.last_tokens = 0

    def gdn_desc(self, slot, proj, ld_proj, tokens, conv_w, a_log, dt_bias, norm_w, out_ref,
                 out, speculative):
        cfg = self.cfg
        desc = L.GdnLayer()
        desc.batch, desc.tokens = self.batch, tokens
        desc.n_k_heads, desc.n_v_heads = cfg.linear_num_key_heads, cfg.linear_num_value_heads
        desc.head_k, desc.head_v = cfg.linear_key_head_dim, cfg.linear_value_head_dim
        desc.conv_kernel, desc.max_spec_tokens = cfg.linear_conv_kernel_dim, self.max_spec_tokens
        desc.speculative, desc.dtype, desc.eps = int(speculative), L.dtype_code(self.dtype), cfg.rms_norm_eps
        desc.proj = out_ref.data_ptr() if proj is None else proj.data_ptr()
        desc.ld_proj = (cfg.conv_dim + cfg.value_dim + 2 * cfg.linear_num_value_heads) if proj is None else ld_proj
        desc.conv_w, desc.a_log, desc.dt_bias, desc.norm_w = (conv_w.data_ptr(), a_log.data_ptr(),
                                                              dt_bias.data_ptr(), norm_w.data_ptr())
        desc.state = self.state[slot].data_ptr()
        desc.conv_hist = self.conv_hist[slot].data_ptr()
        desc.pending = self.pending[slot].data_ptr()
        desc.replay_n, desc.conv_off, desc.parity = (self.replay_n.data_ptr(), self.conv_off.data_ptr(),
                                                     self.parity.data_ptr())
        desc.out = out_ref.data_ptr() if out is None else out.data_ptr()
        desc.ld_out = cfg.value_dim if out is None else out.stride(0)
        return desc
