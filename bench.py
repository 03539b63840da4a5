"""Benchmark: generated tok/s of the qwen3_5 MTP speculative-decoding step (2B shape, bf16,
batch 64 per GPU, 2048-token prompts, k=3 recurrent MTP drafts, greedy), and the verify
step's fraction of the HBM roofline.

    python bench.py [--gpus N --steps K --warmup W]          # this implementation
    python bench.py --impl reference [...]                   # the installed reference, host CPU

One step = draft k tokens with the MTP head → verify [pending, d1..dk] through the 24-layer
hybrid stack → accept → keep a prefix by index → emit, for all sequences of this GPU. The
step runs as three CUDA graphs (draft / verify / accept+commit) so each phase is timed with
CUDA events on its stream. Inputs are far larger than L2 (4 GB of weights, 2.4 GB of GDN
state, 1.8 GB of KV per step), so no L2 flush is needed between steps.

Multi-GPU (torchrun): one process per GPU, each its own replica and its own 64 sequences
(weak scaling, the headline; sequences are independent, no collective on the data path).
At N > 1 the same run also times BASELINE's global batch of 64 split over the GPUs (64/N per
GPU, strong scaling) and reports it under "strong". Rank 0 prints one JSON line; times are
the max over ranks.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "generated tok/s (batch 64, k=3) at 1/2/4/8 B200; verify-step HBM % of peak"
UNIT = "tok/s"
# DRAM bytes (read + write) of one GDN layer update at the step's shape (64 sequences, 32 value
# heads of 128x128, T=4): gdn_chunk_kernel from an ncu capture of `bench.py --workload gdn`,
# which runs exactly that launch (147.91 MB read + 76.97 MB written; some state write-back is
# still in L2 when the kernel ends). gdn_prep_kernel's few MB are not included.
GDN_TRAFFIC_PER_LAUNCH = 224_875_008
GDN_TRAFFIC_SOURCE = "ncu dram__bytes_read.sum + dram__bytes_write.sum of gdn_chunk_kernel, bench.py --workload gdn"


# ─────────────────────────────────────────── helpers ───────────────────────────────────────────

def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"], d["bf16_tflops"], "measured"
    return 6650.0, 1590.0, "fallback"


def dist_setup():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import datetime
        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                             device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return ws, rank, local


def barrier(ws):
    if ws > 1:
        torch.distributed.barrier()


def reduce_max(x: float, ws: int) -> float:
    if ws == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def reduce_sum(x: float, ws: int) -> float:
    if ws == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.SUM)
    return float(t.item())


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 50 ms during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.idx = device_index
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.p = None

    def start(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                       "-i", str(self.idx), "-lms", "50"], stdout=self.f,
                                      stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None

    def stop(self):
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.p.kill()
        self.f.flush()
        rows = [l.strip().split(", ") for l in open(self.f.name) if l.strip()]
        sm = [float(r[1]) for r in rows if len(r) >= 9 and r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if len(r) >= 9 and r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows if len(r) >= 9 for i in range(4) if r[5 + i].strip() == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def verify_step_bytes(cfg, B, T, ctx_lens):
    """Algorithmic HBM bytes of one verify forward (the minimum any implementation moves):
    every weight except the embedding table once (lm_head counted once; the embedding gather
    is B·T rows), the K/V of every visible key once plus the T new rows written, the fp32
    GDN state read once and written once, the conv window read and written."""
    from lollm_b200.qwen3_5.weights import param_specs
    elt = 2
    w = 0
    for name, shape in param_specs(cfg, with_mtp=False):
        if name == "model.embed_tokens.weight":
            continue
        w += math.prod(shape) * elt
    if cfg.tie_word_embeddings:
        w += cfg.vocab_size * cfg.hidden_size * elt
    n_attn, n_gdn = len(cfg.attn_layers), len(cfg.gdn_layers)
    kv_row = n_attn * cfg.num_key_value_heads * cfg.head_dim * 2 * elt
    kv = sum(kv_row * (L + T) for L in ctx_lens) + kv_row * T * B
    state = 2 * n_gdn * B * cfg.linear_num_value_heads * cfg.linear_key_head_dim * cfg.linear_value_head_dim * 4
    conv = 2 * n_gdn * B * cfg.conv_dim * (cfg.linear_conv_kernel_dim - 1) * elt
    return {"weights": w, "kv": kv, "gdn_state": state, "conv": conv, "total": w + kv + state + conv}


# ─────────────────────────────────────────── CPU arm ───────────────────────────────────────────

REF_DIR = os.path.join(ROOT, "baseline", "_ref")


def stock_reference(cfg, raw_cfg, seed=0):
    """The installed reference (baseline/_ref): its own `qwen3_5.weights.load` and
    `qwen3_5.mtp.load_mtp` build the stock `Qwen3_5Model` and `MTP` modules from seeded
    random-init N(0, 0.02) weights (HF names), bf16 on the CPU. Returns (modules dict)."""
    if not os.path.isdir(os.path.join(REF_DIR, "qwen3_5")):
        raise FileNotFoundError(f"the reference is not installed under {REF_DIR}")
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    from qwen3_5 import mtp as RM
    from qwen3_5 import weights as RW
    from qwen3_5.kv import Qwen3_5Cache as RefCache
    from lollm_b200.qwen3_5.weights import random_init
    w = random_init(cfg, seed, dtype=torch.bfloat16, generator="torch")
    model = RW.load(raw_cfg, dict(w), "hf", device="cpu", dtype=torch.bfloat16)
    mtp = RM.load_mtp(model, dict(w), "hf", device="cpu", dtype=torch.bfloat16)
    del w
    return {"model": model, "mtp": mtp, "Cache": RefCache}


def stock_prefilled_cache(ref, cfg, batch, ctx, seed=1):
    """A stock `Qwen3_5Cache` holding `ctx` positions for every sequence: seeded random
    post-RoPE K/V (B, n_kv, ctx, hd) in bf16 for the attention layers, and (conv (B, C, K-1)
    bf16, recurrent (B, Hv, dk, dv) fp32 N(0, 0.1)) for the GDN layers. A 2048-token CPU
    prefill of 64 sequences would take hours; the step's cost does not depend on the values."""
    g = torch.Generator().manual_seed(seed)
    dt = torch.bfloat16
    cache = ref["Cache"](cfg.num_hidden_layers)
    for i in range(cfg.num_hidden_layers):
        if cfg.layer_type(i) == "full_attention":
            shp = (batch, cfg.num_key_value_heads, ctx, cfg.head_dim)
            cache.layers[i] = (torch.randn(*shp, generator=g).to(dt), torch.randn(*shp, generator=g).to(dt))
        else:
            cache.layers[i] = (torch.randn(batch, cfg.conv_dim, cfg.linear_conv_kernel_dim - 1, generator=g).to(dt),
                               torch.randn(batch, cfg.linear_num_value_heads, cfg.linear_key_head_dim,
                                           cfg.linear_value_head_dim, generator=g) * 0.1)
    cache.seen_tokens = ctx
    return cache


def stock_spec_step(ref, past, hidden_last, pending, k):
    """One greedy speculative step of the reference's `generate_mtp` (src/qwen3_5/mtp.py:
    127-162) on a batch, through the stock modules: k MTP drafts (mtp(hidden, emb) →
    lm_head → argmax; depth d > 1 feeds the previous depth's pre-norm MTP output, read off
    the head's final norm, and its token), `past.clone()` snapshot, one (B, k+1) verify
    forward, exact-match accept, and on a rejection the snapshot restored and the kept
    tokens re-run. The stock cache holds one length for the whole batch, so the batch keeps
    the common accepted prefix (every sequence commits a+1 tokens, a = the smallest
    acceptance). Returns (past, hidden_last (B,1,H), pending (B,), tokens committed)."""
    model, mtp = ref["model"], ref["mtp"]
    pre = {}
    hook = mtp.norm.register_forward_hook(lambda m, inp, out: pre.__setitem__("x", inp[0]))
    try:
        h, tok, drafts = hidden_last, pending, []
        for _ in range(k):
            emb = model.model.embed_tokens(tok[:, None])
            tok = model.lm_head(mtp(h, emb))[:, -1].argmax(-1)
            drafts.append(tok)
            h = pre["x"]
    finally:
        hook.remove()
    ids = torch.cat([pending[:, None], torch.stack(drafts, 1)], dim=1)
    snap = past.clone()
    logits, past, hidden = model(ids, past, return_hidden=True)
    tgt = logits.argmax(-1)                                   # (B, k+1)
    match = (ids[:, 1:] == tgt[:, :k]).int().cumprod(dim=1).sum(dim=1)
    a = int(match.min())
    if a == k:
        return past, hidden[:, k:k + 1], tgt[:, k], ids.shape[0] * (k + 1)
    _, past, h1 = model(ids[:, :a + 1], snap, return_hidden=True)
    return past, h1[:, -1:], tgt[:, a], ids.shape[0] * (a + 1)


def stock_reference_sample(cfg, batch, ctx, k, steps, warmup, budget_s):
    """Time the reference's own CPU path: the installed stock modules at `batch` sequences of
    context `ctx`, greedy, k drafts, with all host threads; at most `steps` timed steps,
    stopping once `budget_s` seconds have passed. Returns a dict, or None with the reason
    when the reference cannot be imported."""
    from lollm_b200.qwen3_5.config import QWEN35_2B
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    torch.set_grad_enabled(False)
    try:
        ref = stock_reference(cfg, QWEN35_2B)
    except Exception as e:  # noqa: BLE001
        return None, f"reference import failed: {type(e).__name__}: {e}"
    past = stock_prefilled_cache(ref, cfg, batch, ctx)
    g = torch.Generator().manual_seed(2)
    hidden = torch.randn(batch, 1, cfg.hidden_size, generator=g).to(torch.bfloat16)
    pending = torch.randint(0, cfg.vocab_size, (batch,), generator=g)
    for _ in range(warmup):
        past, hidden, pending, _ = stock_spec_step(ref, past, hidden, pending, k)
    toks, n, t0 = 0, 0, time.perf_counter()
    while n < steps:
        past, hidden, pending, c = stock_spec_step(ref, past, hidden, pending, k)
        toks += c
        n += 1
        if time.perf_counter() - t0 > budget_s:
            break
    secs = time.perf_counter() - t0
    sample = (f"{n} speculative steps (of {steps} asked, {budget_s:.0f} s budget; {warmup} warm-up) x {batch} "
              f"sequences at context {ctx}, k={k}, greedy: the installed reference's stock Qwen3_5Model / MTP / "
              f"Qwen3_5Cache (generate_mtp's draft, clone, verify, restore + recompute) in bf16 on {threads} host threads")
    return {"value": toks / secs, "unit": UNIT, "cores": threads, "kind": "reference", "sample": sample,
            "steps": n, "seconds": secs, "tokens": toks}, None


def run_reference_arm(args, cfg, ws, rank):
    """The reference's own CPU path, timed on the host cores: the installed stock modules
    (baseline/_ref) at the GPU arm's per-GPU batch and context, greedy, k drafts. It has no
    multi-GPU path: under torchrun only rank 0 runs (one CPU measurement per box) and the other
    ranks exit without work, so at N > 1 the line still describes one process serving
    `batch` sequences on the host cores."""
    if rank != 0:
        return
    warm = min(args.warmup, args.ref_warmup)
    cb, why = stock_reference_sample(cfg, args.batch, args.prompt, args.k, args.steps, warm, args.ref_budget_s)
    if cb is None:
        print(json.dumps({"impl": "reference", "unavailable": why}), flush=True)
        return
    n, secs, tps = cb.pop("steps"), cb.pop("seconds"), cb["value"]
    cb.pop("tokens")
    line = {"metric": METRIC, "value": tps, "unit": UNIT, "n_gpus": args.gpus, "steps": n,
            "warmup": warm, "ms_per_step": 1000 * secs / max(n, 1), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded random-init weights, random prefilled state)",
            "impl": "reference",
            "config": dict(config_block(args, cfg), global_batch=args.batch,
                           parallelism=f"one CPU process on the box's host cores (rank 0 of {args.gpus}; "
                                       "the reference has no multi-GPU path)"),
            "cpu_baseline": cb,
            "e2e": {"value": tps, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def config_block(args, cfg):
    return {"workload": "qwen3_5 2B-shape MTP speculative decode step (BASELINE configs[1])",
            "batch_per_gpu": args.batch, "global_batch": args.batch * args.gpus,
            "prompt_len": args.prompt, "k": args.k, "hidden": cfg.hidden_size,
            "layers": cfg.num_hidden_layers, "vocab": cfg.vocab_size, "sampling": "greedy",
            "parallelism": f"replicas x{args.gpus} (sequence-sharded, no collective)",
            "l2": "inputs larger than L2 (weights 4 GB + GDN state 2.4 GB per step)"}


# ─────────────────────────────────────────── GPU arm ───────────────────────────────────────────

def run_gpu_arm(args, cfg, ws, rank, local):
    from lollm_b200.qwen3_5 import MTP, Qwen3_5Model, SpecDecoder
    from lollm_b200.qwen3_5.weights import load_checkpoint, random_init
    dev = torch.device("cuda", local)
    t_setup = time.perf_counter()
    # identical replicas on every rank (same seed), generated on the device
    w = random_init(cfg, 0, dtype=torch.bfloat16, device=dev, generator="torch")
    params = load_checkpoint(cfg, w, device=dev)
    n_steps_total = args.warmup + 2 * args.steps + 4
    max_len = args.prompt + (n_steps_total + 2) * (args.k + 1) + 16
    model = Qwen3_5Model(cfg, params, dtype=torch.bfloat16, device=dev, max_positions=max_len + 64)
    mtp = MTP(model, params)
    del w, params
    dec = SpecDecoder(model, mtp, args.batch, args.k, max_len, out_capacity=n_steps_total * (args.k + 1) + 8)
    g = torch.Generator(device=dev)
    g.manual_seed(1000 + rank)
    prompts = torch.randint(0, cfg.vocab_size, (args.batch, args.prompt), generator=g, device=dev)
    torch.cuda.synchronize()
    t_pf = time.perf_counter()
    dec.prefill(prompts, chunk=args.prefill_chunk)
    torch.cuda.synchronize()
    prefill_s = time.perf_counter() - t_pf
    dec.step()                                       # one eager step (warms workspaces)
    graphs = capture_split(dec)
    full = capture_full(dec, graphs)
    launches_per_step = graph_kernel_nodes([full])
    stream = torch.cuda.current_stream()
    for _ in range(args.warmup):
        full.replay()
    torch.cuda.synchronize()

    if ws > 1:
        # every rank reached the timed region: a rank lost during set-up is named here, on the
        # host, before any rank enters the timed region's collectives
        from lollm_b200.ranks import PeerGuard
        PeerGuard(torch.distributed.distributed_c10d._get_default_store(), rank, ws,
                  timeout_s=300.0).checkpoint("timed")

    # ---------------- timed region: device-resident inputs
    n0 = int(dec.n_out.sum())
    ctx_lens = dec.cache.seq_lens.tolist()
    clocks = ClockSampler(local)
    barrier(ws)
    torch.cuda.synchronize()
    clocks.start()
    time.sleep(0.3)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if args.profile:
        torch.cuda.profiler.start()       # ncu --profile-from-start off: only the timed steps
    start.record(stream)
    for s in range(args.steps):
        full.replay()                     # one CUDA graph per step: draft, verify, accept
    end.record(stream)
    torch.cuda.synchronize()
    if args.profile:
        torch.cuda.profiler.stop()
    barrier(ws)
    clk = clocks.stop()
    elapsed_ms = start.elapsed_time(end)
    tokens = int(dec.n_out.sum()) - n0
    max_ms = reduce_max(elapsed_ms, ws)
    tot_tokens = reduce_sum(tokens, ws)
    value = tot_tokens / (max_ms / 1000.0)

    # ---------------- e2e: public API with host buffers (H2D pending ids, D2H committed tokens)
    # Every step: H2D of the pending ids from pinned host memory, D2H of the step's token block
    # and accepted counts into pinned host memory, D2H of the next pending ids (the next step's
    # H2D reads them back: stream order carries the round trip through host memory). The host
    # reads step s's counts once step s's copies have landed, while step s+1 runs (two pinned
    # buffers), so it never leaves the GPU idle waiting for the host.
    # (Host buffers are contiguous: a strided pinned view would make torch stage the copy
    # through pageable memory synchronously.)
    B, T = args.batch, args.k + 1
    h_ids = torch.empty(B, 1, dtype=torch.int64, pin_memory=True)
    h_acc = [torch.empty(B, dtype=torch.int32, pin_memory=True) for _ in range(2)]
    h_tok = [torch.empty(B, T, dtype=torch.int64, pin_memory=True) for _ in range(2)]
    landed = [torch.cuda.Event() for _ in range(2)]
    h_ids.copy_(dec.ids[:, :1].cpu())
    barrier(ws)
    torch.cuda.synchronize()
    e2e_tokens = 0
    es, ee = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    es.record(stream)
    for s in range(args.steps):
        j = s & 1
        dec.ids[:, :1].copy_(h_ids, non_blocking=True)
        h_tok[j].copy_(dec.ids, non_blocking=True)          # the token block this step verifies
        full.replay()
        h_acc[j].copy_(dec.accept_n, non_blocking=True)
        h_ids.copy_(dec.ids[:, :1], non_blocking=True)
        landed[j].record(stream)
        if s > 0:                                         # the previous step's result, on the host
            landed[j ^ 1].synchronize()
            e2e_tokens += int(h_acc[j ^ 1].sum()) + B
    landed[(args.steps - 1) & 1].synchronize()
    e2e_tokens += int(h_acc[(args.steps - 1) & 1].sum()) + B
    ee.record(stream)
    torch.cuda.synchronize()
    barrier(ws)
    e2e_ms = reduce_max(es.elapsed_time(ee), ws)
    e2e_value = reduce_sum(e2e_tokens, ws) / (e2e_ms / 1000.0)
    h2d = B * 1 * 8
    d2h = B * 4 + B * T * 8 + B * 8

    # ---------------- per-phase device time: the same steps replayed as three graphs with
    # events between them (after the timed region, on the live decoding state)
    n_ph = max(3, min(args.steps, 10))
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(n_ph)]
    for s in range(n_ph):
        replay_split(graphs, ev[s], stream)
    torch.cuda.synchronize()
    phase = {"draft": [], "verify": [], "accept": []}
    for e in ev:
        phase["draft"].append(e[0].elapsed_time(e[1]))
        phase["verify"].append(e[1].elapsed_time(e[2]))
        phase["accept"].append(e[2].elapsed_time(e[3]))
    verify_ms = statistics.mean(phase["verify"])

    # ---------------- roofline of the verify step (HBM-bound): algorithmic bytes / time
    hbm, tflops, src = peaks()
    vb = verify_step_bytes(cfg, B, T, ctx_lens)
    achieved = vb["total"] / (verify_ms / 1000.0) / 1e9
    acc_rate = (tokens / (args.steps * B) - 1.0) / args.k
    # ---------------- the dominant kernel, timed live inside the step (after the timed region)
    live = live_kernel_times(dec, graphs, max(3, min(args.steps, 10)))
    n_gdn, gdn_ms, gdn_tot = live["gdn_verify"]
    gdn_bytes = gdn_launch_bytes(cfg, B, T)
    gdn_achieved = gdn_bytes / (gdn_ms / 1000.0) / 1e9
    out = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": max_ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded random-init weights, uniform random prompt ids)",
        "config": config_block(args, cfg), "clocks": clk,
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": launches_per_step * args.steps,
        "roofline": {"kernel": "qsp_gdn_verify = gdn_prep_kernel + gdn_chunk_kernel (one GDN layer of the verify forward, live in the step)",
                     "bound": "hbm", "achieved": gdn_achieved, "peak": hbm, "unit": "GB/s",
                     "frac": gdn_achieved / hbm, "peak_source": src,
                     "traffic": GDN_TRAFFIC_PER_LAUNCH, "traffic_source": GDN_TRAFFIC_SOURCE,
                     "algorithmic_bytes_per_launch": gdn_bytes, "launches_per_step": n_gdn,
                     "ms_per_launch": gdn_ms},
        "step_roofline": {"kernel": "verify phase (24-layer forward, T=k+1, all kernels)", "bound": "hbm",
                          "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                          "algorithmic_bytes": vb},
        "live_kernels_ms_per_step": {LIVE_CLASSES[k]: {"launches": v[0], "ms_per_launch": v[1], "ms_per_step": v[2]}
                                     for k, v in live.items()},
        "live_kernels_note": LIVE_NOTE,
        "live_kernels_sum_ms": sum(v[2] for v in live.values()),
        "phases_ms": {k: statistics.mean(v) for k, v in phase.items()},
        "acceptance_rate": acc_rate, "tokens_per_step_per_seq": tokens / (args.steps * B),
        "prefill_s": prefill_s, "setup_s": time.perf_counter() - t_setup,
    }
    if ws > 1 and args.global_batch % ws == 0 and args.global_batch // ws != args.batch:
        del graphs, full, dec
        torch.cuda.empty_cache()
        out["strong"] = strong_scaling(args, cfg, model, mtp, ws, rank, local)
    return out


def strong_scaling(args, cfg, model, mtp, ws, rank, local):
    """The same step at a FIXED global batch (`--global-batch`, BASELINE's 64) split over the
    ranks: global_batch / N sequences per GPU (8 at N = 8, i.e. 32 verify rows). Timed like
    the headline (barrier + synchronize around K graph replays, max over ranks); reports the
    whole-job tok/s, the verify phase against its HBM roofline at that batch, and the live
    per-class kernel times that name the limiting kernel."""
    from lollm_b200.qwen3_5 import SpecDecoder
    dev = torch.device("cuda", local)
    B = args.global_batch // ws
    n_steps_total = args.warmup + args.steps + 4
    max_len = args.prompt + (n_steps_total + 2) * (args.k + 1) + 16
    dec = SpecDecoder(model, mtp, B, args.k, max_len, out_capacity=n_steps_total * (args.k + 1) + 8)
    g = torch.Generator(device=dev)
    g.manual_seed(2000 + rank)
    dec.prefill(torch.randint(0, cfg.vocab_size, (B, args.prompt), generator=g, device=dev), chunk=args.prefill_chunk)
    dec.step()
    graphs = capture_split(dec)
    full = capture_full(dec, graphs)
    stream = torch.cuda.current_stream()
    for _ in range(args.warmup):
        full.replay()
    n0 = int(dec.n_out.sum())
    ctx_lens = dec.cache.seq_lens.tolist()
    barrier(ws)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(args.steps):
        full.replay()
    end.record(stream)
    torch.cuda.synchronize()
    barrier(ws)
    max_ms = reduce_max(start.elapsed_time(end), ws)
    tokens = reduce_sum(int(dec.n_out.sum()) - n0, ws)
    n_ph = max(3, min(args.steps, 10))
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(n_ph)]
    for e in ev:
        replay_split(graphs, e, stream)
    torch.cuda.synchronize()
    verify_ms = statistics.mean(e[1].elapsed_time(e[2]) for e in ev)
    draft_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in ev)
    hbm, _, src = peaks()
    vb = verify_step_bytes(cfg, B, args.k + 1, ctx_lens)
    live = live_kernel_times(dec, graphs, n_ph)
    del graphs, full
    return {"global_batch": args.global_batch, "batch_per_gpu": B, "verify_rows_per_gpu": B * (args.k + 1),
            "value": tokens / (max_ms / 1000.0), "unit": UNIT, "ms_per_step": max_ms / args.steps,
            "phases_ms": {"draft": draft_ms, "verify": verify_ms},
            "verify_roofline": {"bound": "hbm", "achieved": vb["total"] / (verify_ms / 1000) / 1e9, "peak": hbm,
                                "unit": "GB/s", "frac": vb["total"] / (verify_ms / 1000) / 1e9 / hbm,
                                "peak_source": src, "algorithmic_bytes": vb["total"]},
            "live_kernels_ms_per_step": {LIVE_CLASSES[k]: {"launches": v[0], "ms_per_launch": v[1], "ms_per_step": v[2]}
                                         for k, v in live.items()},
            "scaling": "strong"}


def capture_split(dec):
    """Three CUDA graphs for one step: MTP drafting, the speculative verify forward, and
    accept + rollback-by-index + commit. Replayed back to back they are exactly dec.step()."""
    from lollm_b200 import kernels as K
    m, B, T, k = dec.model, dec.B, dec.T, dec.k

    def draft():
        dec.mtp.draft(dec.hidden_last, dec.ids, k)

    def verify():
        dec._ws = m._forward_into(dec.ids, dec.cache, B, T, True)

    def accept():
        ws = m.workspace(B, T, dec.cache)
        K.greedy_verify(ws.logits, B, T, dec.ids[:, 1:], T, dec.accept_n, dec.next_tok, dec.amax)
        dec.cache.accept(dec.accept_n)
        K.select_rows(ws.x, B, T, dec.accept_n, dec.hidden_last)
        K.commit_tokens(B, T, dec.ids, dec.accept_n, dec.next_tok, dec.out, dec.n_out)

    graphs = []
    capture_split.last_fns = (draft, verify, accept)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        draft(); verify(); accept()          # one eager warm-up step on the capture stream
    torch.cuda.current_stream().wait_stream(s)
    for fn in (draft, verify, accept):
        gph = torch.cuda.CUDAGraph(keep_graph=True)
        with torch.cuda.graph(gph):
            fn()
        gph.instantiate()
        graphs.append(gph)
    return graphs


def capture_full(dec, graphs):
    """The whole step (draft, verify, accept) as one CUDA graph: kernels at the phase
    boundaries keep their programmatic dependencies instead of waiting for a graph launch."""
    fns = capture_split.last_fns
    gph = torch.cuda.CUDAGraph(keep_graph=True)
    with torch.cuda.graph(gph):
        for fn in fns:
            fn()
    gph.instantiate()
    return gph


def graph_kernel_nodes(graphs) -> int:
    """Kernel nodes in the captured step graphs (every one is a libqsp kernel: the step calls
    no torch op that launches work), counted through the driver API."""
    import ctypes as C
    cu = C.CDLL("libcuda.so.1")
    total = 0
    for gph in graphs:
        h = C.c_void_p(gph.raw_cuda_graph())
        n = C.c_size_t(0)
        if cu.cuGraphGetNodes(h, None, C.byref(n)) != 0:
            raise RuntimeError("cuGraphGetNodes failed")
        nodes = (C.c_void_p * n.value)()
        if cu.cuGraphGetNodes(h, nodes, C.byref(n)) != 0:
            raise RuntimeError("cuGraphGetNodes failed")
        for i in range(n.value):
            t = C.c_int(-1)
            if cu.cuGraphNodeGetType(C.c_void_p(nodes[i]), C.byref(t)) != 0:
                raise RuntimeError("cuGraphNodeGetType failed")
            total += int(t.value == 0)          # CU_GRAPH_NODE_TYPE_KERNEL
    return total


LIVE_CLASSES = {"gdn_verify": "gdn_prep_kernel + gdn_chunk_kernel", "attn_verify": "attn_ws_kernel + attn_combine_kernel",
                "gemm": "qsp_gemm plain (in_proj, q|k|v, vocabulary)",
                "gemm_residual_rmsnorm": "qsp_gemm + residual/RMSNorm (out, o, down)",
                "gemm_swiglu": "qsp_gemm + SwiGLU (gate|up)"}


LIVE_NOTE = ("each class is timed between two events recorded around its launches inside the captured verify "
             "forward; an event between two kernels stops the next kernel from starting early (programmatic "
             "dependent launch), so these per-launch times are upper bounds and their sum exceeds phases_ms.verify. "
             "The qsp_gemm kernels are the planner's: at 256 rows gemm_pair_kernel (in_proj, q|k|v; gate|up with "
             "SwiGLU in its epilogue), gemm_pairp_kernel (vocabulary), gemm_tc_kernel split-K + "
             "splitk_residual_rmsnorm_kernel (out, o, down)")


def live_kernel_times(dec, graphs, steps):
    """Per-launch device time of the verify forward's kernel classes, measured inside the real
    step: the verify phase is captured once more with an external (timing) event recorded
    before and after every launch of each class, and the step (draft, instrumented verify,
    accept) is replayed `steps` times on the live decoding state. Returns
    {class: (launches per step, mean ms per launch, total ms per step)}."""
    from lollm_b200 import kernels as K
    m, B, T = dec.model, dec.B, dec.T
    pairs = []
    orig = {n: getattr(K, n) for n in LIVE_CLASSES}

    def wrap(name, fn):
        def timed(*a, **kw):
            e0 = torch.cuda.Event(enable_timing=True, external=True)
            e1 = torch.cuda.Event(enable_timing=True, external=True)
            e0.record()
            r = fn(*a, **kw)
            e1.record()
            pairs.append((name, e0, e1))
            return r
        return timed

    gph = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    try:
        for n, fn in orig.items():
            setattr(K, n, wrap(n, fn))
        with torch.cuda.stream(s):
            with torch.cuda.graph(gph, stream=s):
                dec._ws = m._forward_into(dec.ids, dec.cache, B, T, True)
    finally:
        for n, fn in orig.items():
            setattr(K, n, fn)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    acc = {}
    for _ in range(steps):
        graphs[0].replay()
        gph.replay()
        graphs[2].replay()
        torch.cuda.synchronize()
        for name, e0, e1 in pairs:
            acc.setdefault(name, []).append(e0.elapsed_time(e1))
    del gph
    out = {}
    for name, v in acc.items():
        n = len(v) // steps
        out[name] = (n, statistics.mean(v), sum(v) / steps)
    return out


def gdn_launch_bytes(cfg, B, T):
    """Algorithmic HBM bytes of one GDN verify launch: the fp32 state read and written once,
    the conv window read and written, the token rows of the projection read (q, k, v, z, a, b)
    and the gated output written."""
    Hv, dk, dv = cfg.linear_num_value_heads, cfg.linear_key_head_dim, cfg.linear_value_head_dim
    C, Vd = cfg.conv_dim, cfg.value_dim
    return (2 * B * Hv * dk * dv * 4 + 2 * B * C * (cfg.linear_conv_kernel_dim - 1) * 2
            + B * T * (C + Vd + 2 * Hv) * 2 + B * T * Vd * 2)


def replay_split(graphs, events=None, stream=None):
    if events is not None:
        events[0].record(stream)
    for i, gph in enumerate(graphs):
        gph.replay()
        if events is not None:
            events[i + 1].record(stream)


# ─────────────────────────────────────── isolated kernels ───────────────────────────────────────

def timed_loop(fn, steps, warmup, stream, between=None):
    """CUDA-event time per call (ms) of `steps` calls of fn (after `warmup`); `between` runs
    before each call. The calls are captured in one CUDA graph and replayed, so host launch
    overhead does not leak into the device time; returns [per-call ms] * steps."""
    for _ in range(warmup):
        if between: between()
        fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        with torch.cuda.graph(g, stream=side):
            for _ in range(steps):
                if between: between()
                fn()
    stream.wait_stream(side)
    torch.cuda.synchronize()
    g.replay()          # warm replay
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    g.replay()
    b.record(stream)
    torch.cuda.synchronize()
    per = a.elapsed_time(b) / steps
    return [per] * steps


def run_gdn_workload(args):
    """one GDN verify update over T=4 tokens for 64 sequences x 32 value
    heads (16 key heads), fp32 128x128 state per head, then a rollback to a random kept prefix
    by index. Units: one launch updates 64x32 head states."""
    from lollm_b200 import _lib as L
    from lollm_b200 import kernels as K
    dev = torch.device("cuda", 0)
    B, Hk, Hv, d, Kc, T = 64, 16, 32, 128, 4, 4
    C, Vd = 2 * Hk * d + Hv * d, Hv * d
    g = torch.Generator(device=dev); g.manual_seed(0)
    rnd = lambda *s: torch.randn(*s, generator=g, device=dev)
    state = rnd(B, Hv, d, d) * 0.1
    Ts = T                                   # max_spec_tokens as the model sets it: k + 1
    hist = torch.zeros(2, B, Kc - 1 + Ts, C, dtype=torch.bfloat16, device=dev)
    pending = torch.zeros(K.gdn_pending_bytes(B, Hk, Hv, d, d, Ts, torch.bfloat16), dtype=torch.uint8, device=dev)
    replay = torch.zeros(B, dtype=torch.int32, device=dev)
    coff = torch.zeros(B, dtype=torch.int32, device=dev)
    parity = torch.zeros(1, dtype=torch.int32, device=dev)
    lens = torch.zeros(B, dtype=torch.int32, device=dev)
    proj = rnd(B * T, C + Vd + 2 * Hv).to(torch.bfloat16)
    # decay exp(-softplus(a + dt_bias) * A), A ~ U[1, 16]: A_log = log(A)
    a_log = torch.log(1 + 15 * torch.rand(Hv, generator=g, device=dev)).to(torch.bfloat16)
    dt_bias = torch.zeros(Hv, dtype=torch.bfloat16, device=dev)
    conv_w = (rnd(C, Kc) * 0.5).to(torch.bfloat16)
    norm_w = torch.ones(d, dtype=torch.bfloat16, device=dev)
    out = torch.empty(B * T, Vd, dtype=torch.bfloat16, device=dev)
    desc = L.GdnLayer()
    desc.batch, desc.tokens, desc.n_k_heads, desc.n_v_heads, desc.head_k, desc.head_v = B, T, Hk, Hv, d, d
    desc.conv_kernel, desc.max_spec_tokens, desc.speculative, desc.dtype, desc.eps = Kc, Ts, 1, L.QSP_BF16, 1e-6
    desc.proj, desc.ld_proj = proj.data_ptr(), proj.stride(0)
    desc.conv_w, desc.a_log, desc.dt_bias, desc.norm_w = conv_w.data_ptr(), a_log.data_ptr(), dt_bias.data_ptr(), norm_w.data_ptr()
    desc.state, desc.conv_hist, desc.pending = state.data_ptr(), hist.data_ptr(), pending.data_ptr()
    desc.replay_n, desc.conv_off, desc.parity = replay.data_ptr(), coff.data_ptr(), parity.data_ptr()
    desc.out, desc.ld_out = out.data_ptr(), out.stride(0)
    acc_all = torch.randint(0, T, (args.warmup + args.steps + 1, B), generator=g, device=dev, dtype=torch.int32)
    it = {"i": 0}

    def between():   # rollback of the previous step to a random kept prefix (index only)
        K.cache_accept(B, T, acc_all[it["i"]], lens, replay, coff)
        it["i"] += 1

    def step():
        K.gdn_verify(desc)
        K.cache_finalize(B, T, True, lens, replay, coff, parity)

    stream = torch.cuda.current_stream()
    if args.profile:
        torch.cuda.profiler.start()
    ms = timed_loop(step, args.steps, args.warmup, stream, between)
    if args.profile:
        torch.cuda.profiler.stop()
    # kernel-only time (finalize is a 2 µs bookkeeping launch): time the GDN launch alone too
    ms_k = timed_loop(lambda: K.gdn_verify(desc), args.steps, 1, stream)
    hbm, _, src = peaks()
    algo = 2 * B * Hv * d * d * 4 + 2 * B * C * (Kc - 1) * 2 + B * T * (C + Vd + 2 * Hv) * 2 + B * T * Vd * 2
    t = statistics.mean(ms_k) / 1000
    return {"metric": "GDN verify update (64 seq x 32 heads, T=4) state GB/s", "value": algo / t / 1e9,
            "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": statistics.mean(ms), "higher_is_better": True, "dtype": "f32 state, bf16 io",
            "data": "synthetic (BASELINE configs[3] shapes)", "config": {"workload": "gdn (BASELINE configs[3])"},
            "roofline": {"kernel": "gdn_prep_kernel + gdn_chunk_kernel", "bound": "hbm", "achieved": algo / t / 1e9, "peak": hbm,
                         "unit": "GB/s", "frac": algo / t / 1e9 / hbm, "peak_source": src, "traffic": None,
                         "algorithmic_bytes_per_launch": algo}}


def run_attn_workload(args):
    """verify attention of T=4 queries x 16 heads (2 kv heads, hd 256)
    for 64 sequences with per-sequence context L ~ U[1024, 32768] over a paged bf16 cache."""
    from lollm_b200 import _lib as L
    from lollm_b200 import kernels as K
    from lollm_b200.qwen3_5.modeling_qwen3_5 import rope_table
    dev = torch.device("cuda", 0)
    B, T, nh, nkv, hd, rd, ps = 64, 4, 16, 2, 256, 64, 64
    lo, hi = (int(x) for x in args.attn_len.split(","))
    g = torch.Generator(device=dev); g.manual_seed(0)
    lens = torch.randint(lo, hi + 1 - T, (B,), generator=g, device=dev, dtype=torch.int32)
    max_pages = (hi + ps - 1) // ps
    # only the pages each sequence uses are allocated, in shuffled order (a paged pool)
    need = [(int(l) + T + ps - 1) // ps for l in lens.tolist()]
    num_pages = sum(need)
    perm = torch.randperm(num_pages, generator=g, device=dev).to(torch.int32)
    page_table = torch.zeros(B, max_pages, dtype=torch.int32, device=dev)
    o = 0
    for b, n in enumerate(need):
        page_table[b, :n] = perm[o:o + n]
        o += n
    kp = torch.empty(num_pages, nkv, ps, hd, dtype=torch.bfloat16, device=dev).normal_(generator=g)
    vp = torch.empty_like(kp).normal_(generator=g)
    qkv = torch.randn(B * T, 2 * nh * hd + 2 * nkv * hd, generator=g, device=dev).to(torch.bfloat16)
    qn = torch.zeros(hd, dtype=torch.bfloat16, device=dev); kn = torch.zeros_like(qn)
    cos, sin = rope_table(rd, 1e7, hi + 8, torch.bfloat16)
    cos, sin = cos.to(dev), sin.to(dev)
    if args.attn_split_len > 0:                  # fixed-length key splits of this many keys
        splits = max(1, (hi + args.attn_split_len - 1) // args.attn_split_len)
    else:                                        # the model's choice for this capacity and batch
        from lollm_b200.qwen3_5.modeling_qwen3_5 import attn_num_splits
        splits = attn_num_splits(max_pages * ps, B * nkv)
    q_buf = torch.empty(B * T, nh * hd, dtype=torch.bfloat16, device=dev)
    out = torch.empty(B * T, nh * hd, dtype=torch.bfloat16, device=dev)
    part = torch.empty(K.attn_workspace_bytes(B, T, nh, hd, splits) // 4, device=dev)
    d = L.AttnLayer()
    d.batch, d.tokens, d.n_heads, d.n_kv_heads, d.head_dim, d.rotary_dim = B, T, nh, nkv, hd, rd
    d.page_size, d.max_pages, d.num_pages, d.dtype, d.eps, d.scale = ps, max_pages, num_pages, L.QSP_BF16, 1e-6, 1 / 16
    d.qkv, d.ld_qkv, d.q_norm_w, d.k_norm_w = qkv.data_ptr(), qkv.stride(0), qn.data_ptr(), kn.data_ptr()
    d.rope_cos, d.rope_sin, d.rope_rows = cos.data_ptr(), sin.data_ptr(), hi + 8
    d.k_pages, d.v_pages, d.page_table, d.seq_lens = kp.data_ptr(), vp.data_ptr(), page_table.data_ptr(), lens.data_ptr()
    d.q_buf, d.out, d.ld_out, d.partial, d.num_splits, d.bad_index = (q_buf.data_ptr(), out.data_ptr(), out.stride(0),
                                                                     part.data_ptr(), splits, 0)
    K.attn_prep(d)
    stream = torch.cuda.current_stream()
    if args.profile:
        torch.cuda.profiler.start()
    ms = timed_loop(lambda: K.attn_verify(d), args.steps, args.warmup, stream)
    if args.profile:
        torch.cuda.profiler.stop()
    hbm, _, src = peaks()
    Ls = lens.tolist()
    algo = sum((l + T) * nkv * hd * 2 * 2 for l in Ls)
    t = statistics.mean(ms) / 1000
    return {"metric": f"verify attention (64 seq, T=4, L~U[{lo},{hi}]) KV GB/s", "value": algo / t / 1e9,
            "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": statistics.mean(ms), "higher_is_better": True, "dtype": "bf16",
            "data": "synthetic (BASELINE configs[2] shapes)",
            "config": {"workload": "attn (BASELINE configs[2] shapes)", "mean_L": sum(Ls) / B, "splits": splits},
            "roofline": {"kernel": "attn_ws_kernel + attn_combine_kernel", "bound": "hbm", "achieved": algo / t / 1e9,
                         "peak": hbm, "unit": "GB/s", "frac": algo / t / 1e9 / hbm, "peak_source": src,
                         "traffic": None, "algorithmic_bytes_per_launch": algo}}


def run_attn_compare_workload(args):
    """The verify attention of configs[2] (64 sequences, T=4, 16 q / 2 kv heads, hd 256,
    scale 1/16, causal over the 4 new rows) at EQUAL context lengths — the reference needs
    one length per batch — timed three ways on the same GPU:
      ours      qsp_attn_verify over the paged cache (GQA in the kernel);
      sdpa      the reference's `attention.torch_attention` (src/attention.py:43-51) on
                (B, 16, L+4, 256) K/V already expanded from 2 to 16 heads, as the reference's
                GatedAttention does before the call (src/qwen3_5/blocks.py:229);
      triton    the reference's `_triton_attn.flash_attention_kv` (src/_triton_attn.py) on
                the same expanded tensors (autotuned once before timing).
    The reference's GQA expansion (repeat_interleave of K and V, per call in the reference)
    is timed separately as `expand_ms` and not included in its attention time. HBM
    roofline for every impl: the unexpanded K/V bytes, Σ_b (L+T)·2·256·2·2.

    The reference's Triton kernel forms element offsets in 32-bit integers (b·stride_b with
    stride_b = H·(L+T)·D, src/_triton_attn.py:64-65): once B·H·(L+T)·D reaches 2^31 they wrap
    and the kernel reads outside its tensors (an illegal memory access here at L = 16384,
    B = 64). Both reference paths are therefore called on batch slices that stay below that
    bound (the reference would have to split the batch the same way), and their time is the
    sum over the slices."""
    from lollm_b200 import _lib as L
    from lollm_b200 import kernels as K
    from lollm_b200.qwen3_5.modeling_qwen3_5 import rope_table
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    dev = torch.device("cuda", 0)
    B, T, nh, nkv, hd, rd, ps = args.batch, 4, 16, 2, 256, 64, 64
    hbm, _, src = peaks()
    rows = []
    for Lc in (int(x) for x in args.attn_equal.split(",")):
        g = torch.Generator(device=dev); g.manual_seed(Lc)
        max_pages = (Lc + T + ps - 1) // ps
        num_pages = B * max_pages
        page_table = torch.arange(num_pages, dtype=torch.int32, device=dev).view(B, max_pages)
        kp = torch.empty(num_pages, nkv, ps, hd, dtype=torch.bfloat16, device=dev).normal_(generator=g)
        vp = torch.empty_like(kp).normal_(generator=g)
        qkv = torch.randn(B * T, 2 * nh * hd + 2 * nkv * hd, generator=g, device=dev).to(torch.bfloat16)
        qn = torch.zeros(hd, dtype=torch.bfloat16, device=dev); kn = torch.zeros_like(qn)
        cos, sin = rope_table(rd, 1e7, Lc + 8, torch.bfloat16)
        cos, sin = cos.to(dev), sin.to(dev)
        lens = torch.full((B,), Lc, dtype=torch.int32, device=dev)
        splits = max(1, (Lc + 511) // 512)
        q_buf = torch.empty(B * T, nh * hd, dtype=torch.bfloat16, device=dev)
        out = torch.empty(B * T, nh * hd, dtype=torch.bfloat16, device=dev)
        part = torch.empty(K.attn_workspace_bytes(B, T, nh, hd, splits) // 4, device=dev)
        d = L.AttnLayer()
        d.batch, d.tokens, d.n_heads, d.n_kv_heads, d.head_dim, d.rotary_dim = B, T, nh, nkv, hd, rd
        d.page_size, d.max_pages, d.num_pages, d.dtype, d.eps, d.scale = ps, max_pages, num_pages, L.QSP_BF16, 1e-6, 1 / 16
        d.qkv, d.ld_qkv, d.q_norm_w, d.k_norm_w = qkv.data_ptr(), qkv.stride(0), qn.data_ptr(), kn.data_ptr()
        d.rope_cos, d.rope_sin, d.rope_rows = cos.data_ptr(), sin.data_ptr(), Lc + 8
        d.k_pages, d.v_pages, d.page_table, d.seq_lens = kp.data_ptr(), vp.data_ptr(), page_table.data_ptr(), lens.data_ptr()
        d.q_buf, d.out, d.ld_out, d.partial, d.num_splits, d.bad_index = (q_buf.data_ptr(), out.data_ptr(), out.stride(0),
                                                                         part.data_ptr(), splits, 0)
        K.attn_prep(d)                       # appends the T new keys at L..L+T-1, writes q_buf
        torch.cuda.synchronize()
        stream = torch.cuda.current_stream()
        ours = statistics.mean(timed_loop(lambda: K.attn_verify(d), args.steps, args.warmup, stream))
        # the same tensors in the reference's layout: q (B, nh, T, hd) post-norm/RoPE,
        # K/V (B, nkv, L+T, hd) contiguous, then expanded to nh heads
        Lt = Lc + T
        kc = kp.view(B, max_pages, nkv, ps, hd).permute(0, 2, 1, 3, 4).reshape(B, nkv, max_pages * ps, hd)[:, :, :Lt].contiguous()
        vc = vp.view(B, max_pages, nkv, ps, hd).permute(0, 2, 1, 3, 4).reshape(B, nkv, max_pages * ps, hd)[:, :, :Lt].contiguous()
        del kp, vp
        q = q_buf.view(B, T, nh, hd).transpose(1, 2).contiguous()
        n_rep = nh // nkv
        expand = lambda: (kc.repeat_interleave(n_rep, dim=1), vc.repeat_interleave(n_rep, dim=1))
        ke, ve = expand()
        del ke, ve
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        ke, ve = expand()                    # eager: a captured loop would hold one copy per call
        e1.record(stream)
        torch.cuda.synchronize()
        exp_ms = e0.elapsed_time(e1)
        import attention as RA
        per = max(1, min(B, ((1 << 31) - 1) // (nh * Lt * hd)))          # sequences per reference call
        slices = [(i, min(B, i + per)) for i in range(0, B, per)]
        print(f"attn_compare L={Lc}: reference calls of {per} sequences", file=sys.stderr, flush=True)

        def sliced(fn):
            return lambda: [fn(q[i:j], ke[i:j], ve[i:j]) for i, j in slices]

        o_ref = torch.cat(sliced(RA.torch_attention)())
        sdpa = statistics.mean(timed_loop(sliced(RA.torch_attention), args.steps, args.warmup, stream))
        # agreement of ours with the reference's SDPA output (ungated: ours applies σ(gate))
        gate = torch.sigmoid(qkv[:, :2 * nh * hd].reshape(B, T, nh, 2 * hd)[..., hd:].float())
        ours_o = out.view(B, T, nh, hd).float()
        ref_o = o_ref.transpose(1, 2).float() * gate
        err = float((ours_o - ref_o).abs().max())
        tri, tri_err = None, None
        try:
            from _triton_attn import flash_attention_kv
            o_tri = torch.cat(sliced(flash_attention_kv)())   # autotune + compile outside the timing
            torch.cuda.synchronize()
            tri = statistics.mean(timed_loop(sliced(flash_attention_kv), args.steps, args.warmup, stream))
            tri_err = float((o_tri.float() - o_ref.float()).abs().max())
        except Exception as e:  # noqa: BLE001
            tri = f"failed: {type(e).__name__}: {str(e)[:200]}"
        algo = B * Lt * nkv * hd * 2 * 2
        gbs = lambda ms: algo / (ms / 1000) / 1e9 if isinstance(ms, float) else None
        rows.append({"L": Lc, "splits": splits, "ref_sequences_per_call": per, "ours_ms": ours, "sdpa_ms": sdpa,
                     "triton_ms": tri,
                     "expand_ms": exp_ms, "ours_frac": gbs(ours) / hbm, "sdpa_frac": gbs(sdpa) / hbm,
                     "triton_frac": (gbs(tri) / hbm) if isinstance(tri, float) else None,
                     "max_abs_diff_ours_vs_sdpa": err, "max_abs_diff_triton_vs_sdpa": tri_err,
                     "algorithmic_bytes": algo})
        del ke, ve, kc, vc, q, o_ref, part
        torch.cuda.empty_cache()
    return {"metric": "verify attention at equal lengths: ours vs the reference's SDPA and Triton kernels",
            "unit": "ms", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "higher_is_better": False,
            "dtype": "bf16", "data": "synthetic (BASELINE configs[2] shapes, equal lengths per batch)",
            "config": {"workload": "attn_compare", "batch": B, "T": T, "heads": f"{nh}q/{nkv}kv", "head_dim": hd},
            "peak_gbs": hbm, "peak_source": src, "rows": rows}


def moe_step_bytes(cfg, model, B, T, ctx_lens, expert_hits):
    """Algorithmic HBM bytes of one verify forward of the MoE model: the dense weights (every
    projection, norms, the lm_head once; not the embedding table), the experts hit in each
    layer (`expert_hits[i]` of them, gate|up + down), the K/V of every visible key plus the T
    new rows, the GDN state read + written and the conv window read + written."""
    elt = 2
    w = 0
    E = cfg.num_experts
    per_expert = (2 * cfg.moe_intermediate_size * cfg.hidden_size + cfg.hidden_size * cfg.moe_intermediate_size) * elt
    from lollm_b200.qwen3_5.weights import param_specs
    for name, shape in param_specs(cfg, with_mtp=False):
        if name == "model.embed_tokens.weight" or ".mlp.experts." in name:
            continue
        w += math.prod(shape) * elt
    if cfg.tie_word_embeddings:
        w += cfg.vocab_size * cfg.hidden_size * elt
    experts = sum(expert_hits) * per_expert
    n_attn, n_gdn = len(cfg.attn_layers), len(cfg.gdn_layers)
    kv_row = n_attn * cfg.num_key_value_heads * cfg.head_dim * 2 * elt
    kv = sum(kv_row * (L + T) for L in ctx_lens) + kv_row * T * B
    state = 2 * n_gdn * B * cfg.linear_num_value_heads * cfg.linear_key_head_dim * cfg.linear_value_head_dim * 4
    conv = 2 * n_gdn * B * cfg.conv_dim * (cfg.linear_conv_kernel_dim - 1) * elt
    return {"dense_weights": w, "experts": experts, "kv": kv, "gdn_state": state, "conv": conv,
            "total": w + experts + kv + state + conv}


def run_moe_step_workload(args, ws, rank, local):
    """the qwen3_5_moe shape (48 layers, 512 experts top-10 + a shared
    expert) in bf16, stochastic speculative decoding at temperature 0.8 with seeded uniforms,
    k=3, 4096-token prompts, `--moe-batch` (256) sequences sharded over the ranks.

    The ~162 GB of weights are generated on the device one tensor at a time (StreamingParams);
    what is left of the GPU holds the state of one resident WAVE of sequences (KV, GDN state,
    conv windows) — about 200 MB per sequence at 4.6k positions — so a rank's sequences run in
    waves: prefill a wave, run its steps, drop its state, next wave. Each wave's steps are one
    CUDA graph replayed with fresh uniforms copied in before every replay. Timed: K steps per
    wave (CUDA events around the replays); value = committed tokens of all waves of all ranks ÷
    the max over ranks of the summed wave times."""
    from lollm_b200.qwen3_5 import MTP, Qwen3_5Model, SpecDecoder
    from lollm_b200.qwen3_5.config import QWEN35_MOE, Qwen3_5Config
    from lollm_b200.qwen3_5.weights import StreamingParams
    dev = torch.device("cuda", local)
    raw = json.loads(json.dumps(QWEN35_MOE))
    if args.moe_layers:
        tc = raw["text_config"]
        tc["num_hidden_layers"] = args.moe_layers
        tc["layer_types"] = tc["layer_types"][:args.moe_layers]
    cfg = Qwen3_5Config.from_hf(raw)
    t0 = time.perf_counter()
    k, T = args.k, args.k + 1
    n_total = args.warmup + args.steps + 2
    max_len = args.moe_prompt + (n_total + 2) * T + 16
    model = Qwen3_5Model(cfg, StreamingParams.random(cfg, 0, device=dev), dtype=torch.bfloat16, device=dev,
                         max_positions=max_len + 64)
    mtp = MTP(model, StreamingParams.random(cfg, 0, device=dev))
    torch.cuda.synchronize()
    build_s = time.perf_counter() - t0
    weight_gb = torch.cuda.memory_allocated(dev) / 1e9
    per_rank = args.moe_batch // ws
    # one sequence's resident state at max_len positions (KV pages, GDN state, conv ring, token
    # ring), measured on a 1-sequence cache so nothing is estimated
    probe = model.new_cache(1, max_len, max_spec_tokens=max(T, 2))
    per_seq = probe.nbytes()
    del probe
    free, _ = torch.cuda.mem_get_info(dev)
    reserve = int(args.moe_reserve_gb * 1e9)
    fit = max(8, int((free - reserve) // per_seq) // 8 * 8)
    n_waves = math.ceil(per_rank / min(per_rank, fit))
    wave = min(fit, math.ceil(per_rank / n_waves / 8) * 8)      # balanced waves
    stream = torch.cuda.current_stream()
    tot_tokens, tot_ms, verify_ms, prefill_s, acc_steps = 0, 0.0, [], 0.0, []
    gen = torch.Generator(device=dev)
    hits = torch.zeros(cfg.num_experts, dtype=torch.int32, device=dev)
    bytes_rows = []
    for wv in range(n_waves):
        B = min(wave, per_rank - wv * wave)
        gen.manual_seed(10_000 * rank + wv)
        dec = SpecDecoder(model, mtp, B, k, max_len, temperature=args.moe_temperature,
                          out_capacity=n_total * T + 8)
        U = {"draft": torch.rand(n_total + 2, B, k, generator=gen, device=dev),
             "accept": torch.rand(n_total + 2, B, k, generator=gen, device=dev),
             "resample": torch.rand(n_total + 2, B, generator=gen, device=dev)}
        dec.u = {key: v[0].clone() for key, v in U.items()}
        prompts = torch.randint(0, cfg.vocab_size, (B, args.moe_prompt), generator=gen, device=dev)
        torch.cuda.synchronize()
        tp = time.perf_counter()
        dec.prefill(prompts, chunk=args.prefill_chunk, u_first=torch.rand(B, generator=gen, device=dev))
        torch.cuda.synchronize()
        prefill_s += time.perf_counter() - tp
        del prompts
        graph = dec.capture(warmup=1)
        si = [1]

        def feed():
            for key, v in U.items():
                dec.u[key].copy_(v[si[0]])
            si[0] += 1

        for _ in range(args.warmup):
            feed()
            graph.replay()
        ctx_lens = dec.cache.seq_lens.tolist()
        n0 = int(dec.n_out.sum())
        barrier(ws)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            feed()
            graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        tot_ms += e0.elapsed_time(e1)
        tot_tokens += int(dec.n_out.sum()) - n0
        acc_steps.append((int(dec.n_out.sum()) - n0) / (args.steps * B))
        # verify phase alone (same wave state), with the experts each layer hit
        ws_ = model.workspace(B, T, dec.cache)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        dec.mtp.draft(dec.hidden_last, dec.ids, k, dec.temperature, dec.u["draft"])
        hits.zero_()
        counts = []
        for lw in model.layers:
            c = torch.zeros(cfg.num_experts, dtype=torch.int32, device=dev)
            lw["moe"].counts_probe = c
            counts.append(c)
        ev[0].record(stream)
        model._forward_into(dec.ids, dec.cache, B, T, True)
        ev[1].record(stream)
        torch.cuda.synchronize()
        verify_ms.append(ev[0].elapsed_time(ev[1]))
        for lw in model.layers:
            lw["moe"].counts_probe = None
        expert_hits = [int((c > 0).sum()) for c in counts]
        bytes_rows.append(moe_step_bytes(cfg, model, B, T, ctx_lens, expert_hits))
        dec.cache.accept(torch.zeros(B, dtype=torch.int32, device=dev))
        del dec, graph, U, ws_
        model._ws.clear()
        mtp._ws.clear()
        torch.cuda.empty_cache()
    max_ms = reduce_max(tot_ms, ws)
    all_tokens = reduce_sum(tot_tokens, ws)
    hbm, _, src = peaks()
    vb = bytes_rows[0]
    v_ms = verify_ms[0]
    return {"metric": "generated tok/s, qwen3_5_moe 48-layer shape, stochastic spec decode (batch 256, k=3, T=0.8)",
            "value": all_tokens / (max_ms / 1000.0), "unit": UNIT, "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": max_ms / (args.steps * n_waves), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded random-init N(0,0.02) weights generated on the device, uniform random prompt ids, seeded uniforms)",
            "config": {"workload": "moe_step (BASELINE configs[4])", "layers": cfg.num_hidden_layers,
                       "experts": cfg.num_experts, "top_k": cfg.num_experts_per_tok, "global_batch": args.moe_batch,
                       "batch_per_gpu": per_rank, "wave": wave, "waves_per_gpu": n_waves,
                       "prompt_len": args.moe_prompt, "k": k, "temperature": args.moe_temperature,
                       "parallelism": f"replicas x{ws}, sequence-sharded, resident waves",
                       "weights_gb_per_gpu": weight_gb, "state_bytes_per_sequence": per_seq,
                       "l2": "inputs larger than L2 (~160 GB of weights per step)"},
            "acceptance_rate": (statistics.mean(acc_steps) - 1.0) / k,
            "roofline": {"kernel": "verify phase (48-layer forward, T=k+1, all kernels), first wave", "bound": "hbm",
                         "achieved": vb["total"] / (v_ms / 1000) / 1e9, "peak": hbm, "unit": "GB/s",
                         "frac": vb["total"] / (v_ms / 1000) / 1e9 / hbm, "peak_source": src, "traffic": None,
                         "algorithmic_bytes": vb, "verify_ms": v_ms},
            "prefill_s": prefill_s, "build_s": build_s, "setup_s": time.perf_counter() - t0}


def run_prefill_workload(args):
    """Prompt prefill of the 2B shape: `--batch` sequences of `--prompt` tokens
    through the commit-all forward in chunks of `--prefill-chunk` (logits at each sequence's
    last position only). Timed with CUDA events over the whole prefill, after one untimed
    prefill of the same shape; reports prompt tokens per second."""
    from lollm_b200.qwen3_5 import MTP, Qwen3_5Model, SpecDecoder
    from lollm_b200.qwen3_5.config import QWEN35_2B, Qwen3_5Config
    from lollm_b200.qwen3_5.weights import load_checkpoint, random_init
    dev = torch.device("cuda", 0)
    cfg = Qwen3_5Config.from_hf(QWEN35_2B)
    params = load_checkpoint(cfg, random_init(cfg, 0, dtype=torch.bfloat16, device=dev, generator="torch"), device=dev)
    model = Qwen3_5Model(cfg, params, dtype=torch.bfloat16, device=dev, max_positions=args.prompt + 64)
    mtp = MTP(model, params)
    del params
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    prompts = torch.randint(0, cfg.vocab_size, (args.batch, args.prompt), generator=g, device=dev)
    ms = []
    stream = torch.cuda.current_stream()
    for rep in range(2):
        dec = SpecDecoder(model, mtp, args.batch, args.k, args.prompt + 16, out_capacity=16)
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if args.profile and rep == 1:
            torch.cuda.profiler.start()
        a.record(stream)
        dec.prefill(prompts, chunk=args.prefill_chunk)
        b.record(stream)
        torch.cuda.synchronize()
        if args.profile and rep == 1:
            torch.cuda.profiler.stop()
        ms.append(a.elapsed_time(b))
        del dec
    toks = args.batch * args.prompt
    return {"metric": "prompt prefill tok/s (2B shape, bf16)", "value": toks / (ms[-1] / 1000), "unit": "tok/s",
            "n_gpus": 1, "steps": 1, "warmup": 1, "ms_per_step": ms[-1], "higher_is_better": True, "dtype": "bf16",
            "data": "synthetic (seeded random-init weights, uniform random prompt ids)",
            "config": {"workload": "prefill (configs[1] prompts)", "batch": args.batch, "prompt_len": args.prompt,
                       "chunk": args.prefill_chunk}, "prefill_s": ms[-1] / 1000}


def run_gemm_workload(args):
    """One projection of the verify step alone: c = a·wᵀ (bf16, fp32 accumulate) with
    M = batch·(k+1) token rows (default: the GDN in_proj shape 256 x 12352 x 2048)."""
    from lollm_b200 import kernels as K
    dev = torch.device("cuda", 0)
    m, n, k = args.m, args.n, args.k_dim
    g = torch.Generator(device=dev); g.manual_seed(0)
    a = torch.randn(m, k, generator=g, device=dev).to(torch.bfloat16)
    # several weight copies rotated so each launch streams its weights from HBM (> L2 in total)
    n_w = 1 if args.l2_resident else max(1, int(math.ceil(256e6 / (n * k * 2))))
    ws = [(torch.randn(n, k, generator=g, device=dev) * 0.02).to(torch.bfloat16) for _ in range(n_w)]
    c = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
    it = {"i": 0}
    epi = args.gemm_epi
    if epi == "swiglu":      # n = 2·inter rows of a [gate; up] weight, SwiGLU of the product out
        act = torch.empty(m, n // 2, dtype=torch.bfloat16, device=dev)
    if epi == "resnorm":     # residual add into c, then the next RMSNorm into y
        y = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
        nw = torch.zeros(n, dtype=torch.bfloat16, device=dev)

    def step():
        w_i = ws[it["i"] % n_w]
        if epi == "swiglu":
            K.gemm_swiglu(a, w_i, act, c)
        elif epi == "resnorm":
            K.gemm_residual_rmsnorm(a, w_i, c, nw, y, 1e-6)
        else:
            K.gemm(a, w_i, c)
        it["i"] += 1

    stream = torch.cuda.current_stream()
    if args.profile:
        torch.cuda.profiler.start()
    ms = timed_loop(step, args.steps, args.warmup, stream)
    if args.profile:
        torch.cuda.profiler.stop()
    hbm, tf, src = peaks()
    t = statistics.mean(ms) / 1000
    algo_b = n * k * 2 + m * k * 2 + m * n * 2
    flops = 2 * m * n * k
    gbs, tfs = algo_b / t / 1e9, flops / t / 1e12
    bound = "hbm" if gbs / hbm >= tfs / tf else "tensor"
    return {"metric": f"gemm {m}x{n}x{k} bf16" + ("" if epi == "store" else f" + {epi}"), "value": tfs, "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": statistics.mean(ms), "higher_is_better": True, "dtype": "bf16",
            "data": "synthetic", "config": {"workload": "gemm", "m": m, "n": n, "k": k, "weight_copies": n_w},
            "roofline": {"kernel": "gemm_tc_kernel (+ split-k merge)", "bound": bound,
                         "achieved": gbs if bound == "hbm" else tfs, "peak": hbm if bound == "hbm" else tf,
                         "unit": "GB/s" if bound == "hbm" else "TFLOP/s",
                         "frac": gbs / hbm if bound == "hbm" else tfs / tf, "peak_source": src, "traffic": None,
                         "hbm_frac": gbs / hbm, "tensor_frac": tfs / tf}}


def run_moe_workload(args):
    """BASELINE configs[4] FFN: one qwen3_5_moe sparse block (hidden 2048, 512 experts top-10
    of width 512, shared expert 512) over the verify rows of `--batch` sequences x (k+1)
    tokens, with the residual add and the next RMSNorm. Random-init N(0, 0.02) weights,
    N(0, 1) inputs. Algorithmic bytes: the weights of every expert hit in the call (read
    once), the router/shared weights and the activations."""
    from lollm_b200.qwen3_5.config import QWEN35_MOE, Qwen3_5Config
    from lollm_b200.qwen3_5.moe import SparseMoeBlock
    dev = torch.device("cuda", 0)
    cfg = Qwen3_5Config.from_hf(QWEN35_MOE)
    H, E, I, Is = cfg.hidden_size, cfg.num_experts, cfg.moe_intermediate_size, cfg.shared_expert_intermediate_size
    m = args.batch * (args.k + 1)
    g = torch.Generator(device=dev); g.manual_seed(0)
    w = lambda *s: (torch.randn(*s, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    P = {"mlp.gate.weight": w(E, H), "mlp.experts.gate_up_proj": w(E, 2 * I, H), "mlp.experts.down_proj": w(E, H, I),
         "mlp.shared_expert.gate_proj.weight": w(Is, H), "mlp.shared_expert.up_proj.weight": w(Is, H),
         "mlp.shared_expert.down_proj.weight": w(H, Is), "mlp.shared_expert_gate.weight": w(1, H)}
    blk = SparseMoeBlock(cfg, P, "", dtype=torch.bfloat16, device=dev)
    del P
    xn = torch.randn(m, H, generator=g, device=dev).to(torch.bfloat16)
    x = torch.randn(m, H, generator=g, device=dev).to(torch.bfloat16)
    nw = w(H)
    y = torch.empty_like(x)
    ws = torch.empty(blk.workspace_bytes(m), dtype=torch.uint8, device=dev)
    counts = torch.zeros(E, dtype=torch.int32, device=dev)

    def step():
        blk(xn, x, nw, y, cfg.rms_norm_eps, m, ws, expert_counts=counts)

    stream = torch.cuda.current_stream()
    if args.profile:
        torch.cuda.profiler.start()
    ms = timed_loop(step, args.steps, args.warmup, stream)
    if args.profile:
        torch.cuda.profiler.stop()
    hbm, _, src = peaks()
    t = statistics.mean(ms) / 1000
    hit = int((counts > 0).sum())
    algo = blk.weight_bytes(counts) + m * H * 2 * 4
    return {"metric": f"MoE FFN layer (configs[4] shape, {m} rows) weight GB/s", "value": algo / t / 1e9,
            "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": statistics.mean(ms), "higher_is_better": True, "dtype": "bf16",
            "data": "synthetic (BASELINE configs[4] FFN shapes, random-init N(0,0.02) weights)",
            "config": {"workload": "moe (BASELINE configs[4] FFN)", "rows": m, "experts_hit": hit,
                       "tokens_per_hit_expert": m * cfg.num_experts_per_tok / max(hit, 1),
                       "l2": "weights 3.2 GB per call (> L2)"},
            "roofline": {"kernel": "qsp_moe_ffn (moe_tc_kernel gate|up + down dominate)", "bound": "hbm",
                         "achieved": algo / t / 1e9, "peak": hbm, "unit": "GB/s", "frac": algo / t / 1e9 / hbm,
                         "peak_source": src, "traffic": None, "algorithmic_bytes_per_launch": algo}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--batch", type=int, default=64, help="sequences per GPU (weak scaling, the headline)")
    ap.add_argument("--global-batch", type=int, default=64,
                    help="N > 1: also time the step with this many sequences split over the GPUs (strong scaling)")
    ap.add_argument("--prompt", type=int, default=2048)
    ap.add_argument("--k", type=int, default=3)
    ap.add_argument("--prefill-chunk", type=int, default=128)
    ap.add_argument("--ref-budget-s", type=float, default=150.0,
                    help="reference arm: stop the timed CPU steps after this many seconds")
    ap.add_argument("--ref-warmup", type=int, default=1, help="reference arm: at most this many warm-up steps")
    ap.add_argument("--cpu-steps", type=int, default=2, help="cpu_baseline: timed reference steps")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--attn-len", default="1024,32768",
                    help="attn workload: per-sequence context lengths ~ U[lo, hi] (configs[2]: 1024,32768)")
    ap.add_argument("--attn-split-len", type=int, default=0,
                    help="attn workload: keys per split (the split count is the longest context over this); "
                         "0: the model's split count for this capacity and batch")
    ap.add_argument("--attn-equal", default="1024,4096,16384,32768",
                    help="attn_compare workload: the equal context lengths to time")
    ap.add_argument("--profile", action="store_true",
                    help="bracket the timed steps with cudaProfilerStart/Stop (for ncu --profile-from-start off)")
    ap.add_argument("--m", type=int, default=256)
    ap.add_argument("--n", type=int, default=12352)
    ap.add_argument("--k-dim", type=int, default=2048)
    ap.add_argument("--l2-resident", action="store_true", help="gemm workload: one weight copy (stays in L2)")
    ap.add_argument("--gemm-epi", choices=["store", "resnorm", "swiglu"], default="store",
                    help="gemm workload: plain product, + residual add and RMSNorm, or SwiGLU of [gate; up]")
    ap.add_argument("--moe-batch", type=int, default=256, help="moe_step: sequences over all GPUs (configs[4]: 256)")
    ap.add_argument("--moe-prompt", type=int, default=4096, help="moe_step: prompt length (configs[4]: 4096)")
    ap.add_argument("--moe-temperature", type=float, default=0.8)
    ap.add_argument("--moe-layers", type=int, default=0, help="moe_step: fewer layers (0 = the 48 of configs[4])")
    ap.add_argument("--moe-reserve-gb", type=float, default=6.0,
                    help="moe_step: device memory kept free of wave state (workspaces)")
    ap.add_argument("--workload", choices=["step", "gdn", "attn", "attn_compare", "gemm", "moe", "moe_step", "prefill"],
                    default="step",
                    help="step: the speculative step (headline); gdn / attn: BASELINE configs[3] / [2] kernels "
                         "alone; attn_compare: configs[2] attention at equal lengths against the reference's "
                         "SDPA and Triton kernels; moe: one configs[4] sparse FFN block")
    args = ap.parse_args()
    from lollm_b200.qwen3_5.config import QWEN35_2B, Qwen3_5Config
    cfg = Qwen3_5Config.from_hf(QWEN35_2B)
    if args.workload == "moe_step":
        ws, rank, local = dist_setup()
        out = run_moe_step_workload(args, ws, rank, local)
        if ws > 1:
            torch.distributed.destroy_process_group()
        if rank == 0:
            print(json.dumps(out), flush=True)
        return
    if args.workload != "step":
        torch.cuda.set_device(0)
        out = {"gdn": run_gdn_workload, "attn": run_attn_workload, "attn_compare": run_attn_compare_workload,
               "gemm": run_gemm_workload, "moe": run_moe_workload, "prefill": run_prefill_workload}[args.workload](args)
        print(json.dumps(out), flush=True)
        return
    if args.impl == "reference":
        ws, rank = int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0"))
        run_reference_arm(args, cfg, ws, rank)
        return
    ws, rank, local = dist_setup()
    args.gpus = ws
    out = run_gpu_arm(args, cfg, ws, rank, local)
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        cb, why = stock_reference_sample(cfg, args.batch, args.prompt, args.k, args.cpu_steps, 1, 30.0)
        if cb is not None:
            for key in ("steps", "seconds", "tokens"):
                cb.pop(key)
        out["cpu_baseline"] = cb if cb is not None else {"unavailable": why}
    if ws > 1:
        torch.distributed.destroy_process_group()
    if rank == 0:
        print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
