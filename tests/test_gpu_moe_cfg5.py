"""BASELINE configs[4] at its real per-layer shapes on the GPU against the reference's own
outputs (tests/golden/golden_moe_cfg5.safetensors, made by make_golden_moe_cfg5.py): hidden
2048, 512 experts top-10 of width 512 plus the shared expert, GDN 16/32 heads of 128,
attention 16/2 heads of 256, vocabulary 151936; one GDN layer, one attention layer and the
MTP head, fp32 (the golden script says why fp32: bf16 routing over 512 experts is a near-tie
for about half of the tokens).

Prefill (12 tokens), a T=4 verify, a decode and the depth-1 MTP draft, each compared on the
reference's 32 best logits of every row, on 1024 fixed vocabulary positions and on the
argmax, at the fp32 bar (1e-4 relative and absolute)."""

import json
import os

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
TOL = dict(rtol=1e-4, atol=1e-4)


@pytest.fixture(scope="module")
def g5():
    from safetensors.torch import load_file
    G = load_file(os.path.join(ROOT, "tests", "golden", "golden_moe_cfg5.safetensors"))
    meta = json.load(open(os.path.join(ROOT, "tests", "golden", "golden_moe_cfg5_meta.json")))
    return G, meta


def _check(G, name, logits):
    lf = logits.float().cpu()
    cols = G["cols"]
    torch.testing.assert_close(lf[..., cols], G[f"{name}.cols"].float(), **TOL)
    torch.testing.assert_close(lf.gather(-1, G[f"{name}.top_i"]), G[f"{name}.top_v"].float(), **TOL)
    top = G[f"{name}.top_v"].float()
    clear = (top[..., 0] - top[..., 1]) > 1e-3          # the reference's pick is not a near-tie
    assert torch.equal(lf.argmax(-1)[clear], G[f"{name}.argmax"][clear])


def test_cfg5_shapes_match_reference(g5):
    from lollm_b200 import qwen3_5 as fam
    from lollm_b200.qwen3_5.config import Qwen3_5Config
    from lollm_b200.qwen3_5.weights import counter_init
    G, meta = g5
    raw = meta["config"]
    cfg = Qwen3_5Config.from_hf(raw)
    # routing is unambiguous in fp32: every router's 10th and 11th logits are apart
    for i in range(meta["router_calls_after_stage"][-1][1]):
        s = G[f"router.{i}"].float().sort(-1, descending=True).values
        k = cfg.num_experts_per_tok
        assert float((s[..., k - 1] - s[..., k]).min()) > 1e-5
    w = counter_init(cfg, meta["weight_seed"], dtype=torch.float32, device="cuda")   # bit-identical to the host's
    model = fam.load(raw, w, dtype=torch.float32, max_positions=64)      # consumes w as it builds
    mtp = fam.load_mtp(model, w)
    del w
    logits, past, hidden = model(G["ids"].cuda(), return_hidden=True)
    _check(G, "prefill", logits)
    logits, past, hidden = model(G["verify.ids"].cuda(), past, return_hidden=True)
    _check(G, "verify", logits)
    logits, past, hidden = model(G["decode.ids"].cuda(), past, return_hidden=True)
    _check(G, "decode", logits)
    torch.testing.assert_close(hidden.float().cpu(), G["decode.hidden"].float(), **TOL)
    ids = torch.zeros(2, 2, dtype=torch.int64, device="cuda")
    ids[:, 0] = G["decode.ids"][:, 0].cuda()
    dl = mtp.draft(hidden[:, -1].contiguous(), ids, 1)
    _check(G, "draft", dl[:, :1])
    assert past.seen_tokens == 17


def test_counter_init_is_bit_identical_on_gpu_and_cpu():
    """The fixture's weights are rebuilt on the GPU: the counter hash must give the host's
    values bit for bit (any slice, any offset)."""
    from lollm_b200.qwen3_5.weights import counter_uniform
    for n, off, seed in ((1 << 20, 0, 4321), (12345, (1 << 33) + 7, 4321), (999, 5, 1)):
        a = counter_uniform(n, off, seed, "cpu")
        b = counter_uniform(n, off, seed, "cuda").cpu()
        assert torch.equal(a, b)
        assert torch.equal(a.to(torch.bfloat16), b.to(torch.bfloat16))
