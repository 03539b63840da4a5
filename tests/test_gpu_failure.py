"""Failure detection on the GPU without a GPU fault: a bounded wait that runs out returns and
reports a status, and the host-side injections (an out-of-range accepted count, NaN logits, a
sequence running past its pages) are flagged on the device and raised on the host. Every case
leaves the context usable (checked by running a GEMM afterwards)."""

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def K():
    from lollm_b200 import kernels
    return kernels


def _context_still_usable():
    a = torch.randn(64, 256, device=DEV).bfloat16()
    w = torch.randn(384, 256, device=DEV).bfloat16()
    c = torch.empty(64, 384, device=DEV, dtype=torch.bfloat16)
    K().gemm(a, w, c)
    torch.testing.assert_close(c.float(), (a.float() @ w.float().T), rtol=2e-2, atol=2e-2)
    assert K().device_status() == 0


def test_bounded_wait_runs_out_and_reports():
    K().device_status(reset=True)
    waited = torch.zeros(1, dtype=torch.int32, device=DEV)
    K().wait_probe(1 << 14, waited)
    torch.cuda.synchronize()                     # the kernel returned: no hang
    assert K().device_status(reset=False) == K().DEV_WAIT_PROBE
    assert K().device_status(reset=True) == K().DEV_WAIT_PROBE
    assert K().device_status() == 0              # cleared
    assert int(waited) > 0                       # it did wait before giving up
    _context_still_usable()


def test_out_of_range_accept_is_clamped_and_flagged():
    B, T = 4, 4
    lens = torch.full((B,), 100, dtype=torch.int32, device=DEV)
    lens += T                                    # after a speculative T=4 forward
    replay = torch.zeros(B, dtype=torch.int32, device=DEV)
    coff = torch.zeros(B, dtype=torch.int32, device=DEV)
    acc = torch.tensor([7, -3, 0, 3], dtype=torch.int32, device=DEV)
    K().cache_accept(B, T, acc, lens, replay, coff)
    keep = [4, 1, 1, 4]                          # clamped into [1, T]
    assert lens.tolist() == [100 + k for k in keep] and replay.tolist() == keep
    assert K().device_status() == K().DEV_BAD_ACCEPT
    _context_still_usable()


@pytest.mark.parametrize("vocab", [1000, 151936])
def test_nan_logits_pick_the_first_nan_and_flag(vocab):
    g = torch.Generator(device=DEV).manual_seed(0)
    rows = torch.randn(6, vocab, device=DEV, generator=g).bfloat16()
    rows[1, 777] = float("nan")
    rows[1, 5] = float("nan")
    rows[3, vocab - 1] = float("nan")
    out = torch.zeros(6, dtype=torch.int64, device=DEV)
    K().argmax_rows(rows, out)
    want = rows.float().cpu().argmax(-1)         # torch: NaN ranks above every number
    assert out.cpu().tolist() == want.tolist() and int(out[1]) == 5 and int(out[3]) == vocab - 1
    assert K().device_status() == K().DEV_NAN_LOGITS
    clean = torch.randn(6, vocab, device=DEV, generator=g).bfloat16()
    K().argmax_rows(clean, out)
    assert out.cpu().tolist() == clean.float().cpu().argmax(-1).tolist()
    assert K().device_status() == 0
    _context_still_usable()


def test_sequence_past_its_pages_is_refused_and_raised():
    """A cache of 16 positions per sequence; a speculative forward of 4 tokens at position 14
    runs past the last page: the writes are refused on the device, flagged, and check()
    raises on the host."""
    from lollm_b200 import qwen3_5 as fam
    from lollm_b200.qwen3_5.config import MICRO, Qwen3_5Config
    from lollm_b200.qwen3_5.weights import random_init
    cfg = Qwen3_5Config.from_hf(MICRO)
    model = fam.load(MICRO, dict(random_init(cfg, 3, generator="numpy")), dtype=torch.float32,
                     max_positions=64)
    # one page per sequence (pages 1 and 4) out of a pool of 6: the other four stay unused
    cache = model.new_cache(2, 16, page_size=16, num_pages=6, page_table=torch.tensor([[1], [4]]))
    model(torch.randint(0, cfg.vocab_size, (2, 14)).cuda(), cache)
    cache.check()                                # within capacity: nothing flagged
    k_before, v_before = cache.k_pages.clone(), cache.v_pages.clone()
    model(torch.randint(0, cfg.vocab_size, (2, 4)).cuda(), cache, speculative=True)
    with pytest.raises(RuntimeError, match="outside its sequence's pages"):
        cache.check()
    # positions 14, 15 were written into pages 1 and 4; 16, 17 had no page, and no other
    # page of the pool was touched
    for now, before in ((cache.k_pages, k_before), (cache.v_pages, v_before)):
        changed = (now != before).flatten(2).any(-1)            # [layers, pages]
        assert changed[:, [1, 4]].all() and not changed[:, [0, 2, 3, 5]].any()
    cache.check()                                # the flag was cleared by the raise
    _context_still_usable()
