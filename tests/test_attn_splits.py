"""The verify attention's split-count rule (`attn_num_splits`, host logic used by the model and
by `bench.py --workload attn`), checked on the CPU: the measured choices at the step's and
configs[2]'s shapes, and that every split the tensor-core kernel is given covers keys.

The kernel cuts a sequence's capacity into splits of ceil(capacity / splits) keys rounded up
to its 32-key tile (`at3_chunk` in qsp_attn_mma.cu); the restatement below is that formula."""

import math

import pytest

from lollm_b200.qwen3_5.modeling_qwen3_5 import attn_num_splits


def _chunk(capacity, splits, tile=32):
    return math.ceil(math.ceil(capacity / splits) / tile) * tile


def test_step_shape_takes_one_split():
    # 64 sequences × 2 kv heads at a 2048-token prompt plus the speculative steps
    assert attn_num_splits(2048 + 64 * 4, 64 * 2) == 1
    assert attn_num_splits(4096, 128) == 1


def test_few_sequences_fill_the_sms():
    # 4 sequences × 2 kv heads: 148 // 8 = 18 splits
    assert attn_num_splits(4096, 8) == 18
    assert attn_num_splits(4096, 8, sms=132) == 16


def test_long_contexts_take_1024_key_splits():
    # contexts up to 32768 keys
    assert attn_num_splits(32768 + 64, 128) == math.ceil((32768 + 64) / 1024)
    assert attn_num_splits(4097, 128) == 5


def test_tiny_capacity_is_capped_at_one_tile_per_split():
    assert attn_num_splits(64, 1) == 2
    assert attn_num_splits(32, 1) == 1
    assert attn_num_splits(1, 1) == 1


def _written_splits(kv_len, chunk):
    """Splits whose key range [s·chunk, min((s+1)·chunk, kv_len)) is not empty: the ones the
    tensor-core kernel writes partials for, and the merge kernel's count 2·ceil(kv_len / chunk)
    of partials read (qsp_attn.cu, attn_combine_kernel)."""
    return math.ceil(kv_len / chunk)


@pytest.mark.parametrize("n_seq_heads", [1, 2, 8, 64, 128, 256, 1024])
def test_every_key_is_in_a_split(n_seq_heads):
    for capacity in range(32, 40000, 97):
        s = attn_num_splits(capacity, n_seq_heads)
        assert 1 <= s <= max(1, math.ceil(capacity / 32))
        chunk = _chunk(capacity, s)
        assert chunk % 32 == 0
        assert s * chunk >= capacity                 # every key of the capacity is in a split
        for kv_len in (1, capacity // 2 + 1, capacity):
            w = _written_splits(kv_len, chunk)
            assert 1 <= w <= s                       # the merge reads only partials that exist
            assert (w - 1) * chunk < kv_len <= w * chunk


def test_benched_shapes_have_no_empty_splits():
    """With few sequences and a short capacity, rounding a split up to whole 32-key tiles can
    leave trailing splits without keys (4096 keys, 8 sequence-heads: 18 splits of 256 keys, 16
    of them used; 4785 keys, one sequence-head: 148 splits of 64 keys, 75 used); the kernel
    skips those items. The benched shapes (the step's 128 sequence-heads at a 2k context,
    configs[2] at up to 32k) have none."""
    for capacity, n_seq_heads in [(2048 + 256, 128), (32768 + 64, 128)]:
        s = attn_num_splits(capacity, n_seq_heads)
        assert (s - 1) * _chunk(capacity, s) < capacity
    for capacity, n_seq_heads, want in [(4096, 8, (18, 256, 16)), (4785, 1, (148, 64, 75))]:
        s = attn_num_splits(capacity, n_seq_heads)
        c = _chunk(capacity, s)
        assert (s, c, _written_splits(capacity, c)) == want
