"""The algorithmic byte counts behind the bench's roofline fractions (`bench.py`
verify_step_bytes and gdn_launch_bytes), restated here by plain arithmetic from the configs[1]
shape (the qwen3_5 2B shape: 24 layers, 18 Gated-DeltaNet + 6 attention; GDN 16 key / 32
value heads of 128; attention 2 kv heads of 256; conv width 4) and pinned to the totals the
bench reports."""

import bench
from lollm_b200.qwen3_5.config import QWEN35_2B, Qwen3_5Config

CFG = Qwen3_5Config.from_hf(QWEN35_2B)
B, T = 64, 4                     # sequences, verify tokens (k = 3)
N_GDN, N_ATTN = 18, 6
HK, HV, DK, DV = 16, 32, 128, 128
NKV, HD = 2, 256
CONV_DIM = 2 * HK * DK + HV * DV     # q, k, v channels of the causal conv
VALUE_DIM = HV * DV


def test_shape_is_the_2b_config():
    assert (len(CFG.gdn_layers), len(CFG.attn_layers)) == (N_GDN, N_ATTN)
    assert (CFG.linear_num_key_heads, CFG.linear_num_value_heads) == (HK, HV)
    assert (CFG.linear_key_head_dim, CFG.linear_value_head_dim) == (DK, DV)
    assert (CFG.num_key_value_heads, CFG.head_dim, CFG.linear_conv_kernel_dim) == (NKV, HD, 4)
    assert CFG.conv_dim == CONV_DIM == 8192


def test_verify_step_bytes():
    lens = [2048 + (37 * i) % 128 for i in range(B)]          # ragged contexts around 2048
    got = bench.verify_step_bytes(CFG, B, T, lens)
    state = 2 * N_GDN * B * HV * DK * DV * 4                 # fp32 state read + written
    conv = 2 * N_GDN * B * CONV_DIM * 3 * 2                  # 3-row bf16 window read + written
    kv_pos = N_ATTN * NKV * HD * 2 * 2                       # K and V, bf16, per position
    kv = kv_pos * (sum(L + T for L in lens) + B * T)         # every visible key read, T rows written
    assert got["gdn_state"] == state == 4_831_838_208
    assert got["conv"] == conv == 113_246_208
    assert got["kv"] == kv
    # every weight but the embedding table once, the tied lm_head once: 1.99 B bf16 parameters
    assert got["weights"] == 3_975_496_448
    assert got["total"] == got["weights"] + kv + state + conv
    assert abs(bench.verify_step_bytes(CFG, B, T, [2048] * B)["total"] - 10.537e9) < 1e6


def test_gdn_launch_bytes():
    got = bench.gdn_launch_bytes(CFG, B, T)
    state = 2 * B * HV * DK * DV * 4
    window = 2 * B * CONV_DIM * 3 * 2
    rows_in = B * T * (CONV_DIM + VALUE_DIM + 2 * HV) * 2    # q, k, v, z, a, b of each token row
    rows_out = B * T * VALUE_DIM * 2                         # gated output
    assert got == state + window + rows_in + rows_out == 283_148_288
