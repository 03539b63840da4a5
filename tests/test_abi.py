"""The C ABI library loads (no GPU needed) and exports every entry point include/qsp.h
declares, with matching ctypes signatures; the product path refuses to run on the CPU."""

import os
import re

import pytest
import torch

from lollm_b200 import _lib as L

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    src = open(os.path.join(ROOT, "include", "qsp.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(qsp_\w+)\s*\(", src)))


def test_library_loads_and_exports_every_declared_symbol():
    lib = L.load()
    names = declared_symbols()
    assert len(names) >= 20
    for n in names:
        assert hasattr(lib, n), f"libqsp.so does not export {n}"
        assert n in L.SIGNATURES, f"no ctypes signature for {n}"
    assert lib.qsp_abi_version() == 1


def test_struct_layouts_match_header():
    # sizes follow natural alignment on x86-64: 11 4-byte fields, padding, 14 8-byte fields
    import ctypes
    assert ctypes.sizeof(L.GdnLayer) == 4 * 11 + 4 + 8 * 14
    assert ctypes.sizeof(L.AttnLayer) % 8 == 0


def test_argument_validation_without_gpu():
    """Invalid arguments are rejected by the host-side checks before any launch."""
    lib = L.load()
    rc = lib.qsp_gemm(None, 1, None, 1, None, 1, 1, 1, 1, 0, 0, None, 0, None)
    assert rc == L.QSP_ERR_INVALID
    assert b"null" in lib.qsp_last_error()
    rc = lib.qsp_cache_finalize(0, 1, 0, None, None, None, None, None)
    assert rc == L.QSP_ERR_INVALID


def test_model_refuses_cpu():
    from lollm_b200.qwen3_5.config import MICRO, Qwen3_5Config
    from lollm_b200.qwen3_5 import Qwen3_5Model
    from lollm_b200.qwen3_5.weights import load_checkpoint, random_init
    cfg = Qwen3_5Config.from_hf(MICRO)
    P = load_checkpoint(cfg, random_init(cfg, 0))
    with pytest.raises(RuntimeError):
        Qwen3_5Model(cfg, P, dtype=torch.float32, device="cpu")


def test_kernel_wrappers_refuse_cpu_tensors():
    from lollm_b200 import kernels as K
    x = torch.zeros(2, 8)
    with pytest.raises(RuntimeError):
        K.rmsnorm(x, torch.zeros(8), x, 1e-6)


def test_static_attention_scratch_limits_without_gpu():
    """qsp_attn_verify_static checks its scratch limit on the host before touching the device."""
    import ctypes
    lib = L.load()
    assert lib.qsp_attn_verify_static(None, None) == L.QSP_ERR_INVALID
    d = L.AttnLayer()
    d.batch, d.tokens, d.n_heads, d.head_dim = 64, 4, 16, 256
    d.num_splits = L.QSP_ATTN_STATIC_SCRATCH_BYTES // lib.qsp_attn_workspace_bytes(64, 4, 16, 256, 1) + 1
    assert lib.qsp_attn_verify_static(ctypes.byref(d), None) == L.QSP_ERR_INVALID
    assert b"static region" in lib.qsp_last_error()
    d.num_splits = 0
    assert lib.qsp_attn_verify_static(ctypes.byref(d), None) == L.QSP_ERR_INVALID
    # a shape whose byte count wraps 64 bits (2^30 rows x 2^31 heads x 2^31 splits x 2 KB)
    # is refused, not reduced to a small number that would pass the limit
    d.batch, d.tokens, d.n_heads, d.num_splits = 1 << 15, 1 << 15, (1 << 31) - 1, (1 << 31) - 1
    assert lib.qsp_attn_verify_static(ctypes.byref(d), None) == L.QSP_ERR_INVALID
    assert b"static region" in lib.qsp_last_error()


def test_wait_probe_limits_without_gpu():
    """The failure-detection probe checks its poll limit on the host before any launch."""
    lib = L.load()
    assert lib.qsp_wait_probe(0, None, None) == L.QSP_ERR_INVALID
    assert lib.qsp_wait_probe((1 << 24) + 1, None, None) == L.QSP_ERR_INVALID
    assert b"polls" in lib.qsp_last_error()


def test_gemm_plans_at_the_step_shapes():
    """The split-K plans behind the verify step's projections, read through the workspace
    query (host-side planning only, no launch; the SM count is the B200's 148): the
    vocabulary projection's last partial round of tiles is split along K into 16 slices of
    fp32 partials (3 tiles of 128 rows x 256 tokens), the 2048 x 6144 down projection takes the
    fewest splits within 3 % of the best estimate (8, not 9), gate|up 3 splits."""
    lib = L.load()
    f4 = 4
    assert lib.qsp_gemm_workspace_bytes(256, 151936, 2048, L.QSP_BF16) == 16 * 256 * 3 * 128 * f4
    assert lib.qsp_gemm_workspace_bytes(64, 151936, 2048, L.QSP_BF16) == 16 * 64 * 3 * 128 * f4
    assert lib.qsp_gemm_workspace_bytes(256, 2048, 6144, L.QSP_BF16) == 8 * 256 * 2048 * f4
    assert lib.qsp_gemm_workspace_bytes(256, 2048, 4096, L.QSP_BF16) == 8 * 256 * 2048 * f4
    assert lib.qsp_gemm_workspace_bytes(256, 12288, 2048, L.QSP_BF16) == 3 * 256 * 12288 * f4
    assert lib.qsp_gemm_workspace_bytes(256, 2048, 4096, L.QSP_F32) == 0   # fp32 runs unsplit
