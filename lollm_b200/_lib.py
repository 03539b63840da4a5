"""ctypes binding of libqsp.so (the C ABI declared in include/qsp.h).

There is no fallback: importing this module on a machine without the built library, or
calling into it without a CUDA device, raises. Every status code other than QSP_OK becomes a
RuntimeError carrying `qsp_last_error()` — the reference's "hard-fail, never guess" policy
(src/qwen3_5/weights.py:57-62).
"""

from __future__ import annotations

import ctypes as C
import os

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("QSP_LIB", os.path.join(_HERE, "libqsp.so"))

QSP_OK, QSP_ERR_INVALID, QSP_ERR_CUDA, QSP_ERR_UNSUPPORTED = 0, 1, 2, 3
QSP_F32, QSP_BF16 = 0, 1
QSP_GEMM_ACCUMULATE = 1
QSP_ATTN_STATIC_SCRATCH_BYTES = 16 << 20   # include/qsp.h

vp, i32, i64, f32, sz = C.c_void_p, C.c_int32, C.c_int64, C.c_float, C.c_size_t


class GdnLayer(C.Structure):
    """Mirror of `qsp_gdn_layer`."""
    _fields_ = [("batch", i32), ("tokens", i32), ("n_k_heads", i32), ("n_v_heads", i32),
                ("head_k", i32), ("head_v", i32), ("conv_kernel", i32), ("max_spec_tokens", i32),
                ("speculative", i32), ("dtype", i32), ("eps", f32),
                ("proj", vp), ("ld_proj", i64), ("conv_w", vp), ("a_log", vp), ("dt_bias", vp),
                ("norm_w", vp), ("state", vp), ("conv_hist", vp), ("pending", vp),
                ("replay_n", vp), ("conv_off", vp), ("parity", vp), ("out", vp), ("ld_out", i64)]


class SampleParams(C.Structure):
    """Mirror of `qsp_sample_params`."""
    _fields_ = [("temperature", f32), ("top_k", i32), ("top_p", f32), ("repetition_penalty", f32),
                ("hist", vp), ("hist_ld", i64), ("hist_n", vp), ("step_ids", vp), ("step_ld", i64),
                ("step_base", i32)]


class AttnLayer(C.Structure):
    """Mirror of `qsp_attn_layer`."""
    _fields_ = [("batch", i32), ("tokens", i32), ("n_heads", i32), ("n_kv_heads", i32),
                ("head_dim", i32), ("rotary_dim", i32), ("page_size", i32), ("max_pages", i32),
                ("num_pages", i32), ("dtype", i32), ("eps", f32), ("scale", f32),
                ("qkv", vp), ("ld_qkv", i64), ("q_norm_w", vp), ("k_norm_w", vp),
                ("rope_cos", vp), ("rope_sin", vp), ("rope_rows", i32), ("k_pages", vp),
                ("v_pages", vp), ("page_table", vp), ("seq_lens", vp), ("q_buf", vp),
                ("out", vp), ("ld_out", i64), ("partial", vp), ("num_splits", i32),
                ("bad_index", vp)]


class MoeLayer(C.Structure):
    """Mirror of `qsp_moe_layer`."""
    _fields_ = [("tokens", i32), ("hidden", i32), ("n_experts", i32), ("top_k", i32), ("inter", i32),
                ("shared_inter", i32), ("norm_topk_prob", i32), ("dtype", i32), ("eps", f32),
                ("xn", vp), ("ld_xn", i64), ("w_in", vp), ("gate_up", vp), ("down", vp),
                ("shared_down", vp), ("x", vp), ("ld_x", i64), ("norm_w", vp), ("y", vp), ("ld_y", i64),
                ("workspace", vp), ("workspace_bytes", sz), ("expert_counts", vp)]


# name -> (restype, argtypes)
SIGNATURES = {
    "qsp_last_error": (C.c_char_p, []),
    "qsp_abi_version": (C.c_int, []),
    "qsp_embed": (C.c_int, [vp, i64, i64, vp, i64, i64, vp, i64, vp, C.c_int, vp]),
    "qsp_rmsnorm": (C.c_int, [vp, i64, vp, vp, i64, i64, i64, f32, C.c_int, vp]),
    "qsp_add_rmsnorm": (C.c_int, [vp, vp, vp, vp, i64, i64, f32, C.c_int, vp]),
    "qsp_swiglu": (C.c_int, [vp, i64, vp, i64, i64, i64, C.c_int, vp]),
    "qsp_gemm": (C.c_int, [vp, i64, vp, i64, vp, i64, i64, i64, i64, C.c_int, C.c_int, vp, sz, vp]),
    "qsp_gemm_workspace_bytes": (sz, [i64, i64, i64, C.c_int]),
    "qsp_gemm_residual_rmsnorm": (C.c_int, [vp, i64, vp, i64, vp, i64, vp, vp, i64, i64, i64, i64, f32, C.c_int,
                                            vp, sz, vp]),
    "qsp_gemm_swiglu": (C.c_int, [vp, i64, vp, i64, vp, i64, vp, i64, i64, i64, i64, C.c_int, vp, sz, vp]),
    "qsp_device_status": (C.c_int, [C.POINTER(i32), i32]),
    "qsp_wait_probe": (C.c_int, [C.c_uint32, vp, vp]),
    "qsp_gdn_verify": (C.c_int, [C.POINTER(GdnLayer), vp]),
    "qsp_gdn_pending_bytes": (sz, [i32, i32, i32, i32, i32, i32, i32]),
    "qsp_attn_prep": (C.c_int, [C.POINTER(AttnLayer), vp]),
    "qsp_attn_verify": (C.c_int, [C.POINTER(AttnLayer), vp]),
    "qsp_attn_workspace_bytes": (sz, [i32, i32, i32, i32, i32]),
    "qsp_attn_verify_static": (C.c_int, [C.POINTER(AttnLayer), vp]),
    "qsp_mtp_single_token_attn": (C.c_int, [vp, i64, i64, vp, i64, vp, i64, i64, i32, i32, i32,
                                            C.c_int, vp]),
    "qsp_select_rows": (C.c_int, [vp, i64, i32, i32, vp, vp, i64, i64, C.c_int, vp]),
    "qsp_argmax_rows": (C.c_int, [vp, i64, i64, i64, vp, i64, C.c_int, vp]),
    "qsp_greedy_verify": (C.c_int, [vp, i64, i32, i32, i64, vp, i64, vp, vp, vp, vp, C.c_int, vp]),
    "qsp_spec_sample": (C.c_int, [vp, i64, vp, i64, i32, i32, i64, f32, vp, i64, vp, vp, vp, vp,
                                  vp, C.c_int, vp]),
    "qsp_sample_rows": (C.c_int, [vp, i64, i64, i64, f32, vp, vp, i64, vp, C.c_int, vp]),
    "qsp_select_workspace_bytes": (sz, [i64, i64]),
    "qsp_filter_workspace_bytes": (sz, [i64, i64]),
    "qsp_sample_filtered": (C.c_int, [vp, i64, i64, i32, i64, C.POINTER(SampleParams), vp, vp, i64, vp, sz,
                                      C.c_int, vp]),
    "qsp_spec_sample_filtered": (C.c_int, [vp, i64, vp, i64, i32, i32, i64, C.POINTER(SampleParams), vp, i64,
                                           vp, vp, vp, vp, vp, sz, C.c_int, vp]),
    "qsp_moe_ffn": (C.c_int, [C.POINTER(MoeLayer), vp]),
    "qsp_moe_router_rows": (i64, [i32, i32]),
    "qsp_moe_workspace_bytes": (sz, [i32, i32, i32, i32, i32, i32, i32]),
    "qsp_cache_finalize": (C.c_int, [i32, i32, i32, vp, vp, vp, vp, vp]),
    "qsp_cache_accept": (C.c_int, [i32, i32, vp, vp, vp, vp, vp]),
    "qsp_commit_tokens": (C.c_int, [i32, i32, vp, vp, vp, vp, i64, vp, vp]),
}

_lib = None


def load():
    """Load libqsp.so once; raises if it is missing or its ABI version differs."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"libqsp.so not found at {LIB_PATH}: build it with "
                           "`python -m lollm_b200.csrc.build` (there is no CPU fallback)")
    lib = C.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if lib.qsp_abi_version() != 1:
        raise RuntimeError("libqsp.so ABI version mismatch")
    _lib = lib
    return lib


def check(rc: int, what: str = "qsp"):
    if rc != QSP_OK:
        msg = load().qsp_last_error().decode(errors="replace")
        raise RuntimeError(f"{what} failed (status {rc}): {msg}")


def call(name: str, *args):
    lib = load()
    rc = getattr(lib, name)(*args)
    check(rc, name)


def dtype_code(dt: torch.dtype) -> int:
    if dt == torch.float32:
        return QSP_F32
    if dt == torch.bfloat16:
        return QSP_BF16
    raise RuntimeError(f"unsupported model dtype {dt} (float32 or bfloat16)")


def ptr(t) -> int:
    return 0 if t is None else t.data_ptr()


def stream_handle(stream=None) -> int:
    s = torch.cuda.current_stream() if stream is None else stream
    return s.cuda_stream


def require_cuda(t: torch.Tensor, name: str):
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor (the qsp path has no CPU fallback)")
