"""qwen3_5 family on the qsp C ABI — manifest mirroring src/qwen3_5/__init__.py:17-23.

    load(raw_config, weights, fmt, device, dtype) -> Qwen3_5Model   (weights.py:40-70)
    load_mtp(model, weights, fmt, device, dtype) -> MTP             (mtp.py:171-189)
"""

from __future__ import annotations

import torch

from .config import Qwen3_5Config, build_config
from .kv import Qwen3_5Cache
from .modeling_qwen3_5 import Qwen3_5Model
from .moe import SparseMoeBlock
from .mtp import MTP, SpecDecoder, generate_mtp
from .weights import load_checkpoint, random_init

MODEL_TYPES = ["qwen3_5", "qwen3_5_moe"]   # the MoE sibling (src/qwen3_5_moe/__init__.py) shares the backbone
DEFAULTS = {"temperature": 0.7, "top_p": 0.8, "top_k": 20, "repetition_penalty": 1.05}


def load(raw_config: dict, weights: dict, fmt: str = "hf", device="cuda", dtype=torch.bfloat16,
         progress=None, **model_kw) -> Qwen3_5Model:
    cfg = build_config(raw_config, fmt)
    params = load_checkpoint(cfg, weights, with_mtp=False, device="cpu")
    if progress is not None:
        progress(1, 1)
    return Qwen3_5Model(cfg, params, dtype=dtype, device=device, **model_kw)


def load_mtp(model: Qwen3_5Model, weights: dict, fmt: str = "hf", device=None, dtype=None) -> MTP:
    if fmt != "hf":
        raise NotImplementedError("qwen3_5 MTP: only hf (safetensors) supported")
    params = load_checkpoint(model.cfg, weights, with_mtp=True, device="cpu")
    return MTP(model, params)


__all__ = ["Qwen3_5Config", "Qwen3_5Cache", "Qwen3_5Model", "MTP", "SpecDecoder", "SparseMoeBlock", "generate_mtp",
           "load", "load_mtp", "random_init", "MODEL_TYPES", "DEFAULTS"]
