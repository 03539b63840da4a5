"""qwen3_5 family on the qsp C ABI — manifest mirroring src/qwen3_5/__init__.py:17-23.

    load(raw_config, weights, fmt, device, dtype) -> Qwen3_5Model   (weights.py:40-70; streams
        the tensors of a dict or a safetensors checkpoint one at a time)
    load_mtp(model, weights, fmt, device, dtype) -> MTP             (mtp.py:171-189)
"""

from __future__ import annotations

import torch

from .config import Qwen3_5Config, build_config
from .kv import Qwen3_5Cache
from .modeling_qwen3_5 import Qwen3_5Model
from .moe import SparseMoeBlock
from .mtp import MTP, SpecDecoder, generate_mtp
from .weights import StreamingParams, load_checkpoint, random_init

MODEL_TYPES = ["qwen3_5", "qwen3_5_moe"]   # the MoE sibling (src/qwen3_5_moe/__init__.py) shares the backbone
DEFAULTS = {"temperature": 0.7, "top_p": 0.8, "top_k": 20, "repetition_penalty": 1.05}


def _source(cfg, weights, with_mtp):
    """A streaming parameter source over an HF-named dict (tensors popped as the model takes
    them, as the reference's load does) or a safetensors file / directory path."""
    if isinstance(weights, StreamingParams):
        return weights
    if isinstance(weights, (str, bytes)) or hasattr(weights, "__fspath__"):
        return StreamingParams.from_safetensors(cfg, str(weights), with_mtp=with_mtp)
    return StreamingParams.from_dict(cfg, weights, consume=True, with_mtp=with_mtp)


def load(raw_config: dict, weights, fmt: str = "hf", device="cuda", dtype=torch.bfloat16,
         progress=None, **model_kw) -> Qwen3_5Model:
    """Build the model on `device`, taking one tensor at a time from `weights` (a dict —
    consumed — or a safetensors path), each shape-checked (RuntimeError on a mismatch or a
    missing tensor)."""
    if fmt != "hf":
        raise NotImplementedError("qwen3_5: only hf (safetensors) supported")
    cfg = build_config(raw_config, fmt)
    model = Qwen3_5Model(cfg, _source(cfg, weights, False), dtype=dtype, device=device, **model_kw)
    if progress is not None:
        progress(1, 1)
    return model


def load_mtp(model: Qwen3_5Model, weights, fmt: str = "hf", device=None, dtype=None) -> MTP:
    if fmt != "hf":
        raise NotImplementedError("qwen3_5 MTP: only hf (safetensors) supported")
    return MTP(model, _source(model.cfg, weights, True))


__all__ = ["Qwen3_5Config", "Qwen3_5Cache", "Qwen3_5Model", "MTP", "SpecDecoder", "SparseMoeBlock", "generate_mtp",
           "load", "load_mtp", "random_init", "StreamingParams", "MODEL_TYPES", "DEFAULTS"]
