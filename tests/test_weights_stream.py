"""The streaming load seam without a GPU: tensors come one at a time from a dict (consumed as
taken) or a safetensors checkpoint, shape-checked, with the reference's hard failures
(src/qwen3_5/weights.py:57-62): a missing tensor or a wrong shape raises RuntimeError."""

import os

import pytest
import torch

from lollm_b200.qwen3_5.config import MICRO, Qwen3_5Config
from lollm_b200.qwen3_5.weights import StreamingParams, load_checkpoint, param_specs, random_init, to_raw


def cfg():
    return Qwen3_5Config.from_hf(MICRO)


def test_dict_source_is_consumed_and_matches_strict_load():
    c = cfg()
    w = random_init(c, 5, generator="numpy")
    want = load_checkpoint(c, dict(w))
    src = StreamingParams.from_dict(c, dict(w))
    assert src.tied
    for name, _ in param_specs(c):
        assert torch.equal(src[name], want[name])
    with pytest.raises(RuntimeError, match="missing tensor"):
        src["model.norm.weight"]                  # already handed over once
    with pytest.raises(RuntimeError, match="tied"):
        src["lm_head.weight"]


def test_shape_mismatch_and_unknown_names_raise():
    c = cfg()
    w = random_init(c, 5, generator="numpy")
    w[to_raw("model.norm.weight")] = torch.zeros(3)
    src = StreamingParams.from_dict(c, w, consume=False)
    with pytest.raises(RuntimeError, match="shape mismatch"):
        src["model.norm.weight"]
    with pytest.raises(RuntimeError, match="no parameter"):
        src["model.layers.99.mlp.down_proj.weight"]


def test_safetensors_file_and_sharded_directory(tmp_path):
    import json
    from safetensors.torch import save_file
    c = cfg()
    w = random_init(c, 6, generator="numpy")
    save_file({k: v.contiguous() for k, v in w.items()}, str(tmp_path / "one.safetensors"))
    names = sorted(w)
    half = len(names) // 2
    shard = tmp_path / "sharded"
    shard.mkdir()
    save_file({k: w[k].contiguous() for k in names[:half]}, str(shard / "a.safetensors"))
    save_file({k: w[k].contiguous() for k in names[half:]}, str(shard / "b.safetensors"))
    json.dump({"weight_map": {k: ("a.safetensors" if i < half else "b.safetensors") for i, k in enumerate(names)}},
              open(shard / "model.safetensors.index.json", "w"))
    for path in (str(tmp_path / "one.safetensors"), str(shard)):
        src = StreamingParams.from_safetensors(c, path, dtype=torch.bfloat16)
        for name, _ in param_specs(c):
            t = src[name]
            assert t.dtype == torch.bfloat16 and torch.equal(t, w[to_raw(name)].to(torch.bfloat16))


def test_random_source_is_order_independent():
    c = cfg()
    a = StreamingParams.random(c, 3, device="cpu", dtype=torch.float32)
    b = StreamingParams.random(c, 3, device="cpu", dtype=torch.float32)
    names = [n for n, _ in param_specs(c)]
    first = {n: a[n] for n in names}
    for n in reversed(names):
        assert torch.equal(b[n], first[n])
    assert abs(float(first["model.embed_tokens.weight"].std()) - 0.02) < 1e-3


def test_counter_init_slices_and_statistics():
    from lollm_b200.qwen3_5.weights import counter_init, counter_uniform
    c = cfg()
    w = counter_init(c, 9, chunk=1000)               # small chunks: the slices must join exactly
    w2 = counter_init(c, 9)
    for k in w:
        assert torch.equal(w[k], w2[k])
    x = counter_uniform(1 << 20, 0, 9, "cpu")
    assert abs(float(x.std()) - 0.02) < 2e-4 and abs(float(x.mean())) < 2e-4
    assert float(x.abs().max()) <= 0.02 * 3 ** 0.5
