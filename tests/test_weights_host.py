"""Checkpoint files on the host: the safetensors + ``config.json`` pair
round-trips bit for bit, sharded directories load whole, and the loader
picks the family and dtype the way ``cev_model::load`` does (load.rs:326-337,
engine.rs:87-124).  No GPU: the models are built on the CPU device."""
import json
import os

import pytest
import torch

from cev_b200 import configs, weights


@pytest.mark.parametrize("make", [configs.tiny_qwen3, configs.tiny_qwen35, configs.tiny_lfm2])
def test_save_load_round_trip_and_family_dispatch(tmp_path, make):
    from cev_b200.hybrid import Lfm2, Qwen35
    from cev_b200.qwen3 import Qwen3
    cfg = make()
    w = weights.init_weights(cfg, 4)
    weights.save(str(tmp_path), cfg, w)
    with open(tmp_path / "config.json") as f:
        assert json.load(f) == cfg
    cfg2, w2 = weights.load(str(tmp_path))
    assert cfg2 == cfg and w2.keys() == w.keys()
    assert all(torch.equal(w[k], w2[k]) and w[k].dtype == w2[k].dtype for k in w)
    _, m = weights.load_decoder(str(tmp_path), "auto", "cpu", arena_rows=64)
    want = {"qwen3": Qwen3, "qwen3_5_text": Qwen35, "lfm2": Lfm2}[cfg["model_type"]]
    assert isinstance(m, want) and m.dtype == torch.float32  # "auto" is f32 off CUDA


def test_sharded_checkpoint_and_gate_parameters_stay_f32(tmp_path):
    from safetensors.torch import save_file
    cfg = configs.tiny_qwen35()
    w = weights.init_weights(cfg, 5)
    names = sorted(w)
    half = len(names) // 2
    with open(tmp_path / "config.json", "w") as f:
        json.dump(cfg, f)
    save_file({k: w[k] for k in names[:half]}, str(tmp_path / "model-00001-of-00002.safetensors"))
    save_file({k: w[k] for k in names[half:]}, str(tmp_path / "model-00002-of-00002.safetensors"))
    _, w2 = weights.load(str(tmp_path), dtype=torch.bfloat16)
    assert w2.keys() == w.keys()
    for k, v in w2.items():
        gate = k.endswith(("A_log", "dt_bias"))
        assert v.dtype == (torch.float32 if gate else torch.bfloat16), k
        assert torch.equal(v, w[k] if gate else w[k].to(torch.bfloat16))


def test_pick_dtype_and_errors(tmp_path):
    assert weights.pick_dtype("auto", "cuda") == torch.bfloat16
    assert weights.pick_dtype("auto", "cpu") == torch.float32
    assert weights.pick_dtype("f32", "cuda") == torch.float32
    assert weights.pick_dtype("bf16", "cpu") == torch.bfloat16
    with pytest.raises(ValueError, match="unknown dtype"):
        weights.pick_dtype("f8", "cpu")
    os.makedirs(tmp_path / "empty")
    with open(tmp_path / "empty" / "config.json", "w") as f:
        json.dump(configs.tiny_qwen3(), f)
    with pytest.raises(FileNotFoundError):
        weights.load(str(tmp_path / "empty"))
