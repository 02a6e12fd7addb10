"""Seeded random-init checkpoints and the safetensors + ``config.json`` pair.

The benchmark models are random-init (no checkpoints are available offline):
linear weights N(0, 0.02), RMSNorm weights 1 (zero-centred norms of Qwen3.5
start at 0, i.e. scale 1), GDN ``A_log``/``dt_bias`` like HF's init.  Names
are the HF names the reference's ``VarBuilder`` reads
(``crates/cev-model/src/qwen3.rs:172-339``, ``qwen35.rs:390-668``,
``lfm2.rs:128-322``).
"""
from __future__ import annotations

import json
import math
import os

import torch


def _shapes(cfg: dict):
    """(name, shape, kind) for every tensor of a checkpoint of ``cfg``."""
    mt = cfg["model_type"]
    h, v, inter = cfg["hidden_size"], cfg["vocab_size"], cfg["intermediate_size"]
    heads, kv = cfg["num_attention_heads"], cfg["num_key_value_heads"]
    d = cfg.get("head_dim") or h // heads
    out = [("model.embed_tokens.weight", (v, h), "lin")]
    for i in range(cfg["num_hidden_layers"]):
        p = f"model.layers.{i}."
        if mt == "qwen3":
            out += [(p + "self_attn.q_proj.weight", (heads * d, h), "lin"),
                    (p + "self_attn.k_proj.weight", (kv * d, h), "lin"),
                    (p + "self_attn.v_proj.weight", (kv * d, h), "lin"),
                    (p + "self_attn.o_proj.weight", (h, heads * d), "lin"),
                    (p + "self_attn.q_norm.weight", (d,), "one"),
                    (p + "self_attn.k_norm.weight", (d,), "one"),
                    (p + "mlp.gate_proj.weight", (inter, h), "lin"),
                    (p + "mlp.up_proj.weight", (inter, h), "lin"),
                    (p + "mlp.down_proj.weight", (h, inter), "lin"),
                    (p + "input_layernorm.weight", (h,), "one"),
                    (p + "post_attention_layernorm.weight", (h,), "one")]
        elif mt.startswith("qwen3_5"):
            if cfg["layer_types"][i] == "linear_attention":
                nk, nv = cfg["linear_num_key_heads"], cfg["linear_num_value_heads"]
                dk, dv = cfg["linear_key_head_dim"], cfg["linear_value_head_dim"]
                conv = 2 * nk * dk + nv * dv
                a = p + "linear_attn."
                out += [(a + "in_proj_qkv.weight", (conv, h), "lin"),
                        (a + "in_proj_z.weight", (nv * dv, h), "lin"),
                        (a + "in_proj_b.weight", (nv, h), "lin"),
                        (a + "in_proj_a.weight", (nv, h), "lin"),
                        (a + "conv1d.weight", (conv, 1, cfg["linear_conv_kernel_dim"]), "conv"),
                        (a + "A_log", (nv,), "alog"),
                        (a + "dt_bias", (nv,), "one"),
                        (a + "norm.weight", (dv,), "one"),
                        (a + "out_proj.weight", (h, nv * dv), "lin")]
            else:
                qo = 2 * heads * d if cfg.get("attn_output_gate", True) else heads * d
                out += [(p + "self_attn.q_proj.weight", (qo, h), "lin"),
                        (p + "self_attn.k_proj.weight", (kv * d, h), "lin"),
                        (p + "self_attn.v_proj.weight", (kv * d, h), "lin"),
                        (p + "self_attn.o_proj.weight", (h, heads * d), "lin"),
                        (p + "self_attn.q_norm.weight", (d,), "zero"),
                        (p + "self_attn.k_norm.weight", (d,), "zero")]
            out += [(p + "mlp.gate_proj.weight", (inter, h), "lin"),
                    (p + "mlp.up_proj.weight", (inter, h), "lin"),
                    (p + "mlp.down_proj.weight", (h, inter), "lin"),
                    (p + "input_layernorm.weight", (h,), "zero"),
                    (p + "post_attention_layernorm.weight", (h,), "zero")]
        elif mt == "lfm2":
            if cfg["layer_types"][i] == "full_attention":
                out += [(p + "self_attn.q_proj.weight", (heads * d, h), "lin"),
                        (p + "self_attn.k_proj.weight", (kv * d, h), "lin"),
                        (p + "self_attn.v_proj.weight", (kv * d, h), "lin"),
                        (p + "self_attn.out_proj.weight", (h, heads * d), "lin"),
                        (p + "self_attn.q_layernorm.weight", (d,), "one"),
                        (p + "self_attn.k_layernorm.weight", (d,), "one")]
            else:
                out += [(p + "conv.in_proj.weight", (3 * h, h), "lin"),
                        (p + "conv.out_proj.weight", (h, h), "lin"),
                        (p + "conv.conv.weight", (h, 1, cfg.get("conv_L_cache", 3)), "conv")]
            out += [(p + "feed_forward.w1.weight", (inter, h), "lin"),
                    (p + "feed_forward.w3.weight", (inter, h), "lin"),
                    (p + "feed_forward.w2.weight", (h, inter), "lin"),
                    (p + "operator_norm.weight", (h,), "one"),
                    (p + "ffn_norm.weight", (h,), "one")]
        else:
            raise ValueError(f"unsupported model_type `{mt}`")
    if mt == "lfm2":
        out.append(("model.embedding_norm.weight", (h,), "one"))
    else:
        out.append(("model.norm.weight", (h,), "zero" if mt.startswith("qwen3_5") else "one"))
    if not cfg.get("tie_word_embeddings", False):
        out.append(("lm_head.weight", (v, h), "lin"))
    return out


def init_weights(cfg: dict, seed: int, dtype=torch.float32, device="cpu") -> dict:
    """Seeded random-init weights for ``cfg``; generated in f32 on ``device``
    in a fixed order, then cast to ``dtype``."""
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    w = {}
    for name, shape, kind in _shapes(cfg):
        if kind == "lin":
            t = torch.empty(shape, dtype=torch.float32, device=device).normal_(0.0, 0.02, generator=gen)
        elif kind == "conv":
            t = torch.empty(shape, dtype=torch.float32, device=device).normal_(0.0, 1.0 / math.sqrt(shape[-1]), generator=gen)
        elif kind == "alog":
            t = torch.empty(shape, dtype=torch.float32, device=device).uniform_(1.0, 16.0, generator=gen).log()
        elif kind == "one":
            t = torch.ones(shape, dtype=torch.float32, device=device)
        else:
            t = torch.zeros(shape, dtype=torch.float32, device=device)
        # The GDN gate parameters stay f32 (the reference upcasts them,
        # qwen35.rs:400-402); everything else takes the model dtype.
        w[name] = t if kind == "alog" or name.endswith("dt_bias") else t.to(dtype)
    return w


def save(dirname: str, cfg: dict, weights: dict) -> None:
    """Write ``config.json`` + ``model.safetensors``."""
    from safetensors.torch import save_file
    os.makedirs(dirname, exist_ok=True)
    with open(os.path.join(dirname, "config.json"), "w") as f:
        json.dump(cfg, f, indent=1)
    save_file({k: v.contiguous().cpu() for k, v in weights.items()}, os.path.join(dirname, "model.safetensors"))


def load(dirname: str, dtype=None, device="cpu"):
    """Read ``config.json`` and every ``*.safetensors`` shard of a checkpoint
    directory (the files ``RepoFiles::weights`` lists, load.rs); returns
    (cfg, weights).  With ``dtype`` every tensor but the f32 GDN gate
    parameters is cast to it."""
    import glob

    from safetensors.torch import load_file
    with open(os.path.join(dirname, "config.json")) as f:
        cfg = json.load(f)
    shards = sorted(glob.glob(os.path.join(dirname, "*.safetensors")))
    if not shards:
        raise FileNotFoundError(f"no *.safetensors in {dirname}")
    w = {}
    for sh in shards:
        w.update(load_file(sh, device=str(device)))
    if dtype is not None:
        w = {k: (v if k.endswith(("A_log", "dt_bias")) else v.to(dtype)) for k, v in w.items()}
    return cfg, w


def pick_dtype(name: str, device) -> torch.dtype:
    """``EngineOptions::dtype`` (engine.rs:108-115): "auto" is bf16 on a CUDA
    device and f32 elsewhere; "f32", "bf16" name theirs."""
    dev = torch.device(device)
    if name == "auto":
        return torch.bfloat16 if dev.type == "cuda" else torch.float32
    if name in ("f32", "float32"):
        return torch.float32
    if name in ("bf16", "bfloat16"):
        return torch.bfloat16
    raise ValueError(f"unknown dtype `{name}`")


def load_decoder(dirname: str, dtype="auto", device="cuda", **kw):
    """``cev_model::load`` (load.rs:326-337) at the model level: detect the
    family from ``config.json``'s ``model_type`` and build it on ``device``
    from the directory's safetensors.  Returns (cfg, model): a
    :class:`cev_b200.qwen3.Qwen3` for ``qwen3``, a
    :class:`cev_b200.hybrid.Qwen35` for ``qwen3_5`` / ``qwen3_5_text``, a
    :class:`cev_b200.hybrid.Lfm2` for ``lfm2``.  ``kw`` go to the model's
    constructor (``arena_rows``, ``max_len``, ...)."""
    dt = pick_dtype(dtype, device) if isinstance(dtype, str) else dtype
    cfg, w = load(dirname)
    mt = cfg.get("model_type")
    if mt == "qwen3":
        from .qwen3 import Qwen3
        return cfg, Qwen3(cfg, w, dt, device, **kw)
    if mt in ("qwen3_5", "qwen3_5_text"):
        from .hybrid import Qwen35
        return cfg, Qwen35(cfg, w, dt, device, **kw)
    if mt == "lfm2":
        from .hybrid import Lfm2
        return cfg, Lfm2(cfg, w, dt, device, **kw)
    raise ValueError(f"unsupported model_type `{mt}`")
