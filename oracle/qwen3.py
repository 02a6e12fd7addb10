"""Qwen3 decoder, prefill-only, with explicit shared-prefix K/V.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).  Restates
``crates/cev-model/src/qwen3.rs`` with weights as a dict of HF-named tensors.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import ops


def linear(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """candle_nn::Linear without bias: ``x @ w^T`` in the model dtype."""
    return torch.matmul(x, w.t())


@dataclass
class LayerKv:
    """K/V of one layer: (1, kv_heads, S, D) each (qwen3.rs:138-143)."""
    k: torch.Tensor
    v: torch.Tensor


@dataclass
class PrefixKv:
    """K/V for every layer of a prefilled prefix (qwen3.rs:265-278)."""
    layers: list
    len: int


class Qwen3:
    """(qwen3.rs:296-402)."""

    def __init__(self, cfg: dict, weights: dict, dtype=torch.float32, max_len: int = 32768):
        self.cfg = cfg
        self.dtype = dtype
        self.w = {k: v.to(dtype) for k, v in weights.items()}
        self.heads = cfg["num_attention_heads"]
        self.kv_heads = cfg["num_key_value_heads"]
        self.hidden = cfg["hidden_size"]
        self.head_dim = cfg.get("head_dim") or self.hidden // self.heads
        self.eps = cfg["rms_norm_eps"]
        self.theta = cfg.get("rope_theta") or (cfg.get("rope_parameters") or {}).get("rope_theta") or 1e6
        self.layers = cfg["num_hidden_layers"]
        self.max_len = min(max_len, cfg.get("max_position_embeddings", max_len))
        tied = cfg.get("tie_word_embeddings", False)
        self.lm_head = self.w["model.embed_tokens.weight"] if tied else self.w["lm_head.weight"]

    def head_rows(self, ids) -> torch.Tensor:
        """LM-head rows of ``ids`` (qwen3.rs:342-344)."""
        return self.lm_head[torch.as_tensor(ids, dtype=torch.long)]

    def _attn(self, i, x, pos, mask, past):
        """``Attention::forward`` (qwen3.rs:190-204)."""
        p = f"model.layers.{i}.self_attn."
        t = x.shape[1]
        d = self.head_dim

        def shape(y, h):
            return y.reshape(1, t, h, d).transpose(1, 2).contiguous()

        q = ops.rms_norm(shape(linear(x, self.w[p + "q_proj.weight"]), self.heads), self.w[p + "q_norm.weight"], self.eps)
        k = ops.rms_norm(shape(linear(x, self.w[p + "k_proj.weight"]), self.kv_heads), self.w[p + "k_norm.weight"], self.eps)
        v = shape(linear(x, self.w[p + "v_proj.weight"]), self.kv_heads)
        cos, sin = ops.rope_cos_sin(pos, d, self.theta, self.dtype)
        q, k = ops.rope(q, cos, sin), ops.rope(k, cos, sin)
        if past is not None:
            k = torch.cat([past.k, k], 2)
            v = torch.cat([past.v, v], 2)
        ctx = ops.attend(q, k, v, mask)
        out = linear(ctx.transpose(1, 2).reshape(1, t, self.heads * d), self.w[p + "o_proj.weight"])
        return out, LayerKv(k, v)

    def _mlp_block(self, i, x):
        """``Layer::mlp_block`` (qwen3.rs:259-262; ``Mlp`` 229-233)."""
        p = f"model.layers.{i}."
        h = ops.rms_norm(x, self.w[p + "post_attention_layernorm.weight"], self.eps)
        g = ops.silu(linear(h, self.w[p + "mlp.gate_proj.weight"]))
        u = linear(h, self.w[p + "mlp.up_proj.weight"])
        return x + linear(g * u, self.w[p + "mlp.down_proj.weight"])

    def _layer(self, i, x, pos, mask, past):
        h, kv = self._attn(i, ops.rms_norm(x, self.w[f"model.layers.{i}.input_layernorm.weight"], self.eps), pos, mask, past)
        return self._mlp_block(i, x + h), kv

    def embed(self, ids) -> torch.Tensor:
        return self.w["model.embed_tokens.weight"][torch.as_tensor(ids, dtype=torch.long)]

    def prefill(self, tokens, chunk: int) -> PrefixKv:
        """Chunked causal prefill of the prefix (qwen3.rs:347-362)."""
        caches = [None] * self.layers
        past = 0
        chunk = max(chunk, 1)
        for s in range(0, len(tokens), chunk):
            part = tokens[s:s + chunk]
            mask = ops.segment_mask([0] * len(part), past)
            pos = torch.arange(past, past + len(part))
            past += len(part)
            x = self.embed(part)[None]
            for i in range(self.layers):
                x, caches[i] = self._layer(i, x, pos, mask, caches[i])
        return PrefixKv(caches, len(tokens))

    def forward_packed(self, past_layers, tokens, pos, mask, gather, keep):
        """One packed pass (qwen3.rs:374-401).  Returns the final-normed
        hidden state at ``gather`` rows (f32) and, for each ``keep`` range of
        new tokens, its per-layer K/V."""
        past_len = 0 if past_layers is None else past_layers[0].k.shape[2]
        pos = torch.as_tensor(pos, dtype=torch.long)
        mask = mask.to(self.dtype)
        kept = [[] for _ in keep]
        x = self.embed(tokens)[None]
        for i in range(self.layers):
            xn = ops.rms_norm(x, self.w[f"model.layers.{i}.input_layernorm.weight"], self.eps)
            h, kv = self._attn(i, xn, pos, mask, None if past_layers is None else past_layers[i])
            for slot, (start, n) in zip(kept, keep):
                slot.append(LayerKv(kv.k[:, :, past_len + start:past_len + start + n].clone(),
                                    kv.v[:, :, past_len + start:past_len + start + n].clone()))
            x = self._mlp_block(i, x + h)
        x = x[0][torch.as_tensor(gather, dtype=torch.long)]
        return ops.rms_norm(x, self.w["model.norm.weight"], self.eps).float(), kept
