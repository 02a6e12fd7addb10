"""Qwen3 decoder, prefill-only, on the B200 kernels.

Mirrors ``crates/cev-model/src/qwen3.rs``: ``prefill`` (chunked causal prefill
of a state prefix, qwen3.rs:347-362), ``forward_packed`` (one packed pass
whose attention pattern is given by segment descriptors instead of an
additive mask, qwen3.rs:374-401) and ``head_rows`` (qwen3.rs:342-344).

Per layer: RMSNorm (fused with the previous residual add) -> one fused
q|k|v projection (cuBLAS) -> per-head RMSNorm + RoPE writing Q and the K/V
arena rows -> packed block-masked attention (tcgen05) -> o_proj -> residual
add + RMSNorm -> fused gate|up projection -> SwiGLU -> down projection.
Linear layers are plain cuBLAS GEMMs through torch; everything else is
this library's kernels.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

from . import ops
from .arena import KvArena


@dataclass
class PrefixKv:
    """A computed prefix: its rows ``[start, start+len)`` in every layer of
    the arena (``PrefixKv``, qwen3.rs:265-278)."""
    arena: KvArena
    start: int
    len: int
    capacity: int
    pins: int = 0
    released: bool = False

    def release(self):
        if not self.released:
            self.arena.release(self.start, self.capacity)
            self.released = True


class Qwen3:
    def __init__(self, cfg: dict, weights: dict, dtype=torch.bfloat16, device="cuda", max_len: int = 32768,
                 arena_rows: int = 65536 + 8192):
        self.cfg = cfg
        self.dtype = dtype
        self.device = torch.device(device)
        H = cfg["hidden_size"]
        self.hidden = H
        self.hq = cfg["num_attention_heads"]
        self.hkv = cfg["num_key_value_heads"]
        self.D = cfg.get("head_dim") or H // self.hq
        self.eps = cfg["rms_norm_eps"]
        self.theta = cfg.get("rope_theta") or (cfg.get("rope_parameters") or {}).get("rope_theta") or 1e6
        self.n_layers = cfg["num_hidden_layers"]
        self.max_len = min(max_len, cfg.get("max_position_embeddings", max_len))
        dev = self.device

        def w(name):
            return weights[name].to(device=dev, dtype=dtype)

        self.embed_w = w("model.embed_tokens.weight")
        self.lm_head = self.embed_w if cfg.get("tie_word_embeddings", False) else w("lm_head.weight")
        self.layers = []
        for i in range(self.n_layers):
            p = f"model.layers.{i}."
            self.layers.append(dict(
                qkv=torch.cat([w(p + "self_attn.q_proj.weight"), w(p + "self_attn.k_proj.weight"),
                               w(p + "self_attn.v_proj.weight")], 0).contiguous(),
                o=w(p + "self_attn.o_proj.weight"),
                qn=w(p + "self_attn.q_norm.weight"), kn=w(p + "self_attn.k_norm.weight"),
                gu=torch.cat([w(p + "mlp.gate_proj.weight"), w(p + "mlp.up_proj.weight")], 0).contiguous(),
                down=w(p + "mlp.down_proj.weight"),
                ln1=w(p + "input_layernorm.weight"), ln2=w(p + "post_attention_layernorm.weight")))
        self.norm_w = w("model.norm.weight")
        self.arena = KvArena(self.n_layers, arena_rows, self.hkv, self.D, dtype, dev)

    def head_rows(self, ids) -> torch.Tensor:
        """LM-head rows of ``ids`` as f32 (qwen3.rs:342-344, engine.rs:155)."""
        return self.lm_head[torch.as_tensor(list(ids), dtype=torch.long, device=self.device)].float()

    # -- the decoder body -------------------------------------------------
    def _layers(self, x: torch.Tensor, pos: torch.Tensor, kv_rows: torch.Tensor, plan: ops.AttnPlan) -> torch.Tensor:
        """Run all layers over x [T, H] (updated in place as the residual
        stream).  Returns the last MLP output (not yet added)."""
        T = x.shape[0]
        hq, hkv, D = self.hq, self.hkv, self.D
        q_buf = torch.empty(T, hq, D, dtype=self.dtype, device=self.device)
        attn = torch.empty(T, hq, D, dtype=self.dtype, device=self.device)
        h = ops.rms_norm(x, self.layers[0]["ln1"], self.eps)
        m = None
        for i, L in enumerate(self.layers):
            if m is not None:
                h = ops.add_rms_norm(x, m, L["ln1"], self.eps, out=h)
            qkv = F.linear(h, L["qkv"])
            ops.qk_norm_rope(qkv, (0, D), hq * D, (hq + hkv) * D, hq, hkv, D, L["qn"], L["kn"], self.eps, False, pos,
                             self.theta, D, q_buf, self.arena.k[i], self.arena.v[i], kv_rows)
            ops.attend_packed(q_buf, self.arena.k[i], self.arena.v[i], plan, out=attn)
            o = F.linear(attn.view(T, hq * D), L["o"])
            h = ops.add_rms_norm(x, o, L["ln2"], self.eps, out=h)
            m = F.linear(ops.swiglu(F.linear(h, L["gu"])), L["down"])
        return m

    def run_tokens(self, tokens, pos, kv_rows, segments) -> torch.Tensor:
        """Embed ``tokens``, run every layer writing K/V to arena rows
        ``kv_rows`` with the attention pattern of ``segments``; returns the
        final residual stream [T, H] (before the final norm)."""
        dev = self.device
        T = len(tokens)
        ids = torch.tensor(tokens, dtype=torch.int32).pin_memory().to(dev, non_blocking=True)
        pos_t = torch.tensor(pos, dtype=torch.int32).pin_memory().to(dev, non_blocking=True)
        rows_t = torch.tensor(kv_rows, dtype=torch.int32).pin_memory().to(dev, non_blocking=True)
        plan = ops.AttnPlan(segments, T, self.arena.capacity, self.hq, self.hkv, self.D, self.dtype, dev)
        x = ops.embed(self.embed_w, ids)
        m = self._layers(x, pos_t, rows_t, plan)
        return ops.residual_add(x, m)

    def prefill_into(self, pk: PrefixKv, tokens, start_pos: int, chunk: int) -> None:
        """Chunked causal prefill of ``tokens`` at positions start_pos.. into
        the rows of ``pk`` right after its first ``start_pos`` rows
        (qwen3.rs:347-362)."""
        chunk = max(chunk, 1)
        done = 0
        while done < len(tokens):
            part = tokens[done:done + chunk]
            past = start_pos + done
            n = len(part)
            seg = [(0, n, pk.start, past, pk.start + past)]
            self.run_tokens(part, list(range(past, past + n)), list(range(pk.start + past, pk.start + past + n)), seg)
            done += n
