"""Recurrent-state decoders (Qwen3.5 Gated DeltaNet hybrid, LFM2 short-conv
hybrid) and the hybrid engine's Codes readout, at the token-id level.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).  Restates
``crates/cev-model/src/qwen35.rs``, ``crates/cev-model/src/lfm2.rs``,
``crates/cev-model/src/decoder.rs`` and ``crates/cev-model/src/hybrid.rs``
(prefill 555-575, rows 595-617, Codes readout 619-641, run 697-739,
PrefixCache 744-772).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import ops
from .engine import Output, PrefixCache, Readout, Request
from .qwen3 import linear


@dataclass
class AttnState:
    """``LayerState::Attn``: (B, kv_heads, S, D) each (decoder.rs:56)."""
    k: torch.Tensor
    v: torch.Tensor


@dataclass
class GdnState:
    """``LayerState::Gdn``: conv (B, C, K-1) model dtype, s (B, H, dk, dv)
    f32 (decoder.rs:58)."""
    conv: torch.Tensor
    s: torch.Tensor


@dataclass
class ConvState:
    """``LayerState::Conv``: (B, C, K-1) model dtype (decoder.rs:60)."""
    last: torch.Tensor


@dataclass
class PrefixState:
    """(decoder.rs:92-99)."""
    layers: list
    len: int
    next_pos: int


def broadcast(st, b: int):
    """``LayerState::broadcast`` (decoder.rs:74-88)."""
    def bc(t):
        return t if t.shape[0] == b else t.expand(b, *t.shape[1:]).contiguous()
    if isinstance(st, AttnState):
        return AttnState(bc(st.k), bc(st.v))
    if isinstance(st, GdnState):
        return GdnState(bc(st.conv), bc(st.s))
    return ConvState(bc(st.last))


class Qwen35:
    """Qwen3.5 text decoder (qwen35.rs:625-752).  ``weights`` are keyed by
    HF names under ``root`` (``model.``)."""

    def __init__(self, cfg: dict, weights: dict, dtype=torch.float32, root="model.", max_len=262144):
        self.cfg = cfg
        self.dtype = dtype
        self.root = root
        self.w = {k: v.to(dtype) for k, v in weights.items()}
        self.wf = {k: v.float() for k, v in weights.items() if k.endswith(("A_log", "dt_bias", "linear_attn.norm.weight"))}
        self.hidden = cfg["hidden_size"]
        self.heads = cfg["num_attention_heads"]
        self.kv_heads = cfg["num_key_value_heads"]
        self.head_dim = cfg.get("head_dim") or self.hidden // self.heads
        self.eps = cfg.get("rms_norm_eps", 1e-6)
        rp = cfg.get("rope_parameters") or {}
        self.theta = rp.get("rope_theta") or cfg.get("rope_theta") or 1e7
        f = rp.get("partial_rotary_factor") or 1.0
        self.rotary_dim = int(self.head_dim * f) & ~1
        self.gate = cfg.get("attn_output_gate", True)
        self.nk = cfg.get("linear_num_key_heads", 16)
        self.nv = cfg.get("linear_num_value_heads", 16)
        self.dk = cfg.get("linear_key_head_dim", 128)
        self.dv = cfg.get("linear_value_head_dim", 128)
        self.kernel = cfg.get("linear_conv_kernel_dim", 4)
        self.layer_types = cfg["layer_types"]
        self.max_len = min(max_len, cfg.get("max_position_embeddings", max_len))
        tied = cfg.get("tie_word_embeddings", False)
        self.lm_head = self.w[root + "embed_tokens.weight"] if tied or "lm_head.weight" not in self.w else self.w["lm_head.weight"]

    def _norm(self, x, name):
        """Zero-centred RMSNorm ``(1 + w)`` (qwen35.rs:160-176)."""
        w = self.w[name]
        return ops.rms_norm(x, (w.float() + 1.0).to(w.dtype), self.eps)

    def head_rows(self, ids):
        return self.lm_head[torch.as_tensor(ids, dtype=torch.long)].float()

    def embed(self, ids):
        return self.w[self.root + "embed_tokens.weight"][torch.as_tensor(ids, dtype=torch.long)]

    def _gdn(self, i, x, state):
        """``GatedDeltaNet::forward`` (qwen35.rs:415-453)."""
        p = f"{self.root}layers.{i}.linear_attn."
        b, t, _ = x.shape
        key_dim, value_dim = self.nk * self.dk, self.nv * self.dv
        conv_dim = 2 * key_dim + value_dim
        mixed = linear(x, self.w[p + "in_proj_qkv.weight"]).transpose(1, 2).contiguous()
        z = linear(x, self.w[p + "in_proj_z.weight"])
        bb = linear(x, self.w[p + "in_proj_b.weight"]).float()
        aa = linear(x, self.w[p + "in_proj_a.weight"]).float()
        if state is None:
            conv_state, s0 = torch.zeros(b, conv_dim, self.kernel - 1, dtype=mixed.dtype), None
        else:
            conv_state, s0 = state.conv, state.s
        full = torch.cat([conv_state, mixed], 2)
        new_conv = full[:, :, t:t + self.kernel - 1].contiguous()
        conved = ops.silu(ops.depthwise_conv1d(full, self.w[p + "conv1d.weight"])).transpose(1, 2)

        def heads(y, h, d):
            return y.reshape(b, t, h, d).transpose(1, 2).contiguous().float()

        q = heads(conved[..., :key_dim], self.nk, self.dk)
        k = heads(conved[..., key_dim:2 * key_dim], self.nk, self.dk)
        v = heads(conved[..., 2 * key_dim:], self.nv, self.dv)
        if self.nv > self.nk:
            g = self.nv // self.nk
            q = q[:, :, None].expand(b, self.nk, g, t, self.dk).reshape(b, self.nv, t, self.dk)
            k = k[:, :, None].expand(b, self.nk, g, t, self.dk).reshape(b, self.nv, t, self.dk)
        beta = torch.sigmoid(bb).transpose(1, 2).contiguous()
        neg_a = -self.wf[p + "A_log"].exp()
        gg = (ops.softplus(aa + self.wf[p + "dt_bias"]) * neg_a).transpose(1, 2).contiguous()
        core, s = ops.chunk_gated_delta_rule(q, k, v, gg, beta, s0)
        core = core.transpose(1, 2).contiguous()
        var = core.pow(2).mean(-1, keepdim=True)
        normed = core / (var + self.eps).sqrt() * self.wf[p + "norm.weight"]
        zz = ops.silu(z.float().reshape(b, t, self.nv, self.dv))
        y = (normed * zz).reshape(b, t, value_dim).to(x.dtype)
        return linear(y, self.w[p + "out_proj.weight"]), GdnState(new_conv, s)

    def _attn(self, i, x, cos, sin, state):
        """Gated attention (qwen35.rs:526-560), causal rows only."""
        p = f"{self.root}layers.{i}.self_attn."
        b, t, _ = x.shape
        h, d = self.heads, self.head_dim
        qg = linear(x, self.w[p + "q_proj.weight"])
        if self.gate:
            qg = qg.reshape(b, t, h, 2 * d)
            q, gate = qg[..., :d], qg[..., d:].reshape(b, t, h * d)
        else:
            q, gate = qg.reshape(b, t, h, d), None
        q = self._norm(q.transpose(1, 2).contiguous(), p + "q_norm.weight")
        k = self._norm(linear(x, self.w[p + "k_proj.weight"]).reshape(b, t, self.kv_heads, d).transpose(1, 2).contiguous(), p + "k_norm.weight")
        v = linear(x, self.w[p + "v_proj.weight"]).reshape(b, t, self.kv_heads, d).transpose(1, 2).contiguous()
        q, k = ops.rope_partial(q, cos, sin), ops.rope_partial(k, cos, sin)
        past = 0
        if state is not None:
            past = state.k.shape[2]
            k = torch.cat([state.k, k], 2)
            v = torch.cat([state.v, v], 2)
        mask = ops.causal_mask(t, past).to(self.dtype)
        ctx = ops.attend(q, k, v, mask)
        out = ctx.transpose(1, 2).reshape(b, t, h * d)
        if gate is not None:
            out = out * torch.sigmoid(gate.float()).to(out.dtype)
        return linear(out, self.w[p + "o_proj.weight"]), AttnState(k, v)

    def forward(self, embeds, pos, state=None, keep=False):
        """``Decoder::forward`` (qwen35.rs:698-751) with text positions."""
        b, t, _ = embeds.shape
        if keep and b != 1:
            raise ValueError("a prefix state is kept for one sequence at a time")
        pos = torch.as_tensor(pos, dtype=torch.long)
        # Text positions: all three mrope axes equal, so every frequency
        # reads the text position (qwen35.rs:221-228).
        cos, sin = ops.rope_cos_sin(pos, self.rotary_dim, self.theta, self.dtype)
        x = embeds.to(self.dtype)
        new_states = []
        for i in range(self.cfg["num_hidden_layers"]):
            past = None if state is None else broadcast(state.layers[i], b)
            h = self._norm(x, f"{self.root}layers.{i}.input_layernorm.weight")
            if self.layer_types[i] == "linear_attention":
                h, st = self._gdn(i, h, past)
            else:
                h, st = self._attn(i, h, cos, sin, past)
            if keep:
                new_states.append(st)
            x = x + h
            p = f"{self.root}layers.{i}."
            hn = self._norm(x, p + "post_attention_layernorm.weight")
            m = linear(ops.silu(linear(hn, self.w[p + "mlp.gate_proj.weight"])) * linear(hn, self.w[p + "mlp.up_proj.weight"]), self.w[p + "mlp.down_proj.weight"])
            x = x + m
        hidden = self._norm(x, self.root + "norm.weight").float()
        new = None
        if keep:
            new = PrefixState(new_states, (0 if state is None else state.len) + t, int(pos.max()) + 1)
        return hidden, new


class Lfm2:
    """LFM2 causal decoder (lfm2.rs:270-431)."""

    def __init__(self, cfg: dict, weights: dict, dtype=torch.float32, root="model.", max_len=128000):
        self.cfg = cfg
        self.dtype = dtype
        self.root = root
        self.w = {k: v.to(dtype) for k, v in weights.items()}
        self.hidden = cfg["hidden_size"]
        self.heads = cfg["num_attention_heads"]
        self.kv_heads = cfg["num_key_value_heads"]
        self.head_dim = cfg.get("head_dim") or self.hidden // self.heads
        self.eps = cfg.get("norm_eps", 1e-5)
        self.theta = cfg.get("rope_theta") or (cfg.get("rope_parameters") or {}).get("rope_theta") or 1e6
        self.kernel = cfg.get("conv_L_cache", 3)
        self.layer_types = cfg["layer_types"]
        self.max_len = min(max_len, cfg.get("max_position_embeddings", max_len))
        self.lm_head = self.w[root + "embed_tokens.weight"]

    def head_rows(self, ids):
        return self.lm_head[torch.as_tensor(ids, dtype=torch.long)].float()

    def embed(self, ids):
        return self.w[self.root + "embed_tokens.weight"][torch.as_tensor(ids, dtype=torch.long)]

    def _conv(self, i, x, state):
        """``ShortConv::forward`` (lfm2.rs:199-219)."""
        p = f"{self.root}layers.{i}.conv."
        bsz, t, _ = x.shape
        d = self.hidden
        bcu = linear(x, self.w[p + "in_proj.weight"]).transpose(1, 2).contiguous()
        b, c, u = bcu[:, :d], bcu[:, d:2 * d], bcu[:, 2 * d:]
        bu = b * u
        last = torch.zeros(bsz, d, self.kernel - 1, dtype=bu.dtype) if state is None else state.last
        full = torch.cat([last, bu], 2)
        new_last = full[:, :, t:t + self.kernel - 1].contiguous()
        z = ops.depthwise_conv1d(full, self.w[p + "conv.weight"])
        if p + "conv.bias" in self.w:
            z = z + self.w[p + "conv.bias"].reshape(1, d, 1)
        y = (c * z).transpose(1, 2).contiguous()
        return linear(y, self.w[p + "out_proj.weight"]), ConvState(new_last)

    def _attn(self, i, x, cos, sin, mask, state):
        """``Attention::forward`` (lfm2.rs:145-171)."""
        p = f"{self.root}layers.{i}.self_attn."
        b, t, _ = x.shape
        h, d = self.heads, self.head_dim
        q = ops.rms_norm(linear(x, self.w[p + "q_proj.weight"]).reshape(b, t, h, d), self.w[p + "q_layernorm.weight"], self.eps).transpose(1, 2).contiguous()
        k = ops.rms_norm(linear(x, self.w[p + "k_proj.weight"]).reshape(b, t, self.kv_heads, d), self.w[p + "k_layernorm.weight"], self.eps).transpose(1, 2).contiguous()
        v = linear(x, self.w[p + "v_proj.weight"]).reshape(b, t, self.kv_heads, d).transpose(1, 2).contiguous()
        q, k = ops.rope(q, cos, sin), ops.rope(k, cos, sin)
        if state is not None:
            k = torch.cat([state.k, k], 2)
            v = torch.cat([state.v, v], 2)
        ctx = ops.attend(q, k, v, mask)
        return linear(ctx.transpose(1, 2).reshape(b, t, h * d), self.w[p + "out_proj.weight"]), AttnState(k, v)

    def forward(self, embeds, pos, state=None, keep=False):
        """``Decoder::forward`` (lfm2.rs:397-430)."""
        b, t, _ = embeds.shape
        if keep and b != 1:
            raise ValueError("a prefix state is kept for one sequence at a time")
        past = 0 if state is None else state.len
        pos = torch.as_tensor(pos, dtype=torch.long)
        cos, sin = ops.rope_cos_sin(pos, self.head_dim, self.theta, self.dtype)
        mask = ops.causal_mask(t, past).to(self.dtype)
        x = embeds.to(self.dtype)
        new_states = []
        for i in range(self.cfg["num_hidden_layers"]):
            prev = None if state is None else broadcast(state.layers[i], b)
            p = f"{self.root}layers.{i}."
            h = ops.rms_norm(x, self.w[p + "operator_norm.weight"], self.eps)
            if self.layer_types[i] == "full_attention":
                h, st = self._attn(i, h, cos, sin, mask, prev)
            else:
                h, st = self._conv(i, h, prev)
            if keep:
                new_states.append(st)
            x = x + h
            hn = ops.rms_norm(x, self.w[p + "ffn_norm.weight"], self.eps)
            f = p + "feed_forward."
            x = x + linear(ops.silu(linear(hn, self.w[f + "w1.weight"])) * linear(hn, self.w[f + "w3.weight"]), self.w[f + "w2.weight"])
        hidden = ops.rms_norm(x, self.w[self.root + "embedding_norm.weight"], self.eps).float()
        new = PrefixState(new_states, past + t, int(pos.max()) + 1) if keep else None
        return hidden, new


class HybridEngine:
    """Hybrid engine, ``Kind::Codes`` readout (hybrid.rs:155-165, 454-772)."""

    def __init__(self, decoder, code_ids, pad_id, prefill_chunk=512, pass_tokens=2048, prefix_cache_tokens=65536):
        self.decoder = decoder
        self.head = decoder.head_rows(code_ids)
        self.pad_id = pad_id
        self.prefill_chunk = prefill_chunk
        self.pass_tokens = pass_tokens
        self.cache = PrefixCache(prefix_cache_tokens)

    def prefill(self, prefix) -> PrefixState:
        """Run the prefix in chunks into a state and cache it (hybrid.rs:555-575)."""
        hit = self.cache.get(prefix)
        if hit is not None:
            return hit
        chunk = max(self.prefill_chunk, 1)
        allemb = self.decoder.embed(prefix)
        state, done = None, 0
        while done < len(prefix):
            n = min(chunk, len(prefix) - done)
            _, state = self.decoder.forward(allemb[done:done + n][None], list(range(done, done + n)), state, keep=True)
            done += n
        self.cache.put(prefix, state)
        return state

    def rows(self, state, rows):
        """Right-padded batch continuing ``state`` (hybrid.rs:595-617)."""
        t = max(len(r) for r in rows)
        ids = []
        for r in rows:
            ids += list(r) + [self.pad_id] * (t - len(r))
        emb = self.decoder.embed(ids).reshape(len(rows), t, -1)
        pos = list(range(state.next_pos, state.next_pos + t))
        hidden, _ = self.decoder.forward(emb, pos, state, keep=False)
        return hidden

    def run(self, req: Request) -> Output:
        """hybrid.rs:697-739 with the Codes readout of 619-641."""
        cached = self.cache.get(req.prefix) is not None
        state = self.prefill(list(req.prefix))
        readouts, start = [], 0
        br = req.suffixes
        while start < len(br):
            end, longest = start + 1, len(br[start])
            while end < len(br):
                l = max(longest, len(br[end]))
                if l * (end + 1 - start) > self.pass_tokens:
                    break
                longest = l
                end += 1
            rows = br[start:end]
            hidden = self.rows(state, rows)
            for i, r in enumerate(rows):
                h = hidden[i, len(r) - 1]
                z = h @ self.head.t()
                k = req.n_options[start + i]
                readouts.append(Readout(z[:k].clone(), h.clone()))
            start = end
        return Output(readouts, len(req.prefix) + sum(len(s) for s in br), cached)

    def run_many(self, reqs):
        return [self.run(r) for r in reqs]
