"""Recurrent-state decoders and the hybrid engine on the B200 kernels.

Mirrors ``crates/cev-model/src/qwen35.rs`` (Gated DeltaNet + gated attention
hybrid), ``crates/cev-model/src/lfm2.rs`` (gated short conv + GQA hybrid),
``crates/cev-model/src/decoder.rs`` (``Decoder::forward``, ``PrefixState``)
and the Codes path of ``crates/cev-model/src/hybrid.rs`` (prefix prefilled
once in chunks into a cached state, then the questions as right-padded rows
continuing it).

State of a prefix (``PrefixState``, decoder.rs:54-105): the attention layers'
K/V rows in the model's arena (one contiguous range shared by every
attention layer), the GDN layers' conv tails and f32 recurrent matrices, and
the short-conv layers' tails.  Rows continuing a state read it in place:
attention through segment descriptors, GDN / conv through batch stride 0
(the reference copies the state B times, decoder.rs:74-88).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

from . import ops
from .arena import KvArena, PrefixCache
from .engine import InputError, Output, Readout, Request


def dist_all_gather(out: torch.Tensor, t: torch.Tensor, split) -> None:
    """Every rank's ``t`` into ``out`` (rank order), over the split's group."""
    import torch.distributed as dist
    dist.all_gather_into_tensor(out, t, group=split.group)


@dataclass
class HybridState:
    arena: KvArena | None
    start: int
    capacity: int
    len: int = 0
    next_pos: int = 0
    gdn: dict = field(default_factory=dict)    # layer -> (conv tail [1,C,K-1], S [1,nv,dk,dv] f32)
    conv: dict = field(default_factory=dict)   # layer -> tail [1,d,K-1]
    pins: int = 0
    released: bool = False

    def release(self):
        if not self.released and self.arena is not None and self.capacity > 0:
            self.arena.release(self.start, self.capacity)
        self.released = True
        self.gdn, self.conv = {}, {}


class _HybridDecoder:
    """Shared layer loop of the two hybrid families."""

    plus_one = False

    def __init__(self, cfg, dtype, device, max_len, arena_rows, split=None):
        self.cfg = cfg
        self.dtype = dtype
        self.device = torch.device(device)
        self.hidden = cfg["hidden_size"]
        self.hq = cfg["num_attention_heads"]
        self.hkv = cfg["num_key_value_heads"]
        self.D = cfg.get("head_dim") or self.hidden // self.hq
        # attention heads this process computes (all, or its KV-head group)
        self.split = split
        self.hq_a, self.hkv_a = (self.hq, self.hkv) if split is None else (split.hq_l, split.hkv_l)
        self.n_layers = cfg["num_hidden_layers"]
        self.attn_layers = [i for i, t in enumerate(cfg["layer_types"]) if t == "full_attention"]
        self.arena_index = {l: j for j, l in enumerate(self.attn_layers)}
        self.arena = KvArena(len(self.attn_layers), arena_rows, self.hkv_a, self.D, dtype, self.device)
        self.max_len = min(max_len, cfg.get("max_position_embeddings", max_len))

    def _w(self, weights, name):
        return weights[name].to(device=self.device, dtype=self.dtype)

    def head_rows(self, ids) -> torch.Tensor:
        return self.lm_head[torch.as_tensor(list(ids), dtype=torch.long, device=self.device)].float()

    def new_state(self, n_tokens: int, cache=None) -> HybridState:
        start = self.arena.alloc(n_tokens, cache) if self.attn_layers and n_tokens > 0 else 0
        return HybridState(self.arena, start, n_tokens if self.attn_layers else 0)

    def forward(self, tokens, B: int, T: int, pos, state: HybridState | None, keep: bool, cache=None):
        """``Decoder::forward`` over B rows of T tokens (flattened,
        row-major) at shared positions ``pos``, continuing ``state``.  With
        ``keep`` (B == 1) the state is extended in place (its arena range
        must have room).  Returns the residual stream [B*T, H] before the
        final norm."""
        if keep and B != 1:
            raise ValueError("a prefix state is kept for one sequence at a time")
        dev = self.device
        n = B * T
        ids = torch.tensor(tokens, dtype=torch.int32).pin_memory().to(dev, non_blocking=True)
        pos_t = torch.tensor(list(pos) * B, dtype=torch.int32).pin_memory().to(dev, non_blocking=True)
        past = 0 if state is None else state.len
        scratch = None
        if self.attn_layers:
            if keep:
                base = state.start + past
                rows = list(range(base, base + T))
                segs = [(0, T, state.start, past, base)]
            else:
                scratch = self.arena.alloc(n, cache)
                rows = list(range(scratch, scratch + n))
                pstart = 0 if state is None else state.start
                segs = [(b * T, T, pstart, past, scratch + b * T) for b in range(B)]
            rows_t = torch.tensor(rows, dtype=torch.int32).pin_memory().to(dev, non_blocking=True)
            plan = ops.AttnPlan(segs, n, self.arena.capacity, self.hq_a, self.hkv_a, self.D, self.dtype, dev)
        try:
            if self._token_split(B, T):
                x = self._layers_token_split(ids, B, T, pos_t, rows_t, plan, state, keep)
            else:
                x = ops.embed(self.embed_w, ids)
                h = ops.rms_norm(x, self.layers[0]["ln1"], self.eps, self.plus_one)
                m = None
                for i, L in enumerate(self.layers):
                    if m is not None:
                        h = ops.add_rms_norm(x, m, L["ln1"], self.eps, self.plus_one, out=h)
                    if L["kind"] == "attn":
                        o = self._attn(i, L, h, pos_t, rows_t, plan)
                    elif L["kind"] == "gdn":
                        o = self._gdn(i, L, h, B, T, state, keep)
                    else:
                        o = self._conv(i, L, h, B, T, state, keep)
                    h = ops.add_rms_norm(x, o, L["ln2"], self.eps, self.plus_one, out=h)
                    m = F.linear(ops.swiglu(F.linear(h, L["gu"])), L["down"])
                ops.residual_add(x, m)
        finally:
            if scratch is not None:
                self.arena.release(scratch, n)
        if keep:
            state.len = past + T
            state.next_pos = max(pos) + 1
        return x

    def _token_split(self, B, T) -> bool:
        """Token-local layers split over the ranks of a KV-head split: a row
        batch by whole rows, a sequence chunk by contiguous runs of at least
        K-1 tokens (shorter chunks run whole on every rank)."""
        sp = self.split
        if sp is None or sp.world < 2 or not sp.sequence_parallel:
            return False
        return B > 1 or T >= sp.world * max(getattr(self, "K", 1) - 1, 1)

    def _token_runs(self, B, T):
        """This rank's token rows [a, b) of the token split, and the run
        length (all but the last runs are full)."""
        sp = self.split
        if B > 1:
            per = -(-B // sp.world)
            return min(B, sp.rank * per) * T, min(B, (sp.rank + 1) * per) * T, per * T
        unit = -(-T // sp.world)
        return min(T, sp.rank * unit), min(T, (sp.rank + 1) * unit), unit

    def _layers_token_split(self, ids, B, T, pos_t, rows_t, plan, state, keep, tails=None):
        """The layer loop with a KV-head split over ranks: attention runs
        this rank's heads on every token (its head outputs gathered across
        ranks), everything token-local -- the output projection, the short
        conv, the MLP, the norms -- runs only on this rank's token rows.
        A row batch splits by whole rows, a sequence chunk into contiguous
        runs in rank order.  The residual stream is all-gathered (NVLink
        peer stores into the fused gather's row buffers, or NCCL) only
        where every token is needed: before each attention layer and, for a
        row batch, at the end.  Between gathers a run's short convs read
        K-1 rows before it, so each layer before them also computes those
        rows (recomputed from the last gathered stream; their outputs are
        dropped once consumed).  With ``keep`` the rank that runs the
        chunk's last token collects every conv layer's new tails (written
        by its conv kernel) and one gather at the end gives them to every
        rank; the returned stream then holds only this rank's rows.
        ``tails``: (read, write) tail buffers by layer for a graph-captured
        chunk."""
        sp = self.split
        n = B * T
        a, b, unit = self._token_runs(B, T)
        K1 = getattr(self, "K", 1) - 1
        kinds = [L["kind"] for L in self.layers]
        if any(k not in ("attn", "conv") for k in kinds):
            raise NotImplementedError("token split: attention and short-conv layers only")
        conv = [i for i, k in enumerate(kinds) if k == "conv"]
        # rows before `a` each layer must also produce: the conv layers up to
        # the next gather read K-1 more each (a row batch never crosses rows)
        need = [0] * len(kinds)
        if B == 1:
            for i in range(len(kinds) - 2, -1, -1):
                need[i] = need[i + 1] + K1 if kinds[i + 1] == "conv" else 0
        fused = sp.fused if sp.fused is not None and sp.fused.hidden == self.hidden else None
        extra = len(conv) * K1 if keep else 0
        if fused is not None and n + extra > fused.max_tokens:
            raise ValueError(f"{n} tokens: the residual buffers hold {fused.max_tokens - extra}")
        owner = keep and B == 1 and b == T and b > a
        if keep:
            # the owner's tails, one (K-1) x d block per conv layer (bytes of a
            # [1, d, K-1] tail each): after the stream in residual buffer 0
            if fused is not None:
                stage = fused.rows[0][n:n + extra]
            else:
                stage = torch.empty(extra, self.hidden, dtype=self.dtype, device=self.device)
        k = 0
        if fused is not None:
            x = ops.embed(self.embed_w, ids, out=fused.rows[0][:n])
        else:
            x = ops.embed(self.embed_w, ids)

        def gather(x, k):
            if fused is not None:
                return fused.gather_rows(k, a, b, n), 1 - k
            sp.gather_rows(x, a, b, unit)
            return x, k

        for i, L in enumerate(self.layers):
            lo = min(b, max(0, a - need[i]))
            if L["kind"] == "attn":
                if i > 0:
                    x, k = gather(x, k)
                h = ops.rms_norm(x, L["ln1"], self.eps, self.plus_one)
                ctx = self._attn_ctx(i, L, h, pos_t, rows_t, plan)
                o = F.linear(ctx[lo:b], L["o"]) if b > lo else None
            else:
                dst = None
                if owner:
                    j = conv.index(i)
                    dst = stage[j * K1:(j + 1) * K1].reshape(-1)[:self.hidden * K1].view(1, self.hidden, K1)
                o = self._conv_rows(i, L, x, lo, b, B, T, state, tails, tail_dst=dst)
            if b > lo:
                xs = x[lo:b]
                hs = ops.add_rms_norm(xs, o, L["ln2"], self.eps, self.plus_one)
                # the MLP's down projection accumulates into the residual rows
                xs.addmm_(ops.swiglu(F.linear(hs, L["gu"])), L["down"].t())
        if not keep:
            x, k = gather(x, k)
            return x
        # the chunk's tails from the rank that ran its last token to every rank
        src = (T - 1) // unit
        if fused is not None:
            fused.gather_rows(0, n, n + (extra if owner else 0), n)
            got = fused.rows[1][n:n + extra]
        else:
            allt = torch.empty(sp.world * extra, self.hidden, dtype=self.dtype, device=self.device)
            dist_all_gather(allt, stage, sp)
            got = allt[src * extra:(src + 1) * extra]
        for j, i in enumerate(conv):
            t = got[j * K1:(j + 1) * K1].reshape(-1)[:self.hidden * K1].view(1, self.hidden, K1)
            if tails is not None:
                tails[1][i].copy_(t)
            else:
                state.conv[i] = t.clone()
        return x

    def _attn_common(self, i, L, h, pos_t, rows_t, plan, q_cols, k_col, v_col, rot, attend=None):
        T = h.shape[0]
        hq, hkv, D = self.hq_a, self.hkv_a, self.D
        qkv = F.linear(h, L["qkv"])
        q = torch.empty(T, hq, D, dtype=self.dtype, device=self.device)
        j = self.arena_index[i]
        ops.qk_norm_rope(qkv, q_cols, k_col, v_col, hq, hkv, D, L["qn"], L["kn"], self.eps, self.plus_one, pos_t,
                         self.theta, rot, q, self.arena.k[j], self.arena.v[j], rows_t)
        return qkv, (attend or ops.attend_packed)(q, self.arena.k[j], self.arena.v[j], plan)


class Qwen35(_HybridDecoder):
    """Qwen3.5 text decoder (qwen35.rs:625-752)."""

    plus_one = True  # zero-centred RMSNorm (qwen35.rs:160-176)

    def __init__(self, cfg: dict, weights: dict, dtype=torch.bfloat16, device="cuda", max_len=262144,
                 arena_rows=65536 + 8192):
        super().__init__(cfg, dtype, device, max_len, arena_rows)
        self.eps = cfg.get("rms_norm_eps", 1e-6)
        rp = cfg.get("rope_parameters") or {}
        self.theta = rp.get("rope_theta") or cfg.get("rope_theta") or 1e7
        self.rot = int(self.D * (rp.get("partial_rotary_factor") or 1.0)) & ~1
        self.gate = cfg.get("attn_output_gate", True)
        self.nk, self.nv = cfg["linear_num_key_heads"], cfg["linear_num_value_heads"]
        self.dk, self.dv = cfg["linear_key_head_dim"], cfg["linear_value_head_dim"]
        self.K = cfg.get("linear_conv_kernel_dim", 4)
        self.C = 2 * self.nk * self.dk + self.nv * self.dv
        w = lambda n: self._w(weights, n)  # noqa: E731
        self.embed_w = w("model.embed_tokens.weight")
        tied = cfg.get("tie_word_embeddings", False) or "lm_head.weight" not in weights
        self.lm_head = self.embed_w if tied else w("lm_head.weight")
        self.layers = []
        for i in range(self.n_layers):
            p = f"model.layers.{i}."
            L = dict(ln1=w(p + "input_layernorm.weight"), ln2=w(p + "post_attention_layernorm.weight"),
                     gu=torch.cat([w(p + "mlp.gate_proj.weight"), w(p + "mlp.up_proj.weight")], 0).contiguous(),
                     down=w(p + "mlp.down_proj.weight"))
            if cfg["layer_types"][i] == "linear_attention":
                a = p + "linear_attn."
                L.update(kind="gdn",
                         proj=torch.cat([w(a + "in_proj_qkv.weight"), w(a + "in_proj_z.weight"),
                                         w(a + "in_proj_b.weight"), w(a + "in_proj_a.weight")], 0).contiguous(),
                         conv_w=w(a + "conv1d.weight").reshape(self.C, self.K).contiguous(),
                         a_log=weights[a + "A_log"].to(self.device, torch.float32),
                         dt_bias=weights[a + "dt_bias"].to(self.device, torch.float32),
                         norm_w=w(a + "norm.weight"), out=w(a + "out_proj.weight"))
            else:
                s = p + "self_attn."
                L.update(kind="attn",
                         qkv=torch.cat([w(s + "q_proj.weight"), w(s + "k_proj.weight"), w(s + "v_proj.weight")],
                                       0).contiguous(),
                         qn=w(s + "q_norm.weight"), kn=w(s + "k_norm.weight"), o=w(s + "o_proj.weight"))
            self.layers.append(L)
        self.norm_w = w("model.norm.weight")

    def _attn(self, i, L, h, pos_t, rows_t, plan):
        """qwen35.rs:526-560: q|gate per head, (1+w) QK-norm, partial RoPE,
        sigmoid output gate."""
        hq, hkv, D = self.hq, self.hkv, self.D
        qw = 2 * D if self.gate else D
        qkv, ctx = self._attn_common(i, L, h, pos_t, rows_t, plan, (0, qw), hq * qw, hq * qw + hkv * D, self.rot)
        T = h.shape[0]
        out = ctx.view(T, hq * D)
        if self.gate:
            ops.sigmoid_gate(out, qkv[:, D:], qkv.stride(0), 2 * D, hq, D)
        return F.linear(out, L["o"])

    def _gdn(self, i, L, h, B, T, state, keep):
        """GatedDeltaNet::forward (qwen35.rs:415-453)."""
        nk, nv, dk, dv, C, K = self.nk, self.nv, self.dk, self.dv, self.C, self.K
        proj = F.linear(h, L["proj"])
        prev = None if state is None else state.gdn.get(i)
        tail_in = None if prev is None else prev[0]
        s_in = None if prev is None else prev[1]
        tail_out = torch.empty(1, C, K - 1, dtype=self.dtype, device=self.device) if keep else None
        s_out = torch.empty(1, nv, dk, dv, dtype=torch.float32, device=self.device) if keep else None
        conv_out = ops.gdn_conv(proj, B, T, C, L["conv_w"], tail_in, tail_out)
        ws = torch.empty(ops.gdn_workspace_size(B, T, nv, dk, dv), dtype=torch.uint8, device=self.device)
        y = ops.gdn_chunk_prefill(conv_out, proj[:, C + nv * dv:], proj.stride(0), proj[:, C:], proj.stride(0),
                                  L["a_log"], L["dt_bias"], L["norm_w"], self.eps, s_in, s_out, B, T, nk, nv, dk, dv,
                                  ws)
        if keep:
            state.gdn[i] = (tail_out, s_out)
        return F.linear(y, L["out"])


class Lfm2(_HybridDecoder):
    """LFM2 causal decoder (lfm2.rs:270-431)."""

    def __init__(self, cfg: dict, weights: dict, dtype=torch.bfloat16, device="cuda", max_len=128000,
                 arena_rows=65536 + 8192, split=None):
        """``split``: a :class:`cev_b200.tp.KvHeadSplit` to run the attention
        layers on this rank's KV-head group (the other ranks hold the rest)."""
        super().__init__(cfg, dtype, device, max_len, arena_rows, split)
        self.eps = cfg.get("norm_eps", 1e-5)
        self.theta = cfg.get("rope_theta") or (cfg.get("rope_parameters") or {}).get("rope_theta") or 1e6
        self.K = cfg.get("conv_L_cache", 3)
        w = lambda n: self._w(weights, n)  # noqa: E731
        self.embed_w = w("model.embed_tokens.weight")
        self.lm_head = self.embed_w
        self.layers = []
        d = self.hidden
        for i in range(self.n_layers):
            p = f"model.layers.{i}."
            f = p + "feed_forward."
            L = dict(ln1=w(p + "operator_norm.weight"), ln2=w(p + "ffn_norm.weight"),
                     gu=torch.cat([w(f + "w1.weight"), w(f + "w3.weight")], 0).contiguous(), down=w(f + "w2.weight"))
            if cfg["layer_types"][i] == "full_attention":
                s = p + "self_attn."
                qkv = torch.cat([w(s + "q_proj.weight"), w(s + "k_proj.weight"), w(s + "v_proj.weight")], 0)
                L.update(kind="attn",
                         qkv=qkv.contiguous() if split is None else split.slice_fused_qkv(qkv),
                         qn=w(s + "q_layernorm.weight"), kn=w(s + "k_layernorm.weight"), o=w(s + "out_proj.weight"))
            else:
                c = p + "conv."
                L.update(kind="conv", in_proj=w(c + "in_proj.weight"), out=w(c + "out_proj.weight"),
                         conv_w=w(c + "conv.weight").reshape(d, self.K).contiguous(),
                         bias=w(c + "conv.bias") if (c + "conv.bias") in weights else None)
            self.layers.append(L)
        self.norm_w = w("model.embedding_norm.weight")

    def _attn_ctx(self, i, L, h, pos_t, rows_t, plan):
        """lfm2.rs:145-171 up to the output projection: the attention output
        of every head, [T, Hq * D]; with a KV-head split, this rank's heads
        and one all-gather of the head outputs (or the gather fused into the
        attention epilogue)."""
        hq, hkv, D = self.hq_a, self.hkv_a, self.D
        fused = self.split.fused if self.split is not None else None
        _, ctx = self._attn_common(i, L, h, pos_t, rows_t, plan, (0, D), hq * D, (hq + hkv) * D, D,
                                   attend=None if fused is None else fused.attend)
        if fused is not None:  # already gathered by the attention epilogue
            return ctx
        ctx = ctx.view(h.shape[0], hq * D)
        return ctx if self.split is None else self.split.gather(ctx)

    def _attn(self, i, L, h, pos_t, rows_t, plan):
        return F.linear(self._attn_ctx(i, L, h, pos_t, rows_t, plan), L["o"])

    def _conv(self, i, L, h, B, T, state, keep):
        """ShortConv::forward (lfm2.rs:199-219)."""
        d, K = self.hidden, self.K
        bcx = F.linear(h, L["in_proj"])
        tail_in = None if state is None else state.conv.get(i)
        tail_out = torch.empty(1, d, K - 1, dtype=self.dtype, device=self.device) if keep else None
        y = ops.short_conv(bcx, B, T, d, L["conv_w"], L["bias"], tail_in, tail_out)
        if keep:
            state.conv[i] = tail_out
        return F.linear(y, L["out"])

    def _conv_rows(self, i, L, x, lo, b, B, T, state, tails=None, tail_dst=None):
        """ShortConv::forward (lfm2.rs:199-219) producing token rows [lo, b)
        of the residual stream x [B*T, H]: whole rows continuing the state's
        tails (B > 1), or rows of one sequence, for which the conv also runs
        over the K-1 rows before lo (their outputs are dropped) unless it
        starts at the sequence's first token, where the state's tails
        precede it.  ``tail_dst``: where the conv kernel writes the
        sequence's new tails (the run that ends the chunk)."""
        d, K = self.hidden, self.K
        tail_prev = tails[0][i] if tails is not None else (None if state is None else state.conv.get(i))
        if b <= lo:
            return None
        if B > 1:
            bcx = F.linear(ops.rms_norm(x[lo:b], L["ln1"], self.eps, self.plus_one), L["in_proj"])
            y = ops.short_conv(bcx, (b - lo) // T, T, d, L["conv_w"], L["bias"], tail_prev, None)
            return F.linear(y, L["out"])
        in_lo = max(0, lo - (K - 1))
        bcx = F.linear(ops.rms_norm(x[in_lo:b], L["ln1"], self.eps, self.plus_one), L["in_proj"])
        y = ops.short_conv(bcx, 1, b - in_lo, d, L["conv_w"], L["bias"], tail_prev if in_lo == 0 else None, tail_dst)
        return F.linear(y[lo - in_lo:], L["out"])


class ChunkGraphs:
    """The full-size prefill chunks of an LFM2 decoder (short-conv and
    attention layers; one GPU, or a KV-head split whose gathers run over
    NVLink peer memory with device-side epochs) replayed from CUDA graphs.

    A 512-token chunk of the cfg5 state is ~150 kernel launches whose host
    cost (Python, torch dispatch, ctypes) rivals their device time; a graph
    replays them with one launch.  Everything a chunk varies lives in
    device memory the graph reads: the token ids, positions and arena rows,
    the attention segment (its prefix length grows chunk by chunk), and the
    short-conv tails, which alternate between two static buffers (a chunk
    reads one and writes the other).  What changes the launches themselves
    -- the split-KV range count the planner picks for the prefix length,
    and which tail buffer is read -- selects the graph, captured on first
    use after one eager run of the same chunk (the chunk is idempotent: it
    rewrites the same K/V rows and tails).  After the last graph chunk the
    state's tails are copied out of the static buffers."""

    def __init__(self, dec: "Lfm2", T: int):
        from ._lib import Segment
        if any(L["kind"] not in ("conv", "attn") for L in dec.layers):
            raise ValueError("chunk graphs: LFM2 decoders only")
        if dec.split is not None and dec.split.fused is None:
            raise ValueError("chunk graphs: a KV-head split needs the fused (peer-memory) gathers")
        self.dec, self.T = dec, T
        dev = dec.device
        # pinned staging ring: a slot is rewritten only after its copy ran
        self.host = [torch.empty(3 * T + 7, dtype=torch.int32).pin_memory() for _ in range(4)]
        self.copied = [None] * len(self.host)
        self.slot = 0
        self.inputs = torch.zeros(3 * T + 7, dtype=torch.int32, device=dev)
        self.ids, self.pos, self.rows = self.inputs[:T], self.inputs[T:2 * T], self.inputs[2 * T:3 * T]
        self.seg = self.inputs[3 * T:]
        self.conv_layers = [i for i, L in enumerate(dec.layers) if L["kind"] == "conv"]
        self.tails = [{i: torch.zeros(1, dec.hidden, dec.K - 1, dtype=dec.dtype, device=dev)
                       for i in self.conv_layers} for _ in range(2)]
        self.graphs = {}
        self.pool = torch.cuda.graph_pool_handle()
        self.sms = torch.cuda.get_device_properties(dev).multi_processor_count
        self._seg_t = Segment

    def _split_count(self, seg) -> int:
        """Split-KV range count the planner picks for this chunk's segment
        (host only)."""
        import ctypes as C

        from ._lib import BF16, F32, check, lib
        dec = self.dec
        arr = (self._seg_t * 1)()
        arr[0].q_start, arr[0].q_len, arr[0].prefix_off, arr[0].prefix_len, arr[0].self_off = seg
        dt = BF16 if dec.dtype == torch.bfloat16 else F32
        tiles, ns, nb = C.c_int32(0), C.c_int32(1), C.c_int64(0)
        check(lib().cevk_attn_schedule(arr, 1, self.T, dec.arena.capacity, dec.hq_a, dec.hkv_a, dec.D, dt,
                                       C.byref(tiles)))
        check(lib().cevk_attn_split_plan(arr, 1, tiles.value, dec.hkv_a, dec.D, dt, self.sms, C.byref(ns),
                                         C.byref(nb)))
        return ns.value if dt == BF16 else 1

    def _body(self, plan, parity: int):
        dec, T = self.dec, self.T
        rd, wr = self.tails[parity], self.tails[1 - parity]
        if dec._token_split(1, T):
            return dec._layers_token_split(self.ids, 1, T, self.pos, self.rows, plan, None, True, tails=(rd, wr))
        x = ops.embed(dec.embed_w, self.ids)
        h = ops.rms_norm(x, dec.layers[0]["ln1"], dec.eps, dec.plus_one)
        m = None
        for i, L in enumerate(dec.layers):
            if m is not None:
                h = ops.add_rms_norm(x, m, L["ln1"], dec.eps, dec.plus_one, out=h)
            if L["kind"] == "attn":
                o = dec._attn(i, L, h, self.pos, self.rows, plan)
            else:
                y = ops.short_conv(F.linear(h, L["in_proj"]), 1, T, dec.hidden, L["conv_w"], L["bias"], rd[i], wr[i])
                o = F.linear(y, L["out"])
            h = ops.add_rms_norm(x, o, L["ln2"], dec.eps, dec.plus_one, out=h)
            m = F.linear(ops.swiglu(F.linear(h, L["gu"])), L["down"])
        ops.residual_add(x, m)
        return x

    def run(self, tokens, state: HybridState, parity: int) -> None:
        """One T-token chunk continuing ``state`` (keep): reads the tails in
        buffer ``parity``, writes the other."""
        dec, T = self.dec, self.T
        past = state.len
        base = state.start + past
        p0 = state.next_pos
        seg = (0, T, state.start, past, base)
        k = self.slot
        self.slot = (k + 1) % len(self.host)
        if self.copied[k] is not None:
            self.copied[k].synchronize()
        host = self.host[k]
        host[:T] = torch.as_tensor(tokens, dtype=torch.int32)
        host[T:2 * T] = torch.arange(p0, p0 + T, dtype=torch.int32)
        host[2 * T:3 * T] = torch.arange(base, base + T, dtype=torch.int32)
        host[3 * T:] = torch.tensor([*seg, 0, 0], dtype=torch.int32)  # tile_start 0, flags 0
        self.inputs.copy_(host, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        self.copied[k] = ev
        for i in self.conv_layers:
            cur = state.conv.get(i)
            if cur is None:
                self.tails[parity][i].zero_()
            elif cur.data_ptr() != self.tails[parity][i].data_ptr():
                self.tails[parity][i].copy_(cur)
        n_split = self._split_count(seg)
        key = (n_split, parity)
        entry = self.graphs.get(key)
        if entry is None:
            plan = ops.AttnPlan([seg], T, dec.arena.capacity, dec.hq_a, dec.hkv_a, dec.D, dec.dtype, dec.device,
                                n_split=n_split)
            plan.dev = self.seg  # the launches read the segment from the static inputs
            cur = torch.cuda.current_stream(dec.device)
            side = torch.cuda.Stream(device=dec.device)
            side.wait_stream(cur)
            with torch.cuda.stream(side):
                self._body(plan, parity)
            cur.wait_stream(side)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, pool=self.pool):
                self._body(plan, parity)
            entry = self.graphs[key] = (g, plan)
        entry[0].replay()
        for i in self.conv_layers:
            state.conv[i] = self.tails[1 - parity][i]
        state.len = past + T
        state.next_pos = p0 + T

    def release_tails(self, state: HybridState) -> None:
        """Give the state its own copies of tails that live in the static
        buffers (the next chunk or request overwrites those)."""
        for i in self.conv_layers:
            t = state.conv.get(i)
            if t is not None and any(t.data_ptr() == b[i].data_ptr() for b in self.tails):
                state.conv[i] = t.clone()


class HybridEngine:
    """Codes readout of the hybrid engine (hybrid.rs:155-165, 454-772)."""

    def __init__(self, decoder: _HybridDecoder, code_ids, pad_id: int, prefill_chunk=512, pass_tokens=2048,
                 prefix_cache_tokens=65536, device_readout=False, chunk_graphs=False):
        """``chunk_graphs``: replay the full-size prefill chunks of an LFM2
        decoder from CUDA graphs (:class:`ChunkGraphs`)."""
        self.device_readout = device_readout  # readouts stay on the device (on-device debias)
        self.decoder = decoder
        self.graphs = ChunkGraphs(decoder, prefill_chunk) if chunk_graphs else None
        self.head = decoder.head_rows(code_ids).contiguous()
        self.pad_id = pad_id
        self.prefill_chunk = prefill_chunk
        self.pass_tokens = pass_tokens
        self.cache = PrefixCache(prefix_cache_tokens)

    def prefill(self, prefix) -> HybridState:
        """The prefix in chunks into a state, cached (hybrid.rs:555-575)."""
        chunk = max(self.prefill_chunk, 1)
        st = self.decoder.new_state(len(prefix), self.cache)
        st.pins += 1
        graphs = getattr(self, "graphs", None)
        try:
            done, k = 0, 0
            while done < len(prefix):
                n = min(chunk, len(prefix) - done)
                if graphs is not None and n == chunk:
                    graphs.run(prefix[done:done + n], st, k & 1)
                    k += 1
                else:
                    self.decoder.forward(prefix[done:done + n], 1, n, range(done, done + n), st, True, self.cache)
                done += n
            if graphs is not None:
                graphs.release_tails(st)
        except BaseException:
            st.pins -= 1
            st.release()
            raise
        return st

    def rows(self, state: HybridState, rows) -> torch.Tensor:
        """A right-padded batch continuing ``state`` (hybrid.rs:595-617);
        returns the residual stream [B*T, H]."""
        t = max(len(r) for r in rows)
        ids = []
        for r in rows:
            ids += list(r) + [self.pad_id] * (t - len(r))
        pos = range(state.next_pos, state.next_pos + t)
        return self.decoder.forward(ids, len(rows), t, pos, state, False, self.cache), t

    def run(self, req: Request) -> Output:
        """hybrid.rs:697-739 with the Codes readout of 619-641."""
        d = self.decoder
        if len(req.prefix) == 0:
            # hybrid.rs:480-484: a Codes request whose questions share no
            # leading token bails (an internal error, not InputError); the
            # state-less row path of hybrid.rs:701 serves only bidirectional
            # whole-prompt rows
            raise RuntimeError("empty shared prefix")
        longest = max(len(req.prefix) + len(s) for s in req.suffixes)
        if longest >= d.max_len:
            raise InputError(f"prompt is {longest} tokens; the context limit is {d.max_len}")
        state = self.cache.get(req.prefix)
        cached = state is not None
        if cached:
            state.pins += 1
        else:
            state = self.prefill(list(req.prefix))
        try:
            readouts, start, br = [], 0, req.suffixes
            while start < len(br):
                end, longest = start + 1, len(br[start])
                while end < len(br):
                    l = max(longest, len(br[end]))
                    if l * (end + 1 - start) > self.pass_tokens:
                        break
                    longest = l
                    end += 1
                rows = br[start:end]
                x, t = self.rows(state, rows)
                g = torch.tensor([i * t + len(r) - 1 for i, r in enumerate(rows)], dtype=torch.int32)
                hid, logits = ops.readout(x, g.to(d.device), d.norm_w, d.eps, d.plus_one, self.head)
                if not self.device_readout:
                    hid, logits = hid.cpu(), logits.cpu()
                for i, r in enumerate(rows):
                    k = req.n_options[start + i]
                    readouts.append(Readout(logits[i, :k].clone(), hid[i].clone()))
                start = end
        finally:
            state.pins -= 1
            if not cached and not self.cache.put(list(req.prefix), state) and not state.pins:
                state.release()
        # a bounded device wait that gave up (an attention pipeline, a peer's
        # head rows) fails the request instead of serving its rows
        ops.device_status()
        return Output(readouts, len(req.prefix) + sum(len(s) for s in req.suffixes), cached)

    def run_many(self, reqs):
        return [self.run(r) for r in reqs]
