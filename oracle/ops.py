"""Op-level restatement of the candle math on the reference's hot path.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Every function names the reference line it follows.  Tensors are torch CPU
tensors; ``dtype`` is the "model dtype" (f32 for exact parity runs, bf16 for
drift checks): like candle, matmuls and stored activations use it while the
softmax, the GDN core and the norms' accumulation run in f32.
"""
from __future__ import annotations

import math

import torch

NEG_INF = float("-inf")


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """candle_nn::ops::rms_norm: ``x * rsqrt(mean(x^2) + eps) * w`` over the
    last dim, accumulated in f32 and returned in x's dtype
    (qwen3.rs:193-194,254-255; lfm2.rs:148-149)."""
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return (y * w.float()).to(x.dtype)


def rope_inv_freq(dim: int, theta: float) -> torch.Tensor:
    """Inverse frequencies: ``1f32 / (theta.powf(i/dim) as f32)``, the power
    in f64 (qwen3.rs:109-112; qwen35.rs:191; lfm2.rs:97)."""
    vals = [1.0 / float(torch.tensor(theta ** (i / dim), dtype=torch.float32)) for i in range(0, dim, 2)]
    return torch.tensor(vals, dtype=torch.float32)


def rope_cos_sin(pos: torch.Tensor, dim: int, theta: float, dtype: torch.dtype):
    """cos/sin at explicit positions, f32 product then cast to the model
    dtype (qwen3.rs:115-117,122 -- the table rows ``index_select``-ed at pos
    are the same numbers)."""
    inv = rope_inv_freq(dim, theta)
    f = pos.to(torch.float32)[:, None] * inv[None, :]
    return f.cos().to(dtype), f.sin().to(dtype)


def rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """candle_nn::rotary_emb::rope (half-split, not interleaved) on
    x (..., T, D) with cos/sin (T, D/2) (qwen3.rs:121-123)."""
    half = x.shape[-1] // 2
    x1, x2 = x[..., :half], x[..., half:]
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1)


def rope_partial(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Rotate the first ``2 * cos.shape[-1]`` dims only (qwen35.rs:231-240)."""
    rot = 2 * cos.shape[-1]
    if rot == x.shape[-1]:
        return rope(x, cos, sin)
    return torch.cat([rope(x[..., :rot], cos, sin), x[..., rot:]], dim=-1)


def repeat_kv(x: torch.Tensor, groups: int) -> torch.Tensor:
    """(B, Hkv, S, D) -> (B, Hkv*groups, S, D), kv head h serving query heads
    h*groups .. h*groups+groups-1 (qwen3.rs:145-151)."""
    if groups == 1:
        return x
    b, h, s, d = x.shape
    return x[:, :, None].expand(b, h, groups, s, d).reshape(b, h * groups, s, d)


def attend(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, mask: torch.Tensor) -> torch.Tensor:
    """Generic (CUDA/CPU) attention of the reference (qwen3.rs:206-220;
    qwen35.rs:563-579; lfm2.rs:160-168): repeat_kv, ``q k^T`` in the model
    dtype, cast to f32, scale, add the additive mask, softmax in f32, cast
    back, ``p v``.  q (B, Hq, T, D); k, v (B, Hkv, S, D); mask broadcastable
    to (B, Hq, T, S)."""
    d = q.shape[-1]
    scale = 1.0 / math.sqrt(d)
    g = q.shape[1] // k.shape[1]
    b, hq, t, _ = q.shape
    s = k.shape[2]
    if b * hq * t * s <= (1 << 27):
        kk, vv = repeat_kv(k, g), repeat_kv(v, g)
        scores = torch.matmul(q, kk.transpose(-1, -2)).float() * scale + mask.float()
        p = torch.softmax(scores, dim=-1).to(v.dtype)
        return torch.matmul(p, vv)
    # Large shapes (long states at the benchmark configs): the same
    # arithmetic one query head at a time, so that the f32 score matrix
    # held at once is (B, 1, T, S) instead of (B, Hq, T, S).  Every row's
    # softmax is independent of the other heads, so the result is the same.
    out = torch.empty(b, hq, t, v.shape[-1], dtype=v.dtype)
    m = mask.float()
    per_head = m.dim() == 4 and m.shape[1] == hq
    for h in range(hq):
        mh = m[:, h:h + 1] if per_head else m
        sc = torch.matmul(q[:, h:h + 1], k[:, h // g:h // g + 1].transpose(-1, -2)).float() * scale + mh
        p = torch.softmax(sc, dim=-1).to(v.dtype)
        out[:, h:h + 1] = torch.matmul(p, v[:, h // g:h // g + 1])
    return out


def segment_mask(segments: list[int], past: int) -> torch.Tensor:
    """Additive mask for ``n`` new tokens after ``past`` cached ones: a new
    token sees every cached token plus earlier new tokens of its own segment
    (qwen3.rs:157-169)."""
    n = len(segments)
    m = torch.zeros(n, past + n)
    seg = torch.tensor(segments)
    i = torch.arange(n)[:, None]
    j = torch.arange(n)[None, :]
    hide = (j > i) | (seg[None, :] != seg[:, None])
    m[:, past:][hide] = NEG_INF
    return m


def causal_mask(t: int, past: int) -> torch.Tensor:
    """(T, past+T): full past, causal over the new tokens
    (lfm2.rs:282-290; qwen35.rs:471-479 ``branch_mask``)."""
    m = torch.zeros(t, past + t)
    i = torch.arange(t)[:, None]
    j = torch.arange(t)[None, :]
    m[:, past:][j > i] = NEG_INF
    return m


def bidirectional_mask(t: int, lengths: list[int]) -> torch.Tensor:
    """(B, T, T) additive mask of ``Attn::Bidirectional`` rows
    (qwen35.rs:483-498, decoder.rs:109-116): every real token of a row sees
    every real token of it, padding columns are hidden, and a padding query
    keeps its own diagonal so its softmax stays finite."""
    b = len(lengths)
    m = torch.zeros(b, t, t)
    for r, n in enumerate(lengths):
        m[r, :, n:] = NEG_INF
        for i in range(n, t):
            m[r, i, i] = 0.0
    return m


def depthwise_conv1d(x: torch.Tensor, kernel: torch.Tensor) -> torch.Tensor:
    """x (B, C, L), kernel (C, 1, K) -> (B, C, L-K+1) as K shifted
    multiply-adds in x's dtype (decoder.rs:137-151)."""
    _, c, l = x.shape
    k = kernel.shape[2]
    out = l + 1 - k
    w = kernel.reshape(1, c, k).to(x.dtype)
    acc = None
    for i in range(k):
        term = x[:, :, i:i + out] * w[:, :, i:i + 1]
        acc = term if acc is None else acc + term
    return acc


def silu(x: torch.Tensor) -> torch.Tensor:
    """candle_nn::ops::silu in x's dtype."""
    return (x.float() * torch.sigmoid(x.float())).to(x.dtype)


def softplus(x: torch.Tensor) -> torch.Tensor:
    """``max(x, 0) + ln(1 + e^{-|x|})`` (qwen35.rs:243-248)."""
    return x.relu() + (torch.exp(-x.abs()) + 1.0).log()


def l2norm(x: torch.Tensor) -> torch.Tensor:
    """``x / sqrt(sum(x^2) + 1e-6)`` over the last dim (qwen35.rs:251-254)."""
    return x / (x.pow(2).sum(-1, keepdim=True) + 1e-6).sqrt()


def inv_unit_lower(m: torch.Tensor) -> torch.Tensor:
    """Inverse of ``I + strict_lower(m)`` over the last two dims by recursive
    block inversion (qwen35.rs:266-296)."""
    n = m.shape[-1]
    lead = m.shape[:-2]
    mm = m.reshape(-1, n, n)
    strict = mm * (torch.tril(torch.ones(n, n, dtype=m.dtype)) - torch.eye(n, dtype=m.dtype))
    return _inv_unit_lower_strict(strict).reshape(*lead, n, n)


def _inv_unit_lower_strict(m: torch.Tensor) -> torch.Tensor:
    """(qwen35.rs:277-296)."""
    b, n, _ = m.shape
    if n == 1:
        return torch.ones(b, 1, 1, dtype=m.dtype)
    h = n // 2
    a = m[:, :h, :h]
    c = m[:, h:, :h]
    d = m[:, h:, h:]
    if n - h == h:
        both = _inv_unit_lower_strict(torch.cat([a, d], 0).contiguous())
        ai, di = both[:b], both[b:]
    else:
        ai, di = _inv_unit_lower_strict(a.contiguous()), _inv_unit_lower_strict(d.contiguous())
    ll = -torch.matmul(torch.matmul(di, c), ai)
    top = torch.cat([ai, torch.zeros(b, h, n - h, dtype=m.dtype)], 2)
    bottom = torch.cat([ll, di], 2)
    return torch.cat([top, bottom], 1)


GDN_CHUNK = 64


def chunk_gated_delta_rule(q, k, v, g, beta, s0=None):
    """The chunked gated delta rule, all f32 (qwen35.rs:301-368).

    q, k (B, H, T, dk); v (B, H, T, dv); g, beta (B, H, T); s0 (B, H, dk, dv).
    Returns (out (B, H, T, dv), state (B, H, dk, dv)).
    """
    C = GDN_CHUNK
    b, h, t, dk = q.shape
    dv = v.shape[3]
    q = l2norm(q.float()) * (dk ** -0.5)
    k = l2norm(k.float())
    v, g, beta = v.float(), g.float(), beta.float()
    pad = (C - t % C) % C
    tp = t + pad
    n = tp // C

    def padt(x):
        if pad == 0:
            return x
        shape = list(x.shape)
        shape[2] = pad
        return torch.cat([x, torch.zeros(shape, dtype=x.dtype)], 2)

    q, k, v, g, beta = padt(q), padt(k), padt(v), padt(g), padt(beta)
    beta4 = beta[..., None]
    v_beta = (v * beta4).reshape(b, h, n, C, dv)
    k_beta = (k * beta4).reshape(b, h, n, C, dk)
    q = q.reshape(b, h, n, C, dk)
    k = k.reshape(b, h, n, C, dk)
    g = g.reshape(b, h, n, C)
    cum = g.cumsum(3)
    pair = cum[..., :, None] - cum[..., None, :]
    lower = torch.tril(torch.ones(C, C))
    pair = (pair + (1.0 - lower) * -1e30).exp()
    kt = k.transpose(-1, -2)
    ut = torch.matmul(k_beta, kt) * pair
    intra = torch.matmul(q, kt) * pair
    ecum = cum.exp()[..., None]
    inv = inv_unit_lower(ut)
    new_values = torch.matmul(inv, v_beta)
    k_cumdecay = torch.matmul(inv, k_beta * ecum)
    qd = q * ecum
    last = cum[..., C - 1:C]
    kd = k * (last - cum).exp()[..., None]
    chunk_decay = last.exp()[..., None]
    s = torch.zeros(b, h, dk, dv) if s0 is None else s0.float().clone()
    outs = []
    for i in range(n):
        v_new = new_values[:, :, i] - torch.matmul(k_cumdecay[:, :, i], s)
        out = torch.matmul(qd[:, :, i], s) + torch.matmul(intra[:, :, i], v_new)
        outs.append(out)
        s = s * chunk_decay[:, :, i] + torch.matmul(kd[:, :, i].transpose(-1, -2), v_new)
    out = torch.stack(outs, 2).reshape(b, h, tp, dv)
    return out[:, :, :t], s


def gated_delta_recurrence(q, k, v, g, beta, s0=None):
    """Token-by-token recurrence the chunked rule must equal; the reference's
    own check (qwen35.rs:788-821).  Same argument shapes as
    :func:`chunk_gated_delta_rule`."""
    b, h, t, dk = q.shape
    dv = v.shape[3]
    qn = l2norm(q.float()) * (dk ** -0.5)
    kn = l2norm(k.float())
    s = torch.zeros(b, h, dk, dv) if s0 is None else s0.float().clone()
    out = torch.zeros(b, h, t, dv)
    for ti in range(t):
        s = s * g[:, :, ti].float().exp()[..., None, None]
        mem = torch.einsum("bhij,bhi->bhj", s, kn[:, :, ti])
        delta = (v[:, :, ti].float() - mem) * beta[:, :, ti].float()[..., None]
        s = s + kn[:, :, ti][..., :, None] * delta[..., None, :]
        out[:, :, ti] = torch.einsum("bhij,bhi->bhj", s, qn[:, :, ti])
    return out, s
