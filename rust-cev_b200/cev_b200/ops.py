"""Op-level entry points over the C ABI, on torch CUDA tensors.

These are the operations the reference runs as candle ops on its hot path
(``Attention::attend``, ``chunk_gated_delta_rule``, ``depthwise_conv1d`` and
the norms / RoPE / readout around them); each wrapper checks dtypes and
devices, passes raw pointers and the current CUDA stream, and raises
``CevkError`` with the library's message on failure.  Nothing here computes
on the CPU.
"""
from __future__ import annotations

import ctypes as C
import math

import torch

from ._lib import BF16, F32, SEG_BIDIRECTIONAL, Segment, check, lib  # noqa: F401 (SEG_BIDIRECTIONAL re-exported)


def _dt(*ts) -> int:
    dt = ts[0].dtype
    for t in ts:
        if t is not None and t.dtype != dt:
            raise TypeError(f"mixed dtypes {dt} / {t.dtype}")
    if dt == torch.bfloat16:
        return BF16
    if dt == torch.float32:
        return F32
    raise TypeError(f"unsupported dtype {dt}")


def _cuda(*ts) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("cev_b200 kernels take CUDA tensors only (no CPU path)")


def _p(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def _s():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


# ---------------------------------------------------------------------------
# Attention.
# ---------------------------------------------------------------------------
class AttnPlan:
    """Segments of one packed attention call, scheduled and on the device.

    ``segs``: iterable of (q_start, q_len, prefix_off, prefix_len, self_off)
    or (..., flags) -- see ``cevk_segment``; ``flags`` ``SEG_BIDIRECTIONAL``
    makes every row see all of its segment's own rows.  Built once per pass
    and shared by every layer.

    ``n_split``: key ranges per work tile (split-KV, for calls whose tiles
    underfill the GPU); None plans it from the SM count
    (``cevk_attn_split_plan``), 1 disables it.  A split plan owns a device
    workspace that serves one call at a time.
    """

    def __init__(self, segs, n_tokens: int, n_kv_rows: int, hq: int, hkv: int, head_dim: int, dtype: torch.dtype,
                 device, n_split: int | None = None):
        segs = list(segs)
        n = len(segs)
        arr = (Segment * max(n, 1))()
        for i, s in enumerate(segs):
            arr[i].q_start, arr[i].q_len, arr[i].prefix_off, arr[i].prefix_len, arr[i].self_off = (int(x) for x in s[:5])
            arr[i].flags = int(s[5]) if len(s) > 5 else 0
        tiles = C.c_int32(0)
        dt = BF16 if dtype == torch.bfloat16 else F32
        check(lib().cevk_attn_schedule(arr, n, n_tokens, n_kv_rows, hq, hkv, head_dim, dt, C.byref(tiles)))
        host = torch.frombuffer(bytearray(bytes(arr)[:n * C.sizeof(Segment)] or b"\0" * C.sizeof(Segment)),
                                dtype=torch.int32).clone()
        self.host = host
        self.dev = host.to(device)
        self.n_segs = n
        self.n_tiles = tiles.value
        self.n_tokens, self.n_kv_rows = n_tokens, n_kv_rows
        self.hq, self.hkv, self.head_dim = hq, hkv, head_dim
        if n_split is None:
            dev = torch.device(device)
            sms = torch.cuda.get_device_properties(dev).multi_processor_count if dev.type == "cuda" else 0
            ns, nb = C.c_int32(1), C.c_int64(0)
            check(lib().cevk_attn_split_plan(arr, n, self.n_tiles, hkv, head_dim, dt, sms, C.byref(ns), C.byref(nb)))
            n_split = ns.value
        self.n_split = max(1, int(n_split)) if dt == BF16 else 1
        ws = lib().cevk_attn_split_workspace_size(self.n_tiles, hkv, head_dim, self.n_split)
        self.workspace = torch.empty(ws, dtype=torch.uint8, device=device) if ws > 0 else None


def attend_packed(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, plan: AttnPlan, scale: float | None = None,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    """Packed block-masked attention (replaces ``Attention::attend`` +
    the engine's additive mask).  q [T, hq, D] (row-strided allowed),
    k/v [S, hkv, D] (row-strided allowed); returns o [T, hq, D]."""
    _cuda(q, k, v)
    dt = _dt(q, k, v)
    T, hq, D = q.shape
    S, hkv, _ = k.shape
    if q.stride(2) != 1 or q.stride(1) != D or k.stride(2) != 1 or k.stride(1) != D or v.stride() != k.stride():
        raise ValueError("attend_packed: heads must be contiguous within a row")
    if out is None:
        out = torch.empty(T, hq, D, dtype=q.dtype, device=q.device)
    scale = 1.0 / math.sqrt(D) if scale is None else scale
    if plan.n_split > 1:
        ws = plan.workspace
        check(lib().cevk_attn_packed_prefill_split(_p(q), _p(k), _p(v), _p(out), T, S, hq, hkv, D, q.stride(0),
                                                   k.stride(0), out.stride(0), _p(plan.dev), plan.n_segs,
                                                   plan.n_tiles, scale, plan.n_split, _p(ws), ws.numel(), dt, _s()))
    else:
        check(lib().cevk_attn_packed_prefill(_p(q), _p(k), _p(v), _p(out), T, S, hq, hkv, D, q.stride(0),
                                             k.stride(0), out.stride(0), _p(plan.dev), plan.n_segs, plan.n_tiles,
                                             scale, dt, _s()))
    return out


# ---------------------------------------------------------------------------
# Norms, RoPE, elementwise.
# ---------------------------------------------------------------------------
def qk_norm_rope(qkv: torch.Tensor, q_cols: tuple, k_col: int, v_col: int, hq: int, hkv: int, head_dim: int,
                 q_norm_w: torch.Tensor, k_norm_w: torch.Tensor, eps: float, plus_one: bool, pos: torch.Tensor,
                 theta: float, rotary_dim: int, q_out: torch.Tensor, k_arena: torch.Tensor, v_arena: torch.Tensor,
                 kv_rows: torch.Tensor) -> None:
    """Per-head RMSNorm + partial RoPE; writes q_out [T, hq, D] and the K/V
    arena rows ``kv_rows``.  ``q_cols`` = (first column, head stride) of the
    queries inside each ``qkv`` row."""
    _cuda(qkv, q_out, k_arena, v_arena, pos, kv_rows)
    dt = _dt(qkv, q_out, k_arena, v_arena, q_norm_w, k_norm_w)
    assert pos.dtype == torch.int32 and kv_rows.dtype == torch.int32
    T = qkv.shape[0]
    base = qkv[:, q_cols[0]:]
    check(lib().cevk_qk_norm_rope(_p(base), qkv.stride(0), q_cols[1], k_col - q_cols[0], v_col - q_cols[0],
                                  _p(q_norm_w), _p(k_norm_w), eps, int(plus_one), _p(pos), float(theta), rotary_dim,
                                  _p(q_out), _p(k_arena), _p(v_arena), k_arena.stride(0), _p(kv_rows), T, hq, hkv,
                                  head_dim, dt, _s()))


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float, plus_one: bool = False, out=None) -> torch.Tensor:
    _cuda(x, w)
    dt = _dt(x, w)
    n, h = x.shape
    out = torch.empty_like(x) if out is None else out
    check(lib().cevk_rms_norm(_p(x), None, None, _p(w), _p(out), n, h, eps, int(plus_one), dt, _s()))
    return out


def add_rms_norm(residual: torch.Tensor, add: torch.Tensor, w: torch.Tensor, eps: float, plus_one: bool = False,
                 out=None) -> torch.Tensor:
    """residual += add (in place); returns rms_norm(residual)."""
    _cuda(residual, add, w)
    dt = _dt(residual, add, w)
    n, h = residual.shape
    out = torch.empty_like(residual) if out is None else out
    check(lib().cevk_rms_norm(None, _p(residual), _p(add), _p(w), _p(out), n, h, eps, int(plus_one), dt, _s()))
    return out


def residual_add(residual: torch.Tensor, add: torch.Tensor) -> torch.Tensor:
    """residual += add in the model dtype (the decoder's ``x = x + h``)."""
    _cuda(residual, add)
    n, h = residual.shape
    check(lib().cevk_rms_norm(None, _p(residual), _p(add), None, None, n, h, 0.0, 0, _dt(residual, add), _s()))
    return residual


def swiglu(gu: torch.Tensor, out=None) -> torch.Tensor:
    _cuda(gu)
    n, two_i = gu.shape
    inter = two_i // 2
    out = torch.empty(n, inter, dtype=gu.dtype, device=gu.device) if out is None else out
    check(lib().cevk_swiglu(_p(gu), _p(out), n, inter, _dt(gu), _s()))
    return out


def embed(table: torch.Tensor, ids: torch.Tensor, out=None) -> torch.Tensor:
    _cuda(table, ids)
    assert ids.dtype == torch.int32
    n = ids.numel()
    out = torch.empty(n, table.shape[1], dtype=table.dtype, device=table.device) if out is None else out
    check(lib().cevk_embed(_p(table), _p(ids), _p(out), n, table.shape[1], table.shape[0], _dt(table), _s()))
    return out


def sigmoid_gate(a: torch.Tensor, gate: torch.Tensor, gate_row_stride: int, gate_head_stride: int, heads: int,
                 head_dim: int, out=None) -> torch.Tensor:
    """out = a * sigmoid(gate); a [T, heads*head_dim]; gate addressed by row
    and head strides (elements) from its data pointer."""
    _cuda(a, gate)
    out = a if out is None else out
    check(lib().cevk_sigmoid_gate(_p(a), _p(gate), gate_row_stride, gate_head_stride, _p(out), a.shape[0], heads,
                                  head_dim, _dt(a, gate), _s()))
    return out


def readout(x: torch.Tensor, rows: torch.Tensor, norm_w: torch.Tensor, eps: float, plus_one: bool,
            code_head: torch.Tensor):
    """Final norm at ``rows`` + f32 logits against ``code_head`` [n_codes, H].
    Returns (hidden f32 [n, H], logits f32 [n, n_codes])."""
    _cuda(x, rows, norm_w, code_head)
    assert code_head.dtype == torch.float32 and rows.dtype == torch.int32
    n = rows.numel()
    H = x.shape[1]
    hid = torch.empty(n, H, dtype=torch.float32, device=x.device)
    logits = torch.empty(n, code_head.shape[0], dtype=torch.float32, device=x.device)
    check(lib().cevk_readout(_p(x), _p(rows), n, _p(norm_w), eps, int(plus_one), _p(code_head), code_head.shape[0],
                             _p(hid), _p(logits), H, _dt(x, norm_w), _s()))
    return hid, logits


# ---------------------------------------------------------------------------
# Recurrent layers.
# ---------------------------------------------------------------------------
def gdn_conv(mixed: torch.Tensor, B: int, T: int, C_: int, conv_w: torch.Tensor, tail_in, tail_out,
             out=None) -> torch.Tensor:
    """mixed: [B*T, >=C] rows (row stride taken from the tensor); conv_w
    [C, K]; tail_in [B or 1, C, K-1] or None; tail_out [B, C, K-1] or None."""
    _cuda(mixed, conv_w, tail_in, tail_out)
    K = conv_w.shape[1]
    out = torch.empty(B * T, C_, dtype=mixed.dtype, device=mixed.device) if out is None else out
    tbs = 0 if tail_in is None or tail_in.shape[0] == 1 else tail_in.stride(0)
    check(lib().cevk_gdn_conv(_p(mixed), mixed.stride(0), _p(conv_w), _p(tail_in), tbs, _p(tail_out), _p(out), B, T,
                              C_, K, _dt(mixed, conv_w), _s()))
    return out


def gdn_workspace_size(B, T, nv, dk, dv) -> int:
    return lib().cevk_gdn_workspace_size(B, T, nv, dk, dv)


def gdn_chunk_prefill(conv_out, ab, ab_row_stride, z, z_row_stride, a_log, dt_bias, norm_w, eps, s_in, s_out,
                      B, T, nk, nv, dk, dv, workspace, out=None) -> torch.Tensor:
    """Chunked gated delta rule + gated RMSNorm; returns y [B*T, nv*dv]."""
    _cuda(conv_out, ab, z, a_log, dt_bias, norm_w, s_in, s_out, workspace)
    C_ = conv_out.shape[1]
    y = torch.empty(B * T, nv * dv, dtype=conv_out.dtype, device=conv_out.device) if out is None else out
    sbs = 0 if s_in is None or s_in.shape[0] == 1 else s_in.stride(0)
    check(lib().cevk_gdn_chunk_prefill(_p(conv_out), C_, _p(ab), ab_row_stride, _p(z), z_row_stride, _p(a_log),
                                       _p(dt_bias), _p(norm_w), eps, _p(s_in), sbs, _p(s_out), _p(y), B, T, nk, nv,
                                       dk, dv, _p(workspace), workspace.numel() * workspace.element_size(),
                                       _dt(conv_out, z), _s()))
    return y


def short_conv(bcx: torch.Tensor, B: int, T: int, d: int, conv_w: torch.Tensor, bias, tail_in, tail_out,
               out=None) -> torch.Tensor:
    """LFM2 gated short conv: bcx [B*T, 3d] -> y [B*T, d]."""
    _cuda(bcx, conv_w, bias, tail_in, tail_out)
    K = conv_w.shape[1]
    out = torch.empty(B * T, d, dtype=bcx.dtype, device=bcx.device) if out is None else out
    tbs = 0 if tail_in is None or tail_in.shape[0] == 1 else tail_in.stride(0)
    check(lib().cevk_short_conv(_p(bcx), _p(conv_w), _p(bias), _p(tail_in), tbs, _p(tail_out), _p(out), B, T, d, K,
                                _dt(bcx, conv_w), _s()))
    return out


def debias(logits: torch.Tensor, cf_logits, span: torch.Tensor, n_options: torch.Tensor, order: torch.Tensor):
    """Served (scores f32, probabilities f64) per question on the device
    (service.rs:288-348).  logits / cf_logits [n_variants, ld] f32 (cf may
    be None), span [n_q + 1], n_options [n_q], order [n_variants, ld] int32."""
    _cuda(logits, span, n_options, order, cf_logits)
    n_q, ld = n_options.shape[0], logits.shape[1]
    scores = torch.empty(n_q, ld, dtype=torch.float32, device=logits.device)
    probs = torch.empty(n_q, ld, dtype=torch.float64, device=logits.device)
    check(lib().cevk_debias(_p(logits), _p(cf_logits), ld, _p(span), _p(n_options), _p(order), n_q, _p(scores),
                            _p(probs), ld, _s()))
    return scores, probs


def device_status() -> None:
    """Synchronise and raise if a bounded device wait gave up."""
    check(lib().cevk_device_status())
