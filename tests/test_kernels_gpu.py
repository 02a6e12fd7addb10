"""Kernel parity on the GPU: every op of the C ABI against the CPU oracle on
the same seeded inputs.  Tolerances: max-abs 2e-2 for bf16 attention / GDN
outputs and 1e-4 for f32 (the bounds the decision forward is held to)."""
import math

import pytest
import torch

from oracle import ops as ref

pytestmark = pytest.mark.gpu

BF16_TOL = 2e-2
F32_TOL = 1e-4


def cuda():
    return torch.device("cuda")


def oracle_segments(q, k, v, segs, scale=None, model_dtype=torch.float32):
    """Attention per segment with the reference's generic path
    (qwen3.rs:206-220) on CPU: prefix rows in full, own rows causally.
    ``model_dtype`` is the dtype the reference computes q k^T and P V in
    (P cast to it before P V); f32 gives the exact result."""
    q, k, v = (x.cpu().to(model_dtype) for x in (q, k, v))
    out = torch.zeros(q.shape)
    for (qs, ql, po, pl, so) in segs:
        if ql == 0:
            continue
        kk = torch.cat([k[po:po + pl], k[so:so + ql]], 0)
        vv = torch.cat([v[po:po + pl], v[so:so + ql]], 0)
        mask = ref.causal_mask(ql, pl).to(model_dtype)
        o = ref.attend(q[qs:qs + ql].transpose(0, 1)[None], kk.transpose(0, 1)[None], vv.transpose(0, 1)[None], mask)
        out[qs:qs + ql] = o[0].transpose(0, 1).float()
    return out


def check_bf16_attention(out, q, k, v, segs, n_tok):
    """The kernel must be within 2e-2 of the exact result (the bound the
    decision forward is held to) AND at least as accurate as the
    reference's own bf16 arithmetic on the same inputs."""
    exact = oracle_segments(q, k, v, segs)
    ref_bf16 = oracle_segments(q, k, v, segs, model_dtype=torch.bfloat16)
    rows = torch.zeros(n_tok, dtype=torch.bool)
    for (qs, ql, *_r) in segs:
        rows[qs:qs + ql] = True
    err = (out.float().cpu()[rows] - exact[rows]).abs().max().item()
    ref_err = (ref_bf16[rows] - exact[rows]).abs().max().item()
    assert err < BF16_TOL, err
    assert err <= ref_err + 1e-4, (err, ref_err)


def rand_attn(n_tok, n_kv, hq, hkv, D, dtype, seed):
    g = torch.Generator().manual_seed(seed)

    def rn(*s):
        x = torch.randn(*s, generator=g)
        return (x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6)).to(dtype).to("cuda")

    return rn(n_tok, hq, D), rn(n_kv, hkv, D), torch.randn(n_kv, hkv, D, generator=g).to(dtype).to("cuda")


CASES = [
    # (hq, hkv, D, segments (q_start, q_len, prefix_off, prefix_len, self_off), n_tok, n_kv)
    (16, 8, 128, [(0, 64, 0, 2048, 2048), (64, 64, 0, 2048, 2112), (128, 64, 2176, 2048, 4224)], 192, 4288),
    (2, 1, 128, [(0, 37, 0, 100, 300), (37, 150, 0, 100, 337), (187, 5, 100, 0, 487)], 192, 492),
    (4, 1, 64, [(0, 70, 0, 513, 600), (70, 33, 513, 64, 670)], 103, 703),
    (8, 2, 256, [(0, 48, 0, 300, 300), (48, 100, 0, 300, 348)], 148, 448),
    (16, 4, 256, [(0, 128, 0, 1000, 1000)], 128, 1128),
    (32, 8, 64, [(0, 64, 0, 700, 700), (64, 3, 0, 700, 764)], 67, 767),
    (8, 8, 128, [(0, 200, 0, 0, 0)], 200, 200),
    # head_dim 64, one and two heads per KV head: a 128-row tile spans two
    # own key blocks, so the odd block (the second softmax group's) is fully
    # masked for half the rows; one-block segments leave that group idle
    (4, 4, 64, [(0, 300, 0, 0, 0)], 300, 300),
    (8, 4, 64, [(0, 5, 0, 0, 0), (5, 130, 0, 70, 135), (135, 64, 70, 1, 265)], 199, 329),
]


@pytest.mark.parametrize("case", range(len(CASES)))
def test_attention_bf16_matches_oracle(case):
    from cev_b200 import ops
    hq, hkv, D, segs, n_tok, n_kv = CASES[case]
    q, k, v = rand_attn(n_tok, n_kv, hq, hkv, D, torch.bfloat16, 100 + case)
    plan = ops.AttnPlan(segs, n_tok, n_kv, hq, hkv, D, torch.bfloat16, "cuda")
    out = ops.attend_packed(q, k, v, plan)
    ops.device_status()
    check_bf16_attention(out, q, k, v, segs, n_tok)


@pytest.mark.parametrize("case", [0, 1, 3])
def test_attention_f32_matches_oracle(case):
    from cev_b200 import ops
    hq, hkv, D, segs, n_tok, n_kv = CASES[case]
    q, k, v = rand_attn(n_tok, n_kv, hq, hkv, D, torch.float32, 200 + case)
    plan = ops.AttnPlan(segs, n_tok, n_kv, hq, hkv, D, torch.float32, "cuda")
    out = ops.attend_packed(q, k, v, plan)
    want = oracle_segments(q, k, v, segs)
    rows = torch.zeros(n_tok, dtype=torch.bool)
    for (qs, ql, *_r) in segs:
        rows[qs:qs + ql] = True
    assert (out.cpu()[rows] - want[rows]).abs().max().item() < F32_TOL


@pytest.mark.parametrize("case", [1, 2, 5, 7, 8])
def test_attention_ignores_nonfinite_rows_outside_segments(case):
    """Rows of K/V outside every segment's visible range may hold anything
    (NaN/Inf garbage of an uninitialised arena): outputs stay exact."""
    from cev_b200 import ops
    hq, hkv, D, segs, n_tok, n_kv = CASES[case]
    q, k, v = rand_attn(n_tok, n_kv, hq, hkv, D, torch.bfloat16, 300 + case)
    used = torch.zeros(n_kv, dtype=torch.bool)
    for (qs, ql, po, pl, so) in segs:
        used[po:po + pl] = True
        used[so:so + ql] = True
    k2, v2 = k.clone(), v.clone()
    k2[~used.cuda()] = float("nan")
    v2[~used.cuda()] = float("inf")
    plan = ops.AttnPlan(segs, n_tok, n_kv, hq, hkv, D, torch.bfloat16, "cuda")
    a = ops.attend_packed(q, k, v, plan)
    b = ops.attend_packed(q, k2, v2, plan)
    rows = torch.zeros(n_tok, dtype=torch.bool)
    for (qs, ql, *_r) in segs:
        rows[qs:qs + ql] = True
    assert torch.equal(a[rows.cuda()], b[rows.cuda()])


def test_attention_repeatable_and_strided_q():
    """Q read through a row stride (a view into a fused projection) gives
    the same bits; two launches agree bit for bit."""
    from cev_b200 import ops
    hq, hkv, D, segs, n_tok, n_kv = CASES[0]
    q, k, v = rand_attn(n_tok, n_kv, hq, hkv, D, torch.bfloat16, 7)
    plan = ops.AttnPlan(segs, n_tok, n_kv, hq, hkv, D, torch.bfloat16, "cuda")
    a = ops.attend_packed(q, k, v, plan)
    wide = torch.zeros(n_tok, hq + 8, D, dtype=q.dtype, device="cuda")
    wide[:, :hq] = q
    b = ops.attend_packed(wide[:, :hq], k, v, plan)
    c = ops.attend_packed(q, k, v, plan)
    assert torch.equal(a, b) and torch.equal(a, c)


def test_attention_cfg2_shape_sampled():
    """The cfg2 workload itself (32 requests x (2048 prefix + 16 x 64)),
    checked against the oracle on a sample of requests."""
    from cev_b200 import workloads
    wb = workloads.AttentionBatch()
    out = wb.run()
    torch.cuda.synchronize()
    from cev_b200 import ops
    ops.device_status()
    for rq in (0, 17, 31):
        segs = [s for s in wb.segments if s[0] // 1024 == rq]
        check_bf16_attention(out, wb.q, wb.k, wb.v, segs, wb.n_tokens)


@pytest.mark.parametrize("dtype,tol", [(torch.bfloat16, 2e-2), (torch.float32, 1e-5)])
@pytest.mark.parametrize("plus_one,rot", [(False, 128), (True, 32), (False, 64)])
def test_qk_norm_rope_matches_oracle(dtype, tol, plus_one, rot):
    from cev_b200 import ops
    torch.manual_seed(1)
    T, hq, hkv, D = 37, 4, 2, 128
    theta = 1e6
    qkv = torch.randn(T, (hq + 2 * hkv) * D).to(dtype)
    qw = (torch.rand(D) * 0.5 + 0.5).to(dtype)
    kw = (torch.rand(D) * 0.5 + 0.5).to(dtype)
    pos = torch.randint(0, 70000, (T,), dtype=torch.int32)
    rows = torch.randperm(64)[:T].to(torch.int32)
    qo = torch.empty(T, hq, D, dtype=dtype, device="cuda")
    ka = torch.zeros(64, hkv, D, dtype=dtype, device="cuda")
    va = torch.zeros(64, hkv, D, dtype=dtype, device="cuda")
    ops.qk_norm_rope(qkv.cuda(), (0, D), hq * D, (hq + hkv) * D, hq, hkv, D, qw.cuda(), kw.cuda(), 1e-6, plus_one,
                     pos.cuda(), theta, rot, qo, ka, va, rows.cuda())
    wq = (qw.float() + 1).to(dtype) if plus_one else qw
    wk = (kw.float() + 1).to(dtype) if plus_one else kw
    x = qkv.float().reshape(T, hq + 2 * hkv, D)
    cos, sin = ref.rope_cos_sin(pos.long(), rot, theta, torch.float32)
    want_q = ref.rope_partial(ref.rms_norm(x[:, :hq].transpose(0, 1).to(dtype), wq, 1e-6).float(), cos, sin).transpose(0, 1)
    want_k = ref.rope_partial(ref.rms_norm(x[:, hq:hq + hkv].transpose(0, 1).to(dtype), wk, 1e-6).float(), cos, sin).transpose(0, 1)
    # bf16: the output is rounded once to bf16 (relative half-ulp 2^-9)
    scale_q = want_q.abs().max().item() if dtype == torch.bfloat16 else 1.0
    scale_k = want_k.abs().max().item() if dtype == torch.bfloat16 else 1.0
    assert (qo.float().cpu() - want_q).abs().max().item() < tol * scale_q
    assert (ka.float().cpu()[rows.long()] - want_k).abs().max().item() < tol * scale_k
    assert torch.equal(va.cpu()[rows.long()], qkv.reshape(T, -1, D)[:, hq + hkv:])


def close(got, want, tol, rel):
    """max |got - want| < tol, relative to max |want| when ``rel`` (a value
    rounded once to bf16 carries a relative half-ulp of 2^-9)."""
    got, want = got.float().cpu(), want.float().cpu()
    scale = want.abs().max().item() if rel else 1.0
    return (got - want).abs().max().item() < tol * max(scale, 1e-6)


@pytest.mark.parametrize("dtype,tol", [(torch.bfloat16, 1e-2), (torch.float32, 1e-5)])
def test_norms_swiglu_embed_readout(dtype, tol):
    from cev_b200 import ops
    rel = dtype == torch.bfloat16
    torch.manual_seed(2)
    n, H, I = 9, 256, 512
    x = torch.randn(n, H).to(dtype)
    add = torch.randn(n, H).to(dtype)
    w = (torch.rand(H) + 0.5).to(dtype)
    out = ops.rms_norm(x.cuda(), w.cuda(), 1e-6)
    assert close(out, ref.rms_norm(x, w, 1e-6), tol, rel)
    res = x.cuda().clone()
    out = ops.add_rms_norm(res, add.cuda(), w.cuda(), 1e-6, plus_one=True)
    s = (x + add)
    assert torch.equal(res.cpu(), s)
    assert close(out, ref.rms_norm(s, (w.float() + 1).to(dtype), 1e-6), tol, rel)
    res2 = x.cuda().clone()
    ops.residual_add(res2, add.cuda())
    assert torch.equal(res2.cpu(), s)
    gu = torch.randn(n, 2 * I).to(dtype)
    y = ops.swiglu(gu.cuda())
    assert close(y, ref.silu(gu[:, :I].float()) * gu[:, I:].float(), tol, rel)
    table = torch.randn(100, H).to(dtype)
    ids = torch.randint(0, 100, (n,), dtype=torch.int32)
    assert torch.equal(ops.embed(table.cuda(), ids.cuda()).cpu(), table[ids.long()])
    head = torch.randn(5, H)
    rows = torch.tensor([0, 4, 8], dtype=torch.int32)
    hid, logits = ops.readout(x.cuda(), rows.cuda(), w.cuda(), 1e-6, False, head.cuda())
    want_h = ref.rms_norm(x[rows.long()], w, 1e-6).float()
    assert close(hid, want_h, tol, rel)
    assert close(logits, hid.cpu() @ head.t(), 1e-4, True)
    a = torch.randn(n, 2 * 64).to(dtype)
    qg = torch.randn(n, 2, 2 * 64).to(dtype)   # per head [q | gate] like Qwen3.5's q_proj
    gated = ops.sigmoid_gate(a.cuda().clone(), qg.cuda()[:, :, 64:], 2 * 2 * 64, 2 * 64, 2, 64)
    want = a.float().reshape(n, 2, 64) * torch.sigmoid(qg[:, :, 64:].float())
    assert close(gated, want.reshape(n, -1), tol, rel)


@pytest.mark.parametrize("dtype,tol", [(torch.bfloat16, 1e-2), (torch.float32, 1e-5)])
@pytest.mark.parametrize("B,T,bcast", [(1, 50, False), (3, 7, True), (2, 1, False)])
def test_short_conv_matches_oracle(dtype, tol, B, T, bcast):
    """lfm2.rs:199-219 with a tail state (broadcast from one prefix or per row)."""
    from cev_b200 import ops
    torch.manual_seed(3)
    d, K = 64, 3
    bcx = torch.randn(B, T, 3 * d).to(dtype)
    w = torch.randn(d, 1, K).to(dtype)
    tail = torch.randn(1 if bcast else B, d, K - 1).to(dtype)
    tail_out = torch.empty(B, d, K - 1, dtype=dtype, device="cuda")
    y = ops.short_conv(bcx.reshape(B * T, 3 * d).cuda(), B, T, d, w.reshape(d, K).cuda(), None, tail.cuda(), tail_out)
    bcu = bcx.transpose(1, 2)
    bu = bcu[:, :d] * bcu[:, 2 * d:]
    full = torch.cat([tail.expand(B, d, K - 1), bu], 2)
    z = ref.depthwise_conv1d(full.float(), w.float())
    want = (bcu[:, d:2 * d].float() * z).transpose(1, 2)
    rel = dtype == torch.bfloat16
    assert close(y.reshape(B, T, d), want, tol, rel)
    assert close(tail_out, full[:, :, T:T + K - 1], tol, rel)


def gdn_inputs(B, T, nk, nv, dk, dv, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    C_ = 2 * nk * dk + nv * dv
    conv_out = (torch.randn(B, T, C_, generator=g) * 0.5).to(dtype)
    ab = torch.randn(B, T, 2 * nv, generator=g).to(dtype)
    z = torch.randn(B, T, nv * dv, generator=g).to(dtype)
    a_log = torch.rand(nv, generator=g) * 2
    dt_bias = torch.rand(nv, generator=g)
    norm_w = (torch.rand(dv, generator=g) + 0.5).to(dtype)
    s0 = torch.randn(1, nv, dk, dv, generator=g) * 0.1
    return conv_out, ab, z, a_log, dt_bias, norm_w, s0


def gdn_oracle(conv_out, ab, z, a_log, dt_bias, norm_w, s0, nk, nv, dk, dv, eps=1e-6):
    """qwen35.rs:432-451 after the conv, on CPU."""
    B, T, _ = conv_out.shape
    c = conv_out.float()
    kd = nk * dk
    q = c[..., :kd].reshape(B, T, nk, dk).transpose(1, 2)
    k = c[..., kd:2 * kd].reshape(B, T, nk, dk).transpose(1, 2)
    v = c[..., 2 * kd:].reshape(B, T, nv, dv).transpose(1, 2)
    rep = nv // nk
    q = q[:, :, None].expand(B, nk, rep, T, dk).reshape(B, nv, T, dk)
    k = k[:, :, None].expand(B, nk, rep, T, dk).reshape(B, nv, T, dk)
    beta = torch.sigmoid(ab[..., :nv].float()).transpose(1, 2)
    g = (ref.softplus(ab[..., nv:].float() + dt_bias) * -a_log.exp()).transpose(1, 2)
    core, s = ref.chunk_gated_delta_rule(q, k, v, g, beta, None if s0 is None else s0.expand(B, nv, dk, dv))
    core = core.transpose(1, 2)
    normed = core / (core.pow(2).mean(-1, keepdim=True) + eps).sqrt() * norm_w.float()
    y = normed * ref.silu(z.float().reshape(B, T, nv, dv))
    return y.reshape(B, T, nv * dv), s


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("hq,hkv,D", [(16, 8, 128), (4, 1, 64), (8, 2, 256)])
def test_attention_bidirectional_rows_match_oracle(dtype, hq, hkv, D):
    """Right-padded rows under ``Attn::Bidirectional`` (qwen35.rs:483-498):
    each row's real tokens are one CEVK_SEG_BIDIRECTIONAL segment; its pad
    tokens a causal segment over the real ones (pads never reach a real
    token).  Real rows are compared with the reference's mask."""
    from cev_b200 import ops
    T, lengths = 150, [150, 37, 1, 129]
    n = T * len(lengths)
    q, k, v = rand_attn(n, n, hq, hkv, D, dtype, 23)
    segs = []
    for r, L in enumerate(lengths):
        base = r * T
        segs.append((base, L, 0, 0, base, ops.SEG_BIDIRECTIONAL))
        if L < T:
            segs.append((base + L, T - L, base, L, base + L))
    plan = ops.AttnPlan(segs, n, n, hq, hkv, D, dtype, "cuda")
    out = ops.attend_packed(q, k, v, plan).float().cpu()
    mask = ref.bidirectional_mask(T, lengths)
    md = torch.float32 if dtype == torch.float32 else torch.bfloat16
    for r, L in enumerate(lengths):
        sl = slice(r * T, (r + 1) * T)
        qq, kk, vv = (x[sl].cpu().to(md).transpose(0, 1)[None] for x in (q, k, v))
        want = ref.attend(qq, kk, vv, mask[r].to(md))[0].transpose(0, 1).float()
        exact = ref.attend(*(x[sl].cpu().float().transpose(0, 1)[None] for x in (q, k, v)), mask[r])[0]
        exact = exact.transpose(0, 1)
        err = (out[sl][:L] - exact[:L]).abs().max().item()
        if dtype == torch.float32:
            assert err < F32_TOL, (r, err)
        else:
            ref_err = (want[:L] - exact[:L]).abs().max().item()
            assert err < BF16_TOL and err <= ref_err + 1e-4, (r, err, ref_err)


@pytest.mark.parametrize("dtype,tol", [(torch.bfloat16, 2e-2), (torch.float32, 1e-4)])
@pytest.mark.parametrize("B,T,with_state", [(1, 150, True), (3, 64, True), (2, 10, False)])
@pytest.mark.parametrize("ws_kind", ["full", "core"])
@pytest.mark.parametrize("dk", [64, 128])
def test_gdn_chunk_prefill_matches_oracle(dtype, tol, B, T, with_state, ws_kind, dk):
    """bf16 with a full workspace runs the tensor-core kernels; a workspace
    holding only the f32 core output runs the SIMT kernel (f32 always does).
    dk = dv = 128 is the cfg4 head shape."""
    from cev_b200 import ops
    nk, nv, dv = 2, 4, dk
    conv_out, ab, z, a_log, dt_bias, norm_w, s0 = gdn_inputs(B, T, nk, nv, dk, dv, dtype, 11)
    s_in = s0.cuda() if with_state else None
    s_out = torch.empty(B, nv, dk, dv, device="cuda")
    size = ops.gdn_workspace_size(B, T, nv, dk, dv) if ws_kind == "full" else B * T * nv * dv * 4
    ws = torch.empty(size, dtype=torch.uint8, device="cuda")
    y = ops.gdn_chunk_prefill(conv_out.reshape(B * T, -1).cuda(), ab.reshape(B * T, -1).cuda(), 2 * nv,
                              z.reshape(B * T, -1).cuda(), nv * dv, a_log.cuda(), dt_bias.cuda(), norm_w.cuda(), 1e-6,
                              s_in, s_out, B, T, nk, nv, dk, dv, ws)
    want_y, want_s = gdn_oracle(conv_out, ab, z, a_log, dt_bias, norm_w, s0 if with_state else None, nk, nv, dk, dv)
    # bf16: y is rounded once to bf16 at the end; the core runs in f32
    rel = dtype == torch.bfloat16
    assert close(y.reshape(B, T, -1), want_y, 1e-2 if rel else tol, rel)
    assert close(s_out, want_s, 1e-3 if rel else tol, rel)


@pytest.mark.parametrize("T,with_state", [(2700, True), (4000, False)])
def test_gdn_long_single_row_runs_in_pieces(T, with_state):
    """A single-row bf16 call of 43+ chunks (dk = dv = 128) runs its prep
    and scan in pieces on two streams, the state carried through s_out: the
    same output bit for bit as the one-launch path (taken when s_out is not
    asked for), and the oracle's within the chunked-prefill tolerance.
    T = 4000 ends in a partial chunk."""
    from cev_b200 import ops
    B, nk, nv, dk, dv = 1, 2, 4, 128, 128
    conv_out, ab, z, a_log, dt_bias, norm_w, s0 = gdn_inputs(B, T, nk, nv, dk, dv, torch.bfloat16, 12)
    s_in = s0.cuda() if with_state else None
    args = (conv_out.reshape(T, -1).cuda(), ab.reshape(T, -1).cuda(), 2 * nv, z.reshape(T, -1).cuda(), nv * dv,
            a_log.cuda(), dt_bias.cuda(), norm_w.cuda(), 1e-6, s_in)
    ws = torch.empty(ops.gdn_workspace_size(B, T, nv, dk, dv), dtype=torch.uint8, device="cuda")
    s_out = torch.full((B, nv, dk, dv), float("nan"), device="cuda")
    y = ops.gdn_chunk_prefill(*args, s_out, B, T, nk, nv, dk, dv, ws)
    y_one = ops.gdn_chunk_prefill(*args, None, B, T, nk, nv, dk, dv, ws)
    torch.cuda.synchronize()
    ops.device_status()
    assert torch.equal(y, y_one)
    want_y, want_s = gdn_oracle(conv_out, ab, z, a_log, dt_bias, norm_w, s0 if with_state else None, nk, nv, dk, dv)
    assert close(y.reshape(B, T, -1), want_y, 1e-2, True)
    assert close(s_out, want_s, 1e-3, True)


@pytest.mark.parametrize("dtype,tol", [(torch.bfloat16, 1e-2), (torch.float32, 1e-5)])
def test_gdn_conv_matches_oracle(dtype, tol):
    from cev_b200 import ops
    torch.manual_seed(4)
    B, T, C_, K = 2, 9, 64, 4
    mixed = torch.randn(B, T, C_ + 16).to(dtype)  # extra columns: a row stride
    w = torch.randn(C_, 1, K).to(dtype)
    tail = torch.randn(1, C_, K - 1).to(dtype)
    tail_out = torch.empty(B, C_, K - 1, dtype=dtype, device="cuda")
    y = ops.gdn_conv(mixed.reshape(B * T, -1).cuda(), B, T, C_, w.reshape(C_, K).cuda(), tail.cuda(), tail_out)
    full = torch.cat([tail.expand(B, C_, K - 1), mixed[..., :C_].transpose(1, 2)], 2)
    want = ref.silu(ref.depthwise_conv1d(full.float(), w.float())).transpose(1, 2)
    assert close(y.reshape(B, T, C_), want, tol, dtype == torch.bfloat16)
    assert torch.equal(tail_out.cpu(), full[:, :, T:T + K - 1].contiguous())


SPLIT_CASES = [
    # cfg5-shaped prefill chunk (one KV head of the 8-way split), a
    # bidirectional segment behind a prefix, ragged prefixes, a prefix-less
    # segment (never split) and head_dim 128 / 256
    (4, 1, 64, [(0, 512, 0, 3000, 3000)], 512, 3512),
    (32, 8, 64, [(0, 200, 0, 1111, 1111, 1), (200, 77, 0, 1111, 1311)], 277, 1388),
    (16, 8, 128, [(0, 64, 0, 2048, 2048), (64, 100, 0, 65, 2112), (164, 40, 0, 0, 2212)], 204, 2252),
    (16, 4, 256, [(0, 128, 0, 1000, 1000)], 128, 1128),
    (2, 1, 128, [(0, 37, 0, 100, 300), (37, 150, 0, 100, 337), (187, 5, 100, 0, 487)], 192, 492),
    (2, 2, 64, [(0, 256, 0, 1900, 2000), (256, 3, 0, 130, 2256)], 259, 2259),
]


@pytest.mark.parametrize("n_split", [None, 2, 3, 7, 32])
@pytest.mark.parametrize("case", range(len(SPLIT_CASES)))
def test_attention_split_kv_matches_oracle(case, n_split):
    """Split-KV (key ranges per tile merged by log-sum-exp) against the
    reference's attention: ranges of every length, more ranges than prefix
    blocks, bidirectional and prefix-less segments.  None = the planner's
    choice for 148 SMs."""
    from cev_b200 import ops
    hq, hkv, D, segs, n_tok, n_kv = SPLIT_CASES[case]
    q, k, v = rand_attn(n_tok, n_kv, hq, hkv, D, torch.bfloat16, 400 + case)
    plan = ops.AttnPlan(segs, n_tok, n_kv, hq, hkv, D, torch.bfloat16, "cuda", n_split=n_split)
    if n_split is not None:
        assert plan.n_split == n_split
    out = ops.attend_packed(q, k, v, plan)
    ops.device_status()
    mask_segs = [s[:5] for s in segs if not (len(s) > 5 and s[5])]
    check_bf16_attention(out, q, k, v, mask_segs, n_tok)
    for s in segs:
        if len(s) > 5 and s[5]:  # bidirectional: own rows in full
            qs, ql, po, pl, so = s[:5]
            kk = torch.cat([k[po:po + pl], k[so:so + ql]]).cpu().float().transpose(0, 1)[None]
            vv = torch.cat([v[po:po + pl], v[so:so + ql]]).cpu().float().transpose(0, 1)[None]
            want = ref.attend(q[qs:qs + ql].cpu().float().transpose(0, 1)[None], kk, vv, torch.zeros(ql, pl + ql))
            assert (out[qs:qs + ql].float().cpu() - want[0].transpose(0, 1)).abs().max().item() < BF16_TOL


@pytest.mark.parametrize("case", [2, 5])
def test_attention_split_kv_ignores_nonfinite_rows(case):
    """Split ranges load only visible K/V rows: NaN/Inf elsewhere in the
    arena leaves the output bits unchanged."""
    from cev_b200 import ops
    hq, hkv, D, segs, n_tok, n_kv = SPLIT_CASES[case]
    q, k, v = rand_attn(n_tok, n_kv, hq, hkv, D, torch.bfloat16, 450)
    used = torch.zeros(n_kv, dtype=torch.bool)
    for (qs, ql, po, pl, so) in segs:
        used[po:po + pl] = True
        used[so:so + ql] = True
    k2, v2 = k.clone(), v.clone()
    k2[~used.cuda()] = float("nan")
    v2[~used.cuda()] = float("inf")
    plan = ops.AttnPlan(segs, n_tok, n_kv, hq, hkv, D, torch.bfloat16, "cuda", n_split=5)
    a = ops.attend_packed(q, k, v, plan)
    b = ops.attend_packed(q, k2, v2, plan)
    ops.device_status()
    assert torch.equal(a, b)


def test_bounded_wait_gives_up_reports_and_leaves_the_context_usable():
    """Failure detection without a fault: a wait on a barrier nothing
    arrives on gives up after ~4M cycles, cevk_device_status reports
    CEVK_E_TIMEOUT with the record, the flag clears, and the next kernels
    run and match the oracle."""
    from cev_b200 import _lib, ops
    lib = _lib.lib()
    assert lib.cevk_device_status() == _lib.OK
    assert lib.cevk_selftest_wait_timeout(1 << 22, None) == _lib.OK
    assert lib.cevk_device_status() == _lib.E_TIMEOUT
    assert "bounded device wait gave up" in lib.cevk_last_error().decode()
    assert lib.cevk_device_status() == _lib.OK
    hq, hkv, D, segs, n_tok, n_kv = CASES[2]
    q, k, v = rand_attn(n_tok, n_kv, hq, hkv, D, torch.bfloat16, 500)
    plan = ops.AttnPlan(segs, n_tok, n_kv, hq, hkv, D, torch.bfloat16, "cuda")
    out = ops.attend_packed(q, k, v, plan)
    ops.device_status()
    check_bf16_attention(out, q, k, v, segs, n_tok)


def test_head_gather_wait_gives_up_when_a_peer_never_signals():
    """The fused head all-gather's bounded wait on one GPU: (1) with both
    ranks' flags raised (the two signals issued from this process, in
    stream order before the wait) the wait passes; (2) with a peer whose
    flag never reaches the epoch the wait gives up after ~2M cycles,
    cevk_device_status reports CEVK_E_TIMEOUT naming the head all-gather
    and the silent rank, the record clears, and the next attention call
    still matches the oracle.  Nothing waits on another process, so no
    kernel depends on a concurrent one."""
    import ctypes as C

    from cev_b200 import _lib, ops
    lib = _lib.lib()
    assert lib.cevk_device_status() == _lib.OK
    ptr = C.c_void_p()
    assert lib.cevk_ipc_alloc(256, C.byref(ptr)) == _lib.OK  # zeroed int32[64]
    try:
        flags = (C.c_void_p * 2)(ptr, ptr)  # both "ranks" publish into this one array
        st = C.c_void_p(torch.cuda.current_stream().cuda_stream)
        for r in (0, 1):
            assert lib.cevk_gather_signal(flags, 2, r, 1, st) == _lib.OK
        assert lib.cevk_gather_wait(ptr, 2, 1, 1 << 21, st) == _lib.OK
        assert lib.cevk_device_status() == _lib.OK
        # epoch 2: rank 0 signals, rank 1 never does
        assert lib.cevk_gather_signal(flags, 2, 0, 2, st) == _lib.OK
        assert lib.cevk_gather_wait(ptr, 2, 2, 1 << 21, st) == _lib.OK
        assert lib.cevk_device_status() == _lib.E_TIMEOUT
        msg = lib.cevk_last_error().decode()
        assert "head all-gather" in msg and "rank 1" in msg and "epoch 2" in msg, msg
        assert lib.cevk_device_status() == _lib.OK
    finally:
        assert lib.cevk_ipc_free(ptr) == _lib.OK
    hq, hkv, D, segs, n_tok, n_kv = CASES[2]
    q, k, v = rand_attn(n_tok, n_kv, hq, hkv, D, torch.bfloat16, 501)
    plan = ops.AttnPlan(segs, n_tok, n_kv, hq, hkv, D, torch.bfloat16, "cuda")
    out = ops.attend_packed(q, k, v, plan)
    ops.device_status()
    check_bf16_attention(out, q, k, v, segs, n_tok)
