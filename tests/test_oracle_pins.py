"""The CPU oracle against the reference's own known-answer tests.

These restate, with the same deterministic inputs and tolerances, the unit
tests the reference ships for this path, so the oracle's arithmetic is pinned
to the reference's before it is used to check the GPU library.
"""
import math

import torch

from oracle import ops
from oracle.engine import Output, Readout
from oracle.service import Question, run_debiased, shifts, softmax


def _det(n, seed):
    """The reference's deterministic fill: ((i+1)(seed+7919) mod 1000)/500 - 1
    (qwen35.rs:781)."""
    return torch.tensor([(((i + 1) * (seed + 7919)) % 1000) / 500.0 - 1.0 for i in range(n)], dtype=torch.float32)


def test_unit_lower_inverse_matches_definition():
    """qwen35.rs:758-774."""
    n = 8
    vals = torch.tensor([((i * 37 % 11) - 5.0) / 7.0 for i in range(n * n)], dtype=torch.float32).reshape(1, 1, n, n)
    strict = vals * (torch.tril(torch.ones(n, n)) - torch.eye(n))
    a = strict + torch.eye(n)
    inv = ops.inv_unit_lower(vals)
    ident = torch.matmul(a, inv).reshape(n, n)
    assert (ident - torch.eye(n)).abs().max().item() < 1e-4


def test_chunked_rule_matches_recurrence():
    """qwen35.rs:776-822: B=1, H=2, T=70, dk=4, dv=3, tolerance 2e-4."""
    b, h, t, dk, dv = 1, 2, 70, 4, 3
    q = _det(b * h * t * dk, 1).reshape(b, h, t, dk)
    k = _det(b * h * t * dk, 2).reshape(b, h, t, dk)
    v = _det(b * h * t * dv, 3).reshape(b, h, t, dv)
    g = _det(b * h * t, 4).reshape(b, h, t).abs() * -0.5
    beta = torch.sigmoid(_det(b * h * t, 5).reshape(b, h, t))
    out, s = ops.chunk_gated_delta_rule(q, k, v, g, beta)
    ref_out, ref_s = ops.gated_delta_recurrence(q, k, v, g, beta)
    assert (out - ref_out).abs().max().item() < 2e-4
    assert (s - ref_s).abs().max().item() < 2e-4


def test_chunked_rule_continues_from_state():
    """Two chunked calls through the state equal one call (the prefix-state
    contract of decoder.rs:54-61)."""
    torch.manual_seed(0)
    b, h, t, dk, dv = 2, 3, 150, 8, 5
    q, k = torch.randn(b, h, t, dk), torch.randn(b, h, t, dk)
    v = torch.randn(b, h, t, dv)
    g = -torch.rand(b, h, t)
    beta = torch.rand(b, h, t)
    full, s_full = ops.chunk_gated_delta_rule(q, k, v, g, beta)
    o1, s1 = ops.chunk_gated_delta_rule(q[:, :, :70], k[:, :, :70], v[:, :, :70], g[:, :, :70], beta[:, :, :70])
    o2, s2 = ops.chunk_gated_delta_rule(q[:, :, 70:], k[:, :, 70:], v[:, :, 70:], g[:, :, 70:], beta[:, :, 70:], s1)
    assert (torch.cat([o1, o2], 2) - full).abs().max().item() < 1e-4
    assert (s2 - s_full).abs().max().item() < 1e-4


def test_rotation_and_shifts():
    """compile.rs:462-476."""
    q = Question([1], [[10], [11], [12]], [2])
    r = q.rotated(1)
    assert r.order == [1, 2, 0]
    assert r.rotated(2).order == [0, 1, 2]
    assert shifts("full", 3, 4) == [0, 1, 2]
    assert shifts("full", 10, 4) == [0, 2, 5, 7]
    assert shifts("calibrate", 10, 4) == [0]
    assert shifts("permute", 1, 4) == [0]


class _PositionInvariant:
    """A backend whose option logit depends only on the option's own ids,
    not on where it is shown: the stand-in ``MockBackend`` plays in
    runtime.rs:184-207.  Suffixes are rendered as head, (code, sep, option)
    per display position, tail."""

    def __init__(self, head_len, tail_len, opt_len):
        self.hl, self.tl, self.ol = head_len, tail_len, opt_len

    def run_many(self, reqs):
        outs = []
        for r in reqs:
            rd = []
            for s, k in zip(r.suffixes, r.n_options):
                body = s[self.hl:len(s) - self.tl]
                z = [float(sum(body[j * (self.ol + 2) + 2:(j + 1) * (self.ol + 2)]) % 97) / 10.0 for j in range(k)]
                rd.append(Readout(torch.tensor(z), torch.zeros(4)))
            outs.append(Output(rd, 0, False))
        return outs


def test_debias_rotations_map_back_to_canonical_options():
    """runtime.rs:184-207: with a position-invariant backend, averaging
    rotations reproduces the undebiased distribution within 1e-5."""
    opts = [[3, 4], [50, 60], [7, 8], [1, 2], [90, 91]]
    q = Question([100, 101], opts, [200])
    be = _PositionInvariant(2, 1, 2)
    codes, sep = [500, 501, 502, 503, 504], 9
    _, plain = run_debiased(be, [1, 2, 3], [q], "none", codes, sep)
    _, perm = run_debiased(be, [1, 2, 3], [q], "permute", codes, sep)
    assert max(abs(a - b) for a, b in zip(plain[0], perm[0])) < 1e-5
    assert plain[0][4] > plain[0][0]


def test_math_softmax():
    """math.rs:7-18 in f64 over f32 logits."""
    p = softmax([1.0, 2.0, 3.0])
    e = [math.exp(v - 3.0) for v in (1.0, 2.0, 3.0)]
    assert all(abs(a - b / sum(e)) < 1e-15 for a, b in zip(p, e))


def test_bidirectional_mask_restates_the_reference():
    """qwen35.rs:483-498: real tokens see all real tokens; pad columns are
    hidden; a pad query keeps its diagonal."""
    from oracle import ops
    m = ops.bidirectional_mask(4, [2, 0])
    inf = float("-inf")
    assert m[0].tolist() == [[0, 0, inf, inf], [0, 0, inf, inf], [0, 0, 0, inf], [0, 0, inf, 0]]
    assert m[1].tolist() == [[0, inf, inf, inf], [inf, 0, inf, inf], [inf, inf, 0, inf], [inf, inf, inf, 0]]


def test_attend_head_by_head_equals_all_heads_at_once():
    """The oracle's memory-bounded attention (one query head at a time, for
    the long states of the benchmark configs) computes what the all-heads
    form does (qwen3.rs:206-220), for a 2-D causal mask and a per-row 4-D
    one."""
    g = torch.Generator().manual_seed(3)
    b, hq, hkv, t, past, d = 2, 4, 2, 300, 120000, 16
    q = torch.randn(b, hq, t, d, generator=g)
    k = torch.randn(b, hkv, past + t, d, generator=g)
    v = torch.randn(b, hkv, past + t, d, generator=g)
    assert b * hq * t * (past + t) > (1 << 27)  # takes the head-by-head path
    for mask in (ops.causal_mask(t, past), ops.causal_mask(t, past)[None, None].expand(b, 1, t, past + t)):
        got = ops.attend(q, k, v, mask)
        kk, vv = ops.repeat_kv(k, 2), ops.repeat_kv(v, 2)
        sc = torch.matmul(q, kk.transpose(-1, -2)) * d ** -0.5 + mask
        want = torch.matmul(torch.softmax(sc, -1), vv)
        assert (got - want).abs().max().item() < 1e-5
