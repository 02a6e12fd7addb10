"""Seeded synthetic workloads with the benchmark shapes.

``attention_batch`` builds the packed-prefill attention microbenchmark
(cfg2): ``n_req`` requests, each a cached prefix of ``prefix`` K/V rows plus
``n_suf`` question suffixes of ``suf_len`` tokens.  Q/K/V are drawn N(0, 1)
and RMS-normalised per head; Q and K are normalised and rotated with RoPE at
their positions (prefix rows at 0..P-1, every suffix restarting at P) by the
library's own norm+RoPE kernel, which also writes K/V into the arena.  Arena layout per
request: its prefix rows, then its suffixes' rows.
"""
from __future__ import annotations

import torch

from . import ops


def visible_pairs(prefix: int, suf_lens) -> int:
    """(query, key) pairs a suffix batch attends to: the whole prefix plus a
    causal triangle over itself."""
    return sum(n * prefix + n * (n + 1) // 2 for n in suf_lens)


def attention_flops(hq: int, head_dim: int, pairs: int) -> float:
    """Effective FLOPs: QK^T and PV, 2 flops per MAC, visible pairs only."""
    return 4.0 * head_dim * hq * pairs


class AttentionBatch:
    def __init__(self, n_req=32, prefix=2048, n_suf=16, suf_len=64, hq=16, hkv=8, head_dim=128, seed=0,
                 dtype=torch.bfloat16, device="cuda", theta=1e6):
        self.n_req, self.prefix, self.n_suf, self.suf_len = n_req, prefix, n_suf, suf_len
        self.hq, self.hkv, self.D = hq, hkv, head_dim
        D = head_dim
        per_req_q = n_suf * suf_len
        per_req_kv = prefix + per_req_q
        self.n_tokens = n_req * per_req_q
        self.n_kv = n_req * per_req_kv
        gen = torch.Generator(device=device)
        gen.manual_seed(seed)
        self.q = torch.empty(self.n_tokens, hq, D, dtype=dtype, device=device)
        self.k = torch.empty(self.n_kv, hkv, D, dtype=dtype, device=device)
        self.v = torch.empty(self.n_kv, hkv, D, dtype=dtype, device=device)
        ones_d = torch.ones(D, dtype=dtype, device=device)
        # Prefix rows of every request (positions 0..P-1): K/V only.
        if prefix > 0:
            raw = torch.randn(n_req * prefix, (hq + 2 * hkv) * D, generator=gen, device=device).to(dtype)
            pos = torch.arange(prefix, device=device, dtype=torch.int32).repeat(n_req)
            rows = (torch.arange(n_req, device=device, dtype=torch.int32)[:, None] * per_req_kv
                    + torch.arange(prefix, device=device, dtype=torch.int32)[None, :]).reshape(-1)
            scratch_q = torch.empty(n_req * prefix, hq, D, dtype=dtype, device=device)
            ops.qk_norm_rope(raw, (0, D), hq * D, (hq + hkv) * D, hq, hkv, D, ones_d, ones_d, 1e-6, False, pos, theta,
                             D, scratch_q, self.k, self.v, rows)
            del scratch_q, raw
        # Suffix rows: queries and their own K/V; positions restart at P.
        raw = torch.randn(self.n_tokens, (hq + 2 * hkv) * D, generator=gen, device=device).to(dtype)
        pos = (prefix + torch.arange(suf_len, device=device, dtype=torch.int32)).repeat(n_req * n_suf)
        r = torch.arange(n_req, device=device, dtype=torch.int32)[:, None] * per_req_kv + prefix
        rows = (r + torch.arange(per_req_q, device=device, dtype=torch.int32)[None, :]).reshape(-1)
        ops.qk_norm_rope(raw, (0, D), hq * D, (hq + hkv) * D, hq, hkv, D, ones_d, ones_d, 1e-6, False, pos, theta, D,
                         self.q, self.k, self.v, rows)
        del raw
        # V is RMS-normalised per head as well (Q and K were by the kernel)
        vf = self.v.float()
        self.v.copy_((vf * torch.rsqrt(vf.pow(2).mean(-1, keepdim=True) + 1e-6)).to(dtype))
        del vf
        self.segments = []
        for rq in range(n_req):
            for j in range(n_suf):
                self.segments.append((rq * per_req_q + j * suf_len, suf_len, rq * per_req_kv, prefix,
                                      rq * per_req_kv + prefix + j * suf_len))
        self.plan = ops.AttnPlan(self.segments, self.n_tokens, self.n_kv, hq, hkv, D, dtype, device)
        self.pairs = visible_pairs(prefix, [suf_len] * (n_req * n_suf))
        self.flops = attention_flops(hq, D, self.pairs)
        self.out = torch.empty_like(self.q)

    def run(self):
        return ops.attend_packed(self.q, self.k, self.v, self.plan, out=self.out)

    def algorithmic_bytes(self) -> int:
        """Bytes a perfect kernel moves per call: Q and O once, each
        request's K/V rows once."""
        e = self.q.element_size()
        return e * (2 * self.q.numel() + self.k.numel() + self.v.numel())


# ---------------------------------------------------------------------------
# Decision requests at the token-id level.
# ---------------------------------------------------------------------------
CODE_BASE = 100  # code j ("A", "B", ...) is token CODE_BASE + j in the synthetic vocabularies
SEP_ID = 13


def make_questions(gen: torch.Generator, n_q: int, lengths, n_opt: int, vocab: int):
    """``n_q`` questions whose rendered suffix has exactly the drawn length:
    head, ``n_opt`` x (code, separator, option ids), tail."""
    from .service import Question
    qs = []
    for i in range(n_q):
        total = int(lengths[i])
        body = total - 2 * n_opt
        opt_len = max(1, body // (2 * n_opt))
        head = max(1, (body - n_opt * opt_len) // 2)
        tail = body - n_opt * opt_len - head
        assert tail >= 1, (total, n_opt)

        def ids(n):
            return torch.randint(200, vocab, (n,), generator=gen).tolist()

        qs.append(Question(ids(head), [ids(opt_len) for _ in range(n_opt)], ids(tail)))
    return qs


def code_ids(n: int):
    return [CODE_BASE + j for j in range(n)]


def decision_request(seed: int, prefix_len: int, n_q: int, len_lo: int, len_hi: int, n_opt: int, vocab: int):
    """A seeded request: (prefix ids, questions).  Prefix ids are uniform in
    [0, vocab); question lengths uniform in [len_lo, len_hi]."""
    gen = torch.Generator().manual_seed(seed)
    prefix = torch.randint(0, vocab, (prefix_len,), generator=gen).tolist()
    lengths = torch.randint(len_lo, len_hi + 1, (n_q,), generator=gen).tolist()
    return prefix, make_questions(gen, n_q, lengths, n_opt, vocab)
