"""Debiased served probabilities at the token-id level.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).  Restates
``run_debiased`` (crates/cev-runtime/src/service.rs:288-348),
``Debias::shifts`` / ``CompiledQuestion::rotated``
(crates/cev-core/src/compile.rs:67-73,128-136) and ``math::{softmax,
log_softmax}`` (crates/cev-core/src/math.rs:7-18).

A question is held as token ids: a head, the options' own ids in canonical
order, and a tail; its prompt suffix shows option ``order[j]`` under code
``j`` (the layout of ``prompt/cev.rs:58-69`` with tokens instead of text).
"""
from __future__ import annotations

import math
import struct
from dataclasses import dataclass, field

from .engine import Request


@dataclass
class Question:
    head: list
    options: list
    tail: list
    order: list = field(default_factory=list)

    def __post_init__(self):
        if not self.order:
            self.order = list(range(len(self.options)))

    def rotated(self, shift: int) -> "Question":
        """Display position j shows canonical option ``order[(j+shift) % k]``
        (compile.rs:67-73)."""
        k = len(self.options)
        return Question(self.head, self.options, self.tail, [self.order[(j + shift) % k] for j in range(k)])

    def render(self, code_ids, sep_id) -> list:
        """Suffix ids: head, then per display position its code, a separator
        and the option shown there, then the tail (prompt/cev.rs:58-69)."""
        ids = list(self.head)
        for j, o in enumerate(self.order):
            ids += [code_ids[j], sep_id] + list(self.options[o])
        return ids + list(self.tail)


def shifts(mode: str, k: int, max_perm: int) -> list:
    """``Debias::shifts`` (compile.rs:128-136)."""
    if mode not in ("permute", "full") or k < 2:
        return [0]
    n = min(k, max(max_perm, 1))
    v = []
    for i in range(n):
        s = i * k // n
        if not v or v[-1] != s:
            v.append(s)
    return v


def calibrates(mode: str) -> bool:
    return mode in ("calibrate", "full")


def softmax(z) -> list:
    """f64 softmax over f32 logits (math.rs:7-12)."""
    z = [float(v) for v in z]
    m = max(z)
    e = [math.exp(v - m) for v in z]
    s = sum(e)
    return [v / s for v in e]


def log_softmax(z) -> list:
    """(math.rs:14-18)."""
    z = [float(v) for v in z]
    m = max(z)
    lse = m + math.log(sum(math.exp(v - m) for v in z))
    return [v - lse for v in z]


def run_debiased(backend, prefix, questions, mode, code_ids, sep_id, cf_prefix=None, max_permutations=4):
    """Served scores per question in canonical option order
    (service.rs:288-348); ``backend`` has ``run_many(list[Request])``.
    Returns (scores, probabilities) per question."""
    variants, spans = [], []
    for q in questions:
        start = len(variants)
        for s in shifts(mode, len(q.options), max_permutations):
            variants.append(q if s == 0 else q.rotated(s))
        spans.append(range(start, len(variants)))
    suffixes = [v.render(code_ids, sep_id) for v in variants]
    n_opts = [len(v.options) for v in variants]
    main = Request(list(prefix), suffixes, n_opts)
    cf = [None] * len(variants)
    if calibrates(mode):
        twin = Request(list(cf_prefix), suffixes, n_opts)
        out, twin_out = backend.run_many([main, twin])
        cf = [r.logits for r in twin_out.readouts]
    else:
        out = backend.run_many([main])[0]
    scores, probs = [], []
    for span in spans:
        k = len(variants[span.start].options)
        n = float(len(span))
        score = [0.0] * k
        for v in span:
            lp = log_softmax(out.readouts[v].logits.tolist())
            base = None if cf[v] is None else log_softmax(cf[v].tolist())
            for pos, opt in enumerate(variants[v].order):
                score[opt] += (lp[pos] - (0.0 if base is None else base[pos])) / n
        # The readout carries the scores as f32 (service.rs:344); the served
        # probabilities are their f64 softmax (service.rs:222, math.rs:7).
        score = [float(struct.unpack("f", struct.pack("f", s))[0]) for s in score]
        scores.append(score)
        probs.append(softmax(score))
    return scores, probs
