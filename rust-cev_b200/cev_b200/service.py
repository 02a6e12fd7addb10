"""Debiased served probabilities over an engine (``run_debiased``).

Mirrors ``crates/cev-runtime/src/service.rs:288-348`` with
``Debias::shifts`` / ``CompiledQuestion::rotated``
(``crates/cev-core/src/compile.rs:67-73,128-136``) and ``math::{softmax,
log_softmax}`` (``crates/cev-core/src/math.rs:7-18``) at the token-id level.
Every rotation variant and its content-free calibration twin go to the
engine in ONE ``run_many`` call, so they share packed passes; the answer
math is f64 on the host, like the reference.

A question is head ids, its options' ids in canonical order and tail ids;
its suffix shows option ``order[j]`` under code ``j`` (the layout of
``prompt/cev.rs:58-69``, tokens instead of text).
"""
from __future__ import annotations

import math
import struct
from dataclasses import dataclass, field

from .engine import Request

MODES = ("none", "calibrate", "permute", "full")


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
        """Display position j shows canonical option ``order[(j + shift) % k]``."""
        k = len(self.options)
        return Question(self.head, self.options, self.tail, [self.order[(j + shift) % k] for j in range(k)])

    def render(self, code_ids, sep_id) -> list:
        ids = list(self.head)
        for j, o in enumerate(self.order):
            ids += [code_ids[j], sep_id] + list(self.options[o])
        return ids + list(self.tail)


def shifts(mode: str, k: int, max_perm: int) -> list:
    """Rotation shifts for k options, at most ``max_perm``, evenly spread."""
    if mode not in ("permute", "full") or k < 2:
        return [0]
    n = min(k, max(max_perm, 1))
    out = []
    for i in range(n):
        s = i * k // n
        if not out or out[-1] != s:
            out.append(s)
    return out


def _f32(x: float) -> float:
    return struct.unpack("f", struct.pack("f", x))[0]


def softmax(z) -> list:
    z = [float(v) for v in z]
    m = max(z)
    e = [math.exp(v - m) for v in z]
    s = sum(e)
    return [v / s for v in e]


def log_softmax(z) -> list:
    z = [float(v) for v in z]
    m = max(z)
    lse = m + math.log(sum(math.exp(v - m) for v in z))
    return [v - lse for v in z]


def run_debiased(engine, prefix, questions, mode, code_ids, sep_id, cf_prefix=None, max_permutations=4,
                 on_device=False):
    """Served (scores, probabilities) per question in canonical option order.
    ``on_device``: the answer math runs on the GPU (``cevk_debias``) over the
    readouts left on the device, and only the k probabilities and scores per
    question come back to the host."""
    if mode not in MODES:
        raise ValueError(f"unknown debias mode `{mode}`")
    if on_device:
        saved = engine.device_readout
        engine.device_readout = True
        try:
            return _run_debiased_device(engine, prefix, questions, mode, code_ids, sep_id, cf_prefix,
                                        max_permutations)
        finally:
            engine.device_readout = saved
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
    if mode in ("calibrate", "full"):
        out, twin = engine.run_many([main, Request(list(cf_prefix), suffixes, n_opts)])
        cf = [r.logits for r in twin.readouts]
    else:
        out = engine.run_many([main])[0]
    return _answers(variants, spans, out, cf)


def run_debiased_many(engine, items, mode, code_ids, sep_id, cf_prefix=None, max_permutations=4):
    """``run_debiased`` over several independent requests ``items`` =
    [(prefix, questions), ...] in one ``Engine.run_many`` call: their
    prefill heads share passes chunk by chunk and their questions share
    packed passes.  Returns one (scores, probabilities) per item, each what
    ``run_debiased`` returns for that item alone."""
    if mode not in MODES:
        raise ValueError(f"unknown debias mode `{mode}`")
    calib = mode in ("calibrate", "full")
    per_item, reqs = [], []
    for prefix, questions in items:
        variants, spans = [], []
        for q in questions:
            start = len(variants)
            for s in shifts(mode, len(q.options), max_permutations):
                variants.append(q if s == 0 else q.rotated(s))
            spans.append(range(start, len(variants)))
        suffixes = [v.render(code_ids, sep_id) for v in variants]
        n_opts = [len(v.options) for v in variants]
        per_item.append((variants, spans))
        reqs.append(Request(list(prefix), suffixes, n_opts))
        if calib:
            reqs.append(Request(list(cf_prefix), suffixes, n_opts))
    outs = engine.run_many(reqs)
    results = []
    for i, (variants, spans) in enumerate(per_item):
        out = outs[2 * i] if calib else outs[i]
        cf = [r.logits for r in outs[2 * i + 1].readouts] if calib else [None] * len(variants)
        results.append(_answers(variants, spans, out, cf))
    return results


def _answers(variants, spans, out, cf):
    """service.rs:330-346: per question the mean over its variants of
    log_softmax(z) (minus the calibration log_softmax) at each display
    position, accumulated at the option shown there; f32 score, softmax."""
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
        score = [_f32(s) for s in score]
        scores.append(score)
        probs.append(softmax(score))
    return scores, probs


def _run_debiased_device(engine, prefix, questions, mode, code_ids, sep_id, cf_prefix, max_permutations):
    import torch

    from . import ops
    variants, span = [], [0]
    for q in questions:
        for s in shifts(mode, len(q.options), max_permutations):
            variants.append(q if s == 0 else q.rotated(s))
        span.append(len(variants))
    suffixes = [v.render(code_ids, sep_id) for v in variants]
    n_opts = [len(v.options) for v in variants]
    main = Request(list(prefix), suffixes, n_opts)
    if mode in ("calibrate", "full"):
        out, twin = engine.run_many([main, Request(list(cf_prefix), suffixes, n_opts)])
    else:
        out, twin = engine.run_many([main])[0], None
    ld = max(n_opts)

    def rows(readouts):
        z = [r.logits for r in readouts]
        if any(t.shape[0] != ld for t in z):
            z = [torch.nn.functional.pad(t, (0, ld - t.shape[0])) for t in z]
        return torch.stack(z).float().contiguous()

    dev = out.readouts[0].logits.device
    order = torch.tensor([list(v.order) + [0] * (ld - len(v.order)) for v in variants], dtype=torch.int32)
    k_q = torch.tensor([len(q.options) for q in questions], dtype=torch.int32)
    scores, probs = ops.debias(rows(out.readouts), None if twin is None else rows(twin.readouts),
                               torch.tensor(span, dtype=torch.int32).to(dev), k_q.to(dev), order.to(dev))
    scores, probs = scores.cpu(), probs.cpu()
    ks = k_q.tolist()
    return ([scores[i, :k].tolist() for i, k in enumerate(ks)], [probs[i, :k].tolist() for i, k in enumerate(ks)])
