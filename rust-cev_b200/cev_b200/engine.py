"""Packed block-mask Qwen3 engine on the B200 kernels.

Mirrors ``Engine::run_many`` / ``plan`` / ``pass`` of
``crates/cev-model/src/engine.rs`` at the token-id level (tokenisation, the
prompt text and the code-vocabulary probe stay with the caller):

* a request's prefix is looked up in the prefix cache; otherwise every
  prefill chunk but the last runs now (engine.rs:249-256) and the last
  chunk (the "tail") rides in the first packed pass with the questions.
  The reference prefills each request's head on its own; here chunk c of
  every uncached head of one ``run_many`` call shares a pass (one segment
  per request, at most ``pass_tokens`` tokens), which gives the projection
  GEMMs several chunks' rows at once -- the requests are independent, so
  each one's K/V and readouts are what it computes alone;
* questions are packed greedily under ``pass_tokens`` (engine.rs:259-287);
* each pass computes its new tokens' K/V straight into arena rows -- tails
  into their prefix's range, question suffixes into scratch rows -- and
  describes who sees what with one segment per tail and per suffix instead
  of the host-built additive mask (engine.rs:389-442): a tail sees its own
  prefix head fully and itself causally; a suffix sees its whole prefix
  (head and tail) fully and itself causally.  Nothing is concatenated;
* the readout gathers each question's last token, applies the final norm
  and scores the code rows in f32 on the device (engine.rs:463-469).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch

from . import ops
from .arena import PrefixCache
from .qwen3 import PrefixKv, Qwen3


class InputError(ValueError):
    """A request-caused failure (``InputError``, backend.rs:10-12)."""


@dataclass
class Request:
    """A compiled request after tokenisation: the shared prefix ids, each
    question's suffix ids and its option count."""
    prefix: list
    suffixes: list
    n_options: list


@dataclass
class Readout:
    """(backend.rs:16-26) option logits in display order and the final hidden
    state at the answer position, both f32 (on the host, or on the device for
    an engine built with ``device_readout``)."""
    logits: torch.Tensor
    hidden: torch.Tensor


@dataclass
class Output:
    readouts: list
    input_tokens: int
    prefix_cached: bool


@dataclass
class _Plan:
    prefix: list
    suffixes: list
    n_options: list
    kv: PrefixKv
    cached: bool
    head: int                       # rows of kv already computed
    tail: range = field(default_factory=lambda: range(0))


class Engine:
    def __init__(self, model: Qwen3, code_ids, prefill_chunk=512, pass_tokens=2048, prefix_cache_tokens=65536,
                 device_readout=False):
        """``device_readout``: readouts stay on the device (for the on-device
        debias epilogue); otherwise they are host tensors like the
        reference's ``BackendOutput``."""
        self.model = model
        self.code_head = model.head_rows(code_ids).contiguous()
        self.prefill_chunk = prefill_chunk
        self.pass_tokens = pass_tokens
        self.cache = PrefixCache(prefix_cache_tokens)
        self.device_readout = device_readout

    # engine.rs:327-363 after tokenisation
    def _plan(self, req: Request) -> _Plan:
        m = self.model
        if len(req.prefix) == 0:
            # an internal error, not a request fault: engine.rs:344-346
            # bails (anyhow) rather than returning InputError
            raise RuntimeError("empty shared prefix")
        longest = max(len(req.prefix) + len(s) for s in req.suffixes)
        if longest >= m.max_len:
            raise InputError(f"prompt is {longest} tokens; the context limit is {m.max_len}")
        kv = self.cache.get(req.prefix)
        if kv is not None:
            kv.pins += 1
            p = _Plan(list(req.prefix), [list(s) for s in req.suffixes], list(req.n_options), kv, True, kv.len)
            p.tail = range(len(p.prefix), len(p.prefix))
            return p
        n = len(req.prefix)
        start = m.arena.alloc(n, self.cache)
        kv = PrefixKv(m.arena, start, 0, n, pins=1)
        return _Plan(list(req.prefix), [list(s) for s in req.suffixes], list(req.n_options), kv, False, 0,
                     range(n, n))

    def run(self, req: Request) -> Output:
        return self.run_many([req])[0]

    def run_many(self, reqs) -> list:
        """engine.rs:242-306."""
        plans = []
        try:
            for r in reqs:
                plans.append(self._plan(r))
            heads = []
            for p in plans:
                if not p.cached:
                    tail = min(len(p.prefix), max(self.prefill_chunk, 1))
                    head = len(p.prefix) - tail
                    if head > 0:
                        heads.append((p, p.prefix[:head]))
                    p.head = head
                    p.kv.len = head
                    p.tail = range(head, len(p.prefix))
            self._prefill_heads(heads)
            items = [(pi, qi) for pi, p in enumerate(plans) for qi in range(len(p.suffixes))]
            readouts = [[None] * len(p.suffixes) for p in plans]
            rest = items
            while rest:
                budget = self.pass_tokens
                for p in plans:
                    budget = max(budget - len(p.tail), 0)
                n = 0
                while n < len(rest):
                    pi, qi = rest[n]
                    ln = len(plans[pi].suffixes[qi])
                    if n > 0 and ln > budget:
                        break
                    budget = max(budget - ln, 0)
                    n += 1
                batch, rest = rest[:n], rest[n:]
                self._pass(plans, batch, readouts)
            # a bounded device wait that gave up fails the call instead of
            # serving its rows
            ops.device_status()
            return [Output(r, len(p.prefix) + sum(len(s) for s in p.suffixes), p.cached)
                    for p, r in zip(plans, readouts)]
        finally:
            for p in plans:
                p.kv.pins -= 1
            for p in plans:
                if self.cache.peek(p.prefix) is not p.kv and not p.kv.pins:
                    p.kv.release()

    def _prefill_heads(self, heads):
        """Causal chunked prefill of every (plan, head ids) in ``heads``
        (qwen3.rs:347-362 per request): chunk c of all heads in one pass of
        at most ``max(pass_tokens, prefill_chunk)`` tokens, one segment per
        head seeing its own earlier chunks fully and itself causally."""
        chunk = max(self.prefill_chunk, 1)
        cap = max(self.pass_tokens, chunk)
        n_chunks = max(((len(h) + chunk - 1) // chunk for _, h in heads), default=0)
        for c in range(n_chunks):
            tokens, pos, rows, segs = [], [], [], []
            for p, head in heads:
                part = head[c * chunk:(c + 1) * chunk]
                if not part:
                    continue
                if tokens and len(tokens) + len(part) > cap:
                    self.model.run_tokens(tokens, pos, rows, segs)
                    tokens, pos, rows, segs = [], [], [], []
                past, n, base = c * chunk, len(part), p.kv.start
                segs.append((len(tokens), n, base, past, base + past))
                tokens.extend(part)
                pos.extend(range(past, past + n))
                rows.extend(range(base + past, base + past + n))
            if tokens:
                self.model.run_tokens(tokens, pos, rows, segs)

    @staticmethod
    def pass_layout(plans, batch, scratch_start):
        """Tokens, positions, K/V destination rows, attention segments and
        readout rows of one packed pass (engine.rs:389-442 without the mask)."""
        tokens, pos, rows, segs, gather = [], [], [], [], []
        for p in plans:
            if len(p.tail) == 0:
                continue
            t0 = len(tokens)
            for j, t in enumerate(p.prefix[p.tail.start:p.tail.stop]):
                tokens.append(t)
                pos.append(p.tail.start + j)
                rows.append(p.kv.start + p.tail.start + j)
            segs.append((t0, len(p.tail), p.kv.start, p.head, p.kv.start + p.head))
        srow = scratch_start
        for pi, qi in batch:
            p = plans[pi]
            s = p.suffixes[qi]
            t0 = len(tokens)
            for j, t in enumerate(s):
                tokens.append(t)
                pos.append(len(p.prefix) + j)
                rows.append(srow + j)
            segs.append((t0, len(s), p.kv.start, len(p.prefix), srow))
            srow += len(s)
            gather.append(len(tokens) - 1)
        return tokens, pos, rows, segs, gather, srow - scratch_start

    def _pass(self, plans, batch, readouts):
        m = self.model
        n_scratch = sum(len(plans[pi].suffixes[qi]) for pi, qi in batch)
        scratch = m.arena.alloc(max(n_scratch, 1), self.cache)
        try:
            tokens, pos, rows, segs, gather, _ = self.pass_layout(plans, batch, scratch)
            x = m.run_tokens(tokens, pos, rows, segs)
            g = torch.tensor(gather, dtype=torch.int32).pin_memory().to(m.device, non_blocking=True)
            hid, logits = ops.readout(x, g, m.norm_w, m.eps, False, self.code_head)
            if not self.device_readout:
                hid, logits = hid.cpu(), logits.cpu()
        finally:
            m.arena.release(scratch, max(n_scratch, 1))
        for p in plans:
            if len(p.tail) == 0:
                continue
            p.kv.len = len(p.prefix)
            p.head = len(p.prefix)
            p.tail = range(len(p.prefix), len(p.prefix))
            if not p.cached:
                self.cache.put(p.prefix, p.kv)
        for (pi, qi), h, z in zip(batch, hid, logits):
            k = plans[pi].n_options[qi]
            readouts[pi][qi] = Readout(z[:k].clone(), h.clone())
