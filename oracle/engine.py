"""Packed block-mask Qwen3 engine at the token-id level.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).  Restates
``Engine::run_many`` / ``pass`` / ``PrefixCache`` of
``crates/cev-model/src/engine.rs`` after tokenisation: a request is already
split into ``prefix`` ids and per-question ``suffixes`` ids (``plan``,
engine.rs:327-363, minus the tokenizer).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch

from .qwen3 import LayerKv, PrefixKv, Qwen3


@dataclass
class Request:
    """A compiled request after tokenisation."""
    prefix: list
    suffixes: list
    n_options: list


@dataclass
class Readout:
    """(backend.rs:16-26) logits of the question's options in display order
    and the final hidden state at the answer position."""
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
    cached: PrefixKv | None
    past: PrefixKv | None
    tail: range = field(default_factory=lambda: range(0))


class PrefixCache:
    """LRU of prefilled prefixes bounded by cached tokens (engine.rs:474-503)."""

    def __init__(self, budget: int):
        self.budget = budget
        self.entries = []

    def get(self, key):
        key = tuple(key)
        for i, (k, kv) in enumerate(self.entries):
            if k == key:
                self.entries.append(self.entries.pop(i))
                return kv
        return None

    def put(self, key, kv):
        key = tuple(key)
        if len(key) > self.budget:
            return
        self.entries = [(k, v) for k, v in self.entries if k != key]
        self.entries.append((key, kv))
        while sum(len(k) for k, _ in self.entries) > self.budget:
            self.entries.pop(0)


class Engine:
    """(engine.rs:53-64, 222-471)."""

    def __init__(self, model: Qwen3, code_ids, prefill_chunk=512, pass_tokens=2048, prefix_cache_tokens=65536):
        self.model = model
        self.code_head = model.head_rows(code_ids).float()
        self.prefill_chunk = prefill_chunk
        self.pass_tokens = pass_tokens
        self.cache = PrefixCache(prefix_cache_tokens)

    def _plan(self, req: Request) -> _Plan:
        """engine.rs:327-363 after tokenisation."""
        if len(req.prefix) == 0:
            raise ValueError("empty shared prefix")
        longest = max(len(req.prefix) + len(s) for s in req.suffixes)
        if longest >= self.model.max_len:
            raise ValueError(f"prompt is {longest} tokens; the context limit is {self.model.max_len}")
        cached = self.cache.get(req.prefix)
        p = _Plan(list(req.prefix), [list(s) for s in req.suffixes], list(req.n_options), cached, cached)
        p.tail = range(len(p.prefix), len(p.prefix))
        return p

    def run(self, req: Request) -> Output:
        return self.run_many([req])[0]

    def run_many(self, reqs):
        """engine.rs:242-306."""
        plans = [self._plan(r) for r in reqs]
        for p in plans:
            if p.cached is None:
                tail = min(len(p.prefix), max(self.prefill_chunk, 1))
                head = len(p.prefix) - tail
                if head > 0:
                    p.past = self.model.prefill(p.prefix[:head], self.prefill_chunk)
                p.tail = range(head, len(p.prefix))
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
        return [Output(r, len(p.prefix) + sum(len(s) for s in p.suffixes), p.cached is not None)
                for p, r in zip(plans, readouts)]

    @staticmethod
    def build_pass(plans, batch):
        """Tokens, positions, owner/segment tags, the additive mask, gather
        rows and keep ranges of one packed pass (engine.rs:367-442)."""
        past_off, past_len = [], 0
        for p in plans:
            past_off.append(past_len)
            past_len += 0 if p.past is None else p.past.len
        tokens, pos, owner, seg, keep = [], [], [], [], []
        tail_at = [None] * len(plans)
        for pi, p in enumerate(plans):
            if len(p.tail) == 0:
                continue
            tail_at[pi] = (len(tokens), len(p.tail))
            keep.append((len(tokens), len(p.tail)))
            for j, t in enumerate(p.prefix[p.tail.start:p.tail.stop]):
                tokens.append(t)
                pos.append(p.tail.start + j)
                owner.append(pi)
                seg.append(0)
        gather = []
        for kk, (pi, qi) in enumerate(batch):
            p = plans[pi]
            for j, t in enumerate(p.suffixes[qi]):
                tokens.append(t)
                pos.append(len(p.prefix) + j)
                owner.append(pi)
                seg.append(kk + 1)
            gather.append(len(tokens) - 1)
        n = len(tokens)
        width = past_len + n
        mask = torch.full((n, width), float("-inf"))
        for i in range(n):
            pi = owner[i]
            plen = 0 if plans[pi].past is None else plans[pi].past.len
            mask[i, past_off[pi]:past_off[pi] + plen] = 0.0
            if tail_at[pi] is not None:
                start, ln = tail_at[pi]
                end = i + 1 if seg[i] == 0 else start + ln
                mask[i, past_len + start:past_len + end] = 0.0
            if seg[i] != 0:
                j = i
                while True:
                    mask[i, past_len + j] = 0.0
                    if j == 0 or seg[j - 1] != seg[i]:
                        break
                    j -= 1
        return dict(tokens=tokens, pos=pos, owner=owner, seg=seg, mask=mask, gather=gather, keep=keep,
                    past_off=past_off, past_len=past_len, tail_at=tail_at)

    def _pass(self, plans, batch, readouts):
        """engine.rs:366-471."""
        pasts = [p.past for p in plans if p.past is not None]
        if not pasts:
            past_layers = None
        elif len(pasts) == 1:
            past_layers = pasts[0].layers
        else:
            past_layers = [LayerKv(torch.cat([p.layers[l].k for p in pasts], 2), torch.cat([p.layers[l].v for p in pasts], 2))
                           for l in range(len(pasts[0].layers))]
        b = self.build_pass(plans, batch)
        hidden, kept = self.model.forward_packed(past_layers, b["tokens"], b["pos"], b["mask"], b["gather"], b["keep"])
        kept = iter(kept)
        for p in plans:
            if len(p.tail) == 0:
                continue
            tail_kv = next(kept)
            if p.past is not None:
                layers = [LayerKv(torch.cat([h.k, t.k], 2), torch.cat([h.v, t.v], 2)) for h, t in zip(p.past.layers, tail_kv)]
            else:
                layers = tail_kv
            kv = PrefixKv(layers, len(p.prefix))
            self.cache.put(p.prefix, kv)
            p.past = kv
            p.tail = range(len(p.prefix), len(p.prefix))
        logits = hidden @ self.code_head.t()
        for (pi, qi), h, z in zip(batch, hidden, logits):
            k = plans[pi].n_options[qi]
            readouts[pi][qi] = Readout(z[:k].clone(), h.clone())
