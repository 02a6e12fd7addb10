"""Device KV arena and the prefix cache over it.

The reference keeps each cached prefix as per-layer K/V tensors and builds
every pass's past by ``Tensor::cat`` (engine.rs:375-387, 447-462); the
attention then reads the concatenation.  Here all K/V rows of a model live
in one preallocated arena per layer, ``[capacity, kv_heads, head_dim]``; a
prefix owns a contiguous row range (head and tail written in place, so the
whole prefix is one range), question suffixes borrow scratch rows for one
pass, and attention reads prefixes in place through segment descriptors.
Nothing is copied when a pass mixes several prefixes (a request and its
calibration twin).  The cache is the reference's LRU bounded by cached
tokens (engine.rs:474-503, hybrid.rs:744-772); evicting an entry frees its
rows.
"""
from __future__ import annotations

import torch


class RowAllocator:
    """First-fit allocator of contiguous row ranges."""

    def __init__(self, capacity: int):
        self.capacity = capacity
        self.free = [(0, capacity)]  # sorted (start, length)

    def alloc(self, n: int) -> int | None:
        for i, (s, l) in enumerate(self.free):
            if l >= n:
                if l == n:
                    self.free.pop(i)
                else:
                    self.free[i] = (s + n, l - n)
                return s
        return None

    def release(self, start: int, n: int) -> None:
        if n <= 0:
            return
        self.free.append((start, n))
        self.free.sort()
        merged = []
        for s, l in self.free:
            if merged and merged[-1][0] + merged[-1][1] == s:
                merged[-1] = (merged[-1][0], merged[-1][1] + l)
            else:
                merged.append((s, l))
        self.free = merged

    def used(self) -> int:
        return self.capacity - sum(l for _, l in self.free)


class KvArena:
    """Per-layer K and V row storage for the attention layers of a model."""

    def __init__(self, n_layers: int, capacity: int, kv_heads: int, head_dim: int, dtype, device):
        self.k = [torch.zeros(capacity, kv_heads, head_dim, dtype=dtype, device=device) for _ in range(n_layers)]
        self.v = [torch.zeros(capacity, kv_heads, head_dim, dtype=dtype, device=device) for _ in range(n_layers)]
        self.rows = RowAllocator(capacity)
        self.capacity = capacity

    def alloc(self, n: int, cache=None) -> int:
        """Rows for ``n`` tokens; evicts least-recently-used cache entries
        when the arena is full."""
        while True:
            s = self.rows.alloc(n)
            if s is not None:
                return s
            if cache is None or not cache.evict_one():
                raise MemoryError(f"KV arena full: {n} rows wanted, {self.capacity - self.rows.used()} free")

    def release(self, start: int, n: int) -> None:
        self.rows.release(start, n)


class PrefixCache:
    """LRU of computed prefixes keyed by token ids (and a media hash),
    bounded by total cached tokens.  Entries are state objects with a
    ``release()`` method that gives their arena rows back and a ``pins``
    count: a state a running request still reads is never evicted."""

    def __init__(self, budget: int):
        self.budget = budget
        self.entries = []  # [(key, state)], oldest first

    def get(self, key):
        key = tuple(key)
        for i, (k, st) in enumerate(self.entries):
            if k == key:
                self.entries.append(self.entries.pop(i))
                return st
        return None

    def peek(self, key):
        """Lookup without touching the LRU order."""
        key = tuple(key)
        for k, st in self.entries:
            if k == key:
                return st
        return None

    def put(self, key, state) -> bool:
        """Insert (or refresh) ``key``; returns False when the key alone is
        over budget (the state is then not cached; engine.rs:493-496)."""
        key = tuple(key)
        if len(key) > self.budget:
            return False
        for i, (k, st) in enumerate(self.entries):
            if k == key:
                self.entries.pop(i)
                if st is not state and not st.pins:
                    st.release()
                break
        self.entries.append((key, state))
        while sum(len(k) for k, _ in self.entries) > self.budget and self.evict_one():
            pass
        return True

    def evict_one(self) -> bool:
        """Drop the least recently used entry nobody is reading."""
        for i, (_, st) in enumerate(self.entries):
            if not st.pins:
                self.entries.pop(i)
                st.release()
                return True
        return False

    def clear(self) -> None:
        while self.evict_one():
            pass
