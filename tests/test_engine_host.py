"""Host-side scheduling of the packed engine without a GPU: the joint
chunked prefill of several requests' prefix heads (one pass per chunk
index, at most pass_tokens tokens, one segment per head seeing its own
earlier chunks fully and itself causally) and the packed-pass layout."""
from types import SimpleNamespace

from cev_b200.engine import Engine


class _Recorder:
    def __init__(self):
        self.calls = []

    def run_tokens(self, tokens, pos, rows, segs):
        self.calls.append((list(tokens), list(pos), list(rows), [tuple(s) for s in segs]))


def _engine(chunk, pass_tokens):
    eng = Engine.__new__(Engine)  # host logic only: no model weights
    eng.model = _Recorder()
    eng.prefill_chunk = chunk
    eng.pass_tokens = pass_tokens
    return eng


def _plan(start):
    return SimpleNamespace(kv=SimpleNamespace(start=start))


def test_joint_prefill_packs_chunk_c_of_every_head():
    eng = _engine(4, 16)
    a, b = _plan(100), _plan(300)
    eng._prefill_heads([(a, list(range(10))), (b, list(range(50, 56)))])
    calls = eng.model.calls
    assert len(calls) == 3  # chunk indices 0, 1, 2 (head a has 3 chunks, b has 2)
    toks, pos, rows, segs = calls[0]
    assert toks == [0, 1, 2, 3, 50, 51, 52, 53]
    assert pos == [0, 1, 2, 3, 0, 1, 2, 3]
    assert rows == [100, 101, 102, 103, 300, 301, 302, 303]
    assert segs == [(0, 4, 100, 0, 100), (4, 4, 300, 0, 300)]
    toks, pos, rows, segs = calls[1]
    assert toks == [4, 5, 6, 7, 54, 55] and pos == [4, 5, 6, 7, 4, 5]
    assert segs == [(0, 4, 100, 4, 104), (4, 2, 300, 4, 304)]  # each sees its own 4 earlier rows
    assert calls[2] == ([8, 9], [8, 9], [108, 109], [(0, 2, 100, 8, 108)])


def test_joint_prefill_splits_a_chunk_index_at_pass_tokens():
    eng = _engine(4, 6)  # room for one 4-token part per pass (cap = max(6, 4))
    heads = [(_plan(0), list(range(8))), (_plan(50), list(range(8))), (_plan(90), list(range(3)))]
    eng._prefill_heads(heads)
    sizes = [len(c[0]) for c in eng.model.calls]
    assert sizes == [4, 4, 3, 4, 4]  # chunk 0: 4 | 4 | 3 (4 + 3 > 6); chunk 1: 4 | 4
    # every token of every head is prefilled exactly once, at its position
    seen = {}
    for toks, pos, rows, segs in eng.model.calls:
        for q0, n, po, pl, so in segs:
            assert pl == pos[q0] and so == po + pl  # own rows follow the head's earlier rows
            for i in range(n):
                seen[(po, pos[q0 + i])] = rows[q0 + i]
    assert len(seen) == 8 + 8 + 3
    assert all(row == start + p for (start, p), row in seen.items())


def test_joint_prefill_of_nothing_runs_nothing():
    eng = _engine(512, 2048)
    eng._prefill_heads([])
    assert eng.model.calls == []


def test_pass_layout_tails_then_suffixes():
    """engine.rs:389-442 without the mask: pending tails first (absolute
    positions, written into their prefix rows, seeing the head fully), then
    each suffix (positions from the prefix end, scratch rows, seeing the
    whole prefix), with one readout row per suffix at its last token."""
    a = SimpleNamespace(prefix=[1, 2, 3, 4, 5], head=3, tail=range(3, 5), kv=SimpleNamespace(start=40),
                        suffixes=[[7, 8], [9]])
    b = SimpleNamespace(prefix=[6, 6], head=2, tail=range(2, 2), kv=SimpleNamespace(start=10),
                        suffixes=[[5, 5, 5]])
    tokens, pos, rows, segs, gather, n_scratch = Engine.pass_layout([a, b], [(0, 1), (1, 0), (0, 0)], 1000)
    assert tokens == [4, 5, 9, 5, 5, 5, 7, 8]
    assert pos == [3, 4, 5, 2, 3, 4, 5, 6]
    assert rows == [43, 44, 1000, 1001, 1002, 1003, 1004, 1005]
    assert segs == [(0, 2, 40, 3, 43), (2, 1, 40, 5, 1000), (3, 3, 10, 2, 1001), (6, 2, 40, 5, 1004)]
    assert gather == [2, 5, 7] and n_scratch == 6


# ---- planning, the prefix cache and the arena rows (engine.rs:327-363, 474-503) ----
import pytest  # noqa: E402
import torch  # noqa: E402

from cev_b200.arena import KvArena, PrefixCache, RowAllocator  # noqa: E402
from cev_b200.engine import InputError, Request  # noqa: E402
from cev_b200.qwen3 import PrefixKv  # noqa: E402


def _planning_engine(max_len=128, rows=1024, budget=65536):
    eng = Engine.__new__(Engine)
    eng.model = SimpleNamespace(max_len=max_len, arena=KvArena(1, rows, 1, 8, torch.float32, "cpu"))
    eng.cache = PrefixCache(budget)
    eng.prefill_chunk, eng.pass_tokens = 16, 64
    return eng


def test_plan_rejects_a_prompt_at_the_context_limit():
    """engine.rs:350-352 on the joint token ids: the longest full prompt
    must stay below max_len (the check_fits slack of engine.rs:513-524 is a
    pre-tokenisation shortcut; token ids here are exact)."""
    eng = _planning_engine(max_len=128)
    p = eng._plan(Request([1] * 100, [[2] * 20, [3] * 27], [1, 1]))
    assert not p.cached and p.kv.capacity == 100
    with pytest.raises(InputError, match="context limit is 128"):
        eng._plan(Request([1] * 100, [[2] * 20, [3] * 28], [1, 1]))
    with pytest.raises(InputError, match="context limit"):
        eng._plan(Request([1] * 128, [[2]], [1]))
    # engine.rs:344-346 bails: an internal error, not a request fault
    with pytest.raises(RuntimeError, match="empty shared prefix") as e:
        eng._plan(Request([], [[2]], [1]))
    assert not isinstance(e.value, InputError)


def test_hybrid_engine_rejects_an_empty_prefix_as_an_internal_error():
    """hybrid.rs:480-484: a Codes request whose questions share no leading
    token bails before any forward (not InputError); a prompt at the context
    limit is an InputError (hybrid.rs:485-488)."""
    from cev_b200.hybrid import HybridEngine
    eng = HybridEngine.__new__(HybridEngine)
    eng.decoder = SimpleNamespace(max_len=64)
    with pytest.raises(RuntimeError, match="empty shared prefix") as e:
        eng.run(Request([], [[1, 2]], [1]))
    assert not isinstance(e.value, InputError)
    with pytest.raises(InputError, match="context limit is 64"):
        eng.run(Request([1] * 60, [[2] * 4], [1]))


def test_plan_reuses_and_pins_a_cached_prefix():
    eng = _planning_engine()
    arena = eng.model.arena
    kv = PrefixKv(arena, arena.alloc(40), 40, 40)
    assert eng.cache.put([5] * 40, kv)
    p = eng._plan(Request([5] * 40, [[1, 2]], [1]))
    assert p.cached and p.kv is kv and kv.pins == 1 and p.head == 40 and len(p.tail) == 0
    q = eng._plan(Request([6] * 40, [[1, 2]], [1]))
    assert not q.cached and q.kv.start != kv.start  # a new range; the cached rows stay


def test_prefix_cache_evicts_least_recent_unpinned_and_frees_rows():
    arena = KvArena(1, 300, 1, 4, torch.float32, "cpu")
    cache = PrefixCache(budget=250)
    states = []
    for i in range(3):
        st = PrefixKv(arena, arena.alloc(100), 100, 100)
        states.append(st)
        assert cache.put([i] * 100, st)
    # 300 cached tokens > 250: the oldest (key 0) went, its rows are free
    assert states[0].released and cache.peek([0] * 100) is None
    assert arena.rows.used() == 200
    states[1].pins = 1  # a running request reads key 1
    cache.get([2] * 100)  # key 2 is now the most recent
    assert cache.evict_one() and states[2].released and not states[1].released
    assert not cache.evict_one()  # only the pinned entry is left
    assert cache.put([9] * 300, PrefixKv(arena, 0, 300, 300)) is False  # over budget alone: not cached


def test_arena_evicts_cache_entries_when_full():
    arena = KvArena(1, 200, 1, 4, torch.float32, "cpu")
    cache = PrefixCache(budget=10_000)
    a = PrefixKv(arena, arena.alloc(150), 150, 150)
    cache.put([1] * 150, a)
    start = arena.alloc(120, cache)  # needs a's rows: a is evicted
    assert a.released and start == 0
    with pytest.raises(MemoryError):
        arena.alloc(100, cache)  # 80 free, nothing left to evict


def test_row_allocator_first_fit_and_merging():
    r = RowAllocator(100)
    a, b, c = r.alloc(30), r.alloc(30), r.alloc(30)
    assert (a, b, c) == (0, 30, 60) and r.alloc(20) is None
    r.release(b, 30)
    assert r.alloc(40) is None and r.alloc(25) == 30  # first fit into the hole
    r.release(30, 25)
    r.release(a, 30)
    r.release(c, 30)
    assert r.free == [(0, 100)] and r.used() == 0  # neighbours merged back


# ---- the hybrid engine's state prefill and padded rows (hybrid.rs:555-617) ----
class _RecordingDecoder:
    def __init__(self):
        self.calls = []

    def new_state(self, n, cache):
        return SimpleNamespace(pins=0, released=False, next_pos=0, release=lambda: None)

    def forward(self, ids, B, T, pos, state, keep, cache):
        self.calls.append((list(ids), B, T, list(pos), keep))
        if keep:
            state.next_pos = max(pos) + 1
        return "x"


def _hybrid(chunk):
    from cev_b200.hybrid import HybridEngine
    eng = HybridEngine.__new__(HybridEngine)  # host logic only
    eng.decoder = _RecordingDecoder()
    eng.pad_id = 0
    eng.prefill_chunk = chunk
    eng.pass_tokens = 64
    eng.cache = PrefixCache(1000)
    return eng


def test_hybrid_prefill_runs_the_state_in_chunks_and_pins_it():
    eng = _hybrid(512)
    st = eng.prefill(list(range(1, 1101)))
    calls = eng.decoder.calls
    assert [(c[1], c[2]) for c in calls] == [(1, 512), (1, 512), (1, 76)]
    assert [c[3][0] for c in calls] == [0, 512, 1024] and calls[-1][3][-1] == 1099
    assert all(c[4] for c in calls) and st.pins == 1 and st.next_pos == 1100


def test_hybrid_rows_are_right_padded_and_continue_the_state():
    eng = _hybrid(512)
    state = SimpleNamespace(next_pos=300)
    x, t = eng.rows(state, [[5, 6, 7], [8, 9, 10, 11, 12], [13]])
    ids, B, T, pos, keep = eng.decoder.calls[0]
    assert (x, t, B, T, keep) == ("x", 5, 3, 5, False)
    assert ids == [5, 6, 7, 0, 0, 8, 9, 10, 11, 12, 13, 0, 0, 0, 0]
    assert pos == [300, 301, 302, 303, 304]  # every row continues at the state's next position
