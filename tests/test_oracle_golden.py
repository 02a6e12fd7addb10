"""The CPU oracle against HF transformers golden vectors and against the
reference's own parity invariants (parity_qwen35.rs:36-90,
parity_models.rs:61-64), all on CPU."""
import json
import os

import pytest
import torch
from safetensors.torch import load_file

from cev_b200 import weights
from oracle import ops
from oracle.engine import Engine, Request
from oracle.hybrid import HybridEngine, Lfm2, Qwen35
from oracle.qwen3 import Qwen3

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def rel(a, b):
    """max |a-b| / max |b| (parity_qwen35.rs:30-33)."""
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-6)).item()


def golden(name):
    meta = json.load(open(os.path.join(GOLD, f"hf_{name}.json")))
    return meta, load_file(os.path.join(GOLD, f"hf_{name}.safetensors"))


def build(name, meta, dtype=torch.float32):
    cfg = meta["config"]
    w = weights.init_weights(cfg, meta["seed"])
    if name == "qwen3":
        return Qwen3(cfg, w, dtype)
    return (Qwen35 if name == "qwen35" else Lfm2)(cfg, w, dtype)


def hidden_rows(name, model, ids):
    n = len(ids)
    if name == "qwen3":
        h, _ = model.forward_packed(None, ids, list(range(n)), ops.segment_mask([0] * n, 0), list(range(n)), [])
        return h
    h, _ = model.forward(model.embed(ids)[None], list(range(n)))
    return h[0]


@pytest.mark.parametrize("name", ["qwen3", "qwen35", "lfm2"])
def test_oracle_matches_transformers(name):
    meta, g = golden(name)
    model = build(name, meta)
    head = model.head_rows(meta["probe_ids"]).float()
    for r in range(meta["rows"]):
        ids = g[f"row{r}.ids"].tolist()
        h = hidden_rows(name, model, ids)
        n = len(ids)
        assert rel(h[n - 1], g[f"row{r}.hidden_last"]) < 2e-4
        assert rel(h[n // 2], g[f"row{r}.hidden_mid"]) < 2e-4
        assert (h[n - 1] @ head.t() - g[f"row{r}.logits_last"]).abs().max().item() < 1e-3


@pytest.mark.parametrize("name", ["qwen35", "lfm2"])
def test_prefix_state_branch_and_padded_row(name):
    """parity_qwen35.rs:69-89: prefix in two chunks into a state, then the
    branch and a right-padded shorter row equal the whole row (rel 2e-3)."""
    meta, g = golden(name)
    model = build(name, meta)
    ids = g["row2.ids"].tolist()
    t = len(ids)
    whole = hidden_rows(name, model, ids)
    split = t // 2
    c1 = split // 2
    _, s1 = model.forward(model.embed(ids[:c1])[None], list(range(c1)), None, keep=True)
    _, s2 = model.forward(model.embed(ids[c1:split])[None], list(range(c1, split)), s1, keep=True)
    assert s2.len == split and s2.next_pos == split
    branch = ids[split:]
    short = branch[:len(branch) // 2]
    rows = branch + short + [0] * (len(branch) - len(short))
    hb, _ = model.forward(model.embed(rows).reshape(2, len(branch), -1), list(range(split, t)), s2)
    assert rel(hb[0, len(branch) - 1], whole[t - 1]) < 2e-3
    assert rel(hb[1, len(short) - 1], whole[split + len(short) - 1]) < 2e-3


def test_packed_pass_equals_independent_questions():
    """README:42-47: every question of a packed block-masked pass sees
    exactly the prefix and itself, so its readout equals a pass with that
    question alone; and a second (prefix-cached) pass agrees within 1e-4
    (parity_models.rs:61-64)."""
    meta, _ = golden("qwen3")
    model = build("qwen3", meta)
    gen = torch.Generator().manual_seed(5)
    prefix = torch.randint(0, 1000, (100,), generator=gen).tolist()
    suffixes = [torch.randint(0, 1000, (n,), generator=gen).tolist() for n in (9, 14, 5, 20)]
    codes = [7, 8, 9, 10]
    eng = Engine(model, codes, prefill_chunk=32, pass_tokens=64)
    out = eng.run(Request(prefix, suffixes, [3, 3, 4, 2]))
    assert not out.prefix_cached
    again = eng.run(Request(prefix, suffixes, [3, 3, 4, 2]))
    assert again.prefix_cached
    for a, b in zip(out.readouts, again.readouts):
        assert (a.logits - b.logits).abs().max().item() < 1e-4
    for qi, s in enumerate(suffixes):
        alone = Engine(model, codes, prefill_chunk=32, pass_tokens=4096).run(Request(prefix, [s], [3]))
        assert (alone.readouts[0].hidden - out.readouts[qi].hidden).abs().max().item() < 1e-4
        # Whole prompt causally, no packing: the last token's hidden state.
        full = prefix + s
        h, _ = model.forward_packed(None, full, list(range(len(full))), ops.segment_mask([0] * len(full), 0), [len(full) - 1], [])
        assert rel(out.readouts[qi].hidden, h[0]) < 2e-4


def test_two_requests_in_one_pass():
    """run_many fuses a request and its calibration twin in one pass
    (service.rs:316-329): each still equals its own run."""
    meta, _ = golden("qwen3")
    model = build("qwen3", meta)
    gen = torch.Generator().manual_seed(6)
    p1 = torch.randint(0, 1000, (40,), generator=gen).tolist()
    p2 = torch.randint(0, 1000, (7,), generator=gen).tolist()
    sfx = [torch.randint(0, 1000, (n,), generator=gen).tolist() for n in (6, 11)]
    codes = [7, 8, 9]
    both = Engine(model, codes, prefill_chunk=16).run_many([Request(p1, sfx, [3, 3]), Request(p2, sfx, [3, 3])])
    for i, p in enumerate((p1, p2)):
        one = Engine(model, codes, prefill_chunk=16).run(Request(p, sfx, [3, 3]))
        for a, b in zip(one.readouts, both[i].readouts):
            assert (a.logits - b.logits).abs().max().item() < 1e-4


def test_hybrid_engine_rows_equal_whole_prompts():
    """hybrid.rs:697-739: each right-padded row continuing the cached prefix
    state reads the same last hidden state as its whole prompt."""
    meta, _ = golden("qwen35")
    model = build("qwen35", meta)
    gen = torch.Generator().manual_seed(7)
    prefix = torch.randint(0, 1000, (90,), generator=gen).tolist()
    sfx = [torch.randint(0, 1000, (n,), generator=gen).tolist() for n in (5, 12, 8)]
    eng = HybridEngine(model, [3, 4, 5], pad_id=0, prefill_chunk=40, pass_tokens=24)
    out = eng.run(Request(prefix, sfx, [3, 3, 3]))
    for s, r in zip(sfx, out.readouts):
        full = prefix + s
        h, _ = model.forward(model.embed(full)[None], list(range(len(full))))
        assert rel(r.hidden, h[0, -1]) < 2e-3
