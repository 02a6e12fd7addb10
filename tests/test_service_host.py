"""The serving layer's host logic without a GPU: several requests through
one run_many call (run_debiased_many) answer exactly as each request does
through run_debiased (service.rs:288-348), with rotations and with a
calibration twin, over a deterministic stand-in engine."""
import torch

from cev_b200 import service, workloads
from cev_b200.engine import Output, Readout


class _FakeEngine:
    """Deterministic logits per (prefix, suffix): enough to compare two
    routes through the answer math; records the run_many batch sizes."""

    def __init__(self):
        self.calls = []

    def run_many(self, reqs):
        self.calls.append(len(reqs))
        outs = []
        for r in reqs:
            readouts = []
            for s, k in zip(r.suffixes, r.n_options):
                g = torch.Generator().manual_seed(hash((tuple(r.prefix[:4]), len(r.prefix), tuple(s))) & 0x7FFFFFFF)
                readouts.append(Readout(torch.randn(k, generator=g) * 2, torch.zeros(1)))
            outs.append(Output(readouts, 0, False))
        return outs


def _items(n, n_opt=4):
    return [workloads.decision_request(300 + i, 64 + 8 * i, 5, 22, 32, n_opt, 1000) for i in range(n)]


def test_many_requests_answer_like_one_at_a_time():
    codes = workloads.code_ids(4)
    items = _items(3)
    eng = _FakeEngine()
    got = service.run_debiased_many(eng, items, "permute", codes, workloads.SEP_ID, max_permutations=2)
    assert eng.calls == [3]  # one engine call for every request
    for (prefix, qs), (scores, probs) in zip(items, got):
        want_s, want_p = service.run_debiased(_FakeEngine(), prefix, qs, "permute", codes, workloads.SEP_ID,
                                              max_permutations=2)
        assert scores == want_s and probs == want_p
        assert all(abs(sum(p) - 1.0) < 1e-12 for p in probs)


def test_many_requests_with_a_calibration_twin():
    codes = workloads.code_ids(3)
    items = _items(2, n_opt=3)
    cf = [7, 8, 9, 10]
    eng = _FakeEngine()
    got = service.run_debiased_many(eng, items, "full", codes, workloads.SEP_ID, cf_prefix=cf, max_permutations=3)
    assert eng.calls == [4]  # each request and its content-free twin
    for (prefix, qs), res in zip(items, got):
        want = service.run_debiased(_FakeEngine(), prefix, qs, "full", codes, workloads.SEP_ID, cf_prefix=cf,
                                    max_permutations=3)
        assert res == want


def test_unknown_mode_is_refused():
    import pytest
    with pytest.raises(ValueError, match="unknown debias mode"):
        service.run_debiased_many(_FakeEngine(), _items(1), "sideways", workloads.code_ids(4), workloads.SEP_ID)
