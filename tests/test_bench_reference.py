"""bench.py's reference arm (the reference algorithm on the host cores) runs
without a GPU and prints the one JSON line the benchmark driver reads, with
the same metric as the GPU arm and its CPU-baseline and e2e records."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_the_contract_line():
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "3",
                          "--warmup", "3"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.strip()]
    d = json.loads(lines[-1])
    assert d["impl"] == "reference" and d["unit"] == "TFLOP/s" and d["higher_is_better"] is True
    assert d["metric"].startswith("packed-prefill attn TFLOP/s") and d["value"] > 0
    assert d["steps"] == 3 and d["warmup"] == 3 and d["n_gpus"] == 1
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["sample"] and cb["value"] == d["value"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
    assert "workload" in d["config"]


def test_decision_flop_accounting():
    """The algorithmic FLOPs behind each decisions line's roofline: cfg3's
    per-request count on its mean shape (8192-token state, 64 suffixes of
    ~88 tokens) is 2 * 6.946e9 linear weights x 13,824 tokens + 4.72e13 of
    visible attention pairs = 2.39e14, 7.47e12 per decision; the GDN core of
    a 512-token cfg4 chunk matches the per-chunk formula of the GDN line."""
    sys.path.insert(0, ROOT)
    import bench
    from cev_b200 import configs
    cfg3 = configs.get("cfg3")
    f = bench.request_flops(cfg3, 8192, [88] * 64, 4)
    assert abs(f / 2.39e14 - 1) < 0.01 and abs(f / 32 / 7.47e12 - 1) < 0.01
    cfg4 = configs.get("cfg4")
    gdn_only = dict(cfg4, num_hidden_layers=1, layer_types=["linear_attention"])
    core = bench.request_flops(gdn_only, 512, [], 0) - 2.0 * bench._layer_linear_params(cfg4, "gdn") * 512
    assert abs(core / bench.gdn_flops(512, 32, 128, 128) - 1) < 1e-9
    # a right-padded row counts its real tokens only, seeing the whole state
    one = dict(cfg3, num_hidden_layers=1)
    d = bench.request_flops(one, 100, [7], 0) - bench.request_flops(one, 100, [], 0)
    lin = 2.0 * bench._layer_linear_params(cfg3, "attn") * 7
    assert abs(d - lin - 4.0 * 128 * 32 * (7 * 100 + 28)) < 1
