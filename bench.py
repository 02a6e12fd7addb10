"""Benchmark of the packed block-masked prefill attention (cfg2 shape).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

One step = one packed attention call over 32 requests x (2048-token cached
prefix + 16 suffixes x 64 tokens), Hq 16 / Hkv 8, head_dim 128, bf16, on
seeded synthetic Q/K/V (N(0,1), RMS-normalised per head, RoPE at positions
restarting at 2048 per suffix).  The metric is effective TFLOP/s:
4 * D * Hq * (visible query-key pairs) per call = 5.585e11 FLOP; masked pairs
do not count.  With --gpus N (torchrun, one rank per GPU) every rank runs its
own batch (weak scaling, no collective on the data path); the time is the max
over ranks.

`--op gdn` / `--op conv` time one kernel alone at a config's layer shape
(the Qwen3.5 gated-delta-rule chunked prefill of cfg4; the LFM2 gated
short conv of cfg5) and print their own line with a roofline; `--op cfg3`,
`cfg4`, `cfg5` run only that config's decisions/sec measurement.  These
lines are for profiling and the per-kernel roofline, not the headline.

`value` is kernel throughput with inputs resident in HBM; `e2e` is the same
metric through the C ABI call with host buffers: pinned host -> device copies
of Q, K, V and the segment table, the call, and the device -> host copy of O
inside the timed region, every step (two buffer sets, so that one step's
upload overlaps the previous step's call and download).  `--impl reference` times the reference algorithm
(the CPU oracle: repeat_kv + matmul + additive mask + softmax + matmul,
qwen3.rs:206-220) on the host cores on a bounded sample.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "rust-cev_b200"))

METRIC = "packed-prefill attn TFLOP/s (% BF16 peak); decisions/sec at 1/2/4/8 B200"
CFG = dict(n_req=32, prefix=2048, n_suf=16, suf_len=64, hq=16, hkv=8, head_dim=128)
WORKLOAD = "cfg2 packed-prefill attention: 32 requests x (2048-token prefix + 16 x 64-token suffixes), Hq16/Hkv8, D128"


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["bf16_tflops"]), float(p["hbm_gbs"]), "measured"
    except Exception:
        return 1590.0, 6650.0, "fallback"


def profiled_traffic():
    """DRAM bytes per launch from the committed ncu summary, if any."""
    path = os.path.join(ROOT, "profiles", "attn_tc_cfg2.md")
    try:
        m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", open(path).read())
        return float(m.group(1)) if m else None
    except OSError:
        return None


class Clocks:
    """nvidia-smi sampling during the timed region."""

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), "--query-gpu=clocks.sm,clocks.max.sm,clocks_event_reasons.active,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
                 "--format=csv,noheader,nounits", "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *a):
        self.lines = []
        if self.proc:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in self.lines:
            f = [x.strip() for x in l.split(",")]
            try:
                sm.append(float(f[0]))
                mx = float(f[1])
            except (ValueError, IndexError):
                continue
            for n, v in zip(names, f[3:7]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def run_reference(args, rank, world):
    """The reference algorithm on the host cores (CPU oracle, f32)."""
    if rank != 0:
        return
    import torch
    sys.path.insert(0, ROOT)
    from oracle import ops as ref
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    c = CFG
    g = torch.Generator().manual_seed(0)
    D, hq, hkv, P, L = c["head_dim"], c["hq"], c["hkv"], c["prefix"], c["suf_len"]
    n_suf = 2  # bounded sample: one request's prefix with 2 of its suffixes per step

    def rn(*s):
        x = torch.randn(*s, generator=g)
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6)

    k = rn(1, hkv, P + n_suf * L, D)
    v = rn(1, hkv, P + n_suf * L, D)
    q = rn(1, hq, n_suf * L, D)
    # one request packed the reference way: K/V concatenated, additive mask
    # over [prefix | all suffixes], each suffix sees the prefix and itself causally
    mask = ref.segment_mask(sum([[j] * L for j in range(n_suf)], []), P)
    flops = 4.0 * D * hq * n_suf * (L * P + L * (L + 1) // 2)

    def step():
        ref.attend(q, k, v, mask)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = (time.perf_counter() - t0) / args.steps
    val = flops / dt / 1e12
    sample = f"{n_suf} of 512 suffixes (1 request prefix) per step, f32, torch CPU, {cores} threads"
    line = {"metric": METRIC, "value": val, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
            "config": {"workload": WORKLOAD, "sample": sample},
            "cpu_baseline": {"value": val, "unit": "TFLOP/s", "cores": cores, "cpu": cpu_model(), "kind": "port",
                             "sample": sample},
            "e2e": {"value": val, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def cpu_baseline_sample():
    """Reference algorithm on a bounded sample (rank 0, N=1 only)."""
    import torch
    sys.path.insert(0, ROOT)
    from oracle import ops as ref
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    c = CFG
    g = torch.Generator().manual_seed(0)
    D, hq, hkv, P, L, n_suf = c["head_dim"], c["hq"], c["hkv"], c["prefix"], c["suf_len"], 4
    x = torch.randn(1, hkv, P + n_suf * L, D, generator=g)
    q = torch.randn(1, hq, n_suf * L, D, generator=g)
    mask = ref.segment_mask(sum([[j] * L for j in range(n_suf)], []), P)
    flops = 4.0 * D * hq * n_suf * (L * P + L * (L + 1) // 2)
    ref.attend(q, x, x, mask)
    reps, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < 10.0:
        ref.attend(q, x, x, mask)
        reps += 1
    dt = (time.perf_counter() - t0) / reps
    return {"value": flops / dt / 1e12, "unit": "TFLOP/s", "cores": cores, "cpu": cpu_model(), "kind": "port",
            "sample": f"1 request prefix + {n_suf} suffixes, f32 torch CPU, {reps} reps over ~10 s"}


def cpu_model() -> str:
    """The host CPU's model name (for the CPU-baseline records)."""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform
    return platform.processor() or "unknown"


GDN_CHUNK = 64


def _layer_linear_params(cfg: dict, kind: str) -> int:
    """Weights one token multiplies through in one layer of ``kind`` (its
    projections and its MLP), i.e. half the linear FLOPs per token."""
    h, inter = cfg["hidden_size"], cfg["intermediate_size"]
    hq, hkv = cfg["num_attention_heads"], cfg["num_key_value_heads"]
    D = cfg.get("head_dim") or h // hq
    mlp = 3 * h * inter
    if kind == "attn":
        qo = 2 * hq * D if cfg.get("attn_output_gate", False) else hq * D
        return h * (qo + 2 * hkv * D) + hq * D * h + mlp
    if kind == "gdn":
        nk, nv = cfg["linear_num_key_heads"], cfg["linear_num_value_heads"]
        dk, dv = cfg["linear_key_head_dim"], cfg["linear_value_head_dim"]
        C = 2 * nk * dk + nv * dv
        return h * (C + nv * dv + 2 * nv) + nv * dv * h + mlp
    if kind == "conv":
        return h * 3 * h + h * h + mlp
    raise ValueError(kind)


def request_flops(cfg: dict, prefix_len: int, row_lens, n_codes: int) -> float:
    """Algorithmic FLOPs of one decision request: a ``prefix_len``-token
    state, causal over itself, then ``row_lens`` question rows (suffixes or
    right-padded rows: their real tokens only), each seeing the whole state
    and itself causally.  Counts the projection / MLP GEMMs (2 FLOP per MAC
    per real token), attention on visible (query, key) pairs only
    (4 * head_dim * Hq per pair), the GDN chunked delta rule per token and
    value head (2 C (3 dk + 2 dv) + 6 dk dv with C = 64) and the code
    readout; padding, masked pairs and the conv taps are not counted."""
    h = cfg["hidden_size"]
    hq = cfg["num_attention_heads"]
    D = cfg.get("head_dim") or h // hq
    types = cfg.get("layer_types") or ["full_attention"] * cfg["num_hidden_layers"]
    tokens = prefix_len + sum(row_lens)
    pairs = prefix_len * (prefix_len + 1) // 2 + sum(n * prefix_len + n * (n + 1) // 2 for n in row_lens)
    total = 0.0
    for t in types:
        kind = {"full_attention": "attn", "linear_attention": "gdn", "conv": "conv"}[t]
        total += 2.0 * _layer_linear_params(cfg, kind) * tokens
        if kind == "attn":
            total += 4.0 * D * hq * pairs
        elif kind == "gdn":
            dk, dv = cfg["linear_key_head_dim"], cfg["linear_value_head_dim"]
            total += (2.0 * GDN_CHUNK * (3 * dk + 2 * dv) + 6.0 * dk * dv) * cfg["linear_num_value_heads"] * tokens
    return total + 2.0 * h * n_codes * len(row_lens)


def decision_rows(name: str, qs, codes, max_permutations: int = 2):
    """Row lengths a request's questions become (every rotation variant's
    rendered suffix), as the engines run them."""
    from cev_b200 import service, workloads
    mode = "none" if name == "cfg5" else "permute"
    out = []
    for q in qs:
        for s in service.shifts(mode, len(q.options), max_permutations):
            out.append(len((q if s == 0 else q.rotated(s)).render(codes, workloads.SEP_ID)))
    return out


def cpu_decisions_baseline(name: str, dev) -> dict:
    """The reference algorithm (the CPU oracle, bf16 like the config) on the
    host cores for one request of config ``name``, timed on a bounded
    sample: each kind of layer the config has runs alone (a one-layer
    oracle model) over each work item of the request -- a prefill chunk at
    a given past length, the packed question pass, the state pass, the
    right-padded rows pass -- on synthetic activations and synthetic cached
    states of the true lengths (the arithmetic does not depend on the
    values).  Prefill-chunk times are fitted linearly in the past length and
    summed over the request's chunks; the request's time is the sum over
    its layers.  Decisions/s = questions per request / that time."""
    import torch
    sys.path.insert(0, ROOT)
    from cev_b200 import configs, weights, workloads
    from oracle import hybrid as ohyb
    from oracle import ops as oops
    from oracle import qwen3 as oq3
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    bf = torch.bfloat16
    g = torch.Generator().manual_seed(5)
    full = configs.get(name)
    codes = workloads.code_ids(4)

    def one_layer(kind):
        cfg = configs.get(name)
        cfg["num_hidden_layers"] = 1
        cfg["vocab_size"] = 1024  # the embedding table is not timed
        if "layer_types" in cfg:
            cfg["layer_types"] = [kind]
        w = {k: v.cpu() for k, v in weights.init_weights(cfg, 7, torch.float32, dev).items()}
        return cfg, w

    def timed_cpu(fn):
        t0 = time.perf_counter()
        fn()
        return time.perf_counter() - t0

    def rnd(*shape, dtype=bf):
        return torch.randn(*shape, generator=g).to(dtype)

    def chunks_total(t_at, n_chunks, chunk, pts):
        """Sum of t(past) over chunks at past 0, chunk, ..., fitted
        linearly through the measured points."""
        xs = [p for p in pts]
        ys = [t_at(p) for p in pts]
        n = len(xs)
        mx, my = sum(xs) / n, sum(ys) / n
        var = sum((x - mx) ** 2 for x in xs)
        b = sum((x - mx) * (y - my) for x, y in zip(xs, ys)) / var if var else 0.0
        a = my - b * mx
        return sum(a + b * (c * chunk) for c in range(n_chunks))

    parts = {}
    if name == "cfg3":
        prefix, qs = workloads.decision_request(1, 8192, 32, 48, 128, 4, 151643)
        rows = decision_rows("cfg3", qs, codes)
        cfg, w = one_layer("full_attention")
        m = oq3.Qwen3(cfg, w, bf)
        hkv, D = cfg["num_key_value_heads"], cfg["head_dim"]

        def chunk(past):
            kv = None if past == 0 else [oq3.LayerKv(rnd(1, hkv, past, D), rnd(1, hkv, past, D))]
            ids = torch.randint(0, 1024, (512,), generator=g).tolist()
            return timed_cpu(lambda: m.forward_packed(kv, ids, list(range(past, past + 512)),
                                                      oops.segment_mask([0] * 512, past), [511], [(0, 512)]))

        m.forward_packed(None, [1] * 16, list(range(16)), oops.segment_mask([0] * 16, 0), [15], [])  # warm-up
        head = 8192 - 512
        parts["prefill chunks"] = chunks_total(chunk, head // 512, 512, [0, head - 512])
        seg = [0] * 512 + sum([[j + 1] * n for j, n in enumerate(rows)], [])
        past = head
        kv = [oq3.LayerKv(rnd(1, hkv, past, D), rnd(1, hkv, past, D))]
        ids = torch.randint(0, 1024, (len(seg),), generator=g).tolist()
        parts["packed pass"] = timed_cpu(lambda: m.forward_packed(kv, ids, list(range(len(seg))),
                                                                  oops.segment_mask(seg, past), [len(seg) - 1], [(0, 512)]))
        t_req = full["num_hidden_layers"] * sum(parts.values())
        n_layers = {"attention": full["num_hidden_layers"]}
    else:
        hybrid_cfg4 = name == "cfg4"
        plen = 16384 if hybrid_cfg4 else 65536
        prefix, qs = workloads.decision_request(2 if hybrid_cfg4 else 3, plen, 32 if hybrid_cfg4 else 64,
                                                32 if hybrid_cfg4 else 64, 128 if hybrid_cfg4 else 64, 4,
                                                full["vocab_size"] - 1)
        rows = decision_rows(name, qs, codes)
        H = full["hidden_size"]
        kinds = ["linear_attention", "full_attention"] if hybrid_cfg4 else ["conv", "full_attention"]
        t_req = 0.0
        n_layers = {}
        for kind in kinds:
            cfg, w = one_layer(kind)
            dec = (ohyb.Qwen35 if hybrid_cfg4 else ohyb.Lfm2)(cfg, w, bf)
            hkv = cfg["num_key_value_heads"]
            D = cfg.get("head_dim") or H // cfg["num_attention_heads"]

            def state(past):
                if kind == "full_attention":
                    st = ohyb.AttnState(rnd(1, hkv, past, D), rnd(1, hkv, past, D))
                elif kind == "conv":
                    st = ohyb.ConvState(rnd(1, H, cfg["conv_L_cache"] - 1))
                else:
                    C = 2 * dec.nk * dec.dk + dec.nv * dec.dv
                    st = ohyb.GdnState(rnd(1, C, dec.kernel - 1), rnd(1, dec.nv, dec.dk, dec.dv, dtype=torch.float32))
                return ohyb.PrefixState([st], past, past)

            def run(b, t, past, keep):
                st = state(past) if past > 0 else None
                x = rnd(b, t, H)
                return timed_cpu(lambda: dec.forward(x, list(range(past, past + t)), st, keep=keep))

            run(1, 16, 0, True)  # warm-up
            n = full["layer_types"].count(kind)
            n_layers[kind] = n
            if hybrid_cfg4:
                t_state = run(1, plen, 0, True)  # the state runs once as one pass
            else:
                t_state = chunks_total(lambda p: run(1, 512, p, True), plen // 512, 512,
                                       [0, plen // 2, plen - 512] if kind == "full_attention" else [512])
            t_rows = run(len(rows), max(rows), plen, False)
            parts[f"{kind} state"] = t_state
            parts[f"{kind} rows"] = t_rows
            t_req += n * (t_state + t_rows)
    n_dec = len(qs)
    return {"value": n_dec / t_req, "unit": "decisions/s", "cores": cores, "cpu": cpu_model(), "kind": "port",
            "sample": f"one {name} request ({n_dec} questions): each layer kind alone through the bf16 CPU oracle "
                      "on synthetic states of the true lengths, per work item ("
                      + ", ".join(f"{k} {v:.2f} s" for k, v in parts.items())
                      + "; prefill chunks fitted linearly in the past length), summed over "
                      + ", ".join(f"{v} {k}" for k, v in n_layers.items())
                      + f" layers: {t_req:.1f} s per request"}


def _sustained_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops_sustained"]), "measured bf16 sustained"
    except Exception:
        return 1400.0, "fallback bf16 sustained"


def _roofline(flops_total: float, seconds: float, world: int) -> dict:
    """Tensor roofline of a decisions run: algorithmic FLOPs / s per GPU
    against the sustained cuBLAS bf16 figure (decision runs are long,
    power-capped steps)."""
    peak, src = _sustained_peak()
    per_gpu = flops_total / seconds / world / 1e12
    return {"bound": "tensor", "achieved": per_gpu, "peak": peak, "unit": "TFLOP/s", "frac": per_gpu / peak,
            "peak_source": src, "flop_total": flops_total}


def decisions_bench(n_req: int, dev, world: int, dist_mod, batch: int = 8):
    """cfg3: Qwen3-8B-shaped decoder (bf16, random init seed 1); per request
    an 8192-token random-id state (head 7680 prefilled in 512-token chunks,
    tail 512 in the packed pass) and 32 questions of U[48,128] tokens with 4
    option codes x 2 rotations, all 64 suffixes in one packed pass; served
    probabilities on the host.  Decisions = questions answered.  Timed end to
    end: token ids in from the host, probabilities out; this rank's
    ``n_req`` requests (the config's 256 over 8 GPUs is 32 per GPU) served
    ``batch`` per run_many call."""
    import torch
    from cev_b200 import configs, service, weights, workloads
    from cev_b200.engine import Engine
    from cev_b200.qwen3 import Qwen3
    cfg = configs.get("cfg3")
    w = weights.init_weights(cfg, 1, torch.bfloat16, dev)
    model = Qwen3(cfg, w, torch.bfloat16, dev, arena_rows=batch * 8192 + 16384)
    del w
    codes = workloads.code_ids(4)
    eng = Engine(model, codes, prefill_chunk=512, pass_tokens=16384, prefix_cache_tokens=batch * 8192)
    rank = int(os.environ.get("RANK", "0"))
    reqs = [workloads.decision_request(10_000 * (rank + 1) + i, 8192, 32, 48, 128, 4, 151643) for i in range(n_req + 1)]
    flops = sum(request_flops(cfg, len(p), decision_rows("cfg3", qs, codes), len(codes)) for p, qs in reqs[1:])

    def one(prefix, qs):
        return service.run_debiased(eng, prefix, qs, "permute", codes, workloads.SEP_ID, max_permutations=2)

    one(*reqs[0])  # warm-up (distinct prefix: no cache hit later)
    eng.cache.clear()
    torch.cuda.synchronize()
    if world > 1:
        dist_mod.barrier()
    t0 = time.perf_counter()
    # each run_many call serves `batch` requests: their prefill chunks and
    # question passes share passes (each request's results are its own)
    for b0 in range(1, n_req + 1, batch):
        results = service.run_debiased_many(eng, reqs[b0:b0 + batch], "permute", codes, workloads.SEP_ID,
                                            max_permutations=2)
        assert all(len(probs) == 32 for _, probs in results)
    torch.cuda.synchronize()
    dt = torch.tensor([time.perf_counter() - t0], device=dev)
    fl = torch.tensor([flops], device=dev, dtype=torch.float64)
    if world > 1:
        dist_mod.all_reduce(dt, op=dist_mod.ReduceOp.MAX)
        dist_mod.all_reduce(fl)
    n_dec = 32 * n_req * world
    del eng, model
    return {"value": n_dec / dt.item(), "unit": "decisions/s", "requests_per_gpu": n_req,
            "requests_total": n_req * world, "batching": f"{batch} requests per run_many call",
            "seconds": dt.item(), "workload": "cfg3 Qwen3-8B-shaped bf16, 8192-token state, 32 questions x 2 rotations",
            "parallelism": f"dp{world}", "roofline": _roofline(fl.item(), dt.item(), world)}


def hybrid_decisions_bench(name: str, n_req: int, dev, world: int, dist_mod):
    """cfg4 (Qwen3.5-shaped GDN hybrid, seed 2, 16384-token state run once
    as one pass, 32 questions of U[32,128] tokens) or cfg5 (LFM2-shaped, seed 3, 65536-token
    state in 512-token chunks, 64 questions of 64 tokens): the state is
    prefilled once into the cached prefix state, the questions run as
    right-padded rows continuing it (hybrid.rs:697-739).  4 option codes,
    2 rotations per question (cfg4) / none (cfg5).  Decisions/s end to end.
    With N > 1 GPUs cfg4 runs its own requests on every rank; cfg5 runs one
    request stream on all ranks with the attention layers split by KV-head
    group (the head outputs gathered by the attention epilogue over NVLink)."""
    import torch
    from cev_b200 import configs, hybrid, service, weights, workloads
    cfg = configs.get(name)
    seed, plen, nq, lo, hi, mode = (2, 16384, 32, 32, 128, "permute") if name == "cfg4" else (3, 65536, 64, 64, 64, "none")
    rank = int(os.environ.get("RANK", "0"))
    split = None
    if name == "cfg5" and world > 1:
        from cev_b200.tp import KvHeadSplit
        split = KvHeadSplit(cfg["num_attention_heads"], cfg["num_key_value_heads"],
                            cfg.get("head_dim") or cfg["hidden_size"] // cfg["num_attention_heads"], rank, world)
        if os.environ.get("CEV_HEAD_GATHER", "fused") == "fused":
            # head outputs gathered by the attention epilogue over NVLink
            # (largest call: 64 right-padded rows x 64 tokens); the token-local
            # layers split by token rows, the residual stream gathered over
            # NVLink peer stores
            split.enable_fused_gather(8192, dev, hidden=cfg["hidden_size"])
            split.sequence_parallel = True
    w = weights.init_weights(cfg, seed, torch.bfloat16, dev)
    if name == "cfg4":
        dec = hybrid.Qwen35(cfg, w, torch.bfloat16, dev, max_len=plen + 1024, arena_rows=plen + 8192)
    else:
        dec = hybrid.Lfm2(cfg, w, torch.bfloat16, dev, max_len=plen + 1024, arena_rows=plen + 8192, split=split)
    del w
    codes = workloads.code_ids(4)
    # cfg4's state is run once: one 16384-token pass; cfg5's is prefilled in 512-token chunks
    # cfg5's 128 state chunks replay from CUDA graphs
    graphs = name == "cfg5" and (split is None or split.fused is not None)
    eng = hybrid.HybridEngine(dec, codes, pad_id=0, prefill_chunk=plen if name == "cfg4" else 512, pass_tokens=8192,
                              prefix_cache_tokens=plen, chunk_graphs=graphs)
    vocab = cfg["vocab_size"] - 1
    stream = 0 if split is not None else rank  # a split model runs the same requests on every rank
    reqs = [workloads.decision_request(20_000 * (stream + 1) + i, plen, nq, lo, hi, 4, vocab) for i in range(n_req + 1)]
    flops = sum(request_flops(cfg, len(p), decision_rows(name, qs, codes), len(codes)) for p, qs in reqs[1:])

    gate = None
    if split is not None:
        # every rank runs each request of the split model: check on the host
        # that all peers are still there before a request's first launch
        from cev_b200.health import StepGate
        gate = StepGate(rank, world, deadline_s=120.0, prefix=f"cev/{name}")
    step = [0]

    def one(prefix, qs):
        if gate is not None:
            step[0] += 1
            gate.enter(step[0])
        return service.run_debiased(eng, prefix, qs, mode, codes, workloads.SEP_ID, max_permutations=2)

    one(*reqs[0])
    eng.cache.clear()
    torch.cuda.synchronize()
    if world > 1:
        dist_mod.barrier()
    t0 = time.perf_counter()
    for prefix, qs in reqs[1:]:
        _, probs = one(prefix, qs)
        assert len(probs) == nq
    torch.cuda.synchronize()
    dt = torch.tensor([time.perf_counter() - t0], device=dev)
    if world > 1:
        dist_mod.all_reduce(dt, op=dist_mod.ReduceOp.MAX)
    streams = 1 if split is not None else world
    gather = None
    if split is not None:
        gather = "fused into the attention epilogue (NVLink peer stores)" if split.fused else "NCCL all-gather"
        if split.fused is not None:
            split.fused.close()
    del eng, dec
    return {"value": nq * n_req * streams / dt.item(), "unit": "decisions/s", "requests_per_stream": n_req,
            "seconds": dt.item(), "workload": f"{name}: {plen}-token state, {nq} questions, rows continuing the state",
            "parallelism": f"kv-head split x{world}" if split is not None else f"dp{world}", "head_gather": gather,
            "roofline": _roofline(flops * streams, dt.item(), world)}


def timed(fn, steps, warmup, stream):
    """Average device time (ms) of fn() over `steps` after `warmup` calls."""
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        fn()
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def gdn_flops(T: int, nv: int, dk: int, dv: int, chunk: int = 64) -> float:
    """Algorithmic FLOPs of the chunked gated delta rule per call: per chunk
    of C tokens and value head, K K^T and Q K^T (2 C^2 dk each), the WY
    products W = T beta K and U = T beta V (2 C^2 dk, 2 C^2 dv), U - W S,
    Q S and the state update K^T U' (2 C dk dv each) and the intra-chunk
    (Q K^T * mask) U' (2 C^2 dv)."""
    n_chunks = (T + chunk - 1) // chunk
    C = chunk
    per = 2 * C * C * (3 * dk + 2 * dv) + 6 * C * dk * dv
    return float(n_chunks * nv * per)


def op_bench(args, dev):
    """One kernel alone at a config's layer shape (synthetic inputs)."""
    import torch
    from cev_b200 import ops
    stream = torch.cuda.current_stream()
    g = torch.Generator(device=dev).manual_seed(7)
    peak_tf, peak_hbm, src = peaks()
    if args.op == "gdn":
        # cfg4 GDN layer, one 512-token prefill chunk continuing a state
        B, T, nk, nv, dk, dv = 1, 512, 16, 32, 128, 128
        C_ = 2 * nk * dk + nv * dv
        conv_out = (torch.randn(B * T, C_, device=dev, generator=g) * 0.5).bfloat16()
        ab = torch.randn(B * T, 2 * nv, device=dev, generator=g).bfloat16()
        z = torch.randn(B * T, nv * dv, device=dev, generator=g).bfloat16()
        a_log = torch.rand(nv, device=dev, generator=g) * 2
        dt_bias = torch.rand(nv, device=dev, generator=g)
        norm_w = (torch.rand(dv, device=dev, generator=g) + 0.5).bfloat16()
        s_in = torch.randn(1, nv, dk, dv, device=dev, generator=g) * 0.1
        s_out = torch.empty(B, nv, dk, dv, device=dev)
        ws = torch.empty(ops.gdn_workspace_size(B, T, nv, dk, dv), dtype=torch.uint8, device=dev)
        y = torch.empty(B * T, nv * dv, dtype=torch.bfloat16, device=dev)

        def fn():
            ops.gdn_chunk_prefill(conv_out, ab, 2 * nv, z, nv * dv, a_log, dt_bias, norm_w, 1e-6, s_in, s_out, B, T, nk,
                                  nv, dk, dv, ws, out=y)
        flops = gdn_flops(T, nv, dk, dv)
        nbytes = (conv_out.numel() + ab.numel() + z.numel() + y.numel()) * 2 + (s_in.numel() + s_out.numel()) * 4
        ms = timed(fn, args.steps, args.warmup, stream)
        ops.device_status()
        tf = flops / (ms / 1e3) / 1e12
        # the cfg4 state pass: the 16384-token state run once through a GDN layer
        Ts = 16384
        conv_s = (torch.randn(Ts, C_, device=dev, generator=g) * 0.5).bfloat16()
        ab_s = torch.randn(Ts, 2 * nv, device=dev, generator=g).bfloat16()
        z_s = torch.randn(Ts, nv * dv, device=dev, generator=g).bfloat16()
        ws_s = torch.empty(ops.gdn_workspace_size(1, Ts, nv, dk, dv), dtype=torch.uint8, device=dev)
        y_s = torch.empty(Ts, nv * dv, dtype=torch.bfloat16, device=dev)

        def fn_state():
            ops.gdn_chunk_prefill(conv_s, ab_s, 2 * nv, z_s, nv * dv, a_log, dt_bias, norm_w, 1e-6, None, s_out, 1, Ts,
                                  nk, nv, dk, dv, ws_s, out=y_s)
        ms_s = timed(fn_state, max(3, args.steps // 10), 3, stream)
        ops.device_status()
        tf_s = gdn_flops(Ts, nv, dk, dv) / (ms_s / 1e3) / 1e12
        line = {"metric": "gdn chunked prefill TFLOP/s (cfg4 layer, one 512-token chunk)", "value": tf,
                "unit": "TFLOP/s", "ms_per_step": ms, "steps": args.steps, "warmup": args.warmup, "dtype": "bf16",
                "config": {"workload": f"B{B} T{T} nk{nk} nv{nv} dk{dk} dv{dv}, chunk 64, state in/out",
                           "flop_per_step": flops, "bytes_per_step": nbytes},
                "state_pass": {"workload": f"B1 T{Ts} (the cfg4 state run once through one GDN layer)",
                               "tflops": tf_s, "ms": ms_s},
                "roofline": {"bound": "tensor (tcgen05, bf16 three-term split; latency of the chunk-sequential scan)",
                             "achieved": tf, "peak": peak_tf, "unit": "TFLOP/s", "frac": tf / peak_tf,
                             "peak_source": src + " bf16 burst",
                             "hbm_gbs": nbytes / (ms / 1e3) / 1e9, "hbm_peak_gbs": peak_hbm}}
    elif args.op == "conv":
        # cfg5 gated short conv layer (d 2048, K 3) over a 16384-token run
        B, T, d, K = 1, 16384, 2048, 3
        bcx = torch.randn(B * T, 3 * d, device=dev, generator=g).bfloat16()
        w = torch.randn(d, K, device=dev, generator=g).bfloat16()
        tail_in = torch.randn(1, d, K - 1, device=dev, generator=g).bfloat16()
        tail_out = torch.empty(B, d, K - 1, dtype=torch.bfloat16, device=dev)
        out = torch.empty(B * T, d, dtype=torch.bfloat16, device=dev)

        def fn():
            ops.short_conv(bcx, B, T, d, w, None, tail_in, tail_out, out=out)
        nbytes = (bcx.numel() + out.numel()) * 2
        ms = timed(fn, args.steps, args.warmup, stream)
        ops.device_status()
        gbs = nbytes / (ms / 1e3) / 1e9
        line = {"metric": "gated short conv GB/s (cfg5 layer)", "value": gbs, "unit": "GB/s", "ms_per_step": ms,
                "steps": args.steps, "warmup": args.warmup, "dtype": "bf16",
                "config": {"workload": f"B{B} T{T} d{d} K{K} (inputs larger than L2)", "bytes_per_step": nbytes},
                "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak_hbm, "unit": "GB/s",
                             "frac": gbs / peak_hbm, "peak_source": src + " copy"}}
    elif args.op == "chunk":
        # cfg5 attention layer, one 512-token prefill chunk after a 32768-token
        # cached prefix: all 8 KV heads (one GPU) and one KV head (a rank of
        # the 8-way KV-head split), planned split-KV against no split
        P, T, D = 32768, 512, 64
        line = {"metric": "prefill-chunk attention TFLOP/s (cfg5 layer, 512 tokens after a 32768-token prefix)",
                "unit": "TFLOP/s", "steps": args.steps, "warmup": args.warmup, "dtype": "bf16",
                "config": {"workload": f"one segment q_len {T}, prefix {P}, head_dim {D}, causal own rows"}}
        for hq, hkv in ((32, 8), (4, 1)):
            q = torch.randn(T, hq, D, device=dev, generator=g).bfloat16()
            k = torch.randn(P + T, hkv, D, device=dev, generator=g).bfloat16()
            v = torch.randn(P + T, hkv, D, device=dev, generator=g).bfloat16()
            o = torch.empty_like(q)
            flops = 4.0 * D * hq * sum(P + i + 1 for i in range(T))
            res = {}
            for name, ns in (("split", None), ("unsplit", 1)):
                plan = ops.AttnPlan([(0, T, 0, P, P)], T, P + T, hq, hkv, D, torch.bfloat16, dev, n_split=ns)
                ms = timed(lambda: ops.attend_packed(q, k, v, plan, out=o), args.steps, args.warmup, stream)
                ops.device_status()
                res[name] = {"tflops": flops / (ms / 1e3) / 1e12, "ms": ms, "n_split": plan.n_split}
            line[f"hq{hq}_hkv{hkv}"] = res
        line["value"] = line["hq32_hkv8"]["split"]["tflops"]
        line["roofline"] = {"bound": "tensor", "achieved": line["value"], "peak": peak_tf, "unit": "TFLOP/s",
                            "frac": line["value"] / peak_tf, "peak_source": src}
    elif args.op == "glue":
        # the bandwidth-bound glue at the decision configs' shapes, inputs
        # larger than L2: QK-norm + RoPE writing K/V into arena rows (cfg5
        # and cfg3 attention layers, 16384 tokens), residual add + RMSNorm
        # and SwiGLU (cfg3 hidden 4096 / intermediate 12288, 16384 tokens)
        res = {}
        n = 16384
        for name, hq, hkv, D, theta in (("qk_norm_rope cfg5 (32/8/8 heads, D 64)", 32, 8, 64, 1e6),
                                        ("qk_norm_rope cfg3 (32/8/8 heads, D 128)", 32, 8, 128, 1e6)):
            qkv = torch.randn(n, (hq + 2 * hkv) * D, device=dev, generator=g).bfloat16()
            q = torch.empty(n, hq, D, dtype=torch.bfloat16, device=dev)
            ka = torch.empty(n, hkv, D, dtype=torch.bfloat16, device=dev)
            va = torch.empty_like(ka)
            wq = torch.ones(D, dtype=torch.bfloat16, device=dev)
            pos = torch.arange(n, device=dev, dtype=torch.int32)
            rows = torch.randperm(n, device=dev, generator=g).to(torch.int32)  # scattered arena rows
            ms = timed(lambda: ops.qk_norm_rope(qkv, (0, D), hq * D, (hq + hkv) * D, hq, hkv, D, wq, wq, 1e-6, False,
                                                pos, theta, D, q, ka, va, rows), args.steps, args.warmup, stream)
            nbytes = 2 * qkv.numel() * 2 + n * 8  # read every head row once, write it once; ids
            res[name] = {"us": ms * 1e3, "gbs": nbytes / (ms / 1e3) / 1e9}
        H, I = 4096, 12288
        x = torch.randn(n, H, device=dev, generator=g).bfloat16()
        a = torch.randn(n, H, device=dev, generator=g).bfloat16()
        wn = torch.ones(H, dtype=torch.bfloat16, device=dev)
        o = torch.empty_like(x)
        ms = timed(lambda: ops.add_rms_norm(x, a, wn, 1e-6, out=o), args.steps, args.warmup, stream)
        res["add_rms_norm cfg3 (hidden 4096)"] = {"us": ms * 1e3, "gbs": 4 * x.numel() * 2 / (ms / 1e3) / 1e9}
        gu = torch.randn(n, 2 * I, device=dev, generator=g).bfloat16()
        so = torch.empty(n, I, dtype=torch.bfloat16, device=dev)
        ms = timed(lambda: ops.swiglu(gu, out=so), args.steps, args.warmup, stream)
        res["swiglu cfg3 (intermediate 12288)"] = {"us": ms * 1e3, "gbs": 3 * n * I * 2 / (ms / 1e3) / 1e9}
        ops.device_status()
        first = next(iter(res.values()))["gbs"]
        line = {"metric": "bandwidth-bound glue GB/s (16384 tokens, bf16)", "value": first, "unit": "GB/s",
                "steps": args.steps, "warmup": args.warmup, "dtype": "bf16", "kernels": res,
                "config": {"workload": "QK-norm + RoPE (cfg5, cfg3 attention layers), residual add + RMSNorm, "
                                       "SwiGLU at 16384 tokens; inputs larger than L2"},
                "roofline": {"bound": "hbm", "achieved": first, "peak": peak_hbm, "unit": "GB/s",
                             "frac": first / peak_hbm, "peak_source": src + " copy",
                             "per_kernel_frac": {k: v["gbs"] / peak_hbm for k, v in res.items()}}}
    else:
        raise SystemExit(f"unknown --op {args.op}")
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=600)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="cevk")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--decisions", type=int, default=32,
                    help="also measure cfg3 decisions/sec on this many requests per GPU (0 = skip; the config's "
                         "256 requests over 8 GPUs are 32 per GPU)")
    ap.add_argument("--batch", type=int, default=8, help="cfg3 requests per run_many call")
    ap.add_argument("--hybrid", type=int, default=4,
                    help="also measure cfg4 and cfg5 decisions/sec on this many requests per GPU (0 = skip)")
    ap.add_argument("--op", default="attn", choices=["attn", "gdn", "conv", "chunk", "glue", "cfg3", "cfg4", "cfg5"],
                    help="attn: the headline line; gdn / conv / chunk / glue: kernels at their layer shapes; "
                         "cfg3/4/5: only that config's decisions/sec")
    ap.add_argument("--requests", type=int, default=2, help="requests per GPU for --op cfg3/cfg4/cfg5")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return

    import torch
    import torch.distributed as dist
    from cev_b200 import ops, workloads

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        # short process-group timeout, non-blocking NCCL communicator init
        from cev_b200 import health
        health.init_distributed("nccl", rank, world, timeout_s=120.0, device=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    if args.op in ("gdn", "conv", "chunk", "glue"):
        if rank == 0:
            op_bench(args, dev)
    elif args.op in ("cfg3", "cfg4", "cfg5"):
        res = (decisions_bench(args.requests, dev, world, dist, args.batch) if args.op == "cfg3" else
               hybrid_decisions_bench(args.op, args.requests, dev, world, dist))
        if rank == 0:
            print(json.dumps({"metric": f"{args.op} decisions/sec", **res}), flush=True)
    if args.op != "attn":
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return

    wb = workloads.AttentionBatch(seed=1000 + rank, device=dev, **CFG)
    stream = torch.cuda.current_stream()
    for _ in range(args.warmup):
        wb.run()
    torch.cuda.synchronize()
    ops.device_status()

    # ---------------- device-resident timing ----------------
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    barrier()
    torch.cuda.synchronize()
    with Clocks(local) as clk:
        time.sleep(1.0)  # let the sampler start before the timed region
        t_all0 = torch.cuda.Event(enable_timing=True)
        t_all1 = torch.cuda.Event(enable_timing=True)
        t_all0.record(stream)
        for i in range(args.steps):
            starts[i].record(stream)
            wb.run()
            ends[i].record(stream)
        t_all1.record(stream)
        torch.cuda.synchronize()
    barrier()
    total_ms = t_all0.elapsed_time(t_all1)
    kern_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    t = torch.tensor([total_ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms = t.item()
    ms_step = total_ms / args.steps
    value = world * wb.flops * args.steps / (total_ms / 1e3) / 1e12
    ops.device_status()

    # ---------------- end to end through the C ABI, host buffers ----------------
    # Every step copies its Q, K, V and segment table from pinned host memory,
    # runs the C-ABI call and copies O back.  Two buffer sets and two streams
    # (copy-in; call + copy-out) let step i+1's upload overlap step i's call
    # and download, as a serving loop would; the copies stay in the timed
    # region.
    import ctypes as C
    from cev_b200._lib import BF16, check, lib
    hq_, hk, hv = (wb.q.cpu().pin_memory(), wb.k.cpu().pin_memory(), wb.v.cpu().pin_memory())
    hseg = wb.plan.host.pin_memory()
    ho = [torch.empty_like(hq_).pin_memory() for _ in range(2)]
    bufs = [(torch.empty_like(wb.q), torch.empty_like(wb.k), torch.empty_like(wb.v), torch.empty_like(wb.q),
             torch.empty_like(wb.plan.dev)) for _ in range(2)]
    h2d = sum(x.numel() * x.element_size() for x in (hq_, hk, hv, hseg))
    d2h = ho[0].numel() * ho[0].element_size()
    s_in, s_run = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_free = [torch.cuda.Event() for _ in range(2)]  # buffer set done (call + download)

    def e2e_step(i):
        dq, dk, dv, do, dseg = bufs[i % 2]
        with torch.cuda.stream(s_in):
            s_in.wait_event(ev_free[i % 2])
            dq.copy_(hq_, non_blocking=True)
            dk.copy_(hk, non_blocking=True)
            dv.copy_(hv, non_blocking=True)
            dseg.copy_(hseg, non_blocking=True)
            ev_in[i % 2].record(s_in)
        with torch.cuda.stream(s_run):
            s_run.wait_event(ev_in[i % 2])
            check(lib().cevk_attn_packed_prefill(
                C.c_void_p(dq.data_ptr()), C.c_void_p(dk.data_ptr()), C.c_void_p(dv.data_ptr()),
                C.c_void_p(do.data_ptr()), wb.n_tokens, wb.n_kv, wb.hq, wb.hkv, wb.D, dq.stride(0), dk.stride(0),
                do.stride(0), C.c_void_p(dseg.data_ptr()), wb.plan.n_segs, wb.plan.n_tiles, 1.0 / wb.D ** 0.5, BF16,
                C.c_void_p(s_run.cuda_stream)))
            ho[i % 2].copy_(do, non_blocking=True)
            ev_free[i % 2].record(s_run)

    for i in range(4):
        e2e_step(i)
    torch.cuda.synchronize()
    e_steps = max(3, min(args.steps, 20))
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(s_in)
    for i in range(e_steps):
        e2e_step(i)
    s_in.wait_stream(s_run)
    e1.record(s_in)
    torch.cuda.synchronize()
    e_ms = torch.tensor([e0.elapsed_time(e1)], device=dev)
    if world > 1:
        dist.all_reduce(e_ms, op=dist.ReduceOp.MAX)
    e2e_val = world * wb.flops * e_steps / (e_ms.item() / 1e3) / 1e12
    if not torch.equal(ho[(e_steps - 1) % 2].to(dev), wb.out):
        raise RuntimeError("end-to-end output differs from the device-resident output")

    peak_tf, peak_hbm, src = peaks()
    avg_kern = statistics.mean(kern_ms[1:] if len(kern_ms) > 1 else kern_ms)
    achieved = wb.flops / (avg_kern / 1e3) / 1e12
    tr = profiled_traffic()
    line = {
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": WORKLOAD, "flop_per_step_per_gpu": wb.flops,
                   "l2": "inputs larger than L2 (Q+K+V+O = %.0f MB per GPU)" % (
                       (2 * wb.q.numel() + wb.k.numel() + wb.v.numel()) * 2 / 1e6),
                   "parallelism": f"dp{world} (independent request batches, no collective)"},
        "pct_of_bf16_peak": 100.0 * (value / world) / peak_tf,
        "e2e": {"value": e2e_val, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak_tf, "unit": "TFLOP/s",
                     "frac": achieved / peak_tf, "peak_source": src + " bf16 burst",
                     "traffic": tr, "algorithmic_bytes": wb.algorithmic_bytes()},
        "clocks": clk.summary(),
        "gpu_launches": args.steps,
    }
    if args.decisions > 0 or args.hybrid > 0:
        del wb, bufs, hq_, hk, hv, ho
        torch.cuda.empty_cache()
    cpu_leg = rank == 0 and world == 1 and not args.no_cpu_baseline
    if args.decisions > 0:
        line["decisions"] = decisions_bench(args.decisions, dev, world, dist, args.batch)
        torch.cuda.empty_cache()
        if cpu_leg:
            line["decisions"]["cpu_baseline"] = cpu_decisions_baseline("cfg3", dev)
    if args.hybrid > 0:
        for name in ("cfg4", "cfg5"):
            line[f"decisions_{name}"] = hybrid_decisions_bench(name, args.hybrid, dev, world, dist)
            torch.cuda.empty_cache()
            if cpu_leg:
                line[f"decisions_{name}"]["cpu_baseline"] = cpu_decisions_baseline(name, dev)
    if cpu_leg:
        line["cpu_baseline"] = cpu_baseline_sample()
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
