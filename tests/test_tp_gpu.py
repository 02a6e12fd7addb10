"""The LFM2 attention layers split by KV-head group over 2 GPUs (NCCL
all-gather of head outputs), with the token-local layers on every token or
split by token rows, against the unsplit model on one GPU: same request,
f32, readouts within 1e-4.  Needs 2 GPUs (skipped otherwise)."""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _request(cfg):
    from cev_b200 import workloads
    codes = workloads.code_ids(3)
    prefix, qs = workloads.decision_request(9, 300, 4, 14, 28, 3, cfg["vocab_size"])
    return codes, prefix, [q.render(codes, workloads.SEP_ID) for q in qs]


def _run(model, cfg, graphs=False):
    from cev_b200 import hybrid
    from cev_b200.engine import Request
    codes, prefix, sfx = _request(cfg)
    eng = hybrid.HybridEngine(model, codes, pad_id=0, prefill_chunk=128, pass_tokens=256, chunk_graphs=graphs)
    out = eng.run(Request(prefix, sfx, [3] * len(sfx)))
    return torch.stack([r.logits.float().cpu() for r in out.readouts])


def _rank(rank, world, port, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    torch.cuda.set_device(rank)
    from datetime import timedelta
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                            timeout=timedelta(seconds=60))
    try:
        from cev_b200 import configs, hybrid, weights
        from cev_b200.tp import KvHeadSplit
        cfg = configs.tiny_lfm2()
        w = weights.init_weights(cfg, 41)
        D = cfg.get("head_dim") or cfg["hidden_size"] // cfg["num_attention_heads"]
        outs = []
        for token_split in (True, False):
            sp = KvHeadSplit(cfg["num_attention_heads"], cfg["num_key_value_heads"], D, rank, world)
            sp.sequence_parallel = token_split
            outs.append(_run(hybrid.Lfm2(cfg, w, torch.float32, f"cuda:{rank}", arena_rows=4096, split=sp), cfg))
        err = None
        if rank == 0:
            whole = _run(hybrid.Lfm2(cfg, w, torch.float32, "cuda:0", arena_rows=4096), cfg)
            err = max((o - whole).abs().max().item() for o in outs)
        dist.barrier()
        q.put((rank, err))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_lfm2_kv_head_split_matches_unsplit():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
        assert p.exitcode == 0
    res = dict(q.get(timeout=10) for _ in range(2))
    assert res[0] is not None and res[0] < 1e-4, res


def _rank_fused(rank, world, port, q):
    """bf16: the split engine with the fused head gather (attention epilogue
    stores into every rank's buffer over NVLink) against the same split
    engine with the NCCL all-gather: same kernels, same bits.  The token
    split with the residual stream over NVLink peer stores agrees with the
    NCCL token split to bf16 noise, and its prefill chunks replayed from
    CUDA graphs (device-side epochs) match its eager chunks bit for bit."""
    import torch.distributed as dist
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    from datetime import timedelta
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                            timeout=timedelta(seconds=60))
    gathers = []
    try:
        from cev_b200 import configs, hybrid, ops, weights
        from cev_b200.tp import KvHeadSplit
        cfg = configs.tiny_lfm2()
        w = weights.init_weights(cfg, 42)
        D = cfg.get("head_dim") or cfg["hidden_size"] // cfg["num_attention_heads"]
        dev = f"cuda:{rank}"

        def run(fused, token_split, graphs=False):
            sp = KvHeadSplit(cfg["num_attention_heads"], cfg["num_key_value_heads"], D, rank, world)
            sp.sequence_parallel = token_split
            if fused:
                gathers.append(sp.enable_fused_gather(1024, dev, hidden=cfg["hidden_size"] if token_split else 0))
            out = _run(hybrid.Lfm2(cfg, w, torch.bfloat16, dev, arena_rows=4096, split=sp), cfg, graphs)
            ops.device_status()
            return out

        nccl, got = run(False, False), run(True, False)
        nccl_ts, fused_ts, graph_ts = run(False, True), run(True, True), run(True, True, graphs=True)
        q.put((rank, (got - nccl).abs().max().item(), (fused_ts - nccl_ts).abs().max().item(),
               (graph_ts - fused_ts).abs().max().item(), (nccl_ts - nccl).abs().max().item(),
               min(g.epoch for g in gathers)))
    finally:
        for g in gathers:
            g.close()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_lfm2_fused_head_gather_matches_nccl_gather():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rank_fused, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
        assert p.exitcode == 0
    res = {v[0]: v[1:] for v in (q.get(timeout=10) for _ in range(2))}
    for r in (0, 1):
        err, err_ts, err_graph, err_split, epochs = res[r]
        assert epochs > 0 and err == 0.0 and err_graph == 0.0, res
        # token split vs not, and peer-store vs NCCL token split (the latter
        # recomputes the conv tails on every rank, the former ships the conv
        # kernel's): same math, other GEMM shapes (bf16)
        assert err_split < 0.1 and err_ts < 0.1, res


def _rank_cfg5(rank, world, port, q):
    """f32, cfg5 layer shapes: the KV-head split with the token split (NCCL
    gathers) against the unsplit model, served probabilities."""
    import torch.distributed as dist
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    torch.cuda.set_device(rank)
    from datetime import timedelta
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                            timeout=timedelta(seconds=120))
    try:
        from cev_b200 import configs, hybrid, service, weights, workloads
        from cev_b200.tp import KvHeadSplit
        cfg = configs.get("cfg5")
        cfg["num_hidden_layers"] = 4
        cfg["layer_types"] = ["conv", "conv", "full_attention", "conv"]
        w = weights.init_weights(cfg, 3, torch.float32, f"cuda:{rank}")
        codes = workloads.code_ids(4)
        plen = 8192
        prefix, qs = workloads.decision_request(30_002, plen, 16, 64, 64, 4, cfg["vocab_size"] - 1)

        def served(split):
            dec = hybrid.Lfm2(cfg, w, torch.float32, f"cuda:{rank}", max_len=plen + 1024, arena_rows=plen + 4096,
                              split=split)
            eng = hybrid.HybridEngine(dec, codes, pad_id=0, prefill_chunk=512, pass_tokens=8192,
                                      prefix_cache_tokens=plen)
            return torch.tensor(service.run_debiased(eng, prefix, qs, "none", codes, workloads.SEP_ID)[1])

        D = cfg.get("head_dim") or cfg["hidden_size"] // cfg["num_attention_heads"]
        sp = KvHeadSplit(cfg["num_attention_heads"], cfg["num_key_value_heads"], D, rank, world)
        sp.sequence_parallel = True
        got = served(sp)
        err = None
        if rank == 0:
            err = (got - served(None)).abs().max().item()
        dist.barrier()
        q.put((rank, err))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_lfm2_token_split_cfg5_shape_served_probabilities():
    """cfg5 layer shapes (hidden 2048, 32 Q / 8 KV heads, head_dim 64, conv
    kernel 3; conv, conv, attention, conv), an 8192-token state in 512-token
    chunks and 16 questions as right-padded rows, f32: the KV-head split with
    the token-local layers on each rank's token rows serves the unsplit
    model's probabilities within 5e-5."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rank_cfg5, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(600)
        assert p.exitcode == 0
    res = dict(q.get(timeout=10) for _ in range(2))
    assert res[0] is not None and res[0] < 5e-5, res
