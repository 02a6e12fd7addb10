"""The KV-head-group split of the attention layers (cev_b200.tp) on two
gloo ranks on CPU: each rank projects and attends its heads with the
oracle's attention (qwen3.rs:206-220 / lfm2.rs:145-171 math), the all-gather
of head outputs must rebuild the unsplit layer's context exactly."""
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import ops as ref


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _layer(hq, hkv, D, H, T, P, seed):
    g = torch.Generator().manual_seed(seed)
    w = torch.randn((hq + 2 * hkv) * D, H, generator=g) * 0.1
    h = torch.randn(P + T, H, generator=g)
    return w, h


def _attend(w, h, hq, hkv, D, P, T):
    """Project, then queries of the last T tokens attend the P prefix rows
    in full and themselves causally (one segment)."""
    x = h @ w.T
    q = x[P:, :hq * D].reshape(T, hq, D).transpose(0, 1)[None]
    k = x[:, hq * D:(hq + hkv) * D].reshape(P + T, hkv, D).transpose(0, 1)[None]
    v = x[:, (hq + hkv) * D:].reshape(P + T, hkv, D).transpose(0, 1)[None]
    o = ref.attend(q, k, v, ref.causal_mask(T, P))
    return o[0].transpose(0, 1).reshape(T, hq * D)


def _rank(rank, world, port, q):
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from cev_b200.tp import KvHeadSplit
        hq, hkv, D, H, T, P = 8, 4, 16, 32, 7, 5
        w, h = _layer(hq, hkv, D, H, T, P, 3)
        sp = KvHeadSplit(hq, hkv, D, rank, world)
        local = _attend(sp.slice_fused_qkv(w), h, sp.hq_l, sp.hkv_l, D, P, T)
        full = sp.gather(local)
        want = _attend(w, h, hq, hkv, D, P, T)
        q.put((rank, (full - want).abs().max().item(), tuple(full.shape)))
    finally:
        dist.destroy_process_group()


def test_kv_head_split_gather_rebuilds_the_unsplit_context():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    res = sorted(q.get(timeout=10) for _ in range(world))
    for rank, err, shape in res:
        assert shape == (7, 8 * 16)
        assert err < 1e-6, (rank, err)


def test_kv_head_split_rejects_uneven_groups():
    import pytest
    from cev_b200.tp import KvHeadSplit
    with pytest.raises(ValueError):
        KvHeadSplit(8, 4, 16, 0, 3)


def _rank_rows(rank, world, port, q):
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from cev_b200.tp import KvHeadSplit
        sp = KvHeadSplit(8, 4, 16, rank, world)
        errs = []
        for n in (6, 5, 1):  # even, uneven, fewer rows than ranks
            want = torch.arange(n * 3, dtype=torch.float32).reshape(n, 3)
            unit = -(-n // world)
            a, b = min(n, rank * unit), min(n, (rank + 1) * unit)
            x = torch.full((n, 3), -1.0)
            x[a:b] = want[a:b]  # only this rank's rows are valid before the gather
            sp.gather_rows(x, a, b, unit)
            errs.append((x - want).abs().max().item())
        q.put((rank, errs))
    finally:
        dist.destroy_process_group()


def test_token_rows_gather_rebuilds_the_stream():
    """KvHeadSplit.gather_rows: each rank's token rows (contiguous runs of
    ceil(n / world), the last ones short or empty) rebuild the whole
    residual stream on every rank."""
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rank_rows, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    for rank, errs in sorted(q.get(timeout=10) for _ in range(world)):
        assert errs == [0.0] * 3, (rank, errs)
