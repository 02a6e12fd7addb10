"""Failure detection on the multi-rank path, on gloo ranks on the CPU (no
GPU is faulted or hung): a rank that leaves between steps, one that dies
without saying so, and one that is only slow (cev_b200.health).  The
survivors learn of a lost peer on the host, before their next step's
collective, and abort the group; a collective a peer never joins ends with
the process group's short timeout instead of hanging.  The reference's
closest behaviour is the server failing a request whose worker panicked
(crates/cev-server/src/lib.rs:58-62)."""
import os
import socket
import time

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q, scenario, deadline):
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    from cev_b200 import health
    health.init_distributed("gloo", rank, world, timeout_s=5.0)
    gate = health.StepGate(rank, world, deadline_s=deadline)
    done = []
    try:
        for step in range(1, 4):
            if rank == 1 and step == 3 and scenario == "leave":
                gate.leave()  # between steps, nothing in flight
                q.put((rank, "left", done, 0.0))
                dist.destroy_process_group()
                return
            if rank == 1 and step == 2 and scenario == "die":
                os._exit(3)  # no goodbye
            if rank == 1 and step == 2 and scenario == "slow":
                time.sleep(0.5)
            t0 = time.monotonic()
            try:
                gate.enter(step)
            except health.PeerLost as e:
                q.put((rank, "lost", e.ranks, time.monotonic() - t0))
                health.abort()
                return
            x = torch.full((4,), float(rank + step))
            dist.all_reduce(x)
            done.append(x[0].item())
        q.put((rank, "ok", done, 0.0))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def _run(scenario, deadline, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q, scenario, deadline)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(60)
    codes = [p.exitcode for p in procs]
    out = {}
    while not q.empty():
        r, what, data, dt = q.get(timeout=5)
        out[r] = (what, data, dt)
    return codes, out


def test_rank_leaving_between_steps_is_seen_before_the_next_step():
    codes, out = _run("leave", deadline=20.0)
    assert codes == [0, 0]
    assert out[1][0] == "left" and out[1][1] == [1.0 + 2.0, 2.0 + 3.0]
    what, ranks, dt = out[0]
    assert what == "lost" and ranks == [1]
    assert dt < 5.0  # seen from the store, long before the 20 s deadline


def test_rank_dying_without_a_word_misses_the_deadline():
    codes, out = _run("die", deadline=1.5)
    assert codes[1] == 3 and codes[0] == 0
    what, ranks, dt = out[0]
    assert what == "lost" and ranks == [1]
    assert 1.5 <= dt < 6.0


def test_slow_rank_within_the_deadline_is_waited_for():
    codes, out = _run("slow", deadline=20.0)
    assert codes == [0, 0]
    for r in (0, 1):
        assert out[r][0] == "ok" and out[r][1] == [3.0, 5.0, 7.0]


def _silent_peer(rank, world, port, q):
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    from cev_b200 import health
    health.init_distributed("gloo", rank, world, timeout_s=2.0)
    if rank == 1:
        time.sleep(8.0)  # never joins the collective, exits later
        q.put((rank, "slept", 0.0))
        return
    t0 = time.monotonic()
    try:
        dist.all_reduce(torch.ones(4))
        q.put((rank, "returned", time.monotonic() - t0))
    except RuntimeError:
        q.put((rank, "timed out", time.monotonic() - t0))


def test_collective_a_peer_never_joins_ends_with_the_group_timeout():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_silent_peer, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(60)
    res = {}
    while not q.empty():
        r, what, dt = q.get(timeout=5)
        res[r] = (what, dt)
    assert res[0][0] == "timed out" and res[0][1] < 7.0, res
