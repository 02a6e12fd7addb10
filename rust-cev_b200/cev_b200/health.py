"""Host-side failure detection for the multi-GPU path.

Only the cfg5 KV-head split runs one request over several ranks; the
data-parallel configs share nothing.  The reference runs one process with
no collective; its closest behaviour is the server catching a worker's
panic and failing that request (``crates/cev-server/src/lib.rs:58-62``).
Here a rank that leaves or dies must not leave its peers blocked in a
collective or in a device wait, so:

* :func:`init_distributed` creates the process group with a short timeout
  and, for NCCL, non-blocking communicator initialisation; torch's NCCL
  watchdog polls the communicator's asynchronous error and aborts it when a
  collective outlives the timeout;
* :class:`StepGate`: before each step (a request of the split engine) every
  rank posts the step number in the process group's store and waits,
  bounded by a host deadline, until every peer has posted it.  A peer that
  posted ``left`` (it leaves between steps, with nothing in flight), or
  that misses the deadline (it died or hangs), raises :class:`PeerLost` on
  the survivors before they launch any kernel or collective of the step;
* :func:`abort` tears the communicator down (``ncclCommAbort`` through
  torch) so that the survivors can exit or form a new group.

The device side is bounded separately: the fused head gather's flag wait
gives up after its cycle limit and reports ``CEVK_E_TIMEOUT`` through
``cevk_device_status``.
"""
from __future__ import annotations

import time
from datetime import timedelta

import torch.distributed as dist


class PeerLost(RuntimeError):
    """A peer rank left or stopped answering between steps."""

    def __init__(self, msg: str, ranks):
        super().__init__(msg)
        self.ranks = sorted(ranks)


def init_distributed(backend: str, rank: int, world: int, timeout_s: float = 60.0, device=None):
    """``init_process_group`` from the usual env variables with a short
    timeout; NCCL communicators are created non-blocking (their
    initialisation errors surface on the host instead of hanging it)."""
    kw = {"backend": backend, "rank": rank, "world_size": world, "timeout": timedelta(seconds=timeout_s)}
    if backend == "nccl":
        opts = dist.ProcessGroupNCCL.Options()
        opts.config.blocking = False
        kw["pg_options"] = opts
        if device is not None:
            kw["device_id"] = device
    dist.init_process_group(**kw)


class StepGate:
    """Step-by-step liveness over the process group's key-value store."""

    LEFT = "left"

    def __init__(self, rank: int, world: int, deadline_s: float = 30.0, store=None, prefix: str = "cev/gate"):
        self.rank, self.world, self.deadline_s = rank, world, deadline_s
        self.store = store if store is not None else dist.distributed_c10d._get_default_store()
        self.prefix = prefix

    def _key(self, r: int) -> str:
        return f"{self.prefix}/{r}"

    def _peek(self, r: int):
        k = self._key(r)
        if not self.store.check([k]):
            return None
        return self.store.get(k).decode()

    def enter(self, step: int) -> None:
        """Post ``step`` and wait until every peer has reached it; raise
        :class:`PeerLost` if one left or the deadline passes."""
        self.store.set(self._key(self.rank), str(step))
        t_end = time.monotonic() + self.deadline_s
        pending = [r for r in range(self.world) if r != self.rank]
        while True:
            still, left = [], []
            for r in pending:
                v = self._peek(r)
                if v == self.LEFT:
                    left.append(r)
                elif v is None or int(v) < step:
                    still.append(r)
            if left:
                raise PeerLost(f"rank(s) {left} left before step {step}", left)
            if not still:
                return
            if time.monotonic() > t_end:
                raise PeerLost(f"rank(s) {still} did not reach step {step} within {self.deadline_s} s", still)
            pending = still
            time.sleep(0.002)

    def leave(self) -> None:
        """Tell the peers this rank is gone (call between steps, with none
        of its kernels or collectives in flight)."""
        self.store.set(self._key(self.rank), self.LEFT)


def abort(group=None) -> None:
    """Abort the process group's communicators (NCCL: ``ncclCommAbort``)
    without waiting for peers; backends without an abort are destroyed."""
    try:
        dist.distributed_c10d._abort_process_group(group)
    except Exception:
        dist.destroy_process_group(group)
