"""KV-head-group split of the attention layers across ranks.

The long-prefix LFM2 case (a 64k-token state) spreads its attention layers
over the GPUs of one node: rank r holds, projects and attends only its group
of KV heads and the query heads that read them, with a KV arena of those
heads alone; one all-gather of the per-head outputs rebuilds the
``[T, Hq * D]`` context the (replicated) output projection reads.  The other
layers run whole on every rank, so every rank ends each layer with the same
activations.  Query head h reads KV head ``h // (Hq / Hkv)`` (lfm2.rs:145-171
via ``repeat_kv``), so contiguous head ranges keep GQA groups whole.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


class KvHeadSplit:
    """Rank ``rank`` of ``world`` owns KV heads ``[rank * Hkv/world, ...)``
    and query heads ``[rank * Hq/world, ...)``."""

    def __init__(self, hq: int, hkv: int, head_dim: int, rank: int, world: int, group=None):
        if world < 1 or hkv % world or hq % hkv:
            raise ValueError(f"{hkv} KV heads do not split over {world} ranks")
        self.hq, self.hkv, self.D = hq, hkv, head_dim
        self.rank, self.world, self.group = rank, world, group
        self.hq_l, self.hkv_l = hq // world, hkv // world
        self.q0, self.kv0 = rank * self.hq_l, rank * self.hkv_l
        self.fused = None  # a FusedHeadGather once enable_fused_gather ran
        # token-local layers on this rank's token rows only, the residual
        # stream all-gathered after each layer (False: every rank runs them
        # on every token)
        self.sequence_parallel = False

    def enable_fused_gather(self, max_tokens: int, device, hidden: int = 0) -> "FusedHeadGather":
        """Gather head outputs from the attention epilogue over NVLink peer
        memory instead of the NCCL all-gather (bf16 models); with ``hidden``
        also the residual stream of the token split (``max_tokens`` rows of
        that width) over peer stores instead of NCCL."""
        self.fused = FusedHeadGather(self, max_tokens, device, self.group, hidden=hidden)
        return self.fused

    def slice_fused_qkv(self, w: torch.Tensor) -> torch.Tensor:
        """Rows of a fused ``q | k | v`` projection weight ``[(Hq + 2 Hkv) D,
        H]`` that this rank computes, in the same q | k | v order."""
        D = self.D
        q = w[self.q0 * D:(self.q0 + self.hq_l) * D]
        k0 = (self.hq + self.kv0) * D
        v0 = (self.hq + self.hkv + self.kv0) * D
        k = w[k0:k0 + self.hkv_l * D]
        v = w[v0:v0 + self.hkv_l * D]
        return torch.cat([q, k, v], 0).contiguous()

    def gather_rows(self, x: torch.Tensor, a: int, b: int, unit: int) -> None:
        """x [n, H]: every rank r's rows [r * unit, min(n, (r + 1) * unit)),
        this rank's being [a, b), gathered into x on every rank (one
        all-gather; in place when n = world * unit)."""
        n, H = x.shape
        if n == self.world * unit and x.is_cuda:  # NCCL gathers in place
            dist.all_gather_into_tensor(x, x[a:b], group=self.group)
            return
        send = x.new_zeros(unit, H)
        send[:b - a] = x[a:b]
        out = x.new_empty(self.world * unit, H)
        dist.all_gather_into_tensor(out, send, group=self.group)
        x.copy_(out[:n])

    def broadcast(self, t: torch.Tensor, src: int) -> None:
        """t from rank ``src`` to every rank, in place."""
        dist.broadcast(t, src, group=self.group)

    def gather(self, ctx: torch.Tensor) -> torch.Tensor:
        """``[T, Hq/world * D]`` per rank -> ``[T, Hq * D]`` in head order
        (one all-gather; NCCL on GPUs, gloo on CPU)."""
        T = ctx.shape[0]
        out = torch.empty(self.world * T, ctx.shape[1], dtype=ctx.dtype, device=ctx.device)
        dist.all_gather_into_tensor(out, ctx.contiguous(), group=self.group)
        return out.view(self.world, T, -1).transpose(0, 1).reshape(T, -1)


class _DeviceView:
    """A raw device allocation seen by torch through __cuda_array_interface__
    (int16 elements, viewed as bf16 by the caller)."""

    def __init__(self, ptr: int, shape):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": "<i2", "data": (ptr, False),
                                         "version": 3, "strides": None}


class FusedHeadGather:
    """The head all-gather of a :class:`KvHeadSplit` fused into the
    attention epilogue (bf16): each rank's attention call stores its heads'
    output rows straight into every rank's gathered ``[T, Hq * D]`` buffer
    over NVLink (CUDA IPC peer pointers, no multicast), raises its epoch
    flag in every rank's flag array, and waits until every rank's flag in
    its own array has reached the epoch; the replicated output projection
    then reads the local buffer.  Two buffers alternate by epoch parity.
    Every rank must make the same sequence of ``attend`` calls."""

    def __init__(self, split: KvHeadSplit, max_tokens: int, device, group=None, limit_cycles: int = 1 << 31,
                 hidden: int = 0):
        import ctypes as C

        from ._lib import check, lib
        self.split, self.world, self.rank = split, split.world, split.rank
        self.width = split.hq * split.D
        self.max_tokens = max_tokens
        self.buf_bytes = max_tokens * self.width * 2
        # residual-stream rows of the token split: two buffers (layer parity)
        self.hidden = hidden
        self.row_bytes = max_tokens * hidden * 2
        self.row_off = 2 * self.buf_bytes
        # flags [world] int32, then this rank's epoch counter (device side:
        # the signal kernel advances it, so graph replays get new epochs)
        self.flag_off = self.row_off + 2 * self.row_bytes
        self.ctr_off = self.flag_off + 128
        self.limit = limit_cycles
        self.epoch = 0  # host count of gathers: picks the head buffer by parity
        self.device = torch.device(device)
        ptr = C.c_void_p()
        check(lib().cevk_ipc_alloc(self.flag_off + 256, C.byref(ptr)))
        self.own = ptr.value
        handle = (C.c_char * 64)()
        check(lib().cevk_ipc_handle(C.c_void_p(self.own), handle))
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self.bases, self.opened = [], []
        for i, hb in enumerate(handles):
            if i == self.rank:
                self.bases.append(self.own)
                continue
            p = C.c_void_p()
            check(lib().cevk_ipc_open((C.c_char * 64).from_buffer_copy(hb), C.byref(p)))
            self.bases.append(p.value)
            self.opened.append(p.value)
        self.flag_ptrs = (C.c_void_p * self.world)(*[b + self.flag_off for b in self.bases])
        self.views = [torch.as_tensor(_DeviceView(self.own + k * self.buf_bytes, (max_tokens, self.width)),
                                      device=self.device).view(torch.bfloat16) for k in (0, 1)]
        self.rows = [torch.as_tensor(_DeviceView(self.own + self.row_off + k * self.row_bytes, (max_tokens, hidden)),
                                     device=self.device).view(torch.bfloat16) for k in (0, 1)] if hidden else []
        self.ctr = C.c_void_p(self.own + self.ctr_off)
        self.ticket = C.c_void_p(self.own + self.ctr_off + 64)  # the row gather's last-block ticket
        self.own_flags = C.c_void_p(self.own + self.flag_off)
        self.group = group

    def _signal_wait(self, s) -> None:
        from ._lib import check, lib
        self.epoch += 1
        check(lib().cevk_gather_sync_dev(self.flag_ptrs, self.world, self.rank, self.ctr, self.own_flags, self.limit,
                                         s))

    def gather_rows(self, k: int, a: int, b: int, n: int) -> torch.Tensor:
        """Rows [a, b) of this rank's residual buffer k stored into every
        rank's buffer 1 - k over NVLink, then the epoch handshake: returns
        this rank's buffer 1 - k, [n, hidden], complete.  (Buffers alternate
        by layer: a peer writes layer l's rows into buffer 1 - k only after
        every rank signalled layer l - 1, i.e. finished reading it.)"""
        import ctypes as C

        from . import ops
        from ._lib import check, lib
        rb = self.hidden * 2
        a = min(a, b)
        dst = (C.c_void_p * self.world)(*[base + self.row_off + (1 - k) * self.row_bytes + a * rb
                                          for base in self.bases])
        src = C.c_void_p(self.own + self.row_off + k * self.row_bytes + a * rb)
        self.epoch += 1
        check(lib().cevk_rows_gather_dev(src, dst, self.world, (b - a) * rb, self.flag_ptrs, self.world, self.rank,
                                         self.ctr, self.own_flags, self.limit, self.ticket, ops._s()))
        return self.rows[1 - k][:n]

    def attend(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, plan, scale=None) -> torch.Tensor:
        """This rank's heads of the packed attention (q [T, Hq/world, D],
        k / v the rank's arena [S, Hkv/world, D]) gathered with every rank's:
        returns the local ``[T, Hq * D]`` rows (valid until the call after
        next)."""
        import ctypes as C
        import math

        from . import ops
        from ._lib import check, lib
        T, hq, D = q.shape
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens in one call; the gathered buffers hold {self.max_tokens}")
        if q.dtype != torch.bfloat16 or plan.n_tokens != T:
            raise ValueError("fused head gather: bf16 and a plan for these tokens")
        scale = 1.0 / math.sqrt(D) if scale is None else scale
        e = self.epoch + 1
        off = (e & 1) * self.buf_bytes + self.split.q0 * D * 2
        dst = (C.c_void_p * self.world)(*[b + off for b in self.bases])
        ws = plan.workspace
        s = ops._s()
        check(lib().cevk_attn_packed_prefill_gather(
            ops._p(q), ops._p(k), ops._p(v), dst, self.world, T, k.shape[0], hq, k.shape[1], D, q.stride(0),
            k.stride(0), self.width, ops._p(plan.dev), plan.n_segs, plan.n_tiles, scale, plan.n_split, ops._p(ws),
            0 if ws is None else ws.numel(), s))
        self._signal_wait(s)
        return self.views[e & 1][:T]

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's, once every rank is
        done writing (call on every rank)."""
        import ctypes as C

        from ._lib import check, lib
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for p in self.opened:
            check(lib().cevk_ipc_close(C.c_void_p(p)))
        self.opened = []
        dist.barrier(group=self.group)
        self.views = []
        check(lib().cevk_ipc_free(C.c_void_p(self.own)))
