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

    def gather(self, ctx: torch.Tensor) -> torch.Tensor:
        """``[T, Hq/world * D]`` per rank -> ``[T, Hq * D]`` in head order
        (one all-gather; NCCL on GPUs, gloo on CPU)."""
        T = ctx.shape[0]
        out = torch.empty(self.world * T, ctx.shape[1], dtype=ctx.dtype, device=ctx.device)
        dist.all_gather_into_tensor(out, ctx.contiguous(), group=self.group)
        return out.view(self.world, T, -1).transpose(0, 1).reshape(T, -1)
