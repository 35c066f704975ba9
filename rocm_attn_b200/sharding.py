"""(batch*head) sharding of the attention forward over the ranks of one box.

Attention heads are independent, so the path partitions with no data-path
collective: rank r of N owns the contiguous flattened (b*H + h) slices
``shard_range(B*H, N, r)`` of q/k/v and produces the same slices of O.  The
only collective is the optional all-gather that assembles the full O on
every rank (used where a full tensor is needed on one rank, e.g. for
checking); it runs over NCCL (NVLink/NVSwitch) on GPUs or gloo on CPUs.
The reference has no multi-GPU code; this module is new.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch

from .workloads import shard_range


def local_view(t: torch.Tensor, world: int, rank: int) -> torch.Tensor:
    """Slices of a contiguous [B, H, L, D] tensor owned by ``rank``, as a
    [1, n_local, L, D] view (no copy)."""
    B, H, L, D = t.shape
    r = shard_range(B * H, world, rank)
    return t.reshape(1, B * H, L, D)[:, r.start:r.stop]


def gather_heads(o_local: torch.Tensor, B: int, H: int, world: int, rank: int,
                 group: Optional[object] = None) -> torch.Tensor:
    """All-gathers every rank's [1, n_r, L, D] slices into the full
    [B, H, L, D] O on every rank.  Shards may differ in size by one slice;
    they are padded to the largest for the collective and trimmed after."""
    import torch.distributed as dist

    _, n_local, L, D = o_local.shape
    sizes = [len(shard_range(B * H, world, r)) for r in range(world)]
    assert n_local == sizes[rank], "local shard does not match the partition"
    n_max = max(sizes)
    send = o_local.reshape(n_local, L, D)
    if n_local < n_max:
        pad = torch.zeros(n_max - n_local, L, D, dtype=o_local.dtype, device=o_local.device)
        send = torch.cat([send, pad], 0)
    recv = torch.empty(world * n_max, L, D, dtype=o_local.dtype, device=o_local.device)
    dist.all_gather_into_tensor(recv, send.contiguous(), group=group)
    if all(n == n_max for n in sizes):
        return recv.view(B, H, L, D)  # equal shards land in order: no copy
    parts = [recv[r * n_max:r * n_max + sizes[r]] for r in range(world)]
    return torch.cat(parts, 0).view(B, H, L, D)


def sharded_forward(attn: Callable, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool, world: int,
                    rank: int, gather: bool = False, group: Optional[object] = None,
                    scale: Optional[float] = None) -> torch.Tensor:
    """Runs ``attn`` on this rank's slices of full [B, H, L, D] tensors.
    Returns the local [1, n_local, Lq, D] output, or the full O when
    ``gather`` is set."""
    B, H = q.shape[:2]
    ql, kl, vl = (local_view(t, world, rank) for t in (q, k, v))
    o_local = attn(ql, kl, vl, causal=causal, scale=scale)
    if not gather:
        return o_local
    return gather_heads(o_local, B, H, world, rank, group=group)
