"""Channel-sharded scan across GPUs (one process per GPU, NCCL over NVLink).

Every (batch, channel) recurrence of the scan is independent, so a long
sequence is split over GPUs by channel: rank r holds channels
[r*Dl, (r+1)*Dl) of delta, Lambda, S and D plus the shared B/C, scans them
locally (time-parallel when the shard is too narrow to fill the GPU), and one
all-gather over the process group returns the full output to every rank. There
is no exchange inside the scan; the all-gather is the only collective.
"""

from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist

__all__ = ["channel_shard", "ssm_scan_cayley_channel_sharded"]


def channel_shard(t: torch.Tensor, rank: int, world: int, dim: int) -> torch.Tensor:
    """The rank's equal slice of ``t`` along the channel dimension ``dim``."""
    n = t.shape[dim]
    if n % world:
        raise ValueError(f"{n} channels do not split evenly over {world} ranks")
    k = n // world
    return t.narrow(dim, rank * k, k)


def ssm_scan_cayley_channel_sharded(delta: torch.Tensor, Lambda: torch.Tensor, B: torch.Tensor,
                                    C: torch.Tensor, S: torch.Tensor, D: torch.Tensor,
                                    group=None, time_chunks: int | str = "auto",
                                    scan_fn: Callable | None = None) -> torch.Tensor:
    """Scan this rank's channel shard and all-gather y over ``group``.

    delta [B,T,Dl], Lambda [Dl,N,4], S [B,T,Dl] or [B,T,Dl,4], D [Dl] are this
    rank's shard (rank order = channel order); B/C are the full shared
    [B,T,N,4] (or the rank's per-channel [B,T,Dl,N,4]). Returns y [B,T,world*Dl,4]
    on every rank. ``scan_fn(delta, Lambda, B, C, S, D) -> y`` replaces the local
    scan (default: ``ssm_scan_cayley`` with ``time_chunks``).
    """
    if scan_fn is None:
        from .ssm_fused import ssm_scan_cayley

        def scan_fn(d, L, Bm, Cm, s, Dk):
            return ssm_scan_cayley(d, L, Bm, Cm, s, Dk, time_chunks=time_chunks)

    y_local = scan_fn(delta, Lambda, B, C, S, D).contiguous()
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    if world == 1:
        return y_local
    bsz, seqlen, dl, _ = y_local.shape
    # ranks' outputs concatenated along dim 0 (the form every backend accepts)
    gathered = torch.empty((world * bsz, seqlen, dl, 4), dtype=y_local.dtype,
                           device=y_local.device)
    dist.all_gather_into_tensor(gathered, y_local, group=group)
    # [G, B, T, Dl, 4] -> [B, T, G*Dl, 4]
    return gathered.view(world, bsz, seqlen, dl, 4).permute(1, 2, 0, 3, 4).reshape(
        bsz, seqlen, world * dl, 4)
