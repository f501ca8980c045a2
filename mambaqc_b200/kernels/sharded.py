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


_side_streams: dict[int, torch.cuda.Stream] = {}


def _side_stream(device: torch.device) -> torch.cuda.Stream:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    st = _side_streams.get(idx)
    if st is None:
        st = _side_streams[idx] = torch.cuda.Stream(device)
    return st


def ssm_scan_cayley_channel_sharded(delta: torch.Tensor, Lambda: torch.Tensor, B: torch.Tensor,
                                    C: torch.Tensor, S: torch.Tensor, D: torch.Tensor,
                                    group=None, time_chunks: int | str = "auto",
                                    scan_fn: Callable | None = None,
                                    segments: int = 1) -> torch.Tensor:
    """Scan this rank's channel shard and all-gather y over ``group``.

    delta [B,T,Dl], Lambda [Dl,N,4], S [B,T,Dl] or [B,T,Dl,4], D [Dl] are this
    rank's shard (rank order = channel order); B/C are the full shared
    [B,T,N,4] (or the rank's per-channel [B,T,Dl,N,4]). Returns y [B,T,world*Dl,4]
    on every rank.

    ``segments`` > 1 cuts the sequence into that many equal time segments,
    scanned in order, each from the previous segment's final state; on CUDA the
    all-gather and reassembly of segment k run on a side stream while segment
    k+1 is scanned, so only the last segment's gather is exposed.

    ``scan_fn(delta, Lambda, B, C, S, D, h0) -> (y, h_T)`` replaces the local
    scan (default: ``ssm_scan_cayley`` with ``time_chunks``).
    """
    if scan_fn is None:
        from .ssm_fused import ssm_scan_cayley

        def scan_fn(d, L, Bm, Cm, s, Dk, h0=None):
            return ssm_scan_cayley(d, L, Bm, Cm, s, Dk, h0=h0, return_final_state=True,
                                   time_chunks=time_chunks)

    world = dist.get_world_size(group) if dist.is_initialized() else 1
    if world == 1:
        return scan_fn(delta, Lambda, B, C, S, D, None)[0]
    bsz, seqlen, dl = delta.shape[:3]
    if segments < 1 or seqlen % segments:
        raise ValueError(f"seq_len {seqlen} does not split into {segments} equal segments")
    seg = seqlen // segments
    on_cuda = delta.is_cuda
    y = torch.empty((bsz, seqlen, world * dl, 4), dtype=delta.dtype, device=delta.device)
    # ranks' outputs concatenated along dim 0 (the form every backend accepts),
    # double-buffered across segments
    bufs = [torch.empty((world * bsz, seg, dl, 4), dtype=delta.dtype, device=delta.device)
            for _ in range(min(2, segments))]
    if on_cuda:
        compute = torch.cuda.current_stream(delta.device)
        comm = _side_stream(delta.device)
        comm.wait_stream(compute)
    h = None
    for k in range(segments):
        sl = slice(k * seg, (k + 1) * seg)
        yk, h = scan_fn(delta[:, sl], Lambda, B[:, sl], C[:, sl], S[:, sl], D, h)
        yk = yk.contiguous()
        buf = bufs[k % len(bufs)]
        if on_cuda:
            done = torch.cuda.Event()
            done.record(compute)
            comm.wait_event(done)
            with torch.cuda.stream(comm):
                dist.all_gather_into_tensor(buf, yk, group=group)
                # [G, B, seg, Dl, 4] -> y[:, seg, G*Dl, 4] (one strided copy)
                y[:, sl].view(bsz, seg, world, dl, 4).copy_(
                    buf.view(world, bsz, seg, dl, 4).permute(1, 2, 0, 3, 4))
            yk.record_stream(comm)
        else:
            dist.all_gather_into_tensor(buf, yk, group=group)
            y[:, sl].view(bsz, seg, world, dl, 4).copy_(
                buf.view(world, bsz, seg, dl, 4).permute(1, 2, 0, 3, 4))
    if on_cuda:
        for b in bufs:
            b.record_stream(comm)
        compute.wait_stream(comm)
    return y
