"""Channel- and time-sharded scans across GPUs (one process per GPU, NCCL over NVLink).

Every (batch, channel) recurrence of the scan is independent, so a long
sequence is split over GPUs by channel: rank r holds channels
[r*Dl, (r+1)*Dl) of delta, Lambda, S and D plus the shared B/C, scans them
locally (time-parallel when the shard is too narrow to fill the GPU), and one
all-gather over the process group returns the full output to every rank. There
is no exchange inside the scan; the all-gather is the only collective.

A sequence can also be split by time (``ssm_scan_cayley_time_sharded``): rank r
holds time range r of every input. The scan is affine in the state, so each
rank first summarises its range as h -> P (x) h + E (a state-only pass from
zero), the ranks all-gather the summaries (2 x B*D*N quaternions each, a few
MB), every rank folds the summaries of the ranks before it into its start
state, and then scans its range from that state. y stays time-sharded; the
final state of the whole sequence is known on every rank.
"""

from __future__ import annotations

import ctypes
from typing import Callable

import torch
import torch.distributed as dist

__all__ = ["channel_shard", "time_shard", "ssm_scan_cayley_channel_sharded",
           "ssm_scan_cayley_time_sharded", "PeerOutput", "channel_push"]


class _CudaArray:
    """A device buffer presented through __cuda_array_interface__ (zero copy)."""

    # bf16 is exposed as int16 and reinterpreted by the caller
    _TYPESTR = {torch.float32: "<f4", torch.bfloat16: "<i2"}

    def __init__(self, ptr: int, shape: tuple, dtype: torch.dtype):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": self._TYPESTR[dtype],
                                         "data": (ptr, False), "version": 3, "strides": None}


class PeerOutput:
    """One output buffer per rank that every rank of the group can write.

    Each rank allocates ``shape`` x ``dtype`` with ``mqc_peer_alloc`` and the
    ranks exchange the IPC handles (an all-gather of 64-byte objects), so
    ``ptrs[r]`` addresses rank r's buffer from this process (peer memory over
    NVLink for r != rank). ``tensor`` is this rank's own buffer as a torch
    tensor. The buffers live until ``close()``.
    """

    def __init__(self, shape: tuple, dtype: torch.dtype, device: torch.device, group=None):
        from .. import _lib
        lib = _lib.load()
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.shape, self.dtype = tuple(shape), dtype
        nbytes = 1
        for n in shape:
            nbytes *= int(n)
        nbytes *= torch.empty((), dtype=dtype).element_size()
        with torch.cuda.device(device):
            own = ctypes.c_void_p()
            handle = ctypes.create_string_buffer(_lib.MQC_PEER_HANDLE_BYTES)
            _lib.check(lib.mqc_peer_alloc(nbytes, ctypes.byref(own), handle), "mqc_peer_alloc")
            handles = [None] * self.world
            dist.all_gather_object(handles, handle.raw, group=group)
            self._own = own.value
            self._opened = []
            ptrs = []
            for r, h in enumerate(handles):
                if r == self.rank:
                    ptrs.append(self._own)
                    continue
                peer = ctypes.c_void_p()
                hb = ctypes.create_string_buffer(h, _lib.MQC_PEER_HANDLE_BYTES)
                _lib.check(lib.mqc_peer_open(hb, ctypes.byref(peer)), "mqc_peer_open")
                self._opened.append(peer.value)
                ptrs.append(peer.value)
        self.ptrs = ptrs
        self.tensor = torch.as_tensor(_CudaArray(self._own, shape, dtype), device=device)
        if dtype == torch.bfloat16:
            self.tensor = self.tensor.view(torch.bfloat16)

    def close_peers(self) -> None:
        """Unmaps the other ranks' buffers."""
        from .. import _lib
        lib = _lib.load()
        for ptr in self._opened:
            lib.mqc_peer_close(ptr)
        self._opened = []

    def close(self) -> None:
        """Unmaps the peers' buffers and frees this rank's own. Every rank that
        mapped this rank's buffer must have unmapped it first."""
        from .. import _lib
        lib = _lib.load()
        self.close_peers()
        self.tensor = None
        if self._own is not None:
            lib.mqc_peer_free(self._own)
            self._own = None


def channel_push(src: torch.Tensor, dst_ptrs: list[int], seq_total: int, ch_total: int,
                 ch_off: int, t_off: int, stream=None) -> None:
    """Writes src [B, seg, Dl, 4] into rows t_off.. and channels ch_off.. of every
    destination [B, seq_total, ch_total, 4] (device addresses, local or peer)
    with ``mqc_channel_push`` on ``stream`` (default: the current stream)."""
    from .. import _lib
    bsz, seg, dl = src.shape[:3]
    arr = (ctypes.c_void_p * len(dst_ptrs))(*dst_ptrs)
    st = stream if stream is not None else torch.cuda.current_stream(src.device)
    _lib.call("mqc_channel_push", src.data_ptr(), arr, len(dst_ptrs), bsz, seg, dl, ch_total,
              ch_off, t_off, seq_total, _lib.dtype_code(src), st.cuda_stream)


_peer_outputs: dict = {}


def _peer_output(shape, dtype, device, group) -> PeerOutput:
    key = (tuple(shape), dtype, str(device), id(group))
    out = _peer_outputs.get(key)
    if out is None:
        out = _peer_outputs[key] = PeerOutput(shape, dtype, device, group)
    return out


def release_peer_outputs() -> None:
    """Closes every cached PeerOutput. Collective: every rank of each buffer's
    group calls it, before the process group is destroyed. Ranks first unmap
    their peers' buffers, then (after a barrier) free their own."""
    _mc_outputs.clear()
    if not _peer_outputs:
        return
    torch.cuda.synchronize()
    groups = {id(o.group): o.group for o in _peer_outputs.values()}
    for out in _peer_outputs.values():
        out.close_peers()
    for g in groups.values():
        dist.barrier(group=g)
    for out in _peer_outputs.values():
        out.close()
    _peer_outputs.clear()


def channel_shard(t: torch.Tensor, rank: int, world: int, dim: int) -> torch.Tensor:
    """The rank's equal slice of ``t`` along the channel dimension ``dim``."""
    n = t.shape[dim]
    if n % world:
        raise ValueError(f"{n} channels do not split evenly over {world} ranks")
    k = n // world
    return t.narrow(dim, rank * k, k)


def time_shard(t: torch.Tensor, rank: int, world: int, dim: int = 1) -> torch.Tensor:
    """The rank's equal slice of ``t`` along the time dimension ``dim``."""
    return channel_shard(t, rank, world, dim)


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
                                    segments: int = 1, gather: str = "nccl") -> torch.Tensor:
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

    ``gather="peer"`` (CUDA, ranks on one node): instead of the collective
    library's all-gather and a permute of its rank-major result, y is written
    straight into its channel columns of every rank's output buffer
    (``PeerOutput``, CUDA IPC) over NVLink. With channel-shared B/C and the
    default scan this happens inside the scan kernel itself
    (``mqc_ssm_scan_fwd_chunked_peer``: every y value is stored to all ranks'
    buffers as it is produced, and ``segments`` is not needed); otherwise each
    scanned segment is pushed by ``mqc_channel_push`` on a side stream under
    the next segment's scan. Two one-element all-reduces on the compute stream
    order the exchange: one on entry (every rank is done with the previous
    result before it is overwritten) and one on exit (every store has landed).
    The returned tensor is this rank's peer buffer, valid until the next call
    with the same shape.

    ``gather="multicast"`` (CUDA, NVSwitch with NVLink SHARP): the output is a
    symmetric-memory tensor bound to a multicast object on every rank, and the
    scan kernel stores each y quaternion once, with ``multimem.st`` to the
    multicast address (``mqc_ssm_scan_fwd_chunked_multicast``); the switch
    writes it into every rank's buffer. Needs the fused conditions above,
    d_state > 16 and a platform with multicast (else RuntimeError). Measured on
    config 5 at 2 GPUs it is much slower than ``"peer"`` (60.2 ms per step
    against 12.7 ms): one 8- or 16-byte multimem store per channel and step is
    far below the transfer size the switch's multicast serves well.
    """
    # the scan kernel itself writes every rank's output: channel-shared B/C, the
    # default scan, a per-channel skip weight, inputs that need no gradient
    fused_peer = (scan_fn is None and B.dim() == 4 and D.dim() == 1 and
                  not (torch.is_grad_enabled() and any(
                      t.requires_grad for t in (delta, Lambda, B, C, S, D))))
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
    if gather == "multicast":
        if not on_cuda:
            raise ValueError("gather='multicast' needs CUDA tensors")
        ds = Lambda.shape[1]
        mc = None
        if fused_peer and 16 < ds <= 256:
            mc = _mc_output((bsz, seqlen, world * dl, 4), delta.dtype, delta.device, group)
        if mc is None or not mc.mc_ptr:
            raise RuntimeError("gather='multicast': no multicast support on this platform, or "
                               "not the fused form (channel-shared B/C, d_state > 16, no grad)")
        return _channel_sharded_mc_fused(delta, Lambda, B, C, S, D, group, time_chunks, mc)
    if gather == "peer":
        if not on_cuda:
            raise ValueError("gather='peer' needs CUDA tensors")
        if fused_peer:
            return _channel_sharded_peer_fused(delta, Lambda, B, C, S, D, group, time_chunks)
        return _channel_sharded_peer(delta, Lambda, B, C, S, D, group, scan_fn, segments)
    if gather != "nccl":
        raise ValueError(f"gather must be 'nccl', 'peer' or 'multicast', got {gather!r}")
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


def _channel_sharded_peer(delta, Lambda, B, C, S, D, group, scan_fn, segments):
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    bsz, seqlen, dl = delta.shape[:3]
    seg = seqlen // segments
    dev = delta.device
    out = _peer_output((bsz, seqlen, world * dl, 4), delta.dtype, dev, group)
    flag = _barrier_flag(dev)
    compute = torch.cuda.current_stream(dev)
    comm = _side_stream(dev)
    dist.all_reduce(flag, group=group)  # every rank is done with the previous result
    comm.wait_stream(compute)
    h = None
    for k in range(segments):
        sl = slice(k * seg, (k + 1) * seg)
        yk, h = scan_fn(delta[:, sl], Lambda, B[:, sl], C[:, sl], S[:, sl], D, h)
        yk = yk.contiguous()
        done = torch.cuda.Event()
        done.record(compute)
        comm.wait_event(done)
        channel_push(yk, out.ptrs, seqlen, world * dl, rank * dl, k * seg, stream=comm)
        yk.record_stream(comm)
    compute.wait_stream(comm)
    dist.all_reduce(flag, group=group)  # every rank's pushes have completed
    return out.tensor


def _channel_sharded_peer_fused(delta, Lambda, B, C, S, D, group, time_chunks):
    from .ssm_fused import _run_scan_chunked, auto_time_chunks
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    bsz, seqlen, dl = delta.shape[:3]
    ds = Lambda.shape[1]
    dev = delta.device
    nc = (auto_time_chunks(bsz, seqlen, dl, ds, dev) if time_chunks == "auto"
          else int(time_chunks))
    if nc > 1 and seqlen // nc <= 8:
        nc = 1
    out = _peer_output((bsz, seqlen, world * dl, 4), delta.dtype, dev, group)
    flag = _barrier_flag(dev)
    dist.all_reduce(flag, group=group)  # every rank is done with the previous result
    _run_scan_chunked(delta, Lambda, B, C, S, D, None, 1e-6, nc, False,
                      peer=(out.ptrs, world * dl, rank * dl))
    dist.all_reduce(flag, group=group)  # every rank's stores have landed
    return out.tensor


class McOutput:
    """A [B, T, channels, 4] output in symmetric memory on every rank of ``group``
    (``torch.distributed._symmetric_memory``), with the multicast address of the
    buffer set when the platform supports NVLink SHARP multicast (``mc_ptr``,
    0 otherwise). ``tensor`` is this rank's buffer."""

    def __init__(self, shape: tuple, dtype: torch.dtype, device: torch.device, group=None):
        import torch.distributed._symmetric_memory as symm
        self.group = group
        self.tensor = symm.empty(shape, dtype=dtype, device=device)
        self.handle = symm.rendezvous(self.tensor,
                                      group if group is not None else dist.group.WORLD)
        ok = bool(self.handle.has_multicast_support())
        self.mc_ptr = int(self.handle.multicast_ptr) if ok else 0


_mc_outputs: dict = {}


def _mc_output(shape, dtype, device, group) -> McOutput | None:
    key = (tuple(shape), dtype, str(device), id(group))
    out = _mc_outputs.get(key)
    if out is None:
        try:
            out = McOutput(shape, dtype, device, group)
        except Exception:  # no symmetric-memory support: callers fall back to "peer"
            out = None
        _mc_outputs[key] = out
    return out


def _channel_sharded_mc_fused(delta, Lambda, B, C, S, D, group, time_chunks, mc: McOutput):
    from .ssm_fused import _run_scan_chunked, auto_time_chunks
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    bsz, seqlen, dl = delta.shape[:3]
    ds = Lambda.shape[1]
    dev = delta.device
    nc = (auto_time_chunks(bsz, seqlen, dl, ds, dev) if time_chunks == "auto"
          else int(time_chunks))
    if nc > 1 and seqlen // nc <= 8:
        nc = 1
    flag = _barrier_flag(dev)
    dist.all_reduce(flag, group=group)  # every rank is done with the previous result
    _run_scan_chunked(delta, Lambda, B, C, S, D, None, 1e-6, nc, False,
                      peer=((mc.mc_ptr,), world * dl, rank * dl, True))
    dist.all_reduce(flag, group=group)  # every rank's stores have landed
    return mc.tensor


_flags: dict[int, torch.Tensor] = {}


def _barrier_flag(device: torch.device) -> torch.Tensor:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    f = _flags.get(idx)
    if f is None:
        f = _flags[idx] = torch.zeros(1, device=device)
    return f


def ssm_scan_cayley_time_sharded(delta: torch.Tensor, Lambda: torch.Tensor, B: torch.Tensor,
                                 C: torch.Tensor, S: torch.Tensor, D: torch.Tensor,
                                 h0: torch.Tensor | None = None, group=None,
                                 time_chunks: int | str = "auto",
                                 summary_fn: Callable | None = None,
                                 carry_fn: Callable | None = None,
                                 scan_fn: Callable | None = None):
    """Scan this rank's time range of a sequence split by time over ``group``.

    The inputs are time shards: delta [B, T/world, D], B/C [B, T/world, N, 4] (or
    per-channel), S [B, T/world, D(,4)], in rank order = time order. Lambda
    [D, N, 4] and the skip D [D] are the full tensors, held on every rank.
    h0 [B, D, N, 4] is the state before step 0, or None.

    Returns (y, h_T):
    - y [B, T/world, D, 4] is this rank's time range of the output;
    - h_T is the state after the last step of the whole sequence, the same on
      every rank.

    The only collective is one all-gather each of the range summaries P and E,
    fp32 [B, D, N, 4] per rank.

    ``summary_fn(delta, Lambda, B, C, S, D) -> (P, E)``,
    ``carry_fn(P_all, E_all, h0) -> (hin, h_T)`` and
    ``scan_fn(delta, Lambda, B, C, S, D, h0) -> (y, h_T)`` replace the GPU
    summary, carry and scan (defaults: ``ssm_scan_summary``,
    ``ssm_scan_carry`` and ``ssm_scan_cayley`` with ``time_chunks``).
    """
    from .ssm_fused import ssm_scan_carry, ssm_scan_cayley, ssm_scan_cayley_resume, ssm_scan_summary

    world = dist.get_world_size(group) if dist.is_initialized() else 1
    if summary_fn is None and scan_fn is None and world > 1:
        # GPU default: the range is summarised once, in time chunks, and its scan
        # resumes from those chunk summaries (one state-only pass in total)
        rank = dist.get_rank(group)
        summ = ssm_scan_summary(delta, Lambda, B, C, S, D, time_chunks=time_chunks,
                                keep_chunks=True)
        P_all, E_all = _gather_summaries(summ.P, summ.E, world, group)
        hin, hT = (carry_fn or ssm_scan_carry)(P_all, E_all, h0)
        y = ssm_scan_cayley_resume(delta, Lambda, B, C, S, D, summ, h0=hin[rank])
        return y, hT

    if summary_fn is None:
        def summary_fn(d, L, Bm, Cm, s, Dk):
            return ssm_scan_summary(d, L, Bm, Cm, s, Dk, time_chunks=time_chunks)
    if carry_fn is None:
        carry_fn = ssm_scan_carry
    if scan_fn is None:
        def scan_fn(d, L, Bm, Cm, s, Dk, hs=None):
            return ssm_scan_cayley(d, L, Bm, Cm, s, Dk, h0=hs, return_final_state=True,
                                   time_chunks=time_chunks)

    if world == 1:
        return scan_fn(delta, Lambda, B, C, S, D, h0)
    rank = dist.get_rank(group)
    P, E = summary_fn(delta, Lambda, B, C, S, D)
    P_all, E_all = _gather_summaries(P, E, world, group)
    hin, hT = carry_fn(P_all, E_all, h0)
    y, _ = scan_fn(delta, Lambda, B, C, S, D, hin[rank])
    return y, hT


def _gather_summaries(P: torch.Tensor, E: torch.Tensor, world: int, group):
    """All-gather of every rank's range summary: ([world, ...], [world, ...])."""
    P_all = torch.empty((world,) + tuple(P.shape), dtype=P.dtype, device=P.device)
    E_all = torch.empty_like(P_all)
    dist.all_gather_into_tensor(P_all.view(world * P.shape[0], *P.shape[1:]), P.contiguous(),
                                group=group)
    dist.all_gather_into_tensor(E_all.view(world * E.shape[0], *E.shape[1:]), E.contiguous(),
                                group=group)
    return P_all, E_all
