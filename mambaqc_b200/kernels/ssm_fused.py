"""Quaternion selective scan on the GPU: drop-in for ``mambaqc.kernels.ssm_fused``.

Reference functions and their replacements:

* ``ssm_step_fused(q, B, S, C, D, h_prev)`` (mambaqc/kernels/ssm_fused.py:258-337)
  -> ``mqc_ssm_step``: one step, h' = q (x) h + B (x) S, y = sum_n C (x) h' + D*S.
* ``ssm_forward_fused(q, B, S, C, D)`` (ssm_fused.py:340-401; a Python loop over
  T with one kernel launch per step) -> one ``mqc_ssm_scan_fwd`` launch with the
  state held in registers for all T steps.
* ``ssm_scan_cayley(delta, Lambda, B, C, S, D)`` -- new: the fused form of
  ``QuaternionMamba2Block._ssm_forward`` lines 214-228
  (models/quaternion_mamba2_block.py): q_t = Cayley(delta_t * Lambda) is formed
  in registers inside the scan, so neither z nor q is ever materialised.

Shapes: B batch, T seq_len, D channels (d_inner), N d_state; quaternions on the
last axis. B/C may be per-channel [B,T,D,N,4] (the reference block's layout) or
shared by all channels [B,T,N,4]; S may be a quaternion signal [B,T,D,4] or a
real one [B,T,D] (embedded as (x, 0, 0, 0), as the block does at :200-202).
The state is fp32 in registers; inputs are float32 or bfloat16 (all the same).
"""

from __future__ import annotations

import ctypes

import torch

from .. import _lib

__all__ = ["ssm_step_fused", "ssm_forward_fused", "ssm_scan_cayley", "ssm_scan_cayley_from_host"]


def _vec_align(dtype: torch.dtype) -> int:
    return 16 if dtype == torch.float32 else 8


def _prep(t: torch.Tensor, align: int) -> torch.Tensor:
    return _lib.aligned_contig(t, align)


def _skip_operand(D: torch.Tensor, bsz: int, seqlen: int, dm: int):
    """fp32 skip weights and their (b, t, d) strides; accepts [D], [B,D] or [B,T,D] (any strides)."""
    Df = D if D.dtype == torch.float32 else D.float()
    if Df.dim() == 1:
        assert Df.shape[0] == dm, f"D shape {tuple(D.shape)} vs channels {dm}"
        return Df, 0, 0, Df.stride(0)
    if Df.dim() == 2:
        assert tuple(Df.shape) == (bsz, dm), f"D shape {tuple(D.shape)}"
        return Df, Df.stride(0), 0, Df.stride(1)
    assert tuple(Df.shape) == (bsz, seqlen, dm), f"D shape {tuple(D.shape)}"
    return Df, Df.stride(0), Df.stride(1), Df.stride(2)


def _run_scan(*, flags: int, q=None, delta=None, Lam=None, B, C, S, D, h0=None,
              return_final_state=False, eps=1e-6, wait_poll_limit=-1, ckpt=None, y=None,
              hT_out=None):
    ref = q if q is not None else delta
    dt = ref.dtype
    bsz, seqlen, dm = ref.shape[0], ref.shape[1], ref.shape[2]
    shared = B.dim() == 4
    ds = B.shape[2] if shared else B.shape[3]
    s_real = S.dim() == 3
    va = _vec_align(dt)
    _lib.require_cuda(ref, B, C, S, D, h0, Lam, what="mambaqc_b200 scan")
    for name, t in (("B", B), ("C", C), ("S", S)):
        if t.dtype != dt:
            raise TypeError(f"{name} dtype {t.dtype} != {dt}")
    Bc = _prep(B, 16 if shared else va)
    Cc = _prep(C, 16 if shared else va)
    Sc = _prep(S, va)
    qc = _prep(q, va) if q is not None else None
    dc = _prep(delta, 4) if delta is not None else None
    Lc = _prep(Lam.float(), 16) if Lam is not None else None
    Df, dsb, dst, dsd = _skip_operand(D, bsz, seqlen, dm)
    h0c = _prep(h0.float(), 16) if h0 is not None else None
    if y is None:
        y = torch.empty(bsz, seqlen, dm, 4, dtype=dt, device=ref.device)
    else:
        assert y.is_contiguous() and y.dtype == dt and tuple(y.shape) == (bsz, seqlen, dm, 4)
        assert y.data_ptr() % va == 0
    if hT_out is not None:
        assert hT_out.is_contiguous() and hT_out.dtype == torch.float32
        assert tuple(hT_out.shape) == (bsz, dm, ds, 4)
        hT = hT_out
    else:
        hT = (torch.empty(bsz, dm, ds, 4, dtype=torch.float32, device=ref.device)
              if return_final_state else None)
    if shared:
        flags |= _lib.MQC_SSM_BC_SHARED
    if s_real:
        flags |= _lib.MQC_SSM_S_REAL
    status = _lib.status_word(ref.device)
    a = _lib.SsmScanArgs(
        batch=bsz, seq_len=seqlen, channels=dm, d_state=ds, dtype=_lib.dtype_code(ref),
        flags=flags, eps=float(eps), reserved0=0,
        delta=_lib.ptr(dc), lambda_=_lib.ptr(Lc), q=_lib.ptr(qc), Bm=Bc.data_ptr(),
        Cm=Cc.data_ptr(), s=Sc.data_ptr(), dskip=Df.data_ptr(), dskip_sb=dsb, dskip_st=dst,
        dskip_sd=dsd, h0=_lib.ptr(h0c), y=y.data_ptr(), hT=_lib.ptr(hT), status=status.data_ptr(),
        wait_poll_limit=int(wait_poll_limit), ckpt=_lib.ptr(ckpt),
        ckpt_every=_lib.MQC_SSM_CKPT_EVERY if ckpt is not None else 0)
    with torch.cuda.device(ref.device):
        _lib.call("mqc_ssm_scan_fwd", ctypes.byref(a), _lib.stream_ptr(ref.device))
    if _lib.sync_checks_enabled():
        _lib.check_device_status(ref.device)
    return y, hT


def _n_ckpt(seqlen: int) -> int:
    k = _lib.MQC_SSM_CKPT_EVERY
    return (seqlen + k - 1) // k - 1


def _sum_to(g: torch.Tensor, like: torch.Tensor) -> torch.Tensor:
    """Reduce a [B,T,D] skip gradient to the shape the skip weight was given in."""
    if like.dim() == 1:
        g = g.sum(dim=(0, 1))
    elif like.dim() == 2:
        g = g.sum(dim=1)
    return g.to(like.dtype)


class _SsmScanCayley(torch.autograd.Function):
    """Fused Cayley + scan with its backward (``mqc_ssm_scan_bwd``)."""

    @staticmethod
    def forward(ctx, delta, Lam, B, C, S, D, h0, eps, wait_poll_limit):
        dt = delta.dtype
        bsz, seqlen, dm = delta.shape
        ds = Lam.shape[1]
        va = _vec_align(dt)
        need_grad = any(ctx.needs_input_grad[:7])
        nck = _n_ckpt(seqlen)
        ckpt = None
        if need_grad and nck > 0:
            ckpt = torch.empty(bsz, nck, dm, ds, 4, dtype=torch.float32, device=delta.device)
        shared = B.dim() == 4
        dc = _prep(delta, 4)
        Lc = _prep(Lam.float(), 16)
        Bc = _prep(B, 16 if shared else va)
        Cc = _prep(C, 16 if shared else va)
        Sc = _prep(S, va)
        h0c = _prep(h0.float(), 16) if h0 is not None else None
        y, hT = _run_scan(flags=0, delta=dc, Lam=Lc, B=Bc, C=Cc, S=Sc, D=D, h0=h0c,
                          return_final_state=True, eps=eps, wait_poll_limit=wait_poll_limit,
                          ckpt=ckpt)
        if need_grad:
            ctx.save_for_backward(dc, Lc, Bc, Cc, Sc, D, h0c, ckpt)
        ctx.eps = eps
        ctx.meta = (Lam.dtype, None if h0 is None else h0.dtype)
        return y, hT

    @staticmethod
    def backward(ctx, gy, ghT):
        dc, Lc, Bc, Cc, Sc, D, h0c, ckpt = ctx.saved_tensors
        lam_dtype, h0_dtype = ctx.meta
        has_h0 = h0_dtype is not None
        dt = dc.dtype
        bsz, seqlen, dm = dc.shape
        ds = Lc.shape[1]
        shared = Bc.dim() == 4
        s_real = Sc.dim() == 3
        va = _vec_align(dt)
        dev = dc.device
        if gy is None:
            gy = torch.zeros(bsz, seqlen, dm, 4, dtype=dt, device=dev)
        gyc = _prep(gy.to(dt), va)
        ghTc = _prep(ghT.float(), 16) if ghT is not None else None
        Df, dsb, dst, dsd = _skip_operand(D, bsz, seqlen, dm)
        ddelta = torch.empty_like(dc)
        dlam_part = torch.empty(bsz, dm, ds, 4, dtype=torch.float32, device=dev)
        if shared:
            dB = torch.zeros(Bc.shape, dtype=torch.float32, device=dev)
            dC = torch.zeros(Cc.shape, dtype=torch.float32, device=dev)
        else:
            dB = torch.empty_like(Bc)
            dC = torch.empty_like(Cc)
        dS = torch.empty_like(Sc)
        dh0 = torch.empty(bsz, dm, ds, 4, dtype=torch.float32, device=dev) if has_h0 else None
        flags = (_lib.MQC_SSM_BC_SHARED if shared else 0) | (_lib.MQC_SSM_S_REAL if s_real else 0)
        a = _lib.SsmScanBwdArgs(
            batch=bsz, seq_len=seqlen, channels=dm, d_state=ds, dtype=_lib.dtype_code(dc),
            flags=flags, eps=float(ctx.eps), ckpt_every=_lib.MQC_SSM_CKPT_EVERY,
            delta=dc.data_ptr(), lambda_=Lc.data_ptr(), Bm=Bc.data_ptr(), Cm=Cc.data_ptr(),
            s=Sc.data_ptr(), dskip=Df.data_ptr(), dskip_sb=dsb, dskip_st=dst, dskip_sd=dsd,
            h0=_lib.ptr(h0c), ckpt=_lib.ptr(ckpt), dy=gyc.data_ptr(), dhT=_lib.ptr(ghTc),
            ddelta=ddelta.data_ptr(), dlambda_part=dlam_part.data_ptr(), dBm=dB.data_ptr(),
            dCm=dC.data_ptr(), ds=dS.data_ptr(), dh0=_lib.ptr(dh0))
        with torch.cuda.device(dev):
            _lib.call("mqc_ssm_scan_bwd", ctypes.byref(a), _lib.stream_ptr(dev))
        # skip weight: dL/dD = <dy, S> (no scan involved)
        gyf = gyc.float()
        dD_full = gyf[..., 0] * Sc.float() if s_real else (gyf * Sc.float()).sum(-1)
        return (ddelta, dlam_part.sum(0).to(lam_dtype), dB.to(dt), dC.to(dt), dS,
                _sum_to(dD_full, D), None if dh0 is None else dh0.to(h0_dtype), None, None)


def auto_time_chunks(bsz: int, seqlen: int, channels: int, d_state: int,
                     device: torch.device | None = None) -> int:
    """Number of time chunks that lets a forward scan fill the GPU.

    1 when batch * channels * d_state state lanes already cover ~2048 lanes per
    SM (config 3 has 393K lanes on 148 SMs); otherwise the smallest power of two
    that does, keeping >= 256 steps per chunk and dividing seq_len.
    """
    props = torch.cuda.get_device_properties(device if device is not None else
                                             torch.cuda.current_device())
    target = props.multi_processor_count * 2048
    lanes = bsz * channels * d_state
    nc = 1
    while lanes * nc < target and seqlen % (2 * nc) == 0 and seqlen // (2 * nc) >= 256:
        nc *= 2
    return nc


def _run_scan_chunked(delta, Lam, B, C, S, D, h0, eps, nchunks, return_final_state,
                      peer=None):
    """Time-parallel forward (``mqc_ssm_scan_fwd_chunked``); no autograd.

    ``peer = (ptrs, ch_total, ch_off[, multicast])``: the channel-sharded form
    (``mqc_ssm_scan_fwd_chunked_peer``) that writes y into every buffer of
    ``ptrs`` ([B, T, ch_total, 4], local or peer memory) at channels
    ch_off.. instead of returning it; y is then None."""
    dt = delta.dtype
    bsz, seqlen, dm = delta.shape
    ds = Lam.shape[1]
    shared = B.dim() == 4
    va = _vec_align(dt)
    dc = _prep(delta, 4)
    Lc = _prep(Lam.float(), 16)
    Bc = _prep(B, 16 if shared else va)
    Cc = _prep(C, 16 if shared else va)
    Sc = _prep(S, va)
    Df, dsb, dst, dsd = _skip_operand(D, bsz, seqlen, dm)
    if dsb != 0 or dst != 0:
        raise ValueError("time-chunked scan needs a per-channel skip weight D [D]")
    h0c = _prep(h0.float(), 16) if h0 is not None else None
    y = (torch.empty(bsz, seqlen, dm, 4, dtype=dt, device=delta.device) if peer is None
         else None)
    hT = (torch.empty(bsz, dm, ds, 4, dtype=torch.float32, device=delta.device)
          if return_final_state else None)
    lib = _lib.load()
    ws_bytes = lib.mqc_ssm_scan_fwd_chunked_workspace_size(bsz, dm, ds, nchunks)
    ws = torch.empty(max(1, ws_bytes // 4), dtype=torch.float32, device=delta.device)
    flags = (_lib.MQC_SSM_BC_SHARED if shared else 0) | (_lib.MQC_SSM_S_REAL if S.dim() == 3 else 0)
    status = _lib.status_word(delta.device)
    a = _lib.SsmScanArgs(
        batch=bsz, seq_len=seqlen, channels=dm, d_state=ds, dtype=_lib.dtype_code(dc),
        flags=flags, eps=float(eps), reserved0=0, delta=dc.data_ptr(), lambda_=Lc.data_ptr(),
        q=None, Bm=Bc.data_ptr(), Cm=Cc.data_ptr(), s=Sc.data_ptr(), dskip=Df.data_ptr(),
        dskip_sb=0, dskip_st=0, dskip_sd=dsd, h0=_lib.ptr(h0c), y=_lib.ptr(y),
        hT=_lib.ptr(hT), status=status.data_ptr(), wait_poll_limit=-1, ckpt=None, ckpt_every=0)
    with torch.cuda.device(delta.device):
        if peer is None:
            _lib.call("mqc_ssm_scan_fwd_chunked", ctypes.byref(a), int(nchunks), ws.data_ptr(),
                      ws_bytes, _lib.stream_ptr(delta.device))
        elif len(peer) == 4 and peer[3]:  # (multicast address,), ch_total, ch_off, True
            ptrs, ch_total, ch_off, _ = peer
            _lib.call("mqc_ssm_scan_fwd_chunked_multicast", ctypes.byref(a), int(nchunks),
                      ws.data_ptr(), ws_bytes, int(ptrs[0]), int(ch_total), int(ch_off),
                      _lib.stream_ptr(delta.device))
        else:
            ptrs, ch_total, ch_off = peer[:3]
            arr = (ctypes.c_void_p * len(ptrs))(*ptrs)
            _lib.call("mqc_ssm_scan_fwd_chunked_peer", ctypes.byref(a), int(nchunks),
                      ws.data_ptr(), ws_bytes, arr, len(ptrs), int(ch_total), int(ch_off),
                      _lib.stream_ptr(delta.device))
    if _lib.sync_checks_enabled():
        _lib.check_device_status(delta.device)
    return y, hT


class RangeSummary:
    """Result of ``ssm_scan_summary(..., keep_chunks=True)``: the range's P and E
    plus the per-chunk summaries (kept in ``workspace``) that
    ``ssm_scan_cayley_resume`` reuses instead of repeating the state-only pass."""

    def __init__(self, P, E, workspace, ws_bytes, nchunks):
        self.P, self.E = P, E
        self.workspace, self.ws_bytes, self.nchunks = workspace, ws_bytes, nchunks


def ssm_scan_summary(delta: torch.Tensor, Lambda: torch.Tensor, B: torch.Tensor,
                     C: torch.Tensor, S: torch.Tensor, D: torch.Tensor, eps: float = 1e-6,
                     time_chunks: int | str = "auto", keep_chunks: bool = False):
    """The affine map of a time range of the scan (no autograd).

    Over the steps of the inputs (shapes as in ``ssm_scan_cayley``) the state
    evolves as h -> P (x) h + E. Returns (P, E), both fp32 [B, D, N, 4]:
    - P = q_{T-1} (x) ... (x) q_0;
    - E = the final state reached from h = 0.

    A time-sharded scan exchanges these summaries between ranks
    (``mqc_ssm_scan_fwd_summary``). ``time_chunks`` splits the range
    time-parallel, as in ``ssm_scan_cayley``. With ``keep_chunks`` a
    ``RangeSummary`` is returned instead, for ``ssm_scan_cayley_resume``.
    """
    dt = delta.dtype
    bsz, seqlen, dm = delta.shape
    ds = Lambda.shape[1]
    shared = B.dim() == 4
    _lib.require_cuda(delta, Lambda, B, C, S, D, what="ssm_scan_summary")
    nc = (auto_time_chunks(bsz, seqlen, dm, ds, delta.device) if time_chunks == "auto"
          else int(time_chunks))
    if seqlen == 0 or seqlen % nc:
        nc = 1
    va = _vec_align(dt)
    dc = _prep(delta, 4)
    Lc = _prep(Lambda.float(), 16)
    Bc = _prep(B, 16 if shared else va)
    Cc = _prep(C, 16 if shared else va)
    Sc = _prep(S, va)
    Df, dsb, dst, dsd = _skip_operand(D, bsz, seqlen, dm)
    P = torch.empty(bsz, dm, ds, 4, dtype=torch.float32, device=delta.device)
    E = torch.empty_like(P)
    lib = _lib.load()
    ws_bytes = lib.mqc_ssm_scan_fwd_summary_workspace_size(bsz, dm, ds, nc)
    ws = torch.empty(max(4, ws_bytes // 4), dtype=torch.float32, device=delta.device)
    flags = (_lib.MQC_SSM_BC_SHARED if shared else 0) | (_lib.MQC_SSM_S_REAL if S.dim() == 3 else 0)
    status = _lib.status_word(delta.device)
    a = _lib.SsmScanArgs(
        batch=bsz, seq_len=seqlen, channels=dm, d_state=ds, dtype=_lib.dtype_code(dc),
        flags=flags, eps=float(eps), reserved0=0, delta=dc.data_ptr(), lambda_=Lc.data_ptr(),
        q=None, Bm=Bc.data_ptr(), Cm=Cc.data_ptr(), s=Sc.data_ptr(), dskip=Df.data_ptr(),
        dskip_sb=dsb, dskip_st=dst, dskip_sd=dsd, h0=None, y=None, hT=None,
        status=status.data_ptr(), wait_poll_limit=-1, ckpt=None, ckpt_every=0)
    with torch.cuda.device(delta.device):
        _lib.call("mqc_ssm_scan_fwd_summary", ctypes.byref(a), int(nc), P.data_ptr(),
                  E.data_ptr(), ws.data_ptr(), ws_bytes, _lib.stream_ptr(delta.device))
    if _lib.sync_checks_enabled():
        _lib.check_device_status(delta.device)
    if keep_chunks:
        return RangeSummary(P, E, ws, ws_bytes, nc)
    return P, E


def ssm_scan_cayley_resume(delta: torch.Tensor, Lambda: torch.Tensor, B: torch.Tensor,
                           C: torch.Tensor, S: torch.Tensor, D: torch.Tensor,
                           summary: RangeSummary, h0: torch.Tensor | None = None,
                           eps: float = 1e-6, return_final_state: bool = False):
    """``ssm_scan_cayley`` (no autograd) of the same inputs that ``summary`` was
    made from, starting from h0: only the carry and the full pass run
    (``mqc_ssm_scan_fwd_chunked_resume``), reusing the summary's chunks."""
    dt = delta.dtype
    bsz, seqlen, dm = delta.shape
    ds = Lambda.shape[1]
    shared = B.dim() == 4
    va = _vec_align(dt)
    dc = _prep(delta, 4)
    Lc = _prep(Lambda.float(), 16)
    Bc = _prep(B, 16 if shared else va)
    Cc = _prep(C, 16 if shared else va)
    Sc = _prep(S, va)
    Df, dsb, dst, dsd = _skip_operand(D, bsz, seqlen, dm)
    h0c = _prep(h0.float(), 16) if h0 is not None else None
    y = torch.empty(bsz, seqlen, dm, 4, dtype=dt, device=delta.device)
    hT = (torch.empty(bsz, dm, ds, 4, dtype=torch.float32, device=delta.device)
          if return_final_state else None)
    flags = (_lib.MQC_SSM_BC_SHARED if shared else 0) | (_lib.MQC_SSM_S_REAL if S.dim() == 3 else 0)
    status = _lib.status_word(delta.device)
    a = _lib.SsmScanArgs(
        batch=bsz, seq_len=seqlen, channels=dm, d_state=ds, dtype=_lib.dtype_code(dc),
        flags=flags, eps=float(eps), reserved0=0, delta=dc.data_ptr(), lambda_=Lc.data_ptr(),
        q=None, Bm=Bc.data_ptr(), Cm=Cc.data_ptr(), s=Sc.data_ptr(), dskip=Df.data_ptr(),
        dskip_sb=dsb, dskip_st=dst, dskip_sd=dsd, h0=_lib.ptr(h0c), y=y.data_ptr(),
        hT=_lib.ptr(hT), status=status.data_ptr(), wait_poll_limit=-1, ckpt=None, ckpt_every=0)
    with torch.cuda.device(delta.device):
        _lib.call("mqc_ssm_scan_fwd_chunked_resume", ctypes.byref(a), int(summary.nchunks),
                  summary.workspace.data_ptr(), summary.ws_bytes, _lib.stream_ptr(delta.device))
    if _lib.sync_checks_enabled():
        _lib.check_device_status(delta.device)
    return (y, hT) if return_final_state else y


def ssm_scan_carry(P: torch.Tensor, E: torch.Tensor, h0: torch.Tensor | None = None):
    """Start states of consecutive time segments from their summaries.

    P, E [S, B, D, N, 4] fp32 (segment s = time range s, in order); h0
    [B, D, N, 4] or None (zero). Returns (hin [S, B, D, N, 4], h_T [B, D, N, 4]):
    H_0 = h0, H_{s+1} = P_s (x) H_s + E_s, hin[s] = H_s, h_T = H_S
    (``mqc_ssm_scan_carry``).
    """
    assert P.shape == E.shape and P.dim() == 5 and P.shape[-1] == 4
    _lib.require_cuda(P, E, h0, what="ssm_scan_carry")
    nseg, bsz, dm, ds, _ = P.shape
    Pc = _prep(P.float(), 16)
    Ec = _prep(E.float(), 16)
    h0c = _prep(h0.float(), 16) if h0 is not None else None
    hin = torch.empty_like(Pc)
    hT = torch.empty(bsz, dm, ds, 4, dtype=torch.float32, device=P.device)
    with torch.cuda.device(P.device):
        _lib.call("mqc_ssm_scan_carry", Pc.data_ptr(), Ec.data_ptr(), _lib.ptr(h0c),
                  hin.data_ptr(), hT.data_ptr(), nseg, bsz, dm * ds, _lib.stream_ptr(P.device))
    return hin, hT


def ssm_scan_cayley(delta: torch.Tensor, Lambda: torch.Tensor, B: torch.Tensor,
                    C: torch.Tensor, S: torch.Tensor, D: torch.Tensor,
                    h0: torch.Tensor | None = None, eps: float = 1e-6,
                    return_final_state: bool = False, wait_poll_limit: int = -1,
                    time_chunks: int | str = "auto"):
    """Fused Cayley + quaternion selective scan (differentiable).

    delta [B,T,D] (positive step sizes), Lambda [D,N,4] (fp32 continuous
    dynamics), B/C [B,T,N,4] shared or [B,T,D,N,4] per-channel, S [B,T,D] real or
    [B,T,D,4], D skip [D] / [B,D] / [B,T,D]. Computes, per (b, d, n),
    q_t = (1 - delta_t Lambda/2)^-1 (x) (1 + delta_t Lambda/2) and
    h_t = q_t (x) h_{t-1} + B_t (x) S_t, y_t = sum_n C_t (x) h_t + D S_t.

    Returns y [B,T,D,4] (dtype of delta), plus the final fp32 state
    h_T [B,D,N,4] when ``return_final_state``. Gradients flow to every tensor
    argument through ``mqc_ssm_scan_bwd`` (states recomputed from checkpoints
    the forward writes every 8 steps when a gradient is needed).

    ``time_chunks``: when no gradient is needed, a long sequence with few
    channels is scanned time-parallel in that many chunks (``"auto"``: enough to
    fill the GPU, see ``auto_time_chunks``; 1 disables it).
    """
    assert delta.dim() == 3, f"delta must be [B,T,D], got {tuple(delta.shape)}"
    assert Lambda.dim() == 3 and Lambda.shape[-1] == 4, "Lambda must be [D,N,4]"
    bsz, seqlen, dm = delta.shape
    ds = Lambda.shape[1]
    assert Lambda.shape[0] == dm
    if B.dim() == 4:
        assert tuple(B.shape) == (bsz, seqlen, ds, 4) and B.shape == C.shape
    else:
        assert tuple(B.shape) == (bsz, seqlen, dm, ds, 4) and B.shape == C.shape
    assert tuple(S.shape) in ((bsz, seqlen, dm), (bsz, seqlen, dm, 4))
    _lib.require_cuda(delta, Lambda, B, C, S, D, h0, what="ssm_scan_cayley")
    needs_grad = torch.is_grad_enabled() and any(
        t is not None and t.requires_grad for t in (delta, Lambda, B, C, S, D, h0))
    if not needs_grad and D.dim() == 1 and wait_poll_limit < 0:
        nc = (auto_time_chunks(bsz, seqlen, dm, ds, delta.device) if time_chunks == "auto"
              else int(time_chunks))
        if nc > 1:
            y, hT = _run_scan_chunked(delta, Lambda, B, C, S, D, h0, eps, nc, return_final_state)
            return (y, hT) if return_final_state else y
    y, hT = _SsmScanCayley.apply(delta, Lambda, B, C, S, D, h0, eps, wait_poll_limit)
    return (y, hT) if return_final_state else y


def ssm_forward_fused(q: torch.Tensor, B: torch.Tensor, S: torch.Tensor, C: torch.Tensor,
                      D: torch.Tensor, h0: torch.Tensor | None = None,
                      return_final_state: bool = False):
    """Full scan over time with explicit operators q [B,T,D,N,4] (zero initial state).

    Mirrors ``ssm_forward_fused`` (mambaqc/kernels/ssm_fused.py:340-401): returns
    y [B,T,D,4]; ``h0`` and ``return_final_state`` are optional extensions.
    """
    assert q.dim() == 5 and q.shape[-1] == 4
    y, hT = _run_scan(flags=_lib.MQC_SSM_Q_GIVEN, q=q, B=B, C=C, S=S, D=D, h0=h0,
                      return_final_state=return_final_state)
    return (y, hT) if return_final_state else y


def ssm_step_fused(q: torch.Tensor, B: torch.Tensor, S: torch.Tensor, C: torch.Tensor,
                   D: torch.Tensor, h_prev: torch.Tensor):
    """One step: (h_new, y). Mirrors ``ssm_step_fused`` (ssm_fused.py:258-337)."""
    bsz, dm, ds, _ = q.shape
    assert B.shape == (bsz, dm, ds, 4)
    assert S.shape == (bsz, dm, 4)
    assert C.shape == (bsz, dm, ds, 4)
    assert D.shape == (bsz, dm)
    assert h_prev.shape == (bsz, dm, ds, 4)
    _lib.require_cuda(q, B, S, C, D, h_prev, what="ssm_step_fused")
    va = _vec_align(q.dtype)
    qc, Bc, Cc, Sc = (_prep(t, va) for t in (q, B, C, S))
    Dc = _prep(D.float(), 4)
    hp = _prep(h_prev.float(), 16)
    h_new = torch.empty(bsz, dm, ds, 4, dtype=torch.float32, device=q.device)
    y = torch.empty(bsz, dm, 4, dtype=q.dtype, device=q.device)
    with torch.cuda.device(q.device):
        _lib.call("mqc_ssm_step", qc.data_ptr(), Bc.data_ptr(), Sc.data_ptr(), Cc.data_ptr(),
                  Dc.data_ptr(), hp.data_ptr(), h_new.data_ptr(), y.data_ptr(), bsz, dm, ds,
                  _lib.dtype_code(qc), _lib.stream_ptr(q.device))
    return h_new.to(h_prev.dtype), y


def ssm_step_cayley(delta: torch.Tensor, Lambda: torch.Tensor, B: torch.Tensor,
                    C: torch.Tensor, S: torch.Tensor, D: torch.Tensor, h: torch.Tensor,
                    eps: float = 1e-6, out: torch.Tensor | None = None) -> torch.Tensor:
    """One decode step of the fused Cayley scan with an in-place state cache.

    delta [B,D], Lambda [D,N,4], B/C [B,N,4] (shared by channels) or [B,D,N,4],
    S real x [B,D] or quaternion [B,D,4], D skip [D], h [B,D,N,4] fp32: the state
    before the step, overwritten with the state after it. Returns y [B,D,4]
    (written into ``out`` when given, e.g. a row of a preallocated trajectory).
    The same step as ``ssm_step_fused`` (ssm_fused.py:258-337 in the reference)
    with q formed from delta and Lambda inside the kernel. No autograd.
    """
    assert delta.dim() == 2 and h.dim() == 4 and h.dtype == torch.float32 and h.is_contiguous()
    assert B.dim() in (3, 4) and C.dim() == B.dim()
    y, _ = _run_scan(flags=0, delta=delta.unsqueeze(1), Lam=Lambda, B=B.unsqueeze(1),
                     C=C.unsqueeze(1), S=S.unsqueeze(1), D=D, h0=h, eps=eps, hT_out=h,
                     y=None if out is None else out.unsqueeze(1))
    return y.squeeze(1)


def _host_segments(seqlen: int) -> int:
    """Time segments for the host pipeline: up to 8, each >= 128 steps."""
    n = 8
    while n > 1 and (seqlen % n or seqlen // n < 128):
        n //= 2
    return n


def ssm_scan_cayley_from_host(delta: torch.Tensor, Lambda: torch.Tensor, B: torch.Tensor,
                              C: torch.Tensor, S: torch.Tensor, D: torch.Tensor,
                              device: torch.device | str | None = None,
                              out: torch.Tensor | None = None, eps: float = 1e-6,
                              segments: int | str = "auto",
                              _bufs: dict | None = None) -> torch.Tensor:
    """``ssm_scan_cayley`` on host (CPU) tensors, through ``mqc_ssm_scan_fwd_host``.

    For inputs that live in host memory: the C entry point cuts the sequence into
    time segments (all batch rows in each) and pipelines them over three
    streams: segment k is copied to the GPU (one strided copy per tensor) while
    segment k-1 is scanned on the current stream (from segment k-2's final
    state, so every scan keeps the whole batch and fills the GPU) and segment
    k-2's output is copied back, so the PCIe transfers in both directions overlap
    the kernels. Pinned host tensors give asynchronous copies (pageable ones work
    but serialise). Returns y [B,T,D,4] in host memory (``out`` if given, pinned
    when allocated here), complete when the current stream is. Forward only (no
    autograd); D is the per-channel skip weight [D]. ``_bufs`` is accepted for
    compatibility and unused (device scratch comes from the library's pool).
    """
    assert delta.dim() == 3 and S.shape[:3] == delta.shape
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    bsz, seqlen, dm = delta.shape
    dt = delta.dtype
    for name, t in (("delta", delta), ("B", B), ("C", C), ("S", S), ("Lambda", Lambda), ("D", D)):
        if t.device.type != "cpu":
            raise ValueError(f"ssm_scan_cayley_from_host: {name} must be a host tensor")
    for name, t in (("B", B), ("C", C), ("S", S)):
        if t.dtype != dt:
            raise TypeError(f"{name} dtype {t.dtype} != {dt}")
    if D.dim() != 1 or D.shape[0] != dm:
        raise ValueError("ssm_scan_cayley_from_host: D must be the per-channel skip weight [D]")
    nseg = _host_segments(seqlen) if segments == "auto" else int(segments)
    if nseg < 1 or seqlen % nseg:
        raise ValueError(f"seq_len {seqlen} does not split into {nseg} equal segments")
    if out is None:
        out = torch.empty(bsz, seqlen, dm, 4, dtype=dt, pin_memory=True)
    assert out.is_contiguous() and out.dtype == dt and tuple(out.shape) == (bsz, seqlen, dm, 4)
    shared = B.dim() == 4
    ds = B.shape[2] if shared else B.shape[3]
    dc, Bc, Cc, Sc = (t.contiguous() for t in (delta, B, C, S))
    Lc = Lambda.float().contiguous()
    Dc = D.float().contiguous()
    flags = (_lib.MQC_SSM_BC_SHARED if shared else 0) | (_lib.MQC_SSM_S_REAL if S.dim() == 3 else 0)
    a = _lib.SsmScanArgs(
        batch=bsz, seq_len=seqlen, channels=dm, d_state=ds, dtype=_lib.dtype_code(dc),
        flags=flags, eps=float(eps), reserved0=0, delta=dc.data_ptr(), lambda_=Lc.data_ptr(),
        q=None, Bm=Bc.data_ptr(), Cm=Cc.data_ptr(), s=Sc.data_ptr(), dskip=Dc.data_ptr(),
        dskip_sb=0, dskip_st=0, dskip_sd=1, h0=None, y=out.data_ptr(), hT=None,
        status=_lib.status_word(dev).data_ptr(), wait_poll_limit=-1, ckpt=None, ckpt_every=0)
    with torch.cuda.device(dev):
        _lib.call("mqc_ssm_scan_fwd_host", ctypes.byref(a), int(nseg), _lib.stream_ptr(dev))
    return out
