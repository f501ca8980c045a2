"""The block's B/C projections fused into its per-channel scan (``mqc_bc_proj_scan_fwd``).

The reference block (``mambaqc/models/quaternion_mamba2_block.py:186-191``)
computes ``B = B_proj(x)`` and ``C = C_proj(x)`` -- real -> quaternion
projections of the activated inner signal x [B, T, d_inner] onto
d_inner * d_state quaternions -- and scans them per channel
(``:214-228``). ``bc_proj_scan`` does both in one kernel: the tensor cores
produce each channel's B/C tile on chip and the scan consumes it from shared
memory, so the two [B, T, d_inner, d_state, 4] activations are never stored.

B and C are rounded to bf16 before the scan uses them, as the bf16 projection
of the reference's autocast does. The backward recomputes B and C with the
unfused projections (cuBLAS) and takes the scan's own backward, so training
pays the projections twice, exactly as activation checkpointing of the block
does, and stores neither.
"""

from __future__ import annotations

import ctypes

import torch

from .. import _lib
from .ssm_fused import _prep, _vec_align, ssm_scan_cayley

__all__ = ["bc_proj_scan", "bc_proj_scan_supported"]


def bc_proj_scan_supported(d_inner: int, d_state: int, in_features: int | None = None) -> bool:
    """Shapes the fused kernel takes: d_state 16, 32 or 64; in_features (the
    projection's input width, d_inner in the block) a multiple of 64."""
    k = d_inner if in_features is None else in_features
    return d_state in (16, 32, 64) and k % 64 == 0 and k >= 64 and d_inner <= 65535


def _run(x, w_b, w_c, delta, Lam, S, D, h0, eps, return_final_state):
    bsz, seqlen, kin = x.shape
    dm = delta.shape[2]
    ds = Lam.shape[1]
    dt = delta.dtype
    xc = _lib.aligned_contig(x.reshape(bsz * seqlen, kin), 16)
    wb = _lib.aligned_contig(w_b, 16)
    wc = _lib.aligned_contig(w_c, 16)
    dc = _prep(delta, 4)
    sc = _prep(S.to(dt), 4)
    Lc = _prep(Lam.float(), 16)
    Df = D.detach().float().contiguous()
    h0c = _prep(h0.float(), 16) if h0 is not None else None
    y = torch.empty(bsz, seqlen, dm, 4, dtype=dt, device=x.device)
    assert y.data_ptr() % _vec_align(dt) == 0
    hT = (torch.empty(bsz, dm, ds, 4, dtype=torch.float32, device=x.device)
          if return_final_state else None)
    status = _lib.status_word(x.device)
    a = _lib.BcProjScanArgs(
        batch=bsz, seq_len=seqlen, channels=dm, d_state=ds, in_features=kin,
        dtype=_lib.dtype_code(delta), eps=float(eps), x=xc.data_ptr(), w_b=wb.data_ptr(),
        w_c=wc.data_ptr(), delta=dc.data_ptr(), s=sc.data_ptr(), lambda_=Lc.data_ptr(),
        dskip=Df.data_ptr(), dskip_sd=1, h0=_lib.ptr(h0c), hT=_lib.ptr(hT), y=y.data_ptr(),
        status=status.data_ptr(), wait_poll_limit=-1)
    with torch.cuda.device(x.device):
        _lib.call("mqc_bc_proj_scan_fwd", ctypes.byref(a), _lib.stream_ptr(x.device))
    if _lib.sync_checks_enabled():
        _lib.check_device_status(x.device)
    return y, hT


def _unfused(x, w_b, w_c, delta, Lam, S, D, h0, eps):
    bsz, seqlen, _ = x.shape
    dm, ds = Lam.shape[0], Lam.shape[1]
    Bq = (x @ w_b.t()).view(bsz, seqlen, dm, ds, 4).to(delta.dtype)
    Cq = (x @ w_c.t()).view(bsz, seqlen, dm, ds, 4).to(delta.dtype)
    return ssm_scan_cayley(delta, Lam, Bq, Cq, S, D, h0=h0, eps=eps)


class _BcProjScan(torch.autograd.Function):
    """Forward: the fused kernel (and the final state, not differentiable).
    Backward: recompute the projections and the scan (unfused, with the scan's
    checkpoints) and differentiate that."""

    @staticmethod
    def forward(ctx, x, w_b, w_c, delta, Lam, S, D, h0, eps, return_final_state):
        y, hT = _run(x, w_b, w_c, delta, Lam, S, D, h0, eps, return_final_state)
        ctx.save_for_backward(x, w_b, w_c, delta, Lam, S, D, h0)
        ctx.eps = eps
        if return_final_state:
            ctx.mark_non_differentiable(hT)
            return y, hT
        return y

    @staticmethod
    def backward(ctx, gy, *unused):
        saved = ctx.saved_tensors
        leaves = [t.detach().requires_grad_(need) if t is not None else None
                  for t, need in zip(saved, ctx.needs_input_grad[:8])]
        with torch.enable_grad():
            y = _unfused(*leaves, ctx.eps)
        inputs = [t for t in leaves if t is not None and t.requires_grad]
        grads = torch.autograd.grad(y, inputs, gy, allow_unused=True) if inputs else []
        it = iter(grads)
        out = [next(it) if (t is not None and t.requires_grad) else None for t in leaves]
        return (*out, None, None)


def bc_proj_scan(x: torch.Tensor, w_b: torch.Tensor, w_c: torch.Tensor, delta: torch.Tensor,
                 Lambda: torch.Tensor, S: torch.Tensor, D: torch.Tensor,
                 h0: torch.Tensor | None = None, eps: float = 1e-6,
                 return_final_state: bool = False):
    """``ssm_scan_cayley(delta, Lambda, (x @ w_b.T).view(...), (x @ w_c.T).view(...), S, D)``
    without storing the projections.

    x [B, T, K] bf16 (the block's activated inner signal); w_b, w_c
    [d_inner * d_state * 4, K] bf16 (``B_proj.weight``, ``C_proj.weight``);
    delta and the real signal S [B, T, d_inner] (fp32 or bf16); Lambda
    [d_inner, d_state, 4]; D the per-channel skip weight [d_inner]; h0 an
    optional initial state [B, d_inner, d_state, 4]. Returns y [B, T, d_inner, 4]
    in delta's dtype, and with ``return_final_state`` also the final state
    [B, d_inner, d_state, 4] fp32 (not differentiable)."""
    assert x.dim() == 3 and delta.dim() == 3 and S.dim() == 3
    bsz, seqlen, kin = x.shape
    dm, ds = Lambda.shape[0], Lambda.shape[1]
    assert delta.shape == (bsz, seqlen, dm) and S.shape == (bsz, seqlen, dm)
    assert Lambda.shape == (dm, ds, 4) and D.shape == (dm,)
    assert w_b.shape == (dm * ds * 4, kin) and w_c.shape == w_b.shape
    assert x.dtype == torch.bfloat16 and w_b.dtype == torch.bfloat16 and w_c.dtype == torch.bfloat16
    assert delta.dtype in (torch.float32, torch.bfloat16) and S.dtype == delta.dtype
    assert h0 is None or h0.shape == (bsz, dm, ds, 4)
    _lib.require_cuda(x, w_b, w_c, delta, Lambda, S, D, h0, what="bc_proj_scan")
    if not bc_proj_scan_supported(dm, ds, kin):
        raise ValueError(f"bc_proj_scan: d_state {ds} / in_features {kin} not supported "
                         "(d_state 16, 32 or 64; in_features a multiple of 64)")
    return _BcProjScan.apply(x, w_b, w_c, delta, Lambda, S, D, h0, eps, bool(return_final_state))
