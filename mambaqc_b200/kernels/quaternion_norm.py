"""Quaternion LayerNorm on the GPU: drop-in for ``mambaqc.kernels.quaternion_norm``.

``quaternion_layer_norm_fused(q, gamma, beta, eps)`` and
``QuaternionLayerNorm(d_model, eps)`` keep the reference names, parameters
(``gamma`` [D] ones, ``beta`` [D,4] zeros) and preconditions
(mambaqc/kernels/quaternion_norm.py:119-215). The math is the reference's
definition (quaternion_norm.py:219-245) for every d_model; the reference Triton
kernel's padded-lane behaviour at non-power-of-two d_model is available as an
opt-in (``padded_compat=True`` or env ``MAMBAQC_COMPAT_LN_PADDED=1``, forward
only). Forward: ``mqc_qln_fwd``; backward: ``mqc_qln_bwd``.
"""

from __future__ import annotations

import os

import torch

from .. import _lib

__all__ = ["quaternion_layer_norm_fused", "QuaternionLayerNorm", "quaternion_layer_norm_linear"]


def _compat_default() -> bool:
    return os.environ.get("MAMBAQC_COMPAT_LN_PADDED", "0") == "1"


class _QLayerNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, gamma, beta, eps, padded_compat):
        dt = q.dtype
        qc = _lib.aligned_contig(q, 16 if dt == torch.float32 else 8)
        bsz, seqlen, dm, _ = qc.shape
        rows = bsz * seqlen
        g32 = _lib.aligned_contig(gamma.detach().float(), 4)
        b32 = _lib.aligned_contig(beta.detach().float(), 16)
        out = torch.empty_like(qc)
        mean = torch.empty(rows, dtype=torch.float32, device=q.device)
        rstd = torch.empty(rows, dtype=torch.float32, device=q.device)
        flags = _lib.MQC_QLN_PADDED_COMPAT if padded_compat else 0
        with torch.cuda.device(q.device):
            _lib.call("mqc_qln_fwd", qc.data_ptr(), g32.data_ptr(), b32.data_ptr(),
                      out.data_ptr(), mean.data_ptr(), rstd.data_ptr(), rows, dm, float(eps),
                      flags, _lib.dtype_code(qc), _lib.stream_ptr(q.device))
        ctx.save_for_backward(qc, g32, mean, rstd)
        ctx.eps = eps
        ctx.padded_compat = padded_compat
        ctx.gamma_dtype, ctx.beta_dtype = gamma.dtype, beta.dtype
        return out

    @staticmethod
    def backward(ctx, g):
        if ctx.padded_compat:
            raise RuntimeError("QuaternionLayerNorm: no backward for the padded-compat form")
        qc, g32, mean, rstd = ctx.saved_tensors
        bsz, seqlen, dm, _ = qc.shape
        rows = bsz * seqlen
        gc = _lib.aligned_contig(g.to(qc.dtype), 16 if qc.dtype == torch.float32 else 8)
        dq = torch.empty_like(qc)
        dgamma = torch.empty(dm, dtype=torch.float32, device=qc.device)
        dbeta = torch.empty(dm, 4, dtype=torch.float32, device=qc.device)
        lib = _lib.load()
        ws_bytes = lib.mqc_qln_bwd_workspace_size(rows, dm)
        ws = torch.empty(max(1, ws_bytes // 4), dtype=torch.float32, device=qc.device)
        with torch.cuda.device(qc.device):
            _lib.call("mqc_qln_bwd", qc.data_ptr(), g32.data_ptr(), gc.data_ptr(),
                      mean.data_ptr(), rstd.data_ptr(), dq.data_ptr(), dgamma.data_ptr(),
                      dbeta.data_ptr(), ws.data_ptr(), ws_bytes, rows, dm, float(ctx.eps),
                      _lib.dtype_code(qc), _lib.stream_ptr(qc.device))
        return dq, dgamma.to(ctx.gamma_dtype), dbeta.to(ctx.beta_dtype), None, None


class _QLNLinear(torch.autograd.Function):
    """LN(q) @ weight^T (+ bias) with the LayerNorm as the GEMM's operand
    prologue (``mqc_qln_linear_fwd``); bf16. The backward recomputes LN(q)
    (``mqc_qln_fwd``) for the weight gradient, takes both GEMMs on cuBLAS and
    the LayerNorm backward on ``mqc_qln_bwd`` with the saved row statistics."""

    @staticmethod
    def forward(ctx, q, gamma, beta, weight, bias, eps):
        qc = _lib.aligned_contig(q, 16)
        bsz, seqlen, dm, _ = qc.shape
        rows = bsz * seqlen
        nout = weight.shape[0]
        w = _lib.aligned_contig(weight, 16)
        bc = bias.contiguous() if bias is not None else None
        g32 = _lib.aligned_contig(gamma.detach().float(), 4)
        b32 = _lib.aligned_contig(beta.detach().float(), 16)
        out = torch.empty(bsz, seqlen, nout, dtype=q.dtype, device=q.device)
        mean = torch.empty(rows, dtype=torch.float32, device=q.device)
        rstd = torch.empty(rows, dtype=torch.float32, device=q.device)
        status = _lib.status_word(q.device)
        with torch.cuda.device(q.device):
            _lib.call("mqc_qln_linear_fwd", qc.data_ptr(), g32.data_ptr(), b32.data_ptr(),
                      w.data_ptr(), _lib.ptr(bc), out.data_ptr(), mean.data_ptr(),
                      rstd.data_ptr(), rows, dm, nout, float(eps), status.data_ptr(),
                      _lib.stream_ptr(q.device))
        if _lib.sync_checks_enabled():
            _lib.check_device_status(q.device)
        ctx.save_for_backward(qc, g32, b32, w, mean, rstd)
        ctx.eps = eps
        ctx.has_bias = bias is not None
        ctx.dtypes = (gamma.dtype, beta.dtype)
        return out

    @staticmethod
    def backward(ctx, gout):
        qc, g32, b32, w, mean, rstd = ctx.saved_tensors
        bsz, seqlen, dm, _ = qc.shape
        rows = bsz * seqlen
        dev = qc.device
        yn = torch.empty_like(qc)
        with torch.cuda.device(dev):
            _lib.call("mqc_qln_fwd", qc.data_ptr(), g32.data_ptr(), b32.data_ptr(),
                      yn.data_ptr(), None, None, rows, dm, float(ctx.eps), 0,
                      _lib.dtype_code(qc), _lib.stream_ptr(dev))
        g2 = gout.reshape(rows, -1).to(qc.dtype)
        dw = g2.t() @ yn.reshape(rows, dm * 4)
        dyn = (g2 @ w).reshape(bsz, seqlen, dm, 4).contiguous()
        dbias = g2.float().sum(0).to(qc.dtype) if ctx.has_bias else None
        dq = torch.empty_like(qc)
        dgamma = torch.empty(dm, dtype=torch.float32, device=dev)
        dbeta = torch.empty(dm, 4, dtype=torch.float32, device=dev)
        lib = _lib.load()
        ws_bytes = lib.mqc_qln_bwd_workspace_size(rows, dm)
        ws = torch.empty(max(1, ws_bytes // 4), dtype=torch.float32, device=dev)
        with torch.cuda.device(dev):
            _lib.call("mqc_qln_bwd", qc.data_ptr(), g32.data_ptr(), dyn.data_ptr(),
                      mean.data_ptr(), rstd.data_ptr(), dq.data_ptr(), dgamma.data_ptr(),
                      dbeta.data_ptr(), ws.data_ptr(), ws_bytes, rows, dm, float(ctx.eps),
                      _lib.dtype_code(qc), _lib.stream_ptr(dev))
        return (dq, dgamma.to(ctx.dtypes[0]), dbeta.to(ctx.dtypes[1]), dw, dbias, None)


def quaternion_layer_norm_linear(q: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor,
                                 weight: torch.Tensor, bias: torch.Tensor | None = None,
                                 eps: float = 1e-5) -> torch.Tensor:
    """``F.linear(quaternion_layer_norm_fused(q, gamma, beta, eps).flatten(-2), weight, bias)``
    in one pass over q: the LayerNorm is applied to each q tile inside the
    projection GEMM (sm_100a tensor cores) and its output is never stored.

    q [B, T, D, 4] bf16 with D a multiple of 16; weight [N, 4D] and bias [N]
    bf16. Returns [B, T, N] bf16. This is the block's
    ``out_proj(norm(y_quat))`` (quaternion_mamba2_block.py:154-157)."""
    assert q.ndim == 4 and q.shape[-1] == 4, f"Expected [B, T, D, 4], got {q.shape}"
    dm = q.shape[2]
    assert gamma.shape == (dm,) and beta.shape == (dm, 4)
    assert weight.ndim == 2 and weight.shape[1] == 4 * dm
    assert q.dtype == torch.bfloat16 and weight.dtype == torch.bfloat16
    assert bias is None or (bias.shape == (weight.shape[0],) and bias.dtype == torch.bfloat16)
    _lib.require_cuda(q, gamma, beta, weight, bias, what="quaternion_layer_norm_linear")
    return _QLNLinear.apply(q, gamma, beta, weight, bias, eps)


def quaternion_layer_norm_fused(q: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor,
                                eps: float = 1e-5, padded_compat: bool | None = None
                                ) -> torch.Tensor:
    """Norm-only LayerNorm of q [B,T,D,4] over D, preserving quaternion directions."""
    assert q.shape[-1] == 4
    assert q.ndim == 4, f"Expected [B, T, D, 4], got {q.shape}"
    assert gamma.shape == (q.shape[2],), f"gamma shape mismatch: {gamma.shape}"
    assert beta.shape == (q.shape[2], 4), f"beta shape mismatch: {beta.shape}"
    _lib.require_cuda(q, gamma, beta, what="quaternion_layer_norm_fused")
    if padded_compat is None:
        padded_compat = _compat_default()
    return _QLayerNorm.apply(q, gamma, beta, eps, bool(padded_compat))


class QuaternionLayerNorm(torch.nn.Module):
    """Learnable quaternion LayerNorm; mirrors quaternion_norm.py:177-215.

    Parameters ``gamma`` [d_model] (ones) and ``beta`` [d_model, 4] (zeros), so
    reference state_dicts load unchanged. Input/output [batch, seq_len, d_model, 4].
    """

    def __init__(self, d_model: int, eps: float = 1e-5):
        super().__init__()
        self.d_model = d_model
        self.eps = eps
        self.gamma = torch.nn.Parameter(torch.ones(d_model))
        self.beta = torch.nn.Parameter(torch.zeros(d_model, 4))

    def forward(self, q: torch.Tensor) -> torch.Tensor:
        return quaternion_layer_norm_fused(q, self.gamma, self.beta, self.eps)

    def extra_repr(self) -> str:
        return f"d_model={self.d_model}, eps={self.eps}"
