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

__all__ = ["quaternion_layer_norm_fused", "QuaternionLayerNorm"]


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
