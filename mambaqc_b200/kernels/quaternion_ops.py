"""Quaternion algebra on the GPU: drop-in for ``mambaqc.kernels.quaternion_ops``.

Same names, argument meaning and preconditions (``assert``) as the reference
(mambaqc/kernels/quaternion_ops.py:259-461); the work runs in
``libmambaqc_b200.so`` (``mqc_qmul``, ``mqc_qmul_strided``, ``mqc_qconj``, ``mqc_qinv``,
``mqc_qnorm``). Inputs must be CUDA float32 or bfloat16 tensors; there is no CPU
path. ``quaternion_multiply`` is differentiable (dp = g (x) conj(q),
dq = conj(p) (x) g), which the reference's Triton path is not.
"""

from __future__ import annotations

import ctypes

import torch

from .. import _lib

__all__ = [
    "quaternion_multiply",
    "quaternion_multiply_batched",
    "quaternion_conjugate",
    "quaternion_inverse",
    "quaternion_norm",
]


def _prep(t: torch.Tensor, what: str) -> torch.Tensor:
    _lib.require_cuda(t, what=what)
    return _lib.aligned_contig(t, 16 if t.dtype == torch.float32 else 8)


def _qmul_raw(p: torch.Tensor, q: torch.Tensor) -> torch.Tensor:
    if p.dtype != q.dtype:
        raise TypeError(f"quaternion_multiply: dtype mismatch {p.dtype} vs {q.dtype}")
    if p.device != q.device:
        raise ValueError(f"quaternion_multiply: operands on {p.device} and {q.device}")
    pc, qc = _prep(p, "quaternion_multiply"), _prep(q, "quaternion_multiply")
    out = torch.empty_like(pc)
    with torch.cuda.device(pc.device):
        _lib.call("mqc_qmul", pc.data_ptr(), qc.data_ptr(), out.data_ptr(), pc.numel() // 4,
                  _lib.dtype_code(pc), _lib.stream_ptr(pc.device))
    return out


def _qconj_raw(q: torch.Tensor) -> torch.Tensor:
    qc = _prep(q, "quaternion_conjugate")
    out = torch.empty_like(qc)
    with torch.cuda.device(qc.device):
        _lib.call("mqc_qconj", qc.data_ptr(), out.data_ptr(), qc.numel() // 4,
                  _lib.dtype_code(qc), _lib.stream_ptr(qc.device))
    return out


class _QuaternionMultiply(torch.autograd.Function):
    @staticmethod
    def forward(ctx, p, q):
        ctx.save_for_backward(p, q)
        return _qmul_raw(p, q)

    @staticmethod
    def backward(ctx, g):
        p, q = ctx.saved_tensors
        gp = gq = None
        if ctx.needs_input_grad[0]:
            gp = _qmul_raw(g, _qconj_raw(q))
        if ctx.needs_input_grad[1]:
            gq = _qmul_raw(_qconj_raw(p), g)
        return gp, gq


def quaternion_multiply(p: torch.Tensor, q: torch.Tensor) -> torch.Tensor:
    """Hamilton product p (x) q on [..., 4] tensors of equal shape.

    Mirrors ``quaternion_multiply`` (mambaqc/kernels/quaternion_ops.py:259-303).
    """
    assert p.shape == q.shape, f"Shape mismatch: {p.shape} vs {q.shape}"
    assert p.shape[-1] == 4, f"Last dim must be 4, got {p.shape[-1]}"
    return _QuaternionMultiply.apply(p, q)


def _strided_ok(t: torch.Tensor) -> bool:
    """Whether ``mqc_qmul_strided`` reads ``t`` in place: quaternion axis
    contiguous, the other strides multiples of a quaternion, vector alignment."""
    align = 16 if t.dtype == torch.float32 else 8
    return (t.stride(-1) == 1 and all(s % 4 == 0 for s in t.stride()[:-1])
            and t.data_ptr() % align == 0)


def _qmul_strided_raw(p: torch.Tensor, q: torch.Tensor) -> torch.Tensor:
    if p.dtype != q.dtype:
        raise TypeError(f"quaternion_multiply_batched: dtype mismatch {p.dtype} vs {q.dtype}")
    _lib.require_cuda(p, what="quaternion_multiply_batched")
    _lib.require_cuda(q, what="quaternion_multiply_batched")
    if p.device != q.device:
        raise ValueError(f"quaternion_multiply_batched: operands on {p.device} and {q.device}")
    if not (_strided_ok(p) and _strided_ok(q)):
        return _qmul_raw(p, q)
    out = torch.empty(p.shape, dtype=p.dtype, device=p.device)
    i64x4 = ctypes.c_int64 * 4
    shape = i64x4(*p.shape[:4])
    ps, qs = i64x4(*p.stride()[:4]), i64x4(*q.stride()[:4])
    with torch.cuda.device(p.device):
        _lib.call("mqc_qmul_strided", p.data_ptr(), q.data_ptr(), out.data_ptr(), shape, ps, qs,
                  _lib.dtype_code(p), _lib.stream_ptr(p.device))
    return out


class _QuaternionMultiplyBatched(torch.autograd.Function):
    @staticmethod
    def forward(ctx, p, q):
        ctx.save_for_backward(p, q)
        return _qmul_strided_raw(p, q)

    @staticmethod
    def backward(ctx, g):
        return _QuaternionMultiply.backward(ctx, g)


def quaternion_multiply_batched(p: torch.Tensor, q: torch.Tensor) -> torch.Tensor:
    """Hamilton product on [batch, seq_len, d_model, d_state, 4] tensors.

    Mirrors ``quaternion_multiply_batched`` (quaternion_ops.py:306-357): like the
    reference kernel, p and q are read through their strides (``mqc_qmul_strided``;
    the quaternion axis must be contiguous, otherwise they are copied first). The
    output is a dense tensor.
    """
    assert p.shape == q.shape
    assert p.shape[-1] == 4
    assert p.ndim == 5, f"Expected 5D tensor, got {p.ndim}D"
    return _QuaternionMultiplyBatched.apply(p, q)


def quaternion_conjugate(q: torch.Tensor) -> torch.Tensor:
    """(a, -b, -c, -d); mirrors ``quaternion_conjugate`` (quaternion_ops.py:360-391)."""
    assert q.shape[-1] == 4
    return _qconj_raw(q)


def quaternion_inverse(q: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """conj(q) / max(|q|^2, eps); mirrors ``quaternion_inverse`` (quaternion_ops.py:394-428)."""
    assert q.shape[-1] == 4
    qc = _prep(q, "quaternion_inverse")
    out = torch.empty_like(qc)
    with torch.cuda.device(qc.device):
        _lib.call("mqc_qinv", qc.data_ptr(), out.data_ptr(), qc.numel() // 4, float(eps),
                  _lib.dtype_code(qc), _lib.stream_ptr(qc.device))
    return out


def quaternion_norm(q: torch.Tensor) -> torch.Tensor:
    """|q| over the last axis -> shape q.shape[:-1]; mirrors quaternion_ops.py:431-461."""
    assert q.shape[-1] == 4
    qc = _prep(q, "quaternion_norm")
    out = torch.empty(qc.shape[:-1], dtype=qc.dtype, device=qc.device)
    with torch.cuda.device(qc.device):
        _lib.call("mqc_qnorm", qc.data_ptr(), out.data_ptr(), qc.numel() // 4,
                  _lib.dtype_code(qc), _lib.stream_ptr(qc.device))
    return out
