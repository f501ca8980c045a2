"""Cayley discretisation on the GPU: drop-in for ``mambaqc.kernels.cayley_transform``.

``cayley_discretization_fused(z, eps)`` keeps the reference signature and
preconditions (mambaqc/kernels/cayley_transform.py:132-195) and runs
``mqc_cayley`` (closed form, one reciprocal per quaternion, 16-byte vector
I/O). It is differentiable through ``mqc_cayley_bwd``.
"""

from __future__ import annotations

import torch

from .. import _lib

__all__ = ["cayley_discretization_fused"]


def _prep(t: torch.Tensor) -> torch.Tensor:
    _lib.require_cuda(t, what="cayley_discretization_fused")
    return _lib.aligned_contig(t, 16 if t.dtype == torch.float32 else 8)


class _Cayley(torch.autograd.Function):
    @staticmethod
    def forward(ctx, z, eps):
        zc = _prep(z)
        q = torch.empty_like(zc)
        with torch.cuda.device(zc.device):
            _lib.call("mqc_cayley", zc.data_ptr(), q.data_ptr(), zc.numel() // 4, float(eps),
                      _lib.dtype_code(zc), _lib.stream_ptr(zc.device))
        ctx.save_for_backward(zc)
        ctx.eps = eps
        return q

    @staticmethod
    def backward(ctx, g):
        (zc,) = ctx.saved_tensors
        gc = _prep(g.to(zc.dtype))
        dz = torch.empty_like(zc)
        with torch.cuda.device(zc.device):
            _lib.call("mqc_cayley_bwd", zc.data_ptr(), gc.data_ptr(), dz.data_ptr(),
                      zc.numel() // 4, float(ctx.eps), _lib.dtype_code(zc),
                      _lib.stream_ptr(zc.device))
        return dz, None


def cayley_discretization_fused(z: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """q = (1 - z/2)^-1 (x) (1 + z/2) for z [batch, seq_len, d_model, d_state, 4].

    |1 - z/2|^2 is clamped below by ``eps``. If Re(z) < 0 then |q| < 1.
    """
    assert z.shape[-1] == 4, f"Last dim must be 4, got {z.shape[-1]}"
    assert z.ndim == 5, f"Expected 5D tensor, got {z.ndim}D"
    return _Cayley.apply(z, eps)
