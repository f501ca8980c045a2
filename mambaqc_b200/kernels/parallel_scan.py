"""Cumulative quaternion product on the GPU: drop-in for ``mambaqc.kernels.parallel_scan``.

``parallel_scan_quaternion(q_sequence)`` keeps the reference signature and
semantics (mambaqc/kernels/parallel_scan.py:171-264 and the sequential
definition at :267-295): cumulative[t] = q[t] (x) q[t-1] (x) ... (x) q[0].
One ``mqc_prefix_prod`` call replaces the reference's per-tree-node launches.
"""

from __future__ import annotations

import torch

from .. import _lib

__all__ = ["parallel_scan_quaternion"]


def parallel_scan_quaternion(q_sequence: torch.Tensor) -> torch.Tensor:
    """Inclusive left-product scan over time of q_sequence [B, T, D, N, 4]."""
    assert q_sequence.shape[-1] == 4
    assert q_sequence.ndim == 5
    _lib.require_cuda(q_sequence, what="parallel_scan_quaternion")
    q = _lib.aligned_contig(q_sequence, 16 if q_sequence.dtype == torch.float32 else 8)
    bsz, seqlen, dm, ds, _ = q.shape
    out = torch.empty_like(q)
    with torch.cuda.device(q.device):
        _lib.call("mqc_prefix_prod", q.data_ptr(), out.data_ptr(), bsz, seqlen, dm * ds,
                  _lib.dtype_code(q), _lib.stream_ptr(q.device))
    return out
