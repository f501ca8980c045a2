"""The real-valued glue of ``QuaternionMamba2Block`` around the scan, fused.

Three differentiable ops, each one streaming CUDA kernel forward and one
backward (``csrc/block_fused.cu``), replacing chains of torch ops in the
reference block (mambaqc/models/quaternion_mamba2_block.py):

* ``causal_conv1d_silu(x, weight, bias)`` = ``silu(CausalConv1d(x))``
  (:140-144; layers/causal_conv1d.py:68-91 pads on the left, transposes to
  [B, D, T] and back). The kernel reads x in place, also as a column slice of the
  in_proj output [B, T, 2*d_inner], and never transposes.
* ``ssm_scan_inputs(u, gate, x)`` = ``(softplus(u), sigmoid(gate) * x)``: the
  scan's step sizes and real signal (:183, :197-198) from the dt_proj and
  gate_proj outputs.
* ``gate_residual(x, z, y)`` = ``x + sigmoid(z) * y`` (:154-164).

All three take fp32 or bf16 activations (one dtype per call) and compute in fp32.
"""

from __future__ import annotations

import torch

from .. import _lib

__all__ = ["causal_conv1d_silu", "ssm_scan_inputs", "gate_residual"]


def _rows(t: torch.Tensor) -> tuple[torch.Tensor, int]:
    """(tensor, row stride in elements) with unit stride along the last dim and
    evenly spaced rows over all leading dims; copies only if needed."""
    if t.stride(-1) != 1:
        t = t.contiguous()
    rs = t.stride(-2) if t.dim() >= 2 else t.shape[-1]
    ok = True
    expect = rs
    for d in range(t.dim() - 2, -1, -1):
        if t.shape[d] > 1 and t.stride(d) != expect:
            ok = False
            break
        expect *= t.shape[d]
    if not ok:
        t = t.contiguous()
        rs = t.shape[-1]
    return t, rs


def _contig(t: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    return t.to(dtype).contiguous()


class _ConvSilu(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias):
        bsz, seqlen, dm = x.shape
        k = weight.shape[-1]
        xs, rs = _rows(x)
        w32 = weight.detach().reshape(dm, k).float().contiguous()
        b32 = bias.detach().float().contiguous() if bias is not None else None
        out = torch.empty(bsz, seqlen, dm, dtype=x.dtype, device=x.device)
        with torch.cuda.device(x.device):
            _lib.call("mqc_conv_silu_fwd", xs.data_ptr(), rs, w32.data_ptr(), _lib.ptr(b32),
                      out.data_ptr(), bsz, seqlen, dm, k, _lib.dtype_code(xs),
                      _lib.stream_ptr(x.device))
        ctx.save_for_backward(xs, w32, b32)
        ctx.rs = rs
        ctx.shape = (bsz, seqlen, dm, k)
        ctx.w_meta = (weight.shape, weight.dtype)
        ctx.b_dtype = bias.dtype if bias is not None else None
        return out

    @staticmethod
    def backward(ctx, g):
        xs, w32, b32 = ctx.saved_tensors
        bsz, seqlen, dm, k = ctx.shape
        gc = _contig(g, xs.dtype)
        dx = torch.empty(bsz, seqlen, dm, dtype=xs.dtype, device=xs.device)
        dw = torch.empty(dm, k, dtype=torch.float32, device=xs.device)
        db = torch.empty(dm, dtype=torch.float32, device=xs.device) if b32 is not None else None
        lib = _lib.load()
        ws_bytes = lib.mqc_conv_silu_bwd_workspace_size(bsz, seqlen, dm, k)
        ws = torch.empty(max(4, ws_bytes // 4), dtype=torch.float32, device=xs.device)
        with torch.cuda.device(xs.device):
            _lib.call("mqc_conv_silu_bwd", xs.data_ptr(), ctx.rs, w32.data_ptr(), _lib.ptr(b32),
                      gc.data_ptr(), dx.data_ptr(), dw.data_ptr(), _lib.ptr(db), bsz, seqlen,
                      dm, k, _lib.dtype_code(xs), ws.data_ptr(), ws_bytes,
                      _lib.stream_ptr(xs.device))
        w_shape, w_dtype = ctx.w_meta
        dw = dw.reshape(w_shape).to(w_dtype)
        if db is not None:
            db = db.to(ctx.b_dtype)
        return dx, dw, db


def causal_conv1d_silu(x: torch.Tensor, weight: torch.Tensor,
                       bias: torch.Tensor | None = None) -> torch.Tensor:
    """silu(causal depthwise conv1d(x)): x [B, T, D] (a column slice of a wider
    tensor is read in place), weight [D, 1, K] or [D, K] with K <= 8 (the
    ``CausalConv1d.conv`` weight), bias [D] or None. Returns [B, T, D] in x's dtype."""
    assert x.dim() == 3, f"x must be [B, T, D], got {tuple(x.shape)}"
    dm = x.shape[2]
    assert weight.shape[0] == dm and weight.numel() % dm == 0, "weight must be [D, 1, K]"
    assert bias is None or tuple(bias.shape) == (dm,)
    _lib.require_cuda(x, weight, bias, what="causal_conv1d_silu")
    return _ConvSilu.apply(x, weight, bias)


class _ScanInputs(torch.autograd.Function):
    @staticmethod
    def forward(ctx, u, gate, x):
        dt = x.dtype
        us, urs = _rows(u.to(dt))
        gs, grs = _rows(gate.to(dt))
        xc = x.contiguous()
        dm = x.shape[-1]
        rows = xc.numel() // dm if dm else 0
        delta = torch.empty_like(xc)
        s = torch.empty_like(xc)
        with torch.cuda.device(x.device):
            _lib.call("mqc_scan_inputs_fwd", us.data_ptr(), urs, gs.data_ptr(), grs,
                      xc.data_ptr(), delta.data_ptr(), s.data_ptr(), rows, dm,
                      _lib.dtype_code(xc), _lib.stream_ptr(x.device))
        ctx.save_for_backward(us, gs, xc)
        ctx.meta = (urs, grs, rows, dm, u.dtype, gate.dtype)
        return delta, s

    @staticmethod
    def backward(ctx, g_delta, g_s):
        us, gs, xc = ctx.saved_tensors
        urs, grs, rows, dm, u_dt, g_dt = ctx.meta
        gd = _contig(g_delta, xc.dtype) if g_delta is not None else None
        gss = _contig(g_s, xc.dtype) if g_s is not None else None
        du = torch.empty_like(xc)
        dg = torch.empty_like(xc)
        dx = torch.empty_like(xc)
        with torch.cuda.device(xc.device):
            _lib.call("mqc_scan_inputs_bwd", us.data_ptr(), urs, gs.data_ptr(), grs,
                      xc.data_ptr(), _lib.ptr(gd), _lib.ptr(gss), du.data_ptr(), dg.data_ptr(),
                      dx.data_ptr(), rows, dm, _lib.dtype_code(xc), _lib.stream_ptr(xc.device))
        return du.to(u_dt), dg.to(g_dt), dx


def ssm_scan_inputs(u: torch.Tensor, gate: torch.Tensor, x: torch.Tensor):
    """(delta, s) = (softplus(u), sigmoid(gate) * x), all [..., D] of one shape;
    returned in x's dtype."""
    assert u.shape == gate.shape == x.shape, "u, gate and x must have one shape"
    _lib.require_cuda(u, gate, x, what="ssm_scan_inputs")
    return _ScanInputs.apply(u, gate, x)


class _GateResidual(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, z, y):
        dt = torch.result_type(x, y)
        dt = torch.promote_types(dt, z.dtype)
        xc = _contig(x, dt)
        yc = _contig(y, dt)
        zs, zrs = _rows(z.to(dt))
        cols = x.shape[-1]
        rows = xc.numel() // cols if cols else 0
        out = torch.empty_like(xc)
        with torch.cuda.device(x.device):
            _lib.call("mqc_gate_residual_fwd", xc.data_ptr(), zs.data_ptr(), zrs, yc.data_ptr(),
                      out.data_ptr(), rows, cols, _lib.dtype_code(xc), _lib.stream_ptr(x.device))
        ctx.save_for_backward(zs, yc)
        ctx.meta = (zrs, rows, cols, x.dtype, z.dtype, y.dtype)
        return out

    @staticmethod
    def backward(ctx, g):
        zs, yc = ctx.saved_tensors
        zrs, rows, cols, x_dt, z_dt, y_dt = ctx.meta
        gc = _contig(g, yc.dtype)
        dz = torch.empty_like(yc)
        dy = torch.empty_like(yc)
        with torch.cuda.device(yc.device):
            _lib.call("mqc_gate_residual_bwd", zs.data_ptr(), zrs, yc.data_ptr(), gc.data_ptr(),
                      dz.data_ptr(), dy.data_ptr(), rows, cols, _lib.dtype_code(yc),
                      _lib.stream_ptr(yc.device))
        return g.to(x_dt), dz.to(z_dt), dy.to(y_dt)


def gate_residual(x: torch.Tensor, z: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
    """x + sigmoid(z) * y for x, z, y of one shape [..., C] (z may be a column
    slice of a wider tensor); computed in the promoted dtype of the three."""
    assert x.shape == z.shape == y.shape, "x, z and y must have one shape"
    _lib.require_cuda(x, z, y, what="gate_residual")
    return _GateResidual.apply(x, z, y)
