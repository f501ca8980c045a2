"""Helpers shared by the GPU parity tests (inputs are generated on the CPU with a
seeded generator, so the oracle and the GPU see identical bits)."""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F

# Tolerances from the hot-path contract: relative L2 error against the fp64 oracle.
RTOL_F32 = 1e-5
RTOL_BF16 = 2e-2

DEV = "cuda"


def rel_l2(a: torch.Tensor, b: torch.Tensor) -> float:
    a = a.detach().double().cpu()
    b = b.detach().double().cpu()
    return (torch.linalg.vector_norm(a - b) / torch.linalg.vector_norm(b).clamp_min(1e-300)).item()


def gen(seed: int) -> torch.Generator:
    return torch.Generator().manual_seed(seed)


def make_lambda(dm: int, ds: int, g: torch.Generator, imag_std: float = 0.5) -> torch.Tensor:
    """Re = -exp(U(log 1e-3, log 1e-1)), Im ~ N(0, imag_std) (config 1 / config 3)."""
    lam = torch.empty(dm, ds, 4, dtype=torch.float64)
    lo, hi = math.log(1e-3), math.log(1e-1)
    lam[..., 0] = -torch.exp(torch.rand(dm, ds, generator=g, dtype=torch.float64) * (hi - lo) + lo)
    lam[..., 1:] = imag_std * torch.randn(dm, ds, 3, generator=g, dtype=torch.float64)
    return lam


def make_scan_inputs(bsz, seqlen, dm, ds, *, shared=True, s_real=True, seed=0,
                     delta_shift=-3.0, bc_scale=None):
    """Config-3 style inputs in float64 on the CPU."""
    g = gen(seed)
    x = torch.randn(bsz, seqlen, dm, generator=g, dtype=torch.float64)
    delta = F.softplus(torch.randn(bsz, seqlen, dm, generator=g, dtype=torch.float64) + delta_shift)
    lam = make_lambda(dm, ds, g)
    scale = bc_scale if bc_scale is not None else 1.0 / math.sqrt(ds)
    shape = (bsz, seqlen, ds, 4) if shared else (bsz, seqlen, dm, ds, 4)
    Bm = torch.randn(*shape, generator=g, dtype=torch.float64) * scale
    Cm = torch.randn(*shape, generator=g, dtype=torch.float64) * scale
    if s_real:
        S = x
    else:
        S = torch.randn(bsz, seqlen, dm, 4, generator=g, dtype=torch.float64)
    Dk = 1.0 + 0.1 * torch.randn(dm, generator=g, dtype=torch.float64)
    return dict(delta=delta, Lambda=lam, B=Bm, C=Cm, S=S, D=Dk)


def to_dev(d: dict, dtype) -> dict:
    out = {}
    for k, v in d.items():
        if k in ("Lambda", "D"):
            out[k] = v.to(DEV, torch.float32)
        else:
            out[k] = v.to(DEV, dtype)
    return out
