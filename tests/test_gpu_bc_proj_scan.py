"""The B/C projections fused into the per-channel scan (``bc_proj_scan`` ->
``mqc_bc_proj_scan_fwd``: tcgen05 GEMM tiles handed to the scan on chip).

Checked against
  (a) the unfused path -- the projections on cuBLAS in bf16 (the reference's
      autocast), viewed per channel, then ``ssm_scan_cayley`` -- which sees the
      same bf16 B/C up to the GEMMs' summation order (rel-L2 < 5e-3);
  (b) the fp64 oracle (``oracle.ref.ssm_scan_cayley`` on B/C projected in fp64
      from the same bf16 x and weights), within the bf16 tolerance of the
      contract (2e-2): the kernel rounds B and C to bf16 as the reference does.
The config-4 block shape (B=4, T=2048, d_inner 1536, d_state 64) is checked on a
channel sample; gradients through the recomputing backward against the unfused
path."""

import pytest
import torch

from oracle import ref
from tests.gpu_util import DEV, RTOL_BF16, gen, make_lambda, rel_l2

pytestmark = pytest.mark.gpu

from mambaqc_b200.kernels import ssm_scan_cayley  # noqa: E402
from mambaqc_b200.kernels.bc_proj_scan import bc_proj_scan  # noqa: E402

UNFUSED_TOL = 5e-3


def _inputs(bsz, seqlen, kin, dm, ds, seed):
    g = gen(seed)
    x = torch.randn(bsz, seqlen, kin, generator=g).bfloat16()
    std = (2.0 / (kin + dm * ds)) ** 0.5  # the reference's real -> quaternion init
    w_b = (torch.randn(dm * ds * 4, kin, generator=g) * std).bfloat16()
    w_c = (torch.randn(dm * ds * 4, kin, generator=g) * std).bfloat16()
    delta = torch.nn.functional.softplus(torch.randn(bsz, seqlen, dm, generator=g) - 3.0)
    s = torch.randn(bsz, seqlen, dm, generator=g)
    lam = make_lambda(dm, ds, g).float()
    dk = 1.0 + 0.1 * torch.randn(dm, generator=g)
    return x, w_b, w_c, delta, lam, s, dk


def _unfused(x, w_b, w_c, delta, lam, s, dk, h0=None, return_final_state=False):
    bsz, seqlen, _ = x.shape
    dm, ds = lam.shape[0], lam.shape[1]
    Bq = (x @ w_b.t()).view(bsz, seqlen, dm, ds, 4).to(delta.dtype)
    Cq = (x @ w_c.t()).view(bsz, seqlen, dm, ds, 4).to(delta.dtype)
    return ssm_scan_cayley(delta, lam, Bq, Cq, s, dk, h0=h0,
                           return_final_state=return_final_state)


def _oracle(x, w_b, w_c, delta, lam, s, dk, chans, h0=None):
    """fp64 oracle on a channel sample (channels are independent recurrences)."""
    bsz, seqlen, _ = x.shape
    ds = lam.shape[1]
    xd = x.double().cpu()
    rows = torch.cat([torch.arange(c * ds * 4, (c + 1) * ds * 4) for c in chans.tolist()])
    Bq = (xd @ w_b.double().cpu()[rows].t()).view(bsz, seqlen, len(chans), ds, 4)
    Cq = (xd @ w_c.double().cpu()[rows].t()).view(bsz, seqlen, len(chans), ds, 4)
    return ref.ssm_scan_cayley(delta.double().cpu()[..., chans], lam.double().cpu()[chans], Bq,
                               Cq, s.double().cpu()[..., chans], dk.double().cpu()[chans],
                               h0=None if h0 is None else h0.double().cpu()[:, chans])


CASES = [
    # (B, T, K, d_inner, d_state, dtype of delta / s / y)
    (2, 200, 64, 3, 16, torch.float32),     # ragged last tile, one K block of 64
    (1, 130, 128, 5, 32, torch.float32),    # one scan warp, two tiles
    (3, 257, 192, 4, 64, torch.float32),    # two scan warps, T one past two tiles
    (2, 96, 256, 6, 64, torch.bfloat16),    # bf16 signals and output, T < one tile
    (1, 1, 64, 2, 16, torch.float32),       # a single step
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: "B{}T{}K{}D{}N{}{}".format(
    *c[:5], "f32" if c[5] == torch.float32 else "bf16"))
def test_bc_proj_scan_matches_unfused_and_oracle(case):
    bsz, seqlen, kin, dm, ds, dt = case
    x, w_b, w_c, delta, lam, s, dk = _inputs(bsz, seqlen, kin, dm, ds, seed=sum(case[:5]))
    h0 = torch.randn(bsz, dm, ds, 4, generator=gen(3)) * 0.3
    dev = [t.to(DEV) for t in (x, w_b, w_c)] + [delta.to(DEV, dt), lam.to(DEV), s.to(DEV, dt),
                                                dk.to(DEV)]
    y, hT = bc_proj_scan(*dev, h0=h0.to(DEV), return_final_state=True)
    y_u, hT_u = _unfused(*dev, h0=h0.to(DEV), return_final_state=True)
    torch.cuda.synchronize()
    assert y.dtype == dt and y.shape == (bsz, seqlen, dm, 4)
    assert rel_l2(y.float(), y_u.float()) < UNFUSED_TOL
    assert rel_l2(hT, hT_u) < UNFUSED_TOL
    chans = torch.arange(dm)
    y_ref, h_ref = _oracle(x, w_b, w_c, delta.to(dt), lam, s.to(dt), dk, chans, h0=h0)
    assert rel_l2(y.float(), y_ref) < RTOL_BF16
    assert rel_l2(hT, h_ref) < RTOL_BF16


def test_bc_proj_scan_is_deterministic():
    x, w_b, w_c, delta, lam, s, dk = _inputs(2, 300, 128, 7, 64, seed=5)
    dev = [t.to(DEV) for t in (x, w_b, w_c, delta, lam, s, dk)]
    y1 = bc_proj_scan(*dev)
    y2 = bc_proj_scan(*dev)
    torch.cuda.synchronize()
    assert torch.equal(y1, y2)


def test_bc_proj_scan_config4_block_channel_sample():
    """The config-4 block shape (B=4, T=2048, d_inner 1536, d_state 64, bf16
    signals): the whole output against the unfused path, and a channel sample
    against the fp64 oracle."""
    bsz, seqlen, dm, ds = 4, 2048, 1536, 64
    g = torch.Generator(device=DEV).manual_seed(11)
    x = torch.randn(bsz, seqlen, dm, generator=g, device=DEV).bfloat16()
    std = (2.0 / (dm + dm * ds)) ** 0.5
    w_b = (torch.randn(dm * ds * 4, dm, generator=g, device=DEV) * std).bfloat16()
    w_c = (torch.randn(dm * ds * 4, dm, generator=g, device=DEV) * std).bfloat16()
    delta = torch.nn.functional.softplus(
        torch.randn(bsz, seqlen, dm, generator=g, device=DEV) - 3.0).bfloat16()
    s = torch.randn(bsz, seqlen, dm, generator=g, device=DEV).bfloat16()
    lam = make_lambda(dm, ds, gen(12)).float().to(DEV)
    dk = torch.ones(dm, device=DEV)
    y = bc_proj_scan(x, w_b, w_c, delta, lam, s, dk)
    y_u = _unfused(x, w_b, w_c, delta, lam, s, dk)
    torch.cuda.synchronize()
    assert rel_l2(y.float(), y_u.float()) < UNFUSED_TOL
    del y_u
    chans = torch.tensor([0, 1, 700, 1535])
    y_ref, _ = _oracle(x, w_b, w_c, delta, lam, s, dk, chans)
    assert rel_l2(y.float().cpu()[..., chans, :], y_ref) < RTOL_BF16


def test_bc_proj_scan_gradients_match_unfused():
    x, w_b, w_c, delta, lam, s, dk = _inputs(2, 150, 128, 4, 32, seed=9)
    gy = torch.randn(2, 150, 4, 4, generator=gen(10)).to(DEV)

    def leaves():
        return [t.to(DEV).requires_grad_() for t in (x, w_b, w_c, delta, lam, s, dk)]

    a = leaves()
    bc_proj_scan(*a).backward(gy)
    b = leaves()
    _unfused(*b).backward(gy)
    for name, ta, tb in zip(("x", "w_b", "w_c", "delta", "Lambda", "s", "D"), a, b):
        assert rel_l2(ta.grad.float(), tb.grad.float()) < 1e-5, name


@pytest.mark.parametrize("dm,ds", [(128, 16), (256, 64)])
def test_block_fused_bc_proj_matches_unfused(dm, ds):
    """QuaternionMamba2Block under bf16 autocast with ``fused_bc_proj`` against
    the same block with cuBLAS projections: output and every parameter gradient
    (config 1: d_model 128, d_state 16; and d_state 64)."""
    from mambaqc_b200.models import QuaternionMamba2Block
    torch.manual_seed(0)
    blk = QuaternionMamba2Block(dm, d_state=ds).to(DEV)
    g = torch.Generator(device=DEV).manual_seed(1)
    x = torch.randn(2, 256, dm, generator=g, device=DEV)
    gout = torch.randn(2, 256, dm, generator=g, device=DEV)
    res = {}
    for fused in (False, True):
        blk.zero_grad(set_to_none=True)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            out = blk(x, fused_bc_proj=fused)
        (out.float() * gout).sum().backward()
        res[fused] = (out.detach().float(), {n: p.grad.detach().float().clone()
                                             for n, p in blk.named_parameters()})
    torch.cuda.synchronize()
    assert rel_l2(res[True][0], res[False][0]) < UNFUSED_TOL
    for n in res[False][1]:
        assert rel_l2(res[True][1][n], res[False][1][n]) < 2e-2, n
