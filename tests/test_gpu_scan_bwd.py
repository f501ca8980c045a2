"""GPU parity of the scan backward (mqc_ssm_scan_bwd through ssm_scan_cayley's
autograd) against torch autograd through the fp64 CPU oracle of the reference
composition (delta*Lambda -> Cayley -> sequential scan). Relative L2 per
gradient: 1e-5 for fp32 inputs (the forward contract's tolerance), 2e-2 for
bf16 inputs with the fp32 state."""

import math

import pytest
import torch

from oracle import ref
from tests.gpu_util import DEV, RTOL_BF16, RTOL_F32, gen, make_scan_inputs, rel_l2, to_dev

pytestmark = pytest.mark.gpu

from mambaqc_b200.kernels import ssm_scan_cayley  # noqa: E402

NAMES = ("delta", "Lambda", "B", "C", "S", "D")


def oracle_grads(inp, gy, h0=None, ghT=None):
    leaves = {k: v.clone().requires_grad_() for k, v in inp.items()}
    h0l = None if h0 is None else h0.clone().requires_grad_()
    y, hT = ref.ssm_scan_cayley(*(leaves[k] for k in NAMES), h0=h0l)
    loss = (y * gy).sum()
    if ghT is not None:
        loss = loss + (hT * ghT).sum()
    loss.backward()
    out = {k: leaves[k].grad for k in NAMES}
    if h0l is not None:
        out["h0"] = h0l.grad
    return y, out


def gpu_grads(inp, gy, dtype, h0=None, ghT=None):
    d = {k: v.requires_grad_() for k, v in to_dev(inp, dtype).items()}
    h0d = None if h0 is None else h0.to(DEV, torch.float32).requires_grad_()
    y, hT = ssm_scan_cayley(*(d[k] for k in NAMES), h0=h0d, return_final_state=True)
    loss = (y.float() * gy.to(DEV, torch.float32)).sum()
    if ghT is not None:
        loss = loss + (hT * ghT.to(DEV, torch.float32)).sum()
    loss.backward()
    out = {k: d[k].grad for k in NAMES}
    if h0d is not None:
        out["h0"] = h0d.grad
    return y, out


CASES = [
    # (B, T, D, N, shared, s_real)
    (2, 37, 8, 16, True, True),
    (2, 37, 8, 16, False, True),
    (2, 37, 8, 16, True, False),
    (2, 37, 8, 16, False, False),
    (1, 24, 5, 64, True, True),     # T a multiple of the checkpoint interval
    (3, 9, 6, 3, True, True),       # masked state lanes
    (1, 19, 3, 100, True, False),   # G = 4
    (1, 8, 4, 16, True, True),      # one sub-block, no checkpoints
    (2, 1, 4, 16, False, True),     # T = 1
    (2, 40, 6, 64, False, True),    # per-channel B/C at d_state 64 (the block's layout)
    (2, 40, 6, 64, False, False),
    (1, 77, 9, 64, False, True),    # ragged sub-blocks, odd channel count
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: "B{}T{}D{}N{}{}{}".format(
    c[0], c[1], c[2], c[3], "sh" if c[4] else "pc", "x" if c[5] else "S"))
def test_scan_backward_fp32(case):
    bsz, seqlen, dm, ds, shared, s_real = case
    inp = make_scan_inputs(bsz, seqlen, dm, ds, shared=shared, s_real=s_real, seed=sum(case[:4]))
    g = gen(7 + sum(case[:4]))
    gy = torch.randn(bsz, seqlen, dm, 4, generator=g, dtype=torch.float64)
    h0 = torch.randn(bsz, dm, ds, 4, generator=g, dtype=torch.float64)
    ghT = torch.randn(bsz, dm, ds, 4, generator=g, dtype=torch.float64)
    y_ref, g_ref = oracle_grads(inp, gy, h0=h0, ghT=ghT)
    y, g_gpu = gpu_grads(inp, gy, torch.float32, h0=h0, ghT=ghT)
    assert rel_l2(y, y_ref) < RTOL_F32
    for k in (*NAMES, "h0"):
        err = rel_l2(g_gpu[k], g_ref[k])
        assert err < RTOL_F32, (k, err)


@pytest.mark.parametrize("shared,s_real,dm", [(True, True, 16), (False, True, 16),
                                              (False, False, 16), (False, True, 9),
                                              (False, False, 7)])
def test_scan_backward_bf16(shared, s_real, dm):
    # odd channel counts put consecutive steps of a bf16 delta / x in alternating
    # halves of a 32-bit word
    inp = make_scan_inputs(2, 40, dm, 64, shared=shared, s_real=s_real, seed=5)
    gy = torch.randn(2, 40, dm, 4, generator=gen(6), dtype=torch.float64)
    h0 = torch.randn(2, dm, 64, 4, generator=gen(7), dtype=torch.float64)
    _, g_ref = oracle_grads(inp, gy, h0=h0)
    _, g_gpu = gpu_grads(inp, gy, torch.bfloat16, h0=h0)
    for k in (*NAMES, "h0"):
        assert rel_l2(g_gpu[k], g_ref[k]) < RTOL_BF16, k
    # against the oracle on the bf16-rounded inputs the error is the rounding of
    # the gradients themselves
    rounded = {k: (v if k in ("Lambda", "D") else v.to(torch.bfloat16).double())
               for k, v in inp.items()}
    _, g_rr = oracle_grads(rounded, gy.float().double(), h0=h0)
    for k in ("delta", "B", "C", "S"):
        assert rel_l2(g_gpu[k], g_rr[k]) < 1e-2, k


def test_scan_backward_without_final_state_gradient_and_no_h0():
    inp = make_scan_inputs(1, 30, 4, 16, shared=False, s_real=False, seed=9)
    gy = torch.randn(1, 30, 4, 4, generator=gen(10), dtype=torch.float64)
    _, g_ref = oracle_grads(inp, gy)
    d = {k: v.requires_grad_() for k, v in to_dev(inp, torch.float32).items()}
    y = ssm_scan_cayley(*(d[k] for k in NAMES))  # no h0, h_T not returned
    (y * gy.to(DEV, torch.float32)).sum().backward()
    for k in NAMES:
        assert rel_l2(d[k].grad, g_ref[k]) < RTOL_F32, k


def test_skip_weight_gradient_layouts():
    """D given as [D] and as the reference's stride-0 [B,T,D] expand of a [D] leaf."""
    inp = make_scan_inputs(2, 20, 6, 8, seed=11)
    gy = torch.randn(2, 20, 6, 4, generator=gen(12), dtype=torch.float64)
    _, g_ref = oracle_grads(inp, gy)
    d = to_dev(inp, torch.float32)
    Dleaf = d["D"].clone().requires_grad_()
    y = ssm_scan_cayley(d["delta"], d["Lambda"], d["B"], d["C"], d["S"],
                        Dleaf.view(1, 1, 6).expand(2, 20, 6))
    (y * gy.to(DEV, torch.float32)).sum().backward()
    assert rel_l2(Dleaf.grad, g_ref["D"]) < RTOL_F32


def test_config3_full_size_backward_channel_sample():
    """Forward + backward at config 3 (B=4, T=2048, D=1536, N=64, shared B/C):
    channels are independent recurrences, so ddelta, dx and dLambda of sampled
    channels are checked against the oracle run on those channels alone."""
    bsz, seqlen, dm, ds = 4, 2048, 1536, 64
    g = gen(0)
    x = torch.randn(bsz, seqlen, dm, generator=g)
    delta = torch.nn.functional.softplus(torch.randn(bsz, seqlen, dm, generator=g) - 3.0)
    lam = torch.empty(dm, ds, 4)
    lam[..., 0] = -torch.exp(torch.empty(dm, ds).uniform_(math.log(1e-3), math.log(1e-1),
                                                          generator=g))
    lam[..., 1:] = 0.5 * torch.randn(dm, ds, 3, generator=g)
    Bm = torch.randn(bsz, seqlen, ds, 4, generator=g) / 8
    Cm = torch.randn(bsz, seqlen, ds, 4, generator=g) / 8
    Dk = torch.ones(dm)
    gy = torch.randn(bsz, seqlen, dm, 4, generator=g)
    dv = delta.to(DEV).requires_grad_()
    lv = lam.to(DEV).requires_grad_()
    xv = x.to(DEV).requires_grad_()
    y = ssm_scan_cayley(dv, lv, Bm.to(DEV), Cm.to(DEV), xv, Dk.to(DEV))
    (y * gy.to(DEV)).sum().backward()
    chans = torch.tensor([0, 41, 777, 1535])
    b = 2
    inp = dict(delta=delta[b:b + 1, :, chans].double(), Lambda=lam[chans].double(),
               B=Bm[b:b + 1].double(), C=Cm[b:b + 1].double(), S=x[b:b + 1, :, chans].double(),
               D=Dk[chans].double())
    _, g_ref = oracle_grads(inp, gy[b:b + 1, :, chans].double())
    cd = chans.to(DEV)
    assert rel_l2(dv.grad[b:b + 1, :, cd], g_ref["delta"]) < RTOL_F32
    assert rel_l2(xv.grad[b:b + 1, :, cd], g_ref["S"]) < RTOL_F32
    # dLambda sums over all 4 batches; the oracle saw batch b only -> compare the
    # per-batch contribution by rerunning the GPU backward on that batch alone
    lv2 = lam.to(DEV).requires_grad_()
    y2 = ssm_scan_cayley(delta[b:b + 1].to(DEV), lv2, Bm[b:b + 1].to(DEV), Cm[b:b + 1].to(DEV),
                         x[b:b + 1].to(DEV), Dk.to(DEV))
    (y2 * gy[b:b + 1].to(DEV)).sum().backward()
    assert rel_l2(lv2.grad[cd], g_ref["Lambda"]) < RTOL_F32


def _config3_perchannel_inputs(dtype, seed):
    """Config-3 inputs with the reference block's per-channel B/C
    [4, 2048, 1536, 64, 4], generated on the GPU (25.8 GB in fp32); the sampled
    channels are copied to the CPU for the oracle, so both see the same bits."""
    bsz, seqlen, dm, ds = 4, 2048, 1536, 64
    g = torch.Generator(device=DEV).manual_seed(seed)
    x = torch.randn(bsz, seqlen, dm, generator=g, device=DEV)
    delta = torch.nn.functional.softplus(torch.randn(bsz, seqlen, dm, generator=g, device=DEV) - 3)
    lam = torch.empty(dm, ds, 4, device=DEV)
    lam[..., 0] = -torch.exp(torch.empty(dm, ds, device=DEV).uniform_(
        math.log(1e-3), math.log(1e-1), generator=g))
    lam[..., 1:] = 0.5 * torch.randn(dm, ds, 3, generator=g, device=DEV)
    Bm = (torch.randn(bsz, seqlen, dm, ds, 4, generator=g, device=DEV) / 8).to(dtype)
    Cm = (torch.randn(bsz, seqlen, dm, ds, 4, generator=g, device=DEV) / 8).to(dtype)
    Dk = 1.0 + 0.1 * torch.randn(dm, generator=g, device=DEV)
    gy = torch.randn(bsz, seqlen, dm, 4, generator=g, device=DEV)
    return dict(delta=delta.to(dtype), Lambda=lam, B=Bm, C=Cm, S=x.to(dtype), D=Dk), gy


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_config3_perchannel_full_size_forward_backward_channel_sample(dtype):
    """Forward + backward at config 3 with per-channel B/C (B=4, T=2048, D=1536,
    N=64), the layout the reference block feeds the scan: y, h_T and every
    gradient of sampled channels against the fp64 oracle run on those channels
    alone (channels are independent recurrences). bf16 inputs are checked
    against the oracle on the same bf16-rounded values (and the bf16-rounded
    upstream gradient the backward receives), so the tolerance covers the
    kernel's fp32 arithmetic and its bf16 output rounding."""
    from mambaqc_b200 import _lib
    inp, gy = _config3_perchannel_inputs(dtype, seed=11 if dtype == torch.float32 else 12)
    leaves = {k: v.requires_grad_() for k, v in inp.items()}
    y, hT = ssm_scan_cayley(*(leaves[k] for k in NAMES), return_final_state=True)
    (y.float() * gy).sum().backward()
    torch.cuda.synchronize()
    _lib.check_device_status(torch.device(DEV))
    f32 = dtype == torch.float32
    tol_y = RTOL_F32 if f32 else RTOL_BF16
    tol_g = RTOL_F32 if f32 else 1e-2
    gy_ref = gy.to(dtype).double().cpu()
    cd = torch.tensor([0, 41, 777, 1535], device=DEV)

    def sample_of(src, b):
        s = dict(delta=src["delta"][b:b + 1, :, cd], Lambda=inp["Lambda"][cd],
                 B=src["B"][b:b + 1, :, cd], C=src["C"][b:b + 1, :, cd],
                 S=src["S"][b:b + 1, :, cd], D=inp["D"][cd])
        return {k: v.detach().double().cpu() for k, v in s.items()}

    for b in (0, 3):
        smp = sample_of(inp, b)
        leaves_ref = {k: v.clone().requires_grad_() for k, v in smp.items()}
        y_ref, h_ref = ref.ssm_scan_cayley(*(leaves_ref[k] for k in NAMES))
        (y_ref * gy_ref[b:b + 1, :, cd.cpu()]).sum().backward()
        assert rel_l2(y[b:b + 1, :, cd], y_ref) < tol_y
        assert rel_l2(hT[b:b + 1, cd], h_ref) < RTOL_F32
        for k in ("delta", "S", "B", "C"):
            err = rel_l2(leaves[k].grad[b:b + 1, :, cd], leaves_ref[k].grad)
            assert err < tol_g, (k, err)
    # dLambda and dD sum over the batch: the contribution of row b alone is
    # checked by rerunning the GPU backward on that row
    b = 1
    one = {k: (v.detach()[b:b + 1] if k not in ("Lambda", "D") else v.detach().clone())
           for k, v in inp.items()}
    lam1 = one["Lambda"].requires_grad_()
    d1 = one["D"].requires_grad_()
    y1 = ssm_scan_cayley(one["delta"], lam1, one["B"], one["C"], one["S"], d1)
    (y1.float() * gy[b:b + 1]).sum().backward()
    smp = sample_of(one, 0)
    _, g_ref = oracle_grads(smp, gy_ref[b:b + 1, :, cd.cpu()])
    assert rel_l2(lam1.grad[cd], g_ref["Lambda"]) < tol_g
    assert rel_l2(d1.grad[cd], g_ref["D"]) < tol_g
    assert torch.isfinite(y.float()).all()
