"""Config 1: one QuaternionMamba2Block forward (fp32), d_model=128, d_state=16,
d_conv=4, expand_factor=2, batch=2, seq_len=256, default torch init under seed 0,
Lambda overridden with Re = -exp(U(log 1e-3, log 1e-1)), Im ~ N(0, 0.5). The
block output and the final SSM state are compared with the fp64 CPU oracle of the
reference block (same weights), plus the golden block made by the reference."""

import pytest
import torch

from oracle import ref
from tests.gpu_util import DEV, RTOL_BF16, RTOL_F32, gen, make_lambda, rel_l2

pytestmark = pytest.mark.gpu

from mambaqc_b200.models import QuaternionMamba2Block  # noqa: E402


def test_golden_block(golden):
    c = golden["block_f64"]
    blk = QuaternionMamba2Block(16, d_state=4).to(DEV)
    blk.load_state_dict({k: v.float() for k, v in c["state_dict"].items()})
    with torch.no_grad():
        out = blk(c["x"].to(DEV, torch.float32))
    assert rel_l2(out, c["out"]) < RTOL_F32


def test_config1_block_forward_and_state():
    torch.manual_seed(0)
    blk = QuaternionMamba2Block(128, d_state=16, d_conv=4, expand_factor=2)
    g = gen(0)
    x = torch.randn(2, 256, 128, generator=g)
    lam = make_lambda(256, 16, g)
    params = {k: v.double() for k, v in blk.state_dict().items()}
    out_ref, h_ref = ref.block_forward(params, x.double(), d_state=16, Lam=lam, return_state=True)
    blk = blk.to(DEV)
    blk.lambda_override = lam.to(DEV, torch.float32)
    with torch.no_grad():
        out, h_T = blk(x.to(DEV), return_ssm_state=True)
    assert rel_l2(out, out_ref) < RTOL_F32
    assert rel_l2(h_T, h_ref) < RTOL_F32


def test_block_backward_matches_oracle_autograd():
    """Forward + backward of a whole block (config-1 width, shorter sequence): every
    parameter's gradient and the input gradient against torch autograd through the
    fp64 oracle block. cuDNN TF32 is switched off so the conv runs in fp32."""
    prev = torch.backends.cudnn.allow_tf32
    torch.backends.cudnn.allow_tf32 = False
    try:
        torch.manual_seed(0)
        blk = QuaternionMamba2Block(128, d_state=16, d_conv=4, expand_factor=2)
        g = gen(3)
        x = torch.randn(2, 64, 128, generator=g)
        gout = torch.randn(2, 64, 128, generator=g)
        params = {k: v.detach().double().requires_grad_() for k, v in blk.state_dict().items()}
        xr = x.double().requires_grad_()
        out_ref = ref.block_forward(params, xr, d_state=16)
        (out_ref * gout.double()).sum().backward()
        blk = blk.to(DEV)
        xg = x.to(DEV).requires_grad_()
        out = blk(xg)
        (out * gout.to(DEV)).sum().backward()
        assert rel_l2(out, out_ref.detach()) < RTOL_F32
        assert rel_l2(xg.grad, xr.grad) < 1e-4
        for name, p in blk.named_parameters():
            err = rel_l2(p.grad, params[name].grad)
            assert err < 1e-4, (name, err)
    finally:
        torch.backends.cudnn.allow_tf32 = prev


def test_config4_block_shape_bf16_autocast():
    """The config-4 base block (d_model 768, d_state 64, d_inner 1536) at B=4,
    T=2048 under bf16 autocast, forward and backward, against the fp64 oracle
    block. The GPU runs the whole shape; the checks use what a sample can pin:
    * the block is causal, so with an upstream gradient that is zero outside
      batch row 0 and steps [0, T0), the output there and every parameter
      gradient depend only on x[0, :T0]; the oracle block runs that prefix;
    * channels are independent recurrences, so the final SSM state of sampled
      channels (all 2048 steps, every batch row) is checked against the oracle
      SSM on those channels alone.
    The projection weights are 604 M parameters each; their gradients are
    compared on the rows of the sampled channels. Tolerance: bf16 (2e-2)."""
    bsz, seqlen, dmod, nst, t0 = 4, 2048, 768, 64, 45
    torch.manual_seed(0)
    blk = QuaternionMamba2Block(dmod, d_state=nst)
    g = gen(4)
    x = torch.randn(bsz, seqlen, dmod, generator=g)
    gout = torch.zeros(bsz, seqlen, dmod)
    gout[0, :t0] = torch.randn(t0, dmod, generator=g)
    params = {k: v.detach().double() for k, v in blk.state_dict().items()}
    blk = blk.to(DEV)
    xg = x.to(DEV).requires_grad_()
    with torch.autocast("cuda", dtype=torch.bfloat16):
        out, h_T = blk(xg, return_ssm_state=True)
    (out.float() * gout.to(DEV)).sum().backward()
    torch.cuda.synchronize()
    from mambaqc_b200 import _lib
    _lib.check_device_status(torch.device(DEV))
    assert torch.isfinite(out.float()).all() and torch.isfinite(h_T).all()

    chans = torch.tensor([0, 700, 1535])
    for b in (0, 3):
        _, h_ref = ref.block_ssm_channels(params, x[b:b + 1].double(), nst, chans)
        assert rel_l2(h_T[b:b + 1, chans.to(DEV)], h_ref) < RTOL_BF16

    leaves = {k: v.clone().requires_grad_() for k, v in params.items()}
    xr = x[:1, :t0].double().requires_grad_()
    out_ref = ref.block_forward(leaves, xr, d_state=nst)
    (out_ref * gout[:1, :t0].double()).sum().backward()
    assert rel_l2(out[:1, :t0], out_ref.detach()) < RTOL_BF16
    assert rel_l2(xg.grad[:1, :t0], xr.grad) < RTOL_BF16
    rows = (chans[:, None] * (nst * 4) + torch.arange(nst * 4)).reshape(-1)
    for name, p in blk.named_parameters():
        want = leaves[name].grad
        got = p.grad
        if name in ("B_proj.weight", "C_proj.weight"):
            got, want = got[rows.to(DEV)], want[rows]
        err = rel_l2(got, want)
        assert err < RTOL_BF16, (name, err)
