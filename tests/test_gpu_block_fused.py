"""The block's fused glue kernels against the torch ops they replace (forward
and backward, fp32 and bf16): the causal conv + SiLU read in place from the
in_proj output, softplus / sigmoid-gate scan inputs, and the output gate +
residual. fp32 is held to rel-L2 1e-5, bf16 to 2e-2."""

import pytest
import torch
import torch.nn.functional as F

from tests.gpu_util import DEV, RTOL_BF16, RTOL_F32, gen, rel_l2

pytestmark = pytest.mark.gpu

from mambaqc_b200.kernels import causal_conv1d_silu, gate_residual, ssm_scan_inputs  # noqa: E402


def _tol(dt):
    return RTOL_F32 if dt == torch.float32 else RTOL_BF16


def _conv_silu_ref(x, w, b):
    k = w.shape[-1]
    xt = F.pad(x.transpose(1, 2), (k - 1, 0))
    return F.silu(F.conv1d(xt, w, b, groups=x.shape[2]).transpose(1, 2))


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("shape", [(2, 256, 256, 4), (3, 37, 20, 4), (1, 5, 7, 3), (2, 70, 12, 8),
                                   (1, 100, 64, 1)])
def test_conv_silu_forward_backward(shape, dt):
    bsz, seqlen, dm, k = shape
    g = gen(sum(shape))
    xz = torch.randn(bsz, seqlen, 2 * dm, generator=g).to(DEV, dt)
    w = (torch.randn(dm, 1, k, generator=g) * 0.5).to(DEV)
    b = (torch.randn(dm, generator=g) * 0.1).to(DEV)
    gout = torch.randn(bsz, seqlen, dm, generator=g).to(DEV, dt)

    xz1 = xz.clone().requires_grad_()
    w1, b1 = w.clone().requires_grad_(), b.clone().requires_grad_()
    y1 = causal_conv1d_silu(xz1[..., :dm], w1, b1)
    (y1.float() * gout.float()).sum().backward()

    xz2 = xz.double().requires_grad_()
    w2, b2 = w.double().requires_grad_(), b.double().requires_grad_()
    y2 = _conv_silu_ref(xz2[..., :dm], w2, b2)
    (y2 * gout.double()).sum().backward()

    assert y1.dtype == dt
    tol = _tol(dt)
    assert rel_l2(y1, y2) < tol
    assert rel_l2(xz1.grad[..., :dm], xz2.grad[..., :dm]) < tol
    assert torch.count_nonzero(xz1.grad[..., dm:]) == 0
    # the parameter gradients sum over (b, t): bf16 inputs round each term
    assert rel_l2(w1.grad, w2.grad) < tol
    assert rel_l2(b1.grad, b2.grad) < tol


def test_conv_silu_without_bias_and_padded_rows():
    g = gen(9)
    x = torch.randn(2, 33, 16, generator=g).to(DEV)
    w = torch.randn(16, 1, 4, generator=g).to(DEV)
    y = causal_conv1d_silu(x, w, None)
    assert rel_l2(y, _conv_silu_ref(x.double(), w.double(), None)) < RTOL_F32
    # a row stride that is not a multiple of 4 takes the one-channel path
    wide = torch.randn(2, 33, 19, generator=g).to(DEV)
    y2 = causal_conv1d_silu(wide[..., 1:17], w, None)
    assert rel_l2(y2, _conv_silu_ref(wide[..., 1:17].double(), w.double(), None)) < RTOL_F32


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("dm", [256, 30])
def test_scan_inputs_forward_backward(dt, dm):
    g = gen(dm)
    u = (torch.randn(3, 50, dm, generator=g) * 8).to(DEV, dt)   # crosses the threshold 20
    u[0, 0, :4] = torch.tensor([25.0, -30.0, 20.0, 19.9])
    gate = torch.randn(3, 50, dm, generator=g).to(DEV, dt)
    x = torch.randn(3, 50, dm, generator=g).to(DEV, dt)
    gd = torch.randn(3, 50, dm, generator=g).to(DEV, dt)
    gs = torch.randn(3, 50, dm, generator=g).to(DEV, dt)

    ins1 = [t.clone().requires_grad_() for t in (u, gate, x)]
    d1, s1 = ssm_scan_inputs(*ins1)
    (d1.float() * gd.float() + s1.float() * gs.float()).sum().backward()

    ins2 = [t.double().requires_grad_() for t in (u, gate, x)]
    d2 = F.softplus(ins2[0])
    s2 = torch.sigmoid(ins2[1]) * ins2[2]
    (d2 * gd.double() + s2 * gs.double()).sum().backward()

    tol = _tol(dt)
    assert d1.dtype == dt and s1.dtype == dt
    assert rel_l2(d1, d2) < tol and rel_l2(s1, s2) < tol
    for a, b in zip(ins1, ins2):
        assert rel_l2(a.grad, b.grad) < tol


def test_scan_inputs_one_output_unused():
    g = gen(4)
    u, gate, x = (torch.randn(2, 8, 12, generator=g).to(DEV).requires_grad_() for _ in range(3))
    d, s = ssm_scan_inputs(u, gate, x)
    d.sum().backward()
    assert rel_l2(u.grad, torch.sigmoid(u.detach())) < RTOL_F32
    assert torch.count_nonzero(gate.grad) == 0 and torch.count_nonzero(x.grad) == 0


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_gate_residual_forward_backward(dt):
    g = gen(21)
    x = torch.randn(2, 40, 128, generator=g).to(DEV, dt)
    xz = torch.randn(2, 40, 512, generator=g).to(DEV, dt)
    y = torch.randn(2, 40, 128, generator=g).to(DEV, dt)
    gout = torch.randn(2, 40, 128, generator=g).to(DEV, dt)

    x1, xz1, y1 = (t.clone().requires_grad_() for t in (x, xz, y))
    o1 = gate_residual(x1, xz1[..., 256:384], y1)
    (o1.float() * gout.float()).sum().backward()
    x2, xz2, y2 = (t.double().requires_grad_() for t in (x, xz, y))
    o2 = x2 + torch.sigmoid(xz2[..., 256:384]) * y2
    (o2 * gout.double()).sum().backward()

    tol = _tol(dt)
    assert rel_l2(o1, o2) < tol
    assert rel_l2(x1.grad, x2.grad) < tol
    assert rel_l2(xz1.grad, xz2.grad) < tol
    assert rel_l2(y1.grad, y2.grad) < tol


def test_block_under_bf16_autocast_matches_fp32():
    """The block in bf16 autocast (bf16 activations through every fused kernel,
    fp32 scan state) against the same block in fp32."""
    from mambaqc_b200.models import QuaternionMamba2Block
    torch.manual_seed(0)
    blk = QuaternionMamba2Block(128, d_state=16).to(DEV)
    x = torch.randn(2, 128, 128, generator=gen(2)).to(DEV)
    with torch.no_grad():
        ref_out = blk(x)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            out = blk(x)
    assert rel_l2(out.float(), ref_out) < RTOL_BF16
