"""The quaternion LayerNorm fused into the output projection
(``quaternion_layer_norm_linear`` -> ``mqc_qln_linear_fwd``, a tcgen05 GEMM
whose operand prologue is the LayerNorm).

Checked against (a) the unfused pair -- the LayerNorm kernel's bf16 output fed
to cuBLAS -- whose bf16 operands differ only where the fused prologue's
Newton-refined reciprocal rounds differently, so the GEMM's summation order and
the output rounding dominate (rel-L2 < 4e-3); and (b) the fp64 oracle
(LayerNorm restated from the reference, then the linear map), within the bf16
tolerance of the contract (2e-2). Gradients of every input against torch
autograd through the unfused pair."""

import pytest
import torch
import torch.nn.functional as F

from oracle import ref
from tests.gpu_util import DEV, RTOL_BF16, gen, rel_l2

pytestmark = pytest.mark.gpu

from mambaqc_b200.kernels import quaternion_layer_norm_fused  # noqa: E402
from mambaqc_b200.kernels.quaternion_norm import quaternion_layer_norm_linear  # noqa: E402

UNFUSED_TOL = 4e-3


def _inputs(bsz, seqlen, dm, nout, bias, seed):
    g = gen(seed)
    q = torch.randn(bsz, seqlen, dm, 4, generator=g)
    gamma = 1.0 + 0.2 * torch.randn(dm, generator=g)
    beta = 0.1 * torch.randn(dm, 4, generator=g)
    w = torch.randn(nout, 4 * dm, generator=g) / (4 * dm) ** 0.5
    b = 0.1 * torch.randn(nout, generator=g) if bias else None
    return q, gamma, beta, w, b


@pytest.mark.parametrize("shape,bias", [((2, 64, 32, 96), False),      # one M tile, N < BN
                                        ((1, 300, 48, 300), True),     # ragged M and N tiles
                                        ((4, 2048, 1536, 768), False)])  # the config-4 block
def test_qln_linear_matches_unfused_and_oracle(shape, bias):
    bsz, seqlen, dm, nout = shape
    q, gamma, beta, w, b = _inputs(bsz, seqlen, dm, nout, bias, seed=sum(shape))
    qd = q.to(DEV, torch.bfloat16)
    gd, bd = gamma.to(DEV), beta.to(DEV)
    wd = w.to(DEV, torch.bfloat16)
    bb = b.to(DEV, torch.bfloat16) if b is not None else None
    out = quaternion_layer_norm_linear(qd, gd, bd, wd, bb)
    yn = quaternion_layer_norm_fused(qd, gd, bd)
    unfused = F.linear(yn.reshape(bsz, seqlen, 4 * dm), wd, bb)
    torch.cuda.synchronize()
    assert out.shape == (bsz, seqlen, nout) and out.dtype == torch.bfloat16
    assert rel_l2(out.float(), unfused.float()) < UNFUSED_TOL
    # fp64 oracle on the bf16-rounded inputs, a row sample for the big shape
    rows = slice(None) if bsz * seqlen <= 4096 else slice(0, 256)
    q64 = qd.double().cpu().reshape(bsz * seqlen, dm, 4)[rows]
    yn64 = ref.layer_norm(q64[None], gamma.double(), beta.double())[0]
    want = yn64.reshape(yn64.shape[0], 4 * dm) @ wd.double().cpu().t()
    if bb is not None:
        want = want + bb.double().cpu()
    got = out.reshape(bsz * seqlen, nout)[rows]
    assert rel_l2(got.float(), want) < RTOL_BF16


def test_qln_linear_backward_matches_unfused():
    bsz, seqlen, dm, nout = 2, 160, 64, 128
    q, gamma, beta, w, b = _inputs(bsz, seqlen, dm, nout, True, seed=5)
    gout = torch.randn(bsz, seqlen, nout, generator=gen(6)).to(DEV, torch.bfloat16)

    def leaves():
        return (q.to(DEV, torch.bfloat16).requires_grad_(), gamma.to(DEV).requires_grad_(),
                beta.to(DEV).requires_grad_(), w.to(DEV, torch.bfloat16).requires_grad_(),
                b.to(DEV, torch.bfloat16).requires_grad_())

    fused = leaves()
    (quaternion_layer_norm_linear(*fused).float() * gout.float()).sum().backward()
    plain = leaves()
    yn = quaternion_layer_norm_fused(plain[0], plain[1], plain[2])
    (F.linear(yn.reshape(bsz, seqlen, 4 * dm), plain[3], plain[4]).float() *
     gout.float()).sum().backward()
    torch.cuda.synchronize()
    for name, a, c in zip(("q", "gamma", "beta", "weight", "bias"), fused, plain):
        err = rel_l2(a.grad.float(), c.grad.float())
        assert err < 1e-2, (name, err)


def test_qln_linear_rejects_unsupported_width():
    q = torch.zeros(1, 8, 20, 4, device=DEV, dtype=torch.bfloat16)  # 20 is not a multiple of 16
    w = torch.zeros(8, 80, device=DEV, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="multiple of 16"):
        quaternion_layer_norm_linear(q, torch.ones(20, device=DEV), torch.zeros(20, 4, device=DEV),
                                     w)


def test_block_fused_norm_out_proj_matches_unfused():
    """QuaternionMamba2Block under bf16 autocast with ``fused_norm_out_proj``
    against the same block with the LayerNorm kernel + cuBLAS: output and every
    parameter gradient."""
    from mambaqc_b200.models import QuaternionMamba2Block
    torch.manual_seed(0)
    blk = QuaternionMamba2Block(128, d_state=16).to(DEV)
    g = torch.Generator(device=DEV).manual_seed(2)
    x = torch.randn(2, 200, 128, generator=g, device=DEV)
    gout = torch.randn(2, 200, 128, generator=g, device=DEV)
    res = {}
    for fused in (False, True):
        blk.fused_norm_out_proj = fused
        blk.zero_grad(set_to_none=True)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            out = blk(x)
        (out.float() * gout).sum().backward()
        res[fused] = (out.detach().float(), {n: p.grad.detach().float().clone()
                                             for n, p in blk.named_parameters()})
    torch.cuda.synchronize()
    assert rel_l2(res[True][0], res[False][0]) < UNFUSED_TOL
    for n in res[False][1]:
        assert rel_l2(res[True][1][n], res[False][1][n]) < 2e-2, n
