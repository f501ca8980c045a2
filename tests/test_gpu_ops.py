"""GPU parity of the elementwise ops, prefix product and LayerNorm (through the
C ABI via the reference-shaped Python API) against the CPU oracle and the golden
fixtures made from the reference. Ports the reference's own property tests
(mambaqc/tests/test_quaternion_ops.py) to the CUDA path."""

import pytest
import torch

from oracle import ref
from tests.gpu_util import DEV, RTOL_BF16, RTOL_F32, gen, rel_l2

pytestmark = pytest.mark.gpu

from mambaqc_b200.kernels import (  # noqa: E402
    cayley_discretization_fused,
    parallel_scan_quaternion,
    quaternion_conjugate,
    quaternion_inverse,
    quaternion_layer_norm_fused,
    quaternion_multiply,
    quaternion_multiply_batched,
    quaternion_norm,
)
from mambaqc_b200.layers import QuaternionLayerNorm  # noqa: E402


def g32(t):
    return t.to(DEV, torch.float32)


# ---------------------------------------------------------------- golden fixtures

def test_golden_algebra(golden):
    c = golden["qmul_f32"]
    assert rel_l2(quaternion_multiply(g32(c["p"]), g32(c["q"])), c["out"]) < RTOL_F32
    c = golden["qconj_f32"]
    assert torch.equal(quaternion_conjugate(g32(c["q"])).cpu(), c["out"])
    c = golden["qinv_f32"]
    assert rel_l2(quaternion_inverse(g32(c["q"]), 1e-6), c["out"]) < RTOL_F32
    c = golden["qnorm_f32"]
    assert rel_l2(quaternion_norm(g32(c["q"])), c["out"]) < RTOL_F32
    c = golden["qinv_eps_clamp"]
    torch.testing.assert_close(quaternion_inverse(g32(c["q"]), 1e-6).cpu().double(), c["out"],
                               rtol=1e-6, atol=1e-6)
    c = golden["qmul_noncommuting_pair"]
    assert torch.equal(quaternion_multiply(g32(c["p"]), g32(c["q"])).cpu(), c["pq"].float())
    assert torch.equal(quaternion_multiply(g32(c["q"]), g32(c["p"])).cpu(), c["qp"].float())


def test_golden_cayley(golden):
    for name in ("cayley_f64", "cayley_f32", "cayley_stable_f64"):
        c = golden[name]
        assert rel_l2(cayley_discretization_fused(g32(c["z"]), c["eps"]), c["out"]) < RTOL_F32, name
    c = golden["cayley_pole_f64"]  # eps clamp active near z = 2
    z32 = g32(c["z"])
    got = cayley_discretization_fused(z32, c["eps"]).cpu().double()
    # ill-conditioned at the pole: compare with the oracle on the fp32-rounded input
    torch.testing.assert_close(got, ref.cayley(z32.cpu().double(), c["eps"]), rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(got, c["out"], rtol=5e-3, atol=1e-3)


def test_golden_prefix(golden):
    for name in ("prefix_f64", "prefix_f32"):
        c = golden[name]
        assert rel_l2(parallel_scan_quaternion(g32(c["q"])), c["out"]) < RTOL_F32, name


def test_golden_layernorm(golden):
    for dm in (16, 24):
        c = golden[f"layernorm_d{dm}_f64"]
        out = quaternion_layer_norm_fused(g32(c["q"]), g32(c["gamma"]), g32(c["beta"]), c["eps"])
        assert rel_l2(out, c["out"]) < RTOL_F32
    c = golden["layernorm_triton_interp_d24"]
    out = quaternion_layer_norm_fused(g32(c["q"]), g32(c["gamma"]), g32(c["beta"]), 1e-5,
                                      padded_compat=True)
    assert rel_l2(out, c["out"]) < RTOL_F32


# ---------------------------------------------------- reference property tests

def test_reference_properties():
    g = gen(11)
    q = g32(torch.randn(1000, 4, generator=g))
    p = g32(torch.randn(1000, 4, generator=g))
    r = g32(torch.randn(1000, 4, generator=g))
    one = torch.zeros_like(q)
    one[:, 0] = 1
    torch.testing.assert_close(quaternion_multiply(q, one), q, atol=1e-6, rtol=0)
    n2 = (q * q).sum(-1)
    qq = quaternion_multiply(q, quaternion_conjugate(q))
    torch.testing.assert_close(qq[:, 0], n2, atol=1e-5, rtol=1e-6)
    assert qq[:, 1:].abs().max() < 1e-5
    qi = q + 0.5
    torch.testing.assert_close(quaternion_multiply(qi, quaternion_inverse(qi)),
                               one, atol=1e-4, rtol=0)
    torch.testing.assert_close(quaternion_multiply(quaternion_multiply(p, q), r),
                               quaternion_multiply(p, quaternion_multiply(q, r)), atol=1e-4, rtol=1e-4)
    torch.testing.assert_close(quaternion_norm(quaternion_multiply(p, q)),
                               quaternion_norm(p) * quaternion_norm(q), rtol=1e-5, atol=1e-5)
    assert torch.equal(quaternion_conjugate(quaternion_conjugate(q)), q)
    q1 = q + 1.0
    torch.testing.assert_close(quaternion_inverse(quaternion_inverse(q1)), q1, atol=1e-4, rtol=1e-4)
    assert (quaternion_norm(q) >= 0).all()
    z = torch.zeros(2, 4, 8, 16, 4, device=DEV)
    ident = torch.zeros_like(z)
    ident[..., 0] = 1
    assert torch.equal(cayley_discretization_fused(z), ident)
    zs = g32(torch.randn(2, 4, 8, 16, 4, generator=g))
    zs[..., 0] = -zs[..., 0].abs() - 0.5
    assert (quaternion_norm(cayley_discretization_fused(zs)) < 1.0).all()
    seq = torch.zeros(2, 10, 8, 16, 4, device=DEV)
    seq[..., 0] = 1
    assert torch.equal(parallel_scan_quaternion(seq), seq)


@pytest.mark.parametrize("shape", [(5, 4), (3, 7, 4), (2, 3, 5, 7, 4), (0, 4), (1, 4)])
def test_qmul_shapes_and_empty(shape):
    g = gen(3)
    p = torch.randn(*shape, generator=g)
    q = torch.randn(*shape, generator=g)
    out = quaternion_multiply(g32(p), g32(q))
    assert out.shape == p.shape
    if p.numel():
        assert rel_l2(out, ref.qmul(p.double(), q.double())) < RTOL_F32


def test_qmul_large_and_noncontiguous_and_bf16():
    g = gen(4)
    p = torch.randn(1 << 20, 4, generator=g)
    q = torch.randn(1 << 20, 4, generator=g)
    truth = ref.qmul(p.double(), q.double())
    assert rel_l2(quaternion_multiply(g32(p), g32(q)), truth) < RTOL_F32
    pb, qb = p.to(DEV, torch.bfloat16), q.to(DEV, torch.bfloat16)
    assert rel_l2(quaternion_multiply(pb, qb), truth) < RTOL_BF16
    p5 = g32(torch.randn(2, 3, 6, 5, 4, generator=g)).transpose(1, 2)  # non-contiguous
    q5 = g32(torch.randn(2, 6, 3, 5, 4, generator=g))
    out = quaternion_multiply_batched(p5, q5)
    assert rel_l2(out, ref.qmul(p5.cpu().double(), q5.cpu().double())) < RTOL_F32


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_qmul_batched_reads_strided_inputs_in_place(dtype, monkeypatch):
    """quaternion_multiply_batched on permuted, sliced and broadcast operands goes
    through the strided kernel (no contiguous copy) and matches the oracle."""
    from mambaqc_b200.kernels import quaternion_ops as qo

    def no_copy(*a, **k):
        raise AssertionError("strided operands were copied to the dense path")

    monkeypatch.setattr(qo, "_qmul_raw", no_copy)
    g = gen(41)
    tol = RTOL_F32 if dtype == torch.float32 else RTOL_BF16
    base_p = torch.randn(3, 2 * 37, 16, 24, 4, generator=g)
    base_q = torch.randn(3, 37, 24, 16, 4, generator=g)
    p = base_p.to(DEV, dtype)[:, ::2]                    # every other step
    q = base_q.to(DEV, dtype).transpose(2, 3)            # d_model <-> d_state
    out = quaternion_multiply_batched(p, q)
    assert out.shape == p.shape and out.is_contiguous()
    assert rel_l2(out, ref.qmul(p.cpu().double(), q.cpu().double())) < tol
    # a broadcast operand (stride 0 over batch and sequence)
    w = torch.randn(1, 1, 16, 24, 4, generator=g).to(DEV, dtype).expand(3, 37, 16, 24, 4)
    out = quaternion_multiply_batched(p, w)
    assert rel_l2(out, ref.qmul(p.cpu().double(), w.cpu().double())) < tol
    # bitwise equal to the dense kernel on the same values
    monkeypatch.undo()
    assert torch.equal(quaternion_multiply_batched(p, q),
                       quaternion_multiply(p.contiguous(), q.contiguous()))


def test_qmul_batched_strided_large_and_gradients():
    """A transposed [2, 256, 768, 64, 4] operand (the config-2 prefix-scan shape)
    and the autograd path of the batched multiply."""
    g = torch.Generator(device=DEV).manual_seed(42)
    p = torch.randn(2, 256, 64, 768, 4, generator=g, device=DEV).transpose(2, 3)
    q = torch.randn(2, 256, 768, 64, 4, generator=g, device=DEV)
    out = quaternion_multiply_batched(p, q)
    sl = (slice(None), slice(0, 256, 17), slice(0, 768, 29))
    assert rel_l2(out[sl], ref.qmul(p[sl].cpu().double(), q[sl].cpu().double())) < RTOL_F32
    del p, q, out
    p64 = torch.randn(2, 5, 3, 7, 4, generator=gen(43), dtype=torch.float64)
    q64 = torch.randn(2, 5, 7, 3, 4, generator=gen(44), dtype=torch.float64).transpose(2, 3)
    w = torch.randn(2, 5, 3, 7, 4, generator=gen(45), dtype=torch.float64)
    pr, qr = p64.clone().requires_grad_(), q64.clone().requires_grad_()
    (ref.qmul(pr, qr) * w).sum().backward()
    pg = g32(p64).requires_grad_()
    qg = g32(q64.transpose(2, 3).contiguous()).transpose(2, 3).detach().requires_grad_()
    (quaternion_multiply_batched(pg, qg) * g32(w)).sum().backward()
    assert rel_l2(pg.grad, pr.grad) < RTOL_F32
    assert rel_l2(qg.grad, qr.grad) < RTOL_F32


def test_qmul_order_matters():
    """Swapping operands must break parity: the Hamilton product is exercised."""
    g = gen(5)
    p = torch.randn(4096, 4, generator=g)
    q = torch.randn(4096, 4, generator=g)
    out = quaternion_multiply(g32(p), g32(q))
    assert rel_l2(out, ref.qmul(q.double(), p.double())) > 0.1


def test_qmul_autograd_matches_oracle():
    g = gen(6)
    p = torch.randn(64, 4, generator=g, dtype=torch.float64)
    q = torch.randn(64, 4, generator=g, dtype=torch.float64)
    w = torch.randn(64, 4, generator=g, dtype=torch.float64)
    pr, qr = p.clone().requires_grad_(), q.clone().requires_grad_()
    (ref.qmul(pr, qr) * w).sum().backward()
    pg, qg = g32(p).requires_grad_(), g32(q).requires_grad_()
    (quaternion_multiply(pg, qg) * g32(w)).sum().backward()
    assert rel_l2(pg.grad, pr.grad) < RTOL_F32
    assert rel_l2(qg.grad, qr.grad) < RTOL_F32


def test_cayley_backward_matches_oracle():
    g = gen(7)
    z = torch.randn(2, 3, 4, 5, 4, generator=g, dtype=torch.float64)
    z[0, 0, 0, 0] = torch.tensor([2.0, 0.0, 0.0, 0.0], dtype=torch.float64)  # clamp active
    w = torch.randn(2, 3, 4, 5, 4, generator=g, dtype=torch.float64)
    zr = z.clone().requires_grad_()
    (ref.cayley(zr, 1e-6) * w).sum().backward()
    zg = g32(z).requires_grad_()
    (cayley_discretization_fused(zg, 1e-6) * g32(w)).sum().backward()
    mask = torch.ones_like(z, dtype=torch.bool)
    mask[0, 0, 0, 0] = False
    assert rel_l2(zg.grad.cpu()[mask], zr.grad[mask]) < 1e-5
    torch.testing.assert_close(zg.grad.cpu().double()[0, 0, 0, 0], zr.grad[0, 0, 0, 0],
                               rtol=1e-4, atol=1e-2)


def test_cayley_denominator_sweep():
    """Real z from -2e3 to just below the pole z = 2: |1 - z/2|^2 spans ~1e-6 .. 1e6, so the
    reciprocal is exercised over 12 decades; every output within a few ulp of fp64."""
    zr = torch.cat([-torch.logspace(-6, 3.3, 4000, dtype=torch.float64),
                    2.0 - torch.logspace(-2.9, 0, 2000, dtype=torch.float64)])
    z = torch.zeros(1, 1, 1, zr.numel(), 4, dtype=torch.float64)
    z[..., 0] = zr
    z[..., 1] = 1e-3 * zr
    z32 = g32(z)
    q = cayley_discretization_fused(z32).cpu().double()
    truth = ref.cayley(z32.cpu().double())
    rel = ((q - truth).norm(dim=-1) / truth.norm(dim=-1)).max().item()
    assert rel < 1e-6, rel


def test_cayley_large_bf16_and_stability():
    g = gen(8)
    z = torch.randn(2, 16, 96, 64, 4, generator=g)
    z[..., 0] = -z[..., 0].abs()
    q = cayley_discretization_fused(g32(z))
    truth = ref.cayley(z.double())
    assert rel_l2(q, truth) < RTOL_F32
    assert (quaternion_norm(q) < 1.0 + 1e-6).all()
    qb = cayley_discretization_fused(z.to(DEV, torch.bfloat16))
    assert rel_l2(qb, truth) < RTOL_BF16


# ------------------------------------------------------------- prefix product

@pytest.mark.parametrize("shape", [(2, 37, 5, 3), (1, 300, 2, 4), (3, 1, 4, 4), (1, 2048, 1, 8)])
def test_prefix_product_shapes(shape):
    """Odd sizes; narrow-and-long shapes take the two-pass chunked path."""
    bsz, seqlen, dm, ds = shape
    g = gen(9)
    u = torch.randn(bsz, seqlen, dm, ds, 4, generator=g, dtype=torch.float64)
    lo = 0.9 if seqlen <= 512 else 0.999  # keep |cum| clear of fp32 underflow for long T
    r = lo + (0.999 - lo) * torch.rand(bsz, seqlen, dm, ds, 1, generator=g, dtype=torch.float64)
    if seqlen > 512:
        r = r + 0.001
    q = u / u.norm(dim=-1, keepdim=True) * r
    out = parallel_scan_quaternion(g32(q))
    truth = ref.prefix_product(q)
    assert rel_l2(out, truth) < RTOL_F32
    # last element equals the manual left product (reference test :257-269)
    manual = q[:, 0]
    for t in range(1, seqlen):
        manual = ref.qmul(q[:, t], manual)
    assert rel_l2(out[:, -1], manual) < RTOL_F32


def test_prefix_bf16():
    g = gen(10)
    u = torch.randn(2, 64, 8, 16, 4, generator=g, dtype=torch.float64)
    q = u / u.norm(dim=-1, keepdim=True) * 0.99
    out = parallel_scan_quaternion(q.to(DEV, torch.bfloat16))
    assert rel_l2(out, ref.prefix_product(q)) < RTOL_BF16


# ----------------------------------------------------------------- LayerNorm

@pytest.mark.parametrize("dm", [1, 7, 24, 768, 1536, 4096])
def test_layernorm_forward(dm):
    g = gen(12)
    q = torch.randn(2, 5, dm, 4, generator=g, dtype=torch.float64)
    gamma = 1 + 0.1 * torch.randn(dm, generator=g, dtype=torch.float64)
    beta = 0.1 * torch.randn(dm, 4, generator=g, dtype=torch.float64)
    out = quaternion_layer_norm_fused(g32(q), g32(gamma), g32(beta), 1e-5)
    assert rel_l2(out, ref.layer_norm(q, gamma, beta, 1e-5)) < RTOL_F32
    outc = quaternion_layer_norm_fused(g32(q), g32(gamma), g32(beta), 1e-5, padded_compat=True)
    assert rel_l2(outc, ref.layer_norm_padded_compat(q, gamma, beta, 1e-5)) < RTOL_F32


def test_layernorm_bf16():
    g = gen(13)
    q = torch.randn(4, 64, 768, 4, generator=g, dtype=torch.float64)
    gamma = torch.ones(768, dtype=torch.float64)
    beta = torch.zeros(768, 4, dtype=torch.float64)
    out = quaternion_layer_norm_fused(q.to(DEV, torch.bfloat16), g32(gamma), g32(beta))
    assert out.dtype == torch.bfloat16
    assert rel_l2(out, ref.layer_norm(q, gamma, beta)) < RTOL_BF16


@pytest.mark.parametrize("dm", [5, 24, 768])
def test_layernorm_backward_matches_oracle(dm):
    g = gen(14)
    q = torch.randn(3, 7, dm, 4, generator=g, dtype=torch.float64)
    gamma = 1 + 0.1 * torch.randn(dm, generator=g, dtype=torch.float64)
    beta = 0.1 * torch.randn(dm, 4, generator=g, dtype=torch.float64)
    w = torch.randn(3, 7, dm, 4, generator=g, dtype=torch.float64)
    qr, gr, br = (t.clone().requires_grad_() for t in (q, gamma, beta))
    (ref.layer_norm(qr, gr, br) * w).sum().backward()
    ln = QuaternionLayerNorm(dm).to(DEV)
    with torch.no_grad():
        ln.gamma.copy_(gamma)
        ln.beta.copy_(beta)
    qg = g32(q).requires_grad_()
    (ln(qg) * g32(w)).sum().backward()
    assert rel_l2(qg.grad, qr.grad) < 1e-4
    assert rel_l2(ln.gamma.grad, gr.grad) < 1e-5
    assert rel_l2(ln.beta.grad, br.grad) < 1e-6


# ------------------------------------------- config 2 at the shapes the bench times

def _cpu64(t):
    return t.detach().double().cpu()


def test_config2_qmul_full_shape():
    """quaternion_multiply on p, q [2^26, 4] fp32 ~ N(0,1) (bench config 2a)."""
    g = torch.Generator(device=DEV).manual_seed(0)
    p = torch.randn(1 << 26, 4, generator=g, device=DEV)
    q = torch.randn(1 << 26, 4, generator=g, device=DEV)
    out = quaternion_multiply(p, q)
    torch.cuda.synchronize()
    assert rel_l2(out, ref.qmul(_cpu64(p), _cpu64(q))) < RTOL_F32


def test_config2_cayley_full_shape():
    """cayley_discretization_fused on z [2,16,768,64,4] with Re z <= 0 (config 2b)."""
    g = torch.Generator(device=DEV).manual_seed(1)
    z = torch.randn(2, 16, 768, 64, 4, generator=g, device=DEV)
    z[..., 0] = -z[..., 0].abs()
    q = cayley_discretization_fused(z)
    torch.cuda.synchronize()
    want = ref.cayley(_cpu64(z))
    assert rel_l2(q, want) < RTOL_F32
    assert bool((quaternion_norm(q) <= 1.0 + 1e-6).all())


def test_config2_prefix_product_full_shape_single_pass():
    """parallel_scan_quaternion on [2,256,768,64,4] with |q| in U(0.9, 0.999)
    (config 2c): 98304 lanes per batch row fill the GPU, so this runs the
    single-pass kernel the bench times. Whole-tensor rel-L2 and a per-step check
    on a few lanes, whose products decay over T."""
    g = torch.Generator(device=DEV).manual_seed(2)
    u = torch.randn(2, 256, 768, 64, 4, generator=g, device=DEV)
    r = torch.rand(2, 256, 768, 64, 1, generator=g, device=DEV) * 0.099 + 0.9
    qs = u / torch.linalg.vector_norm(u, dim=-1, keepdim=True) * r
    del u, r
    out = parallel_scan_quaternion(qs)
    torch.cuda.synchronize()
    want = ref.prefix_product(_cpu64(qs))
    assert rel_l2(out, want) < RTOL_F32
    lanes = [(0, 0), (767, 63), (300, 17)]
    for b in (0, 1):
        for d, n in lanes:
            got = _cpu64(out[b, :, d, n])
            exp = want[b, :, d, n]
            err = (got - exp).norm(dim=-1) / exp.norm(dim=-1)
            assert float(err.max()) < 1e-5


def test_config2_layernorm_full_shape():
    """QuaternionLayerNorm on [4,2048,768,4] fp32 (config 2d), gamma = 1, beta = 0
    as in the bench, and with random gamma/beta."""
    g = torch.Generator(device=DEV).manual_seed(3)
    x = torch.randn(4, 2048, 768, 4, generator=g, device=DEV)
    gamma = torch.ones(768, device=DEV)
    beta = torch.zeros(768, 4, device=DEV)
    out = quaternion_layer_norm_fused(x, gamma, beta)
    torch.cuda.synchronize()
    assert rel_l2(out, ref.layer_norm(_cpu64(x), _cpu64(gamma), _cpu64(beta))) < RTOL_F32
    gamma = 1.0 + 0.1 * torch.randn(768, generator=g, device=DEV)
    beta = 0.1 * torch.randn(768, 4, generator=g, device=DEV)
    out = quaternion_layer_norm_fused(x, gamma, beta)
    torch.cuda.synchronize()
    assert rel_l2(out, ref.layer_norm(_cpu64(x), _cpu64(gamma), _cpu64(beta))) < RTOL_F32
