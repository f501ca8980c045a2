"""Pin the CPU oracle to the reference: every golden fixture, CPU only.

The fixtures in tests/golden/reference_golden.pt were produced by running the
reference's own functions (tests/golden/make_golden.py). The oracle restates
them; here we check the restatement reproduces each fixture.
"""

import torch
import torch.nn.functional as F

from oracle import ref


def _close(a, b, rtol, atol):
    assert a.shape == b.shape, (a.shape, b.shape)
    torch.testing.assert_close(a, b, rtol=rtol, atol=atol)


def test_qmul_qconj_qinv_qnorm(golden):
    for tag, tol in (("f64", 1e-14), ("f32", 1e-6)):
        c = golden[f"qmul_{tag}"]
        _close(ref.qmul(c["p"], c["q"]), c["out"], tol, tol)
        c = golden[f"qconj_{tag}"]
        _close(ref.qconj(c["q"]), c["out"], 0, 0)
        c = golden[f"qinv_{tag}"]
        _close(ref.qinv(c["q"], 1e-6), c["out"], tol, tol)
        c = golden[f"qnorm_{tag}"]
        _close(ref.qnorm(c["q"]), c["out"], tol, tol)
    c = golden["qinv_eps_clamp"]
    _close(ref.qinv(c["q"], 1e-6), c["out"], 1e-14, 1e-14)


def test_noncommuting_pair(golden):
    c = golden["qmul_noncommuting_pair"]
    _close(ref.qmul(c["p"], c["q"]), c["pq"], 0, 0)
    _close(ref.qmul(c["q"], c["p"]), c["qp"], 0, 0)
    assert not torch.allclose(c["pq"], c["qp"])


def test_cayley(golden):
    for name, tol in (("cayley_f64", 1e-13), ("cayley_f32", 2e-6),
                      ("cayley_stable_f64", 1e-13), ("cayley_pole_f64", 1e-12)):
        c = golden[name]
        _close(ref.cayley(c["z"], c["eps"]), c["out"], tol, tol)


def test_prefix_product(golden):
    c = golden["prefix_f64"]
    _close(ref.prefix_product(c["q"]), c["out"], 1e-13, 1e-13)
    c = golden["prefix_f32"]
    _close(ref.prefix_product(c["q"]), c["out"], 1e-5, 1e-5)


def test_layer_norm(golden):
    for dm in (16, 24):
        c = golden[f"layernorm_d{dm}_f64"]
        _close(ref.layer_norm(c["q"], c["gamma"], c["beta"], c["eps"]), c["out"], 1e-12, 1e-12)


def test_layer_norm_triton_padded_lanes(golden):
    """The reference Triton LN kernel at d_model=24 follows the padded-lane form."""
    c = golden["layernorm_triton_interp_d24"]
    compat = ref.layer_norm_padded_compat(c["q"], c["gamma"], c["beta"], 1e-5)
    _close(compat, c["out"], 1e-5, 1e-5)
    exact = ref.layer_norm(c["q"], c["gamma"], c["beta"], 1e-5)
    assert (exact - c["out"]).abs().max() > 1e-2  # the kernel differs from the math


def test_ssm_step_and_forward(golden):
    c = golden["ssm_step_f64"]
    h_new, y = ref.ssm_step(c["q"], c["B"], c["S"], c["C"], c["D"], c["h_prev"])
    _close(h_new, c["h_new"], 1e-13, 1e-13)
    _close(y, c["y"], 1e-13, 1e-13)
    c = golden["ssm_forward_f64"]
    y, _ = ref.ssm_forward(c["q"], c["B"], c["S"], c["C"], c["D"])
    _close(y, c["y"], 1e-12, 1e-12)


def test_scan_cayley_shared(golden):
    c = golden["scan_cayley_shared_f64"]
    for slab in (64, 5):
        y, hT = ref.ssm_scan_cayley(c["delta"], c["Lambda"], c["B"], c["C"], c["x"], c["D"],
                                    t_slab=slab)
        _close(y, c["y"], 1e-12, 1e-12)
        _close(hT, c["h_T"], 1e-12, 1e-12)


def test_block_forward(golden):
    c = golden["block_f64"]
    cfg = c["config"]
    out = ref.block_forward(c["state_dict"], c["x"], d_state=cfg["d_state"], d_conv=cfg["d_conv"])
    _close(out, c["out"], 1e-12, 1e-12)


def test_block_lambda_override_matches_params(golden):
    c = golden["block_f64"]
    sd = c["state_dict"]
    lam = ref.lambda_from_params(sd["Lambda_alpha"], sd["Lambda_imag"])
    out = ref.block_forward(sd, c["x"], d_state=4, Lam=lam)
    _close(out, c["out"], 1e-12, 1e-12)
    assert torch.all(lam[..., 0] < 0)
    assert torch.allclose(lam[..., 0], -F.softplus(sd["Lambda_alpha"]))
