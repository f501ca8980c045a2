"""GPU parity of the selective scan (fused Cayley + scan, explicit-q scan, single
step) against the fp64 CPU oracle and the golden fixtures from the reference.

Tolerances (relative L2 over the whole output): 1e-5 for fp32 inputs, 2e-2 for
bf16 inputs with the fp32 state."""

import math

import pytest
import torch

from oracle import ref
from tests.gpu_util import DEV, RTOL_BF16, RTOL_F32, gen, make_scan_inputs, rel_l2, to_dev

pytestmark = pytest.mark.gpu

from mambaqc_b200 import _lib  # noqa: E402
from mambaqc_b200.kernels import (  # noqa: E402
    cayley_discretization_fused,
    quaternion_norm,
    ssm_forward_fused,
    ssm_scan_cayley,
    ssm_step_fused,
)


def oracle_scan(inp, h0=None):
    return ref.ssm_scan_cayley(inp["delta"], inp["Lambda"], inp["B"], inp["C"], inp["S"],
                               inp["D"], h0=h0)


def run_scan(inp, dtype, h0=None):
    d = to_dev(inp, dtype)
    y, hT = ssm_scan_cayley(d["delta"], d["Lambda"], d["B"], d["C"], d["S"], d["D"],
                            h0=None if h0 is None else h0.to(DEV, torch.float32),
                            return_final_state=True)
    torch.cuda.synchronize()
    _lib.check_device_status(torch.device(DEV))
    return y, hT


# ----------------------------------------------------------------- golden

def test_golden_fused_scan(golden):
    c = golden["scan_cayley_shared_f64"]
    inp = dict(delta=c["delta"], Lambda=c["Lambda"], B=c["B"], C=c["C"], S=c["x"], D=c["D"])
    y, hT = run_scan(inp, torch.float32)
    assert rel_l2(y, c["y"]) < RTOL_F32
    assert rel_l2(hT, c["h_T"]) < RTOL_F32


def test_golden_explicit_q_forward_and_step(golden):
    c = golden["ssm_forward_f64"]
    y = ssm_forward_fused(*(c[k].to(DEV, torch.float32) for k in ("q", "B", "S", "C")),
                          c["D"].to(DEV, torch.float32))
    assert rel_l2(y, c["y"]) < RTOL_F32
    c = golden["ssm_step_f64"]
    h_new, y = ssm_step_fused(*(c[k].to(DEV, torch.float32) for k in ("q", "B", "S", "C", "D",
                                                                      "h_prev")))
    assert rel_l2(h_new, c["h_new"]) < RTOL_F32
    assert rel_l2(y, c["y"]) < RTOL_F32


# ------------------------------------------------------------ fused scan grid

CASES = [
    # (B, T, D, N, shared, s_real)
    (2, 37, 8, 16, True, True),
    (2, 37, 8, 16, False, True),
    (2, 37, 8, 16, True, False),
    (2, 37, 8, 16, False, False),
    (1, 100, 13, 64, True, True),     # D not a multiple of anything, T % chunk != 0
    (3, 65, 5, 3, True, True),        # N < lanes: masked state lanes
    (1, 33, 7, 100, True, True),      # N not a power of two (NG=32, G=4)
    (1, 20, 3, 200, False, True),     # N > 128 (G=8)
    (1, 16, 300, 8, True, False),     # many channels, small N
    (1, 1, 4, 16, True, True),        # T = 1
    (4, 64, 1, 64, True, True),       # one channel
    (2, 70, 10, 64, False, True),     # per-channel B/C at d_state 64 (the block's layout)
    (2, 70, 10, 64, False, False),
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: "B{}T{}D{}N{}{}{}".format(
    c[0], c[1], c[2], c[3], "sh" if c[4] else "pc", "x" if c[5] else "S"))
def test_fused_scan_fp32(case):
    bsz, seqlen, dm, ds, shared, s_real = case
    inp = make_scan_inputs(bsz, seqlen, dm, ds, shared=shared, s_real=s_real, seed=sum(case[:4]))
    y, hT = run_scan(inp, torch.float32)
    y_ref, h_ref = oracle_scan(inp)
    assert rel_l2(y, y_ref) < RTOL_F32
    assert rel_l2(hT, h_ref) < RTOL_F32


@pytest.mark.parametrize("shared", [True, False])
def test_fused_scan_bf16(shared):
    inp = make_scan_inputs(2, 96, 24, 64, shared=shared, s_real=True, seed=21)
    y, hT = run_scan(inp, torch.bfloat16)
    assert y.dtype == torch.bfloat16
    y_ref, h_ref = oracle_scan(inp)
    assert rel_l2(y, y_ref) < RTOL_BF16
    assert rel_l2(hT, h_ref) < RTOL_BF16
    # against the oracle on the bf16-rounded inputs the error is output rounding only
    rounded = {k: (v if k in ("Lambda", "D") else v.to(torch.bfloat16).double())
               for k, v in inp.items()}
    y_rr, _ = oracle_scan(rounded)
    assert rel_l2(y, y_rr) < 5e-3


def test_fused_scan_initial_state_and_chaining():
    """Scanning [0, T) equals scanning [0, T/2) then [T/2, T) from its final state."""
    inp = make_scan_inputs(2, 80, 9, 16, shared=True, s_real=False, seed=31)
    g = gen(32)
    h0 = torch.randn(2, 9, 16, 4, generator=g, dtype=torch.float64)
    y, hT = run_scan(inp, torch.float32, h0=h0)
    y_ref, h_ref = oracle_scan(inp, h0=h0)
    assert rel_l2(y, y_ref) < RTOL_F32 and rel_l2(hT, h_ref) < RTOL_F32
    half = {k: (v[:, :40] if k not in ("Lambda", "D") else v) for k, v in inp.items()}
    rest = {k: (v[:, 40:] if k not in ("Lambda", "D") else v) for k, v in inp.items()}
    y1, h1 = run_scan(half, torch.float32, h0=h0)
    y2, h2 = run_scan(rest, torch.float32, h0=h1.double().cpu())
    assert rel_l2(torch.cat([y1, y2], 1), y_ref) < RTOL_F32
    assert rel_l2(h2, h_ref) < RTOL_F32


def test_fused_scan_order_matters():
    """A scan with the Hamilton products reversed must fail parity."""
    inp = make_scan_inputs(1, 40, 6, 16, shared=True, s_real=False, seed=41)
    y, _ = run_scan(inp, torch.float32)

    def _rev(p, q):
        a0, a1, a2, a3 = q.unbind(-1)
        b0, b1, b2, b3 = p.unbind(-1)
        return torch.stack((a0 * b0 - a1 * b1 - a2 * b2 - a3 * b3,
                            a0 * b1 + a1 * b0 + a2 * b3 - a3 * b2,
                            a0 * b2 - a1 * b3 + a2 * b0 + a3 * b1,
                            a0 * b3 + a1 * b2 - a2 * b1 + a3 * b0), dim=-1)

    saved = ref.qmul
    try:
        ref.qmul = _rev  # plant the mistake in the oracle, on the CPU
        y_rev, _ = oracle_scan(inp)
    finally:
        ref.qmul = saved
    y_ref, _ = oracle_scan(inp)
    assert rel_l2(y, y_ref) < RTOL_F32
    assert rel_l2(y, y_rev) > 1e-2


def test_stability_invariant_from_delta_lambda():
    """|q| < 1 whenever Re(delta * Lambda) < 0, for the operators the scan forms."""
    inp = make_scan_inputs(2, 16, 32, 64, seed=51)
    z = inp["delta"][..., None, None] * inp["Lambda"][None, None]
    assert (z[..., 0] < 0).all()
    q = cayley_discretization_fused(z.to(DEV, torch.float32))
    assert (quaternion_norm(q) < 1.0).all()
    # closed form: |q|^2 = ((1+a)^2 + |v|^2) / ((1-a)^2 + |v|^2), a = Re z / 2
    a = z[..., 0] / 2
    vv = (z[..., 1:] / 2).pow(2).sum(-1)
    n2 = ((1 + a) ** 2 + vv) / ((1 - a) ** 2 + vv)
    assert rel_l2(quaternion_norm(q) ** 2, n2) < RTOL_F32


def test_explicit_q_scan_matches_fused():
    """ssm_forward_fused on materialised q = Cayley(delta Lambda) equals the fused op."""
    inp = make_scan_inputs(2, 50, 6, 16, shared=False, s_real=False, seed=61)
    d = to_dev(inp, torch.float32)
    z = d["delta"][..., None, None] * d["Lambda"][None, None]
    q = cayley_discretization_fused(z)
    y_q = ssm_forward_fused(q, d["B"], d["S"], d["C"], d["D"])
    y_f = ssm_scan_cayley(d["delta"], d["Lambda"], d["B"], d["C"], d["S"], d["D"])
    y_ref, _ = oracle_scan(inp)
    assert rel_l2(y_q, y_ref) < RTOL_F32
    assert rel_l2(y_f, y_ref) < RTOL_F32


def test_skip_weight_layouts():
    """D as [D], [B,D] and a stride-0 [B,T,D] expand (the reference passes the latter)."""
    inp = make_scan_inputs(2, 24, 7, 8, seed=71)
    d = to_dev(inp, torch.float32)
    y1 = ssm_scan_cayley(d["delta"], d["Lambda"], d["B"], d["C"], d["S"], d["D"])
    y2 = ssm_scan_cayley(d["delta"], d["Lambda"], d["B"], d["C"], d["S"],
                         d["D"].view(1, 1, 7).expand(2, 24, 7))
    y3 = ssm_scan_cayley(d["delta"], d["Lambda"], d["B"], d["C"], d["S"],
                         d["D"].view(1, 7).expand(2, 7).contiguous())
    assert torch.equal(y1, y2) and torch.equal(y1, y3)


def test_device_timeout_is_reported_and_context_survives():
    """A bounded wait forced to give up (poll limit 0) reports a status the host
    turns into an exception; the kernel drains its copies and the context stays usable."""
    inp = make_scan_inputs(1, 64, 8, 16, shared=True, seed=81)
    d = to_dev(inp, torch.float32)
    ssm_scan_cayley(d["delta"], d["Lambda"], d["B"], d["C"], d["S"], d["D"], wait_poll_limit=0)
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="timed out"):
        _lib.check_device_status(torch.device(DEV))
    y, _ = run_scan(inp, torch.float32)  # a normal call afterwards works
    y_ref, _ = oracle_scan(inp)
    assert rel_l2(y, y_ref) < RTOL_F32


def test_deterministic_bitwise():
    inp = make_scan_inputs(2, 128, 40, 64, seed=91)
    y1, h1 = run_scan(inp, torch.float32)
    y2, h2 = run_scan(inp, torch.float32)
    assert torch.equal(y1, y2) and torch.equal(h1, h2)


def test_config3_full_size_channel_sample():
    """Config 3 at full size (B=4, T=2048, D=1536, N=64, shared B/C, fp32):
    every (b, d) recurrence is independent, so a sample of channels is checked
    against the oracle run on just those channels for all 2048 steps."""
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
    y, hT = ssm_scan_cayley(delta.to(DEV), lam.to(DEV), Bm.to(DEV), Cm.to(DEV), x.to(DEV),
                            Dk.to(DEV), return_final_state=True)
    torch.cuda.synchronize()
    _lib.check_device_status(torch.device(DEV))
    chans = torch.tensor([0, 1, 41, 42, 777, 1535])
    for b in (0, 3):
        y_ref, h_ref = ref.ssm_scan_cayley(
            delta[b:b + 1, :, chans].double(), lam[chans].double(), Bm[b:b + 1].double(),
            Cm[b:b + 1].double(), x[b:b + 1, :, chans].double(), Dk[chans].double())
        assert rel_l2(y[b:b + 1, :, chans.to(DEV)], y_ref) < RTOL_F32
        assert rel_l2(hT[b:b + 1, chans.to(DEV)], h_ref) < RTOL_F32
    assert torch.isfinite(y).all()


def test_host_buffer_entry_point_matches_device_entry_point():
    """ssm_scan_cayley_from_host (pipelined host->device->host) equals the device call."""
    from mambaqc_b200.kernels import ssm_scan_cayley_from_host
    inp = make_scan_inputs(3, 40, 10, 16, shared=True, s_real=True, seed=101)
    d = to_dev(inp, torch.float32)
    y_dev = ssm_scan_cayley(d["delta"], d["Lambda"], d["B"], d["C"], d["S"], d["D"])
    host = {k: v.float().pin_memory() for k, v in inp.items()}
    bufs = {}
    # one segment (same kernel as the device call: bit for bit), then four
    # segments chained through the final state (pieces of 5 and 10 steps; the
    # 5-step ones take the short-sequence kernel, whose sum over n runs in another
    # lane order, so equal up to rounding)
    for segments in (1, 1, 4, 4):
        y_host = ssm_scan_cayley_from_host(host["delta"], host["Lambda"], host["B"], host["C"],
                                           host["S"], host["D"], device=DEV, _bufs=bufs,
                                           segments=segments)
        torch.cuda.synchronize()
        assert y_host.device.type == "cpu"
        if segments == 1:
            assert torch.equal(y_host, y_dev.cpu())
        else:
            assert rel_l2(y_host, y_dev) < 1e-6


@pytest.mark.parametrize("shared,dtype", [(False, torch.float32), (True, torch.bfloat16)])
def test_host_buffer_entry_point_layouts(shared, dtype):
    """Per-channel B/C and bf16 through the host-buffer entry point, in segments."""
    from mambaqc_b200.kernels import ssm_scan_cayley_from_host
    inp = make_scan_inputs(2, 48, 7, 12, shared=shared, s_real=True, seed=202)
    d = to_dev(inp, dtype)
    y_dev = ssm_scan_cayley(d["delta"], d["Lambda"], d["B"], d["C"], d["S"], d["D"])
    host = {k: v.cpu().pin_memory() for k, v in d.items()}
    y_host = ssm_scan_cayley_from_host(host["delta"], host["Lambda"], host["B"], host["C"],
                                       host["S"], host["D"], device=DEV, segments=3)
    torch.cuda.synchronize()
    # pieces of 8, 16, 16, 8 steps (the short ones on the short-sequence kernel)
    assert rel_l2(y_host, y_dev) < (1e-6 if dtype == torch.float32 else 5e-3)


@pytest.mark.parametrize("shared,dtype", [(True, torch.float32), (False, torch.float32),
                                          (True, torch.bfloat16)])
def test_decode_step_with_state_cache(shared, dtype):
    """ssm_step_cayley updates the state cache in place; six steps equal the
    six-step scan bit for bit, and the first step matches the oracle."""
    from mambaqc_b200.kernels import ssm_step_cayley
    inp = make_scan_inputs(3, 6, 20, 16, shared=shared, s_real=True, seed=303)
    d = to_dev(inp, dtype)
    h0 = torch.randn(3, 20, 16, 4, generator=gen(9)).to(DEV)
    y_scan, h_scan = ssm_scan_cayley(d["delta"], d["Lambda"], d["B"], d["C"], d["S"], d["D"],
                                     h0=h0, return_final_state=True)
    h = h0.clone()
    ys = [ssm_step_cayley(d["delta"][:, t], d["Lambda"], d["B"][:, t], d["C"][:, t],
                          d["S"][:, t], d["D"], h) for t in range(6)]
    torch.cuda.synchronize()
    assert torch.equal(torch.stack(ys, 1), y_scan)
    assert torch.equal(h, h_scan)
    # first step against the fp64 oracle
    y_ref, h_ref = ref.ssm_scan_cayley(inp["delta"][:, :1], inp["Lambda"], inp["B"][:, :1],
                                       inp["C"][:, :1], inp["S"][:, :1], inp["D"],
                                       h0=h0.double().cpu())
    tol = RTOL_F32 if dtype == torch.float32 else RTOL_BF16
    assert rel_l2(ys[0], y_ref[:, 0]) < tol


@pytest.mark.parametrize("case", [
    # (B, D, N, s_real, dtype): batch rows not a multiple of the kernel's row
    # block, channel counts not a multiple of a CTA's channels, N from 1 to 64
    (1, 1, 1, True, torch.float32),
    (5, 37, 3, True, torch.float32),
    (7, 13, 16, False, torch.float32),
    (4, 96, 33, True, torch.float32),
    (6, 50, 64, False, torch.float32),
    (9, 40, 64, True, torch.bfloat16),
    (3, 21, 18, False, torch.bfloat16),  # bf16 channel-shared B/C needs an even N
    # more than 32 rows: the state-streaming kernel (ragged row ranges and
    # channel blocks)
    (40, 37, 64, True, torch.float32),
    (33, 13, 3, False, torch.float32),
    (70, 50, 64, True, torch.bfloat16),
    (48, 100, 16, False, torch.float32),
], ids=lambda c: "B{}D{}N{}{}{}".format(c[0], c[1], c[2], "x" if c[3] else "S",
                                      "f32" if c[4] == torch.float32 else "bf16"))
def test_decode_kernel_odd_shapes(case):
    """One decode step (T = 1, channel-shared B/C, state cache in place) against
    the fp64 oracle, with and without an initial state."""
    from mambaqc_b200.kernels import ssm_step_cayley
    bsz, dm, ds, s_real, dtype = case
    inp = make_scan_inputs(bsz, 1, dm, ds, shared=True, s_real=s_real, seed=bsz * 100 + dm + ds)
    d = to_dev(inp, dtype)
    tol = RTOL_F32 if dtype == torch.float32 else RTOL_BF16
    for with_h0 in (False, True):
        h0 = (torch.randn(bsz, dm, ds, 4, generator=gen(ds), dtype=torch.float64) if with_h0
              else torch.zeros(bsz, dm, ds, 4, dtype=torch.float64))
        h = h0.to(DEV, torch.float32)
        y = ssm_step_cayley(d["delta"][:, 0], d["Lambda"], d["B"][:, 0], d["C"][:, 0],
                            d["S"][:, 0], d["D"], h)
        torch.cuda.synchronize()
        y_ref, h_ref = ref.ssm_scan_cayley(inp["delta"], inp["Lambda"], inp["B"], inp["C"],
                                           inp["S"], inp["D"], h0=h0)
        assert rel_l2(y, y_ref[:, 0]) < tol
        assert rel_l2(h, h_ref) < tol


def test_config3_full_size_bf16_channel_sample():
    """Config 3 at full size with bf16 inputs (fp32 state): the oracle runs in fp64
    on the bf16-rounded inputs of a channel sample, so h_T differs only by the
    kernel's fp32 rounding and y by its final bf16 rounding."""
    bsz, seqlen, dm, ds = 4, 2048, 1536, 64
    g = gen(5)
    x = torch.randn(bsz, seqlen, dm, generator=g).bfloat16()
    delta = torch.nn.functional.softplus(torch.randn(bsz, seqlen, dm, generator=g) - 3.0).bfloat16()
    lam = torch.empty(dm, ds, 4)
    lam[..., 0] = -torch.exp(torch.empty(dm, ds).uniform_(math.log(1e-3), math.log(1e-1),
                                                          generator=g))
    lam[..., 1:] = 0.5 * torch.randn(dm, ds, 3, generator=g)
    Bm = (torch.randn(bsz, seqlen, ds, 4, generator=g) / 8).bfloat16()
    Cm = (torch.randn(bsz, seqlen, ds, 4, generator=g) / 8).bfloat16()
    Dk = 1.0 + 0.1 * torch.randn(dm, generator=g)
    y, hT = ssm_scan_cayley(delta.to(DEV), lam.to(DEV), Bm.to(DEV), Cm.to(DEV), x.to(DEV),
                            Dk.to(DEV), return_final_state=True)
    torch.cuda.synchronize()
    _lib.check_device_status(torch.device(DEV))
    assert y.dtype == torch.bfloat16 and hT.dtype == torch.float32
    chans = torch.tensor([0, 3, 64, 1000, 1535])
    for b in (1, 2):
        y_ref, h_ref = ref.ssm_scan_cayley(
            delta[b:b + 1, :, chans].double(), lam[chans].double(), Bm[b:b + 1].double(),
            Cm[b:b + 1].double(), x[b:b + 1, :, chans].double(), Dk[chans].double())
        assert rel_l2(hT[b:b + 1, chans.to(DEV)], h_ref) < RTOL_F32
        assert rel_l2(y[b:b + 1, :, chans.to(DEV)], y_ref) < RTOL_BF16
    assert torch.isfinite(y.float()).all()
