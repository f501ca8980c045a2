"""Time-chunked (time-parallel) scan forward vs the sequential GPU scan and the
fp64 oracle: pass 1 (chunk end state + operator product), the on-device carry
and pass 2 must reproduce the sequential recurrence."""

import pytest
import torch

from oracle import ref
from tests.gpu_util import DEV, RTOL_BF16, RTOL_F32, gen, make_scan_inputs, rel_l2, to_dev

pytestmark = pytest.mark.gpu

from mambaqc_b200.kernels import ssm_scan_cayley  # noqa: E402
from mambaqc_b200.kernels.ssm_fused import auto_time_chunks  # noqa: E402


def run(inp, dtype, nc, h0=None):
    d = to_dev(inp, dtype)
    with torch.no_grad():
        y, hT = ssm_scan_cayley(d["delta"], d["Lambda"], d["B"], d["C"], d["S"], d["D"],
                                h0=None if h0 is None else h0.to(DEV, torch.float32),
                                return_final_state=True, time_chunks=nc)
    torch.cuda.synchronize()
    return y, hT


@pytest.mark.parametrize("shared,s_real", [(True, True), (False, True), (True, False)])
def test_chunked_matches_oracle(shared, s_real):
    inp = make_scan_inputs(1, 1024, 4, 16, shared=shared, s_real=s_real, seed=3)
    h0 = torch.randn(1, 4, 16, 4, generator=gen(4), dtype=torch.float64)
    y_ref, h_ref = ref.ssm_scan_cayley(*(inp[k] for k in ("delta", "Lambda", "B", "C", "S", "D")),
                                       h0=h0)
    for nc in (2, 4, 8):
        y, hT = run(inp, torch.float32, nc, h0=h0)
        assert rel_l2(y, y_ref) < RTOL_F32, nc
        assert rel_l2(hT, h_ref) < RTOL_F32, nc


@pytest.mark.parametrize("shape", [(1, 4096, 12, 64), (2, 2048, 5, 16), (1, 1024, 3, 100)])
def test_chunked_matches_sequential_gpu_scan(shape):
    bsz, seqlen, dm, ds = shape
    inp = make_scan_inputs(bsz, seqlen, dm, ds, shared=True, s_real=True, seed=sum(shape))
    y1, h1 = run(inp, torch.float32, 1)
    for nc in (2, 16, 32):
        y, hT = run(inp, torch.float32, nc)
        # both are fp32 evaluations of the same recurrence in different orders
        assert rel_l2(y, y1) < RTOL_F32, nc
        assert rel_l2(hT, h1) < RTOL_F32, nc


def test_chunked_bf16_config5_like():
    """bf16 inputs, fp32 state, a narrow channel shard of a long sequence."""
    inp = make_scan_inputs(1, 8192, 8, 64, shared=True, s_real=True, seed=11)
    y1, _ = run(inp, torch.float32, 1)
    nc = auto_time_chunks(1, 8192, 8, 64)
    assert nc > 1
    yb, _ = run(inp, torch.bfloat16, "auto")
    assert yb.dtype == torch.bfloat16
    assert rel_l2(yb, y1) < RTOL_BF16


def test_auto_chunks_policy():
    assert auto_time_chunks(4, 2048, 1536, 64) == 1          # config 3 fills the GPU
    assert auto_time_chunks(1, 65536, 1536, 64) >= 2          # config 5 on one GPU
    assert auto_time_chunks(1, 65536, 192, 64) >= 16          # config 5 shard of 8 GPUs
    assert auto_time_chunks(1, 300, 4, 16) == 1               # too short to split


def test_config5_full_size_chunked_vs_sequential():
    """Config 5 at full size (B=1, T=65536, D=1536, N=64, bf16 inputs, fp32 state):
    the time-chunked scan must reproduce the sequential one, and both must match
    the fp64 oracle on a sample of channels over all 65536 steps."""
    bsz, seqlen, dm, ds = 1, 65536, 1536, 64
    g = gen(21)
    x = torch.randn(bsz, seqlen, dm, generator=g).bfloat16()
    delta = torch.nn.functional.softplus(torch.randn(bsz, seqlen, dm, generator=g) - 3.0).bfloat16()
    lam = torch.empty(dm, ds, 4)
    lam[..., 0] = -torch.exp(torch.empty(dm, ds).uniform_(-6.9078, -2.3026, generator=g))
    lam[..., 1:] = 0.5 * torch.randn(dm, ds, 3, generator=g)
    Bm = (torch.randn(bsz, seqlen, ds, 4, generator=g) / 8).bfloat16()
    Cm = (torch.randn(bsz, seqlen, ds, 4, generator=g) / 8).bfloat16()
    Dk = torch.ones(dm)
    dev = [t.to(DEV) for t in (delta, lam, Bm, Cm, x, Dk)]
    assert auto_time_chunks(bsz, seqlen, dm, ds) > 1
    with torch.no_grad():
        y_c, h_c = ssm_scan_cayley(*dev, return_final_state=True, time_chunks="auto")
        y_s, h_s = ssm_scan_cayley(*dev, return_final_state=True, time_chunks=1)
    torch.cuda.synchronize()
    assert rel_l2(h_c, h_s) < RTOL_F32
    assert rel_l2(y_c.float(), y_s.float()) < RTOL_BF16
    chans = torch.tensor([0, 777, 1535])
    y_ref, h_ref = ref.ssm_scan_cayley(
        delta[:, :, chans].double(), lam[chans].double(), Bm.double(), Cm.double(),
        x[:, :, chans].double(), Dk[chans].double(), t_slab=4096)
    ci = chans.to(DEV)
    for y, h in ((y_c, h_c), (y_s, h_s)):
        # bf16 inputs with an fp32 state: the contract bound is RTOL_BF16; the
        # inputs are exact in the oracle, so h_T is held to the fp32 rounding
        # accumulated over 65536 steps as well (about 1.2e-5 measured)
        assert rel_l2(h[:, ci], h_ref) < min(RTOL_BF16, 5e-5)
        assert rel_l2(y[:, :, ci], y_ref) < RTOL_BF16


# ------------------------------------------------------------ time-sharded scan

def test_scan_summary_matches_oracle():
    """(P, E) of a range: P the left-ordered product of the Cayley steps, E the
    final state from zero, with and without time chunks inside the range."""
    from mambaqc_b200.kernels import ssm_scan_summary
    inp = make_scan_inputs(2, 512, 5, 16, shared=True, s_real=True, seed=31)
    q = ref.cayley(inp["delta"][..., None, None] * inp["Lambda"][None, None])
    P_ref = torch.zeros(2, 5, 16, 4, dtype=torch.float64)
    P_ref[..., 0] = 1
    for t in range(512):
        P_ref = ref.qmul(q[:, t], P_ref)
    E_ref = ref.ssm_scan_cayley(*(inp[k] for k in ("delta", "Lambda", "B", "C", "S", "D")))[1]
    d = to_dev(inp, torch.float32)
    for nc in (1, 4, "auto"):
        P, E = ssm_scan_summary(d["delta"], d["Lambda"], d["B"], d["C"], d["S"], d["D"],
                                time_chunks=nc)
        assert rel_l2(P, P_ref) < RTOL_F32, nc
        assert rel_l2(E, E_ref) < RTOL_F32, nc


@pytest.mark.parametrize("shared,s_real,dtype", [(True, True, torch.float32),
                                                 (True, True, torch.bfloat16),
                                                 (False, True, torch.float32),
                                                 (True, False, torch.float32)])
def test_time_sharded_scan_emulated_on_one_gpu(shared, s_real, dtype):
    """The time-sharded decomposition with 4 ranks emulated in turn on one GPU:
    per-range summaries, the carry over ranks, and each range scanned from its
    start state reproduce the unsharded scan (y and the final state)."""
    from mambaqc_b200.kernels import ssm_scan_carry, ssm_scan_summary
    from mambaqc_b200.kernels.sharded import time_shard
    world = 4
    inp = make_scan_inputs(2, 2048, 24, 16, shared=shared, s_real=s_real, seed=41)
    d = to_dev(inp, dtype)
    h0 = torch.randn(2, 24, 16, 4, generator=gen(42)).to(DEV)
    keys = ("delta", "Lambda", "B", "C", "S", "D")
    with torch.no_grad():
        y_full, h_full = ssm_scan_cayley(*(d[k] for k in keys), h0=h0, return_final_state=True,
                                         time_chunks=1)
        parts = []
        for r in range(world):
            parts.append({k: (d[k] if k in ("Lambda", "D") else time_shard(d[k], r, world))
                          for k in keys})
        sums = [ssm_scan_summary(*(p[k] for k in keys)) for p in parts]
        hin, hT = ssm_scan_carry(torch.stack([s[0] for s in sums]),
                                 torch.stack([s[1] for s in sums]), h0)
        ys = [ssm_scan_cayley(*(p[k] for k in keys), h0=hin[r], time_chunks=1)
              for r, p in enumerate(parts)]
    torch.cuda.synchronize()
    y = torch.cat(ys, dim=1)
    assert rel_l2(hT, h_full) < RTOL_F32
    tol = RTOL_F32 if dtype == torch.float32 else RTOL_BF16
    assert rel_l2(y.float(), y_full.float()) < tol


@pytest.mark.parametrize("nc", [1, 4, 8])
def test_resume_from_summary_equals_chunked_scan(nc):
    """A range scanned by resuming from its summary's chunks (carry + full pass)
    gives the time-chunked scan's y bit for bit with the same chunks, and the
    emulated 4-rank time-sharded scan built on it matches the unsharded scan."""
    from mambaqc_b200.kernels import ssm_scan_carry, ssm_scan_cayley_resume, ssm_scan_summary
    from mambaqc_b200.kernels.sharded import time_shard
    keys = ("delta", "Lambda", "B", "C", "S", "D")
    inp = make_scan_inputs(1, 4096, 12, 64, shared=True, s_real=True, seed=51)
    d = to_dev(inp, torch.bfloat16)
    h0 = torch.randn(1, 12, 64, 4, generator=gen(52)).to(DEV)
    with torch.no_grad():
        y_c, h_c = ssm_scan_cayley(*(d[k] for k in keys), h0=h0, return_final_state=True,
                                   time_chunks=nc)
        summ = ssm_scan_summary(*(d[k] for k in keys), time_chunks=nc, keep_chunks=True)
        y_r, h_r = ssm_scan_cayley_resume(*(d[k] for k in keys), summary=summ, h0=h0,
                                          return_final_state=True)
        world = 4
        parts = [{k: (d[k] if k in ("Lambda", "D") else time_shard(d[k], r, world)) for k in keys}
                 for r in range(world)]
        summs = [ssm_scan_summary(*(p[k] for k in keys), time_chunks=nc, keep_chunks=True)
                 for p in parts]
        hin, hT = ssm_scan_carry(torch.stack([s.P for s in summs]),
                                 torch.stack([s.E for s in summs]), h0)
        ys = [ssm_scan_cayley_resume(*(p[k] for k in keys), summary=s, h0=hin[r])
              for r, (p, s) in enumerate(zip(parts, summs))]
    torch.cuda.synchronize()
    assert torch.equal(y_r, y_c)
    # with one batch row the chunked scan takes h_T from its full pass, the
    # resumed scan from the carry: the same state, rounded differently
    assert rel_l2(h_r, h_c) < RTOL_F32
    y_full, h_full = ssm_scan_cayley(*(d[k] for k in keys), h0=h0, return_final_state=True,
                                     time_chunks=1)
    assert rel_l2(hT, h_full) < RTOL_F32
    assert rel_l2(torch.cat(ys, dim=1).float(), y_full.float()) < RTOL_BF16
