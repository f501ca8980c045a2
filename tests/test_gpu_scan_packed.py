"""The packed-FP32 scan kernel (the default for channel-shared B/C) against the
unpacked warp-specialised kernel (selected with MQC_SCAN_IMPL=scalar in a child
process): both compute every state with the same rounded operations in the same
order, so y, h_T and the checkpoints must agree bit for bit, for every lane
mapping (d_state 1 .. 256, padded and unpadded), both input dtypes and both
signal kinds."""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

from tests.gpu_util import make_scan_inputs, to_dev

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]

CASES = [
    # (batch, seq_len, d_inner, d_state, s_real, dtype)
    (2, 100, 70, 64, True, "float32"),
    (1, 67, 33, 1, True, "float32"),
    (2, 40, 9, 16, False, "float32"),
    (1, 50, 20, 38, True, "bfloat16"),
    (2, 33, 12, 200, False, "bfloat16"),
    (1, 65, 300, 256, True, "float32"),
]


def _run(case, out_path=None):
    """Runs one case through the default dispatch; returns (y, h_T)."""
    from mambaqc_b200.kernels import ssm_scan_cayley

    bsz, seqlen, dm, ds, s_real, dtype = case
    inp = to_dev(make_scan_inputs(bsz, seqlen, dm, ds, s_real=s_real, seed=ds + seqlen),
                 getattr(torch, dtype))
    h0 = torch.randn(bsz, dm, ds, 4, generator=torch.Generator().manual_seed(7)).cuda()
    y, hT = ssm_scan_cayley(inp["delta"], inp["Lambda"], inp["B"], inp["C"], inp["S"], inp["D"],
                            h0=h0, return_final_state=True, time_chunks=1)
    torch.cuda.synchronize()
    res = (y.cpu(), hT.cpu())
    if out_path is not None:
        torch.save(res, out_path)
    return res


def _run_scalar(case, tmp_path):
    out = tmp_path / "scalar.pt"
    code = (
        "import sys; sys.path.insert(0, %r); "
        "from tests.test_gpu_scan_packed import _run; _run(%r, %r)" % (str(ROOT), case, str(out))
    )
    env = dict(os.environ, MQC_SCAN_IMPL="scalar")
    subprocess.run([sys.executable, "-c", code], check=True, env=env, cwd=str(ROOT), timeout=600)
    return torch.load(out)


@pytest.mark.parametrize("case", CASES, ids=lambda c: "x".join(map(str, c)))
def test_packed_kernel_bitwise_equals_scalar_kernel(case, tmp_path):
    y, hT = _run(case)
    y_s, hT_s = _run_scalar(case, tmp_path)
    assert torch.equal(y, y_s), (y.double() - y_s.double()).abs().max().item()
    assert torch.equal(hT, hT_s), (hT - hT_s).abs().max().item()
