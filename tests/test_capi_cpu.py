"""C-ABI checks that need no GPU: the library loads, exports every symbol that
include/mambaqc_b200.h declares, and rejects bad arguments before touching the
device (validation happens on the host, so these calls never launch)."""

import ctypes
import re
import shutil
import subprocess
from pathlib import Path

import pytest
import torch

from mambaqc_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "mambaqc_b200.h"

INVALID, MISALIGNED, UNSUPPORTED = 1, 2, 3

# The validation tests pass fake device pointers that must be rejected on the
# host. They are kept off machines with a GPU, so that a future bug in the
# validation can never turn one of them into a launch on a bogus address.
no_gpu = pytest.mark.skipif(torch.cuda.is_available(),
                            reason="fake-pointer validation tests run only on GPU-less hosts")


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^MQC_API\s+[\w\s\*]+?\b(mqc_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_entry_points():
    names = declared_symbols()
    for expected in ("mqc_qmul", "mqc_cayley", "mqc_prefix_prod", "mqc_ssm_scan_fwd",
                     "mqc_ssm_step", "mqc_qln_fwd", "mqc_qln_bwd"):
        assert expected in names


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in declared_symbols():
        assert hasattr(lib, name), f"{name} declared in the header but not exported"
    # and the Python binding knows every declared entry point
    assert set(declared_symbols()) <= set(_lib.exported_symbols())


def test_version_and_status_strings():
    lib = _lib.load()
    assert lib.mqc_version().decode().count(".") == 2
    assert lib.mqc_status_string(0) == b"success"
    assert b"timed out" in lib.mqc_status_string(5)
    assert lib.mqc_status_string(999) == b"unknown status"


def _c_offsets(struct, fields, tmp_path):
    """sizeof and offsetof of a header struct, from a tiny C program built with gcc."""
    src = tmp_path / "layout.c"
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "mambaqc_b200.h"',
             "int main(void) {", f'  printf("%zu\\n", sizeof({struct}));']
    lines += [f'  printf("%zu\\n", offsetof({struct}, {f}));' for f in fields]
    lines += ["  return 0;", "}"]
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", f"-I{HEADER.parent}", str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split()
    return [int(v) for v in out]


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
@pytest.mark.parametrize("cstruct,pystruct", [("mqc_ssm_scan_args", "SsmScanArgs"),
                                              ("mqc_ssm_scan_bwd_args", "SsmScanBwdArgs"),
                                              ("mqc_bc_proj_scan_args", "BcProjScanArgs")])
def test_struct_layout_matches_header(cstruct, pystruct, tmp_path):
    py = getattr(_lib, pystruct)
    fields = [f for f, _ in py._fields_]
    got = _c_offsets(cstruct, fields, tmp_path)
    assert got[0] == ctypes.sizeof(py)
    assert got[1:] == [getattr(py, f).offset for f in fields]


@no_gpu
def test_elementwise_argument_validation_without_gpu():
    lib = _lib.load()
    fake = 0x10000  # never dereferenced: validation fails before any launch
    assert lib.mqc_qmul(fake, fake, fake, 4, 7, None) == INVALID
    assert b"dtype" in lib.mqc_last_error()
    assert lib.mqc_qmul(fake, fake, fake, -1, 0, None) == INVALID
    assert lib.mqc_qmul(None, fake, fake, 4, 0, None) == INVALID
    assert lib.mqc_qmul(fake + 4, fake, fake, 4, 0, None) == MISALIGNED
    assert lib.mqc_qinv(fake, fake + 2, 4, 1e-6, 1, None) == MISALIGNED
    i64x4 = ctypes.c_int64 * 4
    shape, st = i64x4(2, 3, 4, 5), i64x4(240, 80, 20, 4)
    assert lib.mqc_qmul_strided(fake, fake, fake, shape, st, i64x4(240, 80, 20, 2), 0,
                                None) == INVALID  # stride not a whole quaternion
    assert lib.mqc_qmul_strided(fake, fake, fake, shape, st, i64x4(240, 80, -20, 4), 0,
                                None) == INVALID  # negative stride
    assert lib.mqc_qmul_strided(fake, fake, fake, shape, st, st, 5, None) == INVALID
    assert lib.mqc_qmul_strided(fake, None, fake, shape, st, st, 0, None) == INVALID
    assert lib.mqc_qmul_strided(fake, fake, fake + 8, shape, st, st, 0, None) == MISALIGNED
    assert lib.mqc_qmul_strided(None, None, None, i64x4(2, 0, 4, 5), st, st, 0, None) == 0
    assert lib.mqc_cayley(fake, fake, 0, 1e-6, 0, None) == 0  # empty input is a no-op
    assert lib.mqc_prefix_prod(fake, fake, 1, 4, -3, 0, None) == INVALID
    assert lib.mqc_prefix_prod(fake + 4, fake, 1, 4, 3, 0, None) == MISALIGNED


@no_gpu
def test_scan_argument_validation_without_gpu():
    lib = _lib.load()
    fake = 0x10000
    base = dict(batch=2, seq_len=8, channels=4, d_state=16, dtype=0, flags=0, eps=1e-6,
                reserved0=0, delta=fake, lambda_=fake, q=None, Bm=fake, Cm=fake, s=fake,
                dskip=fake, dskip_sb=0, dskip_st=0, dskip_sd=1, h0=None, y=fake, hT=None,
                status=None, wait_poll_limit=-1)

    def call(**kw):
        a = _lib.SsmScanArgs(**{**base, **kw})
        return lib.mqc_ssm_scan_fwd(ctypes.byref(a), None)

    assert call(dtype=3) == INVALID
    assert call(flags=0x80) == INVALID
    assert call(d_state=300) == UNSUPPORTED
    assert b"d_state" in lib.mqc_last_error()
    assert call(delta=None) == INVALID
    assert call(flags=_lib.MQC_SSM_Q_GIVEN, q=None) == INVALID
    assert call(y=fake + 4) == MISALIGNED
    assert call(flags=_lib.MQC_SSM_BC_SHARED, Bm=fake + 8, dtype=1) == MISALIGNED
    assert call(flags=_lib.MQC_SSM_BC_SHARED, dtype=1, d_state=15) == UNSUPPORTED
    assert call(dskip=None) == INVALID
    assert call(batch=70000) == UNSUPPORTED
    assert call(seq_len=0) == 0  # nothing to do


@no_gpu
def test_bc_proj_scan_argument_validation_without_gpu():
    """mqc_bc_proj_scan_fwd rejects bad arguments on the host, before any launch."""
    lib = _lib.load()
    fake = 0x10000
    base = dict(batch=2, seq_len=8, channels=4, d_state=64, in_features=128, dtype=1, eps=1e-6,
                x=fake, w_b=fake, w_c=fake, delta=fake, s=fake, lambda_=fake, dskip=fake,
                dskip_sd=1, h0=None, hT=None, y=fake, status=None, wait_poll_limit=-1)

    def call(**kw):
        a = _lib.BcProjScanArgs(**{**base, **kw})
        return lib.mqc_bc_proj_scan_fwd(ctypes.byref(a), None)

    assert call(dtype=3) == INVALID
    assert call(d_state=48) == UNSUPPORTED
    assert b"d_state" in lib.mqc_last_error()
    assert call(in_features=100) == UNSUPPORTED
    assert b"in_features" in lib.mqc_last_error()
    assert call(w_c=None) == INVALID
    assert call(x=fake + 8) == MISALIGNED
    assert call(y=fake + 4) == MISALIGNED
    assert call(channels=70000) == UNSUPPORTED
    assert call(batch=-1) == INVALID
    assert call(seq_len=0) == 0  # nothing to do


@no_gpu
def test_multicast_scan_argument_validation_without_gpu():
    """mqc_ssm_scan_fwd_chunked_multicast rejects bad arguments on the host."""
    lib = _lib.load()
    fake = 0x10000
    base = dict(batch=1, seq_len=64, channels=4, d_state=32, dtype=0,
                flags=_lib.MQC_SSM_BC_SHARED | _lib.MQC_SSM_S_REAL, eps=1e-6, reserved0=0,
                delta=fake, lambda_=fake, q=None, Bm=fake, Cm=fake, s=fake, dskip=fake,
                dskip_sb=0, dskip_st=0, dskip_sd=1, h0=None, y=None, hT=None, status=None,
                wait_poll_limit=-1, ckpt=None, ckpt_every=0)

    def call(ymc=fake, ch_total=8, ch_off=0, nchunks=2, **kw):
        a = _lib.SsmScanArgs(**{**base, **kw})
        return lib.mqc_ssm_scan_fwd_chunked_multicast(ctypes.byref(a), nchunks, None, 0, ymc,
                                                      ch_total, ch_off, None)

    assert call(d_state=16) == UNSUPPORTED  # four lanes per channel are needed
    assert b"d_state" in lib.mqc_last_error()
    assert call(flags=_lib.MQC_SSM_S_REAL) == UNSUPPORTED  # per-channel B/C
    assert call(ymc=None) == INVALID
    assert call(ymc=fake + 8) == MISALIGNED
    assert call(ch_off=6) == INVALID  # channels [6, 10) outside 8
    assert call(nchunks=64) == UNSUPPORTED  # chunks of one step


@no_gpu
def test_host_scan_argument_validation_without_gpu():
    """mqc_ssm_scan_fwd_host rejects bad arguments before any CUDA call."""
    lib = _lib.load()
    fake = 0x10000
    base = dict(batch=2, seq_len=8, channels=4, d_state=16, dtype=0,
                flags=_lib.MQC_SSM_BC_SHARED | _lib.MQC_SSM_S_REAL, eps=1e-6, reserved0=0,
                delta=fake, lambda_=fake, q=None, Bm=fake, Cm=fake, s=fake, dskip=fake,
                dskip_sb=0, dskip_st=0, dskip_sd=1, h0=None, y=fake, hT=None, status=None,
                wait_poll_limit=-1)

    def call(segments=2, **kw):
        a = _lib.SsmScanArgs(**{**base, **kw})
        return lib.mqc_ssm_scan_fwd_host(ctypes.byref(a), segments, None)

    assert call(segments=3) == INVALID  # 8 steps do not split into 3
    assert b"segments" in lib.mqc_last_error()
    assert call(segments=0) == INVALID
    assert call(dskip_st=1) == UNSUPPORTED  # the skip weight must be per channel
    assert call(flags=_lib.MQC_SSM_Q_GIVEN) == UNSUPPORTED
    assert call(y=None) == INVALID
    assert call(dtype=7) == INVALID
    assert call(batch=0) == 0  # nothing to do


@no_gpu
def test_layernorm_argument_validation_without_gpu():
    lib = _lib.load()
    fake = 0x10000
    assert lib.mqc_qln_fwd(fake, fake, fake, fake, None, None, 4, 8, 1e-5, 0x10, 0, None) == INVALID
    assert lib.mqc_qln_fwd(fake, fake, fake, fake, None, None, 4, 100000, 1e-5, 0, 0, None) == UNSUPPORTED
    assert lib.mqc_qln_fwd(fake + 4, fake, fake, fake, None, None, 4, 8, 1e-5, 0, 0, None) == MISALIGNED
    need = lib.mqc_qln_bwd_workspace_size(64, 8)
    assert need > 0 and lib.mqc_qln_bwd_workspace_size(0, 8) == 0
    assert lib.mqc_qln_bwd(fake, fake, fake, fake, fake, fake, fake, fake, fake, need - 1, 64, 8,
                           1e-5, 0, None) == INVALID
    assert b"workspace" in lib.mqc_last_error()


def test_python_api_has_no_cpu_path():
    from mambaqc_b200.kernels import (cayley_discretization_fused, parallel_scan_quaternion,
                                      quaternion_multiply, ssm_scan_cayley)
    from mambaqc_b200.layers import QuaternionLayerNorm
    p = torch.randn(3, 4)
    with pytest.raises(RuntimeError, match="CUDA"):
        quaternion_multiply(p, p)
    with pytest.raises(RuntimeError, match="CUDA"):
        cayley_discretization_fused(torch.zeros(1, 1, 1, 1, 4))
    with pytest.raises(RuntimeError, match="CUDA"):
        parallel_scan_quaternion(torch.zeros(1, 2, 1, 1, 4))
    with pytest.raises(RuntimeError, match="CUDA"):
        QuaternionLayerNorm(4)(torch.zeros(1, 1, 4, 4))
    with pytest.raises(RuntimeError, match="CUDA"):
        ssm_scan_cayley(torch.ones(1, 2, 3), torch.zeros(3, 4, 4), torch.zeros(1, 2, 4, 4),
                        torch.zeros(1, 2, 4, 4), torch.zeros(1, 2, 3), torch.ones(3))


def test_reference_preconditions_raise_assertion():
    from mambaqc_b200.kernels import (cayley_discretization_fused, quaternion_layer_norm_fused,
                                      quaternion_multiply, ssm_step_fused)
    with pytest.raises(AssertionError):
        quaternion_multiply(torch.zeros(3, 4), torch.zeros(2, 4))
    with pytest.raises(AssertionError):
        quaternion_multiply(torch.zeros(3, 3), torch.zeros(3, 3))
    with pytest.raises(AssertionError):
        cayley_discretization_fused(torch.zeros(2, 3, 4))
    with pytest.raises(AssertionError):
        quaternion_layer_norm_fused(torch.zeros(1, 2, 3, 4), torch.ones(4), torch.zeros(3, 4))
    with pytest.raises(AssertionError):
        ssm_step_fused(torch.zeros(1, 2, 3, 4), torch.zeros(1, 2, 3, 4), torch.zeros(1, 2, 3),
                       torch.zeros(1, 2, 3, 4), torch.zeros(1, 2), torch.zeros(1, 2, 3, 4))


@no_gpu
def test_block_glue_argument_validation_without_gpu():
    """The block glue entry points reject bad arguments before any CUDA call."""
    lib = _lib.load()
    fake = 0x10000
    # conv: kernel size outside 1..8, row stride below the channel count, bad dtype
    assert lib.mqc_conv_silu_fwd(fake, 16, fake, None, fake, 2, 8, 16, 9, 0, None) == UNSUPPORTED
    assert lib.mqc_conv_silu_fwd(fake, 8, fake, None, fake, 2, 8, 16, 4, 0, None) == INVALID
    assert b"row stride" in lib.mqc_last_error()
    assert lib.mqc_conv_silu_fwd(fake, 16, fake, None, fake, 2, 8, 16, 4, 5, None) == INVALID
    assert lib.mqc_conv_silu_fwd(fake, 16, fake, None, fake, 0, 8, 16, 4, 0, None) == 0
    need = lib.mqc_conv_silu_bwd_workspace_size(2, 64, 16, 4)
    assert need > 0 and lib.mqc_conv_silu_bwd_workspace_size(2, 64, 16, 9) == 0
    assert lib.mqc_conv_silu_bwd(fake, 16, fake, None, fake, fake, fake, None, 2, 64, 16, 4, 0,
                                 fake, need - 1, None) == INVALID
    assert b"workspace" in lib.mqc_last_error()
    # elementwise glue: null pointers, strides below the width
    assert lib.mqc_scan_inputs_fwd(fake, 16, None, 16, fake, fake, fake, 4, 16, 0, None) == INVALID
    assert lib.mqc_scan_inputs_fwd(fake, 8, fake, 16, fake, fake, fake, 4, 16, 0, None) == INVALID
    assert lib.mqc_gate_residual_fwd(fake, fake, 8, fake, fake, 4, 16, 0, None) == INVALID
    assert lib.mqc_gate_residual_bwd(fake, 16, fake, fake, fake, fake, 4, 16, 3, None) == INVALID
    assert lib.mqc_scan_inputs_bwd(fake, 16, fake, 16, fake, None, None, fake, fake, fake, 0, 16,
                                   0, None) == 0


@no_gpu
def test_time_shard_entry_points_validation_without_gpu():
    """Range summary, carry and resume reject bad arguments before any CUDA call."""
    lib = _lib.load()
    fake = 0x10000
    base = dict(batch=1, seq_len=64, channels=4, d_state=16, dtype=0,
                flags=_lib.MQC_SSM_BC_SHARED | _lib.MQC_SSM_S_REAL, eps=1e-6, reserved0=0,
                delta=fake, lambda_=fake, q=None, Bm=fake, Cm=fake, s=fake, dskip=fake,
                dskip_sb=0, dskip_st=0, dskip_sd=1, h0=None, y=None, hT=None, status=None,
                wait_poll_limit=-1)

    def summary(nchunks=1, P=fake, E=fake, **kw):
        a = _lib.SsmScanArgs(**{**base, **kw})
        return lib.mqc_ssm_scan_fwd_summary(ctypes.byref(a), nchunks, P, E, None, 0, None)

    assert summary(h0=fake) == INVALID  # the summary is the map from the zero state
    assert b"zero state" in lib.mqc_last_error()
    assert summary(hT=fake) == INVALID
    assert summary(flags=_lib.MQC_SSM_Q_GIVEN) == UNSUPPORTED
    assert summary(nchunks=0) == INVALID
    assert summary(P=fake + 4) == INVALID
    assert summary(nchunks=3) == INVALID  # 64 steps do not split into 3 chunks
    assert summary(nchunks=4) == INVALID  # chunks need a workspace
    assert b"workspace" in lib.mqc_last_error()
    assert lib.mqc_ssm_scan_fwd_summary_workspace_size(1, 4, 16, 4) == \
        lib.mqc_ssm_scan_fwd_chunked_workspace_size(1, 4, 16, 4)
    assert lib.mqc_ssm_scan_fwd_summary_workspace_size(1, 4, 16, 1) == 0
    # carry
    assert lib.mqc_ssm_scan_carry(fake, fake, None, fake, fake, -1, 1, 64, None) == INVALID
    assert lib.mqc_ssm_scan_carry(None, fake, None, fake, fake, 2, 1, 64, None) == INVALID
    assert lib.mqc_ssm_scan_carry(fake + 8, fake, None, fake, fake, 2, 1, 64, None) == MISALIGNED
    assert lib.mqc_ssm_scan_carry(fake, fake, None, fake, fake, 2, 0, 64, None) == 0
    # resume needs the summary's workspace
    a = _lib.SsmScanArgs(**{**base, "y": fake})
    assert lib.mqc_ssm_scan_fwd_chunked_resume(ctypes.byref(a), 4, None, 0, None) == INVALID
    assert b"workspace" in lib.mqc_last_error()
    assert lib.mqc_ssm_scan_fwd_chunked_resume(ctypes.byref(a), 3, None, 0, None) == INVALID
