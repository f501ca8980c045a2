"""ctypes binding of ``libmambaqc_b200.so`` (the C ABI in ``include/mambaqc_b200.h``).

The library is built in-tree (``python -m mambaqc_b200.csrc.build``) and loaded
from this package's folder. There is no CPU fallback: every op of this package
requires CUDA tensors and this library; a missing library raises at first use.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

# MAMBAQC_B200_LIBRARY points at another build of the same library (to compare builds).
LIB_PATH = Path(os.environ.get("MAMBAQC_B200_LIBRARY")
                or Path(__file__).resolve().parent / "libmambaqc_b200.so")

MQC_DTYPE_F32 = 0
MQC_DTYPE_BF16 = 1

MQC_OK = 0
MQC_ERR_DEVICE_TIMEOUT = 5
MQC_DEVICE_STATUS_TIMEOUT = 0x1

MQC_SSM_Q_GIVEN = 0x1
MQC_SSM_BC_SHARED = 0x2
MQC_SSM_S_REAL = 0x4

MQC_QLN_PADDED_COMPAT = 0x1

_c_void_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int
_f32 = ctypes.c_float


class SsmScanArgs(ctypes.Structure):
    """Mirror of ``mqc_ssm_scan_args``."""

    _fields_ = [
        ("batch", _i64), ("seq_len", _i64), ("channels", _i64), ("d_state", _i64),
        ("dtype", ctypes.c_int32), ("flags", ctypes.c_int32), ("eps", _f32),
        ("reserved0", ctypes.c_int32),
        ("delta", _c_void_p), ("lambda_", _c_void_p), ("q", _c_void_p), ("Bm", _c_void_p),
        ("Cm", _c_void_p), ("s", _c_void_p), ("dskip", _c_void_p),
        ("dskip_sb", _i64), ("dskip_st", _i64), ("dskip_sd", _i64),
        ("h0", _c_void_p), ("y", _c_void_p), ("hT", _c_void_p), ("status", _c_void_p),
        ("wait_poll_limit", _i64), ("ckpt", _c_void_p), ("ckpt_every", _i64),
    ]


MQC_SSM_CKPT_EVERY = 8


class SsmScanBwdArgs(ctypes.Structure):
    """Mirror of ``mqc_ssm_scan_bwd_args``."""

    _fields_ = [
        ("batch", _i64), ("seq_len", _i64), ("channels", _i64), ("d_state", _i64),
        ("dtype", ctypes.c_int32), ("flags", ctypes.c_int32), ("eps", _f32),
        ("ckpt_every", ctypes.c_int32),
        ("delta", _c_void_p), ("lambda_", _c_void_p), ("Bm", _c_void_p), ("Cm", _c_void_p),
        ("s", _c_void_p), ("dskip", _c_void_p),
        ("dskip_sb", _i64), ("dskip_st", _i64), ("dskip_sd", _i64),
        ("h0", _c_void_p), ("ckpt", _c_void_p), ("dy", _c_void_p), ("dhT", _c_void_p),
        ("ddelta", _c_void_p), ("dlambda_part", _c_void_p), ("dBm", _c_void_p),
        ("dCm", _c_void_p), ("ds", _c_void_p), ("dh0", _c_void_p),
    ]


class BcProjScanArgs(ctypes.Structure):
    """Mirror of ``mqc_bc_proj_scan_args``."""

    _fields_ = [
        ("batch", _i64), ("seq_len", _i64), ("channels", _i64), ("d_state", _i64),
        ("in_features", _i64), ("dtype", ctypes.c_int32), ("eps", _f32),
        ("x", _c_void_p), ("w_b", _c_void_p), ("w_c", _c_void_p), ("delta", _c_void_p),
        ("s", _c_void_p), ("lambda_", _c_void_p), ("dskip", _c_void_p), ("dskip_sd", _i64),
        ("h0", _c_void_p), ("hT", _c_void_p), ("y", _c_void_p), ("status", _c_void_p),
        ("wait_poll_limit", _i64),
    ]


# name -> (argtypes); every function returns int status unless listed in _STR_FUNCS
_SIGNATURES = {
    "mqc_qmul": [_c_void_p, _c_void_p, _c_void_p, _i64, _i32, _c_void_p],
    "mqc_qmul_strided": [_c_void_p, _c_void_p, _c_void_p, ctypes.POINTER(_i64),
                         ctypes.POINTER(_i64), ctypes.POINTER(_i64), _i32, _c_void_p],
    "mqc_qconj": [_c_void_p, _c_void_p, _i64, _i32, _c_void_p],
    "mqc_qinv": [_c_void_p, _c_void_p, _i64, _f32, _i32, _c_void_p],
    "mqc_qnorm": [_c_void_p, _c_void_p, _i64, _i32, _c_void_p],
    "mqc_cayley": [_c_void_p, _c_void_p, _i64, _f32, _i32, _c_void_p],
    "mqc_cayley_bwd": [_c_void_p, _c_void_p, _c_void_p, _i64, _f32, _i32, _c_void_p],
    "mqc_prefix_prod": [_c_void_p, _c_void_p, _i64, _i64, _i64, _i32, _c_void_p],
    "mqc_prefix_prod_noalloc": [_c_void_p, _c_void_p, _i64, _i64, _i64, _i32, _c_void_p],
    "mqc_ssm_scan_fwd": [ctypes.POINTER(SsmScanArgs), _c_void_p],
    "mqc_ssm_scan_fwd_host": [ctypes.POINTER(SsmScanArgs), _i64, _c_void_p],
    "mqc_ssm_scan_bwd": [ctypes.POINTER(SsmScanBwdArgs), _c_void_p],
    "mqc_ssm_scan_fwd_chunked": [ctypes.POINTER(SsmScanArgs), _i64, _c_void_p, ctypes.c_size_t,
                                 _c_void_p],
    "mqc_ssm_step": [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
                     _c_void_p, _c_void_p, _i64, _i64, _i64, _i32, _c_void_p],
    "mqc_qln_fwd": [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
                    _i64, _i64, _f32, _i32, _i32, _c_void_p],
    "mqc_qln_bwd": [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
                    _c_void_p, _c_void_p, _c_void_p, ctypes.c_size_t, _i64, _i64, _f32, _i32,
                    _c_void_p],
}
_SIGNATURES["mqc_probe_fp32_fma"] = [_c_void_p, _i64, ctypes.POINTER(_i64), _c_void_p]
_SIGNATURES.update({
    "mqc_conv_silu_fwd": [_c_void_p, _i64, _c_void_p, _c_void_p, _c_void_p, _i64, _i64, _i64,
                          _i64, _i32, _c_void_p],
    "mqc_conv_silu_bwd": [_c_void_p, _i64, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
                          _c_void_p, _c_void_p, _i64, _i64, _i64, _i64, _i32, _c_void_p,
                          ctypes.c_size_t, _c_void_p],
    "mqc_scan_inputs_fwd": [_c_void_p, _i64, _c_void_p, _i64, _c_void_p, _c_void_p, _c_void_p,
                            _i64, _i64, _i32, _c_void_p],
    "mqc_scan_inputs_bwd": [_c_void_p, _i64, _c_void_p, _i64, _c_void_p, _c_void_p, _c_void_p,
                            _c_void_p, _c_void_p, _c_void_p, _i64, _i64, _i32, _c_void_p],
    "mqc_gate_residual_fwd": [_c_void_p, _c_void_p, _i64, _c_void_p, _c_void_p, _i64, _i64,
                              _i32, _c_void_p],
    "mqc_gate_residual_bwd": [_c_void_p, _i64, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
                              _i64, _i64, _i32, _c_void_p],
    "mqc_ssm_scan_fwd_summary": [ctypes.POINTER(SsmScanArgs), _i64, _c_void_p, _c_void_p,
                                 _c_void_p, ctypes.c_size_t, _c_void_p],
    "mqc_ssm_scan_carry": [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i64, _i64,
                           _i64, _c_void_p],
    "mqc_ssm_scan_fwd_chunked_resume": [ctypes.POINTER(SsmScanArgs), _i64, _c_void_p,
                                        ctypes.c_size_t, _c_void_p],
    "mqc_peer_alloc": [ctypes.c_size_t, ctypes.POINTER(_c_void_p), _c_void_p],
    "mqc_peer_free": [_c_void_p],
    "mqc_peer_open": [_c_void_p, ctypes.POINTER(_c_void_p)],
    "mqc_peer_close": [_c_void_p],
    "mqc_ssm_scan_fwd_chunked_peer": [ctypes.POINTER(SsmScanArgs), _i64, _c_void_p,
                                      ctypes.c_size_t, ctypes.POINTER(_c_void_p), _i32, _i64,
                                      _i64, _c_void_p],
    "mqc_qln_linear_fwd": [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
                           _c_void_p, _c_void_p, _i64, _i64, _i64, _f32, _c_void_p, _c_void_p],
    "mqc_bc_proj_scan_fwd": [ctypes.POINTER(BcProjScanArgs), _c_void_p],
    "mqc_ssm_scan_fwd_chunked_multicast": [ctypes.POINTER(SsmScanArgs), _i64, _c_void_p,
                                           ctypes.c_size_t, _c_void_p, _i64, _i64, _c_void_p],
    "mqc_channel_push": [_c_void_p, ctypes.POINTER(_c_void_p), _i32, _i64, _i64, _i64, _i64,
                         _i64, _i64, _i64, _i32, _c_void_p],
})
MQC_PEER_HANDLE_BYTES = 64
_SIZE_FUNCS = {"mqc_qln_bwd_workspace_size": [_i64, _i64],
               "mqc_ssm_scan_fwd_chunked_workspace_size": [_i64, _i64, _i64, _i64],
               "mqc_conv_silu_bwd_workspace_size": [_i64, _i64, _i64, _i64],
               "mqc_ssm_scan_fwd_summary_workspace_size": [_i64, _i64, _i64, _i64]}
_STR_FUNCS = {"mqc_version": [], "mqc_status_string": [_i32], "mqc_last_error": []}

_lock = threading.Lock()
_lib = None


def load() -> ctypes.CDLL:
    """Load the shared library once (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"mambaqc_b200: {LIB_PATH.name} is not built; run "
                    "`python -m mambaqc_b200.csrc.build` (nvcc, sm_100a)")
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, args in _SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = args
                fn.restype = _i32
            for name, args in _SIZE_FUNCS.items():
                fn = getattr(lib, name)
                fn.argtypes = args
                fn.restype = ctypes.c_size_t
            for name, args in _STR_FUNCS.items():
                fn = getattr(lib, name)
                fn.argtypes = args
                fn.restype = ctypes.c_char_p
            _lib = lib
    return _lib


def exported_symbols() -> list[str]:
    return sorted([*_SIGNATURES, *_SIZE_FUNCS, *_STR_FUNCS])


def check(rc: int, what: str) -> None:
    if rc != MQC_OK:
        lib = load()
        detail = lib.mqc_last_error().decode(errors="replace")
        status = lib.mqc_status_string(rc).decode(errors="replace")
        raise RuntimeError(f"{what} failed: {status} ({rc}): {detail}")


def call(name: str, *args) -> None:
    lib = load()
    check(getattr(lib, name)(*args), name)


def dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.float32:
        return MQC_DTYPE_F32
    if t.dtype == torch.bfloat16:
        return MQC_DTYPE_BF16
    raise TypeError(f"mambaqc_b200: unsupported dtype {t.dtype} (float32 or bfloat16)")


def require_cuda(*tensors: torch.Tensor, what: str = "mambaqc_b200") -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError(
                f"{what}: CUDA tensors required (this package has no CPU path); got {t.device}")


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def aligned_contig(t: torch.Tensor, align: int = 16) -> torch.Tensor:
    """Contiguous tensor whose data pointer is ``align``-byte aligned (copy if needed)."""
    t = t.contiguous()
    if t.data_ptr() % align:
        t = t.clone()
    return t


_status_words: dict[int, torch.Tensor] = {}


def status_word(device: torch.device) -> torch.Tensor:
    """Per-device int32 word the scan kernels OR MQC_DEVICE_STATUS_* bits into."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    w = _status_words.get(idx)
    if w is None:
        w = torch.zeros(1, dtype=torch.int32, device=f"cuda:{idx}")
        _status_words[idx] = w
    return w


def sync_checks_enabled() -> bool:
    return os.environ.get("MAMBAQC_B200_SYNC_CHECK", "0") == "1"


def check_device_status(device: torch.device | None = None, reset: bool = True) -> None:
    """Synchronise and raise if any kernel on ``device`` reported a device-side timeout."""
    devs = [device] if device is not None else [torch.device(f"cuda:{i}") for i in _status_words]
    for d in devs:
        w = status_word(d)
        val = int(w.item())
        if reset and val:
            w.zero_()
        if val & MQC_DEVICE_STATUS_TIMEOUT:
            raise RuntimeError("mambaqc_b200: a bounded device-side wait timed out "
                               f"(status 0x{val:x} on {d}); results of that launch are invalid")
