"""ctypes binding of ``libadaattn_b200.so`` (the C ABI in include/adaattn_b200.h).

The library is built in-tree (``adaattn_b200/build.py``). There is no
fallback: if the library is missing or cannot be loaded, every device entry
point raises.
"""

from __future__ import annotations

import ctypes
import os
import re
import threading
from ctypes import (POINTER, Structure, c_char_p, c_double, c_float, c_int32,
                    c_int64, c_size_t, c_uint64, c_void_p)

import torch

from .config import AttentionError, KernelError, MemoryError, NumericalError, ShapeError

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libadaattn_b200.so")
HEADER = os.path.join(os.path.dirname(PKG), "include", "adaattn_b200.h")

ADA_OK = 0
ADA_ERR = {
    -1: "INVALID", -2: "SHAPE", -3: "DTYPE", -4: "DEVICE", -5: "LAYOUT",
    -6: "LAUNCH", -7: "TIMEOUT", -8: "WORKSPACE", -9: "UNSUPPORTED", -10: "CUDA",
}
ADA_ERR_TIMEOUT = -7

ADA_F32, ADA_F16, ADA_BF16, ADA_E4M3, ADA_BOOL, ADA_I32, ADA_I64, ADA_F64 = range(8)
DTYPE_CODE = {
    torch.float32: ADA_F32, torch.float16: ADA_F16, torch.bfloat16: ADA_BF16,
    torch.float8_e4m3fn: ADA_E4M3, torch.bool: ADA_BOOL, torch.uint8: ADA_BOOL,
    torch.int32: ADA_I32, torch.int64: ADA_I64, torch.float64: ADA_F64,
}
SUMMARY_LEN = 12


class AdaTensor(Structure):
    _fields_ = [("data", c_void_p), ("dtype", c_int32), ("ndim", c_int32),
                ("shape", c_int64 * 4), ("stride", c_int64 * 4)]


class AdaAnalyzeParams(Structure):
    _fields_ = [("rank_threshold", c_double), ("scale", c_float), ("eps", c_float),
                ("enable_adaptive_rank", c_int32), ("enable_adaptive_precision", c_int32),
                ("default_precision", c_int32), ("allow_fp8", c_int32),
                ("granularity", c_int32), ("sample_stride", c_int32),
                ("reserved", c_int32 * 2)]


class AdaFwdParams(Structure):
    _fields_ = [("scale", c_float), ("causal", c_int32), ("fp8_mode", c_int32),
                ("static_precision", c_int32), ("static_low_rank", c_int32),
                ("reserved", c_int32 * 3)]


_T = POINTER(AdaTensor)
_SIGNATURES = {
    "ada_abi_version": (c_int32, []),
    "ada_get_last_error": (c_int32, [c_char_p, c_size_t]),
    "ada_poll_device_status": (c_int32, [c_void_p]),
    "ada_analyze_workspace_bytes": (c_size_t, [c_int64, c_int64]),
    "ada_analyze": (c_int32, [_T, _T, POINTER(AdaAnalyzeParams), c_void_p, c_void_p,
                              c_void_p, c_void_p, c_size_t, c_void_p]),
    "ada_analyze_noalloc": (c_int32, [_T, _T, POINTER(AdaAnalyzeParams), c_void_p, c_void_p,
                                      c_void_p, c_void_p]),
    "ada_attn_fwd_workspace_bytes": (c_size_t, [_T, _T, _T, _T, c_void_p,
                                               POINTER(AdaFwdParams), c_int32, c_int32]),
    "ada_attn_fwd": (c_int32, [_T, _T, _T, _T, _T, c_void_p, POINTER(AdaFwdParams),
                               c_int32, c_int32, _T, c_void_p, c_size_t, c_void_p]),
    "ada_attn_fwd_host_buffer_bytes": (c_size_t, [_T, _T, _T, _T, POINTER(AdaFwdParams), c_int64]),
    "ada_attn_fwd_host": (c_int32, [_T, _T, _T, _T, POINTER(AdaFwdParams), _T, c_int64, c_void_p,
                                    c_size_t, c_void_p]),
    "ada_flash_attention_forward": (c_int32, [_T, _T, _T, c_float, c_int32, _T, c_void_p]),
    "ada_compute_entropy": (c_int32, [_T, c_void_p, c_void_p]),
    "ada_estimate_effective_rank": (c_int32, [_T, c_void_p, c_void_p]),
    "ada_determine_target_ranks": (c_int32, [c_void_p, c_int64, c_int64, c_int64, c_double,
                                             c_void_p, c_void_p]),
    "ada_debug_bounded_wait": (c_int32, [c_uint64, c_void_p]),
    "ada_attn_bwd_workspace_bytes": (c_size_t, [c_int64, c_int64, c_int64]),
    "ada_attn_bwd": (c_int32, [_T, _T, _T, _T, _T, _T, c_void_p, c_int32, POINTER(AdaFwdParams),
                               _T, _T, _T, c_void_p, c_size_t, c_void_p]),
    "ada_linear": (c_int32, [_T, _T, _T, _T, c_int32, _T, c_void_p]),
    "ada_layer_norm": (c_int32, [_T, _T, _T, c_float, _T, c_void_p]),
    "ada_record_statistics": (c_int32, [c_void_p, _T, _T, _T, c_void_p]),
    "ada_rsvd_workspace_bytes": (c_size_t, [_T, _T, c_int32]),
    "ada_rsvd": (c_int32, [_T, _T, c_int32, c_int32, _T, _T, _T, c_void_p, c_size_t, c_void_p]),
}

_lock = threading.Lock()
_lib = None


def header_functions():
    """Names of the functions include/adaattn_b200.h declares."""
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(ada_[a-z0-9_]+)\s*\(", text)))


def load():
    """Load the shared library once (raises if it is missing)."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise AttentionError(
                    f"{LIB_PATH} is missing: build it with adaattn_b200.build.build()")
            lib = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in _SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(512)
    load().ada_get_last_error(buf, 512)
    return buf.value.decode(errors="replace")


def check(rc: int, what: str) -> None:
    if rc == ADA_OK:
        return
    msg = f"{what}: {ADA_ERR.get(rc, rc)}: {last_error()}"
    if rc == -2:
        raise ShapeError(msg)
    if rc == -3:
        raise TypeError(msg)
    if rc == -8:
        raise MemoryError(msg)
    raise KernelError(msg, rc)


_I64x4 = c_int64 * 4


def tensor(t: torch.Tensor) -> AdaTensor:
    """Describe a torch tensor (up to 4-D) for the C ABI; no copy."""
    nd = t.dim()
    if nd > 4:
        raise ShapeError(f"at most 4 dimensions, got {nd}")
    code = DTYPE_CODE.get(t.dtype)
    if code is None:
        raise TypeError(f"unsupported dtype {t.dtype}")
    return AdaTensor(t.data_ptr() if t.numel() > 0 else 0, code, nd, _I64x4(*t.shape), _I64x4(*t.stride()))


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t) -> int:
    return 0 if t is None else t.data_ptr()


def poll_device_status(device: torch.device) -> None:
    """Raise if a kernel recorded an error (e.g. a bounded wait timed out)."""
    rc = load().ada_poll_device_status(c_void_p(stream_ptr(device)))
    if rc == ADA_ERR_TIMEOUT:
        raise KernelError(f"device wait timed out: {last_error()}", rc)
    check(rc, "device status")


__all__ = ["AdaTensor", "AdaAnalyzeParams", "AdaFwdParams", "load", "check", "tensor",
           "stream_ptr", "ptr", "header_functions", "last_error", "poll_device_status",
           "NumericalError", "SUMMARY_LEN"]
