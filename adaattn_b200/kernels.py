"""Kernel-level entry points with the names and argument meanings of the
reference's ``adaattn.kernels`` (src/adaattn/kernels/__init__.py:56-252) and
its native module ``_adaattn_cuda`` (src/adaattn/kernels/bindings.cpp:140-189).

All of them run on the C ABI; CPU tensors raise (there is no CPU path).
"""

from __future__ import annotations

from ctypes import c_void_p
from typing import Optional

import torch
from torch import Tensor

from . import _lib, core
from .config import PrecisionMode


def is_cuda_available() -> bool:
    """True when the sm_100a library loads and a CUDA device is present
    (kernels/__init__.py:51-53)."""
    try:
        _lib.load()
    except Exception:
        return False
    return torch.cuda.is_available()


def flash_attention_forward(q: Tensor, k: Tensor, v: Tensor,
                            softmax_scale: Optional[float] = None,
                            causal: bool = False) -> Tensor:
    """Attention on [B, N, H, D] tensors (bindings.cpp:21-68).

    Computes in the tensors' dtype: fp16/bf16 on the tensor cores, fp32 on
    the CUDA cores; returns a [B, N, H, D] tensor.
    """
    core._require_cuda(q, k, v)
    out = torch.empty_like(q, memory_format=torch.contiguous_format)
    lib = _lib.load()
    scale = -1.0 if softmax_scale is None else float(softmax_scale)
    with torch.cuda.device(q.device):
        rc = lib.ada_flash_attention_forward(_lib.tensor(q), _lib.tensor(k), _lib.tensor(v),
                                             scale, int(bool(causal)), _lib.tensor(out),
                                             _lib.stream_ptr(q.device))
    _lib.check(rc, "ada_flash_attention_forward")
    return out


_PRECISION = {"fp16": PrecisionMode.FP16, "bf16": PrecisionMode.BF16,
              "fp32": PrecisionMode.FP32, "fp8": PrecisionMode.FP8}


def adaptive_attention_forward(q: Tensor, k: Tensor, v: Tensor,
                               target_rank: Optional[int] = None, precision: str = "fp16",
                               softmax_scale: Optional[float] = None,
                               causal: bool = False) -> Tensor:
    """Dense attention at a requested precision on [B, N, H, D]
    (kernels/__init__.py:124-213, bindings.cpp:73-96).

    Like the native binding, ``target_rank`` does not change the result: the
    sequence-sketch approximation of the Python fallback draws a fresh random
    projection on every call and is not reproduced.
    """
    core._require_cuda(q, k, v)
    prec = _PRECISION.get(precision, PrecisionMode.FP32)
    d = q.shape[-1]
    scale = softmax_scale if softmax_scale is not None else d ** -0.5
    out = core.attention_forward(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                 scale=scale, causal=causal, static_precision=prec)
    return out.transpose(1, 2)


def compute_entropy(attn_weights: Tensor) -> Tensor:
    """-sum w * log(w + 1e-10) over the last dimension (bindings.cpp:101-109)."""
    core._require_cuda(attn_weights)
    w = attn_weights.contiguous()
    out = torch.empty(w.shape[:-1], dtype=torch.float32, device=w.device)
    lib = _lib.load()
    with torch.cuda.device(w.device):
        rc = lib.ada_compute_entropy(_lib.tensor(w), c_void_p(out.data_ptr()),
                                     _lib.stream_ptr(w.device))
    _lib.check(rc, "ada_compute_entropy")
    return out.to(w.dtype)


def estimate_effective_rank(attn_weights: Tensor) -> Tensor:
    """exp(mean over the second-last dimension of the row entropy)
    (bindings.cpp:114-118)."""
    core._require_cuda(attn_weights)
    w = attn_weights.contiguous()
    out = torch.empty(w.shape[:-2], dtype=torch.float32, device=w.device)
    lib = _lib.load()
    with torch.cuda.device(w.device):
        rc = lib.ada_estimate_effective_rank(_lib.tensor(w), c_void_p(out.data_ptr()),
                                             _lib.stream_ptr(w.device))
    _lib.check(rc, "ada_estimate_effective_rank")
    return out.to(w.dtype)


def determine_target_ranks(effective_rank: Tensor, min_rank: int = 8, max_rank: int = 128,
                           threshold: float = 32.0) -> Tensor:
    """clamp(1.5 * rank) where rank < threshold, else max_rank, as int64
    (bindings.cpp:123-135)."""
    core._require_cuda(effective_rank)
    e = effective_rank.float().contiguous()
    out = torch.empty(e.shape, dtype=torch.int64, device=e.device)
    lib = _lib.load()
    with torch.cuda.device(e.device):
        rc = lib.ada_determine_target_ranks(c_void_p(e.data_ptr()), e.numel(), int(min_rank),
                                            int(max_rank), float(threshold),
                                            c_void_p(out.data_ptr()), _lib.stream_ptr(e.device))
    _lib.check(rc, "ada_determine_target_ranks")
    return out


__all__ = ["is_cuda_available", "flash_attention_forward", "adaptive_attention_forward",
           "compute_entropy", "estimate_effective_rank", "determine_target_ranks"]
