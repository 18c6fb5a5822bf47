"""Configuration types and error classes of the AdaAttention interface.

These mirror the reference's public names and meanings so code written
against hkevin01/AdaAttn keeps working: ``PrecisionMode`` and
``AttentionConfig`` (src/adaattn/attention/base.py:81-235) and the error
hierarchy (base.py:29-78). The member names, defaults, validation rules and
error messages are the interface; the code is this package's own.
"""

from __future__ import annotations

from dataclasses import dataclass
from enum import Enum
from typing import Optional, Tuple

import torch


class AttentionError(Exception):
    """Base class of attention errors (base.py:29-32)."""


class ShapeError(AttentionError):
    """Tensor shapes do not fit together (base.py:35-52)."""

    def __init__(self, message: str, expected_shape: Optional[Tuple] = None,
                 actual_shape: Optional[Tuple] = None) -> None:
        self.expected_shape = expected_shape
        self.actual_shape = actual_shape
        if expected_shape and actual_shape:
            message = f"{message}. Expected shape: {expected_shape}, got: {actual_shape}"
        super().__init__(message)


class MemoryError(AttentionError):  # noqa: A001 - the reference's name
    """Device memory exhausted (base.py:55-72)."""

    def __init__(self, message: str, required_memory: Optional[int] = None,
                 available_memory: Optional[int] = None) -> None:
        self.required_memory = required_memory
        self.available_memory = available_memory
        if required_memory and available_memory:
            message = (f"{message}. Required: {required_memory / 1e9:.2f} GB, "
                       f"Available: {available_memory / 1e9:.2f} GB")
        super().__init__(message)


class NumericalError(AttentionError):
    """NaN or Inf in a result (base.py:75-78)."""


class KernelError(AttentionError):
    """A C-ABI call returned an error status (code = ADA_ERR_*)."""

    def __init__(self, message: str, code: int) -> None:
        self.code = code
        super().__init__(message)


class PrecisionMode(Enum):
    """Arithmetic precision of an attention head (base.py:81-109).

    ``code`` is the C-ABI precision code: the index of the reference's
    ``_precision_distribution`` (adaattn.py:480-485), AUTO = 4.
    """

    FP32 = 1
    FP16 = 2
    BF16 = 3
    FP8 = 4
    AUTO = 5

    @classmethod
    def from_dtype(cls, dtype: torch.dtype) -> "PrecisionMode":
        return {torch.float32: cls.FP32, torch.float16: cls.FP16,
                torch.bfloat16: cls.BF16}.get(dtype, cls.FP32)

    def to_dtype(self) -> torch.dtype:
        # base.py:106-107: FP8 and AUTO compute in float16 in the reference.
        return {PrecisionMode.FP32: torch.float32, PrecisionMode.FP16: torch.float16,
                PrecisionMode.BF16: torch.bfloat16, PrecisionMode.FP8: torch.float16,
                PrecisionMode.AUTO: torch.float16}[self]

    @property
    def code(self) -> int:
        return {PrecisionMode.FP32: 0, PrecisionMode.FP16: 1, PrecisionMode.BF16: 2,
                PrecisionMode.FP8: 3, PrecisionMode.AUTO: 4}[self]

    @classmethod
    def from_code(cls, code: int) -> "PrecisionMode":
        return (cls.FP32, cls.FP16, cls.BF16, cls.FP8, cls.AUTO)[int(code)]

    @classmethod
    def coerce(cls, value) -> "PrecisionMode":
        """Accept this enum, the reference's enum (by member name) or a name."""
        if isinstance(value, cls):
            return value
        name = getattr(value, "name", value)
        if isinstance(name, str) and name.upper() in cls.__members__:
            return cls[name.upper()]
        raise ValueError(f"not a precision mode: {value!r}")


@dataclass
class AttentionConfig:
    """Attention knobs, with the reference's field names and defaults
    (base.py:176-235)."""

    embed_dim: int = 512
    num_heads: int = 8
    dropout: float = 0.0
    precision: PrecisionMode = PrecisionMode.AUTO
    allow_precision_fallback: bool = True
    min_precision: PrecisionMode = PrecisionMode.FP16
    enable_adaptive_rank: bool = False
    min_rank_ratio: float = 0.1
    max_rank_ratio: float = 1.0
    rank_threshold: float = 0.95
    max_memory_fraction: float = 0.9
    enable_gradient_checkpointing: bool = False
    attention_clamp_value: float = 1e4
    softmax_temperature: float = 1.0
    eps: float = 1e-6
    enable_profiling: bool = False
    enable_nan_check: bool = True
    verbose: bool = False

    def validate(self) -> None:
        if self.embed_dim <= 0:
            raise ValueError(f"embed_dim must be positive, got {self.embed_dim}")
        if self.num_heads <= 0:
            raise ValueError(f"num_heads must be positive, got {self.num_heads}")
        if self.embed_dim % self.num_heads != 0:
            raise ValueError(f"embed_dim ({self.embed_dim}) must be divisible by "
                             f"num_heads ({self.num_heads})")
        if not 0.0 <= self.dropout < 1.0:
            raise ValueError(f"dropout must be in [0, 1), got {self.dropout}")
        if not 0.0 < self.min_rank_ratio <= self.max_rank_ratio <= 1.0:
            raise ValueError(
                f"Invalid rank ratio range: [{self.min_rank_ratio}, {self.max_rank_ratio}]")
        if not 0.0 < self.max_memory_fraction <= 1.0:
            raise ValueError(
                f"max_memory_fraction must be in (0, 1], got {self.max_memory_fraction}")

    @property
    def head_dim(self) -> int:
        return self.embed_dim // self.num_heads
