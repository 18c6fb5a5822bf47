"""adaattn_b200: the AdaAttn attention-forward path on B200 (sm_100a).

Public surface, mirroring hkevin01/AdaAttn's attention package:
``AdaAttention`` (module), ``PrecisionMode``, ``AttentionConfig`` and the error
types; ``analyze`` / ``attention_forward`` for [B, H, N, D] tensors; and
``adaattn_b200.kernels`` for the reference's kernel-level functions.
"""

from .config import (AttentionConfig, AttentionError, KernelError, MemoryError,
                     NumericalError, PrecisionMode, ShapeError)
from .core import DecisionTable, analyze, attention_forward, attention_forward_host
from .attention import AdaAttention

__all__ = [
    "AdaAttention", "AttentionConfig", "AttentionError", "KernelError", "MemoryError",
    "NumericalError", "PrecisionMode", "ShapeError", "DecisionTable", "analyze",
    "attention_forward",
    "attention_forward_host",
]

__version__ = "0.1.0"
