"""``AdaAttention``: the reference's module interface over the sm_100a kernels.

Constructor, ``forward`` signature, parameter and buffer names, statistics
keys and error behaviour follow src/adaattn/attention/adaattn.py:57-552 and
src/adaattn/attention/base.py:329-622, so the module drops into the
reference's examples/transformer_integration.py and a reference
``state_dict`` loads into it. What differs is where the work runs:

* the analyzer, the branch choice and the per-precision arithmetic run on the
  GPU with no host synchronisation; decisions are made per (b, h) slice by
  default (``decision_granularity="head"``) or once per call exactly like the
  reference (``"global"``);
* heads deciding FP8 run real tile-scaled E4M3 tensor-core arithmetic
  (``fp8_compute="e4m3"``) or the reference's fp16 stand-in (``"fp16"``);
* the reference's per-call ``gc.collect()`` / ``empty_cache()`` and the
  flash_attn bypass (base.py:281-326, adaattn.py:421-445) are not reproduced.
"""

from __future__ import annotations

import logging
import math
from typing import Literal, Optional, Tuple

import torch
import torch.nn as nn
from torch import Tensor

from . import core
from .config import (AttentionConfig, MemoryError, NumericalError, PrecisionMode,
                     ShapeError)

logger = logging.getLogger(__name__)


class _AttentionGrad(torch.autograd.Function):
    """Autograd for the fused attention core (the reference gets its
    gradients from ATen, tests/unit/test_adaattn_unified.py:146-159).

    The forward has already run (the fused kernels wrote ``merged``); this
    node only records what the backward needs. Its backward calls
    ``ada_attn_bwd`` per branch: dense heads on q, k; low-rank heads on
    q_low = q Wᵀ, k_low = k Wᵀ (recomputed in the inputs' dtype, as the
    forward projects them), then chains W: dq += dq_low W, dW = Σ dq_lowᵀ q +
    dk_lowᵀ k. Gradients are those of softmax(q kᵀ·scale + mask) v evaluated
    in fp32 at the operands' values, whatever precision the head's forward
    used.
    """

    @staticmethod
    def forward(ctx, merged, q, k, v, w_down, table, mask, scale, causal, low_possible):
        ctx.save_for_backward(merged, q, k, v, w_down)
        ctx.table, ctx.mask, ctx.scale, ctx.causal = table, mask, scale, causal
        ctx.low_possible = low_possible
        return merged

    @staticmethod
    def backward(ctx, grad):
        merged, q, k, v, w_down = ctx.saved_tensors
        out = merged.transpose(1, 2)
        dout = grad.transpose(1, 2)
        table, mask = ctx.table, ctx.mask
        kw = dict(scale=ctx.scale, causal=ctx.causal, table=table, attention_mask=mask)
        dq, dk, dv = core.attention_backward(q, k, v, out, dout, low_rank=False, **kw)
        dw = None
        if table is not None and ctx.low_possible and w_down is not None:
            q_low = nn.functional.linear(q, w_down.to(q.dtype))
            k_low = nn.functional.linear(k, w_down.to(k.dtype))
            dql, dkl, dvl = core.attention_backward(q_low, k_low, v, out, dout, low_rank=True, **kw)
            wf = w_down.float()
            dq = dq + torch.matmul(dql, wf)
            dk = dk + torch.matmul(dkl, wf)
            dv = dv + dvl
            if ctx.needs_input_grad[4]:
                dw = (torch.einsum("bhnr,bhnd->rd", dql, q.float())
                      + torch.einsum("bhnr,bhnd->rd", dkl, k.float())).to(w_down.dtype)
        return (None, dq.to(q.dtype), dk.to(k.dtype), dv.to(v.dtype), dw, None, None, None, None,
                None)


class AdaAttention(nn.Module):
    """Adaptive precision and rank attention (AdaAttn) on B200."""

    def __init__(
        self,
        embed_dim: int = 512,
        num_heads: int = 8,
        dropout: float = 0.0,
        enable_adaptive_rank: bool = True,
        rank_ratio: float = 0.5,
        rank_estimation_method: Literal["entropy", "power", "random"] = "entropy",
        rank_threshold: float = 0.95,
        enable_adaptive_precision: bool = True,
        default_precision: PrecisionMode = PrecisionMode.FP16,
        allow_fp8: bool = False,
        enable_gpu_optimization: bool = True,
        causal: bool = False,
        bias: bool = True,
        config: Optional[AttentionConfig] = None,
        decision_granularity: Literal["head", "global"] = "head",
        fp8_compute: Literal["e4m3", "fp16"] = "e4m3",
        sample_stride: int = 1,
        **kwargs,
    ) -> None:
        super().__init__()
        default_precision = PrecisionMode.coerce(default_precision)
        if config is None:
            config = AttentionConfig(
                embed_dim=embed_dim, num_heads=num_heads, dropout=dropout,
                enable_adaptive_rank=enable_adaptive_rank, rank_threshold=rank_threshold,
                precision=default_precision, **kwargs)
        config.validate()
        self.config = config
        self._metrics = None
        if decision_granularity not in ("head", "global"):
            raise ValueError("decision_granularity must be 'head' or 'global'")
        if fp8_compute not in ("e4m3", "fp16"):
            raise ValueError("fp8_compute must be 'e4m3' or 'fp16'")
        self.decision_granularity = decision_granularity
        self.fp8_compute = fp8_compute
        self.sample_stride = int(sample_stride)

        self.enable_adaptive_rank = enable_adaptive_rank
        self.enable_adaptive_precision = enable_adaptive_precision
        self.rank_ratio = rank_ratio
        self.rank_estimation_method = rank_estimation_method
        self.rank_threshold = rank_threshold
        self.default_precision = default_precision
        self.allow_fp8 = allow_fp8
        self.causal = causal
        self.enable_gpu_optimization = enable_gpu_optimization

        self.q_proj = nn.Linear(embed_dim, embed_dim, bias=bias)
        self.k_proj = nn.Linear(embed_dim, embed_dim, bias=bias)
        self.v_proj = nn.Linear(embed_dim, embed_dim, bias=bias)
        self.out_proj = nn.Linear(embed_dim, embed_dim, bias=bias)
        if enable_adaptive_rank:
            max_rank = max(1, int(self.head_dim * rank_ratio))
            self.rank_proj_down = nn.Linear(self.head_dim, max_rank, bias=False)
            self.rank_proj_up = nn.Linear(max_rank, self.head_dim, bias=False)
        else:
            self.rank_proj_down = None
            self.rank_proj_up = None
        self.attn_dropout = nn.Dropout(dropout)
        self.resid_dropout = nn.Dropout(dropout)
        self.scale = 1.0 / math.sqrt(self.head_dim)

        self.register_buffer("_call_count", torch.tensor(0))
        # Fractional in per-head mode (share of heads on the low-rank branch).
        self.register_buffer("_low_rank_calls", torch.tensor(0.0, dtype=torch.float64))
        self.register_buffer("_precision_distribution", torch.zeros(4))
        self.last_decisions: Optional[core.DecisionTable] = None
        self._reset_parameters()

    # -- reference properties -------------------------------------------------
    @property
    def embed_dim(self) -> int:
        return self.config.embed_dim

    @property
    def num_heads(self) -> int:
        return self.config.num_heads

    @property
    def head_dim(self) -> int:
        return self.config.head_dim

    @property
    def metrics(self):
        return self._metrics

    def _reset_parameters(self) -> None:
        # adaattn.py:169-183
        for proj in (self.q_proj, self.k_proj, self.v_proj, self.out_proj):
            nn.init.xavier_uniform_(proj.weight)
            if proj.bias is not None:
                nn.init.zeros_(proj.bias)
        if self.rank_proj_down is not None:
            nn.init.orthogonal_(self.rank_proj_down.weight)
        if self.rank_proj_up is not None:
            nn.init.orthogonal_(self.rank_proj_up.weight)

    def _load_from_state_dict(self, state_dict, prefix, local_metadata, strict,
                              missing_keys, unexpected_keys, error_msgs):
        # A reference state dict may carry the flash_attn call counter.
        state_dict.pop(prefix + "_flash_calls", None)
        super()._load_from_state_dict(state_dict, prefix, local_metadata, strict,
                                      missing_keys, unexpected_keys, error_msgs)

    # -- validation (base.py:389-464) -------------------------------------------
    def _validate_inputs(self, query, key, value, attention_mask=None) -> None:
        for name, t in (("query", query), ("key", key), ("value", value)):
            if not isinstance(t, Tensor):
                raise TypeError(f"{name} must be a Tensor, got {type(t)}")
        for name, t in (("query", query), ("key", key), ("value", value)):
            if t.ndim != 3:
                raise ShapeError(f"{name} must be 3D (batch, seq, embed_dim)",
                                 expected_shape=("batch", "seq", "embed_dim"),
                                 actual_shape=tuple(t.shape))
        if query.size(0) != key.size(0) or query.size(0) != value.size(0):
            raise ShapeError(f"Batch sizes must match: query={query.size(0)}, "
                             f"key={key.size(0)}, value={value.size(0)}")
        if key.size(1) != value.size(1):
            raise ShapeError(f"Key and value sequence lengths must match: "
                             f"key={key.size(1)}, value={value.size(1)}")
        if query.size(2) != self.embed_dim:
            raise ShapeError("Query embedding dimension mismatch",
                             expected_shape=(None, None, self.embed_dim),
                             actual_shape=tuple(query.shape))
        if attention_mask is not None and attention_mask.ndim not in (2, 3, 4):
            raise ShapeError(
                f"attention_mask must be 2D, 3D, or 4D, got {attention_mask.ndim}D")

    def _check_numerical_stability(self, tensor: Tensor, name: str = "tensor") -> None:
        # base.py:466-492
        if not self.config.enable_nan_check:
            return
        if tensor.is_cuda and torch.cuda.is_current_stream_capturing():
            # A forward being captured into a CUDA graph cannot read the
            # device; the check runs on eager forwards only.
            return
        if torch.isnan(tensor).any():
            raise NumericalError(f"NaN values detected in {name}. "
                                 "Consider using higher precision or gradient clipping.")
        if torch.isinf(tensor).any():
            raise NumericalError(f"Inf values detected in {name}. "
                                 "Consider reducing learning rate or using gradient clipping.")

    # -- forward ---------------------------------------------------------------
    def forward(self, query: Tensor, key: Tensor, value: Tensor,
                attention_mask: Optional[Tensor] = None, need_weights: bool = False
                ) -> Tuple[Tensor, Optional[Tensor]]:
        """[B, N, E] in, ([B, Nq, E], None) out -- base.py:538-613."""
        self._validate_inputs(query, key, value, attention_mask)
        try:
            output, weights = self._forward_impl(query, key, value, attention_mask,
                                                 need_weights)
            self._check_numerical_stability(output, "attention output")
            return output, weights
        except torch.cuda.OutOfMemoryError as e:
            raise MemoryError(f"GPU out of memory: {e}") from e

    def forward_with_residual(self, x: Tensor, attention_mask: Optional[Tensor] = None) -> Tensor:
        """``x + self(x, x, x)[0]`` for self-attention, the residual sum of the
        host transformer block (examples/transformer_integration.py:47-48)
        fused into out_proj's epilogue (rounded like the two PyTorch ops:
        out_proj's result, then the sum). The output dropout must be inactive
        (eval mode or p = 0)."""
        if self.training and self.resid_dropout.p > 0:
            raise RuntimeError("forward_with_residual needs the output dropout inactive (eval() or p=0)")
        self._validate_inputs(x, x, x, attention_mask)
        try:
            output, _ = self._forward_impl(x, x, x, attention_mask, residual=x)
            self._check_numerical_stability(output, "attention output")
            return output
        except torch.cuda.OutOfMemoryError as e:
            raise MemoryError(f"GPU out of memory: {e}") from e

    @staticmethod
    def _dense_on_tensor_cores(x: Tensor) -> bool:
        # The tensor-core layer (core.linear) serves 16-bit CUDA tensors; fp32
        # layers stay on the reference's own fp32 Linear, whose rounding a
        # tensor-core product would change.
        return x.is_cuda and x.dtype in (torch.bfloat16, torch.float16)

    def _linear(self, layer: nn.Linear, x: Tensor, residual: Optional[Tensor] = None) -> Tensor:
        if self._dense_on_tensor_cores(x):
            return core.linear(x, layer.weight, layer.bias, residual=residual)
        y = layer(x)
        return y if residual is None else residual + y

    def _forward_impl(self, query, key, value, attention_mask=None, need_weights=False, residual=None):
        # adaattn.py:396-460 without the flash_attn branch.
        b, nq, _ = query.shape
        nk = key.shape[1]
        h, d = self.num_heads, self.head_dim
        if query is key and key is value:
            # Self-attention: one GEMM against the stacked q/k/v weights
            # (same values as the three Linears); q, k, v are column views.
            w, bias = self._stacked_qkv()
            if self._dense_on_tensor_cores(query):
                qkv = core.linear(query, w, bias)
            else:
                qkv = torch.nn.functional.linear(query, w, bias)
            e = self.embed_dim
            q, k, v = (qkv[..., i * e:(i + 1) * e].view(b, nq, h, d).transpose(1, 2) for i in range(3))
        else:
            q = self._linear(self.q_proj, query).view(b, nq, h, d).transpose(1, 2)
            k = self._linear(self.k_proj, key).view(b, nk, h, d).transpose(1, 2)
            v = self._linear(self.v_proj, value).view(b, nk, h, d).transpose(1, 2)
        merged = torch.empty(b, nq, h, d, dtype=q.dtype, device=q.device)
        attn_out, _ = self.attention_core(q, k, v, attention_mask, out=merged.transpose(1, 2))
        w_down = self.rank_proj_down.weight if self.rank_proj_down is not None else None
        if torch.is_grad_enabled() and (any(t.requires_grad for t in (q, k, v))
                                        or (w_down is not None and w_down.requires_grad)):
            merged = _AttentionGrad.apply(merged, q, k, v, w_down, self.last_decisions,
                                          attention_mask, self.scale, self.causal,
                                          self.enable_adaptive_rank)
        if residual is not None:
            return self._linear(self.out_proj, merged.view(b, nq, self.embed_dim), residual), None
        output = self.resid_dropout(self._linear(self.out_proj, merged.view(b, nq, self.embed_dim)))
        return output, None

    def _stacked_qkv(self) -> Tuple[Tensor, Optional[Tensor]]:
        """[3E, E] weight and [3E] bias of q_proj, k_proj, v_proj stacked; kept
        between calls (outside the state dict) until a parameter changes,
        rebuilt on every call when autograd tracks the parameters."""
        ws = (self.q_proj.weight, self.k_proj.weight, self.v_proj.weight)
        bs = (self.q_proj.bias, self.k_proj.bias, self.v_proj.bias)
        has_bias = all(t is not None for t in bs)
        if torch.is_grad_enabled() and any(t.requires_grad for t in ws + (bs if has_bias else ())):
            return torch.cat(ws), (torch.cat(bs) if has_bias else None)
        params = ws + (bs if has_bias else ())
        key = tuple((t.data_ptr(), t._version, t.dtype, t.device) for t in params)
        if getattr(self, "_qkv_key", None) != key:
            with torch.no_grad():
                self._qkv_w = torch.cat(ws)
                self._qkv_b = torch.cat(bs) if has_bias else None
            self._qkv_key = key
        return self._qkv_w, self._qkv_b

    def attention_core(self, q: Tensor, k: Tensor, v: Tensor,
                       attention_mask: Optional[Tensor] = None, out: Optional[Tensor] = None
                       ) -> Tuple[Tensor, Optional[core.DecisionTable]]:
        """Adaptive attention on [B, H, N, D] -- adaattn.py:462-504.

        Returns (output [B, H, Nq, D], the decision table or None when the
        decisions are fixed by the configuration).
        """
        if self.training and self.attn_dropout.p > 0:
            raise NotImplementedError(
                "attention-probability dropout in training mode is not part of the fused "
                "forward kernels; use eval() or dropout=0")
        if q.shape[2] == 0 or k.shape[2] == 0:
            raise ValueError("math domain error: the analyzer sample is empty")
        w_down = self.rank_proj_down.weight if self.rank_proj_down is not None else None
        if w_down is not None and w_down.dtype != q.dtype:
            raise RuntimeError(
                f"rank_proj_down is {w_down.dtype} but the inputs are {q.dtype}; cast the "
                "module to the input dtype (the reference's Linear fails the same way)")
        static = not self.enable_adaptive_precision and not (
            self.enable_adaptive_rank and self.rank_proj_down is not None)
        fp8_mode = self.fp8_compute
        table = None
        if static and not self.config.enable_profiling:
            out = core.attention_forward(
                q, k, v, scale=self.scale, causal=self.causal, table=None,
                static_precision=self.default_precision, static_low_rank=False,
                attention_mask=attention_mask, fp8_mode=fp8_mode, out=out)
            self._record_static()
        else:
            table = core.analyze(
                q, k, scale=self.scale, eps=self.config.eps, rank_threshold=self.rank_threshold,
                enable_adaptive_rank=self.enable_adaptive_rank and self.rank_proj_down is not None,
                enable_adaptive_precision=self.enable_adaptive_precision,
                default_precision=self.default_precision, allow_fp8=self.allow_fp8,
                granularity=self.decision_granularity, sample_stride=self.sample_stride)
            out = core.attention_forward(
                q, k, v, scale=self.scale, causal=self.causal, table=table, w_down=w_down,
                attention_mask=attention_mask,
                possible_mask=core.possible_precisions(self.enable_adaptive_precision,
                                                       self.default_precision, self.allow_fp8),
                low_rank_possible=self.enable_adaptive_rank and w_down is not None,
                fp8_mode=fp8_mode, out=out)
            self._record(table)
        self.last_decisions = table
        return out, table

    # -- statistics (adaattn.py:476-486, :506-544) ------------------------------
    def _record(self, table: core.DecisionTable) -> None:
        # One launch, on the device, in the buffers' dtypes (ada_record_statistics).
        core.record_statistics(table.summary, self._call_count, self._low_rank_calls,
                               self._precision_distribution)

    def _record_static(self) -> None:
        self._call_count += 1
        idx = self.default_precision.code if self.default_precision.code < 4 else 0
        self._precision_distribution[idx] += 1

    def get_statistics(self) -> dict:
        call_count = int(self._call_count.item())
        if call_count > 0:
            low_rank_ratio = float(self._low_rank_calls.item()) / call_count
            dist = (self._precision_distribution / call_count).tolist()
        else:
            low_rank_ratio = 0.0
            dist = [0.0, 0.0, 0.0, 0.0]
        return {
            "call_count": call_count,
            "low_rank_ratio": low_rank_ratio,
            "precision_distribution": {"FP32": dist[0], "FP16": dist[1], "BF16": dist[2],
                                       "FP8": dist[3]},
            "flash_calls": 0,
            "flash_ratio": 0.0,
            "gpu_optimizations_available": True,
            "flash_attention_available": False,
            "decision_granularity": self.decision_granularity,
        }

    def extra_repr(self) -> str:
        return (f"embed_dim={self.embed_dim}, num_heads={self.num_heads}, "
                f"head_dim={self.head_dim}, dropout={self.config.dropout}, "
                f"adaptive_rank={self.enable_adaptive_rank}, "
                f"adaptive_precision={self.enable_adaptive_precision}")
