"""Functional core of the hot path on [B, H, N, D] device tensors.

``analyze`` is the runtime analyzer (K1) and ``attention_forward`` the
adaptive attention core (K2 / K3 + operand preparation). Both enqueue work on
the current CUDA stream and never synchronise with the host: decisions live
in device memory and are read by the kernels directly.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import torch

from . import _lib
from .config import PrecisionMode, ShapeError


@dataclass
class DecisionTable:
    """Per-(b, h) decisions of one call, in device memory.

    decisions  int32 [B, H, 2]: precision code (FP32=0, FP16=1, BF16=2, FP8=3,
               AUTO=4) and the low-rank flag.
    head_stats float32 [B, H, 4]: normalized entropy, max |score|, max prob,
               effective rank (ne * min(Nq, Nk)).
    summary    float32 [12]: the call-level statistics and counts (see
               ADA_SUM_* in include/adaattn_b200.h).
    """

    decisions: torch.Tensor
    head_stats: torch.Tensor
    summary: torch.Tensor
    granularity: str
    head_sum: Optional[torch.Tensor] = None  # [B, H] sums of normalised row entropies

    @property
    def precision(self) -> torch.Tensor:
        return self.decisions[..., 0]

    @property
    def low_rank(self) -> torch.Tensor:
        return self.decisions[..., 1].bool()

    def as_dict(self) -> dict:
        """Host copy (synchronises) for logging."""
        names = ("FP32", "FP16", "BF16", "FP8", "AUTO")
        prec = self.precision.cpu()
        low = self.low_rank.cpu()
        return {
            "precision": [[names[int(p)] for p in row] for row in prec.tolist()],
            "low_rank": low.tolist(),
            "head_stats": self.head_stats.cpu().tolist(),
        }


def _require_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError(
                "adaattn_b200 runs on CUDA devices only (sm_100a); got a tensor on "
                f"{t.device}. There is no CPU path.")


def possible_precisions(enable_adaptive_precision: bool, default: PrecisionMode,
                        allow_fp8: bool) -> int:
    """Bit mask of the precision codes the analyzer can choose."""
    if not enable_adaptive_precision:
        return 1 << default.code
    m = (1 << PrecisionMode.FP32.code) | (1 << PrecisionMode.BF16.code) | (1 << default.code)
    m |= 1 << (PrecisionMode.FP8.code if allow_fp8 else PrecisionMode.FP16.code)
    return m


def analyze(q: torch.Tensor, k: torch.Tensor, *, scale: float, eps: float = 1e-6,
            rank_threshold: float = 0.95, enable_adaptive_rank: bool = True,
            enable_adaptive_precision: bool = True,
            default_precision: PrecisionMode = PrecisionMode.FP16, allow_fp8: bool = False,
            granularity: str = "head", sample_stride: int = 1) -> DecisionTable:
    """Run the analyzer (adaattn.py:228-289) on q, k [B, H, N, D].

    granularity "head": one decision per (b, h) slice (the reference's
    analyzer applied to that slice); "global": the reference's single
    decision for the whole call, written to every slice.
    """
    _require_cuda(q, k)
    lib = _lib.load()
    b, h = q.shape[0], q.shape[1]
    dev = q.device
    decisions = torch.empty(b, h, 2, dtype=torch.int32, device=dev)
    stats = torch.empty(b, h, 4, dtype=torch.float32, device=dev)
    summary = torch.empty(_lib.SUMMARY_LEN, dtype=torch.float32, device=dev)
    ws_bytes = lib.ada_analyze_workspace_bytes(b, h)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
    p = _lib.AdaAnalyzeParams()
    p.rank_threshold = float(rank_threshold)
    p.scale = float(scale)
    p.eps = float(eps)
    p.enable_adaptive_rank = int(bool(enable_adaptive_rank))
    p.enable_adaptive_precision = int(bool(enable_adaptive_precision))
    p.default_precision = PrecisionMode.coerce(default_precision).code
    p.allow_fp8 = int(bool(allow_fp8))
    if granularity not in ("head", "global"):
        raise ValueError(f"granularity must be 'head' or 'global', got {granularity!r}")
    p.granularity = 0 if granularity == "head" else 1
    p.sample_stride = int(sample_stride)
    tq, tk = _lib.tensor(q), _lib.tensor(k)
    with torch.cuda.device(dev):
        rc = lib.ada_analyze(tq, tk, p, decisions.data_ptr(), stats.data_ptr(),
                             summary.data_ptr(), ws.data_ptr(), ws.numel(),
                             _lib.stream_ptr(dev))
    _lib.check(rc, "ada_analyze")
    head_sum = ws[:b * h * 4].view(torch.float32).view(b, h) if b * h else None
    return DecisionTable(decisions, stats, summary, granularity, head_sum)


def expand_mask(mask: Optional[torch.Tensor], b: int, h: int, nq: int, nk: int
                ) -> Optional[torch.Tensor]:
    """Broadcast a reference-style mask to a [B, H, Nq, Nk] view.

    2-D [B, Nk] and 3-D [B, Nq, Nk] masks follow adaattn.py:320-324; a 4-D
    mask is used as given (size-1 dimensions broadcast).
    """
    if mask is None:
        return None
    if mask.dim() == 2:
        m = mask[:, None, None, :]
    elif mask.dim() == 3:
        m = mask[:, None, :, :]
    elif mask.dim() == 4:
        m = mask
    else:
        raise ShapeError(f"attention_mask must be 2D, 3D, or 4D, got {mask.dim()}D")
    if m.dtype == torch.bool:
        m = m.view(torch.uint8)  # same bytes; the kernels read nonzero as keep
    elif m.dtype not in (torch.float32, torch.float16, torch.bfloat16):
        m = m.float()
    return m.expand(b, h, nq, nk)


def attention_forward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, scale: float,
                      causal: bool = False, table: Optional[DecisionTable] = None,
                      static_precision: PrecisionMode = PrecisionMode.FP16,
                      static_low_rank: bool = False, w_down: Optional[torch.Tensor] = None,
                      attention_mask: Optional[torch.Tensor] = None,
                      possible_mask: Optional[int] = None, low_rank_possible: bool = False,
                      fp8_mode: str = "e4m3", out: Optional[torch.Tensor] = None
                      ) -> torch.Tensor:
    """Adaptive attention core on [B, H, N, D] (adaattn.py:462-504).

    With ``table`` every slice follows its own decision; without it every
    slice uses ``static_precision`` / ``static_low_rank``. ``out`` may be any
    [B, H, Nq, D] view with unit innermost stride (e.g. a transposed
    [B, Nq, H, D] buffer, so merging heads afterwards costs nothing).
    """
    _require_cuda(q, k, v)
    lib = _lib.load()
    b, h, nq, d = q.shape
    nk = k.shape[2]
    if out is None:
        out = torch.empty(b, nq, h, d, dtype=q.dtype, device=q.device).transpose(1, 2)
    if nq == 0 or b * h == 0:
        return out
    if nk == 0:
        raise ShapeError("key sequence is empty")
    mask4 = expand_mask(attention_mask, b, h, nq, nk)
    p = _lib.AdaFwdParams()
    p.scale = float(scale)
    p.causal = int(bool(causal))
    p.fp8_mode = 0 if fp8_mode == "e4m3" else 1
    p.static_precision = PrecisionMode.coerce(static_precision).code
    p.static_low_rank = int(bool(static_low_rank))
    dec_ptr = table.decisions.data_ptr() if table is not None else None
    if table is not None and possible_mask is None:
        possible_mask = 0x1F
    pm = int(possible_mask or 0)
    lowp = int(bool(low_rank_possible))
    tq, tk, tv, to = (_lib.tensor(t) for t in (q, k, v, out))
    w_keep = w_down.detach().contiguous() if w_down is not None else None
    tw = _lib.tensor(w_keep) if w_keep is not None else None
    tm = _lib.tensor(mask4) if mask4 is not None else None
    ws_bytes = lib.ada_attn_fwd_workspace_bytes(tq, tk, tv, tw, dec_ptr, p, pm, lowp)
    ws = torch.empty(max(int(ws_bytes), 1), dtype=torch.uint8, device=q.device)
    with torch.cuda.device(q.device):
        rc = lib.ada_attn_fwd(tq, tk, tv, tw, tm, dec_ptr, p, pm, lowp, to,
                              ws.data_ptr(), ws.numel(), _lib.stream_ptr(q.device))
    _lib.check(rc, "ada_attn_fwd")
    return out


def attention_backward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out: torch.Tensor,
                       dout: torch.Tensor, *, scale: float, causal: bool = False,
                       table: Optional[DecisionTable] = None, low_rank: bool = False,
                       attention_mask: Optional[torch.Tensor] = None):
    """Gradients (dq, dk, dv) of out = softmax(q kᵀ·scale + mask) v on
    [B, H, N, D] views, fp32 arithmetic at the operands' values
    (``ada_attn_bwd``); returned as contiguous fp32 tensors.

    With ``table`` only the heads whose low-rank flag equals ``low_rank`` are
    computed (the others' gradients stay zero): dense heads pass q, k; low-rank
    heads pass q_low, k_low and chain ``rank_proj_down`` themselves.
    """
    _require_cuda(q, k, v, out, dout)
    lib = _lib.load()
    b, h, nq, dqk = q.shape
    nk, dv_ = k.shape[2], v.shape[3]
    dev = q.device
    dq = torch.zeros(b, h, nq, dqk, dtype=torch.float32, device=dev)
    dk = torch.zeros(b, h, nk, dqk, dtype=torch.float32, device=dev)
    dv = torch.zeros(b, h, nk, dv_, dtype=torch.float32, device=dev)
    if b * h == 0 or nq == 0 or nk == 0:
        return dq, dk, dv
    mask4 = expand_mask(attention_mask, b, h, nq, nk)
    p = _lib.AdaFwdParams()
    p.scale = float(scale)
    p.causal = int(bool(causal))
    ws = torch.empty(max(int(lib.ada_attn_bwd_workspace_bytes(b, h, nq)), 1), dtype=torch.uint8, device=dev)
    tm = _lib.tensor(mask4) if mask4 is not None else None
    dec = table.decisions.data_ptr() if table is not None else None
    with torch.cuda.device(dev):
        rc = lib.ada_attn_bwd(_lib.tensor(q), _lib.tensor(k), _lib.tensor(v), _lib.tensor(out),
                              _lib.tensor(dout), tm, dec, int(bool(low_rank)), p, _lib.tensor(dq),
                              _lib.tensor(dk), _lib.tensor(dv), ws.data_ptr(), ws.numel(),
                              _lib.stream_ptr(dev))
    _lib.check(rc, "ada_attn_bwd")
    return dq, dk, dv


_ACTIVATIONS = {None: 0, "none": 0, "gelu": 1}


def _linear_launch(x2: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor],
                   r2: Optional[torch.Tensor], act: int) -> torch.Tensor:
    """One ada_linear call on 2-D views; y rows padded to 8 elements (16 bytes)
    and returned as a view of the first N columns."""
    lib = _lib.load()
    m, n = x2.shape[0], weight.shape[0]
    n_pad = (n + 7) // 8 * 8
    y = torch.empty(m, n_pad, dtype=x2.dtype, device=x2.device)[:, :n]
    tb = _lib.tensor(bias) if bias is not None else None
    tr = _lib.tensor(r2) if r2 is not None else None
    dev = x2.device
    args = (_lib.tensor(x2), _lib.tensor(weight), tb, tr, act, _lib.tensor(y))
    if dev.index == torch.cuda.current_device():
        rc = lib.ada_linear(*args, torch.cuda.current_stream(dev).cuda_stream)
    else:
        with torch.cuda.device(dev):
            rc = lib.ada_linear(*args, torch.cuda.current_stream(dev).cuda_stream)
    _lib.check(rc, "ada_linear")
    return y


def _unflat(y: torch.Tensor, lead) -> torch.Tensor:
    if len(lead) == 1:
        return y
    return y.unflatten(0, lead) if len(lead) else y[0]


def _rows(t: torch.Tensor) -> torch.Tensor:
    """[..., K] as a 2-D [M, K] view with unit column stride and 16-byte
    aligned rows (a copy only when the layout cannot be read in place)."""
    t2 = t if t.dim() == 2 else t.reshape(-1, t.shape[-1])
    if t2.shape[0] > 1 and t2.shape[1] > 1 and (
            t2.stride(1) != 1 or (t2.stride(0) * t2.element_size()) % 16 or t2.data_ptr() % 16):
        t2 = t2.contiguous()
    elif t2.data_ptr() % 16:
        t2 = t2.clone()
    return t2


class _LinearGrad(torch.autograd.Function):
    """Gradients of y = act(x Wᵀ + b) + r. The forward runs on ada_linear;
    the backward is the Linear's own pair of GEMMs (and GELU's derivative at
    the recomputed pre-activation), in the inputs' dtype like ATen's."""

    @staticmethod
    def forward(ctx, x, weight, bias, residual, act):
        ctx.act = act
        ctx.has_bias = bias is not None
        ctx.has_r = residual is not None
        ctx.save_for_backward(x, weight, bias)
        x2 = _rows(x)
        r2 = _rows(residual) if residual is not None else None
        return _unflat(_linear_launch(x2, weight, bias, r2, act), x.shape[:-1])

    @staticmethod
    def backward(ctx, dy):
        x, weight, bias = ctx.saved_tensors
        dh = dy
        if ctx.act == 1:
            h = _unflat(_linear_launch(_rows(x), weight, bias, None, 0), x.shape[:-1])
            hf = h.float()
            cdf = 0.5 * (1.0 + torch.erf(hf * 0.7071067811865476))
            pdf = torch.exp(-0.5 * hf * hf) * 0.3989422804014327
            dh = (dy.float() * (cdf + hf * pdf)).to(dy.dtype)
        dx = dh.matmul(weight) if ctx.needs_input_grad[0] else None
        dw = dh.reshape(-1, dh.shape[-1]).t().matmul(x.reshape(-1, x.shape[-1])) \
            if ctx.needs_input_grad[1] else None
        db = dh.reshape(-1, dh.shape[-1]).sum(0) if ctx.has_bias and ctx.needs_input_grad[2] else None
        dr = dy if ctx.has_r and ctx.needs_input_grad[3] else None
        return dx, dw, db, dr, None


def linear(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor] = None, *,
           residual: Optional[torch.Tensor] = None, activation: Optional[str] = None) -> torch.Tensor:
    """``act(x @ weight.T + bias) + residual`` on the tensor cores (``ada_linear``):
    the module's q/k/v projections and out_proj (adaattn.py:411-418, :457)
    and the host block's feed-forward, as one launch each with the bias,
    the GELU (erf form) and the residual sum fused into the epilogue.

    x [..., K] and weight [N, K] (nn.Linear's layout) are bf16 or fp16 on an
    sm_100 device; K must be a multiple of 8. The result [..., N] rounds like
    the PyTorch ops it replaces (Linear, then GELU, then the sum, each in the
    inputs' dtype); its rows are padded to 16 bytes in memory. Autograd is
    supported (the backward uses the Linear's own GEMMs).
    """
    _require_cuda(x, weight, bias, residual)
    act = _ACTIVATIONS.get(activation)
    if act is None:
        raise ValueError(f"activation must be None or 'gelu', got {activation!r}")
    if x.dtype not in (torch.bfloat16, torch.float16):
        raise TypeError(f"linear runs in bf16 or fp16, got {x.dtype}")
    if weight.dtype != x.dtype or (bias is not None and bias.dtype != x.dtype) or (
            residual is not None and residual.dtype != x.dtype):
        raise TypeError("x, weight, bias and residual must share one dtype")
    if x.shape[-1] != weight.shape[1]:
        raise ShapeError(f"x has {x.shape[-1]} features, weight expects {weight.shape[1]}")
    if residual is not None and tuple(residual.shape) != tuple(x.shape[:-1]) + (weight.shape[0],):
        raise ShapeError(f"residual must be {tuple(x.shape[:-1]) + (weight.shape[0],)}, "
                         f"got {tuple(residual.shape)}")
    w = weight if (weight.stride(-1) == 1 and (weight.stride(0) * 2) % 16 == 0
                   and weight.data_ptr() % 16 == 0) else weight.contiguous()
    if torch.is_grad_enabled() and any(t is not None and t.requires_grad
                                       for t in (x, weight, bias, residual)):
        return _LinearGrad.apply(x, w, bias, residual, act)
    y = _linear_launch(_rows(x), w, bias, _rows(residual) if residual is not None else None, act)
    return _unflat(y, x.shape[:-1])


def layer_norm(x: torch.Tensor, weight: Optional[torch.Tensor], bias: Optional[torch.Tensor],
               eps: float = 1e-5) -> torch.Tensor:
    """``nn.LayerNorm`` over the last dimension (``ada_layer_norm``), the host
    block's norms (examples/transformer_integration.py:44-45, 81): fp32 mean
    and variance, the result rounded once to x's dtype (bf16 or fp16). No
    autograd: callers that need gradients use ``nn.LayerNorm`` itself."""
    _require_cuda(x, weight, bias)
    if x.dtype not in (torch.bfloat16, torch.float16):
        raise TypeError(f"layer_norm runs in bf16 or fp16, got {x.dtype}")
    e = x.shape[-1]
    for t in (weight, bias):
        if t is not None and (t.dtype != x.dtype or tuple(t.shape) != (e,)):
            raise ShapeError(f"weight and bias must be [{e}] in {x.dtype}")
    x2 = _rows(x)
    y = torch.empty(x2.shape, dtype=x.dtype, device=x.device)
    w = weight.contiguous() if weight is not None else None
    b = bias.contiguous() if bias is not None else None
    lib = _lib.load()
    with torch.cuda.device(x.device):
        rc = lib.ada_layer_norm(_lib.tensor(x2), _lib.tensor(w) if w is not None else None,
                                _lib.tensor(b) if b is not None else None, float(eps), _lib.tensor(y),
                                _lib.stream_ptr(x.device))
    _lib.check(rc, "ada_layer_norm")
    return y.view(x.shape)


def record_statistics(summary: torch.Tensor, call_count: torch.Tensor, low_rank_calls: torch.Tensor,
                      precision_distribution: torch.Tensor) -> None:
    """Add one call's decision summary to the module's running statistics in
    place, on the device and without a host sync (``ada_record_statistics``;
    adaattn.py:486-498): call_count += 1, low_rank_calls += n_lowrank / total,
    precision_distribution += counts / total, each ratio in its buffer's dtype."""
    _require_cuda(summary, call_count, low_rank_calls, precision_distribution)
    if summary.dtype != torch.float32 or not summary.is_contiguous() or summary.numel() < _lib.SUMMARY_LEN:
        raise ShapeError("summary must be a contiguous float32 decision summary")
    lib = _lib.load()
    with torch.cuda.device(summary.device):
        rc = lib.ada_record_statistics(summary.data_ptr(), _lib.tensor(call_count), _lib.tensor(low_rank_calls),
                                       _lib.tensor(precision_distribution), _lib.stream_ptr(summary.device))
    _lib.check(rc, "ada_record_statistics")


def _host_params(scale, causal, static_precision, static_low_rank, fp8_mode):
    p = _lib.AdaFwdParams()
    p.scale = float(scale)
    p.causal = int(bool(causal))
    p.fp8_mode = 0 if fp8_mode == "e4m3" else 1
    p.static_precision = PrecisionMode.coerce(static_precision).code
    p.static_low_rank = int(bool(static_low_rank))
    return p


def host_buffer_bytes(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, scale: float,
                      static_precision: PrecisionMode = PrecisionMode.FP16,
                      static_low_rank: bool = False, w_down: Optional[torch.Tensor] = None,
                      chunk_slices: int = 0) -> int:
    """Device staging bytes `attention_forward_host` needs for these host operands."""
    lib = _lib.load()
    p = _host_params(scale, False, static_precision, static_low_rank, "e4m3")
    tw = _lib.tensor(w_down.detach().contiguous()) if w_down is not None else None
    need = int(lib.ada_attn_fwd_host_buffer_bytes(_lib.tensor(q), _lib.tensor(k), _lib.tensor(v), tw, p,
                                                  int(chunk_slices)))
    if need == 0:
        raise ShapeError(f"ada_attn_fwd_host_buffer_bytes: {_lib.last_error()}")
    return need


def attention_forward_host(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, scale: float,
                           causal: bool = False,
                           static_precision: PrecisionMode = PrecisionMode.FP16,
                           static_low_rank: bool = False, w_down: Optional[torch.Tensor] = None,
                           fp8_mode: str = "e4m3", out: Optional[torch.Tensor] = None,
                           device: Optional[torch.device] = None, chunk_slices: int = 0,
                           buffer: Optional[torch.Tensor] = None) -> torch.Tensor:
    """`attention_forward` for host-resident [B, H, N, D] operands (contiguous;
    pinned memory lets the copies overlap): chunks of (b, h) slices are copied in,
    computed and copied out on overlapping streams (``ada_attn_fwd_host``).
    Every slice takes ``static_precision`` / ``static_low_rank``. Returns the
    host ``out`` (allocated pinned when not given); it is complete once the
    current stream of ``device`` is. ``buffer``: an optional device uint8
    tensor reused as the staging buffer."""
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    if dev.type != "cuda":
        raise TypeError("device must be a CUDA device")
    for t in (q, k, v):
        if t.is_cuda:
            raise TypeError("attention_forward_host takes host tensors; use attention_forward")
        if not t.is_contiguous():
            raise ShapeError("host operands must be contiguous [B, H, N, D]")
    lib = _lib.load()
    if out is None:
        out = torch.empty(q.shape, dtype=q.dtype).pin_memory()
    p = _host_params(scale, causal, static_precision, static_low_rank, fp8_mode)
    w_keep = w_down.detach().to(dev).contiguous() if w_down is not None else None
    tw = _lib.tensor(w_keep) if w_keep is not None else None
    tq, tk, tv, to = (_lib.tensor(t) for t in (q, k, v, out))
    need = int(lib.ada_attn_fwd_host_buffer_bytes(tq, tk, tv, tw, p, int(chunk_slices)))
    if need == 0:
        raise ShapeError(f"ada_attn_fwd_host_buffer_bytes: {_lib.last_error()}")
    if buffer is None or buffer.numel() < need or buffer.device != dev:
        buffer = torch.empty(max(need, 1), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        rc = lib.ada_attn_fwd_host(tq, tk, tv, tw, p, to, int(chunk_slices), buffer.data_ptr(),
                                   buffer.numel(), _lib.stream_ptr(dev))
    _lib.check(rc, "ada_attn_fwd_host")
    return out


def default_scale(head_dim: int) -> float:
    return 1.0 / math.sqrt(head_dim)
