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
