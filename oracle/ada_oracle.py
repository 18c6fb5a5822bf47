"""CPU restatement of the AdaAttn attention-forward hot path (the oracle).

TEST INFRASTRUCTURE ONLY. Nothing in the shipped package imports this module;
the CUDA path is checked against it on the same seeded inputs.

Each function restates one piece of the reference's algorithm in plain PyTorch
CPU code, keeping the reference's dtype semantics (matmul / softmax / entropy in
the tensor's own dtype, FP16-for-FP8 and so on) because decision parity depends
on them. Citations are ``path:line`` inside the hkevin01/AdaAttn project.

Pinning: ``tests/golden/make_golden.py`` runs the reference itself on seeded
inputs and stores its decisions and outputs under ``tests/golden/``;
``tests/test_oracle_golden.py`` checks this module against those fixtures and
against the reference's own known-answer tests (entropy, randomized SVD).

Precision codes follow the reference's ``_precision_distribution`` order
(src/adaattn/attention/adaattn.py:480-485): FP32=0, FP16=1, BF16=2, FP8=3,
plus AUTO=4 (computes in fp16, counted in slot 0 by the reference's
``.get(precision, 0)``).
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional, Tuple

import torch
import torch.nn.functional as F

__all__ = [
    "FP32", "FP16", "BF16", "FP8", "AUTO", "PREC_NAMES", "compute_dtype",
    "OracleConfig", "sample_stats", "head_entropy_sums", "decide", "analyze", "analyze_per_head",
    "apply_masks", "dense_attention", "low_rank_attention", "adaptive_forward",
    "module_forward",
    "fp8_quantize_tiles", "fp8_dense_attention", "randomized_svd",
    "rsvd_sketch", "E4M3_MAX", "FP8_TILE",
    "kernel_flash_attention_forward", "kernel_adaptive_attention_forward",
    "compute_entropy", "estimate_effective_rank", "determine_target_ranks",
    "attention_grads", "attention_grads_from_out", "linear_layer",
]

FP32, FP16, BF16, FP8, AUTO = 0, 1, 2, 3, 4
PREC_NAMES = ("FP32", "FP16", "BF16", "FP8", "AUTO")

# src/adaattn/attention/base.py:100-109 -- PrecisionMode.to_dtype; FP8 and AUTO
# both compute in float16.
_COMPUTE_DTYPE = {
    FP32: torch.float32,
    FP16: torch.float16,
    BF16: torch.bfloat16,
    FP8: torch.float16,
    AUTO: torch.float16,
}

E4M3_MAX = 448.0
FP8_TILE = 128


def compute_dtype(prec: int) -> torch.dtype:
    return _COMPUTE_DTYPE[prec]


@dataclass
class OracleConfig:
    """Knobs of AdaAttention that steer the hot path.

    Defaults mirror src/adaattn/attention/adaattn.py:57-79 and
    src/adaattn/attention/base.py:203 (eps).
    """

    enable_adaptive_rank: bool = True
    enable_adaptive_precision: bool = True
    rank_threshold: float = 0.95
    default_precision: int = FP16
    allow_fp8: bool = False
    causal: bool = False
    eps: float = 1e-6


def sample_stats(q: torch.Tensor, k: torch.Tensor, scale: float, eps: float
                 ) -> Tuple[float, float, float, int]:
    """Statistics of the analyzer sample, computed in the inputs' dtype.

    Follows src/adaattn/attention/adaattn.py:248-275: the first
    S = min(64, Nq, Nk) queries and keys, scores = q_s k_s^T * scale,
    softmax, per-row entropy -sum p*log(p+eps), normalised by log(S) and
    averaged over every (batch, head, row) of the tensors passed in.

    Returns (normalized_entropy, max|score|, max prob, S).
    """
    n_q, n_k = q.shape[2], k.shape[2]
    s = min(64, n_q, n_k)
    scores = torch.matmul(q[:, :, :s], k[:, :, :s].transpose(-2, -1)) * scale
    probs = F.softmax(scores, dim=-1)
    row_entropy = -(probs * torch.log(probs + eps)).sum(dim=-1)
    ne = (row_entropy / math.log(s)).mean().item()
    return ne, scores.abs().max().item(), probs.max().item(), s


def head_entropy_sums(q: torch.Tensor, k: torch.Tensor, scale: float, eps: float
                      ) -> Tuple[torch.Tensor, torch.Tensor, int]:
    """Per-(b, h) pieces of the analyzer's call-level statistics.

    Same arithmetic as sample_stats (adaattn.py:248-263) up to the mean: the
    per-row normalised entropies (in the inputs' dtype), summed per slice in
    fp32, and per-slice max |score| and max prob. Returns (sums [B, H],
    stats [B, H, 4] with max|score| at [..., 1] and max prob at [..., 2], S).
    """
    n_q, n_k = q.shape[2], k.shape[2]
    s = min(64, n_q, n_k)
    scores = torch.matmul(q[:, :, :s], k[:, :, :s].transpose(-2, -1)) * scale
    probs = F.softmax(scores, dim=-1)
    row_entropy = -(probs * torch.log(probs + eps)).sum(dim=-1)
    ne_rows = row_entropy / math.log(s)
    sums = ne_rows.float().sum(dim=-1)
    stats = torch.zeros(*q.shape[:2], 4)
    stats[..., 1] = scores.abs().amax(dim=(-1, -2)).float()
    stats[..., 2] = probs.amax(dim=(-1, -2)).float()
    return sums, stats, s


def decide(ne: float, max_score: float, max_prob: float, cfg: OracleConfig
           ) -> Tuple[bool, int]:
    """Rank and precision ladder of src/adaattn/attention/adaattn.py:268-287.

    NaN statistics compare False everywhere, exactly as Python floats do.
    """
    low_rank = bool(cfg.enable_adaptive_rank and ne < cfg.rank_threshold)
    if max_score > 50.0 or max_prob > 0.95:
        prec = FP32
    elif ne > 0.8:
        prec = FP8 if cfg.allow_fp8 else FP16
    elif ne < 0.3:
        prec = BF16
    else:
        prec = cfg.default_precision
    if not cfg.enable_adaptive_precision:
        prec = cfg.default_precision
    return low_rank, prec


def analyze(q: torch.Tensor, k: torch.Tensor, cfg: OracleConfig, scale: float
            ) -> dict:
    """One decision for the whole call (the reference's own granularity).

    src/adaattn/attention/adaattn.py:228-289; effective rank is
    ne * min(Nq, Nk) (:266).
    """
    ne, ms, mp, _ = sample_stats(q, k, scale, cfg.eps)
    low_rank, prec = decide(ne, ms, mp, cfg)
    return {
        "low_rank": low_rank, "precision": prec, "ne": ne,
        "max_score": ms, "max_prob": mp,
        "effective_rank": ne * min(q.shape[2], k.shape[2]),
    }


def analyze_per_head(q: torch.Tensor, k: torch.Tensor, cfg: OracleConfig,
                     scale: float) -> dict:
    """The reference analyzer applied to every (b, h) slice on its own.

    Returns tensors [B, H]: low_rank (bool), precision (int), ne, max_score,
    max_prob (float64, the values the reference's ``.item()`` would give).
    """
    b_sz, h_sz = q.shape[0], q.shape[1]
    low = torch.zeros(b_sz, h_sz, dtype=torch.bool)
    prec = torch.zeros(b_sz, h_sz, dtype=torch.int32)
    ne = torch.zeros(b_sz, h_sz, dtype=torch.float64)
    ms = torch.zeros_like(ne)
    mp = torch.zeros_like(ne)
    for b in range(b_sz):
        for h in range(h_sz):
            d = analyze(q[b:b + 1, h:h + 1], k[b:b + 1, h:h + 1], cfg, scale)
            low[b, h] = d["low_rank"]
            prec[b, h] = d["precision"]
            ne[b, h], ms[b, h], mp[b, h] = d["ne"], d["max_score"], d["max_prob"]
    return {"low_rank": low, "precision": prec, "ne": ne, "max_score": ms,
            "max_prob": mp}


def apply_masks(scores: torch.Tensor, causal: bool,
                attention_mask: Optional[torch.Tensor], dt: torch.dtype
                ) -> torch.Tensor:
    """Causal and user masks of src/adaattn/attention/adaattn.py:312-329.

    Causal is top-left aligned: key j is hidden from query i when j > i.
    A 2-D mask is [B, Nk], 3-D is [B, Nq, Nk], 4-D is used as given. Boolean
    masks keep True positions; float masks are added in the compute dtype.
    """
    if causal:
        n_q, n_k = scores.shape[-2], scores.shape[-1]
        hide = torch.ones(n_q, n_k, dtype=torch.bool).triu(1)
        scores = scores.masked_fill(hide, float("-inf"))
    if attention_mask is not None:
        m = attention_mask
        if m.ndim == 2:
            m = m[:, None, None, :]
        elif m.ndim == 3:
            m = m[:, None]
        if m.dtype == torch.bool:
            scores = scores.masked_fill(~m, float("-inf"))
        else:
            scores = scores + m.to(dt)
    return scores


def _softmax_in_precision(scores: torch.Tensor, prec: int, dt: torch.dtype
                          ) -> torch.Tensor:
    # adaattn.py:331-334 / :386-389: FP16 and FP8 take the softmax in fp32 and
    # cast back; FP32, BF16 and AUTO take it in the compute dtype itself.
    if prec in (FP16, FP8):
        return F.softmax(scores.float(), dim=-1).to(dt)
    return F.softmax(scores, dim=-1)


def dense_attention(q, k, v, prec: int, scale: float, causal: bool,
                    attention_mask=None, cast_back: bool = True,
                    compute: Optional[torch.dtype] = None) -> torch.Tensor:
    """Dense branch, src/adaattn/attention/adaattn.py:291-339 (eval mode).

    Scores are clamped to the fp16 range for FP16 and FP8 (:309-310).
    cast_back=False returns the result in the compute dtype, before the
    reference's final cast to the inputs' dtype (:339). ``compute`` replaces
    the precision's compute dtype (float64 gives the exact value the FP32
    branch approximates).
    """
    dt = compute or compute_dtype(prec)
    qc, kc, vc = q.to(dt), k.to(dt), v.to(dt)
    scores = torch.matmul(qc, kc.transpose(-2, -1)) * scale
    if prec in (FP16, FP8):
        scores = torch.clamp(scores, min=-65504, max=65504)
    scores = apply_masks(scores, causal, attention_mask, dt)
    probs = _softmax_in_precision(scores, prec, dt)
    out = torch.matmul(probs, vc)
    return out.to(q.dtype) if cast_back else out


def low_rank_attention(q, k, v, w_down: torch.Tensor, prec: int, scale: float,
                       causal: bool, attention_mask=None, cast_back: bool = True,
                       compute: Optional[torch.dtype] = None) -> torch.Tensor:
    """Low-rank branch, src/adaattn/attention/adaattn.py:341-394 (eval mode).

    q and k go through the learned head-dim projection ``rank_proj_down``
    (weight [r, D], no bias) in the inputs' dtype, then scores use the
    module's 1/sqrt(D) scale on the r-dimensional products; V stays full
    width. No clamp on this branch. cast_back=False returns the result in
    the compute dtype, before the final cast to the inputs' dtype (:394);
    ``compute`` replaces the compute dtype as in dense_attention (the
    projection stays in the inputs' dtype).
    """
    dt = compute or compute_dtype(prec)
    w = w_down.to(q.dtype)
    q_low = F.linear(q, w).to(dt)
    k_low = F.linear(k, w).to(dt)
    vc = v.to(dt)
    scores = torch.matmul(q_low, k_low.transpose(-2, -1)) * scale
    scores = apply_masks(scores, causal, attention_mask, dt)
    probs = _softmax_in_precision(scores, prec, dt)
    out = torch.matmul(probs, vc)
    return out.to(q.dtype) if cast_back else out


def _slice_mask(mask, b: int, h: int):
    if mask is None:
        return None
    if mask.ndim in (2, 3):
        return mask[b:b + 1]
    return mask[b:b + 1, (h if mask.shape[1] > 1 else 0):][:, :1]


def adaptive_forward(q, k, v, cfg: OracleConfig, scale: float,
                     w_down: Optional[torch.Tensor] = None,
                     granularity: str = "head", attention_mask=None,
                     fp8_mode: str = "reference") -> Tuple[torch.Tensor, dict]:
    """The adaptive dispatcher, src/adaattn/attention/adaattn.py:462-504.

    granularity "global" is the reference's own behaviour: one decision per
    call. "head" applies the same analyzer and branch to each (b, h) slice.
    fp8_mode "reference" computes FP8 heads in fp16 like base.py:106;
    "e4m3" uses the tile-scaled E4M3 restatement below.
    Returns (output [B,H,Nq,D], decisions).
    """
    def run(qs, ks, vs, low, prec, mask):
        if low and w_down is not None:
            if prec == FP8 and fp8_mode == "e4m3":
                return fp8_dense_attention(qs, ks, vs, scale, cfg.causal, mask,
                                           w_down=w_down)
            return low_rank_attention(qs, ks, vs, w_down, prec, scale,
                                      cfg.causal, mask)
        if prec == FP8 and fp8_mode == "e4m3":
            return fp8_dense_attention(qs, ks, vs, scale, cfg.causal, mask)
        return dense_attention(qs, ks, vs, prec, scale, cfg.causal, mask)

    if granularity == "global":
        d = analyze(q, k, cfg, scale)
        out = run(q, k, v, d["low_rank"], d["precision"], attention_mask)
        return out, d
    d = analyze_per_head(q, k, cfg, scale)
    out = torch.empty(q.shape[0], q.shape[1], q.shape[2], v.shape[3],
                      dtype=q.dtype)
    for b in range(q.shape[0]):
        for h in range(q.shape[1]):
            out[b:b + 1, h:h + 1] = run(
                q[b:b + 1, h:h + 1], k[b:b + 1, h:h + 1], v[b:b + 1, h:h + 1],
                bool(d["low_rank"][b, h]), int(d["precision"][b, h]),
                _slice_mask(attention_mask, b, h))
    return out, d


def module_forward(query, key, value, state_dict: dict, num_heads: int,
                   cfg: OracleConfig, granularity: str = "global",
                   attention_mask=None, fp8_mode: str = "reference"
                   ) -> Tuple[torch.Tensor, dict]:
    """AdaAttention.forward in eval mode, src/adaattn/attention/adaattn.py:396-460.

    Projections E->E, split into heads [B, H, N, D], the adaptive core, merge
    heads, output projection. The flash_attn branch (:421-445) is never taken
    on CPU tensors, so it is not restated.
    """
    sd = state_dict
    b_sz, n_q, e = query.shape
    n_k = key.shape[1]
    d = e // num_heads

    def proj(x, name):
        return F.linear(x, sd[f"{name}.weight"], sd.get(f"{name}.bias"))

    q = proj(query, "q_proj").view(b_sz, n_q, num_heads, d).transpose(1, 2)
    k = proj(key, "k_proj").view(b_sz, n_k, num_heads, d).transpose(1, 2)
    v = proj(value, "v_proj").view(b_sz, n_k, num_heads, d).transpose(1, 2)
    w_down = sd.get("rank_proj_down.weight")
    out, dec = adaptive_forward(q, k, v, cfg, 1.0 / math.sqrt(d), w_down,
                                granularity, attention_mask, fp8_mode)
    out = out.transpose(1, 2).contiguous().view(b_sz, n_q, e)
    return proj(out, "out_proj"), dec


# --------------------------------------------------------------------------
# FP8-E4M3 restatement (the build's real FP8 heads).
#
# The reference's "FP8" computes in fp16 (base.py:106), so a real E4M3 kernel
# needs its own oracle: the same per-tile quantisation the kernel performs,
# followed by fp32 arithmetic. Scheme:
#   Q: one scale per (b, h, 128-row query tile), K: one per (b, h, 128-row key
#   tile), V: one per (b, h); scale = amax / 448 (1 when amax is 0),
#   x8 = e4m3(x / scale) (round to nearest even, |x/scale| <= 448).
#   S_j = (Q8 K8_j^T) * sq * sk_j * softmax_scale; running row max m;
#   P8 = e4m3(exp(S_j - m) * 448); O += P8 V8; l += sum(exp(S_j - m));
#   out = O * sv / (448 * l).
# --------------------------------------------------------------------------

def fp8_quantize_tiles(x: torch.Tensor, tile: Optional[int] = FP8_TILE
                       ) -> Tuple[torch.Tensor, torch.Tensor]:
    """Per-(b, h, row-tile) E4M3 quantisation of x [B, H, N, D] (fp32 math).

    tile=None gives one scale per (b, h). Returns (dequantised fp32 values,
    scales [B, H, n_tiles]).
    """
    xf = x.float()
    b_sz, h_sz, n, d = xf.shape
    t = n if tile is None else tile
    n_tiles = max(1, -(-n // t))
    pad = n_tiles * t - n
    xp = F.pad(xf, (0, 0, 0, pad)) if pad else xf
    xt = xp.view(b_sz, h_sz, n_tiles, t, d)
    amax = xt.abs().amax(dim=(-1, -2))
    scale = torch.where(amax > 0, amax / E4M3_MAX, torch.ones_like(amax))
    q8 = (xt / scale[..., None, None]).to(torch.float8_e4m3fn)
    deq = q8.float() * scale[..., None, None]
    return deq.view(b_sz, h_sz, n_tiles * t, d)[:, :, :n], scale


def fp8_dense_attention(q, k, v, scale: float, causal: bool,
                        attention_mask=None, w_down=None,
                        block: int = FP8_TILE) -> torch.Tensor:
    """Tile-scaled E4M3 attention, computed block by block like the kernel.

    With w_down given, q and k are first projected (in the inputs' dtype,
    as adaattn.py:357-358) and the projected values are quantised.
    """
    if w_down is not None:
        w = w_down.to(q.dtype)
        q = F.linear(q, w)
        k = F.linear(k, w)
    qd, _ = fp8_quantize_tiles(q)
    kd, _ = fp8_quantize_tiles(k)
    vd, _ = fp8_quantize_tiles(v, tile=None)
    n_q, n_k = qd.shape[2], kd.shape[2]
    scores = torch.matmul(qd, kd.transpose(-2, -1)) * scale
    scores = apply_masks(scores, causal, attention_mask, torch.float32)
    out = torch.zeros(qd.shape[0], qd.shape[1], n_q, vd.shape[3])
    m = torch.full((qd.shape[0], qd.shape[1], n_q, 1), float("-inf"))
    l = torch.zeros_like(m)
    for j0 in range(0, n_k, block):
        s = scores[..., j0:j0 + block]
        m_new = torch.maximum(m, s.amax(dim=-1, keepdim=True))
        alpha = torch.where(m_new == float("-inf"), torch.ones_like(m),
                            torch.exp(m - m_new))
        p = torch.where(m_new == float("-inf"), torch.zeros_like(s),
                        torch.exp(s - m_new))
        p8 = (p * E4M3_MAX).to(torch.float8_e4m3fn).float()
        out = out * alpha + torch.matmul(p8, vd[:, :, j0:j0 + block])
        l = l * alpha + p.sum(dim=-1, keepdim=True)
        m = m_new
    return (out / (E4M3_MAX * l)).to(q.dtype)


# --------------------------------------------------------------------------
# Randomized SVD, src/adaattn/linalg/low_rank.py:56-109.
# --------------------------------------------------------------------------

def randomized_svd(a: torch.Tensor, rank: int, omega: torch.Tensor,
                   n_power: int = 2, qr: str = "householder"
                   ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Halko-style truncated SVD with the Gaussian sketch passed in.

    The reference draws omega [..., n, k] with k = min(rank + 10, min(m, n))
    from torch.randn (low_rank.py:80-83); passing it makes the algorithm
    deterministic. qr="householder" is the reference's torch.linalg.qr
    (:93); qr="cholesky" is CholeskyQR (Q = Y R^-1 with R = chol(Y^T Y)^T),
    the form the GPU path uses.
    """
    y = torch.matmul(a, omega)
    for _ in range(n_power):
        y = torch.matmul(a, torch.matmul(a.transpose(-2, -1), y))
    if qr == "householder":
        qm, _ = torch.linalg.qr(y)
    else:
        g = torch.matmul(y.transpose(-2, -1), y)
        r_up = torch.linalg.cholesky(g).transpose(-2, -1)
        qm = torch.linalg.solve_triangular(r_up, y, upper=True, left=False)
    bm = torch.matmul(qm.transpose(-2, -1), a)
    ub, s, vh = torch.linalg.svd(bm, full_matrices=False)
    u = torch.matmul(qm, ub)
    return u[..., :rank], s[..., :rank], vh[..., :rank, :]


def rsvd_sketch(shape_batch, n: int, rank: int, m: int, seed: int,
                oversample: int = 10, dtype=torch.float32) -> torch.Tensor:
    """Seeded Gaussian sketch of the reference's shape [..., n, k]."""
    k = min(rank + oversample, min(m, n))
    g = torch.Generator().manual_seed(seed)
    return torch.randn(*shape_batch, n, k, generator=g, dtype=dtype)


# --------------------------------------------------------------------------
# Kernel-level ops of the reference's native module _adaattn_cuda
# (src/adaattn/kernels/bindings.cpp:21-135) and the Python fallbacks that
# adaattn.kernels runs when that module is absent (kernels/__init__.py:81-213).
# Tensors are [B, N, H, D] here, as in those functions.
# --------------------------------------------------------------------------

def kernel_flash_attention_forward(q, k, v, softmax_scale: Optional[float] = None,
                                   causal: bool = False) -> torch.Tensor:
    """flash_attention_forward: bindings.cpp:21-68, kernels/__init__.py:81-120.

    Scores, softmax and P.V in the tensors' own dtype, causal mask
    triu(ones(N, N), 1) filled with -inf; returns [B, N, H, D].
    """
    n = q.shape[1]
    scale = softmax_scale if softmax_scale is not None else q.shape[-1] ** -0.5
    qt, kt, vt = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
    scores = torch.matmul(qt, kt.transpose(-2, -1)) * scale
    if causal:
        mask = torch.triu(torch.ones(n, n, dtype=torch.bool), diagonal=1)
        scores = scores.masked_fill(mask, float("-inf"))
    probs = torch.softmax(scores, dim=-1)
    return torch.matmul(probs, vt).transpose(1, 2)


_KERNEL_PRECISION = {"fp16": torch.float16, "bf16": torch.bfloat16}


def kernel_adaptive_attention_forward(q, k, v, precision: str = "fp16",
                                      softmax_scale: Optional[float] = None,
                                      causal: bool = False) -> torch.Tensor:
    """adaptive_attention_forward, dense branch (target_rank None):
    kernels/__init__.py:151-213.

    Cast to the requested precision ("fp16", "bf16", anything else fp32),
    softmax taken in fp32 and cast back, result cast to the inputs' dtype.
    (The native binding, bindings.cpp:73-96, ignores target_rank; the Python
    fallback's low-rank branch draws a fresh random projection per call and
    has no fixed answer to restate.)
    """
    orig = q.dtype
    dt = _KERNEL_PRECISION.get(precision, torch.float32)
    n = q.shape[1]
    scale = softmax_scale if softmax_scale is not None else q.shape[-1] ** -0.5
    qt, kt, vt = (t.to(dt).transpose(1, 2) for t in (q, k, v))
    scores = torch.matmul(qt, kt.transpose(-2, -1)) * scale
    if causal:
        mask = torch.triu(torch.ones(n, n, dtype=torch.bool), diagonal=1)
        scores = scores.masked_fill(mask, float("-inf"))
    probs = torch.softmax(scores.float(), dim=-1).to(dt)
    return torch.matmul(probs, vt).transpose(1, 2).to(orig)


def compute_entropy(attn_weights: torch.Tensor) -> torch.Tensor:
    """-(w * log(w + 1e-10)).sum(-1): bindings.cpp:101-109."""
    return -(attn_weights * torch.log(attn_weights + 1e-10)).sum(-1)


def estimate_effective_rank(attn_weights: torch.Tensor) -> torch.Tensor:
    """exp(mean(entropy, -1)): bindings.cpp:114-118."""
    return torch.exp(compute_entropy(attn_weights).mean(-1))


def determine_target_ranks(effective_rank: torch.Tensor, min_rank: int = 8,
                           max_rank: int = 128, threshold: float = 32.0) -> torch.Tensor:
    """where(rank < threshold, (rank * 1.5).clamp(min, max) as int64, max_rank):
    bindings.cpp:123-135 (defaults from :183-188)."""
    return torch.where(effective_rank < threshold,
                       (effective_rank * 1.5).clamp(min_rank, max_rank).to(torch.int64),
                       torch.full_like(effective_rank, max_rank).to(torch.int64))


# --------------------------------------------------------------------------
# Gradients (the reference differentiates through ATen autograd,
# tests/unit/test_adaattn_unified.py:146-159).
# --------------------------------------------------------------------------

def attention_grads_from_out(q, k, v, out, dout, scale: float, causal: bool,
                             attention_mask=None, w_down=None):
    """The attention backward in float64 by its standard formulas, with the
    row term Delta = sum(dO * out) taken from the given forward output (as
    a backward that does not store probabilities computes it):
    P = softmax(z), dV = Pᵀ dO, dS = P (dO Vᵀ - Delta), dQ = scale dS K,
    dK = scale dSᵀ Q; with w_down, Q, K are the projections (rounded in
    their dtype) and dq = dq_low W, dW = dq_lowᵀ q + dk_lowᵀ k.
    Returns (dq, dk, dv, dw or None) in float64."""
    if w_down is not None:
        qa = F.linear(q, w_down.to(q.dtype)).double()
        ka = F.linear(k, w_down.to(k.dtype)).double()
    else:
        qa, ka = q.double(), k.double()
    vd, od, gd = v.double(), out.double(), dout.double()
    z = apply_masks(torch.matmul(qa, ka.transpose(-2, -1)) * scale, causal, attention_mask, torch.float64)
    p = torch.softmax(z, dim=-1)
    dv = torch.matmul(p.transpose(-2, -1), gd)
    delta = (gd * od).sum(-1, keepdim=True)
    ds = p * (torch.matmul(gd, vd.transpose(-2, -1)) - delta)
    dq = torch.matmul(ds, ka) * scale
    dk = torch.matmul(ds.transpose(-2, -1), qa) * scale
    dw = None
    if w_down is not None:
        wd = w_down.double()
        dw = torch.einsum("bhnr,bhnd->rd", dq, q.double()) + torch.einsum("bhnr,bhnd->rd", dk, k.double())
        dq, dk = torch.matmul(dq, wd), torch.matmul(dk, wd)
    return dq, dk, dv, dw


def attention_grads(q, k, v, dout, scale: float, causal: bool, attention_mask=None,
                    w_down=None):
    """float64 autograd of out = softmax(q kᵀ·scale + mask) v (top-left causal,
    bool masks hide keys, float masks are added); with w_down, q and k are
    first projected in their own dtype (adaattn.py:357-358) and the
    projection's rounding is passed through as the identity.
    Returns (dq, dk, dv, dw or None) in float64."""
    qd = q.detach().double().requires_grad_(True)
    kd = k.detach().double().requires_grad_(True)
    vd = v.detach().double().requires_grad_(True)
    wd = None
    if w_down is not None:
        wd = w_down.detach().double().requires_grad_(True)
        ql = F.linear(q, w_down.to(q.dtype)).double()
        kl = F.linear(k, w_down.to(k.dtype)).double()
        # values of the rounded projection, gradients of the exact one
        qa = F.linear(qd, wd)
        ka = F.linear(kd, wd)
        qa = qa + (ql - qa).detach()
        ka = ka + (kl - ka).detach()
    else:
        qa, ka = qd, kd
    z = torch.matmul(qa, ka.transpose(-2, -1)) * scale
    z = apply_masks(z, causal, attention_mask, torch.float64)
    out = torch.matmul(torch.softmax(z, dim=-1), vd)
    out.backward(dout.double())
    return qd.grad, kd.grad, vd.grad, (wd.grad if wd is not None else None)


# --------------------------------------------------------------------------
# The dense layers on either side of the path: nn.Linear (the module's q/k/v
# projections, adaattn.py:411-418, and out_proj, :457) and the host block's
# feed-forward / residual sums (examples/transformer_integration.py:33-58).
# --------------------------------------------------------------------------

def linear_layer(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor] = None,
                 activation: Optional[str] = None, residual: Optional[torch.Tensor] = None
                 ) -> Tuple[torch.Tensor, torch.Tensor]:
    """y = act(x Wᵀ + b) + r with PyTorch's rounding points for 16-bit tensors:
    the Linear's result is rounded to x's dtype, then GELU's (erf form,
    nn.GELU()), then the residual sum's. The products are summed exactly
    (float64), so the only difference from a device result is the device's
    fp32 accumulation order.

    Returns (y in x's dtype, the float64 sum x Wᵀ + b before any rounding,
    for error bounds).
    """
    dt = x.dtype
    h64 = x.double() @ weight.double().t()
    if bias is not None:
        h64 = h64 + bias.double()
    y = h64.to(dt)
    if activation == "gelu":
        y = F.gelu(y.float()).to(dt)
    elif activation is not None:
        raise ValueError(f"unknown activation {activation!r}")
    if residual is not None:
        y = (y.float() + residual.float()).to(dt)
    return y, h64

