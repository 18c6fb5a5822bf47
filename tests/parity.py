"""Per-precision output tolerances shared by the GPU parity tests.

Bars (stated here once, used by every parity test):
  FP32 heads   max|got - ref_fp32| <= max(1e-5 * m, 2 * max|ref_fp32 - ref_fp64|)
               where the fp32 arithmetic's own error is large (scores of 1e3
               and more make the softmax sensitive to the order of the fp32
               sums), twice the reference's fp32-vs-float64 error is the bar;
               for low-rank heads of 16-bit inputs, also the effect of
               rounding q_low / k_low to the inputs' dtype (a projection
               summing in another order may round a few elements the other
               way): max|ref_fp32(projection in fp32) - ref_fp32|.
  FP16 heads   max|got - ref_fp16| <= 2e-3 * m16
               (also AUTO, and FP8 heads in the reference's fp16 mode)
  BF16 heads   max|got - ref_fp32| <= max(2e-3 * m, 1.5 * max|ref_bf16 - ref_fp32|)
               the reference takes its softmax in bf16 (adaattn.py:333-334); a
               fused fp32 softmax is closer to the fp32 result, so the bar is
               taken against ref_fp32 and the reference's own bf16 error
               widens it only where that error exceeds 2e-3 * m.
  FP8 (E4M3)   max|got - ref_fp32| <= 1.5 * max|fp8_oracle - ref_fp32| + 1e-3 * m
  with m = max(1, max|ref_fp32|), m16 = max(1, max|ref_fp16|), where ref_* is
  the CPU oracle's restatement of the reference on the same inputs at that
  precision (dense or low-rank branch as decided).

Rounding of the result: ref_fp32 and ref_fp16 are taken before the
reference's final cast to the inputs' dtype (adaattn.py:339, :394); the
kernel's output has been through that cast, so each bar admits the most the
cast can move a value: half the spacing of the output dtype at the largest
output magnitude (0 for fp32 outputs), plus half the fp16 spacing where the
reference itself ends in fp16. At the dense BF16 workload's magnitudes
(|out| < 0.5) the slack is at most 2^-10.

Every check records (label, precision, error, bar) in RESULTS; the test
session prints the largest error and error/bar ratio per precision.
"""

from __future__ import annotations

import math

import torch

import oracle as O

RESULTS = []  # (label, precision name, max-abs error, bar)

_MANT = {torch.float16: 10, torch.bfloat16: 7}
_MIN_EXP = {torch.float16: -14, torch.bfloat16: -126}


def half_spacing(dtype, magnitude: float) -> float:
    """Half the gap between adjacent values of ``dtype`` at ``magnitude``:
    the largest change rounding a value of that size to ``dtype`` makes."""
    if dtype not in _MANT or magnitude <= 0.0 or not math.isfinite(magnitude):
        return 0.0
    e = max(math.floor(math.log2(magnitude)), _MIN_EXP[dtype])
    return 0.5 * 2.0 ** (e - _MANT[dtype])


def record(label: str, prec_name: str, err: float, bar: float) -> None:
    RESULTS.append((label, prec_name, float(err), float(bar)))


def reference_outputs(q, k, v, prec, low, scale, causal, mask=None, w_down=None):
    def run(p, cast_back=True, compute=None):
        if low:
            return O.low_rank_attention(q, k, v, w_down, p, scale, causal, mask,
                                        cast_back=cast_back, compute=compute)
        return O.dense_attention(q, k, v, p, scale, causal, mask, cast_back=cast_back,
                                 compute=compute)
    return run


def _amax(t) -> float:
    if t.numel() == 0:
        return 0.0
    a = t.abs()
    a = a[torch.isfinite(a)]
    return a.max().item() if a.numel() else 0.0


def _maxdiff(a, b) -> float:
    return (a - b).abs().max().item() if a.numel() else 0.0


def check_head(got, q, k, v, prec, low, scale, causal, mask=None, w_down=None,
               fp8_mode="e4m3", label=""):
    """Assert one slice's output meets the bar for its precision; returns the
    max-abs error.

    ref_fp32 is the oracle's fp32 result before the final cast to the inputs'
    dtype, so only the kernel's own cast needs the rounding slack; the FP16
    reference is compared in fp16 (one more rounding, at fp16 spacing).
    """
    out_dtype = got.dtype
    got = got.float().cpu()
    run = reference_outputs(q, k, v, prec, low, scale, causal, mask, w_down)
    ref32 = run(O.FP32, cast_back=False).float()
    m = max(1.0, _amax(ref32))
    mag = max(_amax(ref32), _amax(got))
    rnd = half_spacing(out_dtype, mag)
    if prec == O.FP32:
        ref64 = run(O.FP32, cast_back=False, compute=torch.float64)
        own = _maxdiff(ref32.double(), ref64)
        if low and q.dtype != torch.float32:
            # q_low / k_low are rounded to the inputs' dtype (F.linear in that
            # dtype, adaattn.py:357-358); a projection that sums in another
            # order can land one unit away on a few elements, which the
            # softmax then amplifies. Bound: how far the whole rounding moves
            # the result (the same branch with the projection kept in fp32).
            proj32 = O.low_rank_attention(q.float(), k.float(), v.float(), w_down.float(), O.FP32,
                                          scale, causal, mask, cast_back=False).float()
            own = max(own, 0.5 * _maxdiff(proj32, ref32))
        err = _maxdiff(got, ref32)
        bar = max(1e-5 * m, 2.0 * own) + rnd
        record(label, "FP32", err, bar)
        assert err <= bar, f"{label} FP32 err {err:.3e} > {bar:.3e} (reference fp32 err {own:.3e})"
        return err
    if prec in (O.FP16, O.AUTO) or (prec == O.FP8 and fp8_mode != "e4m3"):
        ref = run(O.FP16 if prec != O.AUTO else O.AUTO, cast_back=False).float()
        err = _maxdiff(got, ref)
        mm = max(1.0, _amax(ref))
        bar = 2e-3 * mm + rnd + half_spacing(torch.float16, mag)
        record(label, "FP16", err, bar)
        assert err <= bar, f"{label} FP16 err {err:.3e} > {bar:.3e}"
        return err
    if prec == O.BF16:
        ref16 = run(O.BF16).float()
        own = _maxdiff(ref16, ref32)
        err = _maxdiff(got, ref32)
        bar = max(2e-3 * m, 1.5 * own) + rnd
        record(label, "BF16", err, bar)
        assert err <= bar, f"{label} BF16 err {err:.3e} > {bar:.3e} (reference bf16 err {own:.3e})"
        return err
    if prec == O.FP8:
        fo = O.fp8_dense_attention(q, k, v, scale, causal, mask,
                                   w_down=w_down if low else None).float()
        own = _maxdiff(fo, ref32)
        err = _maxdiff(got, ref32)
        bar = 1.5 * own + 1e-3 * m + rnd
        record(label, "FP8", err, bar)
        assert err <= bar, f"{label} FP8 err {err:.3e} > {bar:.3e} (oracle fp8 err {own:.3e})"
        return err
    raise AssertionError(f"unknown precision {prec}")


def summary_lines():
    """One line per precision: checks, largest error, largest error / bar."""
    by = {}
    for label, p, err, bar in RESULTS:
        n, e, r, lab = by.get(p, (0, 0.0, 0.0, ""))
        ratio = err / bar if bar > 0 else 0.0
        if ratio > r:
            lab = label
        by[p] = (n + 1, max(e, err), max(r, ratio), lab)
    return [f"{p:5s} checks {n:4d}  max err {e:.3e}  max err/bar {r:.3f} ({lab})"
            for p, (n, e, r, lab) in sorted(by.items())]


def near_threshold(ne, ms, mp, cfg, dtype) -> bool:
    """True when a statistic sits within epsilon of a decision threshold.

    epsilon = max(1e-3 relative, two units in the last place of the inputs'
    dtype at that threshold): statistics are quantised to the inputs' dtype by
    the reference's own arithmetic.
    """
    ulp = {torch.float32: 2.0 ** -23, torch.float16: 2.0 ** -10, torch.bfloat16: 2.0 ** -7}[dtype]

    def close(x, thr):
        return abs(x - thr) <= max(1e-3 * abs(thr), 2 * ulp * abs(thr))

    return (close(ne, cfg.rank_threshold) or close(ne, 0.8) or close(ne, 0.3)
            or close(ms, 50.0) or close(mp, 0.95))
