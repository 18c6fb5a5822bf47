"""Per-precision output tolerances shared by the GPU parity tests.

Bars (stated here once, used by every parity test):
  FP32 heads   max|got - ref_fp32| <= 1e-5 * max(1, max|ref_fp32|)
  FP16 heads   max|got - ref_fp16| <= 2e-3 * max(1, max|ref_fp16|)
               (also AUTO, and FP8 heads in the reference's fp16 mode)
  BF16 heads   max|got - ref_fp32| <= max(2e-3 * m, 1.5 * max|ref_bf16 - ref_fp32|)
               with m = max(1, max|ref_fp32|): the reference takes its softmax
               in bf16, a fused fp32 softmax is closer to the fp32 result.
  FP8 (E4M3)   max|got - ref_fp32| <= 1.5 * max|fp8_oracle - ref_fp32| + 1e-3 * m
  where ref_* is the CPU oracle's restatement of the reference on the same
  inputs at that precision (dense or low-rank branch as decided). Each bar
  also admits one unit in the last place of the output dtype (2^-7 * m for
  bf16 outputs, 2^-10 * m for fp16, 0 for fp32): the reference casts its
  result back to the inputs' dtype.
"""

from __future__ import annotations

import torch

import oracle as O


def reference_outputs(q, k, v, prec, low, scale, causal, mask=None, w_down=None):
    def run(p):
        if low:
            return O.low_rank_attention(q, k, v, w_down, p, scale, causal, mask)
        return O.dense_attention(q, k, v, p, scale, causal, mask)
    return run


def output_ulp(dtype) -> float:
    """Largest relative spacing of the output dtype: the reference casts its
    result back to the inputs' dtype (adaattn.py:339, :394), so two results
    that agree before that cast may still differ by one unit there."""
    return {torch.float32: 0.0, torch.float16: 2.0 ** -10, torch.bfloat16: 2.0 ** -7}[dtype]


def check_head(got, q, k, v, prec, low, scale, causal, mask=None, w_down=None,
               fp8_mode="e4m3", label=""):
    """Assert one slice's output meets the bar for its precision.

    Every bar below gets one output-dtype unit (output_ulp * m) added, since
    both sides end in the inputs' dtype.
    """
    qo = output_ulp(got.dtype)
    got = got.float().cpu()
    run = reference_outputs(q, k, v, prec, low, scale, causal, mask, w_down)
    ref32 = run(O.FP32).float()
    m = max(1.0, ref32.abs().max().item()) if ref32.numel() else 1.0
    if prec == O.FP32:
        err = (got - ref32).abs().max().item()
        bar = 1e-5 * m + qo * m
        assert err <= bar, f"{label} FP32 err {err:.3e} > {bar:.3e}"
        return err
    if prec in (O.FP16, O.AUTO) or (prec == O.FP8 and fp8_mode != "e4m3"):
        ref = run(O.FP16 if prec != O.AUTO else O.AUTO).float()
        err = (got - ref).abs().max().item()
        mm = max(1.0, ref.abs().max().item())
        bar = 2e-3 * mm + qo * mm
        assert err <= bar, f"{label} FP16 err {err:.3e} > {bar:.3e}"
        return err
    if prec == O.BF16:
        ref16 = run(O.BF16).float()
        own = (ref16 - ref32).abs().max().item()
        err = (got - ref32).abs().max().item()
        bar = max(2e-3 * m, 1.5 * own) + qo * m
        assert err <= bar, f"{label} BF16 err {err:.3e} > {bar:.3e} (reference bf16 err {own:.3e})"
        return err
    if prec == O.FP8:
        fo = O.fp8_dense_attention(q, k, v, scale, causal, mask,
                                   w_down=w_down if low else None).float()
        own = (fo - ref32).abs().max().item()
        err = (got - ref32).abs().max().item()
        bar = 1.5 * own + 1e-3 * m + qo * m
        assert err <= bar, f"{label} FP8 err {err:.3e} > {bar:.3e} (oracle fp8 err {own:.3e})"
        return err
    raise AssertionError(f"unknown precision {prec}")


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
