"""The on-device analyzer vs the reference's decisions (golden fixtures) and the
oracle's statistics.

Decisions must be identical except for heads whose statistic lies within
epsilon of a threshold (tests/parity.py: near_threshold).
"""

import pytest
import torch

import oracle as O
from adaattn_b200 import PrecisionMode, analyze
from adaattn_b200.workloads import WORKLOADS, make_qkv
from golden_util import CASE_NAMES, PREC_CODE, inputs, load, oracle_config
from parity import near_threshold

pytestmark = pytest.mark.gpu


def _analyze(q, k, cfg, scale, granularity, dev):
    return analyze(q.to(dev), k.to(dev), scale=scale, eps=cfg.eps,
                   rank_threshold=cfg.rank_threshold,
                   enable_adaptive_rank=cfg.enable_adaptive_rank,
                   enable_adaptive_precision=cfg.enable_adaptive_precision,
                   default_precision=PrecisionMode.from_code(cfg.default_precision),
                   allow_fp8=cfg.allow_fp8, granularity=granularity)


def _ulp(dtype):
    return {torch.float32: 2.0 ** -23, torch.float16: 2.0 ** -10, torch.bfloat16: 2.0 ** -7}[dtype]


@pytest.mark.parametrize("name", CASE_NAMES)
def test_per_head_decisions_match_reference(name, cuda_device):
    rec = load(name)
    q, k, _ = inputs(rec)
    cfg = oracle_config(rec)
    t = _analyze(q, k, cfg, rec["scale"], "head", cuda_device)
    prec = t.precision.cpu()
    low = t.low_rank.cpu()
    ref = rec["per_head"]
    want_prec = torch.tensor([[PREC_CODE[p] for p in row] for row in ref["precision"]])
    stats = O.analyze_per_head(q, k, cfg, rec["scale"])
    mism = 0
    for b in range(rec["batch"]):
        for h in range(rec["heads"]):
            same = int(prec[b, h]) == int(want_prec[b, h]) and bool(low[b, h]) == bool(ref["low_rank"][b, h])
            if not same:
                assert near_threshold(float(stats["ne"][b, h]), float(stats["max_score"][b, h]),
                                      float(stats["max_prob"][b, h]), cfg, q.dtype), \
                    f"{name} b{b}h{h}: got ({int(prec[b, h])},{bool(low[b, h])}) " \
                    f"want ({int(want_prec[b, h])},{bool(ref['low_rank'][b, h])})"
                mism += 1
    assert mism <= max(1, rec["batch"] * rec["heads"] // 16)


@pytest.mark.parametrize("name", CASE_NAMES)
def test_head_statistics_match_oracle(name, cuda_device):
    rec = load(name)
    q, k, _ = inputs(rec)
    cfg = oracle_config(rec)
    t = _analyze(q, k, cfg, rec["scale"], "head", cuda_device)
    hs = t.head_stats.cpu().double()
    st = O.analyze_per_head(q, k, cfg, rec["scale"])
    u = _ulp(q.dtype)
    torch.testing.assert_close(hs[..., 0], st["ne"], rtol=0, atol=2 * u + 1e-6)
    torch.testing.assert_close(hs[..., 1], st["max_score"], rtol=2 * u + 1e-6, atol=1e-6)
    torch.testing.assert_close(hs[..., 2], st["max_prob"], rtol=2 * u + 1e-6, atol=1e-6)


@pytest.mark.parametrize("name", CASE_NAMES)
def test_global_decision_matches_reference(name, cuda_device):
    rec = load(name)
    q, k, _ = inputs(rec)
    cfg = oracle_config(rec)
    t = _analyze(q, k, cfg, rec["scale"], "global", cuda_device)
    g = O.analyze(q, k, cfg, rec["scale"])
    summ = t.summary.cpu()
    prec = t.precision.cpu()
    assert (prec == prec.flatten()[0]).all()
    same = (int(prec.flatten()[0]) == PREC_CODE[rec["global"]["precision"]]
            and bool(t.low_rank.cpu().flatten()[0]) == rec["global"]["low_rank"])
    if not same:
        assert near_threshold(g["ne"], g["max_score"], g["max_prob"], cfg, q.dtype)
    assert abs(float(summ[0]) - g["ne"]) <= 2 * _ulp(q.dtype) + 1e-6
    assert float(summ[9]) == 1.0


def test_workload_decisions_precision_mix(cuda_device):
    """Per-head precision of the precision-mix workload (one batch row)."""
    w = WORKLOADS["precision_mix"].scaled(batch=1, heads=32, seq=512)
    q, k, _ = make_qkv(w, seed=0)
    for allow in (False, True):
        cfg = O.OracleConfig(causal=True, allow_fp8=allow)
        t = _analyze(q, k, cfg, 128 ** -0.5, "head", cuda_device)
        st = O.analyze_per_head(q, k, cfg, 128 ** -0.5)
        got = t.precision.cpu()
        bad = [(h, int(got[0, h]), int(st["precision"][0, h])) for h in range(32)
               if int(got[0, h]) != int(st["precision"][0, h])
               and not near_threshold(float(st["ne"][0, h]), float(st["max_score"][0, h]),
                                      float(st["max_prob"][0, h]), cfg, q.dtype)]
        assert not bad, bad


def test_sample_stride_knob(cuda_device):
    """Strided sampling (opt-in) reads rows 0, s, 2s, ...: same as the
    reference analyzer applied to the strided rows."""
    w = WORKLOADS["adaptive_mix"].scaled(batch=1, heads=4, seq=512)
    q, k, _ = make_qkv(w, seed=0)
    cfg = O.OracleConfig()
    t = analyze(q.to(cuda_device), k.to(cuda_device), scale=0.125, sample_stride=8)
    st = O.analyze_per_head(q[:, :, ::8], k[:, :, ::8], cfg, 0.125)
    torch.testing.assert_close(t.head_stats.cpu().double()[..., 0], st["ne"], rtol=0, atol=1e-5)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("d", [192, 256])
def test_head_statistics_wide_heads(d, dtype, cuda_device):
    """Head dims above 128 with a full 64-row sample: the 16-byte load path
    needs more than one round of loads per thread (S * D / 8 > 1024 groups)."""
    g = torch.Generator().manual_seed(13)
    q = (torch.randn(2, 3, 100, d, generator=g) * 0.7).to(dtype)
    k = (torch.randn(2, 3, 90, d, generator=g) * 0.7).to(dtype)
    scale = d ** -0.5
    cfg = O.OracleConfig()
    t = _analyze(q, k, cfg, scale, "head", cuda_device)
    hs = t.head_stats.cpu().double()
    st = O.analyze_per_head(q, k, cfg, scale)
    u = _ulp(dtype)
    torch.testing.assert_close(hs[..., 0], st["ne"], rtol=0, atol=2 * u + 1e-6)
    torch.testing.assert_close(hs[..., 1], st["max_score"], rtol=2 * u + 1e-6, atol=1e-6)
    torch.testing.assert_close(hs[..., 2], st["max_prob"], rtol=2 * u + 1e-6, atol=1e-6)
    # a strided view (not 16-byte rows) takes the scalar path: same statistics
    qs = torch.zeros(2, 3, 100, d + 1, dtype=dtype, device=cuda_device)[..., :d]
    qs.copy_(q.to(cuda_device))
    t2 = _analyze(qs, k, cfg, scale, "head", cuda_device)
    torch.testing.assert_close(t2.head_stats.cpu(), t.head_stats.cpu(), rtol=0, atol=0)
