"""Parity at the benchmark workloads' full shapes against the CPU oracle.

The kernels run over the whole workload (every (b, h) slice, the persistent
scheduler at full size); the oracle then checks sampled slices, all of their
rows, and every head's decision:

  dense_bf16     B8 H32 N4096 D128 bf16 causal, forced BF16 / dense: slices
                 (0,0), (3,17), (7,31) against the fp32 oracle with the flat
                 2e-3 max-abs bar (plus the parity.py bar, which also reports
                 the error against the reference's own bf16 arithmetic).
  low_rank_mix   B4 H16 N8192 D128 bf16: decisions of all 64 heads; outputs of
                 one low-rank-key head and one full-rank head at the decided
                 (branch, precision).
  precision_mix  B8 H32 N2048 D128 bf16 causal: decisions of all 256 heads with
                 allow_fp8 off and on; outputs of one head of every (branch,
                 precision) that occurs.
"""

import math

import pytest
import torch

import oracle as O
from adaattn_b200 import AdaAttention, PrecisionMode, analyze, attention_forward
from adaattn_b200.workloads import WORKLOADS, make_qkv
from parity import check_head, half_spacing, near_threshold, record

pytestmark = pytest.mark.gpu


def _slice(t, b, h):
    return t[b:b + 1, h:h + 1].cpu()


def test_dense_bf16_full_shape(cuda_device):
    w = WORKLOADS["dense_bf16"]
    q, k, v = make_qkv(w, seed=0, device=str(cuda_device))
    scale = 1.0 / math.sqrt(w.head_dim)
    out = attention_forward(q, k, v, scale=scale, causal=True,
                            static_precision=PrecisionMode.BF16, static_low_rank=False)
    torch.cuda.synchronize()
    for b, h in [(0, 0), (3, 17), (7, 31)]:
        qs, ks, vs, os_ = (_slice(t, b, h) for t in (q, k, v, out))
        ref32 = O.dense_attention(qs, ks, vs, O.FP32, scale, True, cast_back=False).float()
        ref_bf16 = O.dense_attention(qs, ks, vs, O.BF16, scale, True).float()
        got = os_.float()
        err = (got - ref32).abs().max().item()
        err_ref = (got - ref_bf16).abs().max().item()
        own = (ref_bf16 - ref32).abs().max().item()
        record(f"dense_bf16/b{b}h{h}/flat", "BF16", err, 2e-3)
        print(f"dense_bf16 b{b} h{h}: max-abs vs fp32 {err:.3e}, vs reference bf16 "
              f"{err_ref:.3e} (reference bf16 vs fp32 {own:.3e}), max|out| {got.abs().max():.3f}")
        assert err <= 2e-3, f"b{b}h{h}: {err:.3e} > 2e-3"
        check_head(os_, qs, ks, vs, O.BF16, False, scale, True, label=f"dense_bf16/b{b}h{h}")


def _decisions_match(t, q, k, cfg, scale, label):
    """Every head's decision equals the oracle's analyzer applied to that
    slice, except heads with a statistic within epsilon of a threshold."""
    st = O.analyze_per_head(q[:, :, :64].cpu(), k[:, :, :64].cpu(), cfg, scale)
    prec, low = t.precision.cpu(), t.low_rank.cpu()
    bad = []
    for b in range(q.shape[0]):
        for h in range(q.shape[1]):
            same = (int(prec[b, h]) == int(st["precision"][b, h])
                    and bool(low[b, h]) == bool(st["low_rank"][b, h]))
            if not same and not near_threshold(float(st["ne"][b, h]), float(st["max_score"][b, h]),
                                               float(st["max_prob"][b, h]), cfg, q.dtype):
                bad.append((b, h, int(prec[b, h]), bool(low[b, h])))
    assert not bad, f"{label}: decisions differ from the oracle: {bad}"
    return prec, low


def _module(w, **kw):
    m = AdaAttention(embed_dim=w.heads * w.head_dim, num_heads=w.heads, **kw)
    return m.to(torch.bfloat16).eval()


def test_low_rank_mix_full_shape(cuda_device):
    w = WORKLOADS["low_rank_mix"]
    q, k, v = make_qkv(w, seed=0, device=str(cuda_device))
    scale = 1.0 / math.sqrt(w.head_dim)
    m = _module(w, causal=False).to(cuda_device)
    w_down = m.rank_proj_down.weight.detach()
    cfg = O.OracleConfig(causal=False)
    with torch.no_grad():
        out, t = m.attention_core(q, k, v)
    torch.cuda.synchronize()
    prec, low = _decisions_match(t, q, k, cfg, scale, "low_rank_mix")
    print("low_rank_mix decisions:", sorted(set(zip(prec.flatten().tolist(), low.flatten().tolist()))))
    wd = w_down.cpu()
    for b, h in [(0, 0), (3, w.heads // 2 + 1)]:   # a low-rank-key head, a full-rank head
        qs, ks, vs, os_ = (_slice(x, b, h) for x in (q, k, v, out))
        check_head(os_, qs, ks, vs, int(prec[b, h]), bool(low[b, h]), scale, False, w_down=wd,
                   label=f"low_rank_mix/b{b}h{h}")


@pytest.mark.parametrize("allow_fp8", [False, True])
def test_precision_mix_full_shape(allow_fp8, cuda_device):
    w = WORKLOADS["precision_mix"]
    q, k, v = make_qkv(w, seed=0, device=str(cuda_device))
    scale = 1.0 / math.sqrt(w.head_dim)
    m = _module(w, causal=True, allow_fp8=allow_fp8).to(cuda_device)
    wd = m.rank_proj_down.weight.detach().cpu()
    cfg = O.OracleConfig(causal=True, allow_fp8=allow_fp8)
    with torch.no_grad():
        out, t = m.attention_core(q, k, v)
    torch.cuda.synchronize()
    prec, low = _decisions_match(t, q, k, cfg, scale, f"precision_mix fp8={allow_fp8}")
    seen = {}
    for b in range(w.batch):
        for h in range(w.heads):
            seen.setdefault((int(prec[b, h]), bool(low[b, h])), (b, h))
    print(f"precision_mix allow_fp8={allow_fp8}: one head per (precision, low rank):", seen)
    if allow_fp8:
        assert any(p == O.FP8 for p, _ in seen), "no FP8 head at allow_fp8=True"
    for (p, lo), (b, h) in sorted(seen.items()):
        qs, ks, vs, os_ = (_slice(x, b, h) for x in (q, k, v, out))
        check_head(os_, qs, ks, vs, p, lo, scale, True, w_down=wd,
                   label=f"precision_mix/fp8={int(allow_fp8)}/b{b}h{h}")
