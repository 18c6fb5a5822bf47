"""End-to-end adaptive core and module vs the reference's own outputs.

The golden fixtures hold what the reference computed (per (b, h) slice and
for the whole call). The GPU path runs the analyzer, takes each slice's
decision on the device and computes it; heads are compared with the bars of
tests/parity.py, directly against the golden rows where the precision's bar is
stated against the reference's own output (FP32, FP16-class), and against the
oracle (pinned bit-exact to the same fixtures) for BF16 and E4M3 heads.
"""

import pytest
import torch

import oracle as O
from adaattn_b200 import AdaAttention, PrecisionMode, analyze, attention_forward
from adaattn_b200.core import possible_precisions
from golden_util import CASE_NAMES, PREC_CODE, inputs, load, module_kwargs, oracle_config
from parity import check_head, half_spacing, record

pytestmark = pytest.mark.gpu


def _core(rec, q, k, v, mask, granularity, dev, fp8_mode):
    cfg = oracle_config(rec)
    dp = PrecisionMode.from_code(cfg.default_precision)
    t = analyze(q.to(dev), k.to(dev), scale=rec["scale"], eps=cfg.eps,
                rank_threshold=cfg.rank_threshold, enable_adaptive_rank=cfg.enable_adaptive_rank,
                enable_adaptive_precision=cfg.enable_adaptive_precision, default_precision=dp,
                allow_fp8=cfg.allow_fp8, granularity=granularity)
    w = rec["w_down"]
    out = attention_forward(
        q.to(dev), k.to(dev), v.to(dev), scale=rec["scale"], causal=cfg.causal, table=t,
        w_down=None if w is None else w.to(dev),
        attention_mask=None if mask is None else mask.to(dev),
        possible_mask=possible_precisions(cfg.enable_adaptive_precision, dp, cfg.allow_fp8),
        low_rank_possible=cfg.enable_adaptive_rank and w is not None, fp8_mode=fp8_mode)
    torch.cuda.synchronize()
    return t, out.cpu(), cfg


@pytest.mark.parametrize("granularity", ["head", "global"])
@pytest.mark.parametrize("name", CASE_NAMES)
def test_golden_outputs(name, granularity, cuda_device):
    rec = load(name)
    q, k, v = inputs(rec)
    rows = rec["rows"]
    masks = {"none": None, **rec["masks"]}
    gkey = "per_head" if granularity == "head" else "global"
    for mname, mask in masks.items():
        t, out, cfg = _core(rec, q, k, v, mask, granularity, cuda_device, "fp16")
        prec = t.precision.cpu()
        low = t.low_rank.cpu()
        golden = rec["outputs"][mname][gkey]
        if granularity == "head":
            ref_prec = [[PREC_CODE[p] for p in row] for row in rec["per_head"]["precision"]]
            ref_low = rec["per_head"]["low_rank"]
        else:
            ref_prec = [[PREC_CODE[rec["global"]["precision"]]] * rec["heads"]] * rec["batch"]
            ref_low = torch.full((rec["batch"], rec["heads"]), rec["global"]["low_rank"])
        for b in range(rec["batch"]):
            for h in range(rec["heads"]):
                p, lo = int(prec[b, h]), bool(low[b, h])
                ms = None if mask is None else mask[b:b + 1]
                sl = (slice(b, b + 1), slice(h, h + 1))
                label = f"{name}/{mname}/{granularity}/b{b}h{h}"
                # full-slice check against the oracle at the decided precision
                full = out[sl]
                check_head(full, q[sl], k[sl], v[sl], p, lo, rec["scale"], cfg.causal, ms,
                           rec["w_down"], fp8_mode="fp16", label=label)
                # direct check against the reference's rows when the decision agrees
                if p == ref_prec[b][h] and lo == bool(ref_low[b, h]) and p in (O.FP32, O.FP16, O.FP8, O.AUTO):
                    g = golden[sl].float()
                    got = full[:, :, rows].float()
                    both_nan = torch.isnan(g).all() and torch.isnan(got).all()
                    if both_nan:
                        continue
                    mag = max(g.abs().max().item(), got.abs().max().item()) if g.numel() else 0.0
                    mm = max(1.0, mag)
                    # both sides end in the inputs' dtype (two roundings); FP16-computed
                    # heads of the reference round once more in fp16 before that
                    bar = ((1e-5 if p == O.FP32 else 2e-3) * mm + 2 * half_spacing(golden.dtype, mag)
                           + (0.0 if p == O.FP32 else half_spacing(torch.float16, mag)))
                    err = (got - g).abs().max().item() if g.numel() else 0.0
                    record(label + "/vs-reference-rows", O.PREC_NAMES[p], err, bar)
                    assert err <= bar, f"{label}: {err:.3e} > {bar:.3e} vs reference"


@pytest.mark.parametrize("name", ["precision_mix_small_fp8"])
def test_golden_fp8_heads_e4m3(name, cuda_device):
    rec = load(name)
    q, k, v = inputs(rec)
    t, out, cfg = _core(rec, q, k, v, None, "head", cuda_device, "e4m3")
    prec, low = t.precision.cpu(), t.low_rank.cpu()
    n_fp8 = 0
    for b in range(rec["batch"]):
        for h in range(rec["heads"]):
            sl = (slice(b, b + 1), slice(h, h + 1))
            check_head(out[sl], q[sl], k[sl], v[sl], int(prec[b, h]), bool(low[b, h]),
                       rec["scale"], cfg.causal, None, rec["w_down"], fp8_mode="e4m3",
                       label=f"b{b}h{h}")
            n_fp8 += int(prec[b, h]) == O.FP8
    assert n_fp8 > 0


def test_module_forward_matches_reference(cuda_device):
    rec = load("module_forward")
    m = AdaAttention(embed_dim=rec["embed_dim"], num_heads=rec["num_heads"],
                     decision_granularity="global").to(cuda_device).eval()
    m.load_state_dict(rec["state_dict"])
    x = rec["x"].to(cuda_device)
    with torch.no_grad():
        y, w = m(x, x, x)
    assert w is None
    y = y.cpu()
    # The reference decided globally; check the decision and the output at its precision.
    # The state dict carries the reference's counters (one call so far): after
    # one more call with the same decision every ratio is unchanged.
    stats = m.get_statistics()
    ref_stats = rec["stats"]
    assert stats["call_count"] == ref_stats["call_count"] + 1
    assert stats["low_rank_ratio"] == pytest.approx(ref_stats["low_rank_ratio"])
    for key, val in ref_stats["precision_distribution"].items():
        assert stats["precision_distribution"][key] == pytest.approx(val)
    prec = int(m.last_decisions.precision.flatten()[0])
    bar = (1e-5 if prec == O.FP32 else 2e-3) * max(1.0, rec["y"].abs().max().item())
    err = (y - rec["y"]).abs().max().item()
    assert err <= bar * 4, f"module output err {err:.3e} (precision {prec})"


@pytest.mark.parametrize("name", ["adaptive_mix", "low_rank_small", "dense_bf16_small"])
def test_module_per_head_mode(name, cuda_device):
    """Module in default per-head mode on [B, N, E] built from a fixture's heads."""
    rec = load(name)
    kw = module_kwargs(rec)
    h, d = rec["heads"], rec["head_dim"]
    q, k, v = inputs(rec)
    dtype = q.dtype
    m = AdaAttention(embed_dim=h * d, num_heads=h, **kw).to(cuda_device).to(dtype).eval()
    if m.rank_proj_down is not None:
        m.rank_proj_down.weight.data.copy_(rec["w_down"].to(cuda_device))
    out, table = m.attention_core(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device))
    cfg = oracle_config(rec)
    if table is None:  # decisions fixed by the configuration (no analyzer pass)
        prec = torch.full((rec["batch"], h), m.default_precision.code)
        low = torch.zeros(rec["batch"], h, dtype=torch.bool)
    else:
        prec, low = table.precision.cpu(), table.low_rank.cpu()
    out = out.cpu()
    for b in range(rec["batch"]):
        for hh in range(h):
            sl = (slice(b, b + 1), slice(hh, hh + 1))
            check_head(out[sl], q[sl], k[sl], v[sl], int(prec[b, hh]), bool(low[b, hh]),
                       rec["scale"], cfg.causal, None, rec["w_down"], label=f"b{b}h{hh}")
    s = m.get_statistics()
    assert s["call_count"] == 1
    assert abs(sum(s["precision_distribution"].values()) - 1.0) < 1e-5
