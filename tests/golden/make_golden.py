"""Generate golden fixtures by running the AdaAttn reference itself.

Run in a container that has the reference checked out (read-only is fine):

    python tests/golden/make_golden.py --reference <reference checkout>/src

(or set ADAATTN_REFERENCE_SRC to that directory).

It imports the reference's ``AdaAttention`` (``adaattn.attention.adaattn`` is
imported first: importing ``adaattn.kernels`` first trips a circular import in
the reference), draws the seeded inputs of ``adaattn_b200.workloads`` at small
sizes, and stores what the reference computes:

* its analyzer decision (``_analyze_attention_pattern``) for the whole call and
  for every (b, h) slice, with the effective rank it returns;
* ``_adaptive_attention_forward`` outputs, per slice and for the whole call, on
  a strided subset of query rows (rows are independent given K and V);
* one module-level ``forward`` with its state dict;
* known answers: a constant query (uniform attention) and the randomized SVD
  of a rank-2 matrix (the reference's own test_low_rank.py case);
* the kernel-level functions of ``adaattn.kernels`` (flash and adaptive
  attention on [B, N, H, D]);
* a small ``AdaptiveTransformer`` from the reference's
  examples/transformer_integration.py: logits and every block's input and
  output.

The fixtures are small ``.pt`` files; the GPU box never needs the reference.
"""

from __future__ import annotations

import argparse
import math
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from adaattn_b200.workloads import WORKLOADS, make_qkv  # noqa: E402

sys.path.insert(0, os.path.dirname(HERE))
from golden_util import (TRANSFORMER, kernel_op_inputs, transformer_ids,  # noqa: E402
                         transformer_state)

ROWS_KEPT = 32

# (fixture name, workload, batch, heads, seq, module kwargs, extra)
CASES = [
    ("adaptive_mix", "adaptive_mix", None, None, None, {}, {}),
    ("precision_mix_small", "precision_mix", 2, 8, 256, {"causal": True}, {}),
    ("precision_mix_small_fp8", "precision_mix", 2, 8, 256,
     {"causal": True, "allow_fp8": True}, {}),
    ("low_rank_small", "low_rank_mix", 1, 4, 512, {}, {}),
    ("dense_bf16_small", "dense_bf16", 1, 2, 384,
     {"causal": True, "enable_adaptive_rank": False,
      "enable_adaptive_precision": False, "default_precision": "BF16"}, {}),
    ("edge_short_causal", "adaptive_mix", 1, 3, 17, {"causal": True}, {}),
    ("edge_cross_masked", "precision_mix", 2, 2, 80, {},
     {"nq": 32, "masks": True}),
]


def _checksum(t: torch.Tensor) -> float:
    return float(t.double().sum().item())


def _row_index(n: int) -> torch.Tensor:
    step = max(1, n // ROWS_KEPT)
    return torch.arange(0, n, step)[:ROWS_KEPT]


def _ref_module(A, PM, head_dim: int, heads: int, dtype, kw: dict, seed: int):
    kw = dict(kw)
    if "default_precision" in kw:
        kw["default_precision"] = getattr(PM, kw["default_precision"])
    torch.manual_seed(seed)
    m = A.AdaAttention(embed_dim=head_dim * heads, num_heads=heads, **kw)
    m = m.to(dtype).eval()
    return m


def run_case(A, PM, name, wname, b, h, n, kw, extra, out_dir):
    w = WORKLOADS[wname].scaled(batch=b, heads=h, seq=n)
    q, k, v = make_qkv(w, seed=0)
    nq = extra.get("nq")
    if nq is not None:
        q = q[:, :, :nq].contiguous()
    m = _ref_module(A, PM, w.head_dim, w.heads, w.dtype, kw, seed=1234)
    w_down = m.rank_proj_down.weight.detach().clone() \
        if m.rank_proj_down is not None else None
    masks = {"none": None}
    if extra.get("masks"):
        g = torch.Generator().manual_seed(7)
        keep = torch.rand(w.batch, k.shape[2], generator=g) > 0.3
        keep[:, 0] = True
        masks["bool2d"] = keep
        masks["float3d"] = torch.randn(w.batch, q.shape[2], k.shape[2],
                                       generator=g)
    rows = _row_index(q.shape[2])
    rec = {
        "workload": wname, "batch": w.batch, "heads": w.heads,
        "seq_q": q.shape[2], "seq_k": k.shape[2], "head_dim": w.head_dim,
        "dtype": str(w.dtype), "module_kwargs": {kk: str(vv) for kk, vv in kw.items()},
        "causal": bool(kw.get("causal", False)),
        "checksum": [_checksum(q), _checksum(k), _checksum(v)],
        "rows": rows, "w_down": w_down, "scale": m.scale,
    }
    with torch.no_grad():
        low, prec, eff = m._analyze_attention_pattern(q, k)
        rec["global"] = {"low_rank": bool(low), "precision": prec.name,
                         "effective_rank": float(eff)}
        dec_low = torch.zeros(w.batch, w.heads, dtype=torch.bool)
        dec_prec = [[None] * w.heads for _ in range(w.batch)]
        dec_eff = torch.zeros(w.batch, w.heads, dtype=torch.float64)
        for bi in range(w.batch):
            for hi in range(w.heads):
                l_, p_, e_ = m._analyze_attention_pattern(
                    q[bi:bi + 1, hi:hi + 1], k[bi:bi + 1, hi:hi + 1])
                dec_low[bi, hi] = bool(l_)
                dec_prec[bi][hi] = p_.name
                dec_eff[bi, hi] = float(e_)
        rec["per_head"] = {"low_rank": dec_low, "precision": dec_prec,
                           "effective_rank": dec_eff}
        outs = {}
        for mname, mask in masks.items():
            o_glob, _ = m._adaptive_attention_forward(q, k, v, mask)
            o_head = torch.empty(w.batch, w.heads, q.shape[2], w.head_dim,
                                 dtype=q.dtype)
            for bi in range(w.batch):
                for hi in range(w.heads):
                    ms = None if mask is None else mask[bi:bi + 1]
                    o, _ = m._adaptive_attention_forward(
                        q[bi:bi + 1, hi:hi + 1], k[bi:bi + 1, hi:hi + 1],
                        v[bi:bi + 1, hi:hi + 1], ms)
                    o_head[bi:bi + 1, hi:hi + 1] = o
            outs[mname] = {"global": o_glob[:, :, rows].clone(),
                           "per_head": o_head[:, :, rows].clone()}
        rec["outputs"] = outs
        rec["masks"] = {kk: vv for kk, vv in masks.items() if vv is not None}
    torch.save(rec, os.path.join(out_dir, f"{name}.pt"))
    return rec


def module_case(A, out_dir):
    """One full AdaAttention.forward on [B, N, E] with its state dict."""
    torch.manual_seed(4321)
    m = A.AdaAttention(embed_dim=128, num_heads=2).eval()
    g = torch.Generator().manual_seed(11)
    x = torch.randn(2, 96, 128, generator=g)
    with torch.no_grad():
        y, _ = m(x, x, x)
    rec = {"state_dict": {kk: vv.clone() for kk, vv in m.state_dict().items()},
           "x": x, "y": y, "stats": m.get_statistics(),
           "embed_dim": 128, "num_heads": 2}
    torch.save(rec, os.path.join(out_dir, "module_forward.pt"))


def kat_case(A, LR, out_dir):
    rec = {}
    m = A.AdaAttention(embed_dim=128, num_heads=2).eval()
    z = torch.zeros(1, 2, 64, 64)
    g = torch.Generator().manual_seed(3)
    kk = torch.randn(1, 2, 64, 64, generator=g)
    with torch.no_grad():
        low, prec, eff = m._analyze_attention_pattern(z, kk)
    rec["uniform"] = {"low_rank": bool(low), "precision": prec.name,
                      "effective_rank": float(eff)}
    # test_low_rank.py:44-59 -- rank-2 matrix, rank=2, oversampling 5.
    g = torch.Generator().manual_seed(5)
    u_true = torch.randn(10, 2, generator=g)
    v_true = torch.randn(5, 2, generator=g)
    a = u_true @ v_true.T
    torch.manual_seed(99)
    u, s, vt = LR.randomized_svd(a, rank=2, num_oversampling=5)
    rec["rsvd_rank2"] = {"A": a, "seed": 99, "oversample": 5, "rank": 2,
                         "U": u, "S": s, "Vh": vt}
    # Batched case of test_low_rank.py:61-69 with a fixed seed.
    g = torch.Generator().manual_seed(6)
    ab = torch.randn(4, 8, 6, generator=g)
    torch.manual_seed(100)
    u, s, vt = LR.randomized_svd(ab, rank=3)
    rec["rsvd_batch"] = {"A": ab, "seed": 100, "oversample": 10, "rank": 3,
                         "U": u, "S": s, "Vh": vt}
    torch.save(rec, os.path.join(out_dir, "kat.pt"))


def kernel_ops_case(K, out_dir):
    """The reference's kernel-level functions (adaattn.kernels) on the seeded
    [B, N, H, D] inputs of golden_util.kernel_op_inputs. Its native module is
    never built, so these are the Python paths its callers actually run
    (kernels/__init__.py:81-213); the entropy helpers exist only in the native
    module (bindings.cpp:101-135), which the oracle restates and the known
    answers of the tests pin."""
    rec = {}
    for name, (q, k, v) in kernel_op_inputs().items():
        with torch.no_grad():
            rec[f"flash_{name}"] = {
                "out": K.flash_attention_forward(q, k, v, None, False),
                "out_causal": K.flash_attention_forward(q, k, v, 0.2, True)}
            rec[f"adaptive_{name}"] = {
                "fp16": K.adaptive_attention_forward(q, k, v, None, "fp16", None, True),
                "bf16": K.adaptive_attention_forward(q, k, v, None, "bf16", None, False),
                "fp32": K.adaptive_attention_forward(q, k, v, None, "fp32", 0.15, True)}
    torch.save(rec, os.path.join(out_dir, "kernel_ops.pt"))


def transformer_case(A, PM, ex_path, out_dir):
    """The reference's examples/transformer_integration.py AdaptiveTransformer
    at a small size (golden_util.TRANSFORMER), eval mode, fp32, with the
    seeded weights of golden_util.transformer_state. Stores the logits and
    every block's output and decision; and, as the precision noise floor of
    each block and of the logits, how far they move when every attention
    decision's precision is replaced by FP32 (same branch)."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("transformer_integration", ex_path)
    ex = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ex)
    model = ex.AdaptiveTransformer(**TRANSFORMER).eval()
    model.load_state_dict(transformer_state(model.state_dict()), strict=False)
    ids = transformer_ids()
    blocks = []

    def force_fp32(att):
        orig = att._analyze_attention_pattern

        def forced(q, k):
            lo, _, ef = orig(q, k)
            return lo, PM.FP32, ef
        att._analyze_attention_pattern = forced

    with torch.no_grad():
        pos = torch.arange(ids.shape[1]).unsqueeze(0)
        x = model.token_embedding(ids) + model.position_embedding(pos)
        for blk in model.blocks:
            att = blk.attention
            y = blk(x)
            low, prec, _ = att._analyze_attention_pattern(
                *[t.view(x.shape[0], x.shape[1], att.num_heads, -1).transpose(1, 2)
                  for t in (att.q_proj(x), att.k_proj(x))])
            force_fp32(att)
            y32 = blk(x)
            del att._analyze_attention_pattern
            blocks.append({"y": y.clone(), "fp32_attention_diff": float((y - y32).abs().max()),
                           "low_rank": bool(low), "precision": prec.name})
            x = y
        logits = model(ids)
        for blk in model.blocks:
            force_fp32(blk.attention)
        logits32 = model(ids)
    torch.save({"config": dict(TRANSFORMER), "logits": logits,
                "fp32_attention_diff": float((logits - logits32).abs().max()), "blocks": blocks},
               os.path.join(out_dir, "transformer_small.pt"))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("ADAATTN_REFERENCE_SRC"),
                    help="the reference's src/ directory (or set ADAATTN_REFERENCE_SRC)")
    ap.add_argument("--out", default=HERE)
    ap.add_argument("--only", nargs="*", default=None,
                    help="fixture names to regenerate (default: all)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("--reference (or ADAATTN_REFERENCE_SRC) is required")
    sys.path.insert(0, args.reference)
    import adaattn.attention.adaattn as A  # noqa: E402  (must come first)
    from adaattn.attention.base import PrecisionMode as PM  # noqa: E402
    import adaattn.linalg.low_rank as LR  # noqa: E402
    import adaattn.kernels as K  # noqa: E402
    torch.set_num_threads(os.cpu_count() or 1)
    want = (lambda n: args.only is None or n in args.only)
    for case in CASES:
        if want(case[0]):
            rec = run_case(A, PM, *case, out_dir=args.out)
            print(case[0], rec["global"], flush=True)
    if want("module_forward"):
        module_case(A, args.out)
    if want("kat"):
        kat_case(A, LR, args.out)
    if want("kernel_ops"):
        kernel_ops_case(K, args.out)
    if want("transformer_small"):
        ex_path = os.path.join(os.path.dirname(os.path.abspath(args.reference)), "examples",
                               "transformer_integration.py")
        transformer_case(A, PM, ex_path, args.out)


if __name__ == "__main__":
    main()
