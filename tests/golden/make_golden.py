"""Generate golden fixtures by running the AdaAttn reference itself.

Run in a container that has the reference checked out (read-only is fine):

    python tests/golden/make_golden.py --reference /root/reference/src

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
  of a rank-2 matrix (the reference's own test_low_rank.py case).

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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default="/root/reference/src")
    ap.add_argument("--out", default=HERE)
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    import adaattn.attention.adaattn as A  # noqa: E402  (must come first)
    from adaattn.attention.base import PrecisionMode as PM  # noqa: E402
    import adaattn.linalg.low_rank as LR  # noqa: E402
    torch.set_num_threads(os.cpu_count() or 1)
    for case in CASES:
        rec = run_case(A, PM, *case, out_dir=args.out)
        print(case[0], rec["global"], flush=True)
    module_case(A, args.out)
    kat_case(A, LR, args.out)


if __name__ == "__main__":
    main()
