"""Throughput of the adaptive path on the five AdaAttn workloads (one GPU).

    python -m adaattn_b200.bench_workloads [--workload NAME] [--steps K]

Each workload runs the analyzer and the adaptive core (per-(b,h) decisions on
the device) on seeded synthetic inputs resident in HBM, timed with CUDA events
after warm-up, and prints one JSON line with the decision mix and the
throughput. FLOPs follow the dense convention 4 B H Nq Nk D (halved under
causal masking); low-rank heads add their projection and use r for Q K^T.
The gpt2_small workload times a 12-layer, 768-wide decoder forward built from
AdaAttention (the reference's examples/transformer_integration.py shape) and
reports tokens/s. The rsvd workload times the randomized SVD of the low-rank
workload's K heads (64 fp32 matrices of 8192 x 128, rank 64).
"""

from __future__ import annotations

import argparse
import json
import math
import sys

import torch

from . import AdaAttention, PrecisionMode, analyze, attention_forward
from .core import possible_precisions
from .host_model import AdaptiveTransformer
from .workloads import GPT2_SMALL, WORKLOADS, make_qkv, make_token_ids


def _time(fn, steps: int, warmup: int = 3) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def adaptive_workload(name: str, steps: int, allow_fp8: bool = False, fp8_mode: str = "e4m3") -> dict:
    w = WORKLOADS[name]
    dev = torch.device("cuda:0")
    q, k, v = make_qkv(w, seed=0, device="cuda")
    d = w.head_dim
    scale = 1.0 / math.sqrt(d)
    r = max(1, int(d * 0.5))
    g = torch.Generator().manual_seed(1)
    w_down = torch.empty(r, d)
    torch.nn.init.orthogonal_(w_down, generator=g)
    w_down = w_down.to(w.dtype).to(dev)
    pm = possible_precisions(True, PrecisionMode.FP16, allow_fp8)

    def step():
        t = analyze(q, k, scale=scale, allow_fp8=allow_fp8)
        attention_forward(q, k, v, scale=scale, causal=w.causal, table=t, w_down=w_down,
                          possible_mask=pm, low_rank_possible=True, fp8_mode=fp8_mode)
        return t

    table = step()
    torch.cuda.synchronize()
    ms = _time(step, steps)
    prec = table.precision.cpu().flatten().tolist()
    low = table.low_rank.cpu().flatten().tolist()
    names = ("FP32", "FP16", "BF16", "FP8", "AUTO")
    mix = {}
    flops = 0.0
    half = 0.5 if w.causal else 1.0
    n = w.seq
    for p, lo in zip(prec, low):
        key = ("L-" if lo else "D-") + names[p]
        mix[key] = mix.get(key, 0) + 1
        if lo:
            flops += (2 * n * n * r + 2 * n * n * d) * half + 4 * n * d * r
        else:
            flops += 4 * n * n * d * half
    return {"workload": name, "shape": f"B{w.batch} H{w.heads} N{n} D{d} {str(w.dtype)[6:]}"
            + (" causal" if w.causal else ""), "allow_fp8": allow_fp8, "fp8_mode": fp8_mode,
            "decisions": mix, "ms": ms, "tflops": flops / (ms * 1e-3) / 1e12,
            "dense_equiv_tflops": w.dense_flops() / (ms * 1e-3) / 1e12,
            "tokens_per_s": w.tokens / (ms * 1e-3)}


def gpt2_workload(steps: int) -> dict:
    c = GPT2_SMALL
    dev = torch.device("cuda:0")
    torch.manual_seed(0)
    model = AdaptiveTransformer(vocab_size=c["vocab"], embed_dim=c["embed_dim"],
                                num_heads=c["num_heads"], num_layers=c["num_layers"],
                                ff_dim=c["ff_dim"], max_seq_len=c["seq"], dropout=0.0)
    model.init_gpt2_weights(std=0.02)
    for m in model.modules():
        if isinstance(m, AdaAttention):
            m.config.enable_nan_check = False
    model = model.to(dev).to(torch.bfloat16).eval()
    ids = make_token_ids(c["batch"], c["seq"], c["vocab"], seed=0, device="cuda")

    def step():
        with torch.no_grad():
            return model(ids)

    ms = _time(step, steps, warmup=2)
    stats = model.get_attention_statistics()
    tokens = c["batch"] * c["seq"]
    return {"workload": "gpt2_small", "shape": f"B{c['batch']} N{c['seq']} E{c['embed_dim']} "
            f"H{c['num_heads']} L{c['num_layers']} bf16", "ms": ms,
            "tokens_per_s": tokens / (ms * 1e-3),
            "attention_precision_layer0": stats[0]["precision_distribution"],
            "low_rank_ratio_layer0": stats[0]["low_rank_ratio"]}


def rsvd_workload(steps: int, n_power: int) -> dict:
    """Randomized SVD of the K heads of the low-rank workload: 64 fp32
    matrices of 8192 x 128, rank 64 (k = 74), one sketch per head."""
    from .linalg import randomized_svd, sketch_width
    w = WORKLOADS["low_rank_mix"]
    _, k, _ = make_qkv(w, seed=0, device="cuda")
    a = k.float().reshape(-1, w.seq, w.head_dim).contiguous()
    rank = w.head_dim // 2
    kw = sketch_width(rank, w.seq, w.head_dim)
    g = torch.Generator(device="cuda").manual_seed(0)
    omega = torch.randn(a.shape[0], w.head_dim, kw, device="cuda", generator=g)

    def step():
        return randomized_svd(a, rank, num_power_iterations=n_power, omega=omega)

    ms = _time(step, steps)
    passes = 2 + 2 * n_power  # A is read by A Omega, each power step (twice) and Q^T A
    return {"workload": "rsvd_k_heads", "shape": f"{a.shape[0]} x {w.seq} x {w.head_dim} fp32",
            "rank": rank, "sketch": kw, "n_power": n_power, "ms": ms,
            "a_passes": passes, "a_gbs": passes * a.numel() * 4 / (ms * 1e-3) / 1e9,
            "matrices_per_s": a.shape[0] / (ms * 1e-3)}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--workload", default="all",
                    choices=["all", "adaptive_mix", "low_rank_mix", "precision_mix", "gpt2_small", "rsvd"])
    ap.add_argument("--steps", type=int, default=10)
    args = ap.parse_args(argv)
    todo = ["adaptive_mix", "low_rank_mix", "precision_mix", "gpt2_small", "rsvd"] \
        if args.workload == "all" else [args.workload]
    for name in todo:
        if name == "rsvd":
            for n_power in (1, 2):
                print(json.dumps(rsvd_workload(args.steps, n_power)), flush=True)
        elif name == "gpt2_small":
            print(json.dumps(gpt2_workload(args.steps)), flush=True)
        elif name == "precision_mix":
            for allow in (False, True):
                print(json.dumps(adaptive_workload(name, args.steps, allow_fp8=allow)), flush=True)
        else:
            print(json.dumps(adaptive_workload(name, args.steps)), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
