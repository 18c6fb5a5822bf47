"""Helpers shared by the tests that read the golden fixtures."""

from __future__ import annotations

import os

import torch

from adaattn_b200.workloads import WORKLOADS, make_qkv

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

PREC_CODE = {"FP32": 0, "FP16": 1, "BF16": 2, "FP8": 3, "AUTO": 4}

CASE_NAMES = [
    "adaptive_mix", "precision_mix_small", "precision_mix_small_fp8",
    "low_rank_small", "dense_bf16_small", "edge_short_causal",
    "edge_cross_masked",
]


def load(name: str) -> dict:
    return torch.load(os.path.join(GOLDEN, f"{name}.pt"), weights_only=True)


def inputs(rec: dict, device: str = "cpu"):
    """Regenerate the fixture's (q, k, v) on the host and check its checksum."""
    w = WORKLOADS[rec["workload"]].scaled(batch=rec["batch"],
                                          heads=rec["heads"], seq=rec["seq_k"])
    q, k, v = make_qkv(w, seed=0)
    q = q[:, :, :rec["seq_q"]].contiguous()
    sums = [float(t.double().sum().item()) for t in (q, k, v)]
    for got, want in zip(sums, rec["checksum"]):
        assert abs(got - want) <= 1e-9 * max(1.0, abs(want)), \
            "seeded input generator drifted from the fixture"
    return q.to(device), k.to(device), v.to(device)


def oracle_config(rec: dict):
    from oracle import OracleConfig
    kw = rec["module_kwargs"]
    cfg = OracleConfig(causal=rec["causal"])
    if "allow_fp8" in kw:
        cfg.allow_fp8 = kw["allow_fp8"] == "True"
    if "enable_adaptive_rank" in kw:
        cfg.enable_adaptive_rank = kw["enable_adaptive_rank"] == "True"
    if "enable_adaptive_precision" in kw:
        cfg.enable_adaptive_precision = kw["enable_adaptive_precision"] == "True"
    if "default_precision" in kw:
        cfg.default_precision = PREC_CODE[kw["default_precision"]]
    return cfg


def module_kwargs(rec: dict) -> dict:
    """Fixture module kwargs as AdaAttention constructor arguments."""
    from adaattn_b200 import PrecisionMode
    out = {}
    for k, v in rec["module_kwargs"].items():
        if k == "default_precision":
            out[k] = PrecisionMode[v]
        elif v in ("True", "False"):
            out[k] = v == "True"
        else:
            out[k] = v
    return out


# ---------------------------------------------------------------------------
# Seeded inputs of the kernel-op and transformer fixtures (the fixtures store
# only the reference's outputs; both sides regenerate the inputs from here).
# ---------------------------------------------------------------------------
KERNEL_OP_DTYPES = (torch.float32, torch.float16, torch.bfloat16)


def kernel_op_inputs() -> dict:
    """{dtype name: (q, k, v)} [B=1, N=150, H=2, D=64] (two 128-row tiles, the
    second ragged), drawn in a fixed order."""
    g = torch.Generator().manual_seed(21)
    out = {}
    for dtype in KERNEL_OP_DTYPES:
        q = (torch.randn(1, 150, 2, 64, generator=g) * 0.5).to(dtype)
        k = (torch.randn(1, 150, 2, 64, generator=g) * 0.5).to(dtype)
        v = torch.randn(1, 150, 2, 64, generator=g).to(dtype)
        out[str(dtype).replace("torch.", "")] = (q, k, v)
    return out


TRANSFORMER = dict(vocab_size=500, embed_dim=128, num_heads=2, num_layers=2, ff_dim=256,
                   max_seq_len=64)


def transformer_state(template: dict, seed: int = 77) -> dict:
    """Weights for the small AdaptiveTransformer as the GPT-2-small workload
    initialises them: every Linear / Embedding weight N(0, 0.02), biases 0,
    LayerNorm weight 1 and bias 0; buffers (call counters) are left alone.
    ``template`` is a state dict giving the names and shapes; values are
    drawn in sorted-name order, so any module with these names gets the
    same weights. The output head is tied to the token embedding, so
    ``head.weight`` is left out (loading it would overwrite the embedding)."""
    g = torch.Generator().manual_seed(seed)
    out = {}
    for name in sorted(template):
        t = template[name]
        if name == "head.weight" or not t.is_floating_point() or name.split(".")[-1].startswith("_"):
            continue
        if "norm" in name:
            val = torch.ones(t.shape) if name.endswith("weight") else torch.zeros(t.shape)
        elif name.endswith("bias"):
            val = torch.zeros(t.shape)
        else:
            val = torch.randn(t.shape, generator=g) * 0.02
        out[name] = val
    return out


def transformer_ids(seed: int = 78) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, TRANSFORMER["vocab_size"], (2, TRANSFORMER["max_seq_len"]), generator=g)
