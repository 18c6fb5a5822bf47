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
