"""Seeded synthetic inputs for the five AdaAttn workloads.

No public dataset is named for this path, so every workload is synthetic with
the shapes and value distributions the workload description gives. All
generators draw from an explicit ``torch.Generator`` so a seed reproduces the
same tensors on the host and on the device it was drawn for.

Workloads (tensors are [B, H, N, D] unless noted):
  adaptive_mix   B2 H8 N512 D64 fp32, non-causal, per-head query temperature
                 exp(U[ln 0.25, ln 4]) so heads span high and low entropy.
  dense_bf16     B8 H32 N4096 D128 bf16 causal, iid N(0,1)/sqrt(D).
  low_rank_mix   B4 H16 N8192 D128 bf16 non-causal; heads [0, H/2) have
                 K = A B^T (A, B N(0,1) with inner rank 32) + 0.01 N(0,1),
                 the rest are full-rank N(0,1).
  precision_mix  B8 H32 N2048 D128 bf16 causal; each (b, h) draws a scale
                 from {0.1, 1, 10, 100} and Q, K, V are N(0,1) * scale.
  gpt2_small     token ids [16, 1024] uniform over a 50257 vocabulary for a
                 12-layer, 768-wide, 12-head decoder.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Dict, Optional, Tuple

import torch


@dataclass(frozen=True)
class Workload:
    name: str
    batch: int
    heads: int
    seq: int
    head_dim: int
    dtype: torch.dtype
    causal: bool
    kind: str
    extra: Dict[str, float] = field(default_factory=dict)

    def scaled(self, batch: Optional[int] = None, heads: Optional[int] = None,
               seq: Optional[int] = None) -> "Workload":
        return Workload(self.name, batch or self.batch, heads or self.heads,
                        seq or self.seq, self.head_dim, self.dtype, self.causal,
                        self.kind, dict(self.extra))

    @property
    def tokens(self) -> int:
        return self.batch * self.seq

    def dense_flops(self) -> float:
        """4 B H Nq Nk D, halved under causal masking (unmasked pairs only)."""
        f = 4.0 * self.batch * self.heads * self.seq * self.seq * self.head_dim
        return f * 0.5 if self.causal else f


WORKLOADS = {
    "adaptive_mix": Workload("adaptive_mix", 2, 8, 512, 64, torch.float32,
                             False, "temperature"),
    "dense_bf16": Workload("dense_bf16", 8, 32, 4096, 128, torch.bfloat16,
                           True, "iid_scaled"),
    "low_rank_mix": Workload("low_rank_mix", 4, 16, 8192, 128, torch.bfloat16,
                             False, "low_rank_keys"),
    "precision_mix": Workload("precision_mix", 8, 32, 2048, 128,
                              torch.bfloat16, True, "scale_mix"),
}

GPT2_SMALL = dict(vocab=50257, embed_dim=768, num_heads=12, num_layers=12,
                  ff_dim=3072, seq=1024, batch=16)


def _randn(shape, g, device):
    return torch.randn(*shape, generator=g, device=device, dtype=torch.float32)


def make_qkv(w: Workload, seed: int = 0, device: str = "cpu"
             ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Draw (q, k, v) for a workload on ``device`` with a seeded generator."""
    g = torch.Generator(device=device).manual_seed(seed)
    shape = (w.batch, w.heads, w.seq, w.head_dim)
    if w.kind == "temperature":
        q = _randn(shape, g, device)
        k = _randn(shape, g, device)
        v = _randn(shape, g, device)
        lo, hi = math.log(0.25), math.log(4.0)
        u = torch.rand(w.heads, generator=g, device=device)
        temp = torch.exp(lo + (hi - lo) * u)
        q = q * temp.view(1, -1, 1, 1)
    elif w.kind == "iid_scaled":
        s = 1.0 / math.sqrt(w.head_dim)
        q = _randn(shape, g, device) * s
        k = _randn(shape, g, device) * s
        v = _randn(shape, g, device) * s
    elif w.kind == "low_rank_keys":
        q = _randn(shape, g, device)
        v = _randn(shape, g, device)
        k = _randn(shape, g, device)
        half = w.heads // 2
        inner = 32
        a = _randn((w.batch, half, w.seq, inner), g, device)
        bm = _randn((w.batch, half, w.head_dim, inner), g, device)
        low = torch.matmul(a, bm.transpose(-2, -1))
        k[:, :half] = low + 0.01 * k[:, :half]
    elif w.kind == "scale_mix":
        choices = torch.tensor([0.1, 1.0, 10.0, 100.0], device=device)
        idx = torch.randint(0, 4, (w.batch, w.heads), generator=g,
                            device=device)
        sc = choices[idx].view(w.batch, w.heads, 1, 1)
        q = _randn(shape, g, device) * sc
        k = _randn(shape, g, device) * sc
        v = _randn(shape, g, device) * sc
    else:
        raise ValueError(f"unknown workload kind {w.kind}")
    return q.to(w.dtype), k.to(w.dtype), v.to(w.dtype)


def scale_mix_choices(w: Workload, seed: int = 0, device: str = "cpu"
                      ) -> torch.Tensor:
    """The per-(b, h) scale drawn by ``make_qkv`` for a scale_mix workload."""
    g = torch.Generator(device=device).manual_seed(seed)
    choices = torch.tensor([0.1, 1.0, 10.0, 100.0], device=device)
    idx = torch.randint(0, 4, (w.batch, w.heads), generator=g, device=device)
    return choices[idx]


def make_token_ids(batch: int, seq: int, vocab: int, seed: int = 0,
                   device: str = "cpu") -> torch.Tensor:
    g = torch.Generator(device=device).manual_seed(seed)
    return torch.randint(0, vocab, (batch, seq), generator=g, device=device)
