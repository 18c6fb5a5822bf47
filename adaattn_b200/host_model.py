"""The decoder that hosts AdaAttention in the GPT-2-small workload.

Same architecture and constructor arguments as the reference's
examples/transformer_integration.py:12-141 (post-LayerNorm blocks, GELU
feed-forward, learned positions, head tied to the token embedding,
non-causal attention), with this package's AdaAttention inside. Used to
measure the module-level throughput of the path; the model itself is not part
of the hot path.
"""

from __future__ import annotations

import torch
import torch.nn as nn

from . import core
from .attention import AdaAttention


def _norm(norm: nn.LayerNorm, x: torch.Tensor) -> torch.Tensor:
    """The block's LayerNorm: one ada_layer_norm launch for 16-bit inputs
    without autograd, nn.LayerNorm (with its backward) otherwise."""
    if (x.is_cuda and x.dtype in (torch.bfloat16, torch.float16) and norm.elementwise_affine
            and norm.weight.dtype == x.dtype and len(norm.normalized_shape) == 1
            and x.shape[-1] % 8 == 0 and x.shape[-1] <= 2048
            and not (torch.is_grad_enabled() and (x.requires_grad or norm.weight.requires_grad))):
        return core.layer_norm(x, norm.weight, norm.bias, norm.eps)
    return norm(x)


class TransformerBlock(nn.Module):
    """examples/transformer_integration.py:12-58."""

    def __init__(self, embed_dim: int, num_heads: int, ff_dim: int, dropout: float = 0.1,
                 enable_adaptive_rank: bool = True, enable_adaptive_precision: bool = True, **attn_kwargs):
        super().__init__()
        self.attention = AdaAttention(embed_dim=embed_dim, num_heads=num_heads, dropout=dropout,
                                      enable_adaptive_rank=enable_adaptive_rank,
                                      enable_adaptive_precision=enable_adaptive_precision, **attn_kwargs)
        self.norm1 = nn.LayerNorm(embed_dim)
        self.norm2 = nn.LayerNorm(embed_dim)
        self.ff = nn.Sequential(nn.Linear(embed_dim, ff_dim), nn.GELU(), nn.Dropout(dropout),
                                nn.Linear(ff_dim, embed_dim), nn.Dropout(dropout))

    def forward(self, x: torch.Tensor, attention_mask=None) -> torch.Tensor:
        if self._fused(x):
            # The same sums with the residual adds, the biases and the GELU in
            # the epilogues of the tensor-core layers (core.linear).
            x = _norm(self.norm1, self.attention.forward_with_residual(x, attention_mask))
            up, down = self.ff[0], self.ff[3]
            f = core.linear(x, up.weight, up.bias, activation="gelu")
            return _norm(self.norm2, core.linear(f, down.weight, down.bias, residual=x))
        attn_out, _ = self.attention(x, x, x, attention_mask=attention_mask)
        x = self.norm1(x + attn_out)
        return self.norm2(x + self.ff(x))

    def _fused(self, x: torch.Tensor) -> bool:
        dropout_off = not self.training or all(
            m.p == 0 for m in (self.ff[2], self.ff[4], self.attention.resid_dropout))
        return (x.is_cuda and x.dtype in (torch.bfloat16, torch.float16) and dropout_off
                and isinstance(self.ff[1], nn.GELU) and self.ff[1].approximate == "none")


class AdaptiveTransformer(nn.Module):
    """examples/transformer_integration.py:61-141."""

    def __init__(self, vocab_size: int, embed_dim: int, num_heads: int, num_layers: int, ff_dim: int,
                 max_seq_len: int = 512, dropout: float = 0.1, enable_adaptive_rank: bool = True,
                 enable_adaptive_precision: bool = True, **attn_kwargs):
        super().__init__()
        self.embed_dim = embed_dim
        self.max_seq_len = max_seq_len
        self.token_embedding = nn.Embedding(vocab_size, embed_dim)
        self.position_embedding = nn.Embedding(max_seq_len, embed_dim)
        self.embed_dropout = nn.Dropout(dropout)
        self.blocks = nn.ModuleList([
            TransformerBlock(embed_dim, num_heads, ff_dim, dropout, enable_adaptive_rank,
                             enable_adaptive_precision, **attn_kwargs)
            for _ in range(num_layers)])
        self.norm = nn.LayerNorm(embed_dim)
        self.head = nn.Linear(embed_dim, vocab_size, bias=False)
        self.head.weight = self.token_embedding.weight
        nn.init.normal_(self.token_embedding.weight, std=0.02)
        nn.init.normal_(self.position_embedding.weight, std=0.02)

    def init_gpt2_weights(self, std: float = 0.02) -> None:
        """Every weight N(0, std), biases zero, LayerNorms identity."""
        for m in self.modules():
            if isinstance(m, (nn.Linear, nn.Embedding)):
                nn.init.normal_(m.weight, std=std)
                if getattr(m, "bias", None) is not None:
                    nn.init.zeros_(m.bias)
            elif isinstance(m, nn.LayerNorm):
                nn.init.ones_(m.weight)
                nn.init.zeros_(m.bias)

    def forward(self, input_ids: torch.Tensor, attention_mask=None) -> torch.Tensor:
        _, seq_len = input_ids.shape
        pos = torch.arange(seq_len, device=input_ids.device).unsqueeze(0)
        x = self.embed_dropout(self.token_embedding(input_ids) + self.position_embedding(pos))
        for block in self.blocks:
            x = block(x, attention_mask=attention_mask)
        return self._logits(_norm(self.norm, x))

    def _logits(self, h: torch.Tensor) -> torch.Tensor:
        """The tied head. A vocabulary that is not a multiple of 64 (50257)
        sends cuBLAS to a slow unaligned GEMM on the GPU, so the weight is
        zero-padded to the next multiple of 64 rows (kept until the weight
        changes) and the logits are returned as a view of the first
        `vocab_size` columns: the values of the plain Linear, rows 64-aligned
        in memory (`reshape(-1, vocab_size)` and row-wise ops work as on a
        dense tensor; copying them out would move 1.6 GB at batch 16 x 1024)."""
        w = self.head.weight
        pad = (-w.shape[0]) % 64
        if not h.is_cuda or pad == 0:
            return self.head(h)
        key = (w.data_ptr(), w._version, w.dtype, w.device)
        if getattr(self, "_head_pad_key", None) != key:
            self._head_pad = torch.nn.functional.pad(w.detach(), (0, 0, 0, pad))
            self._head_pad_key = key
        wp = self._head_pad if not torch.is_grad_enabled() else torch.nn.functional.pad(w, (0, 0, 0, pad))
        return torch.matmul(h, wp.t())[..., : w.shape[0]]

    def get_attention_statistics(self):
        stats = []
        for i, block in enumerate(self.blocks):
            s = block.attention.get_statistics()
            s["layer"] = i
            stats.append(s)
        return stats
