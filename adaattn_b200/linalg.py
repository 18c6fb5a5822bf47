"""Randomized truncated SVD on the GPU, mirroring adaattn.linalg.low_rank.

``randomized_svd`` has the reference's signature and return convention
(src/adaattn/linalg/low_rank.py:56-109): A [..., m, n] -> U [..., m, rank],
S [..., rank] (descending), Vh [..., rank, n], with the sketch width
k = min(rank + num_oversampling, min(m, n)). Two keyword extensions make it
testable against the reference on the same numbers: ``omega`` passes the
Gaussian sketch [..., n, k] (drawn with ``torch.randn`` like low_rank.py:83
when omitted) and ``generator`` seeds that draw.

The work runs in libadaattn_b200's ``ada_rsvd``: panel GEMMs on the tcgen05
tensor cores (tf32 head/tail split), fp64 Gram matrices, CholeskyQR2 in place
of Householder QR, and an fp64 Jacobi eigen-solve of B B^T for the small SVD.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch

from . import _lib
from .config import ShapeError


def sketch_width(rank: int, m: int, n: int, num_oversampling: int = 10) -> int:
    """k of low_rank.py:80."""
    return min(rank + num_oversampling, min(m, n))


def randomized_svd(A: torch.Tensor, rank: int, num_oversampling: int = 10,
                   num_power_iterations: int = 2, *, omega: Optional[torch.Tensor] = None,
                   generator: Optional[torch.Generator] = None
                   ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Truncated SVD of A by the randomized range finder (low_rank.py:56-109)."""
    if A.dim() < 2:
        raise ShapeError(f"A must have at least 2 dimensions, got {A.dim()}")
    if not A.is_cuda:
        raise ValueError("randomized_svd runs on a CUDA tensor")
    if A.dtype != torch.float32:
        raise TypeError(f"randomized_svd takes float32 input, got {A.dtype}")
    *batch, m, n = A.shape
    k = sketch_width(rank, m, n, num_oversampling)
    if rank < 1 or rank > k:
        raise ValueError(f"rank {rank} outside [1, {k}]")
    a3 = A.reshape(-1, m, n)
    nb = a3.shape[0]
    if omega is None:
        omega = torch.randn(*batch, n, k, device=A.device, dtype=A.dtype, generator=generator)
    if tuple(omega.shape) != (*batch, n, k):
        raise ShapeError(f"omega must be {(*batch, n, k)}, got {tuple(omega.shape)}")
    om3 = omega.to(device=A.device, dtype=torch.float32).reshape(nb, n, k)
    u = torch.empty(nb, m, rank, device=A.device, dtype=torch.float32)
    s = torch.empty(nb, rank, device=A.device, dtype=torch.float32)
    vh = torch.empty(nb, rank, n, device=A.device, dtype=torch.float32)
    if nb == 0:
        return u.reshape(*batch, m, rank), s.reshape(*batch, rank), vh.reshape(*batch, rank, n)
    lib = _lib.load()
    ta, tom = _lib.tensor(a3), _lib.tensor(om3)
    tu, ts, tvh = _lib.tensor(u), _lib.tensor(s), _lib.tensor(vh)
    ws_bytes = int(lib.ada_rsvd_workspace_bytes(ta, tom, int(rank)))
    if ws_bytes == 0:
        _lib.check(-1, "ada_rsvd_workspace_bytes")
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=A.device)
    with torch.cuda.device(A.device):
        rc = lib.ada_rsvd(ta, tom, int(rank), int(num_power_iterations), tu, ts, tvh,
                          ws.data_ptr(), ws.numel(), _lib.stream_ptr(A.device))
    _lib.check(rc, "ada_rsvd")
    return u.reshape(*batch, m, rank), s.reshape(*batch, rank), vh.reshape(*batch, rank, n)


def low_rank_approx(A: torch.Tensor, rank: int, method: str = "randomized", *,
                    omega: Optional[torch.Tensor] = None,
                    generator: Optional[torch.Generator] = None) -> torch.Tensor:
    """U diag(S) Vh from ``randomized_svd`` (low_rank.py:156-181, method
    "randomized"); the reconstruction product is a plain torch matmul."""
    if method != "randomized":
        raise ValueError("only method='randomized' runs on this path")
    u, s, vh = randomized_svd(A, rank, omega=omega, generator=generator)
    return torch.matmul(u * s.unsqueeze(-2), vh)


__all__ = ["randomized_svd", "low_rank_approx", "sketch_width"]
