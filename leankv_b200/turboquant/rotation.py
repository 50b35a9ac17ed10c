"""Rotations of head vectors (prototype/turboquant/rotation.py).

Three families, all orthogonal (R^T R = I) and applied as x @ R^T:
  random_orthogonal    Q of the QR factorisation of a seeded Gaussian matrix, columns
                       signed by diag(R) (rotation.py:25-49)
  hadamard             the Sylvester Walsh-Hadamard matrix / sqrt(d) (rotation.py:52-76)
  randomized_hadamard  H diag(s) with seeded s in {-1, +1} (rotation.py:79-106)
The matrices are generated on the host with the same torch RNG calls as the
prototype, so a seed gives the same matrix.  On CUDA tensors the two Hadamard
families are applied with the fused butterfly kernel (x @ (H diag s)^T =
FWHT(x * s)); dense matrices go through a GEMM.
"""
from __future__ import annotations

import math
from typing import Optional

import torch

from .. import ops


def _require_pow2(d: int) -> None:
    if d <= 0 or d & (d - 1):
        raise ValueError(f"d must be power of 2, got {d}")


def random_orthogonal(d: int, seed: Optional[int] = None) -> torch.Tensor:
    """d x d orthogonal matrix from the QR factorisation of a seeded N(0, 1) matrix."""
    if seed is not None:
        torch.manual_seed(seed)
    gauss = torch.randn(d, d)
    q, r = torch.linalg.qr(gauss)
    return q * torch.sign(torch.diag(r)).unsqueeze(0)


def hadamard_matrix(d: int) -> torch.Tensor:
    """Normalized Sylvester Walsh-Hadamard matrix of order d (a power of two)."""
    _require_pow2(d)
    h = torch.ones(1, 1)
    while h.shape[0] < d:
        h = torch.cat([torch.cat([h, h], 1), torch.cat([h, -h], 1)], 0)
    return h / math.sqrt(d)


def randomized_hadamard(d: int, seed: Optional[int] = None) -> torch.Tensor:
    """H diag(s): columns of the normalized Hadamard matrix signed by seeded s in {-1, +1}."""
    if seed is not None:
        torch.manual_seed(seed)
    h = hadamard_matrix(d)
    s = (torch.randint(0, 2, (d,)) * 2 - 1).float()
    return h * s.unsqueeze(0)


def fast_hadamard_transform(x: torch.Tensor) -> torch.Tensor:
    """Normalized Walsh-Hadamard transform over the last dimension (butterfly, CUDA kernel)."""
    d = x.shape[-1]
    _require_pow2(d)
    if not x.is_cuda:
        raise ValueError("leankv_b200.turboquant runs on CUDA tensors")
    y = x.to(torch.float32).contiguous().clone()
    ops.hadamard_(y, d)
    return y.to(x.dtype) if x.dtype != torch.float32 else y


def apply_rotation(x: torch.Tensor, rotation: torch.Tensor) -> torch.Tensor:
    """x @ R^T over the last dimension."""
    return x @ rotation.T


def apply_inverse_rotation(x: torch.Tensor, rotation: torch.Tensor) -> torch.Tensor:
    """x @ R (R^-1 = R^T for an orthogonal R)."""
    return x @ rotation


def generate_per_layer_rotations(n_layers: int, head_dim: int, strategy: str = "randomized_hadamard",
                                 base_seed: int = 42) -> list[torch.Tensor]:
    """One rotation per layer, layer l seeded with base_seed + l (the Hadamard matrix ignores seeds)."""
    makers = {
        "random_orthogonal": lambda s: random_orthogonal(head_dim, seed=s),
        "hadamard": lambda s: hadamard_matrix(head_dim),
        "randomized_hadamard": lambda s: randomized_hadamard(head_dim, seed=s),
    }
    if strategy not in makers:
        raise ValueError(f"Unknown rotation strategy: {strategy}. Choose from {list(makers)}")
    return [makers[strategy](base_seed + layer) for layer in range(n_layers)]


def hadamard_signs(rotation: torch.Tensor) -> Optional[torch.Tensor]:
    """s with R = H diag(s) when R is a (randomized) normalized Hadamard matrix, else None.

    H's first row is constant, so s_j = sign(R[0, j]); R is accepted only when it
    equals H diag(s) exactly (entries +-1/sqrt(d) in the Sylvester sign pattern).
    """
    d = rotation.shape[-1]
    if d & (d - 1) or rotation.shape != (d, d):
        return None
    r = rotation.detach().float().cpu()
    s = torch.sign(r[0])
    if torch.any(s == 0):
        return None
    if not torch.equal(r, hadamard_matrix(d) * s.unsqueeze(0)):
        return None
    return s
