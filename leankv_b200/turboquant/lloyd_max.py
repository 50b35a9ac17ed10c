"""Lloyd-Max codebooks of the rotated-coordinate distribution (prototype/turboquant/lloyd_max.py).

After an orthogonal rotation each coordinate of a unit vector in R^d follows
f(x) ~ (1 - x^2)^((d-3)/2) on (-1, 1), close to N(0, 1/d) for d >= 32.  The
codebook is the Lloyd-Max quantizer of that density: levels start evenly spaced
over the support, then alternate boundaries = midpoints of adjacent levels and
levels = E[X | bin] (adaptive quadrature), until the mean squared error changes
by less than tol.  The iteration, its initialisation, support (+-4 sigma for the
Gaussian approximation) and stopping rule follow lloyd_max.py:57-140, so the
same (bits, dim) yields the prototype's codebook.  Codebooks are computed once
per (levels, dim) on the host and cached.
"""
from __future__ import annotations

import math
from typing import Tuple, Union

import numpy as np
import torch

BITS_TO_LEVELS = {2: 4, 2.5: 6, 3: 8, 3.125: 9, 3.5: 12, 4: 16}
SUPPORTED_BITS = sorted(BITS_TO_LEVELS)

_codebook_cache: dict = {}


def n_levels_for(bits: Union[int, float]) -> int:
    return BITS_TO_LEVELS[bits] if bits in BITS_TO_LEVELS else round(2 ** bits)


def beta_pdf(x: float, d: int) -> float:
    """Density of one coordinate of a uniform point on the unit sphere in R^d."""
    from scipy.special import gamma
    if abs(x) >= 1.0:
        return 0.0
    c = gamma(d / 2) / (np.sqrt(np.pi) * gamma((d - 1) / 2))
    return c * (1 - x ** 2) ** ((d - 3) / 2)


def gaussian_pdf(x: float, variance: float) -> float:
    """Density of N(0, variance)."""
    return np.exp(-x ** 2 / (2 * variance)) / np.sqrt(2 * np.pi * variance)


def lloyd_max_1d(pdf_func, support: Tuple[float, float], n_levels: int, max_iter: int = 200,
                 tol: float = 1e-10) -> Tuple[np.ndarray, np.ndarray, float]:
    """Lloyd-Max quantizer of a 1-D density on `support`: (levels, boundaries, mse)."""
    from scipy import integrate
    a, b = support
    levels = np.linspace(a + (b - a) / (2 * n_levels), b - (b - a) / (2 * n_levels), n_levels)
    prev = float("inf")
    mse = prev
    for _ in range(max_iter):
        cuts = np.concatenate([[a], (levels[:-1] + levels[1:]) / 2, [b]])
        centroids = np.zeros(n_levels)
        for i in range(n_levels):
            mass, _ = integrate.quad(pdf_func, cuts[i], cuts[i + 1])
            first, _ = integrate.quad(lambda t: t * pdf_func(t), cuts[i], cuts[i + 1])
            centroids[i] = first / mass if mass > 1e-15 else levels[i]
        levels = centroids
        mse = 0.0
        for i in range(n_levels):
            part, _ = integrate.quad(lambda t: (t - levels[i]) ** 2 * pdf_func(t), cuts[i], cuts[i + 1])
            mse += part
        if abs(prev - mse) < tol:
            break
        prev = mse
    return levels, (levels[:-1] + levels[1:]) / 2, mse


def compute_codebook(bits: Union[int, float], dim: int = 128,
                     use_gaussian_approx: bool = True) -> Tuple[np.ndarray, np.ndarray, float]:
    """Lloyd-Max codebook for `bits` (2, 2.5, 3, 3.125, 3.5, 4 or 2**bits levels) at head_dim `dim`."""
    n = n_levels_for(bits)
    if use_gaussian_approx and dim >= 32:
        var = 1.0 / dim
        sd = np.sqrt(var)
        return lloyd_max_1d(lambda t: gaussian_pdf(t, var), (-4 * sd, 4 * sd), n)
    return lloyd_max_1d(lambda t: beta_pdf(t, dim), (-1.0, 1.0), n)


def get_precomputed_codebook(bits: Union[int, float], dim: int = 128) -> Tuple[torch.Tensor, torch.Tensor]:
    """Cached (levels, boundaries) float32 tensors for (bits, dim)."""
    key = (n_levels_for(bits), dim)
    if key not in _codebook_cache:
        levels, bounds, _ = compute_codebook(bits, dim)
        _codebook_cache[key] = (torch.tensor(levels, dtype=torch.float32), torch.tensor(bounds, dtype=torch.float32))
    return _codebook_cache[key]


def quantize_scalar(x: torch.Tensor, boundaries: torch.Tensor) -> torch.Tensor:
    """Codebook indices #{b : boundaries[b] < x} (torch.bucketize, right=False)."""
    return torch.bucketize(x, boundaries)


def dequantize_scalar(indices: torch.Tensor, levels: torch.Tensor) -> torch.Tensor:
    """levels[indices]."""
    return levels[indices]
