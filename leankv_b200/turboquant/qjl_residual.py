"""1-bit QJL residual correction (prototype/turboquant/qjl_residual.py).

After scalar quantization the residual r = x - Q(x) is stored as sign bits
(r >= 0, packed 8 per byte with bit i of byte j holding element 8j + i) plus
the mean |r| of the vector; decoding adds (2 sign - 1) * mean|r|.  The fused
GPU encoder computes these inside tq_proto_encode_cuda; the helpers below are
the tensor-level functions of the prototype's interface.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

_BITS = (1, 2, 4, 8, 16, 32, 64, 128)


def compute_residual(original: torch.Tensor, reconstructed: torch.Tensor) -> torch.Tensor:
    return original - reconstructed


def encode_qjl_residual(residual: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """(sign bits as bool, mean |residual| over the last dimension)."""
    return residual >= 0, residual.abs().mean(dim=-1)


def decode_qjl_residual(signs: torch.Tensor, mean_abs: torch.Tensor) -> torch.Tensor:
    return (signs.float() * 2 - 1) * mean_abs.unsqueeze(-1)


def pack_signs(signs: torch.Tensor) -> torch.Tensor:
    """bool (..., d) -> uint8 (..., d/8), bit i of byte j = element 8j + i."""
    d = signs.shape[-1]
    if d % 8:
        raise ValueError(f"Dimension must be divisible by 8, got {d}")
    w = torch.tensor(_BITS, dtype=torch.uint8, device=signs.device)
    return (signs.view(*signs.shape[:-1], d // 8, 8).to(torch.uint8) * w).sum(dim=-1).to(torch.uint8)


def unpack_signs(packed: torch.Tensor, d: int) -> torch.Tensor:
    w = torch.tensor(_BITS, dtype=torch.uint8, device=packed.device)
    return ((packed.unsqueeze(-1) & w) > 0).view(*packed.shape[:-1], d)


class QJLResidual:
    """Sign + mean-magnitude residual codec."""

    def encode(self, residual: torch.Tensor, pack: bool = True) -> Tuple[torch.Tensor, torch.Tensor]:
        signs, mean_abs = encode_qjl_residual(residual)
        return (pack_signs(signs) if pack else signs), mean_abs

    def decode(self, signs: torch.Tensor, mean_abs: torch.Tensor, d: Optional[int] = None,
               packed: bool = True) -> torch.Tensor:
        if packed:
            if d is None:
                raise ValueError("Must provide d when signs are packed")
            signs = unpack_signs(signs, d)
        return decode_qjl_residual(signs, mean_abs)

    def memory_bits_per_element(self, d: int) -> float:
        return 1.0 + 32.0 / d
