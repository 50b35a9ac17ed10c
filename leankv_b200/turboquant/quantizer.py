"""TurboQuantizer: rotation + Lloyd-Max scalar quantization + optional QJL residual
(prototype/turboquant/quantizer.py:45-247), running on the GPU.

quantize() makes one launch of the fused per-vector encoder
(tq_proto_encode_cuda): Hadamard-family rotations, the per-vector L2 norm (of
the unrotated vector) or per-group max |x|, normalisation by (scale + 1e-10),
the codebook search (torch.bucketize semantics), and the QJL sign bits and mean
|residual|.  Dense random-orthogonal rotations are applied by a GEMM first.
dequantize() is one launch of the fused decoder (tq_proto_decode_cuda),
including the inverse Hadamard rotation when requested.  Inputs are computed
in float32 (bf16 / fp16 inputs are widened exactly).
"""
from __future__ import annotations

import ctypes as C
import math
from typing import NamedTuple, Optional, Union

import torch

from .. import _lib as L
from ..ops import _DTYPES, _stream
from .lloyd_max import BITS_TO_LEVELS, get_precomputed_codebook
from .qjl_residual import QJLResidual
from .rotation import apply_rotation, generate_per_layer_rotations, hadamard_signs

SUPPORTED_DIMS = (32, 64, 128, 256)


class QuantizedKV(NamedTuple):
    """Packed per-vector representation."""
    indices: torch.Tensor                 # uint8 codebook indices, (..., head_dim)
    qjl_signs: Optional[torch.Tensor]     # uint8 packed residual signs, (..., head_dim // 8)
    qjl_mean_abs: Optional[torch.Tensor]  # float32 mean |residual|, (...)
    norms: torch.Tensor                   # float32 per-vector norms (...) or per-group max (..., n_groups)


def _f32_array(t: torch.Tensor):
    vals = [float(v) for v in t.detach().cpu().reshape(-1)]
    return (C.c_float * max(len(vals), 1))(*vals)


class TurboQuantizer:
    """Per-layer rotation + Lloyd-Max codebook (+ QJL) quantizer of head vectors on a CUDA device."""

    def __init__(self, n_layers: int, head_dim: int, bits: Union[int, float] = 3, group_size: Optional[int] = None,
                 rotation_strategy: str = "randomized_hadamard", use_qjl: bool = True, seed: int = 42,
                 device: str = "cuda"):
        self.n_layers = n_layers
        self.head_dim = head_dim
        self.bits = bits
        self.group_size = min(group_size, head_dim) if group_size is not None else head_dim
        self.use_qjl = use_qjl
        self.device = device
        if head_dim % self.group_size != 0:
            raise AssertionError(f"head_dim ({head_dim}) must be divisible by group_size ({self.group_size})")
        self.n_groups = head_dim // self.group_size
        dev = torch.device(device)
        if dev.type != "cuda":
            raise ValueError("leankv_b200.turboquant runs on CUDA devices (device='cuda')")
        if head_dim not in SUPPORTED_DIMS:
            raise ValueError(f"head_dim {head_dim} not supported (supported: {SUPPORTED_DIMS})")
        if self.group_size & (self.group_size - 1):
            raise ValueError(f"group_size {self.group_size} must be a power of two")
        self.rotation_strategy = rotation_strategy
        self.rotations = [r.to(dev) for r in generate_per_layer_rotations(n_layers, head_dim, rotation_strategy, seed)]
        # Hadamard-family rotations run in the fused kernel as FWHT(x * s)
        self._structured = []
        for r in self.rotations:
            s = hadamard_signs(r)
            self._structured.append((s is not None, None if s is None else s.to(dev).contiguous()))
        self.levels, self.boundaries = get_precomputed_codebook(bits, head_dim)
        self.levels = self.levels.to(dev)
        self.boundaries = self.boundaries.to(dev)
        self._levels_c = _f32_array(self.levels)
        self._bounds_c = _f32_array(self.boundaries)
        self._n_levels = int(self.levels.numel())
        self.qjl = QJLResidual() if use_qjl else None

    # ── encode / decode through the fused kernels ──
    def _encode(self, x: torch.Tensor, layer_idx: Optional[int], rotate: bool, group: int, qjl: bool) -> QuantizedKV:
        if not x.is_cuda:
            raise ValueError("leankv_b200.turboquant runs on CUDA tensors")
        if x.shape[-1] != self.head_dim:
            raise ValueError(f"last dimension {x.shape[-1]} != head_dim {self.head_dim}")
        if x.dtype not in _DTYPES:
            x = x.float()
        x = x.contiguous()
        lead = tuple(x.shape[:-1])
        rows = x.numel() // self.head_dim
        xr = None
        signs = None
        if rotate:
            structured, signs = self._structured[layer_idx]
            if not structured:
                xr = apply_rotation(x.float(), self.rotations[layer_idx]).contiguous()
        idx = torch.empty(*lead, self.head_dim, dtype=torch.uint8, device=x.device)
        norms = torch.empty(*lead, *(() if group >= self.head_dim else (self.head_dim // group,)),
                            dtype=torch.float32, device=x.device)
        qs = torch.empty(*lead, self.head_dim // 8, dtype=torch.uint8, device=x.device) if qjl else None
        qm = torch.empty(*lead, dtype=torch.float32, device=x.device) if qjl else None
        L.check(L.load().tq_proto_encode_cuda(
            x.data_ptr(), _DTYPES[x.dtype], xr.data_ptr() if xr is not None else None, rows, self.head_dim,
            int(rotate and xr is None), signs.data_ptr() if signs is not None else None, group, self._n_levels,
            self._levels_c, self._bounds_c, idx.data_ptr(), norms.data_ptr(),
            qs.data_ptr() if qs is not None else None, qm.data_ptr() if qm is not None else None, _stream(x)))
        return QuantizedKV(indices=idx, qjl_signs=qs, qjl_mean_abs=qm, norms=norms)

    def _decode(self, qkv: QuantizedKV, layer_idx: Optional[int], inverse_rotate: bool, group: int,
                use_qjl: bool) -> torch.Tensor:
        idx = qkv.indices.contiguous()
        if not idx.is_cuda:
            raise ValueError("leankv_b200.turboquant runs on CUDA tensors")
        rows = idx.numel() // self.head_dim
        y = torch.empty(idx.shape, dtype=torch.float32, device=idx.device)
        qs = qkv.qjl_signs.contiguous() if use_qjl and qkv.qjl_signs is not None else None
        qm = qkv.qjl_mean_abs.contiguous().float() if qs is not None else None
        structured, signs = (self._structured[layer_idx] if inverse_rotate else (True, None))
        L.check(L.load().tq_proto_decode_cuda(
            idx.data_ptr(), qkv.norms.contiguous().float().data_ptr(), rows, self.head_dim, group,
            qs.data_ptr() if qs is not None else None, qm.data_ptr() if qm is not None else None, self._n_levels,
            self._levels_c, int(inverse_rotate and structured), signs.data_ptr() if signs is not None else None,
            y.data_ptr(), _stream(idx)))
        if inverse_rotate and not structured:
            y = y @ self.rotations[layer_idx]
        return y

    # ── prototype interface ──
    def quantize(self, x: torch.Tensor, layer_idx: int) -> QuantizedKV:
        """Quantize (batch, n_heads, seq_len, head_dim) head vectors for cache storage."""
        return self._encode(x, layer_idx, True, self.group_size, self.qjl is not None)

    def dequantize(self, qkv: QuantizedKV, layer_idx: int, apply_inverse_rot: bool = False) -> torch.Tensor:
        """Reconstruct (rotated space unless apply_inverse_rot) float32 vectors."""
        return self._decode(qkv, layer_idx, apply_inverse_rot, self.group_size, self.qjl is not None)

    def quantize_for_attention(self, q: torch.Tensor, layer_idx: int) -> torch.Tensor:
        """Rotate queries into the keys' rotated space."""
        structured, signs = self._structured[layer_idx]
        if structured and q.is_cuda:
            from .. import ops
            y = q.float() * signs if signs is not None else q.float().clone()
            y = y.contiguous()
            ops.hadamard_(y, self.head_dim)
            return y
        return apply_rotation(q, self.rotations[layer_idx])

    def memory_bits_per_element(self) -> float:
        total = math.log2(BITS_TO_LEVELS.get(self.bits, round(2 ** self.bits)))
        if self.use_qjl:
            total += 1.0 + 32.0 / self.head_dim
        return total + 32.0 / self.group_size

    def compression_ratio(self, baseline_bits: int = 16) -> float:
        return baseline_bits / self.memory_bits_per_element()

    def __repr__(self) -> str:
        return (f"TurboQuantizer(layers={self.n_layers}, head_dim={self.head_dim}, "
                f"bits={self.bits}, group_size={self.group_size}, qjl={self.use_qjl}, "
                f"effective_bits={self.memory_bits_per_element():.2f}, "
                f"compression={self.compression_ratio():.1f}x)")
