"""Torch-tensor front end of the C ABI (device pointers, current CUDA stream).

Every op requires CUDA tensors and raises otherwise: there is no CPU path.
Packed blocks are uint8 tensors whose last two dims are (n_blocks, 18) for
TQ4_0 or (n_blocks, 14) for TQ3_0 — the byte layout of src/ggml-tq.h:131-141.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib as L

QK = L.QK
TQ2_0, TQ3_0, TQ4_0 = L.TYPE_TQ2_0, L.TYPE_TQ3_0, L.TYPE_TQ4_0
BLOCK_BYTES = L.BLOCK_BYTES
_DTYPES = {torch.float32: L.DTYPE_F32, torch.float16: L.DTYPE_F16, torch.bfloat16: L.DTYPE_BF16}


def _stream(t: torch.Tensor) -> C.c_void_p:
    return C.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _need_cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        if not isinstance(t, torch.Tensor) or not t.is_cuda:
            raise ValueError("leankv_b200 ops take CUDA tensors only (there is no CPU fallback)")


def _qtype(qtype) -> int:
    q = {2: TQ2_0, 3: TQ3_0, 4: TQ4_0, "tq2_0": TQ2_0, "tq3_0": TQ3_0, "tq4_0": TQ4_0}.get(qtype)
    if q is None:
        raise ValueError(f"unknown TQ type {qtype!r}")
    return q


def quantize(x: torch.Tensor, qtype=4, fwht_head_dim: int = 0, opt_passes: int = 0,
             out: torch.Tensor | None = None, rht_seed: int | None = None, row_len: int | None = None) -> torch.Tensor:
    """[FWHT per fwht_head_dim run] + TQ quantize of a contiguous f32/f16/bf16 tensor.

    Returns uint8 blocks shaped (*x.shape[:-1], x.shape[-1] // 32, block_bytes).
    Bit-exact with hadamard_transform_row + quantize_row_tq*_0_ref
    (src/ggml-tq.c) on x.float(); opt_passes=2 with qtype=3 is LeanKV's TQ3
    optimal rounding (scripts/tq3_rounding.py:74-125).  With rht_seed, every row of
    row_len elements (default: the last dimension) is first rotated as
    randomized_hadamard_transform_row(row, row_len, fwht_head_dim, rht_seed).
    """
    _need_cuda(x)
    q = _qtype(qtype)
    if x.dtype not in _DTYPES:
        raise TypeError(f"unsupported dtype {x.dtype}")
    if not x.is_contiguous():
        raise ValueError("x must be contiguous")
    if x.shape[-1] % QK:
        raise ValueError("the last dimension must be a multiple of 32")
    shape = (*x.shape[:-1], x.shape[-1] // QK, BLOCK_BYTES[q])
    if out is None:
        out = torch.empty(shape, dtype=torch.uint8, device=x.device)
    else:
        _need_cuda(out)
        if out.dtype != torch.uint8 or out.numel() != x.numel() // QK * BLOCK_BYTES[q] or not out.is_contiguous():
            raise ValueError("out must be a contiguous uint8 tensor of the block size")
    if rht_seed is not None:
        L.check(L.load().tq_quantize_randomized_cuda(q, x.data_ptr(), _DTYPES[x.dtype], out.data_ptr(), x.numel(),
                                                     int(row_len or x.shape[-1]), int(fwht_head_dim),
                                                     int(rht_seed) & 0xFFFFFFFF, int(opt_passes), _stream(x)))
        return out
    L.check(L.load().tq_quantize_cuda(q, x.data_ptr(), _DTYPES[x.dtype], out.data_ptr(), x.numel(),
                                      int(fwht_head_dim), int(opt_passes), _stream(x)))
    return out


def dequantize(blocks: torch.Tensor, qtype=4, dtype: torch.dtype = torch.float32,
               out: torch.Tensor | None = None) -> torch.Tensor:
    """dequantize_row_tq*_0 over uint8 blocks (..., n_blocks, block_bytes) -> (..., n_blocks*32)."""
    _need_cuda(blocks)
    q = _qtype(qtype)
    if blocks.dtype != torch.uint8 or not blocks.is_contiguous():
        raise ValueError("blocks must be a contiguous uint8 tensor")
    bb = BLOCK_BYTES[q]
    if blocks.numel() % bb:
        raise ValueError("block buffer size is not a multiple of the block size")
    nb = blocks.numel() // bb
    if blocks.dim() >= 2 and blocks.shape[-1] == bb:
        shape = (*blocks.shape[:-2], blocks.shape[-2] * QK)
    else:
        shape = (nb * QK,)
    if out is None:
        out = torch.empty(shape, dtype=dtype, device=blocks.device)
    else:
        _need_cuda(out)
        if out.numel() != nb * QK or not out.is_contiguous() or out.dtype not in _DTYPES:
            raise ValueError("bad out tensor")
    L.check(L.load().tq_dequantize_cuda(q, blocks.data_ptr(), out.data_ptr(), _DTYPES[out.dtype], nb * QK,
                                        _stream(blocks)))
    return out


def hadamard_(x: torch.Tensor, head_dim: int) -> torch.Tensor:
    """In-place hadamard_transform_row (src/ggml-tq.c:398-404) on a contiguous float32 tensor."""
    _need_cuda(x)
    if x.dtype != torch.float32 or not x.is_contiguous():
        raise ValueError("x must be a contiguous float32 tensor")
    L.check(L.load().tq_hadamard_cuda(x.data_ptr(), x.numel(), int(head_dim), _stream(x)))
    return x


def kv_append(src: torch.Tensor, cache: torch.Tensor, pos: torch.Tensor | None = None, qtype=None,
              rotate: bool = True, opt_passes: int = 0, overflow: torch.Tensor | None = None) -> torch.Tensor:
    """Quantize-on-write of new head rows into a packed KV cache (tq_kv_append_cuda).

    src [batch, n_kv_heads, n_new, head_dim] (f32/f16/bf16); cache uint8
    [batch, n_kv_heads, capacity, head_dim/32, block_bytes]; row t of (b, h) lands
    in token slot pos[b] + t (pos: int32 CUDA tensor [batch], None = slot t).
    rotate applies the head_dim Hadamard rotation first.  Slots outside the
    capacity are skipped and counted into overflow (int32 CUDA tensor [1]) when
    given.  Returns cache.
    """
    _need_cuda(src, cache)
    if src.dim() != 4 or not src.is_contiguous() or src.dtype not in _DTYPES:
        raise ValueError("src must be a contiguous f32/f16/bf16 [batch, n_kv_heads, n_new, head_dim] tensor")
    if cache.dim() != 5 or cache.dtype != torch.uint8 or not cache.is_contiguous():
        raise ValueError("cache must be a contiguous uint8 [batch, n_kv_heads, capacity, head_dim/32, bytes] tensor")
    B, H, n_new, D = src.shape
    if qtype is None:
        qtype = TQ4_0 if cache.shape[-1] == BLOCK_BYTES[TQ4_0] else TQ3_0
    q = _qtype(qtype)
    if cache.shape[0] != B or cache.shape[1] != H or cache.shape[3] * QK != D or cache.shape[4] != BLOCK_BYTES[q]:
        raise ValueError(f"cache shape {tuple(cache.shape)} does not match src {tuple(src.shape)} / type {q}")
    if pos is not None:
        _need_cuda(pos)
        if pos.dtype != torch.int32 or pos.numel() != B or not pos.is_contiguous():
            raise ValueError("pos must be a contiguous int32 [batch] tensor")
    if overflow is not None:
        _need_cuda(overflow)
        if overflow.dtype != torch.int32:
            raise ValueError("overflow must be an int32 tensor")
    L.check(L.load().tq_kv_append_cuda(q, src.data_ptr(), _DTYPES[src.dtype], cache.data_ptr(), B, H, D,
                                       cache.shape[2], n_new, pos.data_ptr() if pos is not None else None,
                                       int(rotate), int(opt_passes),
                                       overflow.data_ptr() if overflow is not None else None, _stream(src)))
    return cache


def kv_append_paged(src: torch.Tensor, pool: torch.Tensor, page_table: torch.Tensor, pos: torch.Tensor | None = None,
                    qtype=None, rotate: bool = True, opt_passes: int = 0,
                    overflow: torch.Tensor | None = None) -> torch.Tensor:
    """kv_append into a paged cache (tq_kv_append_paged_cuda).

    pool uint8 [num_pages, n_kv_heads, page_size, head_dim/32, block_bytes];
    page_table int32 CUDA [batch, max_pages_per_seq]: token slot s of sequence b
    lives in pool page page_table[b, s // page_size] at row s % page_size.  Rows
    whose slot is past max_pages_per_seq * page_size, or whose page id is outside
    the pool, are skipped and counted into overflow.  Returns pool.
    """
    from .attention import make_pages
    _need_cuda(src, pool, page_table)
    if src.dim() != 4 or not src.is_contiguous() or src.dtype not in _DTYPES:
        raise ValueError("src must be a contiguous f32/f16/bf16 [batch, n_kv_heads, n_new, head_dim] tensor")
    if pool.dim() != 5 or pool.dtype != torch.uint8 or not pool.is_contiguous():
        raise ValueError("pool must be a contiguous uint8 [num_pages, n_kv_heads, page_size, head_dim/32, bytes] tensor")
    B, H, n_new, D = src.shape
    if qtype is None:
        qtype = TQ4_0 if pool.shape[-1] == BLOCK_BYTES[TQ4_0] else TQ3_0
    q = _qtype(qtype)
    if pool.shape[1] != H or pool.shape[3] * QK != D or pool.shape[4] != BLOCK_BYTES[q]:
        raise ValueError(f"pool shape {tuple(pool.shape)} does not match src {tuple(src.shape)} / type {q}")
    if page_table.dtype != torch.int32 or page_table.dim() != 2 or page_table.shape[0] != B \
            or not page_table.is_contiguous():
        raise ValueError("page_table must be a contiguous int32 [batch, max_pages_per_seq] tensor")
    if pos is not None:
        _need_cuda(pos)
        if pos.dtype != torch.int32 or pos.numel() != B or not pos.is_contiguous():
            raise ValueError("pos must be a contiguous int32 [batch] tensor")
    if overflow is not None:
        _need_cuda(overflow)
        if overflow.dtype != torch.int32:
            raise ValueError("overflow must be an int32 tensor")
    pg = make_pages(page_table, pool.shape[0], pool.shape[2])
    L.check(L.load().tq_kv_append_paged_cuda(q, src.data_ptr(), _DTYPES[src.dtype], pool.data_ptr(), B, H, D,
                                             C.byref(pg), n_new, pos.data_ptr() if pos is not None else None,
                                             int(rotate), int(opt_passes),
                                             overflow.data_ptr() if overflow is not None else None, _stream(src)))
    return pool


TQ2_1_BYTES = 44   # block_tq2_1: a TQ3_0 block and three TQ2_0 blocks per 128 elements


def quantize_tq2_1(x: torch.Tensor) -> torch.Tensor:
    """TQ2_1 blocks (the fork's static mixed-precision type, tq_quantize_tq2_1_cuda) of a contiguous
    f32/f16/bf16 tensor whose last dim is a multiple of 128: uint8 (..., last / 128, 44).  No
    rotation is applied (rotate first with hadamard_ when the rows should be rotated)."""
    _need_cuda(x)
    if x.dtype not in _DTYPES or not x.is_contiguous() or x.dim() == 0 or x.shape[-1] % 128:
        raise ValueError("x must be a contiguous f32/f16/bf16 tensor whose last dim is a multiple of 128")
    out = torch.empty((*x.shape[:-1], x.shape[-1] // 128, TQ2_1_BYTES), dtype=torch.uint8, device=x.device)
    L.check(L.load().tq_quantize_tq2_1_cuda(x.data_ptr(), _DTYPES[x.dtype], out.data_ptr(), x.numel(), _stream(x)))
    return out


def dequantize_tq2_1(blocks: torch.Tensor) -> torch.Tensor:
    """float32 (..., n_blocks * 128) from uint8 TQ2_1 blocks (..., n_blocks, 44)."""
    _need_cuda(blocks)
    if blocks.dtype != torch.uint8 or not blocks.is_contiguous() or blocks.dim() < 2 \
            or blocks.shape[-1] != TQ2_1_BYTES:
        raise ValueError("blocks must be a contiguous uint8 (..., n_blocks, 44) tensor")
    out = torch.empty((*blocks.shape[:-2], blocks.shape[-2] * 128), dtype=torch.float32, device=blocks.device)
    L.check(L.load().tq_dequantize_tq2_1_cuda(blocks.data_ptr(), out.data_ptr(), out.numel(), _stream(blocks)))
    return out


def requantize(blocks: torch.Tensor, src_qtype, dst_qtype) -> torch.Tensor:
    """Blocks of src_qtype -> blocks of dst_qtype (dequantize + quantize per block, one kernel;
    requantize_tq4_to_tq3 / tq3_to_tq2 / tq4_to_tq2 of src/ggml-tq.c:329-357)."""
    _need_cuda(blocks)
    a, b = _qtype(src_qtype), _qtype(dst_qtype)
    if blocks.dtype != torch.uint8 or not blocks.is_contiguous() or blocks.numel() % BLOCK_BYTES[a]:
        raise ValueError("blocks must be a contiguous uint8 tensor of whole blocks")
    nb = blocks.numel() // BLOCK_BYTES[a]
    shape = (*blocks.shape[:-1], BLOCK_BYTES[b]) if blocks.dim() >= 1 and blocks.shape[-1] == BLOCK_BYTES[a] \
        else (nb, BLOCK_BYTES[b])
    out = torch.empty(shape, dtype=torch.uint8, device=blocks.device)
    L.check(L.load().tq_requantize_cuda(a, blocks.data_ptr(), b, out.data_ptr(), nb * QK, _stream(blocks)))
    return out


def hadamard_randomized_(x: torch.Tensor, head_dim: int, seed: int, row_len: int | None = None) -> torch.Tensor:
    """In-place randomized_hadamard_transform_row (src/ggml-tq.c:383-412) on every row of row_len
    elements (default: the last dimension) of a contiguous float32 tensor."""
    _need_cuda(x)
    if x.dtype != torch.float32 or not x.is_contiguous():
        raise ValueError("x must be a contiguous float32 tensor")
    L.check(L.load().tq_hadamard_randomized_cuda(x.data_ptr(), x.numel(), int(row_len or x.shape[-1]), int(head_dim),
                                                 int(seed) & 0xFFFFFFFF, _stream(x)))
    return x


class OutlierConfig(C.Structure):
    """Mirror of tq_outlier_config (src/ggml-tq-outlier.h:44-64, include/leankv_tq.h)."""
    _fields_ = [("head_dim", C.c_int), ("n_outlier", C.c_int), ("n_normal", C.c_int), ("outlier_frac", C.c_float),
                ("outlier_tier", C.c_int), ("normal_tier", C.c_int), ("perm", C.c_int * 256),
                ("inv_perm", C.c_int * 256), ("channel_var", C.c_float * 256)]


TIER_TQ2, TIER_TQ3, TIER_TQ4 = 0, 1, 2
_TIER_BYTES = {TIER_TQ2: 10, TIER_TQ3: 14, TIER_TQ4: 18}


def identify_outliers(calib: torch.Tensor, outlier_frac: float = 0.25, outlier_tier: int = TIER_TQ3,
                      normal_tier: int = TIER_TQ2) -> OutlierConfig:
    """Per-channel variance ranking of calibration data [n_tokens, head_dim] (float32, CUDA)
    -> outlier configuration (tq_identify_outliers, src/ggml-tq-outlier.c:97-170)."""
    _need_cuda(calib)
    if calib.dtype != torch.float32 or calib.dim() != 2 or not calib.is_contiguous():
        raise ValueError("calib must be a contiguous float32 [n_tokens, head_dim] tensor")
    cfg = OutlierConfig()
    L.check(L.load().tq_outlier_identify_cuda(C.byref(cfg), calib.data_ptr(), calib.shape[0], calib.shape[1],
                                              float(outlier_frac), int(outlier_tier), int(normal_tier), _stream(calib)))
    return cfg


def mixed_quantize(x: torch.Tensor, cfg: OutlierConfig) -> tuple[torch.Tensor, torch.Tensor]:
    """Channel-permuted two-tier quantization of head vectors x [..., head_dim]
    (tq_mixed_quantize per vector) -> (outlier blocks, normal blocks) uint8."""
    _need_cuda(x)
    if x.dtype not in _DTYPES or not x.is_contiguous() or x.shape[-1] != cfg.head_dim:
        raise ValueError("x must be a contiguous f32/f16/bf16 tensor with head_dim last")
    n_vec = x.numel() // cfg.head_dim
    ob = torch.empty(*x.shape[:-1], cfg.n_outlier // QK, _TIER_BYTES[cfg.outlier_tier], dtype=torch.uint8, device=x.device)
    nb = torch.empty(*x.shape[:-1], cfg.n_normal // QK, _TIER_BYTES[cfg.normal_tier], dtype=torch.uint8, device=x.device)
    L.check(L.load().tq_mixed_quantize_cuda(C.byref(cfg), x.data_ptr(), _DTYPES[x.dtype], n_vec, ob.data_ptr(),
                                            nb.data_ptr(), _stream(x)))
    return ob, nb


def mixed_dequantize(outlier_blocks: torch.Tensor, normal_blocks: torch.Tensor, cfg: OutlierConfig) -> torch.Tensor:
    """Inverse of mixed_quantize: float32 [..., head_dim] in the original channel order."""
    _need_cuda(outlier_blocks, normal_blocks)
    lead = outlier_blocks.shape[:-2] if cfg.n_outlier else normal_blocks.shape[:-2]
    n_vec = 1
    for s in lead:
        n_vec *= s
    y = torch.empty(*lead, cfg.head_dim, dtype=torch.float32, device=outlier_blocks.device)
    L.check(L.load().tq_mixed_dequantize_cuda(C.byref(cfg), outlier_blocks.contiguous().data_ptr(),
                                              normal_blocks.contiguous().data_ptr(), n_vec, y.data_ptr(),
                                              _stream(outlier_blocks)))
    return y
