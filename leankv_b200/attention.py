"""Fused decode attention over packed TurboQuant K/V caches (torch front end).

Cache tensors are uint8 with shape [batch, n_kv_heads, capacity, head_dim/32, bytes]
of TQ4_0 (18-byte) or, for K, TQ3_0 (14-byte) or TQ2_0 (10-byte) blocks (src/ggml-tq.h:125-141);
head_dim is 128 or 256 and capacity even.  K and V hold Hadamard-rotated rows
(quantize with fwht_head_dim=head_dim); the query is rotated inside, and the
output rotated back, so the result is attention in the original space.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib as L
from .ops import _DTYPES, _need_cuda, _stream


class AttnArgs(C.Structure):
    """Mirror of tq_decode_attention_args (include/leankv_tq.h)."""
    _fields_ = [
        ("batch", C.c_int), ("n_q_heads", C.c_int), ("n_kv_heads", C.c_int), ("head_dim", C.c_int),
        ("q", C.c_void_p), ("q_dtype", C.c_int),
        ("k_cache", C.c_void_p), ("k_type", C.c_int),
        ("v_cache", C.c_void_p), ("v_type", C.c_int),
        ("kv_capacity", C.c_int64),
        ("kv_len", C.c_void_p),
        ("max_kv_len", C.c_int64),
        ("sm_scale", C.c_float),
        ("rotate_q", C.c_int),
        ("v_rotated", C.c_int),
        ("out", C.c_void_p), ("out_dtype", C.c_int),
        ("lse", C.c_void_p),
        ("workspace", C.c_void_p), ("workspace_bytes", C.c_size_t),
    ]


class KVPages(C.Structure):
    """Mirror of tq_kv_pages (include/leankv_tq.h): a paged cache's page table."""
    _fields_ = [("page_table", C.c_void_p), ("max_pages_per_seq", C.c_int64), ("num_pages", C.c_int64),
                ("page_size", C.c_int)]


def make_pages(page_table: torch.Tensor, num_pages: int, page_size: int) -> KVPages:
    pg = KVPages()
    pg.page_table = page_table.data_ptr()
    pg.max_pages_per_seq = page_table.shape[1]
    pg.num_pages = int(num_pages)
    pg.page_size = int(page_size)
    return pg


def _bind():
    lib = L.load()
    lib.tq_decode_attention_workspace_size.restype = C.c_size_t
    lib.tq_decode_attention_workspace_size.argtypes = [C.POINTER(AttnArgs)]
    lib.tq_decode_attention_cuda.restype = C.c_int
    lib.tq_decode_attention_cuda.argtypes = [C.POINTER(AttnArgs), C.c_void_p]
    lib.tq_decode_attention_paged_cuda.restype = C.c_int
    lib.tq_decode_attention_paged_cuda.argtypes = [C.POINTER(AttnArgs), C.POINTER(KVPages), C.c_void_p]
    lib.tq_lse_combine_cuda.restype = C.c_int
    lib.tq_lse_combine_cuda.argtypes = [C.c_int, C.c_int64, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p,
                                        C.c_void_p, C.c_void_p]
    return lib


_workspaces: dict = {}


def _workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    key = (device.type, device.index)
    ws = _workspaces.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _workspaces[key] = ws
    return ws


def make_args(q, k_cache, v_cache, kv_len=None, max_kv_len=0, sm_scale=0.0, rotate_q=True, v_rotated=True,
              out=None, lse=None, k_type=4, v_type=4):
    B, Hq, D = q.shape
    Hkv, cap = k_cache.shape[1], k_cache.shape[2]
    a = AttnArgs()
    a.batch, a.n_q_heads, a.n_kv_heads, a.head_dim = B, Hq, Hkv, D
    a.q, a.q_dtype = q.data_ptr(), _DTYPES[q.dtype]
    a.k_cache, a.k_type = k_cache.data_ptr(), k_type
    a.v_cache, a.v_type = v_cache.data_ptr(), v_type
    a.kv_capacity = cap
    a.kv_len = kv_len.data_ptr() if kv_len is not None else None
    a.max_kv_len = int(max_kv_len)
    a.sm_scale = float(sm_scale)
    a.rotate_q, a.v_rotated = int(rotate_q), int(v_rotated)
    a.out, a.out_dtype = out.data_ptr(), _DTYPES[out.dtype]
    a.lse = lse.data_ptr() if lse is not None else None
    return a


def decode_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                     kv_len: torch.Tensor | None = None, max_kv_len: int | None = None,
                     sm_scale: float | None = None, rotate_q: bool = True, v_rotated: bool = True,
                     out_dtype: torch.dtype = torch.float32, return_lse: bool = False,
                     out: torch.Tensor | None = None, lse_out: torch.Tensor | None = None):
    """softmax(q~ K^T * sm_scale) V over packed caches; q [B, Hq, D] -> out [B, Hq, D].

    kv_len: int32 CUDA tensor [B] of valid tokens (default: the whole capacity);
    max_kv_len: host-side upper bound of kv_len used to plan the split-KV work
    (default: the capacity).  out / lse_out: preallocated contiguous [B, Hq, D]
    and float32 [B, Hq] destinations (lse_out implies the lse is written).
    """
    _check_caches(q, k_cache, v_cache)
    kv_len = _check_len(kv_len, q.shape[0])
    out, lse = _outputs(q, out_dtype, out, lse_out, return_lse)
    a = make_args(q, k_cache, v_cache, kv_len, max_kv_len or 0, sm_scale or 0.0, rotate_q, v_rotated, out, lse,
                  _btype(k_cache), _btype(v_cache))
    lib = _bind()
    need = lib.tq_decode_attention_workspace_size(C.byref(a))
    if need == 0:
        # argument error: let the launch report it with a message
        L.check(lib.tq_decode_attention_cuda(C.byref(a), _stream(q)))
    ws = _workspace(q.device, need)
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    L.check(lib.tq_decode_attention_cuda(C.byref(a), _stream(q)))
    return (out, lse) if return_lse else out


def decode_attention_paged(q: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor, page_table: torch.Tensor,
                           kv_len: torch.Tensor, max_kv_len: int | None = None, sm_scale: float | None = None,
                           rotate_q: bool = True, v_rotated: bool = True, out_dtype: torch.dtype = torch.float32,
                           return_lse: bool = False, out: torch.Tensor | None = None,
                           lse_out: torch.Tensor | None = None):
    """decode_attention over paged caches (tq_decode_attention_paged_cuda).

    k_pool / v_pool: uint8 [num_pages, n_kv_heads, page_size, head_dim/32, bytes];
    page_table: int32 CUDA [B, max_pages_per_seq], row b listing the pool pages of
    sequence b's tokens in order; kv_len: int32 CUDA [B].  Bit-identical to
    decode_attention on the same tokens stored contiguously.
    """
    _check_caches(q, k_pool, v_pool)
    kv_len = _check_len(kv_len, q.shape[0])
    _need_cuda(page_table)
    if page_table.dtype != torch.int32 or page_table.dim() != 2 or page_table.shape[0] != q.shape[0] \
            or not page_table.is_contiguous():
        raise ValueError("page_table must be a contiguous int32 [batch, max_pages_per_seq] tensor")
    if k_pool.shape[:3] != v_pool.shape[:3]:
        raise ValueError("K and V pools must have the same pages, heads and page size")
    num_pages, _, page_size = k_pool.shape[:3]
    out, lse = _outputs(q, out_dtype, out, lse_out, return_lse)
    a = make_args(q, k_pool, v_pool, kv_len, max_kv_len or 0, sm_scale or 0.0, rotate_q, v_rotated, out, lse,
                  _btype(k_pool), _btype(v_pool))
    a.kv_capacity = page_table.shape[1] * page_size
    pg = make_pages(page_table, num_pages, page_size)
    lib = _bind()
    need = lib.tq_decode_attention_workspace_size(C.byref(a))
    if need:
        ws = _workspace(q.device, need)
        a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    L.check(lib.tq_decode_attention_paged_cuda(C.byref(a), C.byref(pg), _stream(q)))
    return (out, lse) if return_lse else out


def _btype(cache: torch.Tensor) -> int:
    return {18: 4, 14: 3, 10: 2}.get(int(cache.shape[-1]), 0)   # 0: rejected by the argument check


def _check_caches(q, k_cache, v_cache) -> None:
    _need_cuda(q, k_cache, v_cache)
    if q.dim() != 3 or not q.is_contiguous():
        raise ValueError("q must be a contiguous [B, Hq, D] tensor")
    if k_cache.dtype != torch.uint8 or v_cache.dtype != torch.uint8:
        raise ValueError("caches must be uint8 block tensors")
    if not (k_cache.is_contiguous() and v_cache.is_contiguous()):
        raise ValueError("caches must be contiguous")


def _check_len(kv_len, batch):
    if kv_len is None:
        return None
    _need_cuda(kv_len)
    if kv_len.dtype != torch.int32 or kv_len.numel() != batch:
        raise ValueError("kv_len must be int32 [batch]")
    return kv_len.contiguous()


def _outputs(q, out_dtype, out, lse_out, return_lse):
    B, Hq, D = q.shape
    if out is None:
        out = torch.empty((B, Hq, D), dtype=out_dtype, device=q.device)
    if lse_out is not None:
        _need_cuda(lse_out)
        if lse_out.dtype != torch.float32 or lse_out.numel() != B * Hq or not lse_out.is_contiguous():
            raise ValueError("lse_out must be a contiguous float32 [B, Hq] tensor")
        return out, lse_out
    return out, (torch.empty((B, Hq), dtype=torch.float32, device=q.device) if return_lse else None)


def last_status(device: torch.device | str | int | None = None) -> int:
    """Kernel-side status of the last decode_attention on `device` (synchronizes its stream).

    0 (TQ_SUCCESS), 7 (TQ_ERROR_TIMEOUT: a bulk copy never completed) or 2
    (TQ_ERROR_UNSUPPORTED: a block scale of magnitude >= 2^15).
    """
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    if dev.type == "cuda" and dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    ws = _workspaces.get((dev.type, dev.index))
    if ws is None:
        return 0
    return int(ws[:4].view(torch.int32).item())


def merge_partials(parts: torch.Tensor, n_parts: int, n_rows: int, head_dim: int, out: torch.Tensor,
                   lse_out: torch.Tensor | None = None) -> torch.Tensor:
    """Log-sum-exp merge of partials packed per part as [o (n_rows*head_dim) | lse (n_rows)] floats.

    parts: contiguous float32 [n_parts * n_rows * (head_dim + 1)] (e.g. the output of
    an all_gather of every rank's packed partial); out: contiguous [n_rows, head_dim]
    of float32/float16/bfloat16 (written); lse_out: optional float32 [n_rows].
    """
    _need_cuda(parts, out)
    stride = n_rows * (head_dim + 1)
    if parts.dtype != torch.float32 or not parts.is_contiguous() or parts.numel() < n_parts * stride:
        raise ValueError("parts must be a contiguous float32 buffer of n_parts packed partials")
    if out.dtype not in _DTYPES or not out.is_contiguous() or out.numel() != n_rows * head_dim:
        raise ValueError("out must be a contiguous [n_rows, head_dim] tensor")
    base = parts.data_ptr()
    L.check(_bind().tq_lse_merge_cuda(n_parts, n_rows, head_dim, base, stride, base + 4 * n_rows * head_dim, stride,
                                      out.data_ptr(), _DTYPES[out.dtype],
                                      lse_out.data_ptr() if lse_out is not None else None, _stream(parts)))
    return out


def lse_combine(o: torch.Tensor, lse: torch.Tensor, return_lse: bool = False):
    """Merge partial results o [P, n, D] (normalized) with natural-log lse [P, n]."""
    _need_cuda(o, lse)
    if o.dtype != torch.float32 or lse.dtype != torch.float32:
        raise ValueError("float32 partials expected")
    o = o.contiguous()
    lse = lse.contiguous()
    P, n, D = o.shape
    out = torch.empty((n, D), dtype=torch.float32, device=o.device)
    lo = torch.empty((n,), dtype=torch.float32, device=o.device) if return_lse else None
    lib = _bind()
    L.check(lib.tq_lse_combine_cuda(P, n, D, o.data_ptr(), lse.data_ptr(), out.data_ptr(),
                                    lo.data_ptr() if lo is not None else None, _stream(o)))
    return (out, lo) if return_lse else out
