"""LeanKVCache: the prototype's HuggingFace-style quantized KV cache
(prototype/turboquant/kv_cache.py:31-245) with GPU-resident packed storage.

Two storage modes.

storage="prototype" (default, the prototype's numerics): keys go through
rotation + Lloyd-Max (+ QJL) in TurboQuantizer; values through Lloyd-Max of the
L2-normalised vector, rotated only when v_rotation is not "none".  update()
returns every cached key (rotated space) and value (original space)
dequantized, like the prototype.  Instead of a Python list of per-call pieces
that is concatenated on every read, each layer keeps its packed codes in device
buffers laid out [token][batch][head] that grow by doubling, so appends are one
copy and the read-out is one decode launch over a contiguous range.

storage="tq_blocks": the layer caches are TurboQuant blocks (TQ3_0 or TQ4_0
keys, TQ4_0 values, src/ggml-tq.h:131-141) in the decode-attention layout
[batch, kv_head, capacity, head_dim / 32, block bytes].  update() quantizes the
new rows on write (head_dim Hadamard rotation fused, tq_kv_append_cuda) and
returns the packed caches; attention() runs the fused decode attention over
them (tq_decode_attention_cuda).  Nothing dequantizes the cache: the
prototype's read-out of the whole cache on every step (kv_cache.py:170-204)
becomes one kernel that reads the packed blocks once.

storage="tq_pages": the same blocks in fixed page pools per layer
(leankv_b200.paged): pages are handed to the batch's sequences as they grow,
so the cache never copies itself to grow and its memory is the pool size set
at construction; attention() runs the paged decode attention
(tq_decode_attention_paged_cuda), bit-identical to the tq_blocks result.
"""
from __future__ import annotations

from typing import Any, Dict, List, Optional, Tuple

import torch

from .. import attention as _attention
from .. import ops as _ops
from .quantizer import QuantizedKV, TurboQuantizer


class _LayerStore:
    """Packed codes of one layer, [capacity, batch, heads, ...] per field."""

    def __init__(self):
        self.len = 0
        self.cap = 0
        self.k: dict = {}
        self.v: dict = {}

    @staticmethod
    def _fields(q: QuantizedKV) -> dict:
        return {n: t for n, t in (("indices", q.indices), ("qjl_signs", q.qjl_signs),
                                  ("qjl_mean_abs", q.qjl_mean_abs), ("norms", q.norms)) if t is not None}

    def append(self, kq: QuantizedKV, vq: QuantizedKV) -> None:
        n = kq.indices.shape[2]
        new = {"k": self._fields(kq), "v": self._fields(vq)}
        if self.len + n > self.cap:
            cap = max(2 * self.cap, self.len + n, 16)
            for side in ("k", "v"):
                old = getattr(self, side)
                grown = {}
                for name, t in new[side].items():
                    shp = (cap, t.shape[0], t.shape[1], *t.shape[3:])
                    buf = torch.empty(shp, dtype=t.dtype, device=t.device)
                    if name in old and self.len:
                        buf[: self.len].copy_(old[name][: self.len])
                    grown[name] = buf
                setattr(self, side, grown)
            self.cap = cap
        for side in ("k", "v"):
            store = getattr(self, side)
            for name, t in new[side].items():
                store[name][self.len: self.len + n].copy_(t.movedim(2, 0))
        self.len += n

    def view(self, side: str) -> QuantizedKV:
        """QuantizedKV over the filled range, in [token, batch, head, ...] layout."""
        s = getattr(self, side)
        get = lambda n: s[n][: self.len] if n in s else None  # noqa: E731
        return QuantizedKV(indices=get("indices"), qjl_signs=get("qjl_signs"), qjl_mean_abs=get("qjl_mean_abs"),
                           norms=get("norms"))


class _BlockStore:
    """TurboQuant blocks of one layer: K and V [batch, kv_head, capacity, head_dim / 32, bytes].

    Capacity grows by doubling (kept even, as the decode attention requires); `pos` is the
    device-side length of every sequence, the append slot of the next rows and the
    attention's kv_len.
    """

    def __init__(self, k_type: int, k_passes: int):
        self.k_type, self.k_passes = k_type, k_passes
        self.len = 0
        self.cap = 0
        self.k = self.v = self.pos = None

    def append(self, k: torch.Tensor, v: torch.Tensor) -> None:
        B, H, n, D = k.shape
        if self.k is not None and (self.k.shape[0] != B or self.k.shape[1] != H):
            raise ValueError("batch and KV-head counts must not change between updates")
        if self.len + n > self.cap:
            cap = max(2 * self.cap, self.len + n, 16)
            cap += cap & 1
            kb = {2: 10, 3: 14, 4: 18}[self.k_type]
            knew = torch.empty(B, H, cap, D // 32, kb, dtype=torch.uint8, device=k.device)
            vnew = torch.empty(B, H, cap, D // 32, 18, dtype=torch.uint8, device=k.device)
            if self.len:
                knew[:, :, : self.len].copy_(self.k[:, :, : self.len])
                vnew[:, :, : self.len].copy_(self.v[:, :, : self.len])
            else:
                self.pos = torch.zeros(B, dtype=torch.int32, device=k.device)
            self.k, self.v, self.cap = knew, vnew, cap
        _ops.kv_append(k.contiguous(), self.k, self.pos, qtype=self.k_type, rotate=True, opt_passes=self.k_passes)
        _ops.kv_append(v.contiguous(), self.v, self.pos, qtype=4, rotate=True)
        self.pos += n
        self.len += n


class _PagedStore:
    """TurboQuant blocks of one layer in fixed page pools (a one-layer PagedKVCache): the batch's
    sequences get pages as they grow, nothing is copied when the cache grows, and the pool size
    (num_pages x page_size tokens over all sequences) is the memory bound."""

    def __init__(self, k_type: int, k_passes: int, num_pages: int, page_size: int):
        self.k_type, self.k_passes = k_type, k_passes
        self.num_pages, self.page_size = num_pages, page_size
        self.cache = None
        self.seqs: list = []
        self.len = 0

    def append(self, k: torch.Tensor, v: torch.Tensor) -> None:
        from ..paged import PagedKVCache
        B, H, n, D = k.shape
        if self.cache is None:
            self.cache = PagedKVCache(1, H, D, self.num_pages, self.page_size, max_seqs=B,
                                      max_pages_per_seq=self.num_pages, k_bits=self.k_type,
                                      k_opt_passes=self.k_passes, device=str(k.device))
            self.seqs = [self.cache.add_sequence() for _ in range(B)]
        elif B != len(self.seqs) or H != self.cache.n_kv_heads:
            raise ValueError("batch and KV-head counts must not change between updates")
        step = self.cache.batch(self.seqs, n)
        self.cache.append(step, 0, k, v)
        self.cache.commit(step)
        self.len += n

    def attention(self, q: torch.Tensor, sm_scale, out_dtype) -> torch.Tensor:
        step = self.cache.batch(self.seqs, 0)   # page rows and lengths, nothing reserved
        return self.cache.attention(step, 0, q, sm_scale=sm_scale, out_dtype=out_dtype)


class LeanKVCache:
    """Quantized KV cache with the interface of transformers.DynamicCache (update / get_seq_length ...)."""

    def __init__(self, n_layers: int, head_dim: int, n_kv_heads: int = 1, k_bits=3, v_bits=4,
                 k_rotation: str = "randomized_hadamard", v_rotation: str = "none", use_qjl: bool = True,
                 seed: int = 42, device: str = "cuda", storage: str = "prototype", k_opt_passes: int = 0,
                 num_pages: int = 0, page_size: int = 16):
        """storage: "prototype" (the prototype's quantizers, dequantized read-out), "tq_blocks"
        (TQ{k_bits}_0 keys and TQ4_0 values as packed blocks that grow by doubling, fused decode
        attention; head_dim 128 or 256; k_opt_passes > 0 applies TQ3 optimal rounding to TQ3_0
        keys) or "tq_pages" (the same blocks in fixed page pools of num_pages pages of page_size
        tokens per layer, shared by the batch's sequences: no copy when the cache grows)."""
        if storage not in ("prototype", "tq_blocks", "tq_pages"):
            raise ValueError("storage must be 'prototype', 'tq_blocks' or 'tq_pages'")
        if storage == "tq_pages" and num_pages <= 0:
            raise ValueError("tq_pages storage needs num_pages > 0 (the pool size per layer)")
        self.storage = storage
        self.n_layers = n_layers
        self.head_dim = head_dim
        self.n_kv_heads = n_kv_heads
        if storage in ("tq_blocks", "tq_pages"):
            if head_dim not in (128, 256):
                raise ValueError(f"{storage} storage needs head_dim 128 or 256 (fused decode attention)")
            if k_bits not in (2, 3, 4) or v_bits != 4:
                raise ValueError(f"{storage} storage holds TQ2_0, TQ3_0 or TQ4_0 keys and TQ4_0 values")
            if k_opt_passes and k_bits != 3:
                raise ValueError("optimal rounding applies to TQ3_0 keys")
            if not str(device).startswith("cuda"):
                raise ValueError(f"{storage} storage lives on a CUDA device")
            self.k_bits, self.v_bits = k_bits, v_bits
            self._blocks = ([_BlockStore(k_bits, k_opt_passes) for _ in range(n_layers)] if storage == "tq_blocks"
                            else [_PagedStore(k_bits, k_opt_passes, num_pages, page_size) for _ in range(n_layers)])
            self._seen_tokens = 0
            return
        self.k_quantizer = TurboQuantizer(n_layers=n_layers, head_dim=head_dim, bits=k_bits,
                                          rotation_strategy=k_rotation, use_qjl=use_qjl, seed=seed, device=device)
        self.v_rotate = v_rotation != "none"
        self.v_quantizer = TurboQuantizer(n_layers=n_layers, head_dim=head_dim, bits=v_bits,
                                          rotation_strategy=v_rotation if self.v_rotate else "hadamard",
                                          use_qjl=False, seed=seed + 1000, device=device)
        self._store = [_LayerStore() for _ in range(n_layers)]
        self._seen_tokens = 0

    # per-layer lists of QuantizedKV, as the prototype exposes them (one entry per layer here,
    # covering every cached token, in [token, batch, head, ...] layout)
    # (storage="tq_blocks": the packed layer caches instead, one uint8 block tensor per layer)
    # (storage="tq_pages": each layer's page pools, [num_pages, kv_head, page_size, head_dim / 32, bytes])
    @property
    def k_cache(self) -> List[List[QuantizedKV]]:
        if self.storage == "tq_blocks":
            return [[b.k[:, :, : b.len]] if b.len else [] for b in self._blocks]
        if self.storage == "tq_pages":
            return [[b.cache.k[0]] if b.len else [] for b in self._blocks]
        return [[s.view("k")] if s.len else [] for s in self._store]

    @property
    def v_cache(self) -> List[List[QuantizedKV]]:
        if self.storage == "tq_blocks":
            return [[b.v[:, :, : b.len]] if b.len else [] for b in self._blocks]
        if self.storage == "tq_pages":
            return [[b.cache.v[0]] if b.len else [] for b in self._blocks]
        return [[s.view("v")] if s.len else [] for s in self._store]

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, layer_idx: int,
               cache_kwargs: Optional[Dict[str, Any]] = None) -> Tuple[torch.Tensor, torch.Tensor]:
        """Store new (batch, n_kv_heads, new_seq, head_dim) K/V; return all cached K (rotated) and V.

        With storage="tq_blocks" the rows are quantized on write and the return value is the packed
        layer caches (uint8 [batch, kv_head, length, head_dim / 32, bytes] views); with "tq_pages"
        the layer's K and V page pools; attend with attention().
        """
        if layer_idx == 0:
            self._seen_tokens += key_states.shape[2]
        if self.storage == "tq_blocks":
            st = self._blocks[layer_idx]
            st.append(key_states, value_states)
            return st.k[:, :, : st.len], st.v[:, :, : st.len]
        if self.storage == "tq_pages":
            st = self._blocks[layer_idx]
            st.append(key_states, value_states)
            return st.cache.k[0], st.cache.v[0]
        kq = self.k_quantizer.quantize(key_states, layer_idx)
        vq = self._quantize_values(value_states, layer_idx)
        self._store[layer_idx].append(kq, vq)
        return self._get_all_keys(layer_idx), self._get_all_values(layer_idx)

    def _quantize_values(self, v: torch.Tensor, layer_idx: int) -> QuantizedKV:
        if self.v_rotate:
            return self.v_quantizer.quantize(v, layer_idx)
        # L2-normalised values, no rotation, no QJL
        return self.v_quantizer._encode(v, None, False, self.head_dim, False)

    def _get_all_keys(self, layer_idx: int) -> Optional[torch.Tensor]:
        s = self._store[layer_idx]
        if not s.len:
            return None
        y = self.k_quantizer.dequantize(s.view("k"), layer_idx, apply_inverse_rot=False)
        return y.permute(1, 2, 0, 3)

    def _get_all_values(self, layer_idx: int) -> Optional[torch.Tensor]:
        s = self._store[layer_idx]
        if not s.len:
            return None
        q = s.view("v")
        if self.v_rotate:
            y = self.v_quantizer.dequantize(q, layer_idx, apply_inverse_rot=True)
        else:
            y = self.v_quantizer._decode(q, None, False, self.head_dim, False)
        return y.permute(1, 2, 0, 3)

    def attention(self, query_states: torch.Tensor, layer_idx: int, sm_scale: float | None = None,
                  out_dtype: torch.dtype | None = None) -> torch.Tensor:
        """softmax(q K^T * sm_scale) V over the packed layer cache for one query token per sequence
        (storage="tq_blocks" or "tq_pages"): query_states (batch, n_q_heads, 1, head_dim) in the
        original space (the kernel rotates it and rotates the output back); returns (batch,
        n_q_heads, 1, head_dim) in out_dtype (default: the query's).  n_q_heads / n_kv_heads must
        be 1 .. 8."""
        if self.storage not in ("tq_blocks", "tq_pages"):
            raise ValueError("attention() needs storage='tq_blocks' or 'tq_pages'")
        st = self._blocks[layer_idx]
        if not st.len:
            raise ValueError("the layer cache is empty")
        q = query_states
        if q.dim() == 4:
            if q.shape[2] != 1:
                raise ValueError("decode attention takes one query token per sequence")
            q = q[:, :, 0]
        if self.storage == "tq_pages":
            return st.attention(q.contiguous(), sm_scale, out_dtype or q.dtype).unsqueeze(2)
        out = _attention.decode_attention(q.contiguous(), st.k, st.v, kv_len=st.pos, max_kv_len=st.len,
                                          sm_scale=sm_scale, out_dtype=out_dtype or q.dtype)
        return out.unsqueeze(2)

    def get_seq_length(self, layer_idx: int = 0) -> int:
        if self.storage in ("tq_blocks", "tq_pages"):
            return self._blocks[layer_idx].len
        return self._store[layer_idx].len

    def get_max_length(self) -> Optional[int]:
        return None

    def get_usable_length(self, new_seq_length: int, layer_idx: int = 0) -> int:
        return self.get_seq_length(layer_idx)

    @property
    def seen_tokens(self) -> int:
        return self._seen_tokens

    def memory_summary(self) -> dict:
        if self.storage in ("tq_blocks", "tq_pages"):
            k_bits = {2: 10, 3: 14, 4: 18}[self.k_bits] * 8 / 32
            v_bits = 18 * 8 / 32
        else:
            k_bits = self.k_quantizer.memory_bits_per_element()
            v_bits = self.v_quantizer.memory_bits_per_element()
        tokens = self.get_seq_length()
        per_tok = self.n_kv_heads * self.head_dim
        k_bytes = tokens * per_tok * k_bits / 8
        v_bytes = tokens * per_tok * v_bits / 8
        fp16 = tokens * per_tok * 2 * 2
        return {"k_bits_per_elem": k_bits, "v_bits_per_elem": v_bits, "total_tokens": tokens,
                "compressed_bytes": (k_bytes + v_bytes) * self.n_layers, "fp16_bytes": fp16 * self.n_layers,
                "compression_ratio": fp16 / max(k_bytes + v_bytes, 1)}

    def __repr__(self) -> str:
        if self.storage in ("tq_blocks", "tq_pages"):
            return (f"LeanKVCache(layers={self.n_layers}, head_dim={self.head_dim}, storage={self.storage}, "
                    f"k=TQ{self.k_bits}_0, v=TQ4_0, tokens={self.get_seq_length()})")
        return (f"LeanKVCache(layers={self.n_layers}, head_dim={self.head_dim}, "
                f"k={self.k_quantizer}, v_rotate={self.v_rotate}, tokens={self.get_seq_length()})")
