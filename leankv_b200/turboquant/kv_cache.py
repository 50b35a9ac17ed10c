"""LeanKVCache: the prototype's HuggingFace-style quantized KV cache
(prototype/turboquant/kv_cache.py:31-245) with GPU-resident packed storage.

Keys: rotation + Lloyd-Max (+ QJL) through TurboQuantizer; values: Lloyd-Max of
the L2-normalised vector, rotated only when v_rotation is not "none".
update() returns every cached key (rotated space) and value (original space)
dequantized, like the prototype.  Instead of a Python list of per-call pieces
that is concatenated on every read, each layer keeps its packed codes in device
buffers laid out [token][batch][head] that grow by doubling, so appends are one
copy and the read-out is one decode launch over a contiguous range.
"""
from __future__ import annotations

from typing import Any, Dict, List, Optional, Tuple

import torch

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


class LeanKVCache:
    """Quantized KV cache with the interface of transformers.DynamicCache (update / get_seq_length ...)."""

    def __init__(self, n_layers: int, head_dim: int, n_kv_heads: int = 1, k_bits=3, v_bits=4,
                 k_rotation: str = "randomized_hadamard", v_rotation: str = "none", use_qjl: bool = True,
                 seed: int = 42, device: str = "cuda"):
        self.n_layers = n_layers
        self.head_dim = head_dim
        self.n_kv_heads = n_kv_heads
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
    @property
    def k_cache(self) -> List[List[QuantizedKV]]:
        return [[s.view("k")] if s.len else [] for s in self._store]

    @property
    def v_cache(self) -> List[List[QuantizedKV]]:
        return [[s.view("v")] if s.len else [] for s in self._store]

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, layer_idx: int,
               cache_kwargs: Optional[Dict[str, Any]] = None) -> Tuple[torch.Tensor, torch.Tensor]:
        """Store new (batch, n_kv_heads, new_seq, head_dim) K/V; return all cached K (rotated) and V."""
        if layer_idx == 0:
            self._seen_tokens += key_states.shape[2]
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

    def get_seq_length(self, layer_idx: int = 0) -> int:
        return self._store[layer_idx].len

    def get_max_length(self) -> Optional[int]:
        return None

    def get_usable_length(self, new_seq_length: int, layer_idx: int = 0) -> int:
        return self.get_seq_length(layer_idx)

    @property
    def seen_tokens(self) -> int:
        return self._seen_tokens

    def memory_summary(self) -> dict:
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
        return (f"LeanKVCache(layers={self.n_layers}, head_dim={self.head_dim}, "
                f"k={self.k_quantizer}, v_rotate={self.v_rotate}, tokens={self.get_seq_length()})")
