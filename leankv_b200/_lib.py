"""ctypes binding of libleankv_tq.so (the C ABI declared in include/leankv_tq.h).

The library is loaded from the package directory (leankv_b200/_lib/).  There
is no CPU fallback: if the library or a CUDA device is missing, calls raise.
"""
from __future__ import annotations

import ctypes as C
import os
import re

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "_lib", "libleankv_tq.so")
HEADER_DIR = os.path.join(os.path.dirname(PKG), "include")

# tq_status values (include/leankv_tq.h)
TQ_SUCCESS = 0
STATUS_NAMES = {0: "TQ_SUCCESS", 1: "TQ_ERROR_INVALID_VALUE", 2: "TQ_ERROR_UNSUPPORTED", 3: "TQ_ERROR_MISALIGNED",
                4: "TQ_ERROR_CUDA", 5: "TQ_ERROR_OUT_OF_MEMORY", 6: "TQ_ERROR_NO_DEVICE", 7: "TQ_ERROR_TIMEOUT"}
# tq_dtype / tq_type
DTYPE_F32, DTYPE_F16, DTYPE_BF16 = 0, 1, 2
TQ_PEER_HANDLE_BYTES = 64   # bytes of a tq_peer_exchange_create handle
TYPE_TQ2_0, TYPE_TQ3_0, TYPE_TQ4_0 = 2, 3, 4
BLOCK_BYTES = {TYPE_TQ2_0: 10, TYPE_TQ3_0: 14, TYPE_TQ4_0: 18}
QK = 32


class TQError(RuntimeError):
    """A libleankv_tq call returned a status other than TQ_SUCCESS."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


_lib: C.CDLL | None = None

_v, _i64, _i32, _f32 = C.c_void_p, C.c_int64, C.c_int, C.c_float

# name -> (restype, argtypes)
SIGNATURES = {
    # drop-in names (src/ggml-tq.h)
    "quantize_row_tq3_0_ref": (None, [_v, _v, _i64]),
    "quantize_row_tq4_0_ref": (None, [_v, _v, _i64]),
    "quantize_row_tq3_0": (None, [_v, _v, _i64]),
    "quantize_row_tq4_0": (None, [_v, _v, _i64]),
    "quantize_row_tq3_0_opt": (None, [_v, _v, _i64]),
    "dequantize_row_tq3_0": (None, [_v, _v, _i64]),
    "dequantize_row_tq4_0": (None, [_v, _v, _i64]),
    "hadamard_transform": (None, [_v, _i32]),
    "hadamard_transform_row": (None, [_v, _i32, _i32]),
    "quantize_row_tq2_0_ref": (None, [_v, _v, _i64]),
    "quantize_row_tq2_0": (None, [_v, _v, _i64]),
    "dequantize_row_tq2_0": (None, [_v, _v, _i64]),
    "requantize_tq4_to_tq3": (None, [_v, _v, _i64]),
    "requantize_tq3_to_tq2": (None, [_v, _v, _i64]),
    "requantize_tq4_to_tq2": (None, [_v, _v, _i64]),
    "randomized_hadamard_transform": (None, [_v, _i32, C.c_uint32]),
    "randomized_hadamard_transform_row": (None, [_v, _i32, _i32, C.c_uint32]),
    # status
    "tq_status_string": (C.c_char_p, [_i32]),
    "tq_last_error_string": (C.c_char_p, []),
    "tq_abi_version": (_i32, []),
    # device API
    "tq_quantize_cuda": (_i32, [_i32, _v, _i32, _v, _i64, _i32, _i32, _v]),
    "tq_dequantize_cuda": (_i32, [_i32, _v, _v, _i32, _i64, _v]),
    "tq_hadamard_cuda": (_i32, [_v, _i64, _i32, _v]),
    "tq_hadamard_randomized_cuda": (_i32, [_v, _i64, _i32, _i32, C.c_uint32, _v]),
    "tq_quantize_randomized_cuda": (_i32, [_i32, _v, _i32, _v, _i64, _i32, _i32, C.c_uint32, _i32, _v]),
    "tq_requantize_cuda": (_i32, [_i32, _v, _i32, _v, _i64, _v]),
    # host API
    "tq_quantize_host": (_i32, [_i32, _v, _i32, _v, _i64, _i32, _i32]),
    "tq_dequantize_host": (_i32, [_i32, _v, _v, _i32, _i64]),
    "tq_hadamard_host": (_i32, [_v, _i64, _i32]),
    "tq_hadamard_randomized_host": (_i32, [_v, _i64, _i32, _i32, C.c_uint32]),
    "tq_requantize_host": (_i32, [_i32, _v, _i32, _v, _i64]),
    # decode attention (argument block pointer; leankv_b200.attention binds the struct type)
    "tq_decode_attention_workspace_size": (C.c_size_t, [_v]),
    "tq_decode_attention_cuda": (_i32, [_v, _v]),
    "tq_decode_attention_static_cuda": (_i32, [_v, _v]),
    "tq_decode_attention_paged_cuda": (_i32, [_v, _v, _v]),
    "tq_lse_combine_cuda": (_i32, [_i32, _i64, _i32, _v, _v, _v, _v, _v]),
    "tq_lse_merge_cuda": (_i32, [_i32, _i64, _i32, _v, _i64, _v, _i64, _v, _i32, _v, _v]),
    # outlier channels (mixed precision); config pointers are host struct pointers
    "tq_identify_outliers": (None, [_v, _v, _i32, _i32, _f32, _i32, _i32]),
    "tq_outlier_config_init_uniform": (None, [_v, _i32, _i32]),
    "tq_mixed_buffer_sizes": (None, [_v, _v, _v]),
    "tq_mixed_effective_bpe": (_f32, [_v]),
    "tq_mixed_quantize": (None, [_v, _v, _v, _v]),
    "tq_mixed_dequantize": (None, [_v, _v, _v, _v]),
    "tq_permute_channels": (None, [_v, _v, _v, _i32]),
    "tq_unpermute_channels": (None, [_v, _v, _v, _i32]),
    "tq_outlier_identify_cuda": (_i32, [_v, _v, _i32, _i32, _f32, _i32, _i32, _v]),
    "tq_mixed_quantize_cuda": (_i32, [_v, _v, _i32, _i64, _v, _v, _v]),
    "tq_mixed_dequantize_cuda": (_i32, [_v, _v, _v, _i64, _v, _v]),
    # TQ2_1 blocks (the fork's static mixed-precision type)
    "tq_quantize_tq2_1_cuda": (_i32, [_v, _i32, _v, _i64, _v]),
    "tq_dequantize_tq2_1_cuda": (_i32, [_v, _v, _i64, _v]),
    # prototype vector codec (levels / boundaries are host float arrays)
    "tq_proto_encode_cuda": (_i32, [_v, _i32, _v, _i64, _i32, _i32, _v, _i32, _i32, _v, _v, _v, _v, _v, _v, _v]),
    "tq_proto_decode_cuda": (_i32, [_v, _v, _i64, _i32, _i32, _v, _v, _i32, _v, _i32, _v, _v, _v]),
    # KV-cache append
    "tq_kv_append_cuda": (_i32, [_i32, _v, _i32, _v, _i32, _i32, _i32, _i64, _i64, _v, _i32, _i32, _v, _v]),
    "tq_kv_append_paged_cuda": (_i32, [_i32, _v, _i32, _v, _i32, _i32, _i32, _v, _i64, _v, _i32, _i32, _v, _v]),
    # split-sequence merge over peer memory (exchange handles are opaque pointers)
    "tq_peer_exchange_create": (_i32, [_i32, _i32, _i64, _i32, C.c_uint32, _v, _v]),
    "tq_peer_exchange_connect": (_i32, [_v, _v]),
    "tq_peer_exchange_merge": (_i32, [_v, _v, _v, _i32, _v, _v]),
    "tq_peer_exchange_attention": (_i32, [_v, _v, _v, _i32, _v, _v]),
    "tq_peer_exchange_status": (_i32, [_v, _v]),
    "tq_peer_exchange_disconnect": (_i32, [_v]),
    "tq_peer_exchange_destroy": (_i32, [_v]),
}


def load() -> C.CDLL:
    """Load (once) and return the library; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing; build it with `python -m leankv_b200.build`")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            if hasattr(L, name):
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
        _lib = L
    return _lib


def check(status: int) -> None:
    if status != TQ_SUCCESS:
        msg = load().tq_last_error_string().decode(errors="replace")
        raise TQError(status, msg or load().tq_status_string(status).decode())


def header_functions() -> list[str]:
    """Every function name declared in include/*.h (for export checks)."""
    names = []
    for fn in sorted(os.listdir(HEADER_DIR)):
        if not fn.endswith(".h"):
            continue
        text = open(os.path.join(HEADER_DIR, fn)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        text = re.sub(r"//[^\n]*", "", text)
        text = re.sub(r"^\s*#.*$", "", text, flags=re.M)
        for m in re.finditer(r"\b([A-Za-z_][A-Za-z0-9_]*)\s*\(([^;{}()]*(?:\([^()]*\)[^;{}()]*)*)\)\s*;", text):
            name = m.group(1)
            if name in ("if", "while", "for", "return", "sizeof", "typedef"):
                continue
            names.append(name)
    return sorted(set(names))
