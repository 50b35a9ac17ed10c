"""The allocation-free decode attention entry point.

tq_decode_attention_static_cuda serves callers that cannot allocate device
memory where they run attention (an allocator-free serving step, a plugin whose
host framework owns all device allocations): its work memory is a fixed static
device array inside the library.  These tests call it through the C ABI and
check it against tq_decode_attention_cuda (caller-provided workspace) on two
calls in a row with different inputs, so a stale scratch from the first call
would show up in the second.  Collected last on purpose.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from leankv_b200 import _lib as L
from leankv_b200 import attention, ops

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
RTOL = 2e-3     # the attention tests' tolerance


def _inputs(seed, B, Hq, Hkv, T, D=128):
    g = torch.Generator(device=DEV).manual_seed(seed)
    kc = ops.quantize(torch.randn(B, Hkv, T, D, device=DEV, generator=g), 4, fwht_head_dim=D)
    vc = ops.quantize(torch.randn(B, Hkv, T, D, device=DEV, generator=g), 4, fwht_head_dim=D)
    q = torch.randn(B, Hq, D, device=DEV, generator=g).half()
    lens = torch.randint(1, T + 1, (B,), device=DEV, generator=g, dtype=torch.int32)
    return q, kc, vc, lens


def _static_call(q, kc, vc, lens):
    lib = attention._bind()
    lib.tq_decode_attention_static_cuda.restype = C.c_int
    lib.tq_decode_attention_static_cuda.argtypes = [C.POINTER(attention.AttnArgs), C.c_void_p]
    out = torch.full(q.shape, float("nan"), dtype=torch.float32, device=DEV)
    lse = torch.full(q.shape[:2], float("nan"), dtype=torch.float32, device=DEV)
    a = attention.make_args(q, kc, vc, lens, 0, 0.0, True, True, out, lse)
    a.workspace, a.workspace_bytes = None, 0
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    L.check(lib.tq_decode_attention_static_cuda(C.byref(a), stream))
    return out, lse


def _compare(got, ref):
    g, r = got.cpu().numpy().astype(np.float64), ref.cpu().numpy().astype(np.float64)
    assert np.isfinite(g).all()
    assert np.abs(g - r).max() <= RTOL * np.abs(r).max() + 1e-5


def test_static_scratch_matches_workspace_entry_point_twice():
    for seed, shape in ((1, (4, 32, 8, 3000)), (2, (3, 16, 2, 778))):
        q, kc, vc, lens = _inputs(seed, *shape)
        out, lse = _static_call(q, kc, vc, lens)
        ref, lref = attention.decode_attention(q, kc, vc, kv_len=lens, return_lse=True)
        torch.cuda.synchronize()
        _compare(out, ref)
        _compare(lse, lref)


def test_static_scratch_rejects_oversized_arguments():
    lib = attention._bind()
    lib.tq_decode_attention_static_cuda.restype = C.c_int
    lib.tq_decode_attention_static_cuda.argtypes = [C.POINTER(attention.AttnArgs), C.c_void_p]
    a = attention.AttnArgs()
    a.batch, a.n_q_heads, a.n_kv_heads, a.head_dim = 4096, 64, 8, 128   # ~170 MB of partials
    a.k_type = a.v_type = 4
    a.kv_capacity = 1024
    a.q = a.out = a.k_cache = a.v_cache = 256
    assert lib.tq_decode_attention_static_cuda(C.byref(a), None) == 1     # TQ_ERROR_INVALID_VALUE
    assert b"fixed scratch" in lib.tq_last_error_string()
