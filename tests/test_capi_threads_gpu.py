"""The ggml drop-in names (src/ggml-tq.h:145-190) called from many host threads at once.

ggml's worker threads call quantize_row_* / dequantize_row_* on disjoint rows of one tensor
concurrently; the reference functions are pure, so that is safe there.  Here each call borrows a
host context (two streams and staging buffers) from a mutex-guarded pool, so concurrent calls run
on separate contexts.  16 threads call quantize_row_tq4_0, dequantize_row_tq4_0 and
quantize_row_tq3_0 on their own 4096-element rows, many times; every result must be bit-exact
with the reference C (oracle/_ref).  A second test prints the per-call latency at ggml row sizes
next to the reference C, which sets the row count below which a caller should batch rows.
"""
import ctypes as C
import threading
import time

import numpy as np
import pytest

from leankv_b200 import _lib as L

pytestmark = pytest.mark.gpu

K = 4096
THREADS, ITERS = 16, 12


def _p(a):
    return a.ctypes.data_as(C.c_void_p)


def _rows(seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal(K).astype(np.float32)
    x[rng.integers(0, K, 8)] *= 20.0
    return x


def test_drop_in_rows_from_16_threads(orc):
    if not orc.ref_available():
        pytest.fail("compiled reference library oracle/_ref is required")
    lib, ref = L.load(), orc.ref_lib()
    bad = []

    def worker(t):
        try:
            for it in range(ITERS):
                x = _rows(1000 * t + it)
                y4 = np.zeros((K // 32, 18), np.uint8)
                y3 = np.zeros((K // 32, 14), np.uint8)
                z = np.zeros(K, np.float32)
                lib.quantize_row_tq4_0(_p(x), _p(y4), K)
                lib.dequantize_row_tq4_0(_p(y4), _p(z), K)
                lib.quantize_row_tq3_0(_p(x), _p(y3), K)
                r4 = np.zeros_like(y4)
                r3 = np.zeros_like(y3)
                rz = np.zeros_like(z)
                ref.quantize_row_tq4_0(_p(x), _p(r4), K)
                ref.dequantize_row_tq4_0(_p(r4), _p(rz), K)
                ref.quantize_row_tq3_0(_p(x), _p(r3), K)
                if not (np.array_equal(y4, r4) and np.array_equal(y3, r3) and
                        np.array_equal(z.view(np.uint32), rz.view(np.uint32))):
                    bad.append((t, it))
        except Exception as e:   # noqa: BLE001 - reported below
            bad.append((t, repr(e)))

    ths = [threading.Thread(target=worker, args=(t,)) for t in range(THREADS)]
    for th in ths:
        th.start()
    for th in ths:
        th.join()
    assert not bad, bad[:5]


def test_drop_in_row_latency(orc):
    """Per-call latency of quantize_row_tq4_0 at ggml row sizes, this library (host pointers:
    copy in, kernel, copy out) against the reference C on one core (printed)."""
    lib, ref = L.load(), orc.ref_lib()
    for k in (128, 4096, 1 << 20):
        x = np.random.default_rng(k).standard_normal(k).astype(np.float32)
        y = np.zeros((k // 32, 18), np.uint8)
        r = np.zeros_like(y)
        n = max(3, min(200, (1 << 22) // k))
        for fn, out in ((lib.quantize_row_tq4_0, y), (ref.quantize_row_tq4_0, r)):
            fn(_p(x), _p(out), k)
        t0 = time.perf_counter()
        for _ in range(n):
            lib.quantize_row_tq4_0(_p(x), _p(y), k)
        ours = (time.perf_counter() - t0) / n
        t0 = time.perf_counter()
        for _ in range(n):
            ref.quantize_row_tq4_0(_p(x), _p(r), k)
        theirs = (time.perf_counter() - t0) / n
        assert np.array_equal(y, r)
        print(f"quantize_row_tq4_0 k={k}: {ours * 1e6:.1f} us here, {theirs * 1e6:.1f} us reference C (1 core)")
