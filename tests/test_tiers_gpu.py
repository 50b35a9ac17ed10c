"""GPU parity of the TQ2_0 type, the tier requantization and the randomized Hadamard
transform with the reference's own compiled C (src/ggml-tq.c, built by oracle/Makefile).

Bar: bit-exact codes, fp16 scales, dequantized floats and transformed floats.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from leankv_b200 import _lib as L
from leankv_b200 import ops

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _data(n, seed, outliers=True):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal(n).astype(np.float32)
    if outliers:
        x[rng.integers(0, n, n // 97)] *= 40.0
    return x


def _edge_rows():
    rng = np.random.default_rng(3)
    rows = [np.zeros(32, np.float32), np.full(32, 0.6498857, np.float32), np.linspace(-1, 1, 32).astype(np.float32)]
    r = rng.standard_normal(32).astype(np.float32); r[5] = np.nan; rows.append(r)
    r = rng.standard_normal(32).astype(np.float32); r[7] = np.inf; rows.append(r)
    rows.append(np.full(32, np.nan, np.float32))
    rows.append((rng.standard_normal(32) * 1e-39).astype(np.float32))
    rows.append((rng.standard_normal(32) * 7e4).astype(np.float32))
    r = (np.array([-0.6498857, 0.0, 0.6498857, -0.2997714] * 8, np.float32) * 3.0); rows.append(r)
    return np.concatenate(rows)


@pytest.mark.parametrize("kind", ["random", "edge"])
def test_tq2_quantize_dequantize_bit_exact(orc, kind):
    x = _data(32 * 4096, 11) if kind == "random" else _edge_rows()
    ref = orc.ref_quantize(2, x)
    got = ops.quantize(torch.from_numpy(x).to(DEV), 2).cpu().numpy().reshape(ref.shape)
    assert np.array_equal(got, ref)
    y = ops.dequantize(torch.from_numpy(ref).to(DEV), 2).cpu().numpy().reshape(-1)
    assert np.array_equal(y.view(np.uint32), orc.ref_dequantize(2, ref).view(np.uint32))


def test_tq2_random_bytes_dequantize(orc):
    rng = np.random.default_rng(4)
    b = rng.integers(0, 256, (777, 10), dtype=np.uint8)
    y = ops.dequantize(torch.from_numpy(b).to(DEV), 2).cpu().numpy().reshape(-1)
    assert np.array_equal(y.view(np.uint32), orc.ref_dequantize(2, b).view(np.uint32))


@pytest.mark.parametrize("src,dst", [(4, 3), (3, 2), (4, 2)])
@pytest.mark.parametrize("kind", ["quantized", "random_bytes"])
def test_requantize_bit_exact(orc, src, dst, kind):
    if kind == "quantized":
        blocks = orc.ref_quantize(src, np.concatenate([_data(32 * 3001, 5), _edge_rows()]))
    else:
        rng = np.random.default_rng(src * 10 + dst)
        blocks = rng.integers(0, 256, (4096, {3: 14, 4: 18}[src]), dtype=np.uint8)
        blocks[:, 1] &= 0x7B   # keep most scales finite; some exponent-31 fields remain via bit 2
    ref = orc.ref_requantize(src, dst, blocks)
    got = ops.requantize(torch.from_numpy(blocks).to(DEV), src, dst).cpu().numpy()
    assert np.array_equal(got, ref)


def test_requantize_chain_equals_direct_path(orc):
    blocks4 = orc.ref_quantize(4, _data(32 * 2048, 9))
    b = torch.from_numpy(blocks4).to(DEV)
    chain = ops.requantize(ops.requantize(b, 4, 3), 3, 2).cpu().numpy()
    assert np.array_equal(chain, orc.ref_requantize(3, 2, orc.ref_requantize(4, 3, blocks4)))


@pytest.mark.parametrize("head_dim,row_len", [(32, 32), (64, 256), (128, 1024), (256, 256), (1024, 2048)])
@pytest.mark.parametrize("seed", [42, 0xFFFFFFF0])
def test_randomized_hadamard_bit_exact(orc, head_dim, row_len, seed):
    x = _data(row_len * 37, head_dim + row_len)
    ref = orc.ref_randomized_fwht(x, row_len, head_dim, seed)
    t = torch.from_numpy(x).to(DEV)
    ops.hadamard_randomized_(t, head_dim, seed, row_len=row_len)
    assert np.array_equal(t.cpu().numpy().view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("qtype,passes", [(2, 0), (3, 0), (4, 0), (3, 2)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_fused_randomized_quantize(orc, qtype, passes, dtype):
    head_dim, row_len, seed = 128, 1024, 7
    x = torch.from_numpy(_data(row_len * 300, qtype)).to(DEV).to(dtype)
    got = ops.quantize(x, qtype, fwht_head_dim=head_dim, opt_passes=passes, rht_seed=seed, row_len=row_len)
    xr = orc.ref_randomized_fwht(x.float().cpu().numpy(), row_len, head_dim, seed)
    if passes:
        ref = ops.quantize(torch.from_numpy(xr).to(DEV), 3, opt_passes=passes).cpu().numpy()
    else:
        ref = orc.ref_quantize(qtype, xr)
    assert np.array_equal(got.cpu().numpy().reshape(ref.shape), ref)


def test_dropin_tier_names_match_reference(orc):
    lib = L.load()
    x = _data(32 * 256, 21)
    y = np.zeros((256, 10), np.uint8)
    lib.quantize_row_tq2_0_ref(x.ctypes.data, y.ctypes.data, x.size)
    assert np.array_equal(y, orc.ref_quantize(2, x))
    d = np.zeros(x.size, np.float32)
    lib.dequantize_row_tq2_0(y.ctypes.data, d.ctypes.data, x.size)
    assert np.array_equal(d.view(np.uint32), orc.ref_dequantize(2, y).view(np.uint32))
    b4 = orc.ref_quantize(4, x)
    for a, b, fn in ((4, 3, lib.requantize_tq4_to_tq3), (4, 2, lib.requantize_tq4_to_tq2)):
        out = np.zeros((256, {3: 14, 2: 10}[b]), np.uint8)
        fn(b4.ctypes.data, out.ctypes.data, x.size)
        assert np.array_equal(out, orc.ref_requantize(a, b, b4))
    b3 = orc.ref_quantize(3, x)
    out = np.zeros((256, 10), np.uint8)
    lib.requantize_tq3_to_tq2(b3.ctypes.data, out.ctypes.data, x.size)
    assert np.array_equal(out, orc.ref_requantize(3, 2, b3))
    z = x[:512].copy()
    lib.randomized_hadamard_transform_row(z.ctypes.data, 512, 128, C.c_uint32(99))
    assert np.array_equal(z.view(np.uint32), orc.ref_randomized_fwht(x[:512], 512, 128, 99).view(np.uint32))
    w = x[:64].copy()
    lib.randomized_hadamard_transform(w.ctypes.data, 64, C.c_uint32(5))
    assert np.array_equal(w.view(np.uint32), orc.ref_randomized_fwht(x[:64], 64, 64, 5).view(np.uint32))
