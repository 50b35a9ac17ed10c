"""GPU parity of the channel-permuted mixed-precision quantization with the
reference's own compiled src/ggml-tq-outlier.c: calibration (channel variances,
permutation, split), blocks and dequantized values bit-exact."""
import ctypes as C

import numpy as np
import pytest
import torch

from leankv_b200 import _lib as L
from leankv_b200 import ops

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _calib(n_tokens, hd, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((n_tokens, hd)).astype(np.float32)
    scales = np.exp(rng.standard_normal(hd)).astype(np.float32)   # distinct channel variances
    x *= scales
    x[:, rng.choice(hd, 5, replace=False)] *= 12.0
    return np.ascontiguousarray(x)


def _ref_config(orc, calib, frac, ot, nt):
    cfg = ops.OutlierConfig()
    orc.ref_lib().tq_identify_outliers(C.byref(cfg), calib.ctypes.data, calib.shape[0], calib.shape[1],
                                        C.c_float(frac), ot, nt)
    return cfg


def _fields(cfg):
    hd = cfg.head_dim
    return (cfg.head_dim, cfg.n_outlier, cfg.n_normal, cfg.outlier_tier, cfg.normal_tier, list(cfg.perm[:hd]),
            list(cfg.inv_perm[:hd]), np.array(cfg.channel_var[:hd], np.float32).view(np.uint32).tolist())


@pytest.mark.parametrize("hd", [64, 128, 256])
@pytest.mark.parametrize("frac,ot,nt", [(0.25, 1, 0), (0.1, 2, 1), (0.3, 2, 0), (0.0, 1, 0), (1.0, 2, 1)])
def test_identify_and_mixed_codec_bit_exact(orc, hd, frac, ot, nt):
    calib = _calib(700, hd, hd + int(frac * 100))
    ref = _ref_config(orc, calib, frac, ot, nt)
    got = ops.identify_outliers(torch.from_numpy(calib).to(DEV), frac, ot, nt)
    assert _fields(got) == _fields(ref)

    x = np.ascontiguousarray(_calib(257, hd, 7 * hd)[:257])
    ob, nb = ops.mixed_quantize(torch.from_numpy(x).to(DEV), got)
    ob, nb = ob.cpu().numpy(), nb.cpu().numpy()
    osz, nsz = C.c_size_t(), C.c_size_t()
    L.load().tq_mixed_buffer_sizes(C.byref(ref), C.byref(osz), C.byref(nsz))
    ro = np.zeros((x.shape[0], max(osz.value, 1)), np.uint8)
    rn = np.zeros((x.shape[0], max(nsz.value, 1)), np.uint8)
    ry = np.zeros_like(x)
    lib = orc.ref_lib()
    for v in range(x.shape[0]):
        lib.tq_mixed_quantize(x[v].ctypes.data, C.byref(ref), ro[v].ctypes.data, rn[v].ctypes.data)
        lib.tq_mixed_dequantize(ro[v].ctypes.data, rn[v].ctypes.data, C.byref(ref), ry[v].ctypes.data)
    assert np.array_equal(ob.reshape(x.shape[0], -1), ro[:, : osz.value])
    assert np.array_equal(nb.reshape(x.shape[0], -1), rn[:, : nsz.value])
    y = ops.mixed_dequantize(torch.from_numpy(ob).to(DEV), torch.from_numpy(nb).to(DEV), got).cpu().numpy()
    assert np.array_equal(y.view(np.uint32), ry.view(np.uint32))
    bits = {0: 2.5, 1: 3.5, 2: 4.5}
    expect = (got.n_outlier * bits[ot] + got.n_normal * bits[nt]) / hd
    assert abs(L.load().tq_mixed_effective_bpe(C.byref(got)) - expect) < 1e-6


def test_dropin_outlier_names(orc):
    lib = L.load()
    calib = _calib(300, 128, 3)
    cfg = ops.OutlierConfig()
    lib.tq_identify_outliers(C.byref(cfg), calib.ctypes.data, 300, 128, C.c_float(0.25), 1, 0)
    assert _fields(cfg) == _fields(_ref_config(orc, calib, 0.25, 1, 0))
    x = calib[5].copy()
    ob = np.zeros(14 * 1, np.uint8)
    nb = np.zeros(10 * 3, np.uint8)
    lib.tq_mixed_quantize(x.ctypes.data, C.byref(cfg), ob.ctypes.data, nb.ctypes.data)
    rob, rnb = np.zeros_like(ob), np.zeros_like(nb)
    orc.ref_lib().tq_mixed_quantize(x.ctypes.data, C.byref(cfg), rob.ctypes.data, rnb.ctypes.data)
    assert np.array_equal(ob, rob) and np.array_equal(nb, rnb)
    y = np.zeros(128, np.float32)
    lib.tq_mixed_dequantize(ob.ctypes.data, nb.ctypes.data, C.byref(cfg), y.ctypes.data)
    ry = np.zeros(128, np.float32)
    orc.ref_lib().tq_mixed_dequantize(rob.ctypes.data, rnb.ctypes.data, C.byref(cfg), ry.ctypes.data)
    assert np.array_equal(y.view(np.uint32), ry.view(np.uint32))
    p = np.zeros(128, np.float32)
    lib.tq_permute_channels(x.ctypes.data, p.ctypes.data, (C.c_int * 128)(*cfg.perm[:128]), 128)
    assert np.array_equal(p, x[np.array(cfg.perm[:128])])
    back = np.zeros(128, np.float32)
    lib.tq_unpermute_channels(p.ctypes.data, back.ctypes.data, (C.c_int * 128)(*cfg.inv_perm[:128]), 128)
    assert np.array_equal(back, x)
    u = ops.OutlierConfig()
    lib.tq_outlier_config_init_uniform(C.byref(u), 64, 0)
    assert u.n_outlier == 0 and u.n_normal == 64 and list(u.perm[:64]) == list(range(64))
