"""The oracle is pinned before it is trusted.

* codec / FWHT restatement == the committed golden fixtures produced by the
  reference C (src/ggml-tq.c), bit for bit, including every edge case;
* the same against the freshly compiled reference C when oracle/_ref is built;
* TQ3 optimal rounding restatement == scripts/tq3_rounding.py (fixtures):
  identical codes and identical stored fp16 scales;
* the reference test suite's printed statistics (src/test-tq.c T2/T3/T6/T9)
  and the published rounding MSE table (docs/RESULTS.md:779-785) reproduce.
"""
import numpy as np
import pytest


def u32(a):
    return np.ascontiguousarray(a, dtype=np.float32).reshape(-1).view(np.uint32)


@pytest.mark.parametrize("t", [3, 4])
def test_codec_matches_reference_fixtures(golden, orc, t):
    g = golden["codec"]
    q = orc.quantize(t, g["x_rot"])
    assert np.array_equal(q, g[f"tq{t}_rot"])
    assert np.array_equal(u32(orc.dequantize(t, q)), u32(g[f"tq{t}_rot_deq"]))
    fw = orc.fwht(g["x_raw"], 128)
    assert np.array_equal(u32(fw), u32(g["fwht128_raw"]))
    assert np.array_equal(orc.quantize(t, fw), g[f"tq{t}_fused"])
    assert np.array_equal(u32(orc.dequantize(t, g[f"tq{t}_rand_bytes"])), u32(g[f"tq{t}_rand_bytes_deq"]))


def test_half_decoder_all_values(golden, orc):
    ref = golden["codec"]["half_decode_all"]
    got = np.array([orc.float_from_half(h) for h in range(65536)], np.float32)
    assert np.array_equal(u32(got), u32(ref))


def test_half_encoder_truncates(orc):
    # src/ggml-tq.h:39-48: truncation, flush below 2^-14, inf at/above 2^16
    assert orc.half_from_float(1.0) == 0x3C00
    assert orc.half_from_float(np.nextafter(np.float32(1.0), np.float32(2)) ) == 0x3C00
    assert orc.half_from_float(1.9999999) == 0x3FFF
    assert orc.half_from_float(2.0 ** -14) == 0x0400
    assert orc.half_from_float(2.0 ** -15) == 0x0000
    assert orc.half_from_float(-2.0 ** -15) == 0x8000
    assert orc.half_from_float(65535.0) == 0x7BFF
    assert orc.half_from_float(65536.0) == 0x7C00
    assert orc.half_from_float(float("inf")) == 0x7C00


def test_fwht_matches_reference_fixtures(golden, orc):
    g = golden["fwht"]
    for l2 in range(0, 11):
        hd = 1 << l2
        assert np.array_equal(u32(orc.fwht(g[f"x_{hd}"], hd)), u32(g[f"y_{hd}"])), hd


@pytest.mark.skipif("not __import__('oracle.oracle', fromlist=['x']).ref_available()")
def test_restatement_matches_compiled_reference_random(orc):
    rng = np.random.default_rng(5)
    for t in (3, 4):
        for scale in (1e-3, 1.0, 300.0):
            x = (rng.standard_normal(32 * 2048) * scale).astype(np.float32)
            x[rng.integers(0, x.size, 20)] *= 50
            assert np.array_equal(orc.quantize(t, x), orc.ref_quantize(t, x))
        rb = rng.integers(0, 256, (4096, orc.BLOCK_BYTES[t]), dtype=np.uint8)
        assert np.array_equal(u32(orc.dequantize(t, rb)), u32(orc.ref_dequantize(t, rb)))
    x = rng.standard_normal(8192).astype(np.float32)
    for hd in (2, 8, 64, 256, 1024, 4096):
        assert np.array_equal(u32(orc.fwht(x, hd)), u32(orc.ref_fwht(x, hd)))


def test_tq3_opt_matches_python_reference(golden, orc):
    g = golden["tq3_opt"]
    blocks, codes, scales = g["blocks"], g["codes"], g["scales"]
    code_mism = half_mism = 0
    for i in range(blocks.shape[0]):
        idx, d, _ = orc.tq3_opt_block(blocks[i], 2, init_f64=True)
        code_mism += not np.array_equal(idx, codes[i])
        half_mism += orc.half_from_float(np.float32(d)) != orc.half_from_float(np.float32(scales[i]))
    assert code_mism == 0
    assert half_mism == 0


def test_tq3_opt_c_init_agrees_with_python_init(golden, orc):
    """The GPU starts from the C float32 nearest assignment; on these blocks it converges identically."""
    b = golden["tq3_opt"]["blocks"]
    q_c, _ = orc.quantize_tq3_opt(b, 2, init_f64=False)
    q_p, _ = orc.quantize_tq3_opt(b, 2, init_f64=True)
    assert (q_c != q_p).any(axis=1).sum() <= 2


def test_tq3_opt_blocks_roundtrip_through_reference_dequant(golden, orc):
    b = golden["tq3_opt"]["blocks"][:500]
    q, moves = orc.quantize_tq3_opt(b, 2)
    assert moves > 0
    rec = orc.dequantize(3, q).reshape(b.shape)
    base = orc.dequantize(3, orc.quantize(3, b)).reshape(b.shape)
    assert np.mean((rec - b) ** 2) < np.mean((base - b) ** 2)


def test_published_rounding_table(golden):
    g = golden["tq3_opt"]
    assert round(float(g["mse_baseline"]), 4) == 0.0316
    assert round(float(g["mse_ls_scale"]), 4) == 0.0298
    assert round(float(g["mse_cd2"]), 4) == 0.0267
    assert round(float(g["mse_cd3"]), 4) == 0.0265


def test_testtq_known_answers(golden, orc):
    g = golden["testtq"]
    assert np.array_equal(orc.quantize(3, g["t2_x"]), g["t2_blocks"])
    assert np.array_equal(orc.quantize(4, g["t3_x"]), g["t3_blocks"])
    assert abs(float(g["t2_mse"]) - 4.2799e-4) < 5e-8 and abs(float(g["t2_cos"]) - 0.984973) < 1e-6
    assert abs(float(g["t3_mse"]) - 1.0023e-4) < 5e-8 and abs(float(g["t3_cos"]) - 0.996639) < 1e-6
    assert abs(float(g["t6_mse"]) - 1.32804e-3) < 5e-8
    assert abs(float(g["t9_cos"]) - 0.991655) < 1e-6
    rot = orc.fwht(g["t6_x"], 64)
    assert np.array_equal(u32(rot), u32(g["t6_rot"]))
    assert np.array_equal(orc.quantize(3, rot), g["t6_blocks"])
    assert np.array_equal(orc.quantize(3, orc.fwht(g["t9_k"], 64)), g["t9_blocks"])


def test_tq3_pack_layout(orc):
    # src/ggml-tq.c:26-43: byte0 = i0 | i1<<3 | (i2&3)<<6, byte1 = i2>>2 | i3<<1 | i4<<4 | (i5&1)<<7, ...
    rng = np.random.default_rng(0)
    for _ in range(50):
        idx = rng.integers(0, 8, 32).astype(np.uint8)
        x = np.array([-1.0, -0.6245203, -0.3513239, -0.1138989, 0.1138989, 0.3513239, 0.6245203, 1.0],
                     np.float32)[idx]
        x[0] = 1.0 if idx[0] == 7 else x[0]
        q = orc.quantize(3, np.where(np.abs(x).max() < 1, np.append(x[:-1], 1.0), x))
        qs = q[0, 2:]
        i = q_idx = np.zeros(32, np.uint8)
        for g in range(4):
            b0, b1, b2 = (int(v) for v in qs[3 * g:3 * g + 3])
            q_idx[8 * g:8 * g + 8] = [b0 & 7, (b0 >> 3) & 7, ((b0 >> 6) & 3) | ((b1 & 1) << 2), (b1 >> 1) & 7,
                                      (b1 >> 4) & 7, ((b1 >> 7) & 1) | ((b2 & 3) << 1), (b2 >> 2) & 7, (b2 >> 5) & 7]
        deq = orc.dequantize(3, q)
        lv = np.array([-1.0, -0.6245203, -0.3513239, -0.1138989, 0.1138989, 0.3513239, 0.6245203, 1.0], np.float32)
        d = orc.float_from_half(int(q[0, 0]) | int(q[0, 1]) << 8)
        assert np.array_equal(deq, lv[i] * np.float32(d))


def test_attention_oracle_matches_dense_softmax(orc):
    """The float64 attention restatement equals a direct numpy evaluation on dequantized K/V."""
    rng = np.random.default_rng(3)
    B, Hq, Hkv, D, T = 2, 4, 2, 64, 96
    q = rng.standard_normal((B, Hq, D)).astype(np.float32)
    kr = orc.fwht(rng.standard_normal((B, Hkv, T, D)).astype(np.float32), D)
    vr = orc.fwht(rng.standard_normal((B, Hkv, T, D)).astype(np.float32), D)
    kb = orc.quantize(4, kr).reshape(B, Hkv, T, D // 32, 18)
    vb = orc.quantize(3, vr).reshape(B, Hkv, T, D // 32, 14)
    lens = np.array([96, 37])
    out, lse = orc.decode_attention(q, kb, 4, vb, 3, Hkv, kv_len=lens)
    kd = orc.dequantize(4, kb).reshape(B, Hkv, T, D).astype(np.float64)
    vd = orc.dequantize(3, vb).reshape(B, Hkv, T, D).astype(np.float64)
    qr = orc.fwht(q, D).astype(np.float64)
    H = np.array([[1.0]])
    while H.shape[0] < D:
        H = np.block([[H, H], [H, -H]])
    H /= np.sqrt(D)
    for b in range(B):
        for h in range(Hq):
            g = h // (Hq // Hkv)
            n = lens[b]
            s = kd[b, g, :n] @ qr[b, h] / np.sqrt(D)
            p = np.exp(s - s.max())
            o = (p / p.sum()) @ vd[b, g, :n]
            np.testing.assert_allclose(out[b, h], H @ o, rtol=1e-5, atol=1e-6)
            np.testing.assert_allclose(lse[b, h], s.max() + np.log(p.sum()), rtol=1e-6)


def test_lse_combine_oracle(orc):
    rng = np.random.default_rng(4)
    o = rng.standard_normal((3, 5, 16)).astype(np.float32)
    lse = rng.standard_normal((3, 5)).astype(np.float32)
    lse[1, 2] = -np.inf
    out, lo = orc.lse_combine(o, lse)
    w = np.exp(lse - lse.max(0))
    np.testing.assert_allclose(out, (w[..., None] * o).sum(0) / w.sum(0)[..., None], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(lo, lse.max(0) + np.log(w.sum(0)), rtol=1e-6)


def test_tq2_dequantize_restatement_equals_reference(orc):
    """The restated TQ2_0 decoder (the decode attention's TQ2 keys) equals the reference
    dequantize_row_tq2_0 on random block bytes, every scale bit pattern included."""
    rng = np.random.default_rng(22)
    blocks = rng.integers(0, 256, size=(20000, 10), dtype=np.uint8)
    blocks[:, :2] = rng.integers(0, 256, size=(20000, 2), dtype=np.uint8)
    y = orc.dequantize(2, blocks)
    ref = orc.ref_dequantize(2, blocks)
    assert np.array_equal(np.isnan(y), np.isnan(ref))
    fin = ~np.isnan(ref)
    assert np.array_equal(y[fin], ref[fin])
