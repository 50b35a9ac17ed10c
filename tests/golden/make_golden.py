"""Generate the golden fixtures in tests/golden/ from the reference itself.

Run where the reference tree is available (it is read, never modified):

    python tests/golden/make_golden.py --reference <reference checkout>

Sources of truth:
  * the reference C (src/ggml-tq.c) compiled unchanged by oracle/Makefile into
    oracle/_ref/libggml_tq_ref.so: FWHT, TQ3_0 / TQ4_0 quantize and dequantize;
  * scripts/tq3_rounding.py imported from the reference tree: TQ3 optimal
    rounding (quantize_coord_descent) and its published MSE table;
  * the input generator of src/test-tq.c, restated in gen_testtq_inputs.c, so
    the reference test suite's printed statistics become known answers.

Fixtures (all .npz):
  codec.npz     edge-case and random rows -> reference codes / dequant values
  fwht.npz      rows for head_dim 1..1024 -> reference hadamard_transform_row
  tq3_opt.npz   blocks -> Python coordinate-descent codes and float64 scales
  testtq.npz    test-tq T2/T3/T6/T9 inputs, reference outputs and statistics
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import oracle as O  # noqa: E402

TQ4_B = np.array([-0.8786519, -0.6748221, -0.5261490, -0.4025170, -0.2928009, -0.1913257, -0.0945769, 0.0,
                  0.0945769, 0.1913257, 0.2928009, 0.4025170, 0.5261490, 0.6748221, 0.8786519], np.float32)
TQ3_B = np.array([-0.8122602, -0.4879221, -0.2326114, 0.0, 0.2326114, 0.4879221, 0.8122602], np.float32)


def edge_rows(rng: np.random.Generator) -> np.ndarray:
    """Already-rotated rows (each 32 elements = one block) that exercise every branch."""
    rows = []
    rows.append(np.zeros(32, np.float32))                                   # amax == 0
    r = rng.standard_normal(32).astype(np.float32); r[5] = np.nan; rows.append(r)   # NaN ignored by amax
    r = rng.standard_normal(32).astype(np.float32); r[7] = np.inf; rows.append(r)   # id = 0, inf*0 = NaN
    r = rng.standard_normal(32).astype(np.float32); r[9] = -np.inf; rows.append(r)
    rows.append(np.full(32, np.nan, np.float32))                             # all NaN
    rows.append((rng.standard_normal(32) * 1e-39).astype(np.float32))       # subnormal amax -> id = inf
    rows.append((rng.standard_normal(32) * 1e-6).astype(np.float32))        # fp16 scale flushed to 0
    rows.append((rng.standard_normal(32) * 7e4).astype(np.float32))         # fp16 scale -> inf field
    rows.append((rng.standard_normal(32) * 6.0e4).astype(np.float32))
    r = np.zeros(32, np.float32); r[0] = 1.0; r[1:16] = TQ4_B; r[16:31] = -TQ4_B; rows.append(r)  # exact ties
    r = np.zeros(32, np.float32); r[0] = -1.0; r[1:8] = TQ3_B; r[8:15] = -TQ3_B; r[15] = -0.0; rows.append(r)
    r = np.zeros(32, np.float32); r[0] = 2.0; r[1:16] = 2 * TQ4_B; r[16:31] = np.nextafter(2 * TQ4_B, 9); rows.append(r)
    r = np.zeros(32, np.float32); r[3] = 3.0; rows.append(r)                # single spike
    rows.append(np.full(32, -0.0, np.float32))
    rows.append(np.full(32, 0.37, np.float32))                              # constant block
    r = np.linspace(-1, 1, 32).astype(np.float32); rows.append(r)
    for _ in range(48):
        rows.append((rng.standard_normal(32) * rng.uniform(0.01, 10)).astype(np.float32))
    return np.stack(rows)


def raw_rows(rng: np.random.Generator, n_tok: int, heads: int, hd: int) -> np.ndarray:
    """N(0,1) K rows with 4 outlier channels per head scaled x20 (the codec workload's distribution)."""
    x = rng.standard_normal((n_tok, heads, hd)).astype(np.float32)
    for h in range(heads):
        ch = rng.choice(hd, 4, replace=False)
        x[:, h, ch] *= 20.0
    return x.reshape(n_tok, heads * hd)


def make_codec(out: str) -> None:
    rng = np.random.default_rng(1234)
    x_rot = edge_rows(rng)
    x_raw = raw_rows(rng, 16, 8, 128)
    fw = O.ref_fwht(x_raw, 128)
    blob = {"x_rot": x_rot, "x_raw": x_raw, "fwht128_raw": fw}
    for t in (3, 4):
        q = O.ref_quantize(t, x_rot)
        blob[f"tq{t}_rot"] = q
        blob[f"tq{t}_rot_deq"] = O.ref_dequantize(t, q)
        qf = O.ref_quantize(t, fw)
        blob[f"tq{t}_fused"] = qf
        blob[f"tq{t}_fused_deq"] = O.ref_dequantize(t, qf)
        rb = rng.integers(0, 256, size=(512, O.BLOCK_BYTES[t]), dtype=np.uint8)
        blob[f"tq{t}_rand_bytes"] = rb
        blob[f"tq{t}_rand_bytes_deq"] = O.ref_dequantize(t, rb)
    # every fp16 scale value decoded by the reference (code 15 = level +1.0, so y == d)
    halves = np.arange(65536, dtype=np.uint32)
    blk = np.zeros((65536, 18), np.uint8)
    blk[:, 0] = halves & 0xFF
    blk[:, 1] = halves >> 8
    blk[:, 2:] = 0xFF
    blob["half_decode_all"] = O.ref_dequantize(4, blk).reshape(65536, 32)[:, 0].copy()
    np.savez_compressed(out, **blob)


def make_fwht(out: str) -> None:
    rng = np.random.default_rng(99)
    blob = {}
    for l2 in range(0, 11):
        hd = 1 << l2
        n = max(hd, 64) * 3
        x = (rng.standard_normal(n) * rng.uniform(0.1, 5)).astype(np.float32)
        blob[f"x_{hd}"] = x
        blob[f"y_{hd}"] = O.ref_fwht(x, hd)
    np.savez_compressed(out, **blob)


def make_tq3_opt(out: str, reference: str) -> None:
    sys.path.insert(0, os.path.join(reference, "scripts"))
    import tq3_rounding as T  # the reference's own prototype

    # the script's own data (np.random.seed(42), scripts/tq3_rounding.py:154-162)
    np.random.seed(42)
    gauss = np.random.randn(10000, 32).astype(np.float64)
    heavy = np.random.standard_t(df=5, size=(10000, 32))
    # published table docs/RESULTS.md:779-785 on the Gaussian set
    mse = {}
    for name, fn, kw in (("baseline", T.quantize_baseline, {}), ("ls_scale", T.quantize_optimal_scale, {}),
                         ("cd2", T.quantize_coord_descent, {"n_passes": 2}),
                         ("cd3", T.quantize_coord_descent, {"n_passes": 3})):
        errs = [np.mean((b - fn(b.copy(), **kw)[0]) ** 2) for b in gauss]
        mse[name] = float(np.mean(errs))
    # float32 blocks (what the C path sees) run through the float64 Python
    rng = np.random.default_rng(7)
    sets = [gauss[:800].astype(np.float32), heavy[:800].astype(np.float32),
            (rng.standard_t(4, size=(300, 32)) * np.exp(rng.standard_normal((300, 1)))).astype(np.float32)]
    edge = np.zeros((6, 32), np.float32)
    edge[1, 3] = 2.0                                  # single spike
    edge[2, :] = 0.5                                  # constant
    edge[3, :] = np.linspace(-1, 1, 32)
    edge[4, ::2] = 1.0; edge[4, 1::2] = -0.1138989    # ties around the inner levels
    edge[5, :] = -TQ3_B[np.arange(32) % 7] * 3.0
    sets.append(edge)
    blocks = np.concatenate(sets)
    codes = np.zeros(blocks.shape, np.uint8)
    scales = np.zeros(blocks.shape[0], np.float64)
    for i, b in enumerate(blocks):
        _, d, idx = T.quantize_coord_descent(b.astype(np.float64), n_passes=2, try_all_levels=False)
        codes[i] = idx
        scales[i] = d
    np.savez_compressed(out, blocks=blocks, codes=codes, scales=scales,
                        mse_baseline=mse["baseline"], mse_ls_scale=mse["ls_scale"],
                        mse_cd2=mse["cd2"], mse_cd3=mse["cd3"])


def make_testtq(out: str) -> None:
    with tempfile.TemporaryDirectory() as td:
        exe = os.path.join(td, "gen")
        subprocess.run(["gcc", "-O2", "-std=c11", "-o", exe, os.path.join(HERE, "gen_testtq_inputs.c"), "-lm"],
                       check=True)
        raw = np.frombuffer(subprocess.run([exe], check=True, capture_output=True).stdout, np.float32)
    t2, t3, t6, k9, q9 = np.split(raw, np.cumsum([1024, 1024, 256, 128 * 64]))

    def stats(a, b):
        a = a.astype(np.float64); b = b.astype(np.float64)
        mse = np.float32(np.sum((a - b) ** 2) / a.size)
        cos = np.float32(np.dot(a, b) / (np.sqrt(np.dot(a, a)) * np.sqrt(np.dot(b, b))))
        return mse, cos

    blob = {"t2_x": t2, "t3_x": t3, "t6_x": t6, "t9_k": k9, "t9_q": q9}
    q = O.ref_quantize(3, t2); d = O.ref_dequantize(3, q)
    blob.update(t2_blocks=q, t2_deq=d)
    blob["t2_mse"], blob["t2_cos"] = stats(t2, d)
    q = O.ref_quantize(4, t3); d = O.ref_dequantize(4, q)
    blob.update(t3_blocks=q, t3_deq=d)
    blob["t3_mse"], blob["t3_cos"] = stats(t3, d)
    rot = O.ref_fwht(t6, 64); q = O.ref_quantize(3, rot); d = O.ref_dequantize(3, q); back = O.ref_fwht(d, 64)
    blob.update(t6_rot=rot, t6_blocks=q, t6_restored=back)
    blob["t6_mse"], blob["t6_cos"] = stats(t6, back)
    k_rot = O.ref_fwht(k9, 64); q_rot = O.ref_fwht(q9, 64)
    q = O.ref_quantize(3, k_rot); kd = O.ref_dequantize(3, q).reshape(128, 64)
    s_orig = k9.reshape(128, 64) @ q9
    s_tq = kd @ q_rot
    blob.update(t9_k_rot=k_rot, t9_q_rot=q_rot, t9_blocks=q)
    blob["t9_cos"] = stats(s_orig, s_tq)[1]
    np.savez_compressed(out, **blob)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="root of the reference checkout (read only)")
    a = ap.parse_args()
    if not os.path.isdir(a.reference):
        sys.exit("reference tree not found; fixtures are generated where it is mounted")
    O.build(os.path.join(a.reference, "src"))
    make_codec(os.path.join(HERE, "codec.npz"))
    make_fwht(os.path.join(HERE, "fwht.npz"))
    make_tq3_opt(os.path.join(HERE, "tq3_opt.npz"), a.reference)
    make_testtq(os.path.join(HERE, "testtq.npz"))
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)), "bytes")


if __name__ == "__main__":
    main()
