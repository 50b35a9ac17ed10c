"""GPU parity of the fused decode attention.

Reference: the float64 oracle (reference dequantization + FWHT + exact softmax),
and at full size a torch float32 evaluation on caches dequantized by the
bit-exact dequantizer.  Every cache is generated as the configs specify: N(0,1)
rows with 4 outlier channels per KV head scaled x20, rotated and quantized.
Tolerance (floating-point kernel, fp16 tensor-core operands, fp32
accumulation): max |out - ref| <= 1e-3 * max |ref| + 1e-5, and
|lse - lse_ref| <= 1e-3 * max(1, |lse_ref|).  The kernel splits both score
operands into fp16 hi + lo parts (q~ and the K codebook) and forms P * d_V in
fp32 before one fp16 rounding, so what remains is the fp16 rounding of the V
codebook (at most 3.1e-4 relative) and of P * d_V (2^-11).
"""
import numpy as np
import pytest
import torch

from leankv_b200 import attention, ops

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
RTOL = 1e-3


def outlier_normal(shape, generator, device=DEV):
    """N(0,1) [..., Hkv, T, D] with 4 outlier channels per KV head scaled x20 (the config-1 generator)."""
    x = torch.randn(*shape, generator=generator, device=device)
    H, D = shape[-3], shape[-1]
    for h in range(H):
        ch = torch.randperm(D, generator=generator, device=device)[:4]
        x[..., h, :, ch] *= 20.0
    return x


def make_cache(B, Hkv, T, D, seed, qtype=4, outliers=True):
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = torch.randn(B, Hkv, T, D, generator=g)
    if outliers:
        for h in range(Hkv):
            ch = torch.randperm(D, generator=g)[:4]
            x[:, h, :, ch] *= 20.0
    blocks = ops.quantize(x.to(DEV).contiguous(), qtype, fwht_head_dim=D)   # rotated + quantized
    return blocks   # [B, Hkv, T, D/32, bb]


def check(out, ref, lse=None, lse_ref=None):
    out = np.asarray(out, np.float64)
    ref = np.asarray(ref, np.float64)
    err = np.abs(out - ref).max()
    tol = RTOL * np.abs(ref).max() + 1e-5
    assert err <= tol, f"max abs err {err:.3g} > tol {tol:.3g}"
    if lse is not None:
        fin = np.isfinite(lse_ref)
        assert np.array_equal(np.isfinite(lse), fin)
        d = np.abs(np.asarray(lse, np.float64)[fin] - lse_ref[fin]).max() if fin.any() else 0.0
        assert d <= RTOL * max(1.0, np.abs(lse_ref[fin]).max() if fin.any() else 1.0)
    return err / max(np.abs(ref).max(), 1e-30)


@pytest.mark.parametrize("grp", [1, 2, 3, 4, 6, 8])
def test_attention_vs_oracle_grp(orc, grp):
    B, Hkv, T, D = 2, 2, 700, 128
    Hq = Hkv * grp
    kc = make_cache(B, Hkv, T, D, 10 + grp)
    vc = make_cache(B, Hkv, T, D, 20 + grp)
    q = torch.randn(B, Hq, D, generator=torch.Generator().manual_seed(grp)).to(torch.float16)
    lens = torch.tensor([700, 333], dtype=torch.int32)
    out, lse = attention.decode_attention(q.to(DEV), kc, vc, kv_len=lens.to(DEV), return_lse=True)
    ref, lref = orc.decode_attention(q.float().numpy(), kc.cpu().numpy(), 4, vc.cpu().numpy(), 4, Hkv,
                                     kv_len=lens.numpy(), nthreads=8)
    rel = check(out.cpu().numpy(), ref, lse.cpu().numpy(), lref)
    print(f"grp {grp}: rel err {rel:.3g}")


@pytest.mark.parametrize("T,lens", [(16, [16]), (34, [1]), (1026, [1026]), (4000, [0]), (5000, [4999]),
                                    (2, [2]), (9000, [8191])])
def test_attention_ragged_lengths(orc, T, lens):
    B, Hkv, D, grp = len(lens), 1, 128, 4
    kc = make_cache(B, Hkv, T, D, 7)
    vc = make_cache(B, Hkv, T, D, 8)
    q = torch.randn(B, Hkv * grp, D, generator=torch.Generator().manual_seed(T))
    lt = torch.tensor(lens, dtype=torch.int32)
    out, lse = attention.decode_attention(q.to(DEV), kc, vc, kv_len=lt.to(DEV), return_lse=True)
    ref, lref = orc.decode_attention(q.numpy(), kc.cpu().numpy(), 4, vc.cpu().numpy(), 4, Hkv,
                                     kv_len=lt.numpy(), nthreads=8)
    check(out.cpu().numpy(), ref, lse.cpu().numpy(), lref)
    if lens[0] == 0:
        assert torch.all(out == 0) and torch.isinf(lse).all() and (lse < 0).all()


@pytest.mark.parametrize("rotate_q,v_rotated", [(True, False), (False, True), (False, False)])
def test_attention_rotation_flags(orc, rotate_q, v_rotated):
    B, Hkv, T, D, grp = 1, 2, 512, 128, 2
    kc = make_cache(B, Hkv, T, D, 3)
    vc = make_cache(B, Hkv, T, D, 4)
    q = torch.randn(B, Hkv * grp, D, generator=torch.Generator().manual_seed(1))
    out = attention.decode_attention(q.to(DEV), kc, vc, rotate_q=rotate_q, v_rotated=v_rotated)
    ref, _ = orc.decode_attention(q.numpy(), kc.cpu().numpy(), 4, vc.cpu().numpy(), 4, Hkv,
                                  rotate_q=rotate_q, v_rotated=v_rotated, nthreads=4)
    check(out.cpu().numpy(), ref)


@pytest.mark.parametrize("qd,od", [(torch.float32, torch.float16), (torch.bfloat16, torch.bfloat16),
                                   (torch.float16, torch.float32)])
def test_attention_dtypes(orc, qd, od):
    B, Hkv, T, D, grp = 2, 1, 300, 128, 8
    kc = make_cache(B, Hkv, T, D, 5)
    vc = make_cache(B, Hkv, T, D, 6)
    q = torch.randn(B, Hkv * grp, D, generator=torch.Generator().manual_seed(2)).to(qd)
    out = attention.decode_attention(q.to(DEV), kc, vc, out_dtype=od)
    assert out.dtype == od
    ref, _ = orc.decode_attention(q.float().numpy(), kc.cpu().numpy(), 4, vc.cpu().numpy(), 4, Hkv, nthreads=4)
    tol_scale = 1.0 if od == torch.float32 else 4.0
    err = (out.float().cpu().numpy() - ref).__abs__().max()
    assert err <= tol_scale * (RTOL * np.abs(ref).max() + 1e-5) + (8e-3 * np.abs(ref).max() if od == torch.bfloat16 else 0)


def test_attention_custom_scale_and_peaky_scores(orc):
    """Large sm_scale makes the softmax nearly one-hot (stresses the running max)."""
    B, Hkv, T, D, grp = 1, 1, 2048, 128, 4
    kc = make_cache(B, Hkv, T, D, 11)
    vc = make_cache(B, Hkv, T, D, 12)
    q = torch.randn(B, grp, D, generator=torch.Generator().manual_seed(3)) * 3
    out, lse = attention.decode_attention(q.to(DEV), kc, vc, sm_scale=0.9, return_lse=True)
    ref, lref = orc.decode_attention(q.numpy(), kc.cpu().numpy(), 4, vc.cpu().numpy(), 4, Hkv, sm_scale=0.9,
                                     nthreads=4)
    check(out.cpu().numpy(), ref, lse.cpu().numpy(), lref)


def torch_reference(q, kc, vc, D):
    """float32 torch evaluation on bit-exact dequantized caches."""
    B, Hkv, T = kc.shape[:3]
    Hq = q.shape[1]
    grp = Hq // Hkv
    kt = 4 if kc.shape[-1] == 18 else 3
    vt = 4 if vc.shape[-1] == 18 else 3
    kd = ops.dequantize(kc.contiguous().reshape(B, Hkv, T * (D // 32), kc.shape[-1]), kt).reshape(B, Hkv, T, D)
    vd = ops.dequantize(vc.contiguous().reshape(B, Hkv, T * (D // 32), vc.shape[-1]), vt).reshape(B, Hkv, T, D)
    H = torch.tensor([[1.0]], device=DEV)
    while H.shape[0] < D:
        H = torch.cat([torch.cat([H, H], 1), torch.cat([H, -H], 1)], 0)
    H = H / np.sqrt(D)
    qr = (q.float() @ H).reshape(B, Hkv, grp, D)
    s = torch.einsum("bhgd,bhtd->bhgt", qr, kd) / np.sqrt(D)
    p = torch.softmax(s, dim=-1)
    o = torch.einsum("bhgt,bhtd->bhgd", p, vd) @ H
    return o.reshape(B, Hq, D), torch.logsumexp(s, dim=-1).reshape(B, Hq)


def test_c3_full_size_tq4(orc):
    """B16 Hq32 Hkv8 D128 ctx 32768, TQ4_0 K/V, fp16 queries: torch fp32 for all, oracle for 2 sequences."""
    B, Hq, Hkv, T, D = 16, 32, 8, 32768, 128
    g = torch.Generator(device=DEV).manual_seed(3)
    kc = ops.quantize(outlier_normal((B, Hkv, T, D), g), 4, fwht_head_dim=D)
    vc = ops.quantize(outlier_normal((B, Hkv, T, D), g), 4, fwht_head_dim=D)
    q = torch.randn(B, Hq, D, device=DEV, generator=g).half()
    out, lse = attention.decode_attention(q, kc, vc, return_lse=True)
    ref, lref = torch_reference(q, kc, vc, D)
    rel = check(out.cpu().numpy(), ref.cpu().numpy(), lse.cpu().numpy(), lref.cpu().numpy())
    print(f"C3 vs torch fp32: rel err {rel:.3g}")
    sel = [0, 9]
    o_ref, l_ref = orc.decode_attention(q[sel].float().cpu().numpy(), kc[sel].cpu().numpy(), 4,
                                        vc[sel].cpu().numpy(), 4, Hkv, nthreads=16)
    rel = check(out[sel].cpu().numpy(), o_ref, lse[sel].cpu().numpy(), l_ref)
    print(f"C3 vs float64 oracle (2 sequences): rel err {rel:.3g}")


def test_lse_combine_matches_oracle(orc):
    rng = np.random.default_rng(5)
    o = rng.standard_normal((4, 33, 128)).astype(np.float32)
    lse = rng.standard_normal((4, 33)).astype(np.float32)
    lse[2, 5] = -np.inf
    lse[:, 7] = -np.inf
    out, lo = attention.lse_combine(torch.from_numpy(o).to(DEV), torch.from_numpy(lse).to(DEV), return_lse=True)
    ref, lref = orc.lse_combine(o, lse)
    np.testing.assert_allclose(out.cpu().numpy(), ref, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(lo.cpu().numpy(), lref, rtol=1e-5, atol=1e-6)


def test_split_by_sequence_combine_equals_full(orc):
    """Attention over a context split in P pieces + lse_combine == attention over the whole context."""
    B, Hkv, T, D, grp, P = 2, 2, 4096, 128, 8, 4
    kc = make_cache(B, Hkv, T, D, 31)
    vc = make_cache(B, Hkv, T, D, 32)
    q = torch.randn(B, Hkv * grp, D, generator=torch.Generator().manual_seed(9)).to(DEV)
    full = attention.decode_attention(q, kc, vc)
    parts, lses = [], []
    for p in range(P):
        sl = slice(p * T // P, (p + 1) * T // P)
        o, l = attention.decode_attention(q, kc[:, :, sl].contiguous(), vc[:, :, sl].contiguous(), return_lse=True)
        parts.append(o.reshape(-1, D))
        lses.append(l.reshape(-1))
    comb = attention.lse_combine(torch.stack(parts), torch.stack(lses)).reshape(full.shape)
    check(comb.cpu().numpy(), full.cpu().numpy())


@pytest.mark.parametrize("grp", [1, 2, 3, 4, 8])
def test_attention_tq3_k_vs_oracle(orc, grp):
    """Mixed TQ3_0 K / TQ4_0 V caches (the long-context split-sequence layout)."""
    B, Hkv, T, D = 2, 2, 900, 128
    kc = make_cache(B, Hkv, T, D, 40 + grp, qtype=3)
    vc = make_cache(B, Hkv, T, D, 50 + grp)
    q = torch.randn(B, Hkv * grp, D, generator=torch.Generator().manual_seed(60 + grp)).to(torch.float16)
    lens = torch.tensor([900, 417], dtype=torch.int32)
    out, lse = attention.decode_attention(q.to(DEV), kc, vc, kv_len=lens.to(DEV), return_lse=True)
    ref, lref = orc.decode_attention(q.float().numpy(), kc.cpu().numpy(), 3, vc.cpu().numpy(), 4, Hkv,
                                     kv_len=lens.numpy(), nthreads=8)
    rel = check(out.cpu().numpy(), ref, lse.cpu().numpy(), lref)
    print(f"TQ3 K grp {grp}: rel err {rel:.3g}")


@pytest.mark.parametrize("kt", [4, 3])
@pytest.mark.parametrize("T,lens", [(2, [2, 1]), (34, [0, 33]), (530, [530, 77]), (3000, [2999, 1500])])
def test_attention_head_dim_256(orc, kt, T, lens):
    """head_dim 256 (warp pairs, identity token order), TQ4_0 or TQ3_0 K, ragged lengths."""
    B, Hkv, D, grp = len(lens), 2, 256, 4
    kc = make_cache(B, Hkv, T, D, 70 + kt, qtype=kt)
    vc = make_cache(B, Hkv, T, D, 80 + kt)
    q = torch.randn(B, Hkv * grp, D, generator=torch.Generator().manual_seed(T)).to(torch.bfloat16)
    lt = torch.tensor(lens, dtype=torch.int32)
    out, lse = attention.decode_attention(q.to(DEV), kc, vc, kv_len=lt.to(DEV), return_lse=True)
    ref, lref = orc.decode_attention(q.float().numpy(), kc.cpu().numpy(), kt, vc.cpu().numpy(), 4, Hkv,
                                     kv_len=lt.numpy(), nthreads=8)
    rel = check(out.cpu().numpy(), ref, lse.cpu().numpy(), lref)
    print(f"D256 K TQ{kt} T {T}: rel err {rel:.3g}")


@pytest.mark.parametrize("D,grp", [(128, 1), (128, 3), (128, 4), (128, 8), (256, 4), (256, 8)])
def test_attention_tq2_k_vs_oracle(orc, D, grp):
    """TQ2_0 K / TQ4_0 V caches (keys in the last tier of a TQ4 -> TQ3 -> TQ2 cache), ragged
    lengths, both query rotations at head_dim 256."""
    B, Hkv, T = 2, 2, 700
    kc = make_cache(B, Hkv, T, D, 140 + grp + D, qtype=2)
    vc = make_cache(B, Hkv, T, D, 150 + grp + D)
    q = torch.randn(B, Hkv * grp, D, generator=torch.Generator().manual_seed(160 + grp + D)).to(torch.float16)
    lens = torch.tensor([T, 251], dtype=torch.int32)
    for rotate in ((True, False) if D == 256 else (True,)):
        out, lse = attention.decode_attention(q.to(DEV), kc, vc, kv_len=lens.to(DEV), return_lse=True,
                                              rotate_q=rotate)
        ref, lref = orc.decode_attention(q.float().numpy(), kc.cpu().numpy(), 2, vc.cpu().numpy(), 4, Hkv,
                                         kv_len=lens.numpy(), rotate_q=rotate, nthreads=8)
        rel = check(out.cpu().numpy(), ref, lse.cpu().numpy(), lref)
        print(f"TQ2 K D {D} grp {grp} rotate {rotate}: rel err {rel:.3g}")


def test_attention_tq2_k_tiered_cache_equals_requantized(orc):
    """A key cache moved down the tiers on the GPU (TQ4 -> TQ2 with the requantize kernel) is
    attended directly: equal to the oracle over the same TQ2 blocks."""
    from leankv_b200 import ops
    B, Hkv, T, D, grp = 2, 2, 512, 128, 4
    k4 = make_cache(B, Hkv, T, D, 170, qtype=4)
    kc = ops.requantize(k4, 4, 2).view(B, Hkv, T, D // 32, 10)
    vc = make_cache(B, Hkv, T, D, 171)
    q = torch.randn(B, Hkv * grp, D, generator=torch.Generator().manual_seed(172)).to(torch.float16)
    out = attention.decode_attention(q.to(DEV), kc, vc)
    ref, _ = orc.decode_attention(q.float().numpy(), kc.cpu().numpy(), 2, vc.cpu().numpy(), 4, Hkv, nthreads=8)
    check(out.cpu().numpy(), ref)


@pytest.mark.parametrize("grp", [1, 2, 3, 8])
@pytest.mark.parametrize("kt", [4, 3])
def test_attention_head_dim_256_grp(orc, kt, grp):
    """head_dim 256 with GQA groups 1, 2 and 8 (group 4 above), f32 q, no rotation of q."""
    B, Hkv, T, D = 2, 2, 700, 256
    kc = make_cache(B, Hkv, T, D, 110 + grp, qtype=kt)
    vc = make_cache(B, Hkv, T, D, 120 + grp)
    q = torch.randn(B, Hkv * grp, D, generator=torch.Generator().manual_seed(130 + grp))
    lt = torch.tensor([T, 333], dtype=torch.int32)
    for rotate in (True, False):
        out, lse = attention.decode_attention(q.to(DEV), kc, vc, kv_len=lt.to(DEV), return_lse=True,
                                              rotate_q=rotate)
        ref, lref = orc.decode_attention(q.numpy(), kc.cpu().numpy(), kt, vc.cpu().numpy(), 4, Hkv,
                                         kv_len=lt.numpy(), rotate_q=rotate, nthreads=8)
        check(out.cpu().numpy(), ref, lse.cpu().numpy(), lref)


@pytest.mark.parametrize("kt", [4, 3])
def test_head_dim_256_many_segments_per_cta(kt):
    """head_dim 256 with 416 (sequence, KV head) pairs of 590-700 tokens: every CTA runs
    three or more segments whose rings hold 4-6 tiles each, so stages are refilled inside
    a segment and across segments (the warp-pair stage-release parities)."""
    B, Hq, Hkv, T, D = 52, 32, 8, 700, 256
    g = torch.Generator(device=DEV).manual_seed(256 + kt)
    kc = ops.quantize(outlier_normal((B, Hkv, T, D), g), kt, fwht_head_dim=D)
    vc = ops.quantize(outlier_normal((B, Hkv, T, D), g), 4, fwht_head_dim=D)
    q = torch.randn(B, Hq, D, device=DEV, generator=g).half()
    lens = torch.tensor([T - 11 * (b % 11) for b in range(B)], dtype=torch.int32, device=DEV)
    out, lse = attention.decode_attention(q, kc, vc, kv_len=lens, max_kv_len=T, return_lse=True)
    for n in sorted(set(lens.tolist())):
        sel = (lens == n).nonzero().flatten()
        ref, lref = torch_reference(q[sel], kc[sel][:, :, :n], vc[sel][:, :, :n], D)
        check(out[sel].cpu().numpy(), ref.cpu().numpy(), lse[sel].cpu().numpy(), lref.cpu().numpy())


def test_attention_tq3_k_rotation_flags(orc):
    B, Hkv, T, D, grp = 1, 2, 300, 128, 8
    kc = make_cache(B, Hkv, T, D, 91, qtype=3)
    vc = make_cache(B, Hkv, T, D, 92)
    q = torch.randn(B, Hkv * grp, D, generator=torch.Generator().manual_seed(93))
    out = attention.decode_attention(q.to(DEV), kc, vc, rotate_q=False, v_rotated=False)
    ref, _ = orc.decode_attention(q.numpy(), kc.cpu().numpy(), 3, vc.cpu().numpy(), 4, Hkv,
                                  rotate_q=False, v_rotated=False, nthreads=4)
    check(out.cpu().numpy(), ref)


def test_c4_shape_tq3k_long_context(orc):
    """64 query / 8 KV heads, head_dim 128, context 131072, TQ3_0 K / TQ4_0 V (batch 2 of the 64)."""
    B, Hq, Hkv, T, D = 2, 64, 8, 131072, 128
    g = torch.Generator(device=DEV).manual_seed(4)
    kc = ops.quantize(outlier_normal((B, Hkv, T, D), g), 3, fwht_head_dim=D)
    vc = ops.quantize(outlier_normal((B, Hkv, T, D), g), 4, fwht_head_dim=D)
    q = torch.randn(B, Hq, D, device=DEV, generator=g).half()
    lens = torch.tensor([T, T - 12345], dtype=torch.int32, device=DEV)
    out, lse = attention.decode_attention(q, kc, vc, kv_len=lens, return_lse=True)
    for b in range(B):
        n = int(lens[b])
        ref, lref = torch_reference(q[b:b + 1], kc[b:b + 1, :, :n], vc[b:b + 1, :, :n], D)
        rel = check(out[b:b + 1].cpu().numpy(), ref.cpu().numpy(), lse[b:b + 1].cpu().numpy(), lref.cpu().numpy())
        print(f"C4 shape seq {b} (len {n}) vs torch fp32: rel err {rel:.3g}")


def test_c5_shape_head_dim_256(orc):
    """8 KV heads, head_dim 256, context 16384 + 1, TQ4_0 K/V (one layer, batch 4 of the 32)."""
    B, Hq, Hkv, T, D = 4, 32, 8, 16385, 256
    g = torch.Generator(device=DEV).manual_seed(5)
    kc = ops.quantize(outlier_normal((B, Hkv, T + 1, D), g), 4, fwht_head_dim=D)
    vc = ops.quantize(outlier_normal((B, Hkv, T + 1, D), g), 4, fwht_head_dim=D)
    q = torch.randn(B, Hq, D, device=DEV, generator=g).to(torch.bfloat16)
    lens = torch.full((B,), T, dtype=torch.int32, device=DEV)
    out, lse = attention.decode_attention(q, kc, vc, kv_len=lens, max_kv_len=T, return_lse=True)
    ref, lref = torch_reference(q, kc[:, :, :T], vc[:, :, :T], D)
    rel = check(out.cpu().numpy(), ref.cpu().numpy(), lse.cpu().numpy(), lref.cpu().numpy())
    print(f"C5 shape vs torch fp32: rel err {rel:.3g}")
