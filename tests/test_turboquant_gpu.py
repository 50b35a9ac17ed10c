"""GPU parity of the prototype interface (leankv_b200.turboquant) with the prototype.

Fixtures: tests/golden/make_proto_golden.py (the prototype run on seeded inputs).
The prototype rotates with a float32 GEMM and reduces norms in its own order; the
CUDA path uses the butterfly and warp reductions, so values agree to float32
rounding.  Bar: per-vector scales and dequantized values within 1e-5 relative;
codebook indices identical except where the normalized value lies within 2e-6
(relative) of a decision boundary — such elements are counted and must stay
rare; QJL sign bits identical wherever the residual is not within rounding of 0.
"""
import numpy as np
import pytest
import torch

from leankv_b200.turboquant import LeanKVCache, TurboQuantizer, qjl_residual

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
CASES = [("a", 128, 3, None, "randomized_hadamard", True, 1),
         ("b", 64, 4, 16, "hadamard", False, 0),
         ("c", 64, 2, None, "random_orthogonal", True, 0),
         ("d", 256, 3, 32, "randomized_hadamard", True, 1),
         ("e", 32, 4, None, "randomized_hadamard", False, 0)]


def _xn64(x, rot, norms, group):
    """float64 normalized rotated values from the prototype's own scales."""
    xr = x.astype(np.float64) @ rot.astype(np.float64).T
    if group is None:
        return xr / (norms[..., None].astype(np.float64) + 1e-10)
    sh = xr.shape
    g = xr.reshape(*sh[:-1], -1, group) / (norms[..., None].astype(np.float64) + 1e-10)
    return g.reshape(sh)


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_quantizer_matches_prototype(golden, case):
    name, hd, bits, gs, strat, qjl, layer = case
    g = golden["proto"]
    tq = TurboQuantizer(n_layers=2, head_dim=hd, bits=bits, group_size=gs, rotation_strategy=strat, use_qjl=qjl,
                        seed=42, device="cuda")
    x = torch.from_numpy(g[f"q{name}_x"]).to(DEV)
    q = tq.quantize(x, layer)
    torch.cuda.synchronize()
    np.testing.assert_allclose(q.norms.cpu().numpy(), g[f"q{name}_norms"], rtol=1e-5, atol=1e-7)

    rot = tq.rotations[layer].cpu().numpy()
    if strat == "random_orthogonal":
        np.testing.assert_allclose(rot, g[f"q{name}_rot"], atol=1e-6)
    idx, ref = q.indices.cpu().numpy(), g[f"q{name}_idx"]
    bad = idx != ref
    xn = _xn64(g[f"q{name}_x"], rot, g[f"q{name}_norms"], gs)
    bounds = tq.boundaries.cpu().numpy().astype(np.float64)
    near = np.min(np.abs(xn[..., None] - bounds), axis=-1) <= 2e-6 * np.maximum(1.0, np.abs(xn))
    assert not np.any(bad & ~near), f"{int((bad & ~near).sum())} index mismatches away from a boundary"
    assert bad.mean() < 1e-3
    print(f"case {name}: {int(bad.sum())} of {bad.size} indices differ, all within 2e-6 of a boundary")

    vec_ok = ~bad.any(-1)
    if qjl:
        sg = qjl_residual.unpack_signs(q.qjl_signs.cpu(), hd).numpy()
        sr = qjl_residual.unpack_signs(torch.from_numpy(g[f"q{name}_signs"]), hd).numpy()
        levels = tq.levels.cpu().numpy().astype(np.float64)
        resid = xn - levels[ref]
        differ = (sg != sr) & vec_ok[..., None]
        assert not np.any(differ & (np.abs(resid) > 1e-6)), "QJL sign differs away from a zero residual"
        np.testing.assert_allclose(q.qjl_mean_abs.cpu().numpy()[vec_ok], g[f"q{name}_mean"][vec_ok], rtol=1e-4,
                                   atol=1e-7)
    for inv, key in ((False, "deq"), (True, "deq_inv")):
        y = tq.dequantize(q, layer, apply_inverse_rot=inv).cpu().numpy()
        r = g[f"q{name}_{key}"]
        scale = np.abs(r).max()
        err = np.abs(y - r)[vec_ok].max() if vec_ok.any() else 0.0
        assert err <= 1e-5 * scale, f"{key}: {err:.3g} > {1e-5 * scale:.3g}"
    qr = tq.quantize_for_attention(x[:, :, :3], layer).cpu().numpy()
    np.testing.assert_allclose(qr, g[f"q{name}_qrot"], rtol=1e-5, atol=1e-5 * np.abs(g[f"q{name}_qrot"]).max())


@pytest.mark.parametrize("tag,vrot", [("kvn", "none"), ("kvr", "randomized_hadamard")])
def test_leankv_cache_matches_prototype(golden, tag, vrot):
    g = golden["proto"]
    cache = LeanKVCache(n_layers=2, head_dim=64, n_kv_heads=2, k_bits=3, v_bits=4, v_rotation=vrot, device="cuda")
    k_in = torch.from_numpy(g[f"{tag}_k_in"]).to(DEV)
    v_in = torch.from_numpy(g[f"{tag}_v_in"]).to(DEV)
    pos = 0
    for n in (5, 1, 1):
        for layer in range(2):
            ak, av = cache.update(k_in[layer, :, :, pos:pos + n].contiguous(), v_in[layer, :, :, pos:pos + n].contiguous(),
                                  layer)
        pos += n
    assert cache.get_seq_length() == int(g[f"{tag}_len"]) == 7
    assert cache.seen_tokens == 7
    for got, key in ((ak, "keys_l1"), (av, "values_l1")):
        r = g[f"{tag}_{key}"]
        d = np.abs(got.cpu().numpy() - r)
        scale = np.abs(r).max()
        # a vector whose index flipped at a boundary differs by a level step; such vectors must be rare
        vec_bad = (d > 1e-5 * scale).any(-1)
        assert vec_bad.mean() < 0.02, f"{key}: {vec_bad.sum()} of {vec_bad.size} vectors differ"
    summ = cache.memory_summary()
    assert summ["total_tokens"] == 7 and summ["compression_ratio"] > 3


def test_cache_growth_many_steps():
    cache = LeanKVCache(n_layers=1, head_dim=128, n_kv_heads=4, device="cuda")
    torch.manual_seed(0)
    ks, vs = [], []
    for n in (3, 40, 1, 1, 17):
        k = torch.randn(2, 4, n, 128, device=DEV)
        v = torch.randn(2, 4, n, 128, device=DEV)
        ks.append(k)
        vs.append(v)
        ak, av = cache.update(k, v, 0)
    full_k, full_v = torch.cat(ks, 2), torch.cat(vs, 2)
    # the stored codes equal one-shot quantization of the whole sequence
    qk = cache.k_quantizer.quantize(full_k, 0)
    assert torch.equal(cache.k_cache[0][0].indices.permute(1, 2, 0, 3).cpu(), qk.indices.cpu())
    assert torch.equal(ak.cpu(), cache.k_quantizer.dequantize(qk, 0).cpu())
    assert ak.shape == (2, 4, 62, 128) and av.shape == (2, 4, 62, 128)
    # values are reconstructed in the original space: relative error of a 4-bit codebook
    rel = ((av - full_v).norm(dim=-1) / full_v.norm(dim=-1)).mean().item()
    assert rel < 0.15
