"""GPU checks of the KV-cache append (quantize-on-write) and the packed partial merge.

Append: every written head row must be bit-identical to tq_quantize_cuda on the
same row (itself bit-exact with the reference C), land in slot pos[b] + t, and
leave every other slot untouched; slots past the capacity are counted, not written.
"""
import numpy as np
import pytest
import torch

from leankv_b200 import attention, ops

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _src(B, H, n, D, dtype, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    x = torch.randn(B, H, n, D, device=DEV, generator=g)
    x[..., :3] *= 15.0
    return x.to(dtype).contiguous()


@pytest.mark.parametrize("qtype,D,dtype,passes", [(4, 128, torch.bfloat16, 0), (3, 128, torch.float16, 0),
                                                  (3, 256, torch.bfloat16, 2), (4, 256, torch.float32, 0),
                                                  (4, 64, torch.float32, 0), (3, 32, torch.bfloat16, 0)])
def test_append_matches_quantize(qtype, D, dtype, passes):
    B, H, cap, n_new = 3, 2, 40, 5
    bb = 18 if qtype == 4 else 14
    src = _src(B, H, n_new, D, dtype, seed=D + qtype)
    fill = 0xA5
    cache = torch.full((B, H, cap, D // 32, bb), fill, dtype=torch.uint8, device=DEV)
    pos = torch.tensor([0, 17, 38], dtype=torch.int32, device=DEV)
    ovf = torch.zeros(1, dtype=torch.int32, device=DEV)
    ops.kv_append(src, cache, pos, qtype=qtype, rotate=True, opt_passes=passes, overflow=ovf)
    ref = ops.quantize(src, qtype, fwht_head_dim=D, opt_passes=passes)      # [B, H, n_new, D/32, bb]
    c = cache.cpu()
    r = ref.cpu()
    written = torch.zeros(B, H, cap, dtype=torch.bool)
    for b, p in enumerate(pos.tolist()):
        for t in range(n_new):
            if p + t < cap:
                assert torch.equal(c[b, :, p + t], r[b, :, t]), (b, t)
                written[b, :, p + t] = True
    assert torch.all(c[~written] == fill)
    assert int(ovf.item()) == H * (38 + n_new - cap)            # sequence 2 runs 3 rows past the capacity


def test_prefill_then_decode_appends_equal_one_shot_quantize():
    """Prefill from slot 0 (pos None) followed by single-token appends == quantizing the whole sequence."""
    B, H, D, n0, steps = 2, 4, 128, 64, 6
    cap = n0 + steps + 2
    full = _src(B, H, n0 + steps, D, torch.bfloat16, seed=7)
    cache = torch.zeros(B, H, cap, D // 32, 18, dtype=torch.uint8, device=DEV)
    ops.kv_append(full[:, :, :n0].contiguous(), cache)
    kv_len = torch.full((B,), n0, dtype=torch.int32, device=DEV)
    for s in range(steps):
        ops.kv_append(full[:, :, n0 + s:n0 + s + 1].contiguous(), cache, kv_len)
        kv_len += 1
    ref = ops.quantize(full, 4, fwht_head_dim=D)
    assert torch.equal(cache[:, :, : n0 + steps], ref)
    assert torch.all(cache[:, :, n0 + steps:] == 0)


def test_append_argument_errors():
    src = torch.zeros(1, 1, 1, 96, device=DEV)
    cache = torch.zeros(1, 1, 4, 3, 18, dtype=torch.uint8, device=DEV)
    with pytest.raises(Exception, match="head_dim"):
        ops.kv_append(src, cache)
    with pytest.raises(ValueError):
        ops.kv_append(torch.zeros(1, 2, 1, 128, device=DEV), torch.zeros(1, 1, 4, 4, 18, dtype=torch.uint8, device=DEV))


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_merge_packed_partials(orc, out_dtype):
    P, n, D = 5, 77, 128
    rng = np.random.default_rng(3)
    o = rng.standard_normal((P, n, D)).astype(np.float32)
    lse = (rng.standard_normal((P, n)) * 3).astype(np.float32)
    lse[1, 4] = -np.inf
    lse[:, 9] = -np.inf
    packed = np.concatenate([o.reshape(P, n * D), lse], axis=1).reshape(-1)
    parts = torch.from_numpy(packed).to(DEV)
    out = torch.empty(n, D, dtype=out_dtype, device=DEV)
    lo = torch.empty(n, dtype=torch.float32, device=DEV)
    attention.merge_partials(parts, P, n, D, out, lo)
    ref, lref = orc.lse_combine(o, lse)
    tol = {torch.float32: 1e-5, torch.float16: 1e-3, torch.bfloat16: 8e-3}[out_dtype]
    np.testing.assert_allclose(out.float().cpu().numpy(), ref, rtol=tol, atol=tol)
    np.testing.assert_allclose(lo.cpu().numpy(), lref, rtol=1e-5, atol=1e-6)
    assert torch.all(out[9] == 0) and lo[9].item() == -np.inf


def test_split_sequence_single_process_emulation(orc):
    """P token shards attended separately, packed, merged == one attention over the whole context."""
    from leankv_b200.distributed import local_lengths, token_shard
    B, Hkv, grp, T, D, P = 2, 2, 8, 3000, 128, 4
    g = torch.Generator(device=DEV).manual_seed(9)
    kc = ops.quantize(torch.randn(B, Hkv, T, D, device=DEV, generator=g), 3, fwht_head_dim=D)
    vc = ops.quantize(torch.randn(B, Hkv, T, D, device=DEV, generator=g), 4, fwht_head_dim=D)
    q = torch.randn(B, Hkv * grp, D, device=DEV, generator=g).half()
    lens = torch.tensor([3000, 1234], dtype=torch.int32, device=DEV)
    n = B * Hkv * grp
    parts = torch.empty(P * n * (D + 1), dtype=torch.float32, device=DEV)
    for r in range(P):
        s0, s1 = token_shard(T, r, P)
        seg = parts[r * n * (D + 1):(r + 1) * n * (D + 1)]
        attention.decode_attention(q, kc[:, :, s0:s1].contiguous(), vc[:, :, s0:s1].contiguous(),
                                   kv_len=local_lengths(lens, s0, s1), out=seg[: n * D].view(B, -1, D),
                                   lse_out=seg[n * D:].view(B, -1))
    out = torch.empty(n, D, dtype=torch.float32, device=DEV)
    attention.merge_partials(parts, P, n, D, out)
    ref, _ = orc.decode_attention(q.float().cpu().numpy(), kc.cpu().numpy(), 3, vc.cpu().numpy(), 4, Hkv,
                                  kv_len=lens.cpu().numpy(), nthreads=8)
    err = np.abs(out.cpu().numpy().reshape(ref.shape) - ref).max()
    assert err <= 2e-3 * np.abs(ref).max() + 1e-5
    assert attention.last_status() == 0
