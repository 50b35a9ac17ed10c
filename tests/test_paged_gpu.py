"""Paged KV caches on the GPU: tq_decode_attention_paged_cuda and tq_kv_append_paged_cuda.

A paged pool holds the same token rows as a contiguous cache, scattered over pages in a
random order through the page table.  The paged decode attention runs the same split-KV
plan over the same tiles as the contiguous kernel, so its outputs and lse must be equal
bit for bit (ragged lengths, page sizes 16 .. 1024, head_dim 128 / 256, TQ3 / TQ4 K,
GQA groups 4 and 8).  The paged append must place exactly the bytes the contiguous
append writes, and count rows it cannot place.  A page id outside the pool is reported
through the attention's status word (that tile reads page 0).
"""
import pytest
import torch

from leankv_b200 import attention, ops

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _cache(B, Hkv, T, D, qtype, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    x = torch.randn(B, Hkv, T, D, device=DEV, generator=g)
    x[..., :: D // 4] *= 20.0   # a few large channels per head
    return ops.quantize(x, qtype, fwht_head_dim=D)


def _scatter(cache, P, spare, seed):
    """Contiguous [B, H, T, nb, bb] -> (pool [num_pages, H, P, nb, bb], page_table [B, T / P])."""
    B, H, T = cache.shape[:3]
    npp = (T + P - 1) // P
    num_pages = B * npp + spare
    g = torch.Generator(device="cpu").manual_seed(seed)
    perm = torch.randperm(num_pages, generator=g)[: B * npp].view(B, npp)
    pool = torch.zeros((num_pages, H, P) + tuple(cache.shape[3:]), dtype=torch.uint8, device=DEV)
    for b in range(B):
        for i in range(npp):
            n = min(P, T - i * P)
            pool[perm[b, i], :, :n] = cache[b, :, i * P: i * P + n]
    return pool, perm.to(torch.int32).to(DEV).contiguous()


@pytest.mark.parametrize("D,kt,grp,P", [(128, 3, 8, 16), (128, 4, 4, 64), (128, 3, 4, 256), (256, 4, 4, 32),
                                        (256, 3, 8, 1024), (128, 4, 8, 128)])
def test_paged_attention_equals_contiguous(D, kt, grp, P):
    B, Hkv = 5, 2
    T = 4 * 1024
    kc = _cache(B, Hkv, T, D, kt, 10 * D + kt)
    vc = _cache(B, Hkv, T, D, 4, 10 * D + kt + 1)
    lens = torch.tensor([T, 1, 0, 3001, 2 * P + 5], dtype=torch.int32, device=DEV)
    q = torch.randn(B, Hkv * grp, D, device=DEV, generator=torch.Generator(device=DEV).manual_seed(P)).half()
    kp, table = _scatter(kc, P, 7, P + D)
    vp, _ = _scatter(vc, P, 7, P + D)
    ref, lref = attention.decode_attention(q, kc, vc, kv_len=lens, max_kv_len=T, return_lse=True)
    assert attention.last_status() == 0
    out, lse = attention.decode_attention_paged(q, kp, vp, table, kv_len=lens, max_kv_len=T, return_lse=True)
    assert attention.last_status() == 0
    assert torch.equal(out, ref)
    assert torch.equal(lse, lref)


def test_paged_attention_bad_page_id_reported():
    B, Hkv, D, P, T = 2, 1, 128, 16, 256
    kc = _cache(B, Hkv, T, D, 4, 1)
    vc = _cache(B, Hkv, T, D, 4, 2)
    kp, table = _scatter(kc, P, 0, 3)
    vp, _ = _scatter(vc, P, 0, 3)
    q = torch.randn(B, 4, D, device=DEV).half()
    lens = torch.tensor([T, T], dtype=torch.int32, device=DEV)
    attention.decode_attention_paged(q, kp, vp, table, kv_len=lens)
    assert attention.last_status() == 0
    bad = table.clone()
    bad[1, 3] = kp.shape[0]   # one past the pool
    attention.decode_attention_paged(q, kp, vp, bad, kv_len=lens)
    assert attention.last_status() == 1   # TQ_ERROR_INVALID_VALUE
    attention.decode_attention_paged(q, kp, vp, table, kv_len=lens)
    assert attention.last_status() == 0   # the next call starts clean


@pytest.mark.parametrize("qtype,P,D", [(3, 16, 128), (4, 64, 128), (4, 32, 256)])
def test_paged_append_equals_contiguous(qtype, P, D):
    B, H, max_pages = 3, 2, 6
    cap = max_pages * P
    g = torch.Generator(device=DEV).manual_seed(qtype + P)
    num_pages = B * max_pages + 3
    perm = torch.randperm(num_pages, generator=torch.Generator().manual_seed(P))[: B * max_pages]
    table = perm.view(B, max_pages).to(torch.int32).to(DEV).contiguous()
    bb = ops.BLOCK_BYTES[qtype]
    cont = torch.zeros(B, H, cap, D // 32, bb, dtype=torch.uint8, device=DEV)
    pool = torch.zeros(num_pages, H, P, D // 32, bb, dtype=torch.uint8, device=DEV)
    pos = torch.tensor([0, 3, 17], dtype=torch.int32, device=DEV)
    ovf_c = torch.zeros(1, dtype=torch.int32, device=DEV)
    ovf_p = torch.zeros(1, dtype=torch.int32, device=DEV)
    for n_new in (P + 3, 1, 2 * P - 1, 5):
        src = torch.randn(B, H, n_new, D, device=DEV, generator=g).to(torch.bfloat16)
        ops.kv_append(src, cont, pos, qtype=qtype, overflow=ovf_c)
        ops.kv_append_paged(src, pool, table, pos, qtype=qtype, overflow=ovf_p)
        pos += n_new
    torch.cuda.synchronize()
    for b in range(B):
        for i in range(max_pages):
            assert torch.equal(pool[table[b, i]], cont[b, :, i * P:(i + 1) * P]), (b, i)
    assert int(ovf_p.item()) == int(ovf_c.item())
    # a page id outside the pool: those rows are skipped and counted
    bad = table.clone()
    bad[0, 0] = -1
    ovf = torch.zeros(1, dtype=torch.int32, device=DEV)
    before = pool.clone()
    ops.kv_append_paged(torch.randn(B, H, 4, D, device=DEV), pool, bad,
                        torch.zeros(B, dtype=torch.int32, device=DEV), qtype=qtype, overflow=ovf)
    assert int(ovf.item()) == 4 * H
    assert torch.equal(pool[table[0, 0]], before[table[0, 0]])


@pytest.mark.parametrize("kt,D", [(3, 128), (4, 256)])
def test_paged_decode_steps_equal_contiguous(kt, D):
    """Prefill + single-token decode steps appended into pages and attended, against the
    same steps on a contiguous cache: equal outputs at every step."""
    B, Hkv, grp, P, max_pages = 3, 2, 4, 16, 40
    cap = P * max_pages
    g = torch.Generator(device=DEV).manual_seed(kt * D)
    num_pages = B * max_pages
    table = torch.randperm(num_pages, generator=torch.Generator().manual_seed(5)).view(B, max_pages)
    table = table.to(torch.int32).to(DEV).contiguous()
    kb = ops.BLOCK_BYTES[kt]
    kc = torch.zeros(B, Hkv, cap, D // 32, kb, dtype=torch.uint8, device=DEV)
    vc = torch.zeros(B, Hkv, cap, D // 32, 18, dtype=torch.uint8, device=DEV)
    kp = torch.zeros(num_pages, Hkv, P, D // 32, kb, dtype=torch.uint8, device=DEV)
    vp = torch.zeros(num_pages, Hkv, P, D // 32, 18, dtype=torch.uint8, device=DEV)
    pos = torch.zeros(B, dtype=torch.int32, device=DEV)
    for step, n in enumerate([37, 1, 1, 1, 20, 1, 1]):
        k = torch.randn(B, Hkv, n, D, device=DEV, generator=g)
        v = torch.randn(B, Hkv, n, D, device=DEV, generator=g)
        ops.kv_append(k, kc, pos, qtype=kt)
        ops.kv_append(v, vc, pos, qtype=4)
        ops.kv_append_paged(k, kp, table, pos, qtype=kt)
        ops.kv_append_paged(v, vp, table, pos, qtype=4)
        pos += n
        q = torch.randn(B, Hkv * grp, D, device=DEV, generator=g).half()
        ref = attention.decode_attention(q, kc, vc, kv_len=pos, max_kv_len=cap)
        out = attention.decode_attention_paged(q, kp, vp, table, kv_len=pos, max_kv_len=cap)
        assert attention.last_status() == 0
        assert torch.equal(out, ref), step
