"""PagedKVCache on the GPU: sequences join and leave between decode steps; at every step
and layer the paged append + attention equals, bit for bit, the contiguous append +
decode attention over the same rows (the same split-KV plan), and a full pool reports
MemoryError without touching the pools."""
import pytest
import torch

from leankv_b200 import attention, ops
from leankv_b200.paged import PagedKVCache

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("D,k_bits,grp,page_size", [(128, 3, 8, 16), (256, 4, 4, 64)])
def test_paged_cache_matches_contiguous(D, k_bits, grp, page_size):
    layers, Hkv, cap = 2, 2, 512
    cache = PagedKVCache(layers, Hkv, D, num_pages=96, page_size=page_size, max_seqs=4,
                         max_pages_per_seq=cap // page_size, k_bits=k_bits)
    kb = 14 if k_bits == 3 else 18
    shadow_k = torch.zeros(layers, 4, Hkv, cap, D // 32, kb, dtype=torch.uint8, device=DEV)
    shadow_v = torch.zeros(layers, 4, Hkv, cap, D // 32, 18, dtype=torch.uint8, device=DEV)
    g = torch.Generator(device=DEV).manual_seed(D + k_bits)
    seqs = [cache.add_sequence(), cache.add_sequence()]
    plan = [("step", 50), ("step", 1), ("join", None), ("step", 1), ("step", 33), ("leave", 0), ("join", None),
            ("step", 1), ("step", 1), ("step", 7)]
    for op, n in plan:
        if op == "join":
            seqs.append(cache.add_sequence())
            continue
        if op == "leave":
            cache.free_sequence(seqs.pop(n))
            continue
        step = cache.batch(seqs, n)
        idx = torch.tensor(seqs, device=DEV)
        for layer in range(layers):
            k = torch.randn(len(seqs), Hkv, n, D, device=DEV, generator=g)
            v = torch.randn(len(seqs), Hkv, n, D, device=DEV, generator=g)
            q = torch.randn(len(seqs), Hkv * grp, D, device=DEV, generator=g).half()
            cache.append(step, layer, k, v)
            out = cache.attention(step, layer, q)
            kc = shadow_k[layer].index_select(0, idx).contiguous()
            vc = shadow_v[layer].index_select(0, idx).contiguous()
            ops.kv_append(k, kc, step.pos, qtype=k_bits)
            ops.kv_append(v, vc, step.pos, qtype=4)
            shadow_k[layer].index_copy_(0, idx, kc)
            shadow_v[layer].index_copy_(0, idx, vc)
            ref = attention.decode_attention(q, kc, vc, kv_len=step.kv_len, max_kv_len=step.max_kv_len,
                                             out_dtype=torch.float16)
            assert attention.last_status() == 0
            assert torch.equal(out, ref), (op, n, layer)
        cache.commit(step)
    assert cache.seq_len(seqs[-1]) == 9 and cache.seq_len(seqs[0]) == 94
    summary = cache.memory_summary()
    assert summary["pages_used"] == sum(-(-cache.seq_len(s) // page_size) for s in seqs)


def test_paged_cache_pool_exhaustion():
    cache = PagedKVCache(1, 1, 128, num_pages=4, page_size=16, max_seqs=2, max_pages_per_seq=4)
    a, b = cache.add_sequence(), cache.add_sequence()
    step = cache.batch([a, b], 32)       # 4 pages
    k = torch.randn(2, 1, 32, 128, device=DEV)
    cache.append(step, 0, k, k)
    cache.commit(step)
    before = cache.k[0].clone()
    with pytest.raises(MemoryError):
        cache.batch([a], 1)
    assert torch.equal(cache.k[0], before)
    cache.free_sequence(b)
    step = cache.batch([a], 1)           # b's pages are free again
    assert cache.pages.free_pages == 1
