"""LeanKVCache with storage="tq_blocks" and "tq_pages": quantize-on-write appends and the fused
decode attention
over the packed cache, against the prototype's flow (dequantize the whole cache, then attend) on
the same blocks, over a prefill and many single-token decode steps (the capacity grows on the way).

Tolerance as the decode-attention tests: max |out - ref| <= 1e-3 * max |ref| + 1e-5.
"""
import numpy as np
import pytest
import torch

from leankv_b200 import ops
from leankv_b200.turboquant import LeanKVCache

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
RTOL = 1e-3


def hadamard(D):
    H = torch.tensor([[1.0]], device=DEV)
    while H.shape[0] < D:
        H = torch.cat([torch.cat([H, H], 1), torch.cat([H, -H], 1)], 0)
    return H / np.sqrt(D)


def dequantize_then_attend(q, kc, vc, D):
    """The prototype's read-out: every cached block dequantized, then float32 attention (q rotated
    into the cache's Hadamard domain, the output rotated back)."""
    B, Hkv, T = kc.shape[:3]
    Hq = q.shape[1]
    kt = 4 if kc.shape[-1] == 18 else 3
    kd = ops.dequantize(kc.contiguous().reshape(B, Hkv, T * (D // 32), kc.shape[-1]), kt).reshape(B, Hkv, T, D)
    vd = ops.dequantize(vc.contiguous().reshape(B, Hkv, T * (D // 32), 18), 4).reshape(B, Hkv, T, D)
    H = hadamard(D)
    qr = (q.float() @ H).reshape(B, Hkv, Hq // Hkv, D)
    s = torch.einsum("bhgd,bhtd->bhgt", qr, kd) / np.sqrt(D)
    o = torch.einsum("bhgt,bhtd->bhgd", torch.softmax(s, dim=-1), vd) @ H
    return o.reshape(B, Hq, D)


def kv_rows(B, H, n, D, g):
    x = torch.randn(B, H, n, D, device=DEV, generator=g)
    x[..., :4] *= 20.0          # outlier channels
    return x.to(torch.bfloat16)


@pytest.mark.parametrize("D,k_bits,passes", [(128, 4, 0), (128, 3, 2), (256, 4, 0), (256, 3, 0)])
def test_blocks_cache_fused_attention_matches_dequantize(D, k_bits, passes):
    B, Hkv, grp, layers, prefill, steps = 3, 2, 4, 2, 300, 24
    g = torch.Generator(device=DEV).manual_seed(D + k_bits)
    cache = LeanKVCache(layers, D, Hkv, k_bits=k_bits, storage="tq_blocks", device="cuda", k_opt_passes=passes)
    worst = 0.0
    for step in range(steps + 1):
        n = prefill if step == 0 else 1
        for layer in range(layers):
            k, v = kv_rows(B, Hkv, n, D, g), kv_rows(B, Hkv, n, D, g)
            kc, vc = cache.update(k, v, layer)
            assert kc.shape[2] == vc.shape[2] == prefill + step
            q = torch.randn(B, Hkv * grp, 1, D, device=DEV, generator=g).to(torch.bfloat16)
            out = cache.attention(q, layer, out_dtype=torch.float32)
            ref = dequantize_then_attend(q[:, :, 0], kc, vc, D)
            err = (out[:, :, 0] - ref).abs().max().item()
            tol = RTOL * ref.abs().max().item() + 1e-5
            assert err <= tol, f"step {step} layer {layer}: {err:.3g} > {tol:.3g}"
            worst = max(worst, err / ref.abs().max().item())
    assert cache.get_seq_length() == prefill + steps
    assert cache.seen_tokens == prefill + steps
    print(f"D {D} TQ{k_bits} K: worst rel err over {steps + 1} updates x {layers} layers {worst:.3g}")


def test_blocks_cache_appends_equal_one_shot_quantize():
    """The packed cache after a prefill and single-token updates holds exactly the blocks of
    quantizing the whole sequence at once."""
    B, Hkv, D, n0, steps = 2, 2, 128, 40, 9
    g = torch.Generator(device=DEV).manual_seed(11)
    full_k, full_v = kv_rows(B, Hkv, n0 + steps, D, g), kv_rows(B, Hkv, n0 + steps, D, g)
    cache = LeanKVCache(1, D, Hkv, k_bits=3, storage="tq_blocks", device="cuda")
    cache.update(full_k[:, :, :n0].contiguous(), full_v[:, :, :n0].contiguous(), 0)
    for s in range(steps):
        kc, vc = cache.update(full_k[:, :, n0 + s:n0 + s + 1].contiguous(),
                              full_v[:, :, n0 + s:n0 + s + 1].contiguous(), 0)
    assert torch.equal(kc, ops.quantize(full_k, 3, fwht_head_dim=D))
    assert torch.equal(vc, ops.quantize(full_v, 4, fwht_head_dim=D))



@pytest.mark.parametrize("D,k_bits,page_size", [(128, 3, 16), (256, 4, 64)])
def test_pages_cache_equals_blocks_cache(D, k_bits, page_size):
    """storage="tq_pages" (fixed page pools) and storage="tq_blocks" (doubling buffers) hold the
    same blocks and run the same split-KV plan: equal attention outputs after every update."""
    B, Hkv, grp, layers, prefill, steps = 3, 2, 4, 2, 300, 12
    g = torch.Generator(device=DEV).manual_seed(D * k_bits + page_size)
    blocks = LeanKVCache(layers, D, Hkv, k_bits=k_bits, storage="tq_blocks", device="cuda")
    pages = LeanKVCache(layers, D, Hkv, k_bits=k_bits, storage="tq_pages", device="cuda",
                        num_pages=B * (-(-(prefill + steps) // page_size)), page_size=page_size)
    for step in range(steps + 1):
        n = prefill if step == 0 else 1
        for layer in range(layers):
            k, v = kv_rows(B, Hkv, n, D, g), kv_rows(B, Hkv, n, D, g)
            blocks.update(k, v, layer)
            kp, vp = pages.update(k, v, layer)
            assert kp.shape[:3] == (pages._blocks[layer].num_pages, Hkv, page_size)
            q = torch.randn(B, Hkv * grp, 1, D, device=DEV, generator=g).to(torch.bfloat16)
            assert torch.equal(pages.attention(q, layer), blocks.attention(q, layer)), (step, layer)
    assert pages.get_seq_length() == blocks.get_seq_length() == prefill + steps
    with pytest.raises(MemoryError):   # the pools hold exactly prefill + steps tokens per sequence
        for _ in range(page_size):
            pages.update(kv_rows(B, Hkv, 1, D, g), kv_rows(B, Hkv, 1, D, g), 0)
