"""tq_peer_exchange on one GPU: the push / arrival count / bounded wait / merge kernel
with a world of one rank (every CTA pushes into its own GPU's buffer), over several
steps so both slot buffers and the never-reset arrival counter are exercised.  The
merge must equal tq_lse_merge_cuda bit for bit (same arithmetic, same order).  The
multi-rank exchange over NVLink is tested in test_multigpu_gpu.py (>= 2 GPUs).
The exchange fused into the decode attention (tq_peer_exchange_attention) must equal the
decode attention followed by the merge, over several steps and interleaved with merge steps.
"""
import numpy as np
import pytest
import torch

from leankv_b200 import attention
from leankv_b200.distributed import PeerExchange

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _part(n, D, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    o = torch.randn(n * D, device=DEV, generator=g)
    lse = torch.randn(n, device=DEV, generator=g) * 4.0
    lse[::7] = -float("inf")   # empty rows: zero output, -inf lse
    return torch.cat([o, lse]).contiguous()


@pytest.mark.parametrize("n,D,dtype", [(4096, 128, torch.float16), (37, 256, torch.float32),
                                       (1, 128, torch.bfloat16), (2051, 128, torch.float32)])
def test_peer_exchange_single_rank_matches_merge(n, D, dtype):
    ex = PeerExchange(n, D)
    try:
        for step in range(5):
            part = _part(n, D, 100 * step + D + n)
            out = torch.empty(n, D, dtype=dtype, device=DEV)
            lse = torch.empty(n, dtype=torch.float32, device=DEV)
            ex.merge(part, out, lse)
            ref = torch.empty_like(out)
            lref = torch.empty_like(lse)
            attention.merge_partials(part, 1, n, D, ref, lref)
            ex.status()
            assert torch.equal(out, ref), step
            assert np.array_equal(lse.cpu().numpy(), lref.cpu().numpy()), step
    finally:
        ex.close()


def test_peer_exchange_unaligned_part_scalar_path():
    """A partial that starts 4 bytes past a 16-byte boundary takes the scalar copy path."""
    n, D = 300, 128
    ex = PeerExchange(n, D)
    try:
        buf = torch.empty(n * (D + 1) + 1, dtype=torch.float32, device=DEV)
        part = buf[1:]
        part.copy_(_part(n, D, 7))
        out = torch.empty(n, D, dtype=torch.float32, device=DEV)
        ex.merge(part, out)
        ref = torch.empty_like(out)
        attention.merge_partials(part.contiguous().clone(), 1, n, D, ref)
        ex.status()
        assert torch.equal(out, ref)
    finally:
        ex.close()


@pytest.mark.parametrize("kt,D,grp", [(3, 128, 8), (4, 256, 4)])
def test_peer_exchange_fused_attention_single_rank(kt, D, grp):
    from leankv_b200 import ops
    B, Hkv, T = 3, 2, 1000
    g = torch.Generator(device=DEV).manual_seed(kt + D)
    kc = ops.quantize(torch.randn(B, Hkv, T, D, device=DEV, generator=g), kt, fwht_head_dim=D)
    vc = ops.quantize(torch.randn(B, Hkv, T, D, device=DEV, generator=g), 4, fwht_head_dim=D)
    lens = torch.tensor([1000, 517, 0], dtype=torch.int32, device=DEV)[:B]
    n = B * Hkv * grp
    ex = PeerExchange(n, D)
    try:
        for step in range(4):
            q = torch.randn(B, Hkv * grp, D, device=DEV, generator=g).half()
            o, lse = attention.decode_attention(q, kc, vc, kv_len=lens, return_lse=True)
            ref = torch.empty(n, D, dtype=torch.float32, device=DEV)
            attention.merge_partials(torch.cat([o.reshape(-1), lse.reshape(-1)]), 1, n, D, ref)
            out = torch.empty(B, Hkv * grp, D, dtype=torch.float32, device=DEV)
            if step == 2:   # a merge step in between keeps the arrival counts in step
                ex.merge(torch.cat([o.reshape(-1), lse.reshape(-1)]).contiguous(), out.view(n, D))
            else:
                ex.attention(q, kc, vc, out, kv_len=lens)
            ex.status()
            assert torch.equal(out.view(n, D), ref), step
    finally:
        ex.close()
