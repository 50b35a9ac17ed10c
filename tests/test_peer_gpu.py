"""tq_peer_exchange on one GPU: the push / arrival count / bounded wait / merge kernel
with a world of one rank (every CTA pushes into its own GPU's buffer), over several
steps so both slot buffers and the never-reset arrival counter are exercised.  The
merge must equal tq_lse_merge_cuda bit for bit (same arithmetic, same order).  The
multi-rank exchange over NVLink is tested in test_multigpu_gpu.py (>= 2 GPUs).
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
