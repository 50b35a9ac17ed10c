"""Split-by-sequence decode attention across GPUs over NCCL (needs >= 2 GPUs).

Each rank holds one token shard of every context; after the all_gather and the
merge, every rank's output must equal the single-GPU attention over the whole
context (same kernels, so the only difference is the split and the merge).
On a single-GPU machine the test is skipped; the exchange logic itself is
covered on CPU ranks by test_distributed_cpu.py.
"""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _caches(dev):
    from leankv_b200 import ops
    B, Hkv, grp, T, D = 4, 8, 8, 20000, 128
    g = torch.Generator(device=dev).manual_seed(21)
    kc = ops.quantize(torch.randn(B, Hkv, T, D, device=dev, generator=g), 3, fwht_head_dim=D)
    vc = ops.quantize(torch.randn(B, Hkv, T, D, device=dev, generator=g), 4, fwht_head_dim=D)
    q = torch.randn(B, Hkv * grp, D, device=dev, generator=g).half()
    lens = torch.tensor([20000, 19999, 7001, 0], dtype=torch.int32, device=dev)
    return q, kc, vc, lens


def _rank(rank, world, port, outdir):
    import datetime
    import torch.distributed as dist
    from leankv_b200 import attention
    from leankv_b200.distributed import SplitSequenceAttention, local_lengths, token_shard
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        q, kc, vc, lens = _caches(dev)
        s0, s1 = token_shard(kc.shape[2], rank, world)
        att = SplitSequenceAttention()
        out = att(q, kc[:, :, s0:s1].contiguous(), vc[:, :, s0:s1].contiguous(), local_lengths(lens, s0, s1),
                  s1 - s0, out_dtype=torch.float32)
        full = attention.decode_attention(q, kc, vc, kv_len=lens)
        np.save(os.path.join(outdir, f"r{rank}.npy"), np.stack([out.cpu().numpy(), full.cpu().numpy()]))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs >= 2 GPUs")
def test_split_sequence_nccl(tmp_path):
    import torch.multiprocessing as mp
    world = min(torch.cuda.device_count(), 8)
    mp.start_processes(_rank, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method="spawn")
    for r in range(world):
        out, full = np.load(tmp_path / f"r{r}.npy")
        err = np.abs(out - full).max()
        assert err <= 1e-3 * np.abs(full).max() + 1e-6, (r, err)
