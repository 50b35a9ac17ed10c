"""Split-by-sequence decode attention across GPUs (needs >= 2 GPUs).

Each rank holds one token shard of every context; after the exchange and the
merge, every rank's output must equal the single-GPU attention over the whole
context (same kernels, so the only difference is the split and the merge).
Two transports: NCCL all_gather + merge kernel, and the peer-memory kernel
(tq_peer_exchange_merge), whose output must equal the NCCL path's bit for bit
over several steps.  A rank that never joins a peer step makes the other
rank's bounded wait run out (TQ_ERROR_TIMEOUT, read on the host).  On a
single-GPU machine the tests are skipped; the exchange logic is covered on CPU
ranks by test_distributed_cpu.py and the peer kernel's single-rank path by
test_peer_gpu.py.
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
        ks, vs, ll = kc[:, :, s0:s1].contiguous(), vc[:, :, s0:s1].contiguous(), local_lengths(lens, s0, s1)
        att = SplitSequenceAttention()
        out = att(q, ks, vs, ll, s1 - s0, out_dtype=torch.float32)
        full = attention.decode_attention(q, kc, vc, kv_len=lens)
        outs = []
        for transport in ("peer", "peer_merge"):
            peer = SplitSequenceAttention(transport=transport)
            for _ in range(3):   # both slot buffers, the arrival counter over several steps
                outs.append(peer(q, ks, vs, ll, s1 - s0, out_dtype=torch.float32).cpu().numpy())
            peer.status()
            peer.close()
        np.save(os.path.join(outdir, f"r{rank}.npy"), np.stack([out.cpu().numpy(), full.cpu().numpy()] + outs))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _rank_absent_peer(rank, world, port, outdir):
    """Rank 0 runs one peer step; the others never do: rank 0's wait must run out and report it."""
    import datetime
    import torch.distributed as dist
    from leankv_b200._lib import TQError
    from leankv_b200.distributed import PeerExchange
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        n, D = 64, 128
        ex = PeerExchange(n, D)
        result = "no step"
        if rank == 0:
            part = torch.zeros(n * (D + 1), dtype=torch.float32, device=dev)
            out = torch.empty(n, D, dtype=torch.float32, device=dev)
            ex.merge(part, out)
            try:
                ex.status()
                result = "ok"
            except TQError as e:
                result = "timeout" if e.status == 7 else f"status {e.status}"
        dist.barrier()
        ex.close()
        with open(os.path.join(outdir, f"absent{rank}.txt"), "w") as f:
            f.write(result)
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs >= 2 GPUs")
def test_split_sequence_nccl(tmp_path):
    import torch.multiprocessing as mp
    world = min(torch.cuda.device_count(), 8)
    mp.start_processes(_rank, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method="spawn")
    for r in range(world):
        out, full, *peer = np.load(tmp_path / f"r{r}.npy")
        err = np.abs(out - full).max()
        assert err <= 1e-3 * np.abs(full).max() + 1e-6, (r, err)
        for step, p in enumerate(peer):
            assert np.array_equal(p, out), (r, step)


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs >= 2 GPUs")
def test_peer_exchange_absent_rank_times_out(tmp_path):
    import torch.multiprocessing as mp
    mp.start_processes(_rank_absent_peer, args=(2, _free_port(), str(tmp_path)), nprocs=2, start_method="spawn")
    assert (tmp_path / "absent0.txt").read_text() == "timeout"
    assert (tmp_path / "absent1.txt").read_text() == "no step"
