"""Host logic of the multi-GPU paths on CPU ranks (gloo, world sizes 2 and 3).

The split-by-sequence attention runs its real exchange (all_gather of packed
[O | lse] partials) with the float64 oracle standing in for the CUDA kernels on
each rank; the merged result must equal the oracle's attention over the whole
context.  The shard helpers are checked for coverage and evenness.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from leankv_b200.distributed import SplitSequenceAttention, batch_shard, local_lengths, token_shard

B, HKV, GRP, T, D = 2, 2, 4, 300, 128
LENS = [300, 131]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _problem():
    from oracle import oracle as O
    rng = np.random.default_rng(11)
    k = rng.standard_normal((B, HKV, T, D), dtype=np.float32)
    v = rng.standard_normal((B, HKV, T, D), dtype=np.float32)
    k[..., :4] *= 20.0
    kc = O.ref_quantize(3, O.ref_fwht(k, D)).reshape(B, HKV, T, D // 32, 14)
    vc = O.ref_quantize(4, O.ref_fwht(v, D)).reshape(B, HKV, T, D // 32, 18)
    q = rng.standard_normal((B, HKV * GRP, D), dtype=np.float32)
    return q, kc, vc


def _cpu_attend(q, k, v, kv_len, max_kv_len, o_out, lse_out):
    from oracle import oracle as O
    o, lse = O.decode_attention(q.numpy(), k.numpy(), 3, v.numpy(), 4, HKV, kv_len=kv_len.numpy())
    o_out.copy_(torch.from_numpy(o))
    lse_out.copy_(torch.from_numpy(lse))


def _cpu_merge(parts, n_parts, n_rows, head_dim, out):
    from oracle import oracle as O
    p = parts[: n_parts * n_rows * (head_dim + 1)].view(n_parts, n_rows * (head_dim + 1))
    o = p[:, : n_rows * head_dim].reshape(n_parts, n_rows, head_dim).numpy()
    lse = p[:, n_rows * head_dim:].numpy()
    m, _ = O.lse_combine(o, lse)
    out.copy_(torch.from_numpy(m))
    return out


def _rank_main(rank, world, port, result_dir, transport="nccl"):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q, kc, vc = _problem()
        s0, s1 = token_shard(T, rank, world)
        lens = local_lengths(torch.tensor(LENS, dtype=torch.int32), s0, s1)
        att = SplitSequenceAttention(attend=_cpu_attend, merge=_cpu_merge, transport=transport)
        assert att.world == world and att.rank == rank
        out = att(torch.from_numpy(q), torch.from_numpy(np.ascontiguousarray(kc[:, :, s0:s1])),
                  torch.from_numpy(np.ascontiguousarray(vc[:, :, s0:s1])), lens, s1 - s0)
        if transport != "nccl":
            # CPU ranks cannot set up the peer exchange: every rank agreed and took NCCL
            assert att.transport == "nccl" and "setup failed" in att.fallback, att.fallback
        att.close()
        np.save(os.path.join(result_dir, f"out{rank}.npy"), out.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_split_sequence_gloo_matches_full_context(orc, tmp_path, world):
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method="spawn")
    q, kc, vc = _problem()
    ref, _ = orc.decode_attention(q, kc, 3, vc, 4, HKV, kv_len=np.array(LENS))
    for r in range(world):
        out = np.load(tmp_path / f"out{r}.npy")
        np.testing.assert_allclose(out, ref, rtol=1e-5, atol=1e-5 * np.abs(ref).max())


@pytest.mark.parametrize("n,world", [(131072, 8), (300, 3), (7, 4), (2, 8), (0, 2), (32, 1)])
def test_token_shard_covers_context(n, world):
    spans = [token_shard(n, r, world) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == n
    for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
        assert a1 == b0 and a0 <= a1
    assert all(s0 % 2 == 0 for s0, _ in spans)


@pytest.mark.parametrize("b,world", [(64, 8), (32, 8), (5, 3), (2, 4)])
def test_batch_shard_even(b, world):
    spans = [batch_shard(b, r, world) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == b
    sizes = [s1 - s0 for s0, s1 in spans]
    assert max(sizes) - min(sizes) <= 1
    assert all(a[1] == c[0] for a, c in zip(spans, spans[1:]))


def test_local_lengths_clamp():
    kv = torch.tensor([0, 5, 100, 1000], dtype=torch.int32)
    assert local_lengths(kv, 64, 128).tolist() == [0, 0, 36, 64]
    assert local_lengths(kv, 0, 64).tolist() == [0, 5, 64, 64]


def test_peer_setup_failure_falls_back_on_every_rank(orc, tmp_path):
    """A peer exchange that cannot be set up on some rank fails on all ranks together (one
    agreement after the same collective steps), and the split attention continues over the
    NCCL path: no rank hangs in a collective the others skipped."""
    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path), "peer_merge"), nprocs=world,
                       start_method="spawn")
    q, kc, vc = _problem()
    ref, _ = orc.decode_attention(q, kc, 3, vc, 4, HKV, kv_len=np.array(LENS))
    for r in range(world):
        out = np.load(tmp_path / f"out{r}.npy")
        np.testing.assert_allclose(out, ref, rtol=1e-5, atol=1e-5 * np.abs(ref).max())
