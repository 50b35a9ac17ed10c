"""Multi-GPU partitioning of the TurboQuant decode path (one process per GPU).

The decode attention divides two ways:

* By (sequence, KV head).  Each rank owns whole contexts, so ranks never
  exchange data: ``batch_shard`` gives the rank's sequence range.  This covers
  the codec and short or medium contexts (the streaming append + decode path).
* By token position, for long contexts.  Every rank holds one contiguous token
  range of every (sequence, KV head) context (``token_shard``).  It computes
  attention over that range together with its log-sum-exp, and the partials are
  merged exactly:

      M = max_r lse_r,   O = sum_r e^{lse_r - M} O_r / sum_r e^{lse_r - M},
      lse = M + log sum_r e^{lse_r - M}

  The single exchange is one all_gather of every rank's packed [O_r | lse_r]
  (batch * n_q_heads * (head_dim + 1) float32 values) over the process group,
  which is NCCL over NVLink on a B200 node.  Each rank then merges the P partials
  itself (tq_lse_merge_cuda), so every rank ends up holding the full output.

  ``transport="peer"`` fuses the exchange into the attention
  (tq_peer_exchange_attention): the decode kernel's CTA that completes a
  (sequence, KV head) pair stores that pair's rows straight into its slot of
  every rank's exchange buffer over NVLink (CUDA IPC mappings, plain peer
  stores) and counts the pair in every rank's arrival counter (system-scope
  atomics), so the transfers of early pairs overlap the attention of later
  ones; a merge kernel then waits (bounded) for all ranks' pairs and merges
  them with the arithmetic of tq_lse_merge_cuda.  ``transport="peer_merge"``
  runs the attention first and then one push + merge kernel per rank
  (tq_peer_exchange_merge).  All transports give bit-identical outputs.  The
  peer transports need one GPU per rank on one node.

The output rotation (FWHT) is linear and is applied inside each rank's partial;
the merge is a convex combination, so it commutes with the rotation.
"""
from __future__ import annotations

import ctypes as C
from typing import Callable

import torch
import torch.distributed as dist

from . import _lib as L
from . import attention
from .ops import _DTYPES, _stream


def batch_shard(batch: int, rank: int, world: int) -> tuple[int, int]:
    """[start, stop) of the sequences owned by `rank` (contiguous, sizes differ by at most one)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad rank / world size")
    base, extra = divmod(batch, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def token_shard(context: int, rank: int, world: int) -> tuple[int, int]:
    """[start, stop) of the token positions held by `rank` for a context of `context` tokens.

    Ranges are contiguous, in rank order, and start on even positions (cache
    capacities stay even, as the decode attention requires); trailing ranks may
    get fewer tokens, or none, when the context is short.
    """
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad rank / world size")
    per = -(-context // world)
    per += per & 1
    start = min(rank * per, context)
    return start, min(start + per, context)


def local_lengths(kv_len: torch.Tensor, start: int, stop: int) -> torch.Tensor:
    """Valid tokens of each sequence inside the shard [start, stop): clamp(kv_len - start, 0, stop - start)."""
    return (kv_len.to(torch.int64) - start).clamp_(0, stop - start).to(torch.int32)


class PeerSetupError(RuntimeError):
    """The peer exchange could not be set up on every rank; raised on all ranks together."""


def _all_ranks_ok(ok: bool, group) -> bool:
    """Collective: True when `ok` holds on every rank of `group`."""
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return ok
    dev = "cuda" if dist.get_backend(group) == "nccl" else "cpu"
    flag = torch.tensor([1 if ok else 0], dtype=torch.int32, device=dev)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=group)
    return bool(flag.item())


class PeerExchange:
    """Exchange buffers of one rank for tq_peer_exchange_merge (CUDA IPC over NVLink).

    Created collectively: every rank of `group` allocates its buffer, the IPC
    handles are all-gathered over the process group (host objects), and every
    rank maps the others'.  Setup is all or nothing: every rank takes the same
    collective steps whatever fails locally, the ranks agree on the outcome, and
    if any rank failed (no CUDA device, two ranks on one GPU, an allocation or a
    mapping refused) every rank unmaps, waits for the others, frees, and raises
    PeerSetupError.  `merge(part, out, lse_out)` then runs one step on the
    current stream; every rank must call it the same number of times, in order.
    `wait_ms` bounds each step's wait for the other ranks (0: 2000 ms).  A wait
    that runs out leaves `out` unmerged and the exchange unusable; `status()`
    reports it, and recovery is `close()` plus a new PeerExchange on every rank.
    `close()` unmaps, waits for all ranks, and frees (collective as well).
    """

    def __init__(self, n_rows: int, head_dim: int, group=None, wait_ms: int = 0):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.n_rows, self.head_dim = n_rows, head_dim
        lib = L.load()
        self._ex = C.c_void_p()
        err = None
        uuid = None
        try:
            dev = torch.cuda.current_device()
            uuid = str(torch.cuda.get_device_properties(dev).uuid)
        except Exception as e:          # no usable CUDA device on this rank
            err = f"rank {self.rank}: no CUDA device ({e})"
        if self.world > 1:
            # the kernel of one rank waits for the kernels of the others: one GPU per rank
            ids = [None] * self.world
            dist.all_gather_object(ids, uuid, group=group)
            if err is None and (None in ids or len(set(ids)) != self.world):
                err = "the peer exchange needs a distinct GPU for every rank"
        raw = b""
        if err is None:
            handle = C.create_string_buffer(L.TQ_PEER_HANDLE_BYTES)
            st = lib.tq_peer_exchange_create(self.world, self.rank, n_rows, head_dim, int(wait_ms),
                                             C.byref(self._ex), handle)
            if st:
                err = f"rank {self.rank}: create: {lib.tq_last_error_string().decode(errors='replace')}"
                self._ex = C.c_void_p()
            else:
                raw = handle.raw
        handles = [raw]
        if self.world > 1:
            handles = [None] * self.world
            dist.all_gather_object(handles, raw, group=group)
        if err is None:
            if any(len(h) != L.TQ_PEER_HANDLE_BYTES for h in handles):
                err = "another rank could not create its exchange buffer"
            else:
                st = lib.tq_peer_exchange_connect(self._ex, b"".join(handles))
                if st:
                    err = f"rank {self.rank}: connect: {lib.tq_last_error_string().decode(errors='replace')}"
        if not _all_ranks_ok(err is None, group):
            # undo in the order of close(): unmap, wait until no rank maps a peer's buffer, free
            if self._ex:
                lib.tq_peer_exchange_disconnect(self._ex)
            if self.world > 1:
                dist.barrier(group=group)
            if self._ex:
                lib.tq_peer_exchange_destroy(self._ex)
                self._ex = C.c_void_p()
            raise PeerSetupError(err or "another rank could not set up the peer exchange")

    def merge(self, part: torch.Tensor, out: torch.Tensor, lse_out: torch.Tensor | None = None) -> torch.Tensor:
        n, D = self.n_rows, self.head_dim
        if part.dtype != torch.float32 or part.numel() != n * (D + 1) or not part.is_contiguous():
            raise ValueError("part must be a contiguous float32 [n_rows * (head_dim + 1)] tensor")
        if out.numel() != n * D or not out.is_contiguous() or out.dtype not in _DTYPES:
            raise ValueError("out must be a contiguous [n_rows, head_dim] float32 / float16 / bfloat16 tensor")
        L.check(L.load().tq_peer_exchange_merge(self._ex, part.data_ptr(), out.data_ptr(), _DTYPES[out.dtype],
                                                lse_out.data_ptr() if lse_out is not None else None,
                                                _stream(part)))
        return out

    def attention(self, q: torch.Tensor, k_shard: torch.Tensor, v_shard: torch.Tensor, out: torch.Tensor,
                  kv_len: torch.Tensor | None = None, max_kv_len: int | None = None, sm_scale: float | None = None,
                  lse_out: torch.Tensor | None = None, rotate_q: bool = True, v_rotated: bool = True) -> torch.Tensor:
        """One step with the exchange fused into the decode attention (tq_peer_exchange_attention): the
        attention over this rank's token shard stores every (sequence, KV head) pair's rows into all
        ranks' slots as soon as the pair is done; a merge kernel waits for every rank and writes the
        merged [B, Hq, D] output to `out`."""
        B, Hq, D = q.shape
        if B * Hq != self.n_rows or D != self.head_dim:
            raise ValueError("q does not match the exchange's rows / head_dim")
        if out.numel() != self.n_rows * D or not out.is_contiguous() or out.dtype not in _DTYPES:
            raise ValueError("out must be a contiguous [B, Hq, D] float32 / float16 / bfloat16 tensor")
        attention._need_cuda(q, k_shard, v_shard, out)
        if kv_len is not None:
            kv_len = kv_len.contiguous()
        k_type = 4 if k_shard.shape[-1] == 18 else 3
        a = attention.make_args(q.contiguous(), k_shard, v_shard, kv_len, max_kv_len or 0, sm_scale or 0.0, rotate_q,
                                v_rotated, out, None, k_type, 4)
        lib = attention._bind()
        need = lib.tq_decode_attention_workspace_size(C.byref(a))
        if need == 0:
            L.check(lib.tq_decode_attention_cuda(C.byref(a), _stream(q)))   # reports the argument error
        ws = attention._workspace(q.device, need)
        a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
        L.check(L.load().tq_peer_exchange_attention(self._ex, C.byref(a), out.data_ptr(), _DTYPES[out.dtype],
                                                    lse_out.data_ptr() if lse_out is not None else None, _stream(q)))
        return out

    def status(self) -> None:
        """Synchronize the current stream and raise if a step's wait ran out."""
        L.check(L.load().tq_peer_exchange_status(self._ex, torch.cuda.current_stream().cuda_stream))

    def close(self) -> None:
        if not self._ex:
            return
        lib = L.load()
        torch.cuda.synchronize()
        L.check(lib.tq_peer_exchange_disconnect(self._ex))
        if self.world > 1:
            dist.barrier(group=self.group)   # no rank frees its buffer while another still maps it
        L.check(lib.tq_peer_exchange_destroy(self._ex))
        self._ex = C.c_void_p()


class SplitSequenceAttention:
    """Decode attention over contexts split across ranks by token position.

    Call it on every rank of `group` with the same query and that rank's shard of
    the caches (``token_shard``); all ranks return the merged output.  Buffers for
    the exchange are allocated once per shape and reused, so steps issue no
    allocation.

    ``attend(q, k, v, kv_len, max_kv_len, o_out, lse_out)`` and
    ``merge(parts, n_parts, n_rows, head_dim, out)`` default to the CUDA
    kernels; they are parameters so that the exchange logic can run on CPU ranks
    (gloo) with CPU stand-ins.  ``transport``: "nccl" (all_gather over the
    process group, then the merge kernel), "peer" (PeerExchange with the
    exchange fused into the decode attention: each pair's rows go to every rank
    over NVLink as soon as the pair is done, then a merge kernel) or
    "peer_merge" (PeerExchange: the attention, then one push + merge kernel over
    NVLink peer memory).  For both peer transports call ``close()`` on every
    rank when done.

    With the peer transport a step whose wait for the other ranks runs out
    (``wait_ms``, 0: 2000 ms) leaves its output unmerged and only records the
    failure on the device: callers must call ``status()``, which synchronizes
    and raises TQError, before trusting any output of the steps so far.
    """

    def __init__(self, group=None, attend: Callable | None = None, merge: Callable | None = None,
                 transport: str = "nccl", wait_ms: int = 0):
        if transport not in ("nccl", "peer", "peer_merge"):
            raise ValueError("transport must be 'nccl', 'peer' or 'peer_merge'")
        if transport == "peer" and attend is not None:
            raise ValueError("the fused peer transport runs the CUDA attention itself; use 'peer_merge' with attend")
        self.transport = transport
        self.fallback = None   # why a peer transport was replaced by NCCL, if it was
        self.wait_ms = wait_ms
        self._peers: dict = {}
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if self.world > 1 else 0
        self._attend = attend or self._cuda_attend
        self._merge = merge or attention.merge_partials
        self._bufs: dict = {}

    @staticmethod
    def _cuda_attend(q, k, v, kv_len, max_kv_len, o_out, lse_out, **kw):
        attention.decode_attention(q, k, v, kv_len=kv_len, max_kv_len=max_kv_len, out=o_out, lse_out=lse_out,
                                   return_lse=True, **kw)

    def _buffers(self, n_rows: int, head_dim: int, device):
        key = (n_rows, head_dim, str(device))
        b = self._bufs.get(key)
        if b is None:
            per = n_rows * (head_dim + 1)
            send = torch.empty(per, dtype=torch.float32, device=device)
            # the all_gather destination; the peer transport gathers into its own exchange buffers
            recv = (torch.empty(self.world * per, dtype=torch.float32, device=device)
                    if self.transport == "nccl" and self.world > 1 else None)
            b = self._bufs[key] = (send, recv)
        return b

    def __call__(self, q: torch.Tensor, k_shard: torch.Tensor, v_shard: torch.Tensor,
                 kv_len_local: torch.Tensor | None = None, max_kv_len: int | None = None,
                 out: torch.Tensor | None = None, out_dtype: torch.dtype = torch.float32, **kw) -> torch.Tensor:
        B, Hq, D = q.shape
        n = B * Hq
        if out is None:
            out = torch.empty((B, Hq, D), dtype=out_dtype, device=q.device)
        if self.transport == "peer":
            ex = self._peer(n, D, q.device)
            if ex is not None:
                return ex.attention(q, k_shard, v_shard, out, kv_len_local, max_kv_len, **kw)
        send, recv = self._buffers(n, D, q.device)
        o_local = send[: n * D].view(B, Hq, D)
        lse_local = send[n * D:].view(B, Hq)
        self._attend(q, k_shard, v_shard, kv_len_local, max_kv_len, o_local, lse_local, **kw)
        if self.transport == "peer_merge":
            ex = self._peer(n, D, q.device)
            if ex is not None:
                ex.merge(send, out.view(n, D))
                return out
        if self.world == 1:
            self._merge(send, 1, n, D, out.view(n, D))
            return out
        if recv is None:   # a peer transport whose setup failed on some rank: all ranks take NCCL
            recv = torch.empty(self.world * send.numel(), dtype=torch.float32, device=send.device)
            self._bufs[(n, D, str(q.device))] = (send, recv)
        dist.all_gather_into_tensor(recv, send, group=self.group)
        self._merge(recv, self.world, n, D, out.view(n, D))
        return out

    def _peer(self, n: int, D: int, device):
        """The exchange for this shape, set up on first use; None after a failed setup, when
        every rank has switched to the NCCL transport (and `fallback` holds the reason)."""
        key = (n, D, str(device))
        ex = self._peers.get(key)
        if ex is None:
            try:
                ex = self._peers[key] = PeerExchange(n, D, self.group, self.wait_ms)
            except PeerSetupError as e:    # raised on every rank together
                self.fallback = f"{self.transport} setup failed ({e}); NCCL all_gather + merge instead"
                self.transport = "nccl"
                return None
        return ex

    def status(self) -> None:
        """Peer transport: synchronize and raise if a step's wait ran out."""
        for ex in self._peers.values():
            ex.status()

    def close(self) -> None:
        """Release the peer exchanges (collective: every rank calls it)."""
        for key in sorted(self._peers):
            self._peers[key].close()
        self._peers.clear()
