#!/usr/bin/env python3
"""Benchmark of the TurboQuant KV-cache hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]

Workloads (synthetic, seeded; shapes and distributions of the LeanKV configs):
  c4      (default) fused decode attention over a TQ3_0 K / TQ4_0 V cache, B64 Hq64 Hkv8 D128,
          context 131072; N > 1 ranks split every context by token position; the decode kernel
          stores each finished pair's (O, lse) into every rank's buffer over NVLink, then a merge
  tq3opt  TQ3_0 + optimal rounding (2 CD passes + LS scale), FWHT fused,
          bf16 [32768 tokens, 8 KV heads, 128]: Student-t(4) x per-channel log-normal scales
  tq4     TQ4_0 quantize (FWHT fused) + dequantize of fp32 [4096, 8, 128], N(0,1) with
          4 outlier channels per head x20
  attn    fused TQ4/TQ4 decode attention, B16 Hq32 Hkv8 D128 ctx 32768 (ranks split the batch)
  c5      streaming append + decode, 80 layers, head_dim 256, 256 decode steps (ranks split the batch)

A step is one pass of the hot path over one batch that is resident in HBM.
`value` is whole-job throughput (all ranks, GB/s of packed KV read for the attention
workloads); `e2e` is the same metric through the public API with host buffers (H2D + D2H
inside the timed region).  One process per GPU (torchrun for N > 1).
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

FALLBACK_HBM_GBS = 6650.0
L2_FLUSH_BYTES = 256 << 20
METRIC = "TQ4/TQ3 KV quantize GB/s; fused decode-attn µs/step; % HBM roofline @1/2/4/8"


# ── helpers ────────────────────────────────────────────────────────────────────

def hbm_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def profile_traffic(workload: str):
    """dram bytes per launch recorded from an ncu capture in profiles/ (None if absent)."""
    path = os.path.join(ROOT, "profiles", "traffic_per_launch.txt")
    try:
        for line in open(path):
            parts = line.split()
            if len(parts) >= 2 and parts[0] == workload:
                return float(parts[1])
    except OSError:
        pass
    return None


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int, period_ms: int = 50):
        self.lines = []
        self.proc = None
        self.device_index = device_index
        self.period_ms = period_ms

    def __enter__(self):
        try:
            import torch
            props = torch.cuda.get_device_properties(self.device_index)
            ident = getattr(props, "pci_bus_id", None)
            sel = []
            if ident is not None:
                sel = ["-i", f"{getattr(props, 'pci_domain_id', 0):08X}:{props.pci_bus_id:02X}:"
                             f"{getattr(props, 'pci_device_id', 0):02X}.0"]
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          f"-lms={self.period_ms}", *sel],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            time.sleep(0.15)
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc is not None:
            time.sleep(0.1)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["active", "hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names[1:], f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_setup():
    import torch
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        # rank 0 prints exactly one JSON line on stdout; NCCL prints its version banner with
        # printf (NCCL_DEBUG=WARN or VERSION) when the communicator is created, so fd 1 points at
        # stderr until the first collective has run (C stdio flushed before it is restored)
        libc = C.CDLL(None)
        sys.stdout.flush()
        saved = os.dup(1)
        os.dup2(2, 1)
        try:
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", local))
            dist.barrier()
        finally:
            libc.fflush(None)
            sys.stdout.flush()
            os.dup2(saved, 1)
            os.close(saved)
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return ws, rank, local


def barrier(ws):
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x: float, ws: int) -> float:
    if ws == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ── workloads ──────────────────────────────────────────────────────────────────

# Workload names as both arms report them (the reference arm uses the same strings).
WORKLOAD = {
    "tq3opt": "TQ3_0 optimal-rounding quantize (2 CD passes + LS scale), FWHT fused",
    "tq4": "C1 TQ4_0 quantize (FWHT fused) + dequantize round trip",
    "attn": "C3 fused TQ4_0/TQ4_0 decode attention (FWHT(q), split-KV, LSE combine, FWHT(o))",
    "c4": "C4 fused TQ3_0-K / TQ4_0-V decode attention, split-KV by sequence",
    "c5": "C5 streaming append + decode, 80-layer TQ4_0 KV cache, one CUDA graph per step",
}
INPUT = {
    "tq3opt": "bf16 [32768 tokens, 8 KV heads, 128], Student-t(4) x log-normal channel scales",
    "tq4": "fp32 [4096 tokens, 8 KV heads, 128], N(0,1) + 4 outlier channels per head x20",
}


def c2_input(seed: int, tokens=32768, heads=8, hd=128):
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    # Student-t(4) = N / sqrt(chi2_4 / 4); chi2_4 = sum of 4 squared normals
    n = torch.randn(tokens, heads, hd, generator=g, device="cuda")
    chi = torch.zeros_like(n)
    for _ in range(4):
        chi += torch.randn(tokens, heads, hd, generator=g, device="cuda") ** 2
    t = n / torch.sqrt(chi / 4.0)
    scale = torch.exp(torch.randn(1, heads, hd, generator=g, device="cuda"))
    return (t * scale).to(torch.bfloat16).contiguous()


def c1_input(seed: int, tokens=4096, heads=8, hd=128):
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(tokens, heads, hd, generator=g, device="cuda")
    for h in range(heads):
        ch = torch.randperm(hd, generator=g, device="cuda")[:4]
        x[:, h, ch] *= 20.0
    return x.contiguous()


class Codec:
    """One workload of the codec family: step() launches the hot path once."""

    def __init__(self, name, rank, tokens=None):
        import torch
        from leankv_b200 import ops
        self.name = name
        if name == "tq3opt":
            self.x = c2_input(2 + 1000 * rank, tokens=tokens or 32768)
            self.qtype, self.hd, self.passes = 3, 128, 2
            self.limiter = ("instruction issue of the float64 coordinate descent (two passes x 32 elements x two "
                            "neighbours per block); DRAM is about 6 % busy, so the HBM fraction is not the bound")
            self.config = {"workload": WORKLOAD["tq3opt"], "input": INPUT["tq3opt"],
                           "blocks_per_step": self.x.numel() // 32}
        else:
            self.x = c1_input(1 + 1000 * rank, tokens=tokens or 4096)
            self.qtype, self.hd, self.passes = 4, 128, 0
            self.config = {"workload": WORKLOAD["tq4"], "input": INPUT["tq4"],
                           "blocks_per_step": self.x.numel() // 32}
        self.round_trip = self.qtype == 4
        self.k = self.x.numel()
        bb = 14 if self.qtype == 3 else 18
        self.y = torch.empty(self.k // 32 * bb, dtype=torch.uint8, device="cuda")
        self.bytes_per_step = self.k * self.x.element_size() + self.k // 32 * bb
        self.ops = ops
        self.launches_per_step = 1
        self.dtype = "bf16->u8 (fp32/fp64 math)" if self.passes else "f32->u8"
        if self.round_trip:
            # dequantize back to fp32 (rotated domain, as dequantize_row_tq4_0 returns it)
            self.xr = torch.empty_like(self.x)
            self.bytes_per_step *= 2
            self.launches_per_step = 2
            self.dtype = "f32->u8->f32"
            self.step()
            rot = self.x.clone()
            ops.hadamard_(rot, self.hd)
            err = (self.xr - rot).double()
            mse = float(err.pow(2).mean())
            self.config["reconstruction_mse"] = round(mse, 8)
            self.config["relative_mse"] = round(mse / float(rot.double().pow(2).mean()), 8)

    def step(self):
        self.ops.quantize(self.x, self.qtype, fwht_head_dim=self.hd, opt_passes=self.passes, out=self.y)
        if self.round_trip:
            self.ops.dequantize(self.y, self.qtype, out=self.xr)

    # end-to-end through the C ABI with pinned host buffers
    def e2e_setup(self):
        import torch
        self.hx = self.x.cpu().pin_memory()
        self.hy = torch.empty(self.y.numel(), dtype=torch.uint8).pin_memory()
        if self.round_trip:
            self.hxr = torch.empty_like(self.hx).pin_memory()

    def e2e_step(self):
        from leankv_b200 import _lib as L
        dt = {2: L.DTYPE_BF16, 4: L.DTYPE_F32}[self.x.element_size()]
        L.check(L.load().tq_quantize_host(self.qtype, C.c_void_p(self.hx.data_ptr()), dt,
                                          C.c_void_p(self.hy.data_ptr()), self.k, self.hd, self.passes))
        if self.round_trip:
            L.check(L.load().tq_dequantize_host(self.qtype, C.c_void_p(self.hy.data_ptr()),
                                                C.c_void_p(self.hxr.data_ptr()), L.DTYPE_F32, self.k))

    def e2e_bytes(self):
        h2d, d2h = self.hx.numel() * self.hx.element_size(), self.hy.numel()
        if self.round_trip:
            h2d, d2h = h2d + self.hy.numel(), d2h + self.hxr.numel() * 4
        return h2d, d2h



def _outlier_rows(g, shape, hd):
    """N(0,1) rows with 4 outlier channels per KV head scaled x20 (the C1 generator); shape [..., H, T, hd]."""
    import torch
    x = torch.randn(*shape, generator=g, device="cuda")
    H = shape[-3]
    for h in range(H):
        ch = torch.randperm(hd, generator=g, device="cuda")[:4]
        x[..., h, :, ch] *= 20.0
    return x


class Attn:
    """Fused decode attention.

    attn (C3): TQ4_0 K/V, B16 Hq32 Hkv8 D128 ctx 32768; ranks split the batch (no collective).
    c4   (C4): TQ3_0 K / TQ4_0 V, B64 Hq64 Hkv8 D128 ctx 131072; ranks split every context by
               token position, then one all_gather of the packed (O, lse) partials over NCCL and a
               log-sum-exp merge on every rank.
    Both keep the total work fixed as ranks are added ("strong" scaling).
    """

    def __init__(self, name, rank, ws, tokens=None, transport="nccl", page_size=0, page_order="shuffled"):
        import torch
        from leankv_b200 import attention, distributed, ops
        self.attention = attention
        self.name = name
        self.ws = ws
        if name == "attn":
            B, Hq, Hkv, D, T, kt = 16, 32, 8, 128, tokens or 32768, 4
            b0, b1 = distributed.batch_shard(B, rank, ws)
            s0, s1 = 0, T
        else:
            B, Hq, Hkv, D, T, kt = 64, 64, 8, 128, tokens or 131072, 3
            b0, b1 = 0, B
            s0, s1 = distributed.token_shard(T, rank, ws)
        Bl, L = b1 - b0, s1 - s0
        g = torch.Generator(device="cuda").manual_seed((3 if name == "attn" else 4) + 1000 * rank)
        kb = 18 if kt == 4 else 14
        kc = torch.empty(Bl, Hkv, L, D // 32, kb, dtype=torch.uint8, device="cuda")
        vc = torch.empty(Bl, Hkv, L, D // 32, 18, dtype=torch.uint8, device="cuda")
        for cache, qt in ((kc, kt), (vc, 4)):          # rotated + quantized rows
            for b in range(Bl):
                ops.quantize(_outlier_rows(g, (Hkv, L, D), D), qt, fwht_head_dim=D, out=cache[b])
        self.kc, self.vc = kc, vc
        self.page_size = page_size
        if page_size:
            # paged layout: the same token rows moved into page pools in a shuffled page order
            if L % page_size or (name == "c4" and ws > 1):
                raise SystemExit("--page-size needs a context that is a multiple of it (and one rank for c4)")
            npp = L // page_size
            perm = (torch.randperm(Bl * npp, generator=torch.Generator().manual_seed(6)) if page_order == "shuffled"
                    else torch.arange(Bl * npp)).cuda()
            self.table = perm.view(Bl, npp).to(torch.int32).contiguous()
            pools = []
            for c in (kc, vc):
                pool = torch.empty((Bl * npp, Hkv, page_size) + tuple(c.shape[3:]), dtype=torch.uint8, device="cuda")
                pool[perm] = c.view(Bl, Hkv, npp, page_size, *c.shape[3:]).transpose(1, 2).reshape(pool.shape)
                pools.append(pool)
            del kc, vc
            self.kc, self.vc = pools
            self.plens = torch.full((Bl,), L, dtype=torch.int32, device="cuda")
            torch.cuda.empty_cache()
        gq = torch.Generator(device="cuda").manual_seed(5)           # the same queries on every rank
        qfull = torch.randn(B, Hq, D, generator=gq, device="cuda").half()
        self.q = qfull[b0:b1].contiguous()
        self.out = torch.empty(Bl, Hq, D, dtype=torch.float16, device="cuda")
        self.L = L
        self.split = name == "c4" and ws > 1
        if self.split:
            self.att = distributed.SplitSequenceAttention(transport=transport)
            self.lens = torch.full((Bl,), L, dtype=torch.int32, device="cuda")
        kv_bytes = self.kc.numel() + self.vc.numel()
        self.bytes_per_step = kv_bytes + self.q.numel() * 2 + self.out.numel() * 2          # this rank
        kv_total = B * Hkv * T * (D // 32) * (kb + 18)
        self.job_bytes = kv_total + B * Hq * D * 2 * 2                                       # all ranks
        self.launches_per_step = 2 if self.split else 1        # decode (+ rank merge)
        self.scaling = "strong"
        self.flush_l2 = False
        self.l2_note = f"KV {kv_total / 1e9:.2f} GB per step (> L2 126 MB), no flush"
        if name == "attn":
            self.config = {"workload": WORKLOAD["attn"],
                           "shape": f"B={B} Hq={Hq} Hkv={Hkv} D={D} ctx={T}, fp16 q/out", "kv_bytes": kv_total}
            self.parallelism = f"batch shards x{ws} (sequences {b0}..{b1 - 1} on rank {rank}), no collective"
        else:
            self.config = {"workload": WORKLOAD["c4"],
                           "shape": f"B={B} Hq={Hq} Hkv={Hkv} D={D} ctx={T}, fp16 q/out", "kv_bytes": kv_total}
        if page_size:
            self.config["cache_layout"] = (f"paged: {page_size}-token pages of every KV head in page pools, "
                                           f"pages in {page_order} order through a page table")
            self.parallelism = (f"token shards x{ws} ({L} tokens per rank); " + (
                "all_gather of packed (O, lse) over NCCL + LSE merge on every rank" if transport == "nccl" else
                "exchange fused into the decode kernel: each pair's (O, lse) stored into every rank's buffer over "
                "NVLink (CUDA IPC peer stores) as soon as the pair is done, system-scope arrival counts, then an "
                "LSE merge kernel" if transport == "peer" else
                "after the decode kernel, one kernel per rank: (O, lse) stored into every rank's buffer over NVLink "
                "(CUDA IPC peer stores), system-scope arrival counts, LSE merge") if ws > 1 else
                "one GPU holds the whole context")
        self.dtype = "TQ blocks -> f16 MMA, f32 accumulate"
        self.e2e_path = "leankv_b200 decode attention, q H2D and out D2H from pinned host memory"

    def step(self):
        if self.split:
            self.att(self.q, self.kc, self.vc, self.lens, self.L, out=self.out)
        elif self.page_size:
            self.attention.decode_attention_paged(self.q, self.kc, self.vc, self.table, kv_len=self.plens,
                                                  max_kv_len=self.L, out=self.out)
        else:
            self.attention.decode_attention(self.q, self.kc, self.vc, out=self.out)

    def e2e_setup(self):
        self.hq = self.q.cpu().pin_memory()
        self.hout = self.out.cpu().pin_memory()

    def e2e_step(self):
        import torch
        self.q.copy_(self.hq, non_blocking=True)
        self.step()
        self.hout.copy_(self.out, non_blocking=True)
        torch.cuda.current_stream().synchronize()

    def e2e_bytes(self):
        return self.hq.numel() * 2, self.hout.numel() * 2



class Stream:
    """C5 streaming append + decode: 80 layers of a KV cache (8 KV heads, head_dim 256, TQ4_0 K/V).

    Prefill quantizes 16384 bf16 tokens per sequence into every layer (quantize-on-write with the
    head_dim Hadamard rotation).  A step is one decode step of all 80 layers: append one token's K
    and V per sequence at its current length, then decode attention (32 query heads, group 4) over
    the grown context.  The 80-layer step (240 kernel launches) is captured once in a CUDA graph
    and replayed; the append slots and lengths live on the device and advance inside the graph.
    Ranks split the batch of 32 ("strong" scaling, no collective).
    """
    LAYERS, HKV, HQ, D, BATCH, DECODE_STEPS = 80, 8, 32, 256, 32, 256
    GROWTH = DECODE_STEPS + 32            # + warm-up and end-to-end steps; capacity stays even

    def __init__(self, rank, ws, tokens=None, layers=None):
        import torch
        from leankv_b200 import attention, distributed, ops
        self.attention, self.ops = attention, ops
        self.nl = layers or self.LAYERS
        b0, b1 = distributed.batch_shard(self.BATCH, rank, ws)
        B = self.B = b1 - b0
        H, D, Hq = self.HKV, self.D, self.HQ
        T0 = tokens or 16384
        cap = self.cap = T0 + self.GROWTH
        nb = D // 32
        self.kc = [torch.empty(B, H, cap, nb, 18, dtype=torch.uint8, device="cuda") for _ in range(self.nl)]
        self.vc = [torch.empty(B, H, cap, nb, 18, dtype=torch.uint8, device="cuda") for _ in range(self.nl)]
        g = torch.Generator(device="cuda").manual_seed(5 + 1000 * rank)
        # prefill: quantize-on-write of every layer's K and V (bf16, head_dim rotation).  The whole input
        # (all layers) cannot be held, so two device-generated chunks of the configured shape and
        # distribution are reused across layers; one untimed launch loads the kernel, then all
        # launches run back to back between two events.
        chunk = max(1, min(B, (1 << 28) // (H * T0 * D)))
        pool = [_outlier_rows(g, (chunk, H, T0, D), D).to(torch.bfloat16) for _ in range(2)]
        ops.kv_append(pool[0][:min(chunk, B)], self.kc[0][:min(chunk, B)])
        pre_bytes, i = 0, 0
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record()
        for l in range(self.nl):
            for cache in (self.kc[l], self.vc[l]):
                for c0 in range(0, B, chunk):
                    c1 = min(B, c0 + chunk)
                    x = pool[i % 2][:c1 - c0]
                    ops.kv_append(x, cache[c0:c1])
                    pre_bytes += x.numel() * 2 + x.numel() // 32 * 18
                    i += 1
        e1.record()
        e1.synchronize()
        pre_ms = e0.elapsed_time(e1)
        del pool
        self.prefill = {"ms": round(pre_ms, 3), "bytes": pre_bytes, "GB_per_s": round(pre_bytes / pre_ms / 1e6, 1),
                        "tokens_per_seq": T0, "launches": self.nl * 2 * ((B + chunk - 1) // chunk)}
        # decode-step inputs for all layers in single buffers (one H2D / D2H each in e2e)
        self.k_new = torch.randn(self.nl, B, H, 1, D, generator=g, device="cuda").to(torch.bfloat16)
        self.v_new = torch.randn(self.nl, B, H, 1, D, generator=g, device="cuda").to(torch.bfloat16)
        self.q = torch.randn(self.nl, B, Hq, D, generator=g, device="cuda").to(torch.bfloat16)
        self.out = torch.empty(self.nl, B, Hq, D, dtype=torch.bfloat16, device="cuda")
        self.pos = torch.full((B,), T0, dtype=torch.int32, device="cuda")     # append slot = current length
        self.len1 = self.pos + 1                                                 # length after the append
        self.T0 = T0
        self.steps_done = 0
        for _ in range(2):                       # eager steps: workspace, kernel attributes, lazy init
            self._body()
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self._body()
        self.steps_done -= 1                     # capture records the step without running it
        self.launches_per_step = self.nl * 3                   # K append, V append, decode
        per_tok = H * nb * 18 * 2                                       # K + V bytes per token and sequence
        self._per_tok = per_tok
        self.scaling = "strong"
        self.flush_l2 = False
        self.l2_note = "cache > 10 GB per rank (> L2 126 MB), no flush"
        self.config = {"workload": WORKLOAD["c5"],
                       "shape": f"batch {self.BATCH} (x{ws} ranks: {B} each) Hkv={H} Hq={Hq} D={D} prefill {T0} "
                                f"+ up to {self.GROWTH} appended tokens, bf16 inputs/outputs",
                       "layers": self.nl, "prefill": self.prefill}
        self.parallelism = f"batch shards x{ws}, all layers local, no collective"
        self.dtype = "bf16 -> TQ4 blocks; TQ4 -> f16 MMA, f32 accumulate"
        self.e2e_path = ("CUDA graph of the 80-layer step; new K/V/q H2D and outputs D2H from pinned host memory "
                         "(one copy each)")
        self.job_ranks = ws

    def _body(self):
        for l in range(self.nl):
            self.ops.kv_append(self.k_new[l], self.kc[l], self.pos)
            self.ops.kv_append(self.v_new[l], self.vc[l], self.pos)
            self.attention.decode_attention(self.q[l], self.kc[l], self.vc[l], kv_len=self.len1,
                                            max_kv_len=self.cap, out=self.out[l])
        self.pos += 1
        self.len1 += 1
        self.steps_done += 1

    @property
    def bytes_per_step(self):
        # K/V read at the mean context of the timed steps + appended rows (bf16 in, blocks out) + q/out
        ctx = self.T0 + self.steps_done + 1      # the step attends over the appended token too
        B, H, D, Hq = self.B, self.HKV, self.D, self.HQ
        per_layer = B * ctx * self._per_tok + 2 * B * H * D * 2 + 2 * B * H * (D // 32) * 18 + 2 * B * Hq * D * 2
        return per_layer * self.nl

    @property
    def job_bytes(self):
        return self.bytes_per_step * self.BATCH // self.B

    def step(self):
        self.graph.replay()
        self.steps_done += 1

    def remaining(self):
        return self.GROWTH - self.steps_done

    def e2e_setup(self):
        self.hk = self.k_new.cpu().pin_memory()
        self.hv = self.v_new.cpu().pin_memory()
        self.hq = self.q.cpu().pin_memory()
        self.hout = self.out.cpu().pin_memory()

    def e2e_step(self):
        import torch
        self.k_new.copy_(self.hk, non_blocking=True)
        self.v_new.copy_(self.hv, non_blocking=True)
        self.q.copy_(self.hq, non_blocking=True)
        self.step()
        self.hout.copy_(self.out, non_blocking=True)
        torch.cuda.current_stream().synchronize()

    def e2e_bytes(self):
        return (self.hk.numel() + self.hv.numel() + self.hq.numel()) * 2, self.hout.numel() * 2



def make_workload(name, rank, tokens, ws=1, layers=None, transport="nccl", page_size=0, page_order="shuffled"):
    if name in ("attn", "c4"):
        return Attn(name, rank, ws, tokens, transport, page_size, page_order)
    if name == "c5":
        return Stream(rank, ws, tokens, layers)
    return Codec(name, rank, tokens)


# ── CPU baselines: one host-side sample per workload, used by both the cpu_baseline leg of
# this arm and the --impl reference arm, so the two report the same work ─────────────────

def cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


NOTE_ATT = ("float64 restatement (reference dequantize_row_tq*_0 + hadamard_transform + exact softmax); "
            "no reference CPU attention exists in-tree")


def _ref_cache(rng, O, qtype, hkv, ctx, d):
    """K or V of one sequence as the reference C writes it: N(0,1) with 4 outlier channels x20,
    hadamard_transform_row over head_dim, quantize_row_tq*_0; [1, hkv, ctx, d/32, block bytes]."""
    import numpy as np
    x = rng.standard_normal((hkv, ctx, d), dtype=np.float32)
    for h in range(hkv):
        x[h, :, rng.permutation(d)[:4]] *= 20.0
    bb = O.BLOCK_BYTES[qtype]
    return O.ref_quantize(qtype, O.ref_fwht(x, d)).reshape(1, hkv, ctx, d // 32, bb)


def cpu_sample(wl: str, nthreads: int):
    """(fn, bytes, kind, sample note) of a bounded host sample of workload `wl`: the inputs are made on
    the host by a seeded generator with the workload's shape and distribution, and fn() runs the
    reference's CPU path (or its C restatement where the reference has none) on `nthreads` threads."""
    import numpy as np
    import torch
    from oracle import oracle as O
    rng = np.random.default_rng(3)
    if wl in ("attn", "c4", "c5"):
        # one sequence (of one layer for C5); the C4 context is cut to 1/8 to keep a step bounded
        Hq, Hkv, D, T, kt = {"attn": (32, 8, 128, 32768, 4), "c4": (64, 8, 128, 131072 // 8, 3),
                             "c5": (32, 8, 256, 16384, 4)}[wl]
        kc, vc = _ref_cache(rng, O, kt, Hkv, T, D), _ref_cache(rng, O, 4, Hkv, T, D)
        q = rng.standard_normal((1, Hq, D), dtype=np.float32)
        nbytes = kc.size + vc.size + (q.size * 2 * 2 if wl != "c5" else 0)
        fn = lambda: O.decode_attention(q, kc, kt, vc, 4, Hkv, nthreads=nthreads)  # noqa: E731
        sample = {"attn": "1 of the 16 sequences per step; ",
                  "c4": "1 of the 64 sequences at 1/8 of the context per step; ",
                  "c5": "1 layer x 1 sequence of the decode step at context 16384, GB/s of cache read; "}[wl] + NOTE_ATT
        return fn, nbytes, "port", sample
    if wl == "tq3opt":
        tokens = 32768 // 16
        g = torch.Generator().manual_seed(2)
        # the workload's distribution: Student-t(4) = N / sqrt(chi2_4 / 4) x log-normal channel scales
        nrm = torch.randn(tokens, 8, 128, generator=g)
        chi = sum(torch.randn(tokens, 8, 128, generator=g) ** 2 for _ in range(4))
        x = (nrm / torch.sqrt(chi / 4.0)) * torch.exp(torch.randn(1, 8, 128, generator=g))
        arr = x.reshape(tokens, -1).to(torch.bfloat16).view(torch.int16).numpy().view("uint16")
        nbytes = arr.size * 2 + arr.size // 32 * 14
        fn = lambda: O.parallel_quantize(arr, 3, 128, nthreads, impl="port", opt_passes=2)  # noqa: E731
        return fn, nbytes, "port", (f"{tokens} of 32768 tokens per step; C restatement of "
                                    "scripts/tq3_rounding.py (no reference C exists) + reference hadamard_transform_row")
    tokens = 4096
    x = rng.standard_normal((tokens, 8, 128), dtype=np.float32)
    for h in range(8):
        x[:, h, rng.permutation(128)[:4]] *= 20.0
    arr = np.ascontiguousarray(x.reshape(tokens, -1))
    nbytes = 2 * (arr.size * 4 + arr.size // 32 * 18)
    fn = lambda: O.parallel_dequantize(O.parallel_quantize(arr, 4, 128, nthreads, impl="reference"),  # noqa: E731
                                       4, arr.shape[1], nthreads)
    return fn, nbytes, "reference", ("full [4096, 8, 128] per step; src/ggml-tq.c hadamard_transform_row + "
                                     "quantize_row_tq4_0 + dequantize_row_tq4_0")


def time_cpu_sample(wl: str, nthreads: int, warmup: int = 1, steps: int = 1):
    fn, nbytes, kind, sample = cpu_sample(wl, nthreads)
    for _ in range(warmup):
        fn()
    t0 = time.perf_counter()
    for _ in range(steps):
        fn()
    dt = (time.perf_counter() - t0) / steps
    return {"value": round(nbytes / dt / 1e9, 4), "unit": "GB/s", "cores": nthreads, "cpu_model": cpu_model(),
            "kind": kind, "sample": sample, "ms_per_sample": round(dt * 1e3, 3)}


def run_ours(args, ws, rank, local):
    import torch
    wl = make_workload(args.workload, rank, args.tokens, ws, args.layers, args.transport, args.page_size,
                       args.page_order)
    if isinstance(wl, Stream):
        budget = wl.remaining() - (0 if args.no_e2e else min(args.steps, 20) + 1)
        if args.warmup + args.steps > budget:
            raise SystemExit(f"c5: warmup + steps must stay within the {budget} free cache slots")
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device="cuda")
    flush_l2 = getattr(wl, "flush_l2", True)
    for _ in range(args.warmup):
        wl.step()
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    step_bytes = []
    barrier(ws)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        t0 = time.perf_counter()
        for i in range(args.steps):
            if flush_l2:
                flush.zero_()                  # evict inputs from L2 between steps
            step_bytes.append(wl.bytes_per_step)
            starts[i].record()
            wl.step()
            ends[i].record()
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
    barrier(ws)
    per = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    ms = statistics.mean(per)
    ms_max = max_over_ranks(ms, ws)
    rank_bytes = statistics.mean(step_bytes)
    job_bytes = getattr(wl, "job_bytes", None)
    job_bytes = job_bytes if job_bytes is not None else rank_bytes * ws
    value = job_bytes / (ms_max * 1e-3) / 1e9
    peak, peak_kind = hbm_peak()
    achieved = rank_bytes / (ms * 1e-3) / 1e9

    # e2e through the public API with host buffers
    e2e = None
    if not args.no_e2e:
        wl.e2e_setup()
        wl.e2e_step()
        n_e2e = min(args.steps, 20 if isinstance(wl, Stream) else 50)
        barrier(ws)
        t0 = time.perf_counter()
        for _ in range(n_e2e):
            wl.e2e_step()
        e2e_s = max_over_ranks((time.perf_counter() - t0) / n_e2e, ws)
        h2d, d2h = wl.e2e_bytes()
        e2e = {"value": round(job_bytes / e2e_s / 1e9, 3), "unit": "GB/s",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "path": getattr(wl, "e2e_path", "tq_quantize_host (C ABI, pinned host buffers)"),
               "steps": n_e2e}

    # a peer-transport step whose wait ran out leaves its output unmerged: check every rank's status
    # (it synchronizes) before any number is reported, and fail the line on an error
    peer_error = None
    if getattr(wl, "att", None) is not None and hasattr(wl.att, "status"):
        try:
            wl.att.status()
        except Exception as e:   # TQError
            peer_error = str(e)
    # every rank learns whether any rank failed, so all take the same exit path
    if max_over_ranks(1.0 if peer_error is not None else 0.0, ws) > 0 and peer_error is None:
        peer_error = "another rank's peer exchange wait ran out"

    out = None
    if rank == 0 and peer_error is None:
        cpu = None
        if ws == 1 and not args.no_cpu_baseline:
            cpu = time_cpu_sample(args.workload, os.cpu_count() or 1)
        is_codec = isinstance(wl, Codec)
        out = {
            "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_max, 6), "higher_is_better": True,
            "scaling": getattr(wl, "scaling", "weak"),
            "vs_baseline": None, "dtype": wl.dtype,
            "data": "synthetic (seeded)",
            "config": {**wl.config,
                       "parallelism": getattr(wl, "parallelism", f"token-row shards x{ws}, no collective"),
                       "l2": getattr(wl, "l2_note", "flushed (256 MiB write) between timed steps"),
                       # a peer transport whose setup failed on some rank: every rank ran NCCL instead
                       **({"transport_fallback": wl.att.fallback}
                          if getattr(getattr(wl, "att", None), "fallback", None) else {})},
            "us_per_step": round(ms_max * 1e3, 2),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                         "traffic": profile_traffic(args.workload),
                         "algorithmic_bytes_per_launch": int(rank_bytes / wl.launches_per_step) if is_codec else None,
                         "algorithmic_bytes_per_step_per_rank": int(rank_bytes),
                         "timed": ("the quantize and dequantize kernels" if getattr(wl, "round_trip", False) else "the kernel")
                                  if is_codec else "the whole step on the launching stream",
                         **({"limiter": wl.limiter} if getattr(wl, "limiter", None) else {})},
            "e2e": e2e,
            "gpu_launches": args.steps * wl.launches_per_step,
            "clocks": clk.summary(),
            "wall_s_timed_region": round(wall, 4),
            "cpu_baseline": cpu,
        }
    if getattr(wl, "att", None) is not None and hasattr(wl.att, "close"):
        wl.att.close()   # peer exchange buffers (collective; a no-op for the NCCL transport)
    if peer_error is not None:
        raise SystemExit(f"peer exchange failed during the timed or e2e steps: {peer_error}")
    return out


def run_reference(args, ws, rank):
    """The reference's CPU implementation of the path on this host's cores, on a bounded sample of
    the same workload (same config, metric and unit as this repository's arm; the same host sample
    as this arm's cpu_baseline leg; nothing of this repository's GPU path involved)."""
    if rank != 0:
        return None
    n = os.cpu_count() or 1
    wl = args.workload
    fn, nbytes, kind, sample = cpu_sample(wl, n)
    config = {"workload": WORKLOAD[wl]}
    if wl in ("attn", "c4", "c5"):
        config["shape"] = {"attn": "B=16 Hq=32 Hkv=8 D=128 ctx=32768, fp16 q/out",
                           "c4": "B=64 Hq=64 Hkv=8 D=128 ctx=131072, fp16 q/out",
                           "c5": "batch 32 (x1 ranks: 32 each) Hkv=8 Hq=32 D=256 prefill 16384 + up to 256 "
                                 "appended tokens, bf16 inputs/outputs"}[wl]
    else:
        config["input"] = INPUT[wl]
    config["parallelism"] = f"{n} host threads"
    scaling = "weak" if wl in ("tq3opt", "tq4") else "strong"
    for _ in range(args.warmup):
        fn()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        fn()
    dt = (time.perf_counter() - t0) / args.steps
    v = nbytes / dt / 1e9
    return {"metric": METRIC, "value": round(v, 4), "unit": "GB/s", "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 4), "higher_is_better": True, "scaling": scaling,
            "vs_baseline": None,
            "dtype": {"tq3opt": "bf16->u8", "tq4": "f32->u8->f32"}.get(wl, "f64"),
            "data": "synthetic (seeded)", "impl": "reference", "config": config,
            "cpu_baseline": {"value": round(v, 4), "unit": "GB/s", "cores": n, "cpu_model": cpu_model(),
                             "kind": kind, "sample": sample},
            "e2e": {"value": round(v, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=None)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["tq3opt", "tq4", "attn", "c4", "c5"], default="c4")
    ap.add_argument("--layers", type=int, default=None, help="c5: override the layer count (profiling runs)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-API measurement (profiling runs)")
    ap.add_argument("--tokens", type=int, default=None, help="override the token count (profiling runs)")
    ap.add_argument("--transport", choices=["peer", "peer_merge", "nccl"], default=None,
                    help="c4 on N > 1 GPUs: rank exchange fused into the attention over NVLink peer memory (peer, "
                         "the default; its parity and timeout tests ran on 2, 4 and 8 B200s), a separate peer "
                         "push + merge kernel (peer_merge) or NCCL all_gather + merge kernel (nccl)")
    ap.add_argument("--page-size", type=int, default=0,
                    help="attn / c4 on one GPU: run the paged decode attention over the same cache stored as "
                         "pages of this many tokens (a power of two, >= 16)")
    ap.add_argument("--page-order", choices=["shuffled", "sequential"], default="shuffled",
                    help="with --page-size: pool pages in a random order, or in sequence order (a fresh pool)")
    args = ap.parse_args()
    if args.steps is None:
        args.steps = 3 if args.impl == "reference" else {"attn": 200, "c4": 50, "c5": Stream.DECODE_STEPS}.get(
            args.workload, 2000)
    if args.warmup is None:
        args.warmup = 3 if args.impl == "reference" else {"c4": 5, "c5": 5}.get(args.workload, 20)
    args.warmup = max(args.warmup, 3)
    if args.transport is None:
        args.transport = "peer"

    if args.impl == "reference":
        ws = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        out = run_reference(args, ws, rank)
        if out is not None:
            print(json.dumps(out), flush=True)
        return

    ws, rank, local = dist_setup()
    out = run_ours(args, ws, rank, local)
    if out is not None:
        print(json.dumps(out), flush=True)
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
