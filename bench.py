#!/usr/bin/env python3
"""Benchmark of the TurboQuant KV-cache hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]

Workloads (synthetic, seeded; shapes and distributions of the LeanKV configs):
  tq3opt  (default) TQ3_0 + optimal rounding (2 CD passes + LS scale), FWHT fused,
          bf16 [32768 tokens, 8 KV heads, 128]: Student-t(4) x per-channel log-normal scales
  tq4     TQ4_0 quantize (FWHT fused) + dequantize of fp32 [4096, 8, 128], N(0,1) with
          4 outlier channels per head x20
  attn    fused TQ4/TQ4 decode attention, B16 Hq32 Hkv8 D128 ctx 32768 (see leankv_b200.attention)

A step is one launch of the hot path over one batch that is resident in HBM.
`value` is whole-job throughput (all ranks); `e2e` is the same metric through the
C-ABI host-pointer API (pinned host buffers, H2D + D2H inside the timed region).
One process per GPU (torchrun for N > 1); the codec shards by token rows with
no collective ("weak" scaling).
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
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
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
            self.config = {"workload": "TQ3_0 optimal-rounding quantize (2 CD passes + LS scale), FWHT fused",
                           "input": "bf16 [32768 tokens, 8 KV heads, 128], Student-t(4) x log-normal channel scales",
                           "blocks_per_step": self.x.numel() // 32}
        else:
            self.x = c1_input(1 + 1000 * rank, tokens=tokens or 4096)
            self.qtype, self.hd, self.passes = 4, 128, 0
            self.config = {"workload": "TQ4_0 quantize, FWHT fused (fp32 [4096, 8, 128], N(0,1) + 4 outlier ch x20)",
                           "blocks_per_step": self.x.numel() // 32}
        self.k = self.x.numel()
        bb = 14 if self.qtype == 3 else 18
        self.y = torch.empty(self.k // 32 * bb, dtype=torch.uint8, device="cuda")
        self.bytes_per_step = self.k * self.x.element_size() + self.k // 32 * bb
        self.ops = ops
        self.launches_per_step = 1
        self.dtype = "bf16->u8 (fp32/fp64 math)" if self.passes else "f32->u8"

    def step(self):
        self.ops.quantize(self.x, self.qtype, fwht_head_dim=self.hd, opt_passes=self.passes, out=self.y)

    # end-to-end through the C ABI with pinned host buffers
    def e2e_setup(self):
        import torch
        self.hx = self.x.cpu().pin_memory()
        self.hy = torch.empty(self.y.numel(), dtype=torch.uint8).pin_memory()

    def e2e_step(self):
        from leankv_b200 import _lib as L
        dt = {2: L.DTYPE_BF16, 4: L.DTYPE_F32}[self.x.element_size()]
        L.check(L.load().tq_quantize_host(self.qtype, C.c_void_p(self.hx.data_ptr()), dt,
                                          C.c_void_p(self.hy.data_ptr()), self.k, self.hd, self.passes))

    def e2e_bytes(self):
        return self.hx.numel() * self.hx.element_size(), self.hy.numel()

    # CPU baseline on a bounded sample of the same workload
    def cpu_run(self, frac_tokens: int, nthreads: int, impl: str):
        import numpy as np
        from oracle import oracle as O
        tokens = self.x.shape[0] // frac_tokens
        xs = self.x[:tokens].reshape(tokens, -1)
        if self.x.dtype == __import__("torch").bfloat16:
            arr = xs.view(__import__("torch").int16).cpu().numpy().view(np.uint16)
        else:
            arr = xs.cpu().numpy()
        t0 = time.perf_counter()
        O.parallel_quantize(arr, self.qtype, self.hd, nthreads, impl=impl, opt_passes=self.passes)
        dt = time.perf_counter() - t0
        sample_bytes = self.bytes_per_step / frac_tokens
        return sample_bytes / dt / 1e9, tokens


class Attn:
    """Fused TQ4/TQ4 decode attention, B16 Hq32 Hkv8 D128 ctx 32768 (3 launches per step)."""

    def __init__(self, rank, tokens=None):
        import torch
        from leankv_b200 import attention, ops
        self.attention = attention
        B, Hq, Hkv, D = 16, 32, 8, 128
        T = tokens or 32768
        g = torch.Generator(device="cuda").manual_seed(3 + 1000 * rank)
        kc = torch.empty(B, Hkv, T, D // 32, 18, dtype=torch.uint8, device="cuda")
        vc = torch.empty_like(kc)
        for cache in (kc, vc):          # N(0,1) rows, 4 outlier channels per head x20, rotated + quantized
            for b in range(B):
                x = torch.randn(Hkv, T, D, generator=g, device="cuda")
                for h in range(Hkv):
                    ch = torch.randperm(D, generator=g, device="cuda")[:4]
                    x[h, :, ch] *= 20.0
                ops.quantize(x, 4, fwht_head_dim=D, out=cache[b])
        self.kc, self.vc = kc, vc
        self.q = torch.randn(B, Hq, D, generator=g, device="cuda").half()
        self.out = torch.empty(B, Hq, D, dtype=torch.float16, device="cuda")
        kv_bytes = kc.numel() + vc.numel()
        self.bytes_per_step = kv_bytes + self.q.numel() * 2 + self.out.numel() * 2
        self.launches_per_step = 3
        self.config = {"workload": "fused TQ4_0/TQ4_0 decode attention (FWHT(q), split-KV, LSE combine, FWHT(o))",
                       "shape": f"B={B} Hq={Hq} Hkv={Hkv} D={D} ctx={T}, fp16 q/out",
                       "kv_bytes": kv_bytes}
        self.dtype = "TQ4 blocks -> f16 MMA, f32 accumulate"

    def step(self):
        self.attention.decode_attention(self.q, self.kc, self.vc, out=self.out)

    def e2e_setup(self):
        self.hq = self.q.cpu().pin_memory()
        self.hout = self.out.cpu().pin_memory()

    def e2e_step(self):
        import torch
        self.q.copy_(self.hq, non_blocking=True)
        self.attention.decode_attention(self.q, self.kc, self.vc, out=self.out)
        self.hout.copy_(self.out, non_blocking=True)
        torch.cuda.current_stream().synchronize()

    def e2e_bytes(self):
        return self.hq.numel() * 2, self.hout.numel() * 2

    def cpu_run(self, frac, nthreads, impl):
        from oracle import oracle as O
        n = max(1, self.q.shape[0] // frac)
        q = self.q[:n].float().cpu().numpy()
        kc, vc = self.kc[:n].cpu().numpy(), self.vc[:n].cpu().numpy()
        t0 = time.perf_counter()
        O.decode_attention(q, kc, 4, vc, 4, self.kc.shape[1], nthreads=nthreads)
        dt = time.perf_counter() - t0
        return self.bytes_per_step * n / self.q.shape[0] / dt / 1e9, n


def make_workload(name, rank, tokens):
    if name == "attn":
        return Attn(rank, tokens)
    return Codec(name, rank, tokens)


def run_ours(args, ws, rank, local):
    import torch
    wl = make_workload(args.workload, rank, args.tokens)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device="cuda")
    flush_l2 = args.workload != "attn"     # the attention step streams 604 MB (> L2) by itself
    for _ in range(args.warmup):
        wl.step()
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    barrier(ws)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        t0 = time.perf_counter()
        for i in range(args.steps):
            if flush_l2:
                flush.zero_()                  # evict inputs from L2 between steps
            starts[i].record()
            wl.step()
            ends[i].record()
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
    barrier(ws)
    per = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    ms = statistics.mean(per)
    ms_max = max_over_ranks(ms, ws)
    value = wl.bytes_per_step * ws / (ms_max * 1e-3) / 1e9
    peak, peak_kind = hbm_peak()
    achieved = wl.bytes_per_step / (ms * 1e-3) / 1e9

    # e2e through the C ABI (host buffers)
    e2e = None
    if not args.no_e2e:
        wl.e2e_setup()
        wl.e2e_step()
        n_e2e = min(args.steps, 50)
        barrier(ws)
        t0 = time.perf_counter()
        for _ in range(n_e2e):
            wl.e2e_step()
        e2e_s = max_over_ranks((time.perf_counter() - t0) / n_e2e, ws)
        h2d, d2h = wl.e2e_bytes()
        e2e = {"value": round(wl.bytes_per_step * ws / e2e_s / 1e9, 3), "unit": "GB/s",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "path": ("leankv_b200.attention.decode_attention, q H2D and out D2H from pinned host memory"
                        if isinstance(wl, Attn) else "tq_quantize_host (C ABI, pinned host buffers)"),
               "steps": n_e2e}

    out = None
    if rank == 0:
        cpu = None
        if ws == 1 and not args.no_cpu_baseline:
            n = os.cpu_count() or 1
            if isinstance(wl, Attn):
                v, nseq = wl.cpu_run(16, n, "port")
                cpu = {"value": round(v, 4), "unit": "GB/s", "cores": n, "kind": "port",
                       "sample": f"{nseq} of {wl.q.shape[0]} sequences (1/16 of the step), {n} threads; float64 "
                                 "restatement: reference dequantize_row_tq4_0 + hadamard_transform + exact softmax"}
            else:
                impl = "port" if wl.passes else "reference"
                v, tokens = wl.cpu_run(16, n, impl)
                cpu = {"value": round(v, 4), "unit": "GB/s", "cores": n,
                       "kind": "port" if wl.passes else "reference",
                       "sample": f"{tokens} of {wl.x.shape[0]} tokens (1/16 of the workload), {n} threads; "
                                 + ("C restatement of scripts/tq3_rounding.py + reference hadamard_transform_row"
                                    if wl.passes else "reference src/ggml-tq.c hadamard_transform_row + quantize_row")}
        out = {
            "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_max, 6), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": wl.dtype,
            "data": "synthetic (seeded)",
            "config": {**wl.config,
                       "parallelism": (f"{ws} independent replicas of the step (batch x KV-head shards), no collective"
                                       if isinstance(wl, Attn) else f"token-row shards x{ws}, no collective"),
                       "l2": ("inputs 604 MB > L2 (126 MB), no flush" if isinstance(wl, Attn)
                              else "flushed (256 MiB write) between timed steps")},
            "us_per_step": round(ms_max * 1e3, 2),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                         "traffic": profile_traffic(args.workload),
                         "algorithmic_bytes_per_launch": wl.bytes_per_step},
            "e2e": e2e,
            "gpu_launches": args.steps * wl.launches_per_step,
            "clocks": clk.summary(),
            "wall_s_timed_region": round(wall, 4),
            "cpu_baseline": cpu,
        }
    return out


def run_reference(args, ws, rank):
    """The reference's CPU implementation of the path on this host's cores."""
    if rank != 0:
        return None
    import torch
    from oracle import oracle as O
    n = os.cpu_count() or 1
    torch.manual_seed(0)
    if args.workload == "attn":
        import numpy as np
        Hq, Hkv, D, T = 32, 8, 128, 32768
        rng = np.random.default_rng(3)
        x = rng.standard_normal((2, Hkv, T, D), dtype=np.float32)
        x[:, :, :, :4] *= 20.0
        blocks = O.ref_quantize(4, O.ref_fwht(x, D)).reshape(2, 1, Hkv, T, D // 32, 18)
        kc, vc = blocks[0], blocks[1]
        q = rng.standard_normal((1, Hq, D), dtype=np.float32)
        bytes_ = kc.size + vc.size + q.size * 4
        fn = lambda: O.decode_attention(q, kc, 4, vc, 4, Hkv, nthreads=n)  # noqa: E731
        kind, sample = "port", ("1 of the 16 sequences of B16 Hq32 Hkv8 D128 ctx 32768 per step; float64 restatement "
                                "(reference dequantize_row_tq4_0 + hadamard_transform + exact softmax), no reference "
                                "CPU attention exists in-tree")
    elif args.workload == "tq3opt":
        tokens = 32768 // 16
        x = torch.randn(tokens, 8 * 128) * torch.exp(torch.randn(1, 8 * 128))
        arr = x.to(torch.bfloat16).view(torch.int16).numpy().view("uint16")
        bytes_ = arr.size * 2 + arr.size // 32 * 14
        fn = lambda: O.parallel_quantize(arr, 3, 128, n, impl="port", opt_passes=2)  # noqa: E731
        kind, sample = "port", f"{tokens} of 32768 tokens per step (bf16 [.., 8, 128]); C restatement of " \
                               "scripts/tq3_rounding.py (no reference C exists) + reference hadamard_transform_row"
    else:
        tokens = 4096
        arr = torch.randn(tokens, 8 * 128).numpy()
        bytes_ = arr.size * 4 + arr.size // 32 * 18
        fn = lambda: O.parallel_quantize(arr, 4, 128, n, impl="reference")  # noqa: E731
        kind, sample = "reference", "full [4096, 8, 128] per step; src/ggml-tq.c hadamard_transform_row + quantize_row_tq4_0"
    for _ in range(args.warmup):
        fn()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        fn()
    dt = (time.perf_counter() - t0) / args.steps
    v = bytes_ / dt / 1e9
    return {"metric": METRIC, "value": round(v, 4), "unit": "GB/s", "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None,
            "dtype": {"tq3opt": "bf16->u8", "tq4": "f32->u8", "attn": "f64"}[args.workload],
            "data": "synthetic (seeded)", "impl": "reference",
            "config": {"workload": args.workload, "parallelism": "host threads"},
            "cpu_baseline": {"value": round(v, 4), "unit": "GB/s", "cores": n, "kind": kind, "sample": sample},
            "e2e": {"value": round(v, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=None)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["tq3opt", "tq4", "attn"], default="tq3opt")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-API measurement (profiling runs)")
    ap.add_argument("--tokens", type=int, default=None, help="override the token count (profiling runs)")
    args = ap.parse_args()
    if args.steps is None:
        args.steps = 3 if args.impl == "reference" else (200 if args.workload == "attn" else 2000)
    if args.warmup is None:
        args.warmup = 3 if args.impl == "reference" else 20
    args.warmup = max(args.warmup, 3)

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
