#!/usr/bin/env python
"""Benchmark of byteprof's decode hot path on B200: the skinny bf16 linear sweep.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N ...

One step = one pass of the sweep: for each OLMo-2-1B linear shape (N, K) in {2048x2048, 8192x2048,
2048x8192, 100352x2048} and each M in {1, 2, 4, 8, 16}, one skinny_mm call y[M, N] = x[M, K] . W^T
(bf16 weights ~ N(0, 0.02), x ~ N(0, 1), fp32 accumulation, bf16 output) on a fresh ring member.
Each shape has a ring of distinct weight buffers totalling >= 256 MiB (> 2x the 126 MB L2), so the
weights come from HBM on every call (cold L2). A step is replayed as a CUDA graph (as the reference's
tools/skinny_bench.py:45-71 times its ring).

`value` = algorithmic bytes (2NK + 2MK + 2MN per call) of all ranks / the max over ranks of the device
time of K steps. `e2e` = the same sweep through the public API (skinny_mm) with the activations copied
from pinned host memory and the outputs read back every step. `roofline` is for the dominant kernel
(the LM-head shape, ~84 % of the bytes). Multi-GPU: independent replicas (no collective on the data path).

--impl reference times the reference's own CPU path for the same sweep (F.linear on the host, as
byteprof's SkinnyLinear runs on a CPU tensor) with all host threads, on rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from datetime import timedelta
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

SHAPES = [(2048, 2048), (8192, 2048), (2048, 8192), (100352, 2048)]  # (N = out, K = in)
MS = (1, 2, 4, 8, 16)
RING_BYTES = 256 * 2**20
INT8_MS = (1, 4, 16)
SCAN_TS = (1, 8, 64, 256)
METRIC = "skinny-GEMM HBM GB/s (% of peak, cold L2) at M=1-16"
PEAK_FALLBACK_GBS = 6650.0


def alg_bytes(m: int, n: int, k: int, kind: str = "bf16") -> int:
    """Bytes one call must move: the weights once (int8: + the [N] scale; int4: packed codes + the
    [K/128, N] bf16 scale and fp16 zero), the activations and the output."""
    if kind == "bf16":
        w = 2 * n * k
    elif kind == "int8":
        w = n * k + 2 * n
    else:
        w = n * k // 2 + 4 * n * (k // 128)
    return w + 2 * m * k + 2 * m * n


# ---- distributed plumbing -------------------------------------------------------------------------

def dist_env() -> tuple[int, int, int]:
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def init_dist(backend: str, timeout_s: float = 120.0) -> None:
    import torch.distributed as dist

    if dist.is_available() and not dist.is_initialized() and int(os.environ.get("WORLD_SIZE", 1)) > 1:
        dist.init_process_group(backend, timeout=timedelta(seconds=timeout_s))


def barrier() -> None:
    import torch.distributed as dist

    if dist.is_available() and dist.is_initialized():
        dist.barrier()


def max_over_ranks(x: float, device: torch.device | None = None) -> float:
    """The maximum of x over all ranks (x itself when not distributed)."""
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()):
        return x
    t = torch.tensor([x], dtype=torch.float64, device=device or "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---- clocks -----------------------------------------------------------------------------------------

class ClockSampler:
    """nvidia-smi samples of the SM clock and throttle reasons while the timed work runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.path = None

    def _gpu_id(self) -> str:
        try:
            p = torch.cuda.get_device_properties(self.device)
            return f"{p.pci_domain_id:08X}:{p.pci_bus_id:02X}:{p.pci_device_id:02X}.0"
        except Exception:  # noqa: BLE001
            vis = os.environ.get("CUDA_VISIBLE_DEVICES")
            return vis.split(",")[self.device] if vis else str(self.device)

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(prefix="bp_clocks_", suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "50",
                 "-i", self._gpu_id()], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        rows = []
        try:
            for line in Path(self.path).read_text().splitlines():
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9 and parts[1].replace(".", "").isdigit():
                    rows.append(parts)
        finally:
            if self.path:
                Path(self.path).unlink(missing_ok=True)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no nvidia-smi samples"], "samples": 0}
        sm = [float(r[1]) for r in rows]
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({nm for r in rows for nm, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": float(rows[0][2]), "reasons": reasons,
                "samples": len(rows), "power_w_max": max(float(r[3]) for r in rows if r[3].replace(".", "").isdigit())}


# ---- the workload -------------------------------------------------------------------------------------

class Sweep:
    """Weight rings, activations and outputs of the bf16 sweep on one device."""

    def __init__(self, device: torch.device, seed: int = 0):
        self.device = device
        self.rings, self.x, self.y = [], [], []
        for si, (n, k) in enumerate(SHAPES):
            ring = max(2, math.ceil(RING_BYTES / (2 * n * k)))
            g = torch.Generator(device=device).manual_seed(seed * 1000 + si)
            self.rings.append([(torch.randn(n, k, generator=g, device=device) * 0.02).to(torch.bfloat16)
                               for _ in range(ring)])
            self.x.append(torch.randn(max(MS), k, generator=g, device=device).to(torch.bfloat16))
            self.y.append(torch.empty(max(MS), n, device=device, dtype=torch.bfloat16))
        self.calls_per_step = len(SHAPES) * len(MS)
        self.bytes_per_step = sum(alg_bytes(m, n, k) for n, k in SHAPES for m in MS)
        # step s uses ring member (len(MS) * s + j) % ring for the j-th M of a shape
        self.period = math.lcm(*(len(r) // math.gcd(len(r), len(MS)) for r in self.rings))

    def step(self, s: int) -> None:
        from byteprof_b200.optim.skinny import skinny_mm

        for si, (n, k) in enumerate(SHAPES):
            ring = self.rings[si]
            for j, m in enumerate(MS):
                skinny_mm(self.x[si][:m], ring[(len(MS) * s + j) % len(ring)], out=self.y[si][:m])


def capture(fn) -> torch.cuda.CUDAGraph:
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    torch.cuda.synchronize()
    return g


def time_graph_replays(g: torch.cuda.CUDAGraph, reps: int) -> float:
    """Device milliseconds of `reps` replays (CUDA events on the replay stream)."""
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    a.record()
    for _ in range(reps):
        g.replay()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b)


def cell_times(sweep: Sweep, peak: float, reps: int = 5) -> dict:
    """Per (shape, M): a graph of one call per ring member, replayed; us per call and GB/s."""
    from byteprof_b200.optim.skinny import skinny_mm

    cells = {}
    for si, (n, k) in enumerate(SHAPES):
        ring = sweep.rings[si]
        for m in MS:
            x, y = sweep.x[si][:m], sweep.y[si][:m]
            g = capture(lambda: [skinny_mm(x, w, out=y) for w in ring])
            time_graph_replays(g, 2)
            ms = time_graph_replays(g, reps)
            us = ms * 1e3 / (reps * len(ring))
            gbs = alg_bytes(m, n, k) / (us * 1e-6) / 1e9
            cells[f"{n}x{k}|M{m}"] = {"us": round(us, 3), "gbs": round(gbs, 1), "frac": round(gbs / peak, 4)}
            del g
    return cells


def int8_cells(device: torch.device, peak: float, reps: int = 5) -> dict:
    from byteprof_b200.optim.skinny import skinny_mm
    from byteprof_b200.quant.int8 import quantize_rowwise_int8

    out = {}
    for si, (n, k) in enumerate(SHAPES):
        ring_n = max(2, math.ceil(RING_BYTES / (n * k)))
        g0 = torch.Generator(device=device).manual_seed(77 + si)
        ring = [quantize_rowwise_int8((torch.randn(n, k, generator=g0, device=device) * 0.02).to(torch.bfloat16))
                for _ in range(ring_n)]
        x = torch.randn(max(INT8_MS), k, generator=g0, device=device).to(torch.bfloat16)
        y = torch.empty(max(INT8_MS), n, device=device, dtype=torch.bfloat16)
        for m in INT8_MS:
            g = capture(lambda: [skinny_mm(x[:m], q, s, out=y[:m]) for q, s in ring])
            time_graph_replays(g, 2)
            us = time_graph_replays(g, reps) * 1e3 / (reps * ring_n)
            gbs = alg_bytes(m, n, k, "int8") / (us * 1e-6) / 1e9
            out[f"{n}x{k}|M{m}"] = {"us": round(us, 3), "gbs": round(gbs, 1), "frac": round(gbs / peak, 4)}
            del g
        del ring
    torch.cuda.empty_cache()
    return out


def int4_cells(device: torch.device, peak: float, reps: int = 5) -> dict:
    """The int4 group-128 weight kind (tile-major format) on the same shapes."""
    from byteprof_b200.optim.skinny import quantize_int4, skinny_mm

    out = {}
    for si, (n, k) in enumerate(SHAPES):
        ring_n = max(2, math.ceil(RING_BYTES / (n * k // 2)))
        g0 = torch.Generator(device=device).manual_seed(99 + si)
        ring = [quantize_int4((torch.randn(n, k, generator=g0, device=device) * 0.02).to(torch.bfloat16))
                for _ in range(ring_n)]
        x = torch.randn(max(INT8_MS), k, generator=g0, device=device).to(torch.bfloat16)
        y = torch.empty(max(INT8_MS), n, device=device, dtype=torch.bfloat16)
        for m in INT8_MS:
            g = capture(lambda: [skinny_mm(x[:m], p, s, z, out=y[:m]) for p, s, z in ring])
            time_graph_replays(g, 2)
            us = time_graph_replays(g, reps) * 1e3 / (reps * ring_n)
            gbs = alg_bytes(m, n, k, "int4") / (us * 1e-6) / 1e9
            out[f"{n}x{k}|M{m}"] = {"us": round(us, 3), "gbs": round(gbs, 1), "frac": round(gbs / peak, 4)}
            del g
        del ring
    torch.cuda.empty_cache()
    return out


VERIFY_KS = (0, 1, 3, 7, 15, 32)


def verify_cells(device: torch.device, peak: float, reps: int = 20) -> dict:
    """The drafting verify round of a Bolmo-shaped local model (encoder + decoder mLSTM layer, LM head):
    one CUDA graph per K, S = K + 1 positions; device time per round and the weight bytes it streams."""
    from byteprof_b200.optim.bolmo_local import BolmoLocal

    m = BolmoLocal(device=device, seed=0)
    wbytes = sum(t.numel() * t.element_size() for layer in (m.enc, m.dec)
                 for t in (layer.w_qkvo, layer.w_if, layer.w_out, layer.w_gu, layer.w_down))
    wbytes += (m.w_in.numel() + m.lm_head.numel()) * 2
    m.capture(VERIFY_KS)
    g0 = torch.Generator(device=device).manual_seed(8)
    m.ids.copy_(torch.randint(0, m.vocab, (m.smax,), generator=g0, device=device))
    out = {}
    for k in VERIFY_KS:
        g = m.graphs[k + 1]
        time_graph_replays(g, 3)
        us = time_graph_replays(g, reps) * 1e3 / reps
        gbs = wbytes / (us * 1e-6) / 1e9
        out[f"K{k}"] = {"us": round(us, 2), "positions_per_s": round((k + 1) / (us * 1e-6), 1),
                        "weight_gbs": round(gbs, 1), "frac": round(gbs / peak, 4)}
    out["weight_bytes"] = wbytes
    del m
    torch.cuda.empty_cache()
    return out


DECODE_PROMPT, DECODE_NEW = 256, 512


def decode_cells(device: torch.device, peak: float, seed: int = 0, reps: int = 20) -> dict:
    """greedy decoding of the random-init Bolmo-1B-shaped byte model, batch 1. The
    prompt (256 uniform-random bytes) is fed byte by byte through the same loop; the 511 steps after it
    produce the remaining generated bytes and are timed on the wall clock (each step ends with its host
    synchronisation, so wall time is the loop's real rate). Per-piece device times come from replaying
    each CUDA graph alone afterwards."""
    from byteprof_b200.optim.bolmo_e2e import BolmoDecoder

    m = BolmoDecoder(device=device, seed=seed)
    m.capture()
    prompt = torch.randint(0, 256, (DECODE_PROMPT,), generator=torch.Generator().manual_seed(seed)).tolist()
    m.reset()
    tok, new_patch = 0, True
    for b in prompt:
        tok, new_patch = m.feed(b, new_patch)
    prompt_patches = m.patches
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(DECODE_NEW - 1):
        tok, new_patch = m.feed(tok, new_patch)
    wall = time.perf_counter() - t0
    gen_patches = m.patches - prompt_patches
    w = m.weights()
    local_bytes = sum(t.numel() * t.element_size() for k, t in w.items()
                      if not k.startswith("glob") and k != "embed") + 2 * m.d  # + the embedding row
    glob_bytes = sum(t.numel() * t.element_size() for k, t in w.items() if k.startswith("glob"))
    per = {}
    for name in ("enc0", "dec0", "glob"):
        g = m.graphs[name]
        time_graph_replays(g, 2)
        per[name] = round(time_graph_replays(g, reps) * 1e3 / reps, 2)
    steps = DECODE_NEW - 1
    streamed = local_bytes * steps + glob_bytes * gen_patches
    out = {
        "bytes_per_s": round(steps / wall, 1), "ms_per_byte": round(wall / steps * 1e3, 4),
        "generated": DECODE_NEW, "timed_steps": steps, "patches_in_timed_steps": gen_patches,
        "prompt_patches": prompt_patches, "device_us": per,
        "weight_bytes": {"local_per_byte": local_bytes, "global_per_patch": glob_bytes},
        "weight_gbs": round(streamed / wall / 1e9, 1), "frac": round(streamed / wall / 1e9 / peak, 4),
        "graphs_per_byte": "enc + dec, + glob on a patch start; one host sync per byte",
    }
    del m
    torch.cuda.empty_cache()
    return out


def scan_cells(device: torch.device, peak: float, reps: int = 20) -> dict:
    """NH=4, dk=dv=512, T positions from a zero state, h and the final state."""
    from byteprof_b200.optim.draft_core import mlstm_scan

    nh, d = 4, 512
    out = {}
    for t in SCAN_TS:
        g0 = torch.Generator(device=device).manual_seed(500 + t)
        q, k, v = ((torch.randn(t, nh, d, generator=g0, device=device) / d ** 0.5).to(torch.bfloat16) for _ in range(3))
        i = torch.randn(t, nh, 1, generator=g0, device=device)
        f = torch.randn(t, nh, 1, generator=g0, device=device) + 3.0
        st_in = (torch.zeros(1, nh, d, d, device=device), torch.zeros(1, nh, d, device=device),
                 torch.zeros(1, nh, 1, device=device))
        st_out = tuple(torch.empty_like(s) for s in st_in)
        h = torch.empty(t, nh, d, device=device, dtype=torch.bfloat16)
        g = capture(lambda: mlstm_scan(st_in, q, k, v, i, f, h, st_out, 1e-6))
        time_graph_replays(g, 3)
        us = time_graph_replays(g, reps) * 1e3 / reps
        # minimum traffic: state read + written once, plus q, k, v, i, f in and h out per position
        nbytes = 2 * (nh * d * d * 4 + nh * d * 4 + nh * 4) + t * (3 * nh * d * 2 + 2 * nh * 4 + nh * d * 2)
        out[f"T{t}"] = {"us": round(us, 2), "us_per_step": round(us / t, 4), "gbs": round(nbytes / (us * 1e-6) / 1e9, 1)}
        del g
    return out


def e2e_sweep(sweep: Sweep, steps: int) -> tuple[float, int, int]:
    """The sweep through the public API with pinned host activations in and outputs out every step.
    Returns (device ms for `steps` steps, h2d bytes / step, d2h bytes / step)."""
    from byteprof_b200.optim.skinny import skinny_mm

    xh = [x.cpu().pin_memory() for x in sweep.x]
    yh = [torch.empty(y.shape, dtype=y.dtype).pin_memory() for y in sweep.y]
    h2d = sum(2 * m * k for n, k in SHAPES for m in MS)
    d2h = sum(2 * m * n for n, k in SHAPES for m in MS)

    def one(s):
        for si, (n, k) in enumerate(SHAPES):
            ring = sweep.rings[si]
            for j, m in enumerate(MS):
                sweep.x[si][:m].copy_(xh[si][:m], non_blocking=True)
                skinny_mm(sweep.x[si][:m], ring[(len(MS) * s + j) % len(ring)], out=sweep.y[si][:m])
                yh[si][:m].copy_(sweep.y[si][:m], non_blocking=True)
        torch.cuda.current_stream().synchronize()  # the step's results are on the host

    for s in range(3):
        one(s)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    a.record()
    for s in range(steps):
        one(s)
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b), h2d, d2h


# ---- CPU path (reference arm and cpu_baseline) ------------------------------------------------------

def cpu_sweep(max_calls: int, min_seconds: float, max_seconds: float, threads: int) -> dict:
    """The reference's CPU path (F.linear on the host, bf16) over the sweep cells, one cell per call in
    sweep order (call c runs cell c mod 20). Stops after max_calls calls, or earlier once max_seconds
    have passed; runs at least until min_seconds have passed or max_calls is reached."""
    from oracle.cpu_path import linear_cpu

    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(0)
    ws = [(torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16) for n, k in SHAPES]
    xs = [torch.randn(max(MS), k, generator=g).to(torch.bfloat16) for n, k in SHAPES]
    cells = [(si, m) for si in range(len(SHAPES)) for m in MS]
    for si in range(len(SHAPES)):  # first-touch of the weights and the BLAS setup
        linear_cpu(xs[si][:1], ws[si])
    nbytes, calls, t0 = 0, 0, time.perf_counter()
    while calls < max_calls or time.perf_counter() - t0 < min_seconds:
        si, m = cells[calls % len(cells)]
        n, k = SHAPES[si]
        linear_cpu(xs[si][:m], ws[si])
        nbytes += alg_bytes(m, n, k)
        calls += 1
        if time.perf_counter() - t0 > max_seconds:
            break
    dt = time.perf_counter() - t0
    return {"value": round(nbytes / dt / 1e9, 3), "unit": "GB/s", "cores": threads, "calls": calls,
            "seconds": round(dt, 2)}


def run_reference(args) -> int:
    """Reference arm: rank 0 times the reference's CPU path; one step = one sweep cell (bounded sample)."""
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    cpu_sweep(max_calls=args.warmup, min_seconds=0.0, max_seconds=60.0, threads=threads)
    res = cpu_sweep(max_calls=args.steps, min_seconds=0.0, max_seconds=150.0, threads=threads)
    sample = (f"{res['calls']} of {args.steps} steps (one sweep cell = one F.linear call per step, cells in sweep "
              f"order) in {res['seconds']} s, torch bf16 on the host = byteprof SkinnyLinear's CPU branch")
    line = {"metric": METRIC, "value": res["value"], "unit": "GB/s", "impl": "reference", "n_gpus": args.gpus,
            "steps": res["calls"], "warmup": args.warmup,
            "ms_per_step": round(res["seconds"] * 1e3 / max(1, res["calls"]), 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "BASELINE configs[1]: bf16 skinny sweep M in {1,2,4,8,16} x OLMo-2-1B shapes",
                       "shapes": [f"{n}x{k}" for n, k in SHAPES], "ms": list(MS)},
            "cpu_baseline": {"kind": "port", "cores": threads, "value": res["value"], "unit": "GB/s", "sample": sample},
            "e2e": {"value": res["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ---- our arm ---------------------------------------------------------------------------------------

def measured_peak() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    except Exception:  # noqa: BLE001
        return PEAK_FALLBACK_GBS, "fallback"


def run_ours(args) -> int:
    rank, world, local = dist_env()
    if not torch.cuda.is_available():
        print(json.dumps({"error": "no CUDA device"}), flush=True)
        return 1
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    init_dist("nccl")
    from byteprof_b200 import _lib

    _lib.lib()
    peak, peak_kind = measured_peak()
    sweep = Sweep(device, seed=rank)
    graphs = [capture(lambda s=s: sweep.step(s)) for s in range(sweep.period)]
    for s in range(args.warmup):
        graphs[s % sweep.period].replay()
    torch.cuda.synchronize()

    with ClockSampler(local) as clk:
        barrier()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for s in range(args.steps):
            graphs[(args.warmup + s) % sweep.period].replay()
        b.record()
        torch.cuda.synchronize()
        barrier()
        ms_local = a.elapsed_time(b)
        cells = cell_times(sweep, peak) if not args.quick else {}
    ms_total = max_over_ranks(ms_local, device)
    del graphs
    value = world * sweep.bytes_per_step * args.steps / (ms_total * 1e-3) / 1e9

    e2e_steps = max(3, args.steps // 20)
    e2e_ms, h2d, d2h = e2e_sweep(sweep, e2e_steps)
    e2e_ms = max_over_ranks(e2e_ms, device)
    e2e_value = world * sweep.bytes_per_step * e2e_steps / (e2e_ms * 1e-3) / 1e9

    extras = {}
    if not args.quick:
        extras["int8"] = int8_cells(device, peak)
        extras["int4"] = int4_cells(device, peak)
        extras["scan"] = scan_cells(device, peak)
        extras["verify"] = verify_cells(device, peak)
        extras["decode"] = decode_cells(device, peak, seed=rank)

    if rank == 0:
        # dominant kernel = the sweep cell with the largest device time per step
        if cells:
            dom_key = max(cells, key=lambda key: cells[key]["us"])
            n_, k_ = (int(v) for v in dom_key.split("|")[0].split("x"))
            m_ = int(dom_key.split("|M")[1])
            achieved = alg_bytes(m_, n_, k_) / (cells[dom_key]["us"] * 1e-6) / 1e9
        else:
            dom_key, achieved = "sweep", value / world
        traffic = _traffic_from_profiles(dom_key)
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_total / args.steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "BASELINE configs[1]: bf16 skinny sweep M in {1,2,4,8,16} x OLMo-2-1B shapes",
                       "shapes": [f"{n}x{k}" for n, k in SHAPES], "ms": list(MS),
                       "parallelism": f"replicas x{world}", "l2": "cold: per-shape weight ring >= 256 MiB (> 2x L2)",
                       "weights": "N(0, 0.02) bf16, x ~ N(0, 1)", "timing": "CUDA graph per step, CUDA events"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": traffic, "peak_kind": peak_kind,
                         "kernel": f"skinny_mm cell {dom_key} (largest time share)"},
            "frac_of_peak": round(value / world / peak, 4),
            "mean_cell_frac": round(statistics.mean(c["frac"] for c in cells.values()), 4) if cells else None,
            "cells": cells,
            "e2e": {"value": round(e2e_value, 1), "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "steps": e2e_steps, "api": "byteprof_b200.optim.skinny.skinny_mm, eager, pinned host x in / y out"},
            "gpu_launches": sweep.calls_per_step * args.steps,
            "clocks": clk.summary(),
            **extras,
        }
        if not args.quick:
            line["cpu_baseline"] = _cpu_baseline()
        print(json.dumps(line), flush=True)
    import torch.distributed as dist

    if dist.is_available() and dist.is_initialized():
        dist.destroy_process_group()
    return 0


def _traffic_from_profiles(cell: str):
    """DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum) of `cell` from a committed
    ncu summary under profiles/ (lines `cell: <N>x<K>|M<m>` and `dram_bytes_per_launch: <bytes>`)."""
    for p in sorted((ROOT / "profiles").glob("*.md")):
        cell_line = traffic = None
        for line in p.read_text().splitlines():
            if line.startswith("cell:"):
                cell_line = line.split(":", 1)[1].strip()
            elif line.startswith("dram_bytes_per_launch:"):
                traffic = int(line.split(":", 1)[1].strip())
        if cell_line == cell and traffic is not None:
            return traffic
    return None


def _cpu_baseline() -> dict:
    threads = os.cpu_count() or 1
    res = cpu_sweep(max_calls=20, min_seconds=10.0, max_seconds=30.0, threads=threads)
    return {"value": res["value"], "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{res['calls']} F.linear calls over the 20 sweep cells in sweep order ({res['seconds']} s), "
                      "torch bf16 on the host = byteprof SkinnyLinear's CPU branch"}


def run_case(args) -> int:
    """One sweep cell alone (for ncu captures): `--case N,K,M[,bf16|int8|int4]`; W eager warm-up calls, then K
    timed calls over a weight ring > 2x L2. Prints a JSON line with us per call and GB/s."""
    from byteprof_b200.optim.skinny import quantize_int4, skinny_mm
    from byteprof_b200.quant.int8 import quantize_rowwise_int8

    parts = args.case.split(",")
    n, k, m = (int(v) for v in parts[:3])
    kind = parts[3] if len(parts) > 3 else "bf16"
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(0)
    wbytes = 2 * n * k if kind == "bf16" else (n * k if kind == "int8" else n * k // 2)
    ring = []
    for _ in range(max(2, math.ceil(RING_BYTES / wbytes))):
        w = (torch.randn(n, k, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        ring.append((w,) if kind == "bf16" else quantize_rowwise_int8(w) if kind == "int8" else quantize_int4(w))
    x = torch.randn(m, k, generator=g, device=dev).to(torch.bfloat16)
    y = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
    for i in range(args.warmup):
        skinny_mm(x, *ring[i % len(ring)], out=y)
    torch.cuda.synchronize()
    if args.graph:  # one graph of a call per ring member, replayed: device time per call without host gaps
        gr = capture(lambda: [skinny_mm(x, *wq, out=y) for wq in ring])
        reps = max(1, args.steps // len(ring))
        time_graph_replays(gr, 2)
        us = time_graph_replays(gr, reps) * 1e3 / (reps * len(ring))
        nb = alg_bytes(m, n, k, kind)
        print(json.dumps({"case": f"{n}x{k}|M{m}|{kind}", "us": round(us, 3), "gbs": round(nb / (us * 1e-6) / 1e9, 1),
                          "bytes": nb, "graph": True, "pdl": os.environ.get("BP_DISABLE_PDL") != "1"}), flush=True)
        return 0
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for i in range(args.steps):
        skinny_mm(x, *ring[(args.warmup + i) % len(ring)], out=y)
    b.record()
    torch.cuda.synchronize()
    us = a.elapsed_time(b) * 1e3 / args.steps
    nb = alg_bytes(m, n, k, kind)
    print(json.dumps({"case": f"{n}x{k}|M{m}|{kind}", "us": round(us, 3), "gbs": round(nb / (us * 1e-6) / 1e9, 1),
                      "bytes": nb, "launches": args.warmup + args.steps}), flush=True)
    return 0


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--quick", action="store_true", help="skip the per-cell, int8, scan and CPU passes")
    ap.add_argument("--case", default=None, help="N,K,M[,bf16|int8|int4]: time one sweep cell alone (ncu captures)")
    ap.add_argument("--graph", action="store_true", help="with --case: time a CUDA graph of the weight ring")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.impl == "reference":
        return run_reference(args)
    if args.case:
        return run_case(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
