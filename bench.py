"""Benchmark of the B200 Q8_0 quantized linear (decode path, HBM-bound).

Workload (the shape sweep's decode rows): the four projection shapes of the shape
sweep -- fused QKV (2048->6144), O (2048->2048), fused gate+up (2048->12288) and
down (6144->2048) -- at M = 1, for 28 distinct layers of Q8_0 weights (the depth of
the 2B decoder).  One step = one pass over all 28 x 4 = 112 projections, i.e. the
Q8_0 linear work of one decode token.  The 1.62 GB of weights is 13x the 126 MB L2,
so no step reads weights from L2 that an earlier one left there.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Output: one JSON line (rank 0).  ``value`` = algorithmic bytes / device time
(N*K*34/32 + 4*M*K + 4*M*N per projection) summed over ranks, in TB/s.
``e2e`` = the same metric through the C ABI with the step's activations copied from
pinned host memory and its outputs read back every step.  ``--impl reference`` times
the candle-CPU restatement (oracle/, the reference's own algorithm) on host cores.
Multi-GPU: every rank runs its own replica of the workload (independent decode
streams, no collective on the data path), so scaling is weak.
"""
from __future__ import annotations

import argparse
import csv
import ctypes
import io
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

SHAPES = [("qkv", 2048, 6144), ("o", 2048, 2048), ("gate_up", 2048, 12288), ("down", 6144, 2048)]
# the sweep adds the real VoxCPM k/v projection (GQA: 2 x 128 of 2048)
SWEEP_SHAPES = SHAPES + [("kv", 2048, 256)]
LAYERS = 28
METRIC = "Q8_0 matmul achieved HBM TB/s (decode GEMV, M=1)"


def algorithmic_bytes(m: int, k: int, n: int) -> int:
    return n * k * 34 // 32 + 4 * m * k + 4 * m * n


def load_peaks() -> tuple[float, str]:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def profile_traffic(name: str):
    """Per-launch DRAM bytes recorded from an ncu capture in profiles/<name> (or None)."""
    p = os.path.join(ROOT, "profiles", name)
    try:
        with open(p) as f:
            for line in f:
                if line.startswith("traffic_bytes_per_launch:"):
                    return float(line.split(":", 1)[1].strip())
    except OSError:
        pass
    return None


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples for one GPU during the timed region."""

    FIELDS = ("pci.bus_id,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, pci_bus: int):
        self.pci_bus = pci_bus
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.15)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, smax, reasons = [], [], set()
        for row in csv.reader(io.StringIO(out)):
            if len(row) < 9:
                continue
            row = [c.strip() for c in row]
            try:
                bus = int(row[0].split(":")[1], 16)
            except (IndexError, ValueError):
                continue
            if bus != self.pci_bus:
                continue
            try:
                sm.append(float(row[1]))
                smax.append(float(row[2]))
            except ValueError:
                continue
            for name, val in zip(("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"),
                                 row[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# --------------------------------------------------------------------------- CPU legs
def cpu_run(threads: int, budget_s: float, layers: int = 2, min_steps: int = 1):
    """candle-CPU restatement timed on host cores over the same projection shapes (M=1).

    Returns (TB/s, projections timed, seconds, description)."""
    import oracle
    from talechime_b200 import synth

    oracle.build()
    rng = np.random.default_rng(0)
    ws = [[(synth.q8_0_blocks(rng, n, k), k, n) for (_, k, n) in SHAPES] for _ in range(layers)]
    xs = {k: rng.standard_normal((1, k), dtype=np.float32) for (_, k, _) in SHAPES}
    oracle.matmul(xs[2048], ws[0][1][0], 2048, threads=threads)  # warm-up
    t0 = time.perf_counter()
    done, nbytes, i = 0, 0, 0
    while True:
        layer = ws[(i // len(SHAPES)) % layers]
        w, k, n = layer[i % len(SHAPES)]
        oracle.matmul(xs[k], w, n, threads=threads)
        nbytes += algorithmic_bytes(1, k, n)
        done += 1
        i += 1
        el = time.perf_counter() - t0
        if el >= budget_s and done >= min_steps:
            break
    return nbytes / el / 1e12, done, el


def run_reference(args, rank: int, world: int) -> None:
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    # each step: one projection (cycling through the 4 shapes of 2 layers), bounded so
    # that --steps K finishes in minutes
    import oracle
    from talechime_b200 import synth

    oracle.build()
    rng = np.random.default_rng(0)
    layers = 2
    ws = [[(synth.q8_0_blocks(rng, n, k), k, n) for (_, k, n) in SHAPES] for _ in range(layers)]
    xs = {k: rng.standard_normal((1, k), dtype=np.float32) for (_, k, _) in SHAPES}
    seq = [ws[li][si] for li in range(layers) for si in range(len(SHAPES))]
    for i in range(args.warmup):
        w, k, n = seq[i % len(seq)]
        oracle.matmul(xs[k], w, n, threads=threads)
    nbytes = 0
    t0 = time.perf_counter()
    for i in range(args.steps):
        w, k, n = seq[i % len(seq)]
        oracle.matmul(xs[k], w, n, threads=threads)
        nbytes += algorithmic_bytes(1, k, n)
    el = time.perf_counter() - t0
    value = nbytes / el / 1e12
    sample = (f"{args.steps} projections (cycling qkv/o/gate_up/down of {layers} layers, M=1) "
              f"with the candle-CPU restatement (oracle/q8_0_oracle.c, scalar vec_dot order)")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": el * 1e3 / max(args.steps, 1),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8xint8->f32",
        "data": "synthetic", "config": config_block(world),
        "cpu_baseline": {"value": value, "unit": "TB/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "TB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def config_block(world: int) -> dict:
    return {"workload": "configs[1] decode rows: qkv 2048->6144, o 2048->2048, gate_up 2048->12288, "
                        "down 6144->2048 at M=1, x 28 layers (one decode token of Q8_0 linears)",
            "m": 1, "layers": LAYERS, "weight_bytes_per_step": sum(algorithmic_bytes(0, k, n) for _, k, n in SHAPES) * LAYERS,
            "l2": "inputs larger than L2: 1.62 GB of distinct weights per step (13x the 126 MB L2)",
            "parallelism": f"replicas x{world}"}


# --------------------------------------------------------------------------- GPU legs
def _device_weight(torch, gen, dev, n, k):
    """Random Q8_0 GGUF blocks generated on the device, uploaded through the C ABI."""
    from talechime_b200 import QMatMul

    nb = k // 32
    blocks = torch.empty((n, nb, 34), dtype=torch.uint8, device=dev)
    qs = torch.randint(-127, 128, (n, nb, 32), generator=gen, device=dev, dtype=torch.int8)
    d = (torch.randn((n, nb), generator=gen, device=dev).abs() * (0.02 / 127.0)).half()
    blocks[:, :, 2:] = qs.view(torch.uint8)
    blocks[:, :, :2] = d.view(torch.uint8).view(n, nb, 2)
    return QMatMul.from_gguf_blocks(blocks, n, k, device=dev)


L2_BYTES = 126 * 1024 * 1024


def shape_weights(torch, dev, gen, k, n, copies=None):
    """Weight copies for time_shape: by default enough that a rotation over them spans
    twice the L2, so every call reads its weights from HBM."""
    if copies is None:
        copies = max(3, -(-2 * L2_BYTES // (n * k * 34 // 32)))
    return [_device_weight(torch, gen, dev, n, k) for _ in range(copies)]


def time_shape(torch, L, dev, stream, gen, m, k, n, reps, mats=None):
    """Device time of one q8lin_forward_ws call (its quantize and matmul launches) for one
    shape: `reps` calls captured in a CUDA graph, so host enqueue time does not hide the
    kernels, each call on the next weight copy of `mats` (shape_weights)."""
    if mats is None:
        mats = shape_weights(torch, dev, gen, k, n)
    copies = len(mats)
    x = torch.randn((m, k), generator=gen, device=dev)
    y = torch.empty((m, n), device=dev)
    need = L.q8lin_workspace_size(mats[0].handle, m)
    ws = torch.empty(max(need, 256), dtype=torch.uint8, device=dev)
    sptr = ctypes.c_void_p(stream.cuda_stream)

    def run(i):
        st = L.q8lin_forward_ws(mats[i % copies].handle, ctypes.c_void_p(x.data_ptr()),
                                ctypes.c_void_p(y.data_ptr()), m, ctypes.c_void_p(ws.data_ptr()), need, sptr)
        if st:
            from talechime_b200 import _lib
            _lib.check(st)

    for i in range(3):
        run(i)
    torch.cuda.synchronize()
    calls = max(reps, copies)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(calls):
            run(i)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    replays = 5
    e0.record(stream)
    for _ in range(replays):
        graph.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / (replays * calls)
    del graph
    return ms


def run_case(args) -> None:
    import torch

    from talechime_b200 import _lib, build

    m, k, n = (int(v) for v in args.case.split(":"))
    build.build()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)
    gen = torch.Generator(device=dev)
    gen.manual_seed(7)
    ms = time_shape(torch, _lib.lib(), dev, stream, gen, m, k, n, max(args.steps, 1))
    ops = 2.0 * m * n * k
    byts = algorithmic_bytes(m, k, n)
    print(json.dumps({"case": {"m": m, "k": k, "n": n}, "us": ms * 1e3, "tflops": ops / ms / 1e9,
                      "gbs": byts / ms / 1e6, "note": "profiling case; not a bench line"}), flush=True)


def run_sweep(torch, L, dev, stream) -> list:
    """The shape sweep: M in {1,4,16,64,256,1024} x the four projection shapes and the
    real k/v shape (2048 -> 256); device time per call from CUDA-graph replays over weight
    copies spanning twice the L2, and the kernel path that served it."""
    from talechime_b200 import _lib

    gen = torch.Generator(device=dev)
    gen.manual_seed(99)
    out = []
    for name, k, n in SWEEP_SHAPES:
        mats = shape_weights(torch, dev, gen, k, n)
        for m in (1, 4, 16, 64, 256, 1024):
            ms = time_shape(torch, L, dev, stream, gen, m, k, n, 20, mats=mats)
            out.append({"shape": name, "m": m, "k": k, "n": n,
                        "path": _lib.PATH_NAMES.get(L.q8lin_dispatch_path(m, k, n), "?"), "us": round(ms * 1e3, 2),
                        "tb_s": round(algorithmic_bytes(m, k, n) / ms / 1e9, 3),
                        "tflop_s": round(2.0 * m * n * k / ms / 1e9, 1), "weight_copies": len(mats)})
        del mats
    return out


def run_prefill(torch, dist, L, dev, stream, mats, rank: int, world: int, m: int = 4096, reps: int = 3) -> dict:
    """The batched-prefill workload, 4 x 1024 tokens (M = 4096), through the Q8_0
    linears of the 28 layers (qkv, o, gate_up, down per layer; the M > 32 tensor-core
    path): one CUDA graph of the 112 calls, device time per pass (CUDA events), max over
    ranks (one independent replica per GPU).  Attention and the elementwise steps of a
    prefill are not part of the Q8_0 linear path and are not timed."""
    gen = torch.Generator(device=dev)
    gen.manual_seed(4096 + rank)
    xs = {k: torch.randn((m, k), generator=gen, device=dev) for k in sorted({q.k for q in mats})}
    ys = {n: torch.empty((m, n), device=dev) for n in sorted({q.n for q in mats})}
    need = max(L.q8lin_workspace_size(q.handle, m) for q in mats)
    ws = torch.empty(max(need, 256), dtype=torch.uint8, device=dev)
    sptr = ctypes.c_void_p(stream.cuda_stream)
    calls = [(q.handle, ctypes.c_void_p(xs[q.k].data_ptr()), ctypes.c_void_p(ys[q.n].data_ptr())) for q in mats]

    def one_pass():
        for h, xp, yp in calls:
            st = L.q8lin_forward_ws(h, xp, yp, m, ctypes.c_void_p(ws.data_ptr()), need, sptr)
            if st:
                from talechime_b200 import _lib
                _lib.check(st)

    one_pass()
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        one_pass()
    graph.replay()
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        graph.replay()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / reps
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    del graph
    flops = sum(2.0 * m * q.n * q.k for q in mats)
    return {"config": f"configs[3]: M = {m} (4 x 1024 tokens) through the Q8_0 linears of {len(mats) // 4} layers "
                      "(qkv 2048->6144, o 2048->2048, gate_up 2048->12288, down 6144->2048), one CUDA graph per pass",
            "ms_per_pass": ms, "tflops": flops / (ms * 1e-3) / 1e12 * world,
            "tokens_per_s_linears": world * m / (ms * 1e-3), "calls_per_pass": len(mats),
            "launches_per_pass": 2 * len(mats)}  # quantize + matmul; no K split at M = 4096


def run_tp_mlp(torch, dist, dev, rank: int, world: int, reps: int = 20) -> dict:
    """Config 4: the Q8_0 SwiGLU MLP at hidden 4096 / intermediate 14336 split over the
    `world` ranks through the C ABI (q8lin_mlp_tp_*: gate/up by output rows, down by input
    blocks, ncclAllReduce on torch's communicator; for one row also the fused down
    projection + NVLink sum).  Device time per forward with CUDA events on the launching
    stream, max over ranks; every rank runs the same launches and collectives.  Every rank
    also times the whole MLP on its own GPU (world 1), so each entry carries the speed-up
    and the strong-scaling efficiency against one GPU."""
    from talechime_b200.tp_mlp import SwiGLUMLP

    hidden, inter = 4096, 14336
    gen = torch.Generator(device=dev)
    gen.manual_seed(4242)  # identical full weights on every rank; each keeps its shards

    def blocks(n, k):
        nb = k // 32
        b = torch.empty((n, nb, 34), dtype=torch.uint8, device=dev)
        b[:, :, 2:] = torch.randint(-127, 128, (n, nb, 32), generator=gen, device=dev,
                                    dtype=torch.int8).view(torch.uint8)
        d = (torch.randn((n, nb), generator=gen, device=dev).abs() * (0.02 / 127.0)).half()
        b[:, :, :2] = d.view(torch.uint8).view(n, nb, 2)
        return b

    gate, up, down = blocks(inter, hidden), blocks(inter, hidden), blocks(hidden, inter)
    mlp = SwiGLUMLP.from_gguf_blocks(gate, up, down, hidden, inter, device=dev, rank=rank, world=world, max_m=256)
    single = mlp if world == 1 else SwiGLUMLP.from_gguf_blocks(gate, up, down, hidden, inter, device=dev, max_m=256)
    fused = (SwiGLUMLP.from_gguf_blocks(gate, up, down, hidden, inter, device=dev, rank=rank, world=world, max_m=1,
                                        fused_decode=True) if world > 1 else None)
    del gate, up, down
    torch.cuda.synchronize(dev)
    stream = torch.cuda.current_stream(dev)

    def time_forward(m_obj, x, n):
        for _ in range(3):
            m_obj.forward(x)
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(n):
            m_obj.forward(x)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        ms = e0.elapsed_time(e1) / n
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    weight_bytes = 3 * inter * hidden * 34 // 32
    out = {"config": f"SwiGLU MLP hidden {hidden} / intermediate {inter}, Q8_0, gate+up column-split, "
                     f"down row-split over {world} GPU(s), q8lin_mlp_tp_forward (ncclAllReduce)",
           "weight_bytes": weight_bytes, "world": world, "per_m": []}
    for m in (1, 16, 256):
        x = torch.randn((m, hidden), generator=gen, device=dev)
        n = reps if m < 256 else max(3, reps // 2)
        ms = time_forward(mlp, x, n)
        ms1 = ms if world == 1 else time_forward(single, x, n)
        out["per_m"].append({"m": m, "ms": ms, "ms_1gpu": ms1, "speedup": ms1 / ms, "efficiency": ms1 / ms / world,
                             "weight_tb_s": weight_bytes / (ms * 1e-3) / 1e12,
                             "tokens_per_s": m / (ms * 1e-3),
                             "tflops": 2.0 * 3 * inter * hidden * m / (ms * 1e-3) / 1e12})
    if fused is not None:
        x = torch.randn((1, hidden), generator=gen, device=dev)
        ms = time_forward(fused, x, reps)
        ms1 = out["per_m"][0]["ms_1gpu"]
        out["m1_fused_allreduce"] = {"m": 1, "ms": ms, "speedup": ms1 / ms, "efficiency": ms1 / ms / world,
                                     "weight_tb_s": weight_bytes / (ms * 1e-3) / 1e12,
                                     "path": "gate_up GEMV, then the down GEMV with SwiGLU in its activation "
                                             "quantization and the cross-GPU sum in its tail (peer stores over "
                                             "NVLink), Q8LIN_TP_FUSED_DECODE"}
        fused.close()
    if single is not mlp:
        single.close()
    mlp.close()
    torch.cuda.synchronize(dev)
    return out


def run_decoder(torch, dist, dev, rank: int, world: int, prefix: int = 128, steps: int = 512) -> dict:
    """Config 2: the ~2B Q8_0 decoder (hidden 2048, 28 layers, 16 x 128 heads, SwiGLU 6144,
    RMSNorm, RoPE, f32 KV cache, vocab 73448; talechime_b200/decoder.py), batch 1: a
    128-token random-id prefix run as one batched forward (Q8Decoder.prefill: device time
    from a CUDA graph of its launches, and the median wall time of 5 host-issued calls),
    then `steps` greedy decode steps replayed from one CUDA graph of a step; device
    time of the decode steps (CUDA events), max over ranks (one independent replica per
    GPU).  Both step implementations are timed: "fused" (one launch per operation, the
    default) and "persistent" (one cooperative launch per step)."""
    from talechime_b200.decoder import DecoderConfig, Q8Decoder, synthetic_weights

    cfg = DecoderConfig(max_t=prefix + steps)
    weights = synthetic_weights(cfg, seed=777, device=dev)
    dec = Q8Decoder(cfg, weights, device=dev)
    del weights
    torch.cuda.synchronize(dev)
    stream = torch.cuda.Stream(dev)
    gen = torch.Generator()
    gen.manual_seed(99)
    ids = torch.randint(0, cfg.vocab, (prefix,), generator=gen).tolist()
    wbytes = dec.weight_bytes_per_step()
    # KV cache read per step at position p: layers * 2 * kv_heads * (p + 1) * head_dim * 4
    kv_bytes = sum(cfg.layers * 2 * cfg.kv_heads * (p + 1) * cfg.head_dim * 4 for p in range(prefix, prefix + steps))
    results = {}
    with torch.cuda.stream(stream):
        dec.reset(ids[0])
        dec.prefill(ids)  # warm-up: workspace growth and kernel attributes
        torch.cuda.synchronize(dev)
        # as the user calls it (host-issued launches, one position read-back): median of 5
        host_ms = []
        for _ in range(5):
            dec.reset(ids[0])
            torch.cuda.synchronize(dev)
            t0 = time.perf_counter()
            dec.prefill(ids)
            torch.cuda.synchronize(dev)
            host_ms.append((time.perf_counter() - t0) * 1e3)
        # device time: the same launches captured once in a CUDA graph and replayed
        tok_d = torch.tensor(ids, dtype=torch.int32, device=dev)
        pgraph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(pgraph, stream=stream):
            dec._prefill_launches(tok_d, 1, prefix, 0)
        pgraph.replay()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(5):
            pgraph.replay()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        del pgraph
    prefill_ms = e0.elapsed_time(e1) / 5
    prefill_host_ms = statistics.median(host_ms)
    for mode in ("fused", "persistent"):
        with torch.cuda.stream(stream):
            dec.reset(ids[0])
            dec.step(mode)  # eager warm-up: workspaces and kernel attributes outside the capture
            dec.reset(ids[0])
            torch.cuda.synchronize(dev)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                dec.step(mode)
            dec.reset(ids[0])
            dec.prefill(ids)  # the prefix as one forward; the decode steps continue from it
            torch.cuda.synchronize(dev)
            if world > 1:
                dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(steps):
                graph.replay()
            e1.record(stream)
            torch.cuda.synchronize(dev)
        ms = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        results[mode] = (ms, int(dec.pos.item()))
        del graph
    ms, final_pos = results["fused"]
    msp, _ = results["persistent"]
    out = {"config": "Q8_0 decoder, hidden 2048, 28 layers, 16 x 128 heads (MHA), SwiGLU 6144, RMSNorm, RoPE, "
                     f"f32 KV cache, vocab 73448; batch 1, {prefix}-token random-id prefix (one batched forward), "
                     f"{steps} greedy steps",
           "prefix_prefill_ms": prefill_ms, "prefix_prefill_tokens_per_s": prefix / (prefill_ms * 1e-3),
           "prefix_prefill_host_issued_ms": prefill_host_ms,
           "tokens_per_s": world * steps / (ms * 1e-3), "ms_per_token": ms / steps,
           "tokens_per_s_persistent": world * steps / (msp * 1e-3), "ms_per_token_persistent": msp / steps,
           "weight_bytes_per_token": wbytes, "kv_bytes_per_token_avg": kv_bytes / steps,
           "hbm_tb_s": (wbytes * steps + kv_bytes) / (ms * 1e-3) / 1e12 * world,
           "launches_per_token": dec.launches_per_step("fused"), "launches_per_token_persistent": 1,
           "final_position": final_pos,
           "graph": "one CUDA graph of a decode step per mode, replayed per token"}
    del dec
    torch.cuda.synchronize(dev)
    return out


def run_decoder_prefill(torch, dist, dev, rank: int, world: int, batch: int = 4, tokens: int = 1024,
                        reps: int = 3) -> dict:
    """The batched-prefill workload as a decoder pass: the same ~2B Q8_0 decoder prefills `batch`
    sequences of `tokens` random ids (M = batch * tokens = 4096 rows through every
    linear) with everything of the prompt pass -- embedding, RMSNorms, RoPE + KV append,
    causal attention, residual adds, SwiGLU, final norm, LM head and greedy pick of each
    sequence's last row (Q8Decoder.prefill).  Device time per pass (CUDA events around the
    call, which starts by reading the position back), max over ranks (one independent
    replica per GPU)."""
    from talechime_b200.decoder import DecoderConfig, Q8Decoder, synthetic_weights

    cfg = DecoderConfig(max_t=tokens)
    weights = synthetic_weights(cfg, seed=4242 + rank, device=dev)
    dec = Q8Decoder(cfg, weights, device=dev, batch=batch)
    del weights
    gen = torch.Generator()
    gen.manual_seed(4243)
    ids = torch.randint(0, cfg.vocab, (batch, tokens), generator=gen)
    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        dec.reset()
        dec.prefill(ids)  # warm-up
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        times = []
        for _ in range(reps):
            dec.reset()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            dec.prefill(ids)
            e1.record(stream)
            torch.cuda.synchronize(dev)
            times.append(e0.elapsed_time(e1))
    ms = statistics.median(times)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    m = batch * tokens
    H = cfg.hidden
    per_layer = cfg.qkv_rows * H + H * cfg.heads * cfg.head_dim + 2 * cfg.inter * H + H * cfg.inter
    linear_flops = 2.0 * m * per_layer * cfg.layers + 2.0 * batch * cfg.vocab * H
    # causal attention: q.k and p.v over (pos + 1) keys for every row and head
    attn_flops = 4.0 * batch * cfg.heads * cfg.head_dim * cfg.layers * sum(p + 1 for p in range(tokens))
    del dec
    torch.cuda.synchronize(dev)
    return {"config": f"configs[3]: the decoder's prompt pass, batch {batch} x {tokens} random-id tokens (M = {m}): "
                      "embedding, per layer rms_norm, qkv, RoPE + KV append, causal attention, o + residual, "
                      "rms_norm, gate_up, SwiGLU, down + residual; final norm, LM head and argmax per sequence",
            "ms_per_pass": ms, "tokens_per_s": world * m / (ms * 1e-3),
            "tflops": (linear_flops + attn_flops) / (ms * 1e-3) / 1e12 * world,
            "linear_gflop": linear_flops / 1e9, "attention_gflop": attn_flops / 1e9}


def run_profile_prefill(args) -> None:
    """A short prompt pass for ncu captures: `--profile-prefill B:T` prefills B sequences
    of T random ids through a decoder of `--layers` layers (max_t = T), once as warm-up
    (launches to skip with ncu -s) and once timed."""
    import torch
    from talechime_b200 import build
    from talechime_b200.decoder import DecoderConfig, Q8Decoder, synthetic_weights

    build.build()
    b, t = (int(v) for v in args.profile_prefill.split(":"))
    dev = torch.device("cuda", 0)
    cfg = DecoderConfig(layers=args.layers, max_t=t)
    weights = synthetic_weights(cfg, seed=4242, device=dev)
    dec = Q8Decoder(cfg, weights, device=dev, batch=b)
    del weights
    ids = torch.randint(0, cfg.vocab, (b, t), generator=torch.Generator().manual_seed(5))
    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        dec.prefill(ids)
        torch.cuda.synchronize(dev)
        dec.reset()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        dec.prefill(ids)
        e1.record(stream)
        torch.cuda.synchronize(dev)
    print(json.dumps({"profile_prefill": {"batch": b, "tokens": t}, "layers": cfg.layers,
                      "ms": e0.elapsed_time(e1), "note": "profiling run; not a bench line"}), flush=True)


def run_profile_decoder(args) -> None:
    """A short decoder run for ncu captures: 4 eager steps (warm-up launches to skip with
    ncu -s), then 8 steps replayed from one CUDA graph, from position 380."""
    import torch
    from talechime_b200 import build
    from talechime_b200.decoder import DecoderConfig, Q8Decoder, synthetic_weights

    build.build()
    dev = torch.device("cuda", 0)
    cfg = DecoderConfig(layers=args.layers, max_t=640)
    weights = synthetic_weights(cfg, seed=777, device=dev)
    dec = Q8Decoder(cfg, weights, device=dev)
    del weights
    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        dec.reset(5)
        dec.pos.fill_(380)
        for _ in range(4):
            dec.step(args.profile_decoder)
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            dec.step(args.profile_decoder)
        dec.pos.fill_(380)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(8):
            graph.replay()
        e1.record(stream)
        torch.cuda.synchronize(dev)
    print(json.dumps({"profile_decoder": args.profile_decoder, "layers": cfg.layers,
                      "launches_per_step": dec.launches_per_step(args.profile_decoder),
                      "us_per_step": e0.elapsed_time(e1) * 1000 / 8}), flush=True)
    del graph


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-budget", type=float, default=10.0, help="seconds for the cpu_baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="skip the end-to-end leg (profiling runs)")
    ap.add_argument("--no-tp-mlp", action="store_true", help="skip the tensor-parallel MLP measurement")
    ap.add_argument("--no-decoder", action="store_true", help="skip the config-2 decoder tokens/s measurement")
    ap.add_argument("--no-prefill", action="store_true",
                    help="skip the config-3 prefill legs (M = 4096 linears, decoder prompt pass)")
    ap.add_argument("--layers", type=int, default=LAYERS,
                    help="layer copies (28 = the benchmark; fewer only for small profiling captures)")
    ap.add_argument("--case", default=None,
                    help="M:K:N -- run one projection shape `--steps` times (profiling), print its timing")
    ap.add_argument("--sweep", action="store_true",
                    help="also time the shape sweep (M x {qkv,o,gate_up,down}) into the line")
    ap.add_argument("--profile-prefill", default=None, metavar="B:T",
                    help="ncu helper: one warm-up and one timed prompt pass of B x T tokens (--layers layers)")
    ap.add_argument("--profile-decoder", default=None, choices=["fused", "persistent", "unfused"],
                    help="profiling run: only the decoder, `--layers` layers, 8 steps replayed from a graph "
                         "after 4 eager warm-up steps from position 380; prints its timing")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        run_reference(args, rank, world)
        return

    import torch
    import torch.distributed as dist

    if args.case:
        run_case(args)
        return
    if args.profile_decoder:
        run_profile_decoder(args)
        return
    if args.profile_prefill:
        run_profile_prefill(args)
        return

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))

    from talechime_b200 import QMatMul, _lib, build

    if rank == 0 or world == 1:
        build.build()
    if world > 1:
        dist.barrier()
    L = _lib.lib()

    # weights: 28 layers x 4 shapes, random Q8_0 blocks generated on the device
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234 + rank)
    mats = []
    for _ in range(args.layers):
        for name, k, n in SHAPES:
            nb = k // 32
            blocks = torch.empty((n, nb, 34), dtype=torch.uint8, device=dev)
            qs = torch.randint(-127, 128, (n, nb, 32), generator=gen, device=dev, dtype=torch.int8)
            d = (torch.randn((n, nb), generator=gen, device=dev).abs() * (0.02 / 127.0)).half()
            blocks[:, :, 2:] = qs.view(torch.uint8)
            blocks[:, :, :2] = d.view(torch.uint8).view(n, nb, 2)
            mats.append(QMatMul.from_gguf_blocks(blocks, n, k, device=dev))
            del blocks, qs, d
    torch.cuda.synchronize()
    xs = {k: torch.randn((1, k), generator=gen, device=dev) for _, k, _ in SHAPES}
    ys = [torch.empty((1, m.n), device=dev) for m in mats]
    # all timed work runs on one non-default stream (graph capture needs one)
    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)
    sptr = ctypes.c_void_p(stream.cuda_stream)
    handles = [m.handle for m in mats]
    xptr = [ctypes.c_void_p(xs[m.k].data_ptr()) for m in mats]
    yptr = [ctypes.c_void_p(y.data_ptr()) for y in ys]
    fwd = L.q8lin_forward

    def step():
        for h, xp, yp in zip(handles, xptr, yptr):
            st = fwd(h, xp, yp, 1, sptr)
            if st:
                _lib.check(st)

    bytes_per_step = sum(algorithmic_bytes(1, k, n) for _, k, n in SHAPES) * args.layers
    launches_per_step = len(mats)

    # Capture one step in a CUDA graph: the device-side timing then measures the
    # kernels back to back without host launch gaps (host cost is in e2e).
    graph = torch.cuda.CUDAGraph()
    for _ in range(2):
        step()
    torch.cuda.synchronize()
    with torch.cuda.graph(graph, stream=stream):
        step()
    torch.cuda.synchronize()

    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    props = torch.cuda.get_device_properties(dev)
    sampler = ClockSampler(props.pci_bus_id)
    sampler.start()
    time.sleep(0.3)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    ev0.record(stream)
    for _ in range(args.steps):
        graph.replay()
    ev1.record(stream)
    torch.cuda.synchronize()
    clocks = sampler.stop()
    ms = ev0.elapsed_time(ev1) / args.steps
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    value = world * bytes_per_step / (ms * 1e-3) / 1e12

    # ---- e2e: through the C ABI, activations from pinned host memory, outputs back
    if args.no_e2e:
        line = {"metric": METRIC, "value": value, "unit": "TB/s", "ms_per_step": ms, "layers": args.layers,
                "clocks": clocks, "note": "profiling run (--no-e2e); not a bench line"}
        if rank == 0:
            print(json.dumps(line), flush=True)
        del graph
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return
    xin = {k: torch.randn((1, k), generator=gen, device=dev).cpu().pin_memory() for _, k, _ in SHAPES}
    yhost = torch.empty(sum(y.numel() for y in ys), dtype=torch.float32).pin_memory()
    yall = torch.cat([y.reshape(-1) for y in ys])
    h2d = sum(v.numel() * 4 for v in xin.values())
    d2h = yhost.numel() * 4
    ycat_views = []
    off = 0
    for y in ys:
        ycat_views.append(yall[off:off + y.numel()])
        off += y.numel()
    yptr2 = [ctypes.c_void_p(v.data_ptr()) for v in ycat_views]

    def e2e_calls():
        for h, xp, yp in zip(handles, xptr, yptr2):
            st = fwd(h, xp, yp, 1, sptr)
            if st:
                _lib.check(st)

    # The step's public-API calls recorded once as a CUDA graph, as the reference's decode
    # loop records its step (crates/voxcpm/src/cuda_graph/replay.rs:46-80), then replayed
    # per step between the H2D copy of the step's inputs and the D2H copy of its outputs.
    e2e_calls()
    torch.cuda.synchronize()
    e2e_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(e2e_graph, stream=stream):
        e2e_calls()
    torch.cuda.synchronize()

    def e2e_step(graphed):
        for k, v in xin.items():
            xs[k].copy_(v, non_blocking=True)
        if graphed:
            e2e_graph.replay()
        else:
            e2e_calls()
        yhost.copy_(yall, non_blocking=True)
        stream.synchronize()

    def time_e2e(graphed):
        for _ in range(args.warmup):
            e2e_step(graphed)
        if world > 1:
            dist.barrier()
        steps = max(1, args.steps // 4)
        torch.cuda.synchronize()
        ev0.record(stream)
        for _ in range(steps):
            e2e_step(graphed)
        ev1.record(stream)
        torch.cuda.synchronize()
        t_ms = ev0.elapsed_time(ev1) / steps
        if world > 1:
            t = torch.tensor([t_ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            t_ms = float(t.item())
        return t_ms, steps

    serial_ms, _ = time_e2e(True)
    eager_ms, _ = time_e2e(False)
    del e2e_graph

    # Pipelined: two buffer sets, each with its own graph of the 112 calls, and one copy
    # stream per direction (a shared one would queue the next step's H2D behind this
    # step's D2H, which waits for this step's compute), so the H2D and D2H of one step
    # overlap the compute of the next; the host still waits for every step's outputs
    # (one step later).
    cs = torch.cuda.Stream(dev)   # H2D
    cs2 = torch.cuda.Stream(dev)  # D2H
    sets = []
    for si in range(2):
        xs_s = {k: torch.empty_like(v) for k, v in xs.items()}
        yall_s = torch.empty_like(yall)
        views, off = [], 0
        for y in ys:
            views.append(yall_s[off:off + y.numel()])
            off += y.numel()
        xp_s = [ctypes.c_void_p(xs_s[m.k].data_ptr()) for m in mats]
        yp_s = [ctypes.c_void_p(v.data_ptr()) for v in views]

        def calls(xp_s=xp_s, yp_s=yp_s):
            for h, xp, yp in zip(handles, xp_s, yp_s):
                st = fwd(h, xp, yp, 1, sptr)
                if st:
                    _lib.check(st)

        calls()
        torch.cuda.synchronize()
        g_s = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_s, stream=stream):
            calls()
        torch.cuda.synchronize()
        sets.append({"xs": xs_s, "yall": yall_s, "graph": g_s,
                     "yhost": torch.empty(yall.numel(), dtype=torch.float32).pin_memory()})
    ev_h2d = [torch.cuda.Event() for _ in range(2)]
    ev_cmp = [torch.cuda.Event() for _ in range(2)]
    ev_d2h = [torch.cuda.Event() for _ in range(2)]

    def pipelined(nsteps):
        for i in range(nsteps):
            b = i % 2
            st_ = sets[b]
            if i >= 2:
                cs.wait_event(ev_cmp[b])  # compute i - 2 is done with this set's inputs
            with torch.cuda.stream(cs):
                for k, v in xin.items():
                    st_["xs"][k].copy_(v, non_blocking=True)
            ev_h2d[b].record(cs)
            stream.wait_event(ev_h2d[b])
            if i >= 2:
                stream.wait_event(ev_d2h[b])  # step i - 2's outputs are out of this set
            st_["graph"].replay()
            ev_cmp[b].record(stream)
            cs2.wait_event(ev_cmp[b])
            with torch.cuda.stream(cs2):
                st_["yhost"].copy_(st_["yall"], non_blocking=True)
            ev_d2h[b].record(cs2)
            if i >= 1:
                ev_d2h[(i - 1) % 2].synchronize()  # the host has step i - 1's outputs
        ev_d2h[(nsteps - 1) % 2].synchronize()

    pipelined(args.warmup)
    if world > 1:
        dist.barrier()
    e2e_steps = max(1, args.steps // 4)
    torch.cuda.synchronize()
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p0.record(cs)
    pipelined(e2e_steps)
    cs2.wait_event(ev_d2h[(e2e_steps - 1) % 2])
    p1.record(cs2)
    torch.cuda.synchronize()
    e2e_ms = p0.elapsed_time(p1) / e2e_steps
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    del sets
    e2e_value = world * bytes_per_step / (e2e_ms * 1e-3) / 1e12

    peak, peak_kind = load_peaks()
    achieved_gbs = (bytes_per_step / launches_per_step) / (ms * 1e-3 / launches_per_step) / 1e9
    traffic = profile_traffic("gemv_q8_0_decode.txt")
    line = {
        "metric": METRIC, "value": value, "unit": "TB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8xint8->f32", "data": "synthetic",
        "config": config_block(world),
        "tokens_per_s_linears_only": world * 1e3 / ms,
        "roofline": {"bound": "hbm", "achieved": achieved_gbs, "peak": peak, "unit": "GB/s",
                     "frac": achieved_gbs / peak, "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)"
                     if peak_kind == "measured" else "fallback 6.65 TB/s",
                     "traffic": traffic, "kernel": "gemv_q8_0_stream_kernel",
                     "bytes_per_launch": bytes_per_step / launches_per_step},
        "e2e": {"value": e2e_value, "unit": "TB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": e2e_ms, "steps": e2e_steps,
                "path": "per step: pinned H2D of the step's x, the 112 q8lin_forward calls (C ABI via ctypes) "
                        "recorded once as a CUDA graph and replayed, D2H of every y into pinned memory, the host "
                        "waiting for each step's outputs; two buffer sets and a copy stream per direction overlap "
                        "one step's copies with the next step's compute",
                "serial": {"value": world * bytes_per_step / (serial_ms * 1e-3) / 1e12, "ms_per_step": serial_ms,
                           "path": "the same with one buffer set and a stream synchronize after every step"},
                "eager": {"value": world * bytes_per_step / (eager_ms * 1e-3) / 1e12, "ms_per_step": eager_ms,
                          "path": "serial, with the 112 q8lin_forward calls issued from the host every step"}},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clocks,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        v, done, el = cpu_run(threads, args.cpu_budget)
        v1, done1, el1 = cpu_run(1, args.cpu_budget / 2)
        line["cpu_baseline"] = {
            "value": v, "unit": "TB/s", "cores": threads, "kind": "port",
            "sample": f"{done} projections (qkv/o/gate_up/down of 2 layers, M=1) in {el:.1f} s with the "
                      f"candle-CPU restatement (oracle/q8_0_oracle.c)",
            "single_thread": {"value": v1, "unit": "TB/s", "cores": 1,
                              "sample": f"{done1} projections in {el1:.1f} s, one thread"}}
    if not args.no_tp_mlp:
        line["tp_mlp"] = run_tp_mlp(torch, dist, dev, rank, world)
    if not args.no_decoder:
        line["decoder"] = run_decoder(torch, dist, dev, rank, world)
    if not args.no_prefill:
        line["prefill"] = run_prefill(torch, dist, L, dev, stream, mats, rank, world)
        line["decoder_prefill"] = run_decoder_prefill(torch, dist, dev, rank, world)
    if args.sweep and rank == 0:
        line["sweep"] = run_sweep(torch, L, dev, stream)
    if rank == 0:
        print(json.dumps(line), flush=True)
    del graph
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
