"""Benchmark of the quantized-matvec hot path (benchmark config C2) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

Workload (benchmark config C2): Q4_1 weights (32-element blocks, f16
scale d ~ U(0.002, 0.02) and min m = -8 d, 4-bit codes uniform), x bf16
~ N(0, 1), batches 1, 8 and 64 over the four shapes 4096x4096, 12288x4096,
4096x12288 and 151936x4096 (the lm-head). One step is the whole sweep: for
each batch, each shape, one `linear` (x prepared once, then the product).
Weights total 462 MB, 3.7x L2, visited in order, so no product finds its
weight in L2 from the previous visit (inputs larger than L2; no flush).

The line's metric is weight-streaming throughput: algorithmic bytes
(weights + x + y of every product) over the step time, in GB/s, also as a
fraction of the nominal 8 TB/s. `value` is device time with inputs resident
(the step replayed as a CUDA graph); `e2e` runs the same step through the
public C ABI with host buffers, copying each x in and each y out inside the
timed region. With N GPUs each rank runs its own sweep on its own weights
(weak scaling: the products shard by rows with no exchange); the time is the
max over ranks.

`--impl reference` times the reference's CPU path for the same products (the
C restatement of CpuOps.linear in oracle/, on every host thread) on a sample
of each matrix's rows, on rank 0 only.
"""

from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

SHAPES = [(4096, 4096), (12288, 4096), (4096, 12288), (151936, 4096)]
BATCHES = [1, 8, 64]
Q4_1, Q8_0 = 3, 8  # GGML type ids
METRIC = "quant matvec HBM GB/s (% of 8 TB/s); decode tok/s at 1/2/4/8 B200"
NOMINAL_HBM_GBS = 8000.0


def algorithmic_bytes(n: int, k: int, b: int) -> int:
    """Weights once, x (bf16) and y (f32) once: N (K/32) 20 + 2 b K + 4 b N."""
    return n * (k // 32) * 20 + 2 * b * k + 4 * b * n


def step_bytes() -> int:
    return sum(algorithmic_bytes(n, k, b) for b in BATCHES for n, k in SHAPES)


def measured_peaks() -> dict:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            data = json.load(f)
        return {"hbm_gbs": float(data["hbm_gbs"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


# ---- clocks ---------------------------------------------------------------------------------
class ClockSampler:
    """nvidia-smi clock and throttle samples (every 20 ms, each stamped on
    arrival) from before the timed region to after it; the summary keeps the
    samples inside the region, or the nearest ones when it is shorter than
    the sampling period."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.samples: list[tuple[float, list[str]]] = []
        self._proc = None
        self._thread = None
        self.window = (0.0, 0.0)

    def start(self):
        try:
            self._proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "20"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True, bufsize=1)
        except (FileNotFoundError, OSError):
            self._proc = None
            return
        self._thread = threading.Thread(target=self._read, daemon=True)
        self._thread.start()
        # let the first samples arrive before the timed region starts
        deadline = time.time() + 3.0
        while not self.samples and time.time() < deadline:
            time.sleep(0.02)

    def _read(self):
        for line in self._proc.stdout:
            self.samples.append((time.time(), [c.strip() for c in line.split(",")]))

    def mark(self, begin: float, end: float):
        self.window = (begin, end)

    def stop(self) -> dict:
        if self._proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.1)
        self._proc.terminate()
        try:
            self._proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self._proc.kill()
        if self._thread:
            self._thread.join(timeout=5)
        begin, end = self.window
        inside = [s for t, s in self.samples if begin - 0.025 <= t <= end + 0.025]
        if not inside and self.samples:
            middle = (begin + end) / 2
            inside = [min(self.samples, key=lambda ts: abs(ts[0] - middle))[1]]
        sm, sm_max, power, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for s in inside:
            try:
                sm.append(float(s[1]))
                sm_max.append(float(s[2]))
                power.append(float(s[3]))
            except (ValueError, IndexError):
                continue
            for name, value in zip(names, s[5:9]):
                if value.strip().lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(sm_max) if sm_max else None,
                "power_w_max": max(power) if power else None,
                "reasons": sorted(reasons), "samples": len(sm),
                "timed_region_s": round(end - begin, 4)}


# ---- the GPU arm ------------------------------------------------------------------------------
def run_gpu(args) -> dict | None:
    import torch
    import torch.distributed as dist

    from drift_b200 import synthetic
    from drift_b200._lib import check
    from drift_b200.ops import CudaOps, Stored

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                timeout=__import__("datetime").timedelta(seconds=120))
    ops = CudaOps(local)
    lib = ops.lib

    # inputs, resident: every rank its own weights (seeded by rank)
    rng = np.random.default_rng(1000 + rank)
    weights = {}
    for n, k in SHAPES:
        weights[(n, k)] = Stored.upload(Q4_1, (n, k), synthetic.quantized(rng, Q4_1, n, k))
    xs, ys = {}, {}
    host_x, host_y = {}, {}
    for b in BATCHES:
        for n, k in SHAPES:
            bits = synthetic.bf16_bits(synthetic.gaussian(rng, b, k))
            xs[(b, n, k)] = torch.from_numpy(bits.view(np.int16)).cuda().view(torch.bfloat16)
            ys[(b, n, k)] = torch.empty(b, n, device="cuda")
            host_x[(b, n, k)] = torch.from_numpy(bits.view(np.int16)).view(
                torch.bfloat16).pin_memory()
            host_y[(b, n, k)] = torch.empty(b, n, dtype=torch.float32).pin_memory()
    ops.reserve_workspace(max(BATCHES), max(k for _, k in SHAPES))

    def step():
        for b in BATCHES:
            for n, k in SHAPES:
                ops.linear(xs[(b, n, k)], weights[(n, k)], ys[(b, n, k)])

    stream = torch.cuda.Stream()
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        for _ in range(2):
            step()  # first calls resolve the library's lazy state outside capture
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph(keep_graph=True)
    with torch.cuda.graph(graph, stream=stream):
        step()
    launches_per_step = count_launches(graph)
    graph.instantiate()

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    wall_begin = time.time()
    start.record()
    for _ in range(args.steps):
        graph.replay()
    end.record()
    torch.cuda.synchronize()
    clocks.mark(wall_begin, time.time())
    clock_info = clocks.stop()
    elapsed_ms = start.elapsed_time(end)
    barrier()
    torch.cuda.synchronize()

    # e2e: the public C ABI with host buffers, copies inside the timed region.
    # As a host of the library pipelines a step: x in on one stream, the
    # product on a second, y out on a third, ordered per buffer by events (a
    # copy in waits for the last product that read its x buffer, a product
    # for its x and for the last copy out of its y buffer), so the copy
    # engines run while the products do. Every byte of every step is copied.
    def created(call, name):
        handle = ctypes.c_void_p()
        check(name, call(ctypes.byref(handle)))
        return handle

    def wait(stream, event):
        check("drift_stream_wait_event", lib.drift_stream_wait_event(stream, event))

    def record(event, stream):
        check("drift_event_record", lib.drift_event_record(event, stream))

    s_in, s_run, s_out = (created(lib.drift_stream_create, "drift_stream_create")
                          for _ in range(3))
    keys = [(b, n, k) for b in BATCHES for n, k in SHAPES]
    copied_in, computed, copied_out = (
        {key: created(lib.drift_event_create, "drift_event_create") for key in keys}
        for _ in range(3))

    def e2e_step():
        for key in keys:
            b, n, k = key
            hx, dx, y, hy = host_x[key], xs[key], ys[key], host_y[key]
            wait(s_in, computed[key])
            check("drift_memcpy_async", lib.drift_memcpy_async(
                ctypes.c_void_p(dx.data_ptr()), ctypes.c_void_p(hx.data_ptr()),
                hx.numel() * 2, 1, s_in))
            record(copied_in[key], s_in)
            wait(s_run, copied_in[key])
            wait(s_run, copied_out[key])
            w = weights[(n, k)]
            check("drift_linear", lib.drift_linear(
                30, ctypes.c_void_p(dx.data_ptr()), Q4_1, ctypes.c_void_p(w.data.data_ptr()),
                ctypes.c_void_p(y.data_ptr()), b, n, k, s_run))
            record(computed[key], s_run)
            wait(s_out, computed[key])
            check("drift_memcpy_async", lib.drift_memcpy_async(
                ctypes.c_void_p(hy.data_ptr()), ctypes.c_void_p(y.data_ptr()),
                hy.numel() * 4, 2, s_out))
            record(copied_out[key], s_out)

    for _ in range(max(1, args.warmup)):
        e2e_step()
    check("drift_device_synchronize", lib.drift_device_synchronize())
    barrier()
    torch.cuda.synchronize()
    e_start, e_end, drained = (created(lib.drift_event_create, "drift_event_create")
                               for _ in range(3))
    record(e_start, s_run)
    wait(s_in, e_start)
    wait(s_out, e_start)
    for _ in range(args.steps):
        e2e_step()
    record(drained, s_out)  # the last copy out (the products waited for every copy in)
    wait(s_run, drained)
    record(e_end, s_run)
    check("drift_device_synchronize", lib.drift_device_synchronize())
    e2e_elapsed = ctypes.c_float()
    check("drift_event_elapsed_time",
          lib.drift_event_elapsed_time(ctypes.byref(e2e_elapsed), e_start, e_end))
    e2e_ms = float(e2e_elapsed.value)
    for handle in [e_start, e_end, drained, *copied_in.values(), *computed.values(),
                   *copied_out.values()]:
        check("drift_event_destroy", lib.drift_event_destroy(handle))
    for handle in (s_in, s_run, s_out):
        check("drift_stream_destroy", lib.drift_stream_destroy(handle))
    h2d = sum(b * k * 2 for b in BATCHES for n, k in SHAPES)
    d2h = sum(b * n * 4 for b in BATCHES for n, k in SHAPES)

    # every product alone (rank 0), and the one with the largest share of the step
    sweep = sweep_table(ops, weights, xs, ys, stream) if rank == 0 else None
    dominant = dominant_kernel(sweep) if sweep else None
    del weights, xs, ys, host_x, host_y
    torch.cuda.empty_cache()
    # benchmark configs C1 (the Q8_0 product) and C3 (the layer ops), rank 0
    configs = (measure_c1_c3(ops, stream, args.cpu_baseline)
               if rank == 0 and args.decode else None)
    read_only = read_only_gbs(lib, stream) if rank == 0 else None

    # benchmark config C4: the dense decoder's decode step, tensor-parallel over the
    # job's GPUs (one NCCL group), tok/s at each batch
    decode = run_decode(args, ops, rank, world, stream) if args.decode else None
    # benchmark config C5: the hybrid MoE decoder, a replica per GPU
    hybrid = run_hybrid(args, ops, rank, world, stream) if args.decode else None

    times = torch.tensor([elapsed_ms, e2e_ms], device="cuda")
    if world > 1:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    elapsed_ms, e2e_ms = float(times[0]), float(times[1])
    del graph
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return None

    traffic, traffic_source = profiled_traffic(dominant["batch"], dominant["shape"])
    total_bytes = step_bytes() * args.steps * world
    value = total_bytes / (elapsed_ms / 1e3) / 1e9
    e2e_value = total_bytes / (e2e_ms / 1e3) / 1e9
    peaks = measured_peaks()
    result = {
        "metric": METRIC,
        "value": round(value, 1),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(elapsed_ms / args.steps, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "q4_1 weights, bf16 x; int8 planes (dp4a, mma.sync s8) and f16 tcgen05 products, f32 out",
        "data": "synthetic (seeded; benchmark config C2 value laws)",
        "config": {
            "workload": "C2 Q4_1 matvec sweep: batches 1/8/64 x shapes 4096x4096, "
                        "12288x4096, 4096x12288, 151936x4096",
            "per_gpu_bytes_per_step": step_bytes(),
            "l2": "inputs larger than L2 (462 MB of weights visited in turn), no flush",
            "parallelism": f"replicas x{world} (weak scaling, no exchange)",
            "fraction_of_8TBs": round(value / world / NOMINAL_HBM_GBS, 4),
            "fraction_of_measured_hbm": round(value / world / peaks["hbm_gbs"], 4),
            "fraction_of_read_only_hbm": round(value / world / read_only, 4),
            # decode tok/s (C4 dense, tensor parallel over the job's GPUs; C5
            # hybrid MoE, expert + head parallel), whole job
            "decode_tok_s": decode_summary(decode, hybrid),
        },
        "e2e": {"value": round(e2e_value, 1), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "gpu_launches": launches_per_step * args.steps,
        "roofline": {
            "bound": "hbm",
            "kernel": f"{dominant['kernel']}, {dominant['shape']}, batch {dominant['batch']}",
            "step_share": round(dominant["share"], 4),
            "achieved": round(dominant["gbs"], 1),
            "peak": peaks["hbm_gbs"],
            "peak_source": peaks["source"] + " (MEASURED_PEAKS.json hbm_gbs, copy)",
            "unit": "GB/s",
            "frac": round(dominant["gbs"] / peaks["hbm_gbs"], 4),
            "read_only_peak": round(read_only, 1),
            "frac_of_read_only": round(dominant["gbs"] / read_only, 4),
            "traffic": traffic,
            "traffic_source": (f"{traffic_source} (ncu dram read + write, one launch)"
                               if traffic_source else None),
            "launch_us": round(dominant["us"], 3),
        },
        "clocks": clock_info,
        "sweep": sweep,
        "decode": decode,
        "decode_hybrid": hybrid,
        "c1_c3": configs,
    }
    if args.cpu_baseline:
        result["cpu_baseline"] = cpu_baseline(seconds=args.cpu_seconds)
    return result


DECODE_CONTEXT = 4096


def decode_summary(decode: dict | None, hybrid: dict | None) -> dict | None:
    """The decode lines' tok/s in one small dict: c4_b1, c4_b16, c5_b1, c5_b16."""
    if not decode and not hybrid:
        return None
    out = {}
    for tag, line in (("c4", decode), ("c5", hybrid)):
        for key, row in (line or {}).items():
            if key.startswith("b") and isinstance(row, dict) and "tok_s" in row:
                out[f"{tag}_{key}"] = row["tok_s"]
    return out


def run_decode(args, ops, rank: int, world: int, stream) -> dict:
    """Decode tok/s of benchmark config C4 (36 layers, hidden 4096, 32 q / 8 kv heads
    of 128, FFN 12288, vocabulary 151936; random-init Q4_1 weights, Q8_0
    embedding; F16 KV caches prefilled with N(0, 1) to 4095 positions): one
    step at position 4095 (4096 keys) captured as a CUDA graph, replayed,
    timed with CUDA events, the slowest rank's time."""
    import torch
    import torch.distributed as dist

    from drift_b200.decoder import DenseConfig, DenseDecoder, DenseWeights
    from drift_b200.tensor_parallel import max_over_ranks

    config = DenseConfig()
    group = dist.group.WORLD if world > 1 else None
    weights = DenseWeights.random(config, rank=rank, world=world)
    peaks = measured_peaks()
    out = {"config": "C4 dense decode, TP over the job's GPUs", "tp": world,
           "context": DECODE_CONTEXT, "weights": "random-init Q4_1 (C2 law), Q8_0 embedding",
           "kv_cache": "F16 paged (the reference's KvCache), prefilled N(0,1)",
           "exchange": (("NVLink peer memory, fused with add + RMSNorm" if args.decode_exchange ==
                         "peer" else "NCCL all-reduce") if world > 1 else None)}
    steps = max(5, min(args.steps, 30))
    for batch in args.decode_batches:
        decoder = DenseDecoder(ops, config, weights, batch, DECODE_CONTEXT, group=group,
                               exchange=args.decode_exchange)
        decoder.prefill_random(DECODE_CONTEXT - 1)
        decoder.capture([DECODE_CONTEXT - 1] * batch, stream)
        for _ in range(3):
            decoder.replay()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        with torch.cuda.stream(stream):
            for _ in range(steps):
                decoder.replay()
        end.record(stream)
        torch.cuda.synchronize()
        ms = max_over_ranks(start.elapsed_time(end) / steps, device="cuda")
        kv_bytes = (2 * config.layers * (config.kv_heads // world) * config.head_dim * 2
                    * DECODE_CONTEXT * batch)
        per_rank = weights.nbytes() + kv_bytes
        out[f"b{batch}"] = {
            "tok_s": round(batch / (ms / 1e3), 1),
            "ms_per_step": round(ms, 4),
            "bytes_per_step_per_gpu": per_rank,
            "fraction_of_measured_hbm": round(per_rank / (ms / 1e3) / 1e9 / peaks["hbm_gbs"], 4),
            "steps": steps,
        }
        decoder.release()
        del decoder
        torch.cuda.empty_cache()
    return out


def run_hybrid(args, ops, rank: int, world: int, stream) -> dict:
    """Decode tok/s of benchmark config C5 (48 layers, hidden 2048: 36 Gated
    DeltaNet layers of 16 heads of 128 and 12 gated full-attention layers of
    16 / 2 heads of 256, each with 512 experts, top-10, FFN 512, and a shared
    expert; random-init Q4_1 weights, F32 routers; DeltaNet states N(0, 0.02),
    F16 caches prefilled with N(0, 1) to 4095 positions): a step captured as a
    CUDA graph, replayed, timed with CUDA events, the slowest rank's time.
    With N GPUs the model is split over them (expert parallelism for the
    experts, DeltaNet and query heads and the lm-head by rank, the two
    exchanges of a layer over the NVLink peer exchange)."""
    import torch
    import torch.distributed as dist

    from drift_b200.hybrid import HybridConfig, HybridDecoder, HybridWeights
    from drift_b200.tensor_parallel import max_over_ranks

    config = HybridConfig()
    weights = HybridWeights.random(config, rank=rank, world=world)
    group = dist.group.WORLD if world > 1 else None
    peaks = measured_peaks()
    per_token = weights.bytes_per_token(config)
    out = {"config": "C5 hybrid MoE decode (Gated DeltaNet + gated attention + 512 experts)",
           "parallelism": (f"expert + head parallel x{world} (NVLink peer exchange)" if world > 1
                           else "one GPU"),
           "context": DECODE_CONTEXT, "weights": "random-init Q4_1 (C2 law), F32 routers",
           "weight_bytes_per_sequence_step_per_gpu": per_token}
    steps = max(5, min(args.steps, 30))
    for batch in args.decode_batches:
        decoder = HybridDecoder(ops, config, weights, batch, DECODE_CONTEXT, group=group)
        decoder.prefill_random(DECODE_CONTEXT - 1)
        decoder.positions.fill_(DECODE_CONTEXT - 1)
        decoder.capture(stream)
        for _ in range(3):
            decoder.replay()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        with torch.cuda.stream(stream):
            for _ in range(steps):
                decoder.replay()
        end.record(stream)
        torch.cuda.synchronize()
        ms = max_over_ranks(start.elapsed_time(end) / steps, device="cuda")
        out[f"b{batch}"] = {
            "tok_s": round(batch / (ms / 1e3), 1),
            "ms_per_step": round(ms, 4),
            "steps": steps,
            "fraction_of_measured_hbm_b1_bytes": round(per_token / (ms / 1e3) / 1e9 / peaks["hbm_gbs"], 4)
            if batch == 1 else None,
        }
        decoder.release()
        del decoder
        torch.cuda.empty_cache()
    del weights
    torch.cuda.empty_cache()
    return out


def measure_c1_c3(ops, stream, cpu: bool) -> dict:
    """C1: the Q8_0 4096 x 4096 product at batch 1 (F32 x; GPU, and the CPU
    oracle on one host thread). C3: the layer ops at batches 1, 8, 16 and 64
    -- RMSNorm of [b, 4096] (with the residual add), SwiGLU of [b, 12288],
    RoPE of q [b, 32, 128] and k [b, 8, 128] (theta 1e6, positions in 0..8191),
    the Q8_0 embedding gather from a 151936 x 4096 table -- each timed as a
    replayed graph of 20 calls, GB/s = the benchmark's algorithmic bytes
    (F32 here: the library's activations are F32) over the time."""
    import time

    import numpy as np
    import torch

    from drift_b200 import synthetic
    from drift_b200.ops import SILU, Rope, RowNorm, Stored

    out = {}
    g = torch.Generator(device="cuda")
    g.manual_seed(11)
    # C1
    n = k = 4096
    w = Stored(Q8_0, (n, k), synthetic.quantized_device(Q8_0, n, k, g))
    copies = rotation(w, 4 * L2_BYTES)
    x = torch.randn(1, k, generator=g, device="cuda")
    y = torch.empty(1, n, device="cuda")

    def c1():
        for c in copies:
            ops.linear(x, c, y)
    ms = timed_graph(c1, stream, 10) / len(copies)
    c1_bytes = n * (k // 32) * 34 + 4 * k + 4 * n
    out["c1"] = {"shape": "4096x4096 Q8_0, b=1", "us": round(ms * 1e3, 2),
                 "gbs": round(c1_bytes / (ms / 1e3) / 1e9, 1)}
    if cpu:
        import oracle
        rng = np.random.default_rng(0)
        wh = synthetic.quantized(rng, Q8_0, n, k)
        xh = rng.standard_normal((1, k)).astype(np.float32)
        start, runs = time.perf_counter(), 0
        while time.perf_counter() - start < 5.0:
            oracle.linear(Q8_0, xh, wh, n, k)
            runs += 1
        elapsed = time.perf_counter() - start
        out["c1"]["cpu_oracle_gbs_1_thread"] = round(c1_bytes * runs / elapsed / 1e9, 3)
    del copies, w
    # C3
    table = Stored(Q8_0, (151936, 4096), synthetic.quantized_device(Q8_0, 151936, 4096, g))
    hidden, ffn = 4096, 12288
    weight = 1 + 0.02 * torch.randn(hidden, generator=g, device="cuda")
    rope = Rope(1e6, 128)
    rows = []
    for b in (1, 8, 16, 64):
        xs = torch.randn(b, hidden, generator=g, device="cuda")
        ys = torch.randn(b, hidden, generator=g, device="cuda")
        normed = torch.empty_like(xs)
        gate = torch.randn(b, ffn, generator=g, device="cuda")
        up = torch.randn(b, ffn, generator=g, device="cuda")
        hid = torch.empty_like(gate)
        q = torch.randn(b, 32, 128, generator=g, device="cuda")
        kk = torch.randn(b, 8, 128, generator=g, device="cuda")
        qo, ko = torch.empty_like(q), torch.empty_like(kk)
        positions = torch.randint(0, 8192, (b,), generator=g, device="cuda", dtype=torch.int32)
        ids = torch.randint(0, 151936, (b,), generator=g, device="cuda", dtype=torch.int32)
        gathered = torch.empty(b, hidden, device="cuda")
        cases = {
            "add_rms_norm": (lambda: ops.add_rms_norm(xs, ys, RowNorm(weight, 1e-6, 0.0, normed)),
                             3 * b * hidden * 4 + hidden * 4),
            "swiglu": (lambda: ops.gated(SILU, gate, up, hid), 3 * b * ffn * 4),
            "rope_q_k": (lambda: (ops.rope(q, positions, rope, qo), ops.rope(kk, positions, rope, ko)),
                         2 * b * 40 * 128 * 4),
            "embedding_q8_0": (lambda: ops.embedding(table, ids, gathered),
                               b * 4352 + b * hidden * 4),
        }
        for name, (fn, nbytes) in cases.items():
            def repeat(fn=fn):
                for _ in range(20):
                    fn()
            ms = timed_graph(repeat, stream, 10) / 20
            rows.append({"op": name, "batch": b, "us": round(ms * 1e3, 2),
                         "gbs": round(nbytes / (ms / 1e3) / 1e9, 1)})
    out["c3"] = rows
    del table
    torch.cuda.empty_cache()
    return out


def profiled_traffic(batch: int, shape: str) -> tuple:
    """DRAM bytes (read + write) of one launch of the product's kernel from a
    committed ncu summary (a line `traffic_bytes b<batch> <shape>: <bytes>`
    in profiles/*.md), and the summary's name; (None, None) if none has it."""
    folder = os.path.join(ROOT, "profiles")
    key = f"traffic_bytes b{batch} {shape}:"
    for name in sorted(os.listdir(folder)) if os.path.isdir(folder) else []:
        try:
            for line in open(os.path.join(folder, name)):
                if line.startswith(key):
                    return int(line.split(":")[1]), f"profiles/{name}"
        except (OSError, ValueError):
            continue
    return None, None


def count_launches(graph) -> int:
    """Kernel nodes in the captured step: the launches one step makes (all of
    them the library's own; the step calls nothing else)."""
    from cuda.bindings import runtime

    handle = runtime.cudaGraph_t(init_value=graph.raw_cuda_graph())
    err, nodes, count = runtime.cudaGraphGetNodes(handle, 0)
    err, nodes, count = runtime.cudaGraphGetNodes(handle, count)
    if err != runtime.cudaError_t.cudaSuccess:
        raise RuntimeError(f"cudaGraphGetNodes: {err}")
    kernels = 0
    for node in nodes[:count]:
        err, kind = runtime.cudaGraphNodeGetType(node)
        kernels += kind == runtime.cudaGraphNodeType.cudaGraphNodeTypeKernel
    return kernels


def timed_graph(fn, stream, repeats: int) -> float:
    """Average ms of fn replayed as a CUDA graph `repeats` times."""
    import torch

    with torch.cuda.stream(stream):
        fn()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        fn()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(repeats):
        graph.replay()
    end.record()
    torch.cuda.synchronize()
    return start.elapsed_time(end) / repeats


L2_BYTES = 126 * 2 ** 20


def rotation(weight, minimum_bytes: int) -> list:
    """Copies of a weight at distinct addresses, enough that cycling through
    them streams `minimum_bytes`: a product never finds its weight in L2."""
    from drift_b200.ops import Stored

    count = max(1, -(-minimum_bytes // weight.data.numel()))
    return [weight] + [Stored(weight.dtype, weight.shape, weight.data.clone())
                       for _ in range(count - 1)]


def product_kernel(batch: int) -> str:
    """The kernel that carries a product of `batch` rows of x (drift_linear's
    dispatch): the tcgen05 product from 32 rows, the ring kernel's integer
    MMA mode for 3-31 (passes of 8), its dp4a mode for 1-2."""
    if batch >= 32:
        return "linear_tc_q4_1 (+ tc_prepare_x)"
    if batch >= 3:
        return "matvec_ring_q4_1_mma (+ quantize_x22_mma)"
    return "matvec_ring_q4_1_dp4a (+ quantize_x22_mma)"


def dominant_kernel(sweep: list) -> dict:
    """The product with the largest share of the step (the sweep times each
    product alone, its weight copies cycling 4x L2 apart): its time, share and
    achieved GB/s of algorithmic bytes."""
    total = sum(r["us"] for r in sweep)
    top = max(sweep, key=lambda r: r["us"])
    n, k = (int(v) for v in top["shape"].split("x"))
    return {"us": top["us"], "gbs": algorithmic_bytes(n, k, top["batch"]) / (top["us"] / 1e6) / 1e9,
            "share": top["us"] / total, "batch": top["batch"], "shape": top["shape"],
            "kernel": product_kernel(top["batch"])}


def read_only_gbs(lib, stream) -> float:
    """The read-only HBM ceiling: the library's read_sum_f32x4 (the reference's
    bandwidth probe, kernels/bandwidth.hip:5-20, launched by name as
    MemoryBandwidth does) over 4 GiB, ten passes, CUDA events."""
    import torch

    from drift_b200._lib import check

    n4 = (4 << 30) // 16
    data = torch.ones(n4 * 4, device="cuda")
    blocks = 148 * 16
    partials = torch.empty(blocks, device="cuda")
    function = ctypes.c_void_p()
    check("drift_module_get_function",
          lib.drift_module_get_function(ctypes.byref(function), None, b"read_sum_f32x4"))
    args = [ctypes.c_void_p(data.data_ptr()), ctypes.c_int64(n4), ctypes.c_void_p(partials.data_ptr())]
    slots = (ctypes.c_void_p * 3)(*[ctypes.cast(ctypes.pointer(a), ctypes.c_void_p) for a in args])
    handle = ctypes.c_void_p(stream.cuda_stream)

    def run():
        check("read_sum_f32x4", lib.drift_module_launch_kernel(function, blocks, 1, 1, 256, 1, 1, 0,
                                                               handle, slots, None))
    run()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(10):
        run()
    end.record(stream)
    torch.cuda.synchronize()
    assert abs(float(partials.double().sum()) - n4 * 4) < 1e-3 * n4 * 4, "read_sum_f32x4 sum"
    del data
    torch.cuda.empty_cache()
    return n4 * 16 * 10 / (start.elapsed_time(end) / 1e3) / 1e9


def sweep_table(ops, weights, xs, ys, stream) -> list:
    """Per (batch, shape): microseconds per product and GB/s, each product
    cycling through copies of its weight that stream 4x L2 between reuses."""
    rows = []
    for n, k in SHAPES:
        copies = rotation(weights[(n, k)], 4 * L2_BYTES)
        for b in BATCHES:
            def fn(b=b, n=n, k=k):
                for w in copies:
                    ops.linear(xs[(b, n, k)], w, ys[(b, n, k)])
            ms = timed_graph(fn, stream, 5 if b == 64 else 10) / len(copies)
            rows.append({"batch": b, "shape": f"{n}x{k}", "us": round(ms * 1e3, 2),
                         "gbs": round(algorithmic_bytes(n, k, b) / (ms / 1e3) / 1e9, 1)})
        del copies
    rows.sort(key=lambda r: (r["batch"], SHAPES.index(tuple(map(int, r["shape"].split("x"))))))
    return rows


# ---- CPU: the reference's path ---------------------------------------------------------------------
def cpu_sample(rng, rows_per_matrix: int):
    import oracle
    from drift_b200 import synthetic

    cases = []
    for n, k in SHAPES:
        rows = min(n, rows_per_matrix)
        w = synthetic.quantized(rng, Q4_1, rows, k)
        for b in BATCHES:
            x = synthetic.bf16_values(synthetic.bf16_bits(synthetic.gaussian(rng, b, k)))
            cases.append((w, x, rows, k, b))
    return cases, oracle


def cpu_baseline(seconds: float) -> dict:
    """The oracle (C restatement of CpuOps.linear, single thread) on a sample:
    the 4096x4096 Q4_1 product at batch 1, repeated for ~`seconds`."""
    import oracle
    from drift_b200 import synthetic

    rng = np.random.default_rng(7)
    n, k = 4096, 4096
    w = synthetic.quantized(rng, Q4_1, n, k)
    x = synthetic.bf16_values(synthetic.bf16_bits(synthetic.gaussian(rng, 1, k)))
    runs, start = 0, time.perf_counter()
    while True:
        oracle.linear(Q4_1, x, w, n, k)
        runs += 1
        if time.perf_counter() - start >= seconds:
            break
    elapsed = time.perf_counter() - start
    gbs = algorithmic_bytes(n, k, 1) * runs / elapsed / 1e9
    return {"value": round(gbs, 4), "unit": "GB/s", "cores": 1, "kind": "port",
            "sample": f"Q4_1 4096x4096 batch 1 x{runs} ({elapsed:.1f} s): C restatement of "
                      "CpuOps.linear (decode per row, Double sums), one thread"}


def run_reference(args) -> dict | None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    import oracle

    threads = oracle.max_threads()
    rng = np.random.default_rng(7)
    rows = 256  # rows sampled per matrix: a bounded share of the sweep
    cases, _ = cpu_sample(rng, rows)
    sample_bytes = sum(algorithmic_bytes(r, k, b) for _, _, r, k, b in cases)

    def step():
        for w, x, r, k, b in cases:
            oracle.linear_threads(Q4_1, x, w, r, k, threads)

    for _ in range(args.warmup):
        step()
    start = time.perf_counter()
    for _ in range(args.steps):
        step()
    elapsed = time.perf_counter() - start
    value = sample_bytes * args.steps / elapsed / 1e9
    sample = (f"{rows} rows of each C2 matrix at batches 1/8/64 per step "
              f"({sample_bytes / 1e6:.1f} MB): C restatement of CpuOps.linear on {threads} "
              "host threads (rows split between threads)")
    return {
        "impl": "reference",
        "metric": METRIC,
        "value": round(value, 4),
        "unit": "GB/s",
        "n_gpus": int(os.environ.get("WORLD_SIZE", "1")),
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(elapsed / args.steps * 1e3, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "q4_1 weights, f32 x (bf16 widened), f64 sums",
        "data": "synthetic (seeded; benchmark config C2 value laws)",
        "config": {"workload": "C2 Q4_1 matvec sweep (row sample), CPU reference path"},
        "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": threads,
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def run_case(spec: str, repeat: int, dtype: int = Q4_1) -> None:
    """`--case B,N,K`: one product, `repeat` times, nothing timed -- the small
    fixed workload the ncu captures run."""
    import torch

    from drift_b200 import synthetic
    from drift_b200.ops import CudaOps, Stored

    b, n, k = (int(v) for v in spec.split(","))
    ops = CudaOps(0)
    rng = np.random.default_rng(7)
    weight = Stored.upload(dtype, (n, k), synthetic.quantized(rng, dtype, n, k))
    bits = synthetic.bf16_bits(synthetic.gaussian(rng, b, k))
    x = torch.from_numpy(bits.view(np.int16)).cuda().view(torch.bfloat16)
    y = torch.empty(b, n, device="cuda")
    for _ in range(repeat):
        ops.linear(x, weight, y)
    torch.cuda.synchronize()
    print(f"case {b}x{n}x{k} dtype {dtype}: {repeat} products, y[0,:4] = {y[0, :4].tolist()}")


def run_hybrid_case(batch: int, layers: int, steps: int) -> None:
    """`--hybrid-case B`: eager decode steps of C5 (with `--decode-layers`
    layers), nothing timed -- the workload of a launch-list capture."""
    import torch

    from drift_b200.hybrid import HybridConfig, HybridDecoder, HybridWeights
    from drift_b200.ops import CudaOps

    torch.cuda.set_device(0)
    config = HybridConfig(layers=min(layers, HybridConfig.layers))
    decoder = HybridDecoder(CudaOps(), config, HybridWeights.random(config), batch,
                            DECODE_CONTEXT)
    decoder.prefill_random(DECODE_CONTEXT - 1)
    decoder.positions.fill_(DECODE_CONTEXT - 1)
    decoder.reserve()
    for _ in range(steps):
        decoder.step()
    torch.cuda.synchronize()
    print(f"hybrid case b{batch} x {config.layers} layers: {steps} steps")


def run_decode_groups(batch: int, layers: int, steps: int) -> None:
    """`--decode-groups B`: per rank, the device time of each op group of the
    C4 and C5 decode steps (`--decode-layers` layers, batch B): the step with
    a CUDA event after each group, captured as a CUDA graph (the events as
    record nodes, so no host launch time shows) and replayed `steps` times
    after two warm-up replays -- which group limits a tensor- or
    expert-parallel step. The event nodes stop each group's launches from
    overlapping the next group's (programmatic dependent launch), so the sum
    is above the plain step's time. An exchange's time on a rank includes its
    wait for the slowest rank. Runs under torchrun like the bench; rank 0
    prints one JSON line."""
    import datetime

    import torch
    import torch.distributed as dist

    from drift_b200.decoder import DenseConfig, DenseDecoder, DenseWeights
    from drift_b200.hybrid import HybridConfig, HybridDecoder, HybridWeights
    from drift_b200.ops import CudaOps

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                timeout=datetime.timedelta(seconds=120))
    group = dist.group.WORLD if world > 1 else None
    ops = CudaOps(local)
    result = {"batch": batch, "layers": layers, "ranks": world, "steps": steps,
              "unit": "us per step"}

    def profile(decoder) -> dict:
        stream = torch.cuda.Stream()
        with torch.cuda.stream(stream):
            decoder.step()  # lazy state resolved outside the capture
        torch.cuda.synchronize()
        decoder.marks = []
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            decoder.step()
        marks, decoder.marks = decoder.marks, None
        for _ in range(2):
            graph.replay()
        torch.cuda.synchronize()
        totals: dict = {}
        for _ in range(steps):
            if world > 1:
                dist.barrier()
            graph.replay()
            torch.cuda.synchronize()
            for (_, before), (name, after) in zip(marks, marks[1:]):
                totals[name] = totals.get(name, 0.0) + before.elapsed_time(after) * 1000
        del graph
        return {name: round(t / steps, 1) for name, t in totals.items()}

    dense = DenseConfig(layers=layers)
    decoder = DenseDecoder(ops, dense, DenseWeights.random(dense, rank=rank, world=world), batch,
                           DECODE_CONTEXT, group=group)
    decoder.prefill_random(DECODE_CONTEXT - 1)
    decoder.positions.fill_(DECODE_CONTEXT - 1)
    decoder.reserve()
    c4 = profile(decoder)
    decoder.release()
    del decoder
    torch.cuda.empty_cache()
    hybrid = HybridConfig(layers=layers)
    decoder = HybridDecoder(ops, hybrid, HybridWeights.random(hybrid, rank=rank, world=world),
                            batch, DECODE_CONTEXT, group=group)
    decoder.prefill_random(DECODE_CONTEXT - 1)
    decoder.positions.fill_(DECODE_CONTEXT - 1)
    decoder.reserve()
    c5 = profile(decoder)
    decoder.release()
    del decoder
    per_rank = [(c4, c5)]
    if world > 1:
        per_rank = [None] * world
        dist.all_gather_object(per_rank, (c4, c5))
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        result["c4"] = [p[0] for p in per_rank]
        result["c5"] = [p[1] for p in per_rank]
        print(json.dumps({"decode_groups": result}), flush=True)


def run_decode_case(batch: int, layers: int, steps: int) -> None:
    """`--decode-case B`: eager decode steps of C4 (with `--decode-layers`
    layers), nothing timed -- the workload of a launch-list capture."""
    import torch

    from drift_b200.decoder import DenseConfig, DenseDecoder, DenseWeights
    from drift_b200.ops import CudaOps

    config = DenseConfig(layers=layers)
    ops = CudaOps(0)
    decoder = DenseDecoder(ops, config, DenseWeights.random(config), batch, DECODE_CONTEXT)
    decoder.prefill_random(DECODE_CONTEXT - 1)
    positions = [DECODE_CONTEXT - 1] * batch
    decoder.positions.copy_(torch.tensor(positions, dtype=torch.int32))
    for _ in range(steps):
        decoder.step(positions)
    torch.cuda.synchronize()
    print(f"decode case: batch {batch}, {layers} layers, {steps} steps")


def main() -> int:
    parser = argparse.ArgumentParser()
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=100)
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--impl", default="drift_b200")
    parser.add_argument("--cpu-seconds", type=float, default=10.0)
    parser.add_argument("--no-cpu-baseline", dest="cpu_baseline", action="store_false")
    parser.add_argument("--no-decode", dest="decode", action="store_false",
                        help="skip the C4 decode tok/s measurement")
    parser.add_argument("--decode-batches", default="1,16")
    parser.add_argument("--decode-exchange", choices=("peer", "nccl"), default="peer",
                        help="tensor-parallel decode: the fused NVLink peer exchange, or NCCL")
    parser.add_argument("--decode-case", type=int, help="B: eager C4 decode steps (profiling)")
    parser.add_argument("--hybrid-case", type=int, help="B: eager C5 decode steps (profiling)")
    parser.add_argument("--decode-groups", type=int,
                        help="B: per-rank device time of each decode op group (profiling)")
    parser.add_argument("--decode-layers", type=int, default=36)
    parser.add_argument("--case", help="B,N,K: run one product --repeat times (profiling)")
    parser.add_argument("--case-dtype", type=int, default=Q4_1)
    parser.add_argument("--repeat", type=int, default=3)
    args = parser.parse_args()
    args.warmup = max(args.warmup, 3)
    args.decode_batches = [int(b) for b in str(args.decode_batches).split(",") if b]
    if args.decode_groups:
        run_decode_groups(args.decode_groups, args.decode_layers, args.repeat)
        return 0
    if args.decode_case:
        run_decode_case(args.decode_case, args.decode_layers, args.repeat)
        return 0
    if args.hybrid_case:
        run_hybrid_case(args.hybrid_case, args.decode_layers, args.repeat)
        return 0
    if args.case:
        run_case(args.case, args.repeat, args.case_dtype)
        return 0
    if args.impl == "reference":
        result = run_reference(args)
    else:
        result = run_gpu(args)
    if result is not None:
        print(json.dumps(result), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
