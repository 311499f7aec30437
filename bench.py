"""Benchmark of the Q4 quantized-linear hot path on B200.

Default workload: the seven Q4_0 linears of one
Llama-2-7B layer (Q, K, V, O: 4096->4096; gate, up: 4096->11008; down:
11008->4096) at decode batch 1, 4 and 16 -- a "step" is one pass over all
3 x 7 GEMVs, issued the way the engine issues them (QKV as one multi call,
O, gate/up as one multi call, down; swamp-engine/src/executor.rs:439-505).
Weights are random-init GGUF Q4_0 blocks from a fixed seed; >= 5 distinct
copies of the layer rotate so every GEMV streams from HBM (the rotation
footprint exceeds 4x the 126 MB L2).

metric: whole-job algorithmic GB/s (weights N*K*18/32 bytes + activations in
+ outputs out). With --gpus N (torchrun, one rank
per GPU) the model has N such layers, each tensor-parallel over the N ranks
(column split Q/K/V/gate/up, row split O/down + all-reduce), so per-GPU
bytes stay fixed (weak scaling).

--impl reference times the reference's CPU path (the C restatement of
swamp-engine forward_linear: per call, full-tensor dequant + f32 row dots,
row-partitioned over host threads) on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "llamanyon.rs_b200"))

SEED = 0x5EED1A11
Q40, Q4K = 2, 12
# (name, K, N) of one Llama-2-7B layer
LAYER = [("q", 4096, 4096), ("k", 4096, 4096), ("v", 4096, 4096), ("o", 4096, 4096),
         ("gate", 4096, 11008), ("up", 4096, 11008), ("down", 11008, 4096)]
TP_MODE = {"q": 1, "k": 1, "v": 1, "gate": 1, "up": 1, "o": 2, "down": 2}
BATCHES = (1, 4, 16)
METRIC = "Q4_0 decode GEMV GB/s (Llama-2-7B layer linears, batch 1/4/16)"


def wbytes(k, n):
    return n * k * 18 // 32


def decode_config(world):
    """The configs[1] workload both arms report (the reference arm times a
    bounded sample of it): N layers at N GPUs, TP N."""
    return {"workload": "configs[1]: Llama-2-7B layer Q4_0 linears (4x 4096->4096, 2x 4096->11008, "
                        "11008->4096) at decode batch 1, 4, 16",
            "batches": list(BATCHES), "layers_per_step": world, "parallelism": f"tp{world}" if world > 1 else "none",
            "l2_policy": "inputs larger than L2: rotating copies of the layer weights, over 4.5x L2 per GPU",
            "bytes_per_step": step_bytes(world)}


def step_bytes(n_layers=1):
    """algorithmic bytes of one step (114,148,352 / 115,085,312 / 118,833,152
    per layer at batch 1/4/16)."""
    tot = 0
    for b in BATCHES:
        for _, k, n in LAYER:
            tot += wbytes(k, n) + b * (k + n) * 4
    return tot * n_layers


def env_int(name, default):
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except FileNotFoundError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# dram__bytes_read.sum + dram__bytes_write.sum of one launch, from an ncu
# capture of the current kernels (profiles/): decode GEMV 4096->11008 batch 1
# (algorithmic 25,406,976 B); prefill GEMM Q4_K 4096->14336 M=512
# (algorithmic weight + activation bytes 41,418,752 B).
NCU_TRAFFIC = {"gemv_4096x11008_b1": 25_466_624, "gemm_q4k_4096x14336_m512": 54_764_032}


def measured_tensor_peak():
    """(burst, sustained) dense bf16 TFLOP/s and where they come from."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["bf16_tflops"]), float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "measured"
    return 1590.0, 1400.0, "fallback"


# Q4_K prefill at M=512 over the Llama-3-8B linear shapes (K, N)
PREFILL_M = 512
PREFILL_SHAPES = [(4096, 4096), (4096, 1024), (4096, 14336), (14336, 4096)]


def prefill_flops():
    return sum(2 * PREFILL_M * n * k for k, n in PREFILL_SHAPES)


# ---------------------------------------------------------------------------
# reference arm / CPU baseline
# ---------------------------------------------------------------------------

def ref_layer(oracle):
    """The configs[1] layer's 7 seeded Q4_0 tensors and the activations of
    each batch, as the reference CPU path consumes them."""
    ws = [(k, n, oracle.gen_weight(Q40, SEED, 500 + i, n, k)) for i, (_, k, n) in enumerate(LAYER)]
    xb = {(b, k): oracle.gen_x(SEED, 900 + 16 * b + k, (b, k)) for b in BATCHES for _, k, _ in LAYER}
    return ws, xb


def ref_step(oracle, sl, xb, threads):
    """One configs[1] step through the routes the reference takes: batch 1
    forward_linear's Q4_0 route (whole-slice dequant + f32 row dots,
    linear.rs:68-87); batches 4 and 16 forward_linear_batch, which sends a
    Q4_0 tensor to fallback_gemv (linear.rs:233-236,336-364): tokens over
    threads, each a dispatched fused_gemv_q4k over the tensor (timed as it
    runs; it does not decode Q4_0). sl: (K, rows, blocks) per tensor."""
    simd = oracle.simd_path() != "none"
    for b in BATCHES:
        for k, r, w in sl:
            if b == 1 or not simd:
                for t in range(b):
                    oracle.forward_linear(Q40, w, xb[(b, k)][t], r, k, threads)
            else:
                oracle.fallback_gemv_dispatched(w, xb[(b, k)], r, k, threads)


def ref_route(oracle):
    if oracle.simd_path() == "none":
        return "batches 4 and 16 as per-token forward_linear calls (no SIMD path on this CPU)"
    return (f"batches 4 and 16 through forward_linear_batch -> fallback_gemv with the dispatched "
            f"{oracle.simd_path()} fused_gemv_q4k (the reference's batched Q4_0 route, linear.rs:233-236,336-364; "
            f"numerically divergent, timed as it runs)")


def cpu_sample(threads, seconds_budget=20.0):
    """The reference CPU path on the whole configs[1] step (batches 1, 4, 16),
    repeated while inside the time budget. Returns (GB/s, steps, seconds,
    sample)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    oracle.build()
    ws, xb = ref_layer(oracle)
    ref_step(oracle, ws, xb, threads)  # warm (page-in)
    t0 = time.perf_counter()
    steps = 0
    while True:
        ref_step(oracle, ws, xb, threads)
        steps += 1
        el = time.perf_counter() - t0
        if el > seconds_budget:
            break
    sample = (f"{steps} whole configs[1] steps (7 Q4_0 tensors at batch 1, 4, 16) in {el:.1f} s: batch 1 "
              f"through forward_linear's Q4_0 route (full-tensor dequant + f32 row dots, "
              f"swamp-engine/src/linear.rs:68-87), {ref_route(oracle)}; {threads} host threads")
    return step_bytes(1) * steps / el / 1e9, steps, el, sample


def cpu_prefill_sample(threads, seconds_budget=8.0):
    """The reference's batched Q4_K path (fused_gemv_q4k_batched, scalar
    order; swamp-engine forward_linear_batch) on a token/row sample of the
    configs[2] shapes. Returns (GFLOP/s, sample description)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    oracle.build()
    toks, rows = 16, 512
    ws = [(k, oracle.gen_weight(Q4K, SEED, 700 + i, rows, k)) for i, (k, _) in enumerate(PREFILL_SHAPES)]
    xs = {k: oracle.gen_x(SEED, 800 + k, (toks, k)) for k, _ in PREFILL_SHAPES}
    oracle.forward_linear_batch(Q4K, ws[0][1], xs[ws[0][0]], rows, ws[0][0], threads)  # page-in
    t0 = time.perf_counter()
    flops, calls = 0, 0
    while True:
        for k, w in ws:
            oracle.forward_linear_batch(Q4K, w, xs[k], rows, k, threads)
            flops += 2 * toks * rows * k
            calls += 1
        el = time.perf_counter() - t0
        if el > seconds_budget:
            break
    return flops / el / 1e12, (f"{calls} forward_linear_batch calls (Q4_K, {toks} tokens x {rows} rows of each "
                               f"configs[2] shape) in {el:.1f} s on {threads} host threads")


def cpu_q4k_decode_variants(threads, seconds_each=3.0):
    """The reference's other Q4_K decode routes on the host, each timed on the
    configs[1] layer's 7 shapes quantized as Q4_K, batch 1 (GB/s of weight +
    activation bytes, like the headline):
      - forward_linear's Q4_K arm with the scalar kernel (fused_gemv_q4k.rs:466-508;
        the parity target), on `threads` threads, on the engine's cap of 6 and on 1;
      - the same arm as the reference dispatches it on this CPU
        (fused_gemv_q4k.rs:59-82 -> VNNI :101-317 or AVX2 :325-392), on the same
        thread counts: numerically divergent from the reference's dequantizer,
        timing only."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    oracle.build()
    ws = [(k, n, oracle.gen_weight(Q4K, SEED, 520 + i, n, k)) for i, (_, k, n) in enumerate(LAYER)]
    x = {k: oracle.gen_x(SEED, 920 + k, (k,)) for _, k, _ in LAYER}
    layer_b = sum(oracle.row_bytes(Q4K, k) * n + (k + n) * 4 for k, n, _ in ws)
    path = oracle.simd_path()

    def run(fn, nthr):
        for k, n, w in ws[:1]:
            fn(w, x[k], n, k, nthr)  # page-in
        t0, layers = time.perf_counter(), 0
        while True:
            for k, n, w in ws:
                fn(w, x[k], n, k, nthr)
            layers += 1
            el = time.perf_counter() - t0
            if el > seconds_each:
                return layer_b * layers / el / 1e9, layers, el

    scalar = lambda w, xx, n, k, t: oracle.forward_linear(Q4K, w, xx, n, k, t)
    disp = lambda w, xx, n, k, t: oracle.forward_linear_dispatched(w, xx, n, k, t)
    out = []
    variants = [("scalar", scalar, "fused_gemv_q4k_scalar (fused_gemv_q4k.rs:466-508), the parity target")]
    if path != "none":
        variants.append(("as-dispatched", disp, f"fused_gemv_q4k as dispatched on this CPU: {path} "
                         f"({'fused_gemv_q4k.rs:101-317' if path == 'avx512-vnni' else 'fused_gemv_q4k.rs:325-392'}); "
                         "numerically divergent, timing only"))
    for name, fn, what in variants:
        # all host threads, the reference engine's own cap of 6 (executor.rs:31), one
        for nthr in sorted({threads, min(6, threads), 1}, reverse=True):
            gbs, layers, el = run(fn, nthr)
            out.append({"variant": f"q4_k {name}", "value": round(gbs, 3), "unit": "GB/s", "cores": nthr,
                        "kind": "port", "sample": f"{layers} passes over the configs[1] layer's 7 shapes as Q4_K, "
                                                  f"batch 1, through forward_linear's Q4_K arm (linear.rs:28-46) "
                                                  f"with {what}, {el:.1f} s on {nthr} host threads"})
    return out


def reference_arm(args):
    """The reference's CPU route on the host cores, same metric and config.

    Each step is a bounded sample of the configs[1] step: the layer's 7 Q4_0
    tensors, cut to their first rows, at batch 1, 4 and 16 through the
    routes the reference takes (ref_step). The row cut keeps the whole
    --steps/--warmup run within about two minutes; GB/s counts the sampled
    bytes. Rank 0 only."""
    rank = env_int("RANK", 0)
    if rank != 0:
        return 0
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    oracle.build()
    threads = os.cpu_count() or 1
    world = env_int("WORLD_SIZE", 1)
    ws, xb = ref_layer(oracle)
    t0 = time.perf_counter()
    ref_step(oracle, ws, xb, threads)  # calibration pass (also pages the weights in)
    t_full = time.perf_counter() - t0
    budget = 120.0 / max(1, args.steps + args.warmup)
    frac = min(1.0, budget / t_full)
    sl = []
    for k, n, w in ws:
        rows = min(n, max(128, int(n * frac) // 128 * 128))
        sl.append((k, rows, w[: rows * oracle.row_bytes(Q40, k)]))
    step_b = sum(wbytes(k, r) + b * (k + r) * 4 for b in BATCHES for k, r, _ in sl)
    for _ in range(args.warmup):
        ref_step(oracle, sl, xb, threads)
    per_step = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        ref_step(oracle, sl, xb, threads)
        per_step.append(time.perf_counter() - t0)
    tot = sum(per_step)
    value = step_b * len(per_step) / tot / 1e9
    sample = (f"per step: the layer's 7 Q4_0 tensors, first {sl[0][1]}/{LAYER[0][2]} .. rows "
              f"({100 * frac:.1f}% of each), batch 1 through forward_linear's Q4_0 route (full-slice dequant + "
              f"f32 row dots, swamp-engine/src/linear.rs:68-87), {ref_route(oracle)}; {threads} host threads")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1000 * tot / len(per_step), 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": decode_config(world),
        "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": sample, "sampled_bytes_per_step": step_b},
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def setup_gpu(args):
    """torch.distributed (one rank per GPU) + the library on this rank's GPU."""
    import torch
    import swamp_gpu as sg
    import build_lib

    rank, world = env_int("RANK", 0), env_int("WORLD_SIZE", 1)
    local = env_int("LOCAL_RANK", 0)
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    if rank == 0:
        build_lib.build()
    if dist:
        dist.barrier()
    gpu = sg.SwampGpu()
    if world > 1:
        uid = gpu.get_unique_id() if rank == 0 else bytes(128)
        t = torch.frombuffer(bytearray(uid), dtype=torch.uint8).cuda()
        dist.broadcast(t, 0)
        gpu.init_rank(rank, world, bytes(t.cpu().numpy().tobytes()), local)
    else:
        gpu.init(1)
    return torch, gpu, dist, rank, world, local


def graph_of(torch, fn):
    """Capture fn() (stream-ordered library calls on the current stream) into a CUDA graph."""
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    return g


def time_graphs(torch, graphs, reps, st):
    """Replay graphs round-robin `reps` times; device ms between two events."""
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(st)
    for j in range(reps):
        graphs[j % len(graphs)].replay()
    e1.record(st)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1)


def gpu_arm(args):
    import numpy as np
    torch, gpu, dist, rank, world, local = setup_gpu(args)

    n_layers = world  # weak scaling: per-GPU bytes fixed
    l2 = torch.cuda.get_device_properties(local).L2_cache_size
    layer_b = sum(wbytes(k, n) for _, k, n in LAYER)
    copies = max(5, int(np.ceil(4.5 * l2 / (layer_b / world))) + 1, n_layers)
    # one seeded tensor per layer linear, generated on the device `copies`
    # times: every copy is a separate allocation, so rotating copies streams
    # from HBM
    model = []
    for c in range(copies):
        layer = {}
        for i, (name, k, n) in enumerate(LAYER):
            layer[name] = gpu.synth_weight(Q40, SEED, 1000 + i, n, k, TP_MODE[name] if world > 1 else 0)
        model.append(layer)
    # K offset of each tensor's shard in x (row split takes a K slice)
    col0 = {name: model[0][name].shard()[3] for name, _, _ in LAYER}
    xs = {b: torch.randn(b, 11008, device="cuda") for b in BATCHES}
    ys = {b: {name: torch.empty(b, 11008, device="cuda") for name, _, _ in LAYER} for b in BATCHES}
    LD = 11008
    # our kernels per call: the activation prep kernel and the GEMV kernel
    def kernels_per_call(b):
        return 2

    def xat(b, name):
        return xs[b].data_ptr() + 4 * col0[name]

    def run_layer(layer, b, st):
        y = ys[b]
        gpu.linear_multi_device([layer["q"], layer["k"], layer["v"]], xat(b, "q"), LD,
                                [y["q"].data_ptr(), y["k"].data_ptr(), y["v"].data_ptr()], [LD] * 3, b, stream=st)
        gpu.linear_device(layer["o"], xat(b, "o"), LD, y["o"].data_ptr(), LD, b, stream=st)
        gpu.linear_multi_device([layer["gate"], layer["up"]], xat(b, "gate"), LD,
                                [y["gate"].data_ptr(), y["up"].data_ptr()], [LD] * 2, b, stream=st)
        gpu.linear_device(layer["down"], xat(b, "down"), LD, y["down"].data_ptr(), LD, b, stream=st)
        return 4 * kernels_per_call(b)

    def step(j):
        """one step = batches 1, 4, 16 over n_layers layers; copies rotate with
        j. Returns the number of our kernel launches."""
        st = torch.cuda.current_stream().cuda_stream
        calls = 0
        for bi, b in enumerate(BATCHES):
            for li in range(n_layers):
                calls += run_layer(model[(j * len(BATCHES) * n_layers + bi * n_layers + li) % copies], b, st)
        return calls

    # warmup (eager: allocates the scratch once), then one graph per rotation offset
    for j in range(args.warmup):
        step(j)
    torch.cuda.synchronize()
    launches_per_step = step(0)
    torch.cuda.synchronize()
    graphs = [graph_of(torch, lambda j=j: step(j)) for j in range(copies)] if not args.eager else None
    for j in range(args.warmup):
        graphs[j % copies].replay() if graphs else step(j)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()

    # ------------------------------------------------------------ timed
    st = torch.cuda.current_stream()
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    if dist:
        dist.barrier()
    if graphs:
        ms = time_graphs(torch, graphs, args.steps, st)
    else:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record(st)
        for j in range(args.steps):
            step(j)
        e1.record(st)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
    if dist:
        dist.barrier()
    clocks = sampler.stop()
    if dist:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_per_step = ms / args.steps
    value = step_bytes(n_layers) * args.steps / (ms / 1e3) / 1e9

    # ------------------------------------------ per-launch roofline pass
    # for each (shape, batch): a graph of `copies` back-to-back single-tensor
    # GEMVs over rotating copies, timed with events; average device time per
    # launch in steady state
    tot_by, tot_us, per_shape = 0.0, 0.0, {}
    reps = 20
    for b in BATCHES:
        for name, k, n in (("q", 4096, 4096), ("gate", 4096, 11008), ("down", 11008, 4096)):
            mult = {"q": 4, "gate": 2, "down": 1}[name]

            def one(name=name, b=b):
                stp = torch.cuda.current_stream().cuda_stream
                for c in range(copies):
                    gpu.linear_device(model[c][name], xat(b, name), LD, ys[b][name].data_ptr(), LD, b, stream=stp)
            g = graph_of(torch, one)
            g.replay()
            ms1 = time_graphs(torch, [g], reps, st)
            us = ms1 * 1e3 / (reps * copies)
            by = (wbytes(k, n) + b * (k + n) * 4) / world
            per_shape[f"{k}x{n}_b{b}"] = round(by / (us * 1e-6) / 1e9, 1)
            tot_by += by * mult
            tot_us += us * mult
            del g
    achieved = tot_by / (tot_us * 1e-6) / 1e9
    peak, peak_kind = measured_peaks()

    # ---------------------------------------------- prefill
    prefill = prefill_bench(torch, gpu, st, args) if world == 1 and not args.no_prefill else None
    upload = gguf_upload_bench(torch, gpu) if world == 1 and not args.no_prefill else None
    q6k = q6k_bench(torch, gpu, st) if world == 1 and not args.no_prefill else None
    decode = model_decode_bench(torch, gpu, args) if world == 1 and not args.no_model else None
    tp_model = tp_model_bench(torch, gpu, args, dist, world) if not args.no_tp_model else None

    # -------------------------------------------------------------- e2e
    # the public host-pointer C ABI: x copied in and y read back on every call
    # every rank calls the host-buffer entry points for its shards (column
    # split: its rows come back; row split: the all-reduced sum); whole-job
    # bytes over the slowest rank's wall time. Inputs and outputs are
    # page-locked host arrays (sg_host_alloc), the outputs reused from call to
    # call as an engine reuses its buffers; the library copies them by DMA.
    names = ("q", "k", "v", "o", "gate", "up", "down")
    e2e_steps = max(1, min(args.steps, args.e2e_steps))

    def host_loop(xh, yh):
        """e2e_steps steps through the host entry points; wall seconds (max
        over ranks) and the bytes copied in and out."""
        h2d = d2h = 0
        for j in range(-1, e2e_steps):  # step -1: untimed warm-up (staging buffers grow once)
            if j == 0:
                if dist:
                    dist.barrier()
                t0 = time.perf_counter()
                h2d = d2h = 0
            for bi, b in enumerate(BATCHES):
                y = yh[b]
                for li in range(n_layers):
                    layer = model[(max(j, 0) * len(BATCHES) * n_layers + bi * n_layers + li) % copies]
                    x4096 = xh[b][:, :4096]
                    if b == 1:
                        gpu.linear_multi([layer["q"], layer["k"], layer["v"]], x4096[0],
                                         outs=[y["q"][0], y["k"][0], y["v"][0]])
                        gpu.linear_multi([layer["gate"], layer["up"]], x4096[0], outs=[y["gate"][0], y["up"][0]])
                    else:
                        for name in ("q", "k", "v", "gate", "up"):
                            gpu.linear(layer[name], x4096, out=y[name])
                    gpu.linear(layer["o"], x4096, out=y["o"])
                    gpu.linear(layer["down"], xh[b], out=y["down"])
                    h2d += b * 4096 * 4 * (2 if b == 1 else 6) + b * 11008 * 4
                    d2h += b * 4 * (5 * 4096 + 2 * 11008)
        el = time.perf_counter() - t0
        if dist:
            t = torch.tensor([el], dtype=torch.float64, device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            el = float(t.item())
        return el, h2d, d2h

    # page-locked host arrays (sg_host_alloc): the library copies them by DMA
    xh = {}
    for b in BATCHES:
        xh[b] = gpu.host_array((b, 11008))
        xh[b][:] = xs[b].cpu().numpy()
    yh = {b: {nm: gpu.host_array((b, model[0][nm].n_rows)) for nm in names} for b in BATCHES}
    el, h2d, d2h = host_loop(xh, yh)
    # ordinary (pageable) arrays, as an engine that keeps Vec<f32> buffers
    # passes them: through the library's staging buffer
    xp = {b: np.array(xh[b]) for b in BATCHES}
    yp = {b: {nm: np.zeros_like(yh[b][nm]) for nm in names} for b in BATCHES}
    el_p, _, _ = host_loop(xp, yp)
    e2e = {"value": round(step_bytes(n_layers) * e2e_steps / el / 1e9, 3), "unit": "GB/s",
           "h2d_bytes_per_step": h2d // e2e_steps, "d2h_bytes_per_step": d2h // e2e_steps,
           "steps": e2e_steps,
           "path": "sg_linear / sg_linear_multi, page-locked host buffers (copy in, launch, copy out, sync per "
                   "call); outputs reused from step to step",
           "pageable_value": round(step_bytes(n_layers) * e2e_steps / el_p / 1e9, 3)}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        gbs, _, _, sample = cpu_sample(threads, seconds_budget=args.cpu_seconds)
        cpu = {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port", "sample": sample,
               "variants": cpu_q4k_decode_variants(threads)}

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_per_step, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None,
            "dtype": "u4 weights x s8 activation digits (3 per value), s32 tensor-core accumulate, f32 epilogue",
            "data": "synthetic (seeded random-init Q4_0 blocks, N(0,1) activations)",
            "config": decode_config(world),
            "run": {"allreduce": gpu.allreduce_path() if world > 1 else None,
                    "execution": "eager" if args.eager else "CUDA graph per step (PDL edges kept)",
                    "l2": f"{copies} rotating layer copies ({copies * layer_b / world / 1e6:.0f} MB per GPU vs L2 "
                          f"{l2 / 1e6:.0f} MB)"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": NCU_TRAFFIC["gemv_4096x11008_b1"],
                         "traffic_launch": "4096x11008 batch 1 (algorithmic 25,406,976 B)", "peak_kind": peak_kind,
                         "traffic_note": "ncu dram bytes of one launch of that shape, per launch like achieved",
                         "kernel": "gemv_kernel (mma.sync u8 x s8, one launch per GEMV, + xprep_kernel), back-to-back in a CUDA graph",
                         "per_shape_gbs": per_shape},
            "e2e": e2e,
            "cpu_baseline": cpu,
            "clocks": clocks,
            "gpu_launches": launches_per_step * args.steps,
            "prefill": prefill,
            "gguf_upload": upload,
            "q6k": q6k,
            "model_decode": decode,
            "tp_model": tp_model,
        }
        if decode and cpu and cpu.get("variants"):
            # the CPU engine runs every token of a step through the Q4_K decode
            # kernel it dispatches (the batched VNNI route loops that kernel
            # over the tokens), so one token costs the model's weight bytes at
            # that kernel's measured rate on all host threads (a full 32-layer
            # CPU run would take minutes per token)
            by = {(v["variant"], v["cores"]): v["value"] for v in cpu["variants"]}
            rate = by.get(("q4_k as-dispatched", cpu["cores"]),
                          by.get(("q4_k scalar", cpu["cores"])))
            if rate:
                for run in decode["runs"].values():
                    run["cpu_extrapolated_tok_s"] = round(rate * 1e9 / decode["weight_bytes_per_step"], 4)
                decode["cpu_extrapolation"] = (f"one token = the model's weight bytes at the host's Q4_K decode "
                                               f"rate ({rate} GB/s, {cpu['cores']} threads)")
        print(json.dumps(line), flush=True)
    graphs = None
    torch.cuda.synchronize()
    for layer in model:
        for w in layer.values():
            w.free()
    gpu.shutdown()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def tp_model_bench(torch, gpu, args, dist, world):
    """a random-init Llama-3-70B-architecture model in Q4_0 (80
    layers, d 8192, 64 query / 8 KV heads, FFN 28672, vocab 128256)
    tensor-parallel over the job's ranks (column split Q/K/V/gate/up, row
    split O/down with the in-place all-reduce of each row-split call), through
    llamanyon.rs_b200/decoder.py. The workload: a 2048-token prefill (32
    sequences x 64 prompt tokens, one pass) followed by batch-32 greedy
    decoding of 128 tokens, each decode step one CUDA graph. Device time with
    CUDA events, max over ranks. Weights are generated on the device (each
    rank its own shards, from the same seeds at every degree)."""
    import numpy as np
    import decoder as dec
    B, P, NEW = 32, 64, args.tp_new
    cfg = dec.DecoderConfig(n_layers=args.tp_layers, d=8192, n_heads=64, n_kv_heads=8, ffn=28672, vocab=128256,
                            dtype=Q40, context_len=1024, max_seq=P + NEW + 64)
    model = dec.SynthModel(gpu, cfg, SEED, stacked=False)
    D = dec.Decoder(gpu, model, n_seqs=B, max_rows=B * P)
    rng = np.random.default_rng(SEED + 70)
    prompts = rng.integers(0, cfg.vocab, size=(B, P))
    st = torch.cuda.Stream()
    ev = lambda: torch.cuda.Event(enable_timing=True)

    def maxr(ms):
        if not dist:
            return ms
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def prefill_rows():
        return D.set_rows(prompts.T.reshape(-1), np.repeat(np.arange(P), B), np.tile(np.arange(B), P))
    with torch.cuda.stream(st):
        rows = prefill_rows()
        D.forward(rows, stream=st.cuda_stream, logits_rows=slice(rows - B, rows), prefill=(B, P, 1, B))  # workspaces
        st.synchronize()
        if dist:
            dist.barrier()
        e0, e1 = ev(), ev()
        e0.record(st)
        rows = prefill_rows()
        D.forward(rows, stream=st.cuda_stream, logits_rows=slice(rows - B, rows), prefill=(B, P, 1, B))
        e1.record(st)
        st.synchronize()
    prefill_ms = maxr(e0.elapsed_time(e1))
    first = D.next[:B].clone()
    seqs = torch.arange(B, dtype=torch.int32, device="cuda")
    with torch.cuda.stream(st):
        def start():
            D.tokens[:B].copy_(first)
            D.pos[:B].fill_(P)
            D.seq[:B].copy_(seqs)
        start()
        D.forward(B, stream=st.cuda_stream, decode=True)  # first use of the decode shapes
        start()
        st.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=st):
            D.forward(B, stream=st.cuda_stream, decode=True)
            D.advance(B)
        for _ in range(3):
            g.replay()
        start()
        st.synchronize()
        if dist:
            dist.barrier()
        steps = NEW - 1
        e2, e3 = ev(), ev()
        e2.record(st)
        for _ in range(steps):
            g.replay()
        e3.record(st)
        st.synchronize()
        toks = D.tokens[:B].cpu().tolist()
        del g
    dec_ms = maxr(e2.elapsed_time(e3))
    step_ms = dec_ms / steps
    peak, peak_kind = measured_peaks()
    tburst, tsust, tkind = measured_tensor_peak()
    mean_len = P + 1 + (steps - 1) / 2
    kv_bytes = 2 * B * cfg.n_layers * (cfg.n_kv_heads // world) * cfg.head_dim * 4 * mean_len
    by = model.weight_bytes() + kv_bytes  # per rank
    gbs = by / (step_ms * 1e-3) / 1e9
    flops = 2 * B * P * (sum(cfg.shape(r)[0] * cfg.shape(r)[1] for r in dec.ROLES) * cfg.n_layers
                         + cfg.d * cfg.vocab / P)  # the head runs on the last position only
    tflops_gpu = flops / world / (prefill_ms * 1e-3) / 1e12
    out = {
        "workload": f"configs[4]: random-init Llama-3-70B-architecture Q4_0, {cfg.n_layers} layers, TP{world}; "
                    f"prefill {B * P} tokens ({B} sequences x {P}), then batch-{B} greedy decode of {NEW} tokens",
        "tp": world,
        "prefill_ms": round(prefill_ms, 2), "prefill_tok_s": round(B * P / (prefill_ms * 1e-3), 1),
        "prefill_roofline": {"bound": "tensor", "achieved": round(tflops_gpu, 1), "peak": tburst, "unit": "TFLOP/s",
                             "frac": round(tflops_gpu / tburst, 4), "per": "GPU", "peak_kind": tkind + " bf16 burst"},
        "decode_ms_per_step": round(step_ms, 4), "decode_tok_s": round(B / (step_ms * 1e-3), 1),
        "e2e_tok_s": round(B * NEW / ((prefill_ms + dec_ms) * 1e-3), 1),
        "decode_roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                            "frac": round(gbs / peak, 4), "per": "GPU", "bytes_per_step_per_gpu": int(by),
                            "peak_kind": peak_kind},
        "allreduce": (("library peer kernel over NVLink (values with epochs, no fence)" if gpu.allreduce_path() == "peer"
                       else "NCCL") + " in-place all-reduce after each row-split linear (O, down): 2 per layer"),
        "tokens_seq0": [t for t in toks[:1]],
    }
    D.free()
    model.free()
    return out


def model_decode_bench(torch, gpu, args):
    """a random-init Llama-3-8B-architecture model in Q4_K (32
    layers, d 4096, 32 query / 8 KV heads, FFN 14336, vocab 128256, Q4_K
    output head) on the device through llamanyon.rs_b200/decoder.py: a
    512-token prompt prefilled in one pass (prefill GEMMs, causal attention
    rows), then greedy decoding, at batch 1 and 8 (independent sequences with
    their own KV-cache slots). Each decode step is one CUDA graph (every
    layer's linears, RMSNorms, RoPE + cache store, attention, SiLU-mul, the
    output head, argmax, the device-side token advance and the D2H copy of
    the step's tokens to pinned host memory); 3 warm-up steps, then the
    position is reset and model_new - 1 steps are timed with CUDA events
    (the first new token comes from the prefill). Weights are generated on
    the device; prompt tokens are seeded uniform over the vocabulary."""
    import numpy as np
    import decoder as dec
    P, NEW = 512, args.model_new
    cfg = dec.DecoderConfig(n_layers=args.model_layers, d=4096, n_heads=32, n_kv_heads=8, ffn=14336,
                            vocab=128256, dtype=Q4K, context_len=2048, max_seq=2048)
    model = dec.SynthModel(gpu, cfg, SEED)
    wbytes_step = model.weight_bytes()
    peak, peak_kind = measured_peaks()
    runs = {}
    for B in (1, 8):
        D = dec.Decoder(gpu, model, n_seqs=B, max_rows=B * P)
        rng = np.random.default_rng(SEED + B)
        prompts = rng.integers(0, cfg.vocab, size=(B, P))
        st = torch.cuda.Stream()
        ev = lambda: torch.cuda.Event(enable_timing=True)
        host_tok = torch.empty(B, dtype=torch.int32, pin_memory=True)
        with torch.cuda.stream(st):
            # rows in (position, sequence) order: the last position's rows are
            # the last B, whose logits the prefill computes
            def prefill_rows():
                return D.set_rows(prompts.T.reshape(-1), np.repeat(np.arange(P), B), np.tile(np.arange(B), P))
            rows = prefill_rows()
            D.forward(rows, stream=st.cuda_stream, logits_rows=slice(rows - B, rows), prefill=(B, P, 1, B))  # first use: workspaces
            st.synchronize()
            e0, e1 = ev(), ev()
            e0.record(st)
            rows = prefill_rows()  # H2D of the prompt inside the timed region
            D.forward(rows, stream=st.cuda_stream, logits_rows=slice(rows - B, rows), prefill=(B, P, 1, B))
            host_tok.copy_(D.next[:B], non_blocking=True)
            e1.record(st)
            st.synchronize()
            prefill_ms = e0.elapsed_time(e1)
            first = D.next[:B].clone()
            seqs = torch.arange(B, dtype=torch.int32, device="cuda")

            def start():
                D.tokens[:B].copy_(first)
                D.pos[:B].fill_(P)
                D.seq[:B].copy_(seqs)
            start()
            D.forward(B, stream=st.cuda_stream, decode=True)  # first use of the decode shapes
            start()
            st.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=st):
                D.forward(B, stream=st.cuda_stream, decode=True)
                D.advance(B)
                host_tok.copy_(D.tokens[:B], non_blocking=True)
            for _ in range(3):
                g.replay()
            start()
            st.synchronize()
            steps = NEW - 1
            e2, e3 = ev(), ev()
            e2.record(st)
            for _ in range(steps):
                g.replay()
            e3.record(st)
            st.synchronize()
            dec_ms = e2.elapsed_time(e3)
            del g
        step_ms = dec_ms / steps
        # algorithmic bytes of a step: every weight once plus the K and V rows
        # attention reads (mean position of the timed steps)
        mean_len = P + 1 + (steps - 1) / 2
        kv_bytes = 2 * B * cfg.n_layers * cfg.n_kv_heads * cfg.head_dim * 4 * mean_len
        by = wbytes_step + kv_bytes
        gbs = by / (step_ms * 1e-3) / 1e9
        runs[f"b{B}"] = {
            "prefill_ms": round(prefill_ms, 2), "prefill_tok_s": round(B * P / (prefill_ms * 1e-3), 1),
            "decode_ms_per_step": round(step_ms, 4), "decode_tok_s": round(B / (step_ms * 1e-3), 1),
            "e2e_tok_s": round(B * NEW / ((prefill_ms + dec_ms) * 1e-3), 1),
            "decode_bytes_per_step": int(by),
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(gbs / peak, 4), "peak_kind": peak_kind},
            "h2d_bytes": B * P * 12, "d2h_bytes_per_step": B * 4}
        D.free()
    model.free()
    return {"workload": f"configs[3]: random-init Llama-3-8B-architecture Q4_K, {cfg.n_layers} layers, prompt {P}, "
                        f"{NEW} new tokens, greedy, batch 1 and 8",
            "weight_bytes_per_step": wbytes_step, "runs": runs,
            "execution": "prefill: one eager pass; decode: one CUDA graph per token",
            "ops": "sg_embed / sg_rmsnorm / sg_linear (stacked QKV, stacked gate+up) / sg_rope_attention (decode; "
                   "sg_rope_kv + sg_attention_prefill at prefill) / "
                   "sg_linear + accumulate (O, down) / sg_silu_mul / sg_argmax"}


def q6k_bench(torch, gpu, st):
    """Q6_K, the dtype real Q4_K_M files keep for ffn_down and the output
    head (Llama-3-8B shapes): decode GEMV GB/s at 1 and 16 tokens
    (algorithmic bytes N*K*210/256 + activations) and prefill GEMM TFLOP/s at
    M=512. Two rotating copies per shape (> L2), CUDA graphs of back-to-back
    calls, device time per call."""
    out = {}
    Q6K = 14
    for (k, n) in ((14336, 4096), (4096, 128256)):
        ws = [gpu.synth_weight(Q6K, SEED, 5000 + c, n, k) for c in range(2)]
        for b in ((1, 16) if n < 100000 else (1,)) + ((PREFILL_M,) if n < 100000 else ()):
            x = torch.randn(b, k, device="cuda")
            y = torch.empty(b, n, device="cuda")

            def one(b=b, x=x, y=y):
                stp = torch.cuda.current_stream().cuda_stream
                for w in ws:
                    gpu.linear_device(w, x.data_ptr(), k, y.data_ptr(), n, b, stream=stp)
            one()
            g = graph_of(torch, one)
            g.replay()
            reps = 10
            us = time_graphs(torch, [g], reps, st) * 1e3 / (reps * len(ws))
            key = f"{k}x{n}_b{b}"
            if b <= 16:
                by = n * k * 210 // 256 + b * (k + n) * 4
                out[key] = {"us": round(us, 2), "gbs": round(by / us / 1e3, 1)}
            else:
                out[key] = {"us": round(us, 2), "tflops": round(2 * b * n * k / us / 1e6, 1)}
            del g
        for w in ws:
            w.free()
    return {"kernels": "gemv_q6k_kernel (CUDA cores) at <= 16 tokens; gemm_kernel (tcgen05) above",
            "per_shape": out}


def gguf_upload_bench(torch, gpu):
    """The GGUF -> device path (sg_gguf_register): one Q4_K 4096->14336
    tensor (33 MB of blocks) in a GGUF file under /tmp, mapped (page cache
    warm) and uploaded with repack; host wall clock around register +
    synchronize, median of 5."""
    import tempfile
    import numpy as np
    import swamp_gpu as sg
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import gguf_writer
    k, n = 4096, 14336
    raw = gpu.synth_blocks(Q4K, SEED, 4000, n, k)
    img, _ = gguf_writer.model_file({"blk.0.ffn_up.weight": (Q4K, n, k, raw)})
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "upload.gguf")
        with open(path, "wb") as f:
            f.write(img)
        g = sg.GgufFile(gpu, path=path)
        t = g.tensor("blk.0.ffn_up.weight")
        times = []
        for _ in range(6):
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            w = g.register(t)
            gpu.synchronize()
            times.append(time.perf_counter() - t0)
            w.free()
        g.close()
    el = statistics.median(times[1:])
    return {"value": round(t.nbytes / el / 1e9, 2), "unit": "GB/s", "bytes": t.nbytes,
            "ms": round(el * 1e3, 3), "tensor": "Q4_K 4096->14336 from a mapped GGUF file (register + repack)"}


def prefill_bench(torch, gpu, st, args):
    """Q4_K prefill GEMM, M=512, the four Llama-3-8B shapes. Each
    shape rotates over distinct weight copies whose bytes together exceed 4x
    the L2 cache (so every call streams its weights from HBM); each shape is
    timed as a CUDA graph of back-to-back calls. TFLOP/s counts 2*M*N*K (one
    product); the kernel issues three bf16 products per k-step (hi/lo operand
    split), so the tensor pipe does 3x that work."""
    import numpy as np
    M = PREFILL_M
    l2 = torch.cuda.get_device_properties(torch.cuda.current_device()).L2_cache_size
    ws, copies_of = {}, {}
    for i, (k, n) in enumerate(PREFILL_SHAPES):
        copies = max(2, int(np.ceil(4 * l2 / (n * k * 144 / 256))) + 1)
        copies_of[(k, n)] = copies
        ws[(k, n)] = [gpu.synth_weight(Q4K, SEED, 2000 + 64 * i + c, n, k) for c in range(copies)]
    x = torch.randn(M, 14336, device="cuda")
    y = torch.empty(M, 14336, device="cuda")
    reps = max(3, min(50, args.prefill_reps))
    per_shape, tot_us = {}, 0.0
    for (k, n), wl in ws.items():
        def one(wl=wl, k=k, n=n):
            stp = torch.cuda.current_stream().cuda_stream
            for w in wl:
                gpu.linear_device(w, x.data_ptr(), k, y.data_ptr(), n, M, stream=stp)
        one()  # eager first call: scratch, kernel attributes
        torch.cuda.synchronize()
        g = graph_of(torch, one)
        for _ in range(3):
            g.replay()
        ms = time_graphs(torch, [g], reps, st)
        us = ms * 1e3 / (reps * len(wl))
        tot_us += us
        per_shape[f"{k}x{n}"] = {"us": round(us, 2), "tflops": round(2 * M * n * k / us / 1e6, 1)}
        del g
    achieved = prefill_flops() / tot_us / 1e6
    burst, sustained, kind = measured_tensor_peak()
    cpu = None
    if not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        tf, sample = cpu_prefill_sample(threads, seconds_budget=min(8.0, args.cpu_seconds))
        cpu = {"value": round(tf * 1e3, 3), "unit": "GFLOP/s", "cores": threads, "kind": "port", "sample": sample}
    for wl in ws.values():
        for w in wl:
            w.free()
    return {"metric": "Q4_K prefill GEMM TFLOP/s (configs[2]: Llama-3-8B linears, M=512)",
            "value": round(achieved, 1), "unit": "TFLOP/s", "flops_per_pass": prefill_flops(),
            "l2_policy": {f"{k}x{n}": f"{c} rotating copies ({c * n * k * 144 / 256 / 1e6:.0f} MB vs L2 "
                                      f"{l2 / 1e6:.0f} MB)" for (k, n), c in copies_of.items()},
            "us_per_pass": round(tot_us, 1), "per_shape": per_shape,
            "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": burst, "unit": "TFLOP/s",
                         "frac": round(achieved / burst, 4), "peak_kind": f"{kind} bf16 dense burst",
                         "tensor_pipe_frac": round(3 * achieved / burst, 4),
                         "traffic": NCU_TRAFFIC["gemm_q4k_4096x14336_m512"],
                         "traffic_launch": "4096x14336 M=512 (algorithmic: weights 33.0 MB + bf16 hi/lo x 8.4 MB)",
                         "kernel": "gemm_kernel (tcgen05 M128 N256 K16 bf16, 3 products per k-step) "
                                   "+ gemm_xprep_kernel"},
            "cpu_baseline": cpu,
            "gpu_launches_per_call": 2}


def profile_arm(args):
    """One tensor shape, eager back-to-back launches (for ncu; not a bench line)."""
    import numpy as np
    torch, gpu, dist, rank, world, local = setup_gpu(args)
    k, n, b = (int(v) for v in args.profile.split(","))
    dtype = Q4K if args.dtype == "q4k" else Q40
    copies = 4
    ws = [gpu.synth_weight(dtype, SEED, 3000 + c, n, k) for c in range(copies)]
    x = torch.randn(b, k, device="cuda")
    y = torch.empty(b, n, device="cuda")
    st = torch.cuda.current_stream()
    for i in range(args.warmup + args.steps):
        if i == args.warmup:
            torch.cuda.synchronize()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(st)
        gpu.linear_device(ws[i % copies], x.data_ptr(), k, y.data_ptr(), n, b, stream=st.cuda_stream)
    e1.record(st)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / args.steps
    by = (n * k * (18 if dtype == Q40 else 144) // (32 if dtype == Q40 else 256)) + b * (k + n) * 4
    print(json.dumps({"profile": args.profile, "dtype": args.dtype, "us_per_call": round(us, 2),
                      "gbs": round(by / us / 1e3, 1), "note": "eager, host-launch bound; for ncu only"}))
    for w in ws:
        w.free()
    gpu.shutdown()
    return 0


def ar_latency_arm(args):
    """Latency of the row-split all-reduce (sg_allreduce_device) per call:
    20 back-to-back calls captured in a CUDA graph, replayed 10 times, device
    time, max over ranks; one JSON line from rank 0 (not a bench line)."""
    torch, gpu, dist, rank, world, local = setup_gpu(args)
    res = {}
    st = torch.cuda.Stream()
    for n in (4096, 16384, 65536, 262144):
        buf = torch.ones(n, device="cuda")
        with torch.cuda.stream(st):
            for _ in range(3):
                gpu.allreduce_device(buf.data_ptr(), n, stream=st.cuda_stream)
            st.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=st):
                for _ in range(20):
                    gpu.allreduce_device(buf.data_ptr(), n, stream=st.cuda_stream)
            g.replay()
            st.synchronize()
            if dist:
                dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            for _ in range(10):
                g.replay()
            e1.record(st)
            st.synchronize()
        us = torch.tensor([e0.elapsed_time(e1) * 1e3 / 200], device="cuda")
        if dist:
            dist.all_reduce(us, op=dist.ReduceOp.MAX)
        res[f"{n * 4 // 1024}KB"] = round(float(us), 2)
        del g
    path = gpu.allreduce_path() if world > 1 else "none"
    gpu.synchronize()
    if dist:
        dist.barrier()
    gpu.shutdown()
    if rank == 0:
        print(json.dumps({"allreduce_latency_us": res, "n_gpus": world, "path": path,
                          "method": "20 calls per CUDA graph, 10 replays, device time, max over ranks"}), flush=True)
    if dist:
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--eager", action="store_true", help="no CUDA graphs")
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--profile", default=None, help="K,N,B: single-shape eager launches (for ncu)")
    ap.add_argument("--dtype", default="q4_0", choices=["q4_0", "q4k"])
    ap.add_argument("--ar-latency", action="store_true", help="all-reduce latency per call (under torchrun)")
    ap.add_argument("--no-prefill", action="store_true", help="skip the configs[2] prefill measurement")
    ap.add_argument("--prefill-reps", type=int, default=20)
    ap.add_argument("--no-model", action="store_true", help="skip the configs[3] model decode measurement")
    ap.add_argument("--model-layers", type=int, default=32, help="configs[3] layers (32 = the named model)")
    ap.add_argument("--model-new", type=int, default=256, help="configs[3] generated tokens")
    ap.add_argument("--no-tp-model", action="store_true", help="skip the configs[4] tensor-parallel model")
    ap.add_argument("--tp-layers", type=int, default=80, help="configs[4] layers (80 = the named model)")
    ap.add_argument("--tp-new", type=int, default=128, help="configs[4] generated tokens")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return reference_arm(args)
    if args.ar_latency:
        return ar_latency_arm(args)
    if args.profile:
        return profile_arm(args)
    return gpu_arm(args)


if __name__ == "__main__":
    sys.exit(main())
