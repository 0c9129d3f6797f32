"""Benchmark of the quantised linear (libsdq) on B200, one JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload cfg2]
    python bench.py --impl reference ...      # the CPU arm (oracle port of the reference)
    torchrun --nproc-per-node N bench.py --gpus N ...

Workloads (the benchmark plan's configurations; data synthetic, seeded):
  cfg2  (default) X bf16 [4096, 12288] . W [3072, 12288]^T, W8 g64  -- configs[1]
  cfg1  X [1024, 3072] . W [3072, 3072]^T, W4
  cfg3  X [M<=8, 3072] . W [18432, 3072]^T, W4 (HBM-bound; reports GB/s)
  cfg5  X [16384, 3072] . W [12288, 3072]^T, W4
  cfg4  the Flux-shaped stack (sdq.flux): 312 linears of one transformer forward (19 double +
        38 single blocks, 512 text + 4096 image tokens, out-proj / MLP down-proj W8, rest W4);
        a step replays the forward's linears as one CUDA graph (value), and the whole forward
        (attention and elementwise work included) is timed beside it
A step is one quantised matmul over the workload's X with the weight resident in HBM.
The default line (cfg2) also carries `secondary`: configs 1, 3 (M = 1, 2, 4, 8) and 5 on
one GPU, each measured the same way with its own device time, roofline fraction and clocks;
and `strong_scaling`: config 5's fixed layer split over the N ranks along its output
features, timed as the GEMM alone and as GEMM + exchange (max over ranks).
With N > 1 ranks each rank holds one workload-sized column shard of a weight N times
as wide (weak scaling) and the [M, N*n] output is all-gathered over NVLink (NCCL).

Timing: W untimed warm-up steps, then K timed steps bracketed by barrier + synchronize.
For cfg1/2/3/5 the K steps run back to back over R rotating copies of the inputs (X, packed
W, scales, biases, Y) that together exceed twice the L2, so no step finds its inputs in L2;
one pair of CUDA events on the launching stream brackets them, and on one GPU the K
launches are replayed as one CUDA graph.  cfg4 and encoders time each step with its own
events after a 256 MiB L2-flushing write.  The total is max-reduced over ranks.  `e2e`
repeats the step eagerly through the public API with the step's X copied from pinned host
memory and the (gathered) Y copied back inside the timed region (L2 flushed before each
step, outside its events); on one GPU that is one sdq_quantized_matmul_host call, which
overlaps the upload, product and download of row chunks.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "stable-diffusion.rs_b200"))

WORKLOADS = {
    # name: (M, K, N, bits, sigma_w, metric kind)
    "cfg1": (1024, 3072, 3072, 4, 0.02, "tflops"),
    "cfg2": (4096, 12288, 3072, 8, 0.01, "tflops"),
    "cfg3": (8, 3072, 18432, 4, 0.02, "gbs"),
    "cfg5": (16384, 3072, 12288, 4, 0.02, "tflops"),
}
# One SeededRng seed per config (the draw of X then W).
SEEDS = {"cfg1": 1, "cfg2": 2, "cfg3": 3, "cfg5": 5}
DESCR = {
    "cfg1": "config 1: X bf16[1024,3072] . W[3072,3072]^T, W4 g64",
    "cfg2": "config 2: X bf16[4096,12288] . W[3072,12288]^T, W8 g64 (Flux MLP down-proj at 1024^2)",
    "cfg3": "config 3: X bf16[8,3072] . W[18432,3072]^T, W4 g64 (adaLN modulation, small-M)",
    "cfg5": "config 5: X bf16[16384,3072] . W[12288,3072]^T, W4 g64",
}


# B200 L2 (126 MB): the timed steps rotate over inputs that exceed it twice.
L2_BYTES = 126 * 1024 * 1024


def algorithmic(m, k, n, bits, world=1):
    """(flops, bytes) of one step on one rank: 2*M*N*K, and packed W + S + B + X + Y (each once)."""
    flops = 2.0 * m * n * k
    byts = n * k * bits / 8 + 2 * n * (k // 64) * 2 + m * k * 2 + m * n * 2
    return flops, byts


def peaks(sustained=False):
    """(HBM GB/s, bf16 TFLOP/s, source).  The burst bf16 figure suits a kernel timed alone; a
    step of tens of milliseconds runs under the power cap and is held to the sustained one."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        tc = p.get("bf16_tflops_sustained", p["bf16_tflops"]) if sustained else p["bf16_tflops"]
        return p["hbm_gbs"], tc, "measured"
    except Exception:
        return 6650.0, 1400.0 if sustained else 1590.0, "fallback"


def traffic_from_profiles(workload):
    """Per-launch DRAM bytes of the dominant kernel from a committed ncu summary, if any."""
    path = os.path.join(ROOT, "profiles", f"traffic_{workload}.txt")
    try:
        for line in open(path):
            if line.startswith("traffic_bytes_per_launch:"):
                return float(line.split(":", 1)[1])
    except OSError:
        pass
    return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.out = out
        else:
            self.out = ""

    def summary(self):
        rows = [r.split(", ") for r in self.out.strip().splitlines() if r.count(",") >= 8]
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = max(float(r[2]) for r in rows if r[2].replace(".", "").isdigit())
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].strip() == "Active"})
        load = [v for v in sm if v > 0.5 * mx] or sm
        return {"sm_mhz": statistics.median(load), "sm_max_mhz": mx, "reasons": reasons,
                "samples": len(rows)}


def cpu_reference(args, wl):
    """The reference's algorithm on the host cores: the oracle port (the reference's MLX CPU
    backend is not installable here), on a bounded sample of the workload's rows."""
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    if wl == "cfg4":
        return cpu_reference_flux(args, O)
    if wl == "encoders":
        sys.path.insert(0, os.path.join(ROOT, "stable-diffusion.rs_b200"))
        from sdq import encoders as E
        shapes = sorted({(n, k, 4) for e in E.ENCODERS for _, n, k, _ in E.layer_linears(e, 512)})
        return cpu_reference_shapes(args, O, shapes, "text-encoder linear shapes (W4)")
    m, k, n, bits, sig, kind = WORKLOADS[wl]
    threads = O.max_threads()
    ms = min(m, 8 if kind == "gbs" else 48)     # sample rows of X per step
    ns = n if kind == "gbs" else min(n, 3072)
    xb, w = O.synthetic_linear(1234, ms, k, ns, sig)
    wq, s, b = O.quantize(w, bits)
    for _ in range(max(1, args.warmup // 3)):
        O.qmatmul(xb, wq, s, b, ns, bits, threads=threads)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        O.qmatmul(xb, wq, s, b, ns, bits, threads=threads)
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    flops, byts = algorithmic(ms, k, ns, bits)
    value = (flops / t / 1e12) if kind == "tflops" else (byts / t / 1e9)
    sample = f"X rows {ms} of {m}, W rows {ns} of {n}, K={k}, W{bits}; median of {len(times)}"
    return value, threads, sample


def cpu_reference_flux(args, O):
    """The oracle over a sample of the Flux stack's linears: 16 rows of X through each distinct
    linear shape of a double block, a single block and a modulation, in TFLOP/s."""
    shapes = [(9216, 3072, 4), (3072, 3072, 8), (12288, 3072, 4), (3072, 12288, 8),
              (21504, 3072, 4), (3072, 15360, 8), (18432, 3072, 4)]
    return cpu_reference_shapes(args, O, shapes, "Flux linear shapes (W4/W8)")


def cpu_reference_shapes(args, O, shapes, label):
    """16 rows of X through each (N, K, bits) of ``shapes`` on all host threads, in TFLOP/s."""
    threads = O.max_threads()
    ms = 16
    cases = []
    for i, (n, k, bits) in enumerate(shapes):
        xb, w = O.synthetic_linear(500 + i, ms, k, n, 1.0 / k ** 0.5)
        cases.append((xb, O.quantize(w, bits), n, bits, 2.0 * ms * n * k))
    times = []
    for it in range(1 + args.steps):
        t0 = time.perf_counter()
        for xb, (wq, s, b), n, bits, _ in cases:
            O.qmatmul(xb, wq, s, b, n, bits, threads=threads)
        if it:
            times.append(time.perf_counter() - t0)
    flops = sum(c[4] for c in cases)
    t = statistics.median(times)
    sample = f"16 rows of X through each of {len(shapes)} {label}; median of {len(times)}"
    return flops / t / 1e12, threads, sample


def run_flux(args, rank, world, local):
    """Config 4: one forward of the Flux-shaped stack, every linear through libsdq.  N > 1 runs
    independent replicas (the stack does not shard here); the time is the max over ranks."""
    import torch
    import sdq
    from sdq import flux

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream()
    cfg = flux.FluxShape()
    total_flops = flux.flops(cfg)
    qw = flux.random_weights(cfg, seed=11, device=dev)
    rope = flux.rope_tables(cfg, device=dev)
    ins = flux.inputs(cfg, seed=12, device=dev)
    lin = flux.LinearsOnly(qw, cfg, seed=13, device=dev)
    flush = torch.empty(256 * 1024 * 1024 // 4, device=dev, dtype=torch.float32)

    def barrier():
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    # warm-up eagerly (first calls configure every kernel variant), then capture both passes
    for _ in range(args.warmup):
        lin()
        flux.forward(qw, *ins, cfg, rope)
    sdq.device_status()
    # The same forward with each linear's elementwise consumers run op by op (the reference's
    # way), to show what the fused output stage saves.
    from sdq.quantized import OpByOp
    opw = OpByOp(qw)
    flux.forward(opw, *ins, cfg, rope)
    g_lin, g_fwd, g_op = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_lin):
        lin()
    with torch.cuda.graph(g_fwd):
        out = flux.forward(qw, *ins, cfg, rope)
    with torch.cuda.graph(g_op):
        flux.forward(opw, *ins, cfg, rope)
    for _ in range(2):
        g_lin.replay()
        g_fwd.replay()
        g_op.replay()
    barrier()
    sdq.device_status()

    def timed(fn, steps):
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        for i in range(steps):
            flush.zero_()
            ev[i][0].record(stream)
            fn()
            ev[i][1].record(stream)
        barrier()
        t = sum(a.elapsed_time(b) for a, b in ev)
        if dist is not None:
            tt = torch.tensor([t], device=dev)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            t = float(tt.item())
        return t / steps

    with ClockSampler(local) as clk:
        lin_ms = timed(g_lin.replay, args.steps)
    fwd_ms = timed(g_fwd.replay, args.steps)
    op_ms = timed(g_op.replay, args.steps)
    sdq.device_status()
    del g_op

    # end to end: the eager forward through the public API with host inputs and output
    hosts = [t.cpu().pin_memory() for t in ins]
    devs = [torch.empty_like(t) for t in ins]
    oh = torch.empty(tuple(out.shape), dtype=out.dtype, pin_memory=True)

    def e2e_step():
        for d, h in zip(devs, hosts):
            d.copy_(h, non_blocking=True)
        o = flux.forward(qw, *devs, cfg, rope)
        oh.copy_(o, non_blocking=True)

    for _ in range(2):
        e2e_step()
    e2e_ms = timed(e2e_step, max(2, args.steps // 2))

    value = total_flops * world / (lin_ms * 1e-3) / 1e12
    hbm, tc, src = peaks(sustained=True)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cv, threads, sample = cpu_reference(argparse.Namespace(steps=3, warmup=3), "cfg4")
        cpu = {"value": cv, "unit": "TFLOP/s", "cores": threads, "kind": "port", "sample": sample}
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        achieved = total_flops / (lin_ms * 1e-3) / 1e12
        print(json.dumps({
            "metric": "qmatmul_tflops", "value": value, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": lin_ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded random-init Flux-shaped weights, quantised by libsdq)",
            "config": {"workload": "cfg4",
                       "descr": "config 4: Flux-schnell-shaped stack, 19 double + 38 single blocks, "
                                "512 txt + 4096 img tokens, hidden 3072, out-proj/MLP-down W8, rest W4; "
                                "gate/residual and GELU/SiLU fused into the linears' output stage",
                       "linears": len(flux.linear_table(cfg)), "qmm_tflop_per_forward": total_flops / 1e12,
                       "packed_weight_bytes": qw.resident_bytes(),
                       "forward_ms": fwd_ms, "qmm_share_of_forward": lin_ms / fwd_ms,
                       "forward_op_by_op_ms": op_ms,
                       "parallelism": "single GPU" if world == 1 else f"{world} replicas",
                       "l2": "weights (8.5 GB) exceed L2; 256 MiB write before every step anyway"},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": tc, "unit": "TFLOP/s",
                         "frac": achieved / tc, "peak_source": f"{src} sustained bf16 (MEASURED_PEAKS.json)",
                         "traffic": None, "kernel_ms": lin_ms},
            "cpu_baseline": cpu,
            "e2e": {"value": total_flops * world / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                    "ms_per_step": e2e_ms,
                    "h2d_bytes_per_step": sum(t.numel() * t.element_size() for t in ins),
                    "d2h_bytes_per_step": out.numel() * out.element_size(),
                    "path": "sdq.flux.forward (every linear through the C ABI), host inputs in, output out"},
            "gpu_launches": args.steps * len(flux.linear_table(cfg)),
            "clocks": clk.summary(),
        }))


def run_encoders(args, rank, world, local):
    """The text encoders' layers (T5-XXL, Qwen3-4B, Qwen2.5-VL-7B, Mistral Small 3.2; W4) at 512
    prompt tokens: one layer's linears per encoder, each encoder's set captured in a CUDA graph.
    N > 1 runs independent replicas; the time is the max over ranks."""
    import torch
    import sdq
    from sdq import encoders as E

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream()
    tokens, bits = 512, 4
    g = torch.Generator(device=dev).manual_seed(21)
    flush = torch.empty(256 * 1024 * 1024 // 4, device=dev, dtype=torch.float32)
    sets = []
    for e in E.ENCODERS:
        calls = []
        for name, n, k, m in E.layer_linears(e, tokens):
            wq, s, b = sdq.quantize(torch.randn(n, k, device=dev, generator=g) * 0.02, 64, bits)
            x = torch.randn(m, k, device=dev, generator=g).to(torch.bfloat16)
            calls.append((x, wq, s, b, torch.empty(m, n, device=dev, dtype=torch.bfloat16)))
        sets.append((e, calls, E.flops(E.layer_linears(e, tokens))))

    def run(calls):
        for x, wq, s, b, y in calls:
            sdq.quantized_matmul(x, wq, s, b, 64, bits, out=y)

    graphs = []
    for e, calls, fl in sets:
        for _ in range(args.warmup):
            run(calls)
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            run(calls)
        graphs.append(gr)
    sdq.device_status()

    def barrier():
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    def timed(fn, steps):
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        for i in range(steps):
            flush.zero_()
            ev[i][0].record(stream)
            fn()
            ev[i][1].record(stream)
        barrier()
        t = sum(a.elapsed_time(b) for a, b in ev)
        if dist is not None:
            tt = torch.tensor([t], device=dev)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            t = float(tt.item())
        return t / steps

    def all_layers():
        for gr in graphs:
            gr.replay()

    barrier()
    with ClockSampler(local) as clk:
        step_ms = timed(all_layers, args.steps)
    per = {e.name: {"ms": timed(gr.replay, args.steps), "gflop": fl / 1e9}
           for (e, _, fl), gr in zip(sets, graphs)}
    for v in per.values():
        v["tflops"] = v["gflop"] / v["ms"]
    sdq.device_status()
    total = sum(fl for _, _, fl in sets)

    # end to end: each layer's input from pinned host memory, its last output back, eager calls
    hosts = [[c[0].cpu().pin_memory() for c in calls] for _, calls, _ in sets]
    outs = [torch.empty(tuple(calls[-1][4].shape), dtype=torch.bfloat16, pin_memory=True) for _, calls, _ in sets]

    def e2e_step():
        for (_, calls, _), hs, oh in zip(sets, hosts, outs):
            for c, h in zip(calls, hs):
                c[0].copy_(h, non_blocking=True)
            run(calls)
            oh.copy_(calls[-1][4], non_blocking=True)

    e2e_step()
    e2e_ms = timed(e2e_step, args.steps)
    hbm, tc, src = peaks()
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cv, threads, sample = cpu_reference(argparse.Namespace(steps=3, warmup=3), "encoders")
        cpu = {"value": cv, "unit": "TFLOP/s", "cores": threads, "kind": "port", "sample": sample}
    del graphs
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        achieved = total / (step_ms * 1e-3) / 1e12
        print(json.dumps({
            "metric": "qmatmul_tflops", "value": total * world / (step_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded random-init weights of each encoder's shapes, quantised by libsdq)",
            "config": {"workload": "encoders",
                       "descr": "one layer's linears of T5-XXL, Qwen3-4B, Qwen2.5-VL-7B and Mistral Small 3.2 "
                                "at 512 prompt tokens, W4 g64",
                       "per_encoder": per, "tokens": tokens,
                       "parallelism": "single GPU" if world == 1 else f"{world} replicas",
                       "l2": "256 MiB write before every step"},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": tc, "unit": "TFLOP/s",
                         "frac": achieved / tc, "peak_source": f"{src} burst bf16 (MEASURED_PEAKS.json)",
                         "traffic": None, "kernel_ms": step_ms},
            "cpu_baseline": cpu,
            "e2e": {"value": total * world / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": e2e_ms,
                    "h2d_bytes_per_step": sum(h.numel() * 2 for hs in hosts for h in hs),
                    "d2h_bytes_per_step": sum(o.numel() * 2 for o in outs),
                    "path": "sdq.quantized_matmul per linear, inputs from and last output to pinned host"},
            "gpu_launches": args.steps * sum(len(c) for _, c, _ in sets),
            "clocks": clk.summary(),
        }))


def _draw(wl_seed, m, k, n_total, sig, rank_rows, dev):
    """The benchmark's inputs: the reference's SeededRng draw (X first, then the whole W), X
    rounded to bf16 and the W rows [lo, hi) quantised by the library."""
    import torch
    import sdq
    lo, hi = rank_rows
    vals = sdq.seeded_normals(wl_seed, m * k + n_total * k, device=dev)
    x = (vals[: m * k] * 1.0).view(m, k).to(torch.bfloat16)
    w = (vals[m * k + lo * k: m * k + hi * k] * sig).view(hi - lo, k)
    return x, w.contiguous()


def measure_single(name, m, k, n, bits, sig, seed, steps, warmup, dev, local):
    """One workload on one GPU, as the headline is measured: K launches back to back over
    rotating input copies larger than twice L2, replayed as one CUDA graph between one pair
    of events, with clocks sampled meanwhile.  Returns the per-workload record of the
    `secondary` block."""
    import torch
    import sdq
    kind = "tflops" if m > 8 else "gbs"
    x, w = _draw(seed, m, k, n, sig, (0, n), dev)
    wq, s, b = sdq.quantize(w, 64, bits)
    del w
    set_bytes = m * k * 2 + wq.numel() * 4 + (s.numel() + b.numel()) * 2 + m * n * 2
    rot = int(min(16, max(2, -(-2 * L2_BYTES // set_bytes))))
    sets = [(x, wq, s, b)] + [(x.clone(), wq.clone(), s.clone(), b.clone()) for _ in range(rot - 1)]
    ys = [torch.empty((m, n), device=dev, dtype=torch.bfloat16) for _ in range(rot)]

    def step(i):
        xi, wqi, si, bi = sets[i % rot]
        sdq.quantized_matmul(xi, wqi, si, bi, 64, bits, out=ys[i % rot])

    for i in range(max(warmup, rot)):
        step(i)
    sdq.device_status()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for i in range(steps):
            step(i)
    graph.replay()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        ev0.record(stream)
        graph.replay()
        ev1.record(stream)
        torch.cuda.synchronize()
    sdq.device_status()
    ms = ev0.elapsed_time(ev1) / steps
    flops, byts = algorithmic(m, k, n, bits)
    hbm, tc, src = peaks()
    if kind == "tflops":
        value, unit, peak = flops / (ms * 1e-3) / 1e12, "TFLOP/s", tc
    else:
        value, unit, peak = byts / (ms * 1e-3) / 1e9, "GB/s", hbm
    del graph, sets, ys
    torch.cuda.empty_cache()
    return {"workload": name, "M": m, "K": k, "N": n, "bits": bits, "value": value, "unit": unit,
            "kernel_ms": ms, "bound": "tensor" if kind == "tflops" else "hbm", "peak": peak,
            "frac": value / peak, "peak_source": f"{src} ({'burst bf16' if kind == 'tflops' else 'copy bandwidth'}, MEASURED_PEAKS.json)",
            "rotating_input_sets": rot, "clocks": clk.summary()}


def secondary_workloads(args, dev, local):
    """The rest of the benchmark plan's metric beside the headline: config 1 (W4, TFLOP/s),
    config 3 at every M it names (W4, HBM GB/s), config 5 on one GPU (W4, TFLOP/s)."""
    out = []
    for name, (m, k, n, bits, sig, _) in (("cfg1", WORKLOADS["cfg1"]), ("cfg5", WORKLOADS["cfg5"])):
        out.append(measure_single(name, m, k, n, bits, sig, SEEDS[name], args.steps, args.warmup, dev, local))
    m3, k3, n3, b3, s3, _ = WORKLOADS["cfg3"]
    for m in (1, 2, 4, 8):
        out.append(measure_single(f"cfg3_m{m}", m, k3, n3, b3, s3, SEEDS["cfg3"], args.steps, args.warmup, dev, local))
    return out


def strong_scaling_cfg5(args, rank, world, dev, comm, dist):
    """Config 5 as specified: one fixed layer (X [16384, 3072], W [12288, 3072] W4) split over
    the ranks along N.  Returns the GEMM-only time (each rank's shard, no exchange) and the
    GEMM + exchange time (the sharded call, its output assembled on every rank), max over
    ranks, with the aggregate TFLOP/s of the whole layer."""
    import torch
    import sdq
    m, k, n_total, bits, sig, _ = WORKLOADS["cfg5"]
    if n_total % world:
        return None
    nl = n_total // world
    x, w = _draw(SEEDS["cfg5"], m, k, n_total, sig, (rank * nl, (rank + 1) * nl), dev)
    wq, s, b = sdq.quantize(w, 64, bits)
    del w
    y_local = torch.empty((m, nl), device=dev, dtype=torch.bfloat16)
    y_shards = torch.empty((world, m, nl), device=dev, dtype=torch.bfloat16)
    y_full = comm.output(m, n_total) if comm is not None else torch.empty((m, n_total), device=dev, dtype=torch.bfloat16)
    stream = torch.cuda.current_stream()

    def timed(fn, steps):
        for _ in range(max(3, args.warmup)):
            fn()
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        t = e0.elapsed_time(e1) / steps
        if dist is not None:
            tt = torch.tensor([t], device=dev)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            t = float(tt.item())
        return t

    gemm_ms = timed(lambda: sdq.quantized_matmul(x, wq, s, b, 64, bits, out=y_local), args.steps)
    if comm is not None:
        total_ms = timed(lambda: sdq.quantized_matmul_sharded(x, wq, s, b, comm, 64, bits, y_shards=y_shards,
                                                              out=y_full), args.steps)
    else:
        total_ms = gemm_ms
    sdq.device_status()
    flops = 2.0 * m * n_total * k
    hbm, tc, src = peaks()
    del x, wq, s, b, y_local, y_shards
    torch.cuda.empty_cache()
    return {"workload": "cfg5 strong scaling", "M": m, "K": k, "N_total": n_total, "N_per_rank": nl, "bits": bits,
            "ranks": world, "gemm_ms": gemm_ms, "gemm_tflops": flops / (gemm_ms * 1e-3) / 1e12,
            "gemm_plus_exchange_ms": total_ms, "gemm_plus_exchange_tflops": flops / (total_ms * 1e-3) / 1e12,
            "exchange_bytes_received_per_rank": (world - 1) * m * nl * 2,
            "frac_of_world_peak_gemm": flops / (gemm_ms * 1e-3) / 1e12 / (tc * world),
            "peak_source": f"{src} burst bf16 x ranks",
            "timing": "eager calls back to back, events on the launching stream, max over ranks"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="cfg2", choices=sorted(list(WORKLOADS) + ["cfg4", "encoders"]))
    ap.add_argument("--impl", default="sdq", choices=["sdq", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-secondary", action="store_true",
                    help="skip the secondary workloads (configs 1, 3, 5) of the default line")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    wl = args.workload
    kind = "tflops" if wl in ("cfg4", "encoders") else WORKLOADS[wl][5]
    metric = "qmatmul_tflops" if kind == "tflops" else "qmatmul_hbm_gbs"
    unit = "TFLOP/s" if kind == "tflops" else "GB/s"

    if args.impl == "reference":
        if rank != 0:
            return
        value, threads, sample = cpu_reference(args, wl)
        print(json.dumps({
            "impl": "reference", "metric": metric, "value": value, "unit": unit, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (SeededRng)",
            "config": {"workload": wl, "descr": DESCR.get(wl, "config 4: Flux-shaped stack" if wl == "cfg4"
                                                          else "text-encoder layers at 512 tokens"),
                       "parallelism": "host threads"},
            "cpu_baseline": {"value": value, "unit": unit, "cores": threads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }))
        return
    if wl == "cfg4":
        return run_flux(args, rank, world, local)
    if wl == "encoders":
        return run_encoders(args, rank, world, local)
    m, k, n, bits, sig, kind = WORKLOADS[wl]

    import torch
    import sdq

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream()

    # ---- data: the reference's documented draw (SeededRng, one seed per config): X first, then
    # the whole [world*n, k] W, each N(0, 1) scaled by sigma; X rounded to bf16, W kept f32 and
    # quantised by the library.  Every rank draws the same sequence and keeps its W rows
    # rank*n .. rank*n + n.
    vals = sdq.seeded_normals(SEEDS[wl], m * k + world * n * k, device=dev)
    x = (vals[: m * k] * 1.0).view(m, k).to(torch.bfloat16)
    w = (vals[m * k + rank * n * k: m * k + (rank + 1) * n * k] * sig).view(n, k)
    wq, s, b = sdq.quantize(w.contiguous(), 64, bits)
    del w, vals
    flush = torch.empty(256 * 1024 * 1024 // 4, device=dev, dtype=torch.float32)
    # The timed steps rotate over R copies of the inputs (X, packed W, scales, biases, Y) that
    # together exceed twice the L2, so that no step finds its inputs in L2 and the steps can
    # run back to back, as consecutive layers do, without a flush between them.
    set_bytes = m * k * 2 + wq.numel() * 4 + (s.numel() + b.numel()) * 2 + m * n * 2
    rot = int(min(16, max(2, -(-2 * L2_BYTES // set_bytes))))
    sets = [(x, wq, s, b)] + [(x.clone(), wq.clone(), s.clone(), b.clone()) for _ in range(rot - 1)]
    comm = None
    if world > 1:
        uid = [sdq.Comm.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        comm = sdq.Comm(uid[0], world, rank)
        y_shards = torch.empty((world, m, n), device=dev, dtype=torch.bfloat16)
        # The communicator's symmetric output: the peers' blocks land in place (no final copy).
        y_full = comm.output(m, world * n)
    y = torch.empty((m, n), device=dev, dtype=torch.bfloat16)
    ys = [y] + [torch.empty_like(y) for _ in range(rot - 1)]

    def step(i=0):
        xi, wqi, si, bi = sets[i % rot]
        if comm is None:
            sdq.quantized_matmul(xi, wqi, si, bi, 64, bits, out=ys[i % rot])
        else:
            sdq.quantized_matmul_sharded(xi, wqi, si, bi, comm, 64, bits, y_shards=y_shards, out=y_full)

    def barrier():
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    for i in range(max(args.warmup, rot)):
        step(i)
    sdq.device_status()

    # ---- device-resident timing (value): K steps back to back over the rotating inputs,
    # one pair of CUDA events around them on the launching stream.  On one GPU the K steps are
    # captured in a CUDA graph first, so that the host's per-call cost (argument checks,
    # tensor-map encoding, launch) does not starve the short kernels; the graph replays the
    # same K kernel launches.
    graph = None
    if comm is None:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for i in range(args.steps):
                step(i)
        graph.replay()
        torch.cuda.synchronize()

    def timed_steps():
        if graph is not None:
            graph.replay()
        else:
            for i in range(args.steps):
                step(i)

    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    with ClockSampler(local) as clk:
        ev0.record(stream)
        timed_steps()
        ev1.record(stream)
        barrier()
    sdq.device_status()
    total_ms = ev0.elapsed_time(ev1)
    if dist is not None:
        t = torch.tensor([total_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
    ms_per_step = total_ms / args.steps

    # ---- the dominant kernel alone (for the roofline): at N = 1 it is the whole step
    if comm is None:
        kern_ms = [ms_per_step]
    else:
        kev0, kev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        kev0.record(stream)
        for i in range(args.steps):
            xi, wqi, si, bi = sets[i % rot]
            sdq.quantized_matmul(xi, wqi, si, bi, 64, bits, out=ys[i % rot])
        kev1.record(stream)
        torch.cuda.synchronize()
        kern_ms = [kev0.elapsed_time(kev1) / args.steps]

    flops, byts = algorithmic(m, k, n, bits)
    if kind == "tflops":
        value = flops * world / (ms_per_step * 1e-3) / 1e12
    else:
        value = byts * world / (ms_per_step * 1e-3) / 1e9

    # ---- end to end through the public API with host buffers
    xh = torch.empty((m, k), dtype=torch.bfloat16, pin_memory=True)
    xh.copy_(x.cpu())
    yh = torch.empty((m, n * world), dtype=torch.bfloat16, pin_memory=True)
    xd = torch.empty_like(x)
    # N > 1: X and Y cross the host link once per step between them: each rank uploads its
    # 1/N of X's rows, NCCL gathers X over NVLink, and each rank reads back its 1/N of the
    # gathered Y's rows (every rank holds the whole Y on the device).
    split = comm is not None and m % world == 0
    rows = m // world if split else m
    xpart = torch.empty((rows, k), device=dev, dtype=torch.bfloat16) if split else None
    e2e_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(args.steps)]
    for i in range(args.warmup + args.steps):
        flush.zero_()
        if i >= args.warmup:
            e2e_ev[i - args.warmup][0].record(stream)
        if comm is None:
            # One call: upload, product and download of row chunks overlap inside it.
            sdq.quantized_matmul_host(xh, wq, s, b, 64, bits, out=yh, x_dev=xd, y_dev=y)
        elif split:
            xpart.copy_(xh[rank * rows:(rank + 1) * rows], non_blocking=True)
            dist.all_gather_into_tensor(xd, xpart)
            sdq.quantized_matmul_sharded(xd, wq, s, b, comm, 64, bits, y_shards=y_shards, out=y_full)
            yh[rank * rows:(rank + 1) * rows].copy_(y_full[rank * rows:(rank + 1) * rows], non_blocking=True)
        else:
            xd.copy_(xh, non_blocking=True)
            sdq.quantized_matmul_sharded(xd, wq, s, b, comm, 64, bits, y_shards=y_shards, out=y_full)
            yh.copy_(y_full, non_blocking=True)
        if i >= args.warmup:
            e2e_ev[i - args.warmup][1].record(stream)
    barrier()
    e2e_ms = sum(a.elapsed_time(bb) for a, bb in e2e_ev)
    if dist is not None:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_step = e2e_ms / args.steps
    e2e_value = (flops if kind == "tflops" else byts) * world / (e2e_step * 1e-3) / (1e12 if kind == "tflops" else 1e9)

    # ---- roofline of the dominant kernel (the qmm kernel, CUDA events around its launches)
    hbm, tc, src = peaks()
    kern_avg = sum(kern_ms) / len(kern_ms)
    if kind == "tflops":
        achieved = flops / (kern_avg * 1e-3) / 1e12
        roof = {"bound": "tensor", "achieved": achieved, "peak": tc, "unit": "TFLOP/s",
                "frac": achieved / tc, "peak_source": f"{src} burst bf16 (MEASURED_PEAKS.json)"}
    else:
        achieved = byts / (kern_avg * 1e-3) / 1e9
        roof = {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                "frac": achieved / hbm, "peak_source": f"{src} copy bandwidth (MEASURED_PEAKS.json)"}
    roof["traffic"] = traffic_from_profiles(wl)
    roof["kernel_ms"] = kern_avg

    # The rest of the metric: configs 1, 3 (M = 1, 2, 4, 8) and 5 on one GPU beside the
    # headline; config 5's strong-scaling split on every run (one GPU: the GEMM alone).
    secondary = None
    if world == 1 and wl == "cfg2" and not args.no_secondary:
        graph = None        # the timed graph is not replayed again: its rotating copies can go
        del sets, ys
        torch.cuda.empty_cache()
        secondary = secondary_workloads(args, dev, local)
    strong = None
    if wl == "cfg2" and not args.no_secondary:
        strong = strong_scaling_cfg5(args, rank, world, dev, comm, dist)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cv, threads, sample = cpu_reference(argparse.Namespace(steps=3, warmup=3), wl)
        cpu = {"value": cv, "unit": unit, "cores": threads, "kind": "port", "sample": sample}

    if comm is not None:
        comm.destroy()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()

    if rank == 0:
        line = {
            "metric": metric, "value": value, "unit": unit, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (SeededRng: splitmix64 + Box-Muller, the reference's documented draw; X then W; W quantised by libsdq)",
            "config": {"workload": wl, "descr": DESCR[wl], "M": m, "K": k, "N_per_rank": n, "bits": bits,
                       "group_size": 64, "global_N": n * world,
                       "parallelism": "single GPU" if world == 1 else
                           f"N-sharded x{world}; the kernel's epilogue stores each output tile into every peer's output over NVLink",
                       "l2": f"inputs larger than L2: steps rotate over {rot} copies of X, W, scales, "
                             f"biases and Y ({rot * set_bytes / 1e6:.0f} MB, L2 {L2_BYTES / 1e6:.0f} MB), "
                             "back to back between one event pair"
                             + (" (the K steps replayed as one CUDA graph)" if world == 1 else ""),
                       "rotating_input_sets": rot},
            "roofline": roof,
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": unit, "ms_per_step": e2e_step,
                    "h2d_bytes_per_step": m * k * 2 * (1 if split or world == 1 else world),
                    "d2h_bytes_per_step": m * n * world * 2 * (1 if split or world == 1 else world),
                    "path": ("sdq.quantized_matmul_host (C ABI): pinned host X in, host Y out, row chunks "
                             "uploaded, multiplied and downloaded in overlap" if world == 1 else
                             "each rank uploads 1/N of X's rows from pinned host memory, NCCL all-gathers X, "
                             "sdq.quantized_matmul_sharded (C ABI), each rank reads back 1/N of the gathered "
                             "Y's rows; bytes are the job's totals" if split else
                             "sdq.quantized_matmul_sharded (C ABI) with pinned host X in, Y out on every rank")},
            # N > 1: the fused path (M > 8) runs the tensor-core kernel, which also stores its
            # tiles into the peers' outputs, and the one-thread wait for the peers' tiles;
            # M <= 8 runs the small-M kernel and the permute (plus NCCL's all-gather).
            "gpu_launches": args.steps * (1 if world == 1 else 2),
            "clocks": clk.summary(),
        }
        if secondary is not None:
            line["secondary"] = secondary
        if strong is not None:
            line["strong_scaling"] = strong
        print(json.dumps(line))


if __name__ == "__main__":
    main()
