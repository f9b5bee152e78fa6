"""Benchmark of the xb200 operator set on B200.

Default workload (N=1): the elementwise / activation suite on flat tensors of
2^28 elements, x, y ~ N(0, 1) from a seed -- vec-add, axpy (alpha 2.5), relu,
leaky_relu (0.01), gelu (tanh form), sigmoid, silu in bf16 and fp32, swiglu
on 2^27 + 2^27, and 2x2 / stride-2 average pooling of a [64, 256, 224, 224]
fp32 tensor.  One step = one pass of every operator over its inputs
(17 kernel launches).  Every input is larger than L2 (126 MB), so no flush is
needed between steps.

Metric: algorithmic HBM bytes (each input read once, each output written
once) per second, aggregated over the step and over all ranks.

Contract:  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl xb200|reference]
Multi-GPU (torchrun, one rank per GPU): every rank runs its own full suite
(weak scaling, no data-path collective); the time is the max over ranks.
``--impl reference`` times the examples' PyTorch CPU expressions (the oracle
port of the reference's CPU path) on the host cores.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "triton-xdna_b200"))

N28 = 1 << 28
N27 = 1 << 27
POOL_SHAPE = (64, 256, 224, 224)


def _peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d["hbm_gbs"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


# ----------------------------------------------------------------------------- workload


def suite_ops():
    """(name, dtype, n_in_elems, n_out_elems, elem_bytes) for each launch of a step."""
    out = []
    for dt, eb in ((torch.bfloat16, 2), (torch.float32, 4)):
        tag = "bf16" if dt == torch.bfloat16 else "f32"
        out += [
            (f"vecadd_{tag}", dt, 2 * N28, N28, eb),
            (f"axpy_{tag}", dt, 2 * N28, N28, eb),
            (f"relu_{tag}", dt, N28, N28, eb),
            (f"leaky_relu_{tag}", dt, N28, N28, eb),
            (f"gelu_tanh_{tag}", dt, N28, N28, eb),
            (f"sigmoid_{tag}", dt, N28, N28, eb),
            (f"silu_{tag}", dt, N28, N28, eb),
            (f"swiglu_{tag}", dt, 2 * N27, N27, eb),
        ]
    n_in = 1
    for s in POOL_SHAPE:
        n_in *= s
    out.append(("avg_pool2d_2x2_f32", torch.float32, n_in, n_in // 4, 4))
    return out


def op_bytes(op) -> int:
    _, _, nin, nout, eb = op
    return (nin + nout) * eb


class DeviceSuite:
    """Device-resident inputs/outputs and the launch sequence of one step."""

    def __init__(self, device, seed: int = 0):
        from xb200 import ops

        self.ops = ops
        g = torch.Generator(device=device).manual_seed(seed)
        self.t = {}
        for dt in (torch.bfloat16, torch.float32):
            x = torch.randn(N28, generator=g, device=device, dtype=torch.float32).to(dt)
            y = torch.randn(N28, generator=g, device=device, dtype=torch.float32).to(dt)
            self.t[dt] = (x, y, torch.empty_like(x))
        self.pool_in = torch.randn(POOL_SHAPE, generator=g, device=device, dtype=torch.float32)
        self.pool_out = torch.empty(POOL_SHAPE[:2] + (POOL_SHAPE[2] // 2, POOL_SHAPE[3] // 2), device=device)

    def run(self, name):
        o = self.ops
        if name.startswith("avg_pool2d"):
            o.avg_pool2d_2x2(self.pool_in, out=self.pool_out)
            return
        dt = torch.bfloat16 if name.endswith("bf16") else torch.float32
        x, y, out = self.t[dt]
        base = name.rsplit("_", 1)[0]
        if base == "vecadd":
            o.vecadd(x, y, out=out)
        elif base == "axpy":
            o.axpy(x, y, 2.5, out=out)
        elif base == "relu":
            o.relu(x, out=out)
        elif base == "leaky_relu":
            o.leaky_relu(x, 0.01, out=out)
        elif base == "gelu_tanh":
            o.gelu_tanh(x, out=out)
        elif base == "sigmoid":
            o.sigmoid(x, out=out)
        elif base == "silu":
            o.silu(x, out=out)
        elif base == "swiglu":
            o.swiglu(x[:N27], y[:N27], out=out[:N27])
        else:
            raise KeyError(name)


# ----------------------------------------------------------------------------- clocks


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms in the background."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = None

    def __enter__(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if self.proc is None or not self.path or not os.path.exists(self.path):
            return None
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        os.unlink(self.path)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": smax, "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------------------- distributed helpers


def _dist_init():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return world, rank, local


def _barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def _max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ----------------------------------------------------------------------------- CPU baseline


def cpu_suite(sample_elems: int, reps: int = 1):
    """Time the oracle (examples' torch CPU expressions) on a bounded sample of
    the suite; returns (GB/s, seconds, threads, description)."""
    sys.path.insert(0, ROOT)
    from oracle import ops as O

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    frac = sample_elems / N28
    g = torch.Generator().manual_seed(0)
    total_bytes = 0
    total_s = 0.0
    pool_planes = max(1, int(POOL_SHAPE[0] * POOL_SHAPE[1] * frac))
    for op in suite_ops():
        name, dt, nin, nout, eb = op
        if name.startswith("avg_pool"):
            x = torch.randn((pool_planes, POOL_SHAPE[2], POOL_SHAPE[3]), generator=g)
            fn = lambda: O.avg_pool2d_2x2(x)  # noqa: E731
            nbytes = x.numel() * 4 * 5 // 4
        else:
            n = max(1024, int(nout * frac))
            x = torch.randn(n, generator=g).to(dt)
            y = torch.randn(n, generator=g).to(dt)
            base = name.rsplit("_", 1)[0]
            fn = {
                "vecadd": lambda: O.vecadd(x, y), "axpy": lambda: O.axpy(x, y, 2.5), "relu": lambda: O.relu(x),
                "leaky_relu": lambda: O.leaky_relu(x, 0.01), "gelu_tanh": lambda: O.gelu_tanh(x),
                "sigmoid": lambda: O.sigmoid(x), "silu": lambda: O.silu(x), "swiglu": lambda: O.swiglu(x, y),
            }[base]
            nbytes = (nin // nout + 1) * n * eb
        fn()  # warm-up
        best = None
        for _ in range(reps):
            t0 = time.perf_counter()
            fn()
            dt_s = time.perf_counter() - t0
            best = dt_s if best is None else min(best, dt_s)
        total_bytes += nbytes
        total_s += best
    desc = f"every suite operator on {sample_elems} elements ({frac:.4f} of the workload), min of {reps}"
    return total_bytes / total_s / 1e9, total_s, threads, desc


# ----------------------------------------------------------------------------- main


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="xb200", choices=["xb200", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=2)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--elements", type=int, default=1 << 28,
                    help="flat tensor length (default 2^28, the workload); smaller values are for profiling only")
    args = ap.parse_args()
    global N28, N27, POOL_SHAPE
    if args.elements != N28:
        N28 = args.elements
        N27 = N28 // 2
        POOL_SHAPE = (max(1, 64 * N28 // (1 << 28)),) + POOL_SHAPE[1:]
    warmup = max(3, args.warmup)

    world, rank, local = _dist_init() if args.impl == "xb200" else (
        int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")), 0)
    ops_list = suite_ops()
    step_bytes = sum(op_bytes(o) for o in ops_list)
    config = {
        "workload": "elementwise/activation suite: 8 ops x {bf16,f32} on 2^28 elements (swiglu 2^27+2^27) "
                    "+ avg_pool2d 2x2/s2 on [64,256,224,224] f32",
        "n_elements": N28,
        "launches_per_step": len(ops_list),
        "bytes_per_step": step_bytes,
        "l2": "every input > 126 MB L2 (no flush needed)",
        "parallelism": f"weak x{world} (independent replicas of the suite, no collective)",
    }

    if args.impl == "reference":
        if rank != 0:
            return
        sample = 1 << 22
        gbs, secs, threads, desc = cpu_suite(sample, reps=1)
        for _ in range(warmup - 1):
            pass
        vals = []
        for _ in range(args.steps):
            v, _, _, _ = cpu_suite(sample, reps=1)
            vals.append(v)
        value = statistics.median(vals)
        line = {
            "impl": "reference", "metric": "elementwise/activation suite algorithmic HBM throughput",
            "value": round(value, 3), "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": warmup,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16+f32",
            "data": "synthetic N(0,1), seed 0", "config": config,
            "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                             "sample": desc},
            "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }
        print(json.dumps(line))
        return

    from xb200 import _lib, kernels

    _lib.load()
    dev = torch.device("cuda", torch.cuda.current_device())
    suite = DeviceSuite(dev, seed=rank)
    stream = torch.cuda.current_stream()

    for _ in range(warmup):
        for o in ops_list:
            suite.run(o[0])
    torch.cuda.synchronize()

    # ---- timed region: K steps, per-launch CUDA events on the launching stream
    evs = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in ops_list]
           for _ in range(args.steps)]
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    _barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        start.record(stream)
        for s in range(args.steps):
            for i, o in enumerate(ops_list):
                evs[s][i][0].record(stream)
                suite.run(o[0])
                evs[s][i][1].record(stream)
        stop.record(stream)
        torch.cuda.synchronize()
    _barrier(world)
    total_ms = start.elapsed_time(stop)
    total_ms = _max_over_ranks(total_ms, world)
    clocks = clk.summary()

    per_op_ms = {o[0]: statistics.mean(evs[s][i][0].elapsed_time(evs[s][i][1]) for s in range(args.steps))
                 for i, o in enumerate(ops_list)}
    ms_per_step = total_ms / args.steps
    value = step_bytes * world / (ms_per_step * 1e-3) / 1e9
    peaks = _peaks()
    hbm = peaks["hbm_gbs"]
    dom = max(ops_list, key=lambda o: per_op_ms[o[0]])
    dom_gbs = op_bytes(dom) / (per_op_ms[dom[0]] * 1e-3) / 1e9
    suite_detail = {o[0]: {"ms": round(per_op_ms[o[0]], 4),
                           "gbs": round(op_bytes(o) / (per_op_ms[o[0]] * 1e-3) / 1e9, 1),
                           "frac": round(op_bytes(o) / (per_op_ms[o[0]] * 1e-3) / 1e9 / hbm, 3)} for o in ops_list}

    # ---- end to end through the public launch API with host (pinned) tensors
    e2e = None
    if rank == 0 and args.e2e_steps > 0:
        e2e = e2e_suite(kernels, dev, args.e2e_steps)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        gbs, secs, threads, desc = cpu_suite(1 << 24, reps=1)
        cpu = {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port", "sample": desc}

    if rank == 0:
        line = {
            "metric": "elementwise/activation suite algorithmic HBM throughput",
            "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": warmup,
            "ms_per_step": round(ms_per_step, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16+f32", "data": "synthetic N(0,1), seed = rank", "config": config,
            "roofline": {"bound": "hbm", "kernel": dom[0], "achieved": round(dom_gbs, 1), "peak": hbm,
                         "peak_source": peaks["source"], "unit": "GB/s", "frac": round(dom_gbs / hbm, 4),
                         "traffic": None},
            "suite": suite_detail,
            "e2e": e2e, "cpu_baseline": cpu, "clocks": clocks, "gpu_launches": len(ops_list) * args.steps,
        }
        print(json.dumps(line))
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


def e2e_suite(kernels, dev, steps: int):
    """Each op through xb200.kernels (the reference-signature launcher) on pinned
    host tensors: host->device copies of every pointer argument, the kernel,
    and the copy of the output back, all inside the timed region."""
    g = torch.Generator().manual_seed(0)
    host = {}
    for dt in (torch.bfloat16, torch.float32):
        x = torch.randn(N28, generator=g).to(dt).pin_memory()
        y = torch.randn(N28, generator=g).to(dt).pin_memory()
        host[dt] = (x, y, torch.empty_like(x).pin_memory())
    pin = torch.randn(POOL_SHAPE, generator=g).pin_memory()
    pout = torch.empty(POOL_SHAPE[:2] + (POOL_SHAPE[2] // 2, POOL_SHAPE[3] // 2)).pin_memory()
    pool_rows = POOL_SHAPE[0] * POOL_SHAPE[1]

    def one_step():
        h2d = d2h = 0
        for name, dt, nin, nout, eb in suite_ops():
            if name.startswith("avg_pool"):
                kernels.avg_pool2d_kernel[(pool_rows,)](pin, pout, POOL_SHAPE[0] * POOL_SHAPE[1], POOL_SHAPE[2],
                                                          POOL_SHAPE[3], BLOCK=1)
                h2d += (pin.numel() + pout.numel()) * 4
                d2h += pout.numel() * 4
                continue
            x, y, out = host[dt]
            base = name.rsplit("_", 1)[0]
            blk = {"BLOCK_SIZE": 1024}
            if base == "vecadd":
                kernels.vecadd[(N28 // 1024,)](x, y, out, N28, BLOCK_SIZE_N=1024)
                h2d += 3 * N28 * eb
            elif base == "axpy":
                kernels.axpy_kernel[(N28 // 1024,)](x, y, out, 2.5, N28, **blk)
                h2d += 3 * N28 * eb
            elif base == "swiglu":
                kernels.swiglu_kernel[(N27 // 1024,)](x[:N27], y[:N27], out[:N27], N27, **blk)
                h2d += 3 * N27 * eb
            else:
                k = {"relu": kernels.relu_kernel, "leaky_relu": kernels.leaky_relu_kernel,
                     "gelu_tanh": kernels.gelu_kernel_gpu, "sigmoid": kernels.sigmoid_kernel,
                     "silu": kernels.silu_kernel}[base]
                k[(N28 // 1024,)](x, out, N28, **blk)
                h2d += 2 * N28 * eb
            d2h += nout * eb
        return h2d, d2h

    one_step()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(steps):
        h2d, d2h = one_step()
    torch.cuda.synchronize()
    secs = (time.perf_counter() - t0) / steps
    step_bytes = sum(op_bytes(o) for o in suite_ops())
    return {"value": round(step_bytes / secs / 1e9, 3), "unit": "GB/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "ms_per_step": round(secs * 1e3, 2),
            "api": "xb200.kernels.<reference kernel>[grid](host tensors...)"}


if __name__ == "__main__":
    main()
