"""Benchmark of the xb200 operator set on B200.

Headline (the default, ``--workload gemm``): the int8 GEMM, int32
accumulate / output, at M = N = K = 16384 with A, B uniform over
[-128, 127] from a seed.  One step = 16 products C_j = A_j B_j, cycling over
4 resident operand sets (every operand is larger than L2, so no flush is
needed).  N = 1 runs the single-GPU tcgen05 kernel; N > 1 runs the N-sharded
kernel (rank r computes columns [r N/P, (r+1) N/P) and its epilogue stores
them into every rank's C over NVLink), so every rank ends with every full C
and the total work is the same at every N (strong scaling).  Before timing,
every rank checks its full C of every operand set: exact int64 row / column
checksums, sampled rows against an fp64 product, and (N > 1) equality with
the single-GPU product; a mismatch exits non-zero.

The same process then measures the metric's other rows as extra keys
(``--no-extras`` skips them): the GEMM sweep (int8 / int8 linear / int16 /
bf16 at 4096^3 .. 16384^3 and the 16 x 8192 x 8192 decode shape; N > 1: the
fused sharded kernel against the NCCL all-gather baseline), the row
reductions (softmax, layernorm, rms_norm, weighted_rms_norm on
[32768, 4096] bf16 + f32), the elementwise / activation suite (2^28
elements), and the Qwen2.5-0.5B and GPT-2 124M forwards (batch 64 x
512-token prefill + 128 greedy decode steps, batch-sharded over the ranks).

Other workloads (``--workload``): ``elementwise``, ``rowreduce``,
``gemm-sweep``, ``qwen``, ``gpt2`` print their own line.

Contract:  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl xb200|reference]
Multi-GPU: torchrun, one rank per GPU over NCCL; times are CUDA events on
each rank, max over ranks.  ``--impl reference`` times the reference's CPU
path (the examples' own CPU expressions, restated in the oracle) on the host
cores on the same sample the xb200 line's ``cpu_baseline`` uses.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "triton-xdna_b200"))
sys.path.insert(0, ROOT)

N28 = 1 << 28
POOL_SHAPE = (64, 256, 224, 224)
ROWS, COLS = 32768, 4096

# headline GEMM
HEAD_MNK = 16384
HEAD_SETS = 4  # resident operand sets (A, B, C), cycled
HEAD_PRODUCTS = 16  # products per step
CPU_SAMPLE_ROWS = 512  # CPU legs: these rows of A times the full B (same N, K as the headline)
METRIC = "GEMM TOPS (i8/bf16) % of TC peak; norm/softmax GB/s % HBM; LLM tokens/s"


def _peaks() -> dict:
    """Roofline denominators: the measured copy bandwidth and bf16 GEMM rate
    of this pool's B200s.  Dense int8 runs at twice the bf16 rate on sm_100
    (4.5 vs 2.25 POPS nominal); no int8 rate is measured, so the int8
    denominator is twice the measured bf16 burst rate (the nominal 4.5 POPS
    fraction is reported beside it)."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        pk = {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
              "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "source": "measured"}
    else:
        pk = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}
    # burst: a kernel timed alone; sustained: back-to-back for about a second
    # under the 1 kW power cap (the headline's timed region)
    pk["i8_tops"] = 2.0 * pk["bf16_tflops"]
    pk["i8_tops_sustained"] = 2.0 * pk["bf16_tflops_sustained"]
    pk["i8_tops_source"] = f"2 x {pk['source']} bf16 TFLOP/s (burst)"
    pk["i8_tops_sustained_source"] = f"2 x {pk['source']} bf16 TFLOP/s (sustained)"
    pk["i8_tops_nominal"] = 4500.0
    return pk


# DRAM traffic per launch / algorithmic bytes, from one ncu capture of the
# kernel (traffic scales with the units processed); see the named summary
# under profiles/.
MEASURED_TRAFFIC_RATIO = {
    "avg_pool2d_2x2_f32": (1000.5 / 1027.6, "profiles/avg_pool2d_f32_16x256x224x224.md"),
}


def _tag(dt):
    return "bf16" if dt == torch.bfloat16 else "f32"


# ----------------------------------------------------------------------------- workloads
#
# A suite workload is a list of ops.  Each op has a name, its algorithmic
# bytes, a device launch (closure over device-resident tensors) and a launch
# through the public reference-signature API on pinned host tensors (for the
# end-to-end number).


class Op:
    def __init__(self, name, nbytes, run, e2e=None, h2d=0, d2h=0, flops=0, peak_key=None):
        self.name, self.nbytes, self.run, self.e2e = name, nbytes, run, e2e
        self.h2d, self.d2h = h2d, d2h
        self.flops, self.peak_key = flops, peak_key


def _pinned_copy(t):
    """A pinned host copy of a device tensor: the end-to-end leg's inputs
    (filled over PCIe, not by CPU random generation, so that every rank sets
    up its host tensors in a second or two)."""
    h = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
    h.copy_(t)
    return h

def elementwise_workload(dev, n: int, seed: int, host: bool):
    from xb200 import kernels
    from xb200 import ops as X

    g = torch.Generator(device=dev).manual_seed(seed)
    half = n // 2
    out = []
    for dt in (torch.bfloat16, torch.float32):
        eb = 2 if dt == torch.bfloat16 else 4
        x = torch.randn(n, generator=g, device=dev, dtype=torch.float32).to(dt)
        y = torch.randn(n, generator=g, device=dev, dtype=torch.float32).to(dt)
        o = torch.empty_like(x)
        hx = hy = ho = None
        if host:
            hx, hy = _pinned_copy(x), _pinned_copy(y)
            ho = torch.empty(hx.shape, dtype=hx.dtype, pin_memory=True)
        t = _tag(dt)
        B = {"BLOCK_SIZE": 1024}
        grid = (max(1, n // 1024),)

        def mk(name, nin, nout, dev_fn, host_fn):
            # the launcher uploads the inputs and brings back the written output,
            # in pieces whose copies overlap (pinned host tensors)
            return Op(f"{name}_{t}", (nin + nout) * eb, dev_fn, host_fn, h2d=nin * eb, d2h=nout * eb)

        out += [
            mk("vecadd", 2 * n, n, lambda x=x, y=y, o=o: X.vecadd(x, y, out=o),
               lambda hx=hx, hy=hy, ho=ho: kernels.vecadd[grid](hx, hy, ho, n, BLOCK_SIZE_N=1024)),
            mk("axpy", 2 * n, n, lambda x=x, y=y, o=o: X.axpy(x, y, 2.5, out=o),
               lambda hx=hx, hy=hy, ho=ho: kernels.axpy_kernel[grid](hx, hy, ho, 2.5, n, **B)),
            mk("relu", n, n, lambda x=x, o=o: X.relu(x, out=o),
               lambda hx=hx, ho=ho: kernels.relu_kernel[grid](hx, ho, n, **B)),
            mk("leaky_relu", n, n, lambda x=x, o=o: X.leaky_relu(x, 0.01, out=o),
               lambda hx=hx, ho=ho: kernels.leaky_relu_kernel[grid](hx, ho, n, **B)),
            mk("gelu_tanh", n, n, lambda x=x, o=o: X.gelu_tanh(x, out=o),
               lambda hx=hx, ho=ho: kernels.gelu_kernel_gpu[grid](hx, ho, n, **B)),
            mk("sigmoid", n, n, lambda x=x, o=o: X.sigmoid(x, out=o),
               lambda hx=hx, ho=ho: kernels.sigmoid_kernel[grid](hx, ho, n, **B)),
            mk("silu", n, n, lambda x=x, o=o: X.silu(x, out=o),
               lambda hx=hx, ho=ho: kernels.silu_kernel[grid](hx, ho, n, **B)),
            mk("swiglu", 2 * half, half, lambda x=x, y=y, o=o: X.swiglu(x[:half], y[:half], out=o[:half]),
               lambda hx=hx, hy=hy, ho=ho: kernels.swiglu_kernel[(max(1, half // 1024),)](
                   hx[:half], hy[:half], ho[:half], half, **B)),
        ]
    planes = max(1, POOL_SHAPE[0] * n // N28) * POOL_SHAPE[1]
    H, W = POOL_SHAPE[2], POOL_SHAPE[3]
    pin = torch.randn((planes, H, W), generator=g, device=dev)
    pout = torch.empty((planes, H // 2, W // 2), device=dev)
    hpin = hpout = None
    if host:
        hpin = _pinned_copy(pin)
        hpout = torch.empty((planes, H // 2, W // 2), pin_memory=True)
    nin, nout = planes * H * W, planes * (H // 2) * (W // 2)
    out.append(Op("avg_pool2d_2x2_f32", (nin + nout) * 4, lambda: X.avg_pool2d_2x2(pin, out=pout),
                  lambda: kernels.avg_pool2d_kernel[(planes,)](hpin, hpout, planes, H, W, BLOCK=1),
                  h2d=nin * 4, d2h=nout * 4))
    config = {
        "workload": suite_workload("elementwise", n),
        "n_elements": n,
        "l2": "every input > 126 MB L2 (no flush needed)" if n * 2 > 126e6 else "inputs may fit in L2",
    }
    return out, config, SUITE_METRICS["elementwise"], "bf16+f32"


SUITE_METRICS = {"elementwise": "elementwise/activation suite algorithmic HBM throughput",
                 "rowreduce": "row-reduction suite algorithmic HBM throughput"}


def suite_workload(kind: str, n: int = None) -> str:
    """The workload description both arms print for the elementwise and
    row-reduction suites (n: flat length of the elementwise tensors)."""
    n = N28 if n is None else n
    if kind == "elementwise":
        half = n // 2
        planes = max(1, POOL_SHAPE[0] * n // N28) * POOL_SHAPE[1]
        return (f"elementwise/activation suite: 8 ops x {{bf16,f32}} on {n} elements "
                f"(swiglu {half}+{half}) + avg_pool2d 2x2/s2 on [{planes // 256},256,224,224] f32")
    rows = max(1, ROWS * n // N28)
    return f"row reductions on [{rows} x {COLS}] bf16 and f32, x~N(0,1)*3"


def rowreduce_workload(dev, n: int, seed: int, host: bool):
    from xb200 import ops as X

    from xb200 import kernels

    rows = max(1, ROWS * n // N28)
    g = torch.Generator(device=dev).manual_seed(seed)
    out = []
    blk = 16  # rows per program of the reference-signature launches
    grid = (max(1, rows // blk),)
    for dt in (torch.bfloat16, torch.float32):
        eb = 2 if dt == torch.bfloat16 else 4
        x = (torch.randn(rows, COLS, generator=g, device=dev) * 3).to(dt)
        gm = (1 + 0.1 * torch.randn(COLS, generator=g, device=dev)).to(dt)
        bt = (0.1 * torch.randn(COLS, generator=g, device=dev)).to(dt)
        y = torch.empty_like(x)
        hx = hg = hy = None
        if host:
            hx, hg = _pinned_copy(x), _pinned_copy(gm)
            hy = torch.empty(hx.shape, dtype=hx.dtype, pin_memory=True)
        t = _tag(dt)
        nb = 2 * rows * COLS * eb
        io = {"h2d": rows * COLS * eb, "d2h": rows * COLS * eb}
        out += [
            Op(f"softmax_{t}", nb, lambda x=x, y=y: X.softmax(x, out=y),
               lambda hx=hx, hy=hy: kernels.softmax_kernel[grid](hx, hy, COLS, 1, COLS, 1, COLS, BLOCK_SIZE=blk),
               **io),
            # the reference's fused layernorm kernel fixes gamma = 1, beta = 0
            # (examples/test_layernorm/test_layernorm.py:46-47), so its launch
            # moves 2 x 4096 fewer parameter bytes than the device line
            Op(f"layernorm_{t}", nb + 2 * COLS * eb, lambda x=x, y=y, gm=gm, bt=bt: X.layernorm(x, gm, bt, 1e-5, out=y),
               lambda hx=hx, hy=hy: kernels._layer_norm_fwd_fused[grid](hx, hy, COLS, 1, COLS, 1, COLS, 1e-5,
                                                                        BLOCK_SIZE=blk), **io),
            Op(f"rms_norm_{t}", nb, lambda x=x, y=y: X.rms_norm(x, None, 1e-6, out=y),
               lambda hx=hx, hy=hy: kernels.rms_norm_kernel[grid](hx, hy, COLS, 1e-6, BLOCK_M=blk, BLOCK_N=COLS),
               **io),
            Op(f"weighted_rms_norm_{t}", nb + COLS * eb, lambda x=x, y=y, gm=gm: X.rms_norm(x, gm, 1e-6, out=y),
               lambda hx=hx, hg=hg, hy=hy: kernels.weighted_rms_norm_kernel[grid](hx, hg, hy, COLS, 1e-6, BLOCK_M=blk,
                                                                                  BLOCK_N=COLS),
               h2d=rows * COLS * eb + COLS * eb, d2h=rows * COLS * eb),
        ]
    config = {"workload": suite_workload("rowreduce", n), "rows": rows,
              "cols": COLS, "l2": "every input > 126 MB L2 (no flush needed)"}
    return out, config, SUITE_METRICS["rowreduce"], "bf16+f32"


GEMM_SIZES = [(256, 256, 256), (1024, 1024, 1024), (4096, 4096, 4096), (8192, 8192, 8192), (16384, 16384, 16384),
              (16, 8192, 8192)]


def gemm_workload(dev, n: int, seed: int, host: bool):
    """The GEMM sweep: int8 (int32 out), int16 (int32 out, wrap-around) and
    bf16 (fp32 accumulate, bf16 out) at M=N=K in {256 .. 16384} and the
    M=16 x 8192 x 8192 decode shape.  Operands are allocated per op and
    freed after timing to bound device memory."""
    from xb200 import ops as X

    g = torch.Generator(device=dev).manual_seed(seed)
    sizes = [s for s in GEMM_SIZES if max(s) <= max(n, 256)] if n != N28 else GEMM_SIZES
    out = []
    for dt in ("i8", "i8nt", "i16", "bf16"):
        for (M, N, K) in sizes:
            def make(M=M, N=N, K=K, dt=dt):
                if dt == "i8nt":  # int8 linear: W [N, K] (K-major B)
                    a = torch.randint(-128, 128, (M, K), generator=g, device=dev, dtype=torch.int8)
                    w = torch.randint(-128, 128, (N, K), generator=g, device=dev, dtype=torch.int8)
                    c = torch.empty((M, N), dtype=torch.int32, device=dev)
                    return lambda: X.linear_i8(a, w, out=c), (a, w, c)
                if dt == "i8":
                    a = torch.randint(-128, 128, (M, K), generator=g, device=dev, dtype=torch.int8)
                    b = torch.randint(-128, 128, (K, N), generator=g, device=dev, dtype=torch.int8)
                    c = torch.empty((M, N), dtype=torch.int32, device=dev)
                    return lambda: X.matmul_i8(a, b, out=c), (a, b, c)
                if dt == "i16":
                    a = torch.randint(-2**15, 2**15, (M, K), generator=g, device=dev, dtype=torch.int16)
                    b = torch.randint(-2**15, 2**15, (K, N), generator=g, device=dev, dtype=torch.int16)
                    c = torch.empty((M, N), dtype=torch.int32, device=dev)
                    ws = torch.empty(2 * (M * K + K * N) + 4096, dtype=torch.uint8, device=dev)
                    return lambda: X.matmul_i16(a, b, out=c, workspace=ws), (a, b, c, ws)
                a = torch.randn((M, K), generator=g, device=dev).to(torch.bfloat16)
                b = torch.randn((K, N), generator=g, device=dev).to(torch.bfloat16)
                c = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
                return lambda: X.matmul_bf16(a, b, torch.bfloat16, out=c), (a, b, c)

            eb = {"i8": 1, "i8nt": 1, "i16": 2, "bf16": 2}[dt]
            ob = 2 if dt == "bf16" else 4
            op = Op(f"gemm_{dt}_{M}x{N}x{K}", (M * K + K * N) * eb + M * N * ob, None, flops=2 * M * N * K,
                    peak_key="bf16_tflops" if dt == "bf16" else "i8_tops")
            op.make = make
            out.append(op)
    config = {"workload": "GEMM sweep M=N=K in {256,1024,4096,8192,16384} + 16x8192x8192, int8 / int16 / bf16",
              "l2": "L2 flushed (256 MB write) before every timed launch"}
    return out, config, "GEMM TOPS", "i8/i16/bf16"



def llm_flops_bytes(kind, cfg, B, S, ctx_end):
    """Algorithmic work of an LLM forward: prefill FLOPs (linears over all
    tokens + causal attention + last-position LM head) and decode bytes per
    step (every weight once + the KV cache read)."""
    D, H, KVH, HD, V, L = cfg.n_embd, cfg.n_head, cfg.n_kv_head, cfg.head_dim, cfg.vocab_size, cfg.n_layer
    if kind == "qwen":
        per_tok = 2 * (D * (H + 2 * KVH) * HD + H * HD * D + 3 * D * cfg.intermediate) * L
    else:  # gpt2: QKV, attention projection, fc and mlp projection
        per_tok = 2 * (3 * D * D + D * D + 2 * D * 4 * D) * L
    attn = 2 * 2 * B * H * HD * (S * (S + 1) // 2) * L
    prefill = per_tok * B * S + attn + 2 * B * D * V
    weights = (per_tok // 2 + D * V) * 2  # bf16 bytes of every weight (LM head tied to the embedding)
    kv_mean = 2 * L * B * KVH * HD * 2 * ((S + ctx_end) / 2)
    return prefill, weights + kv_mean


LLM_WORKLOADS = {
    "qwen": "Qwen2.5-0.5B architecture (24 layers, hidden 896, 14/2 heads, MLP 4864, vocab 151936)",
    "gpt2": "GPT-2 124M architecture (12 layers, hidden 768, 12 heads, MLP 3072, vocab 50257, learned positions)",
}


def _llm_model(kind, dev):
    if kind == "qwen":
        from xb200.qwen import Qwen2Model, QwenConfig, random_weights
        cfg = QwenConfig()
        return cfg, Qwen2Model(random_weights(cfg, seed=0), cfg, device=dev, rope_len=1024)
    from xb200.gpt2 import GPT2Config, GPT2Model, random_weights
    cfg = GPT2Config.variant("gpt2")
    return cfg, GPT2Model(random_weights(cfg, seed=0), cfg, device=dev)


def llm_bench(args, world, rank, local, dev, kind, steps, warmup, cpu_leg):
    """Batch B x S prompt prefill + `new` greedy decode steps (CUDA-graph
    replays), batch-sharded over the ranks (replicated weights, no
    collective).  Returns the line (tokens/s over all ranks, max-over-ranks
    times)."""
    from xb200 import ops as X

    B_total, S, new = args.qwen_batch, args.qwen_prompt, args.qwen_new
    if B_total % world:
        raise SystemExit(f"batch {B_total} does not split over {world} ranks")
    B = B_total // world
    cfg, model = _llm_model(kind, dev)
    g = torch.Generator().manual_seed(1000 + rank)
    ids_host = torch.randint(0, cfg.vocab_size, (B, S), generator=g).pin_memory()
    ids = ids_host.to(dev)
    toks_host = torch.empty((B, new), dtype=torch.int64).pin_memory()
    # kernels one step launches: count an eager step (graph replays re-run the
    # kernels recorded at capture, which the counter saw once)
    n0 = X.launch_count()
    model.generate(ids, new)
    launches_per_step = X.launch_count() - n0
    groups = args.decode_groups if B % args.decode_groups == 0 else 1
    # decode steps replay CUDA graphs, `groups` groups of sequences on their own streams
    graphs = None if args.qwen_eager else model.decode_graphs(B, S, new, groups=groups)
    cache = model.new_cache(B, S + new) if graphs is None else None

    def step():
        return model.generate(ids, new, cache=cache, graphs=graphs)

    for _ in range(max(1, warmup)):
        step()
    peaks = _peaks()
    pre, dec = [], []
    _barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        for _ in range(steps):
            _, t = step()
            pre.append(t["prefill_ms"])
            dec.append(t["decode_ms"])
    _barrier(world)
    pre_ms = _max_over_ranks(statistics.mean(pre), world)
    dec_ms = _max_over_ranks(statistics.mean(dec), world)
    # end to end through the public API: prompt ids from pinned host memory,
    # generation, generated ids back to the host, every step
    e2e = []
    for _ in range(max(1, args.e2e_steps)):
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        ev0.record()
        ids.copy_(ids_host, non_blocking=True)
        toks, _ = model.generate(ids, new, cache=cache, graphs=graphs)
        toks_host.copy_(toks, non_blocking=True)
        ev1.record()
        torch.cuda.synchronize()
        e2e.append(ev0.elapsed_time(ev1))
    e2e_ms = _max_over_ranks(statistics.mean(e2e), world)
    flops, dec_bytes = llm_flops_bytes(kind, cfg, B, S, S + new)
    prefill_tps = B_total * S / (pre_ms * 1e-3)
    decode_tps = B_total * (new - 1) / (dec_ms * 1e-3)
    total_tps = B_total * (S + new) / ((pre_ms + dec_ms) * 1e-3)
    tflops = flops / (pre_ms * 1e-3) / 1e12
    dec_gbs = dec_bytes * (new - 1) / (dec_ms * 1e-3) / 1e9
    cpu = llm_cpu_baseline(kind, cfg) if cpu_leg else None
    groups = 1 if graphs is None else groups
    del graphs, model, cache
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return {
        "metric": "LLM tokens/s (prefill + decode)", "value": round(total_tps, 1), "unit": "tokens/s",
        "n_gpus": world, "steps": steps, "warmup": warmup,
        "ms_per_step": round(pre_ms + dec_ms, 2), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic random ids, random-init weights (seed 0)",
        "config": {"workload": f"{LLM_WORKLOADS[kind]}: batch {B_total} x {S} prefill + {new} greedy decode",
                   "global_batch": B_total, "seq_len": S, "new_tokens": new,
                   "parallelism": f"batch-sharded x{world} (replicated weights, no collective)",
                   "l2": "weights re-read every step; decode steps replay CUDA graphs",
                   "decode_groups": groups},
        "prefill_tokens_per_s": round(prefill_tps, 1), "decode_tokens_per_s": round(decode_tps, 1),
        "prefill_ms": round(pre_ms, 2), "decode_ms": round(dec_ms, 2),
        "roofline": {"bound": "tensor (prefill) / hbm (decode)",
                     "prefill": {"achieved": round(tflops, 1), "unit": "TFLOP/s", "peak": peaks["bf16_tflops"],
                                 "frac": round(tflops / peaks["bf16_tflops"], 4)},
                     "decode": {"achieved": round(dec_gbs, 1), "unit": "GB/s", "peak": peaks["hbm_gbs"],
                                "frac": round(dec_gbs / peaks["hbm_gbs"], 4)},
                     "peak_source": peaks["source"]},
        "e2e": {"value": round(B_total * (S + new) / (e2e_ms * 1e-3), 1), "unit": "tokens/s",
                "h2d_bytes_per_step": ids_host.numel() * 8 * world,
                "d2h_bytes_per_step": toks_host.numel() * 8 * world, "ms_per_step": round(e2e_ms, 2),
                "api": f"{LLM_WORKLOADS[kind].split(' (')[0]} generate(ids copied from pinned host memory) -> tokens "
                       "to host"},
        "gpu_launches": launches_per_step * steps,
        "cpu_baseline": cpu, "clocks": clk.summary(),
    }


def llm_cpu_baseline(kind, cfg):
    """The oracle forward on the host cores: one 128-token prefill + 4 decode
    steps of one sequence (a bounded sample of the workload)."""
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    if kind == "qwen":
        from oracle.qwen import OracleQwen as Oracle
        from xb200.qwen import random_weights
    else:
        from oracle.gpt2 import OracleGPT2 as Oracle
        from xb200.gpt2 import random_weights
    orc = Oracle(random_weights(cfg, seed=0), cfg)
    ids = torch.randint(0, cfg.vocab_size, (1, 128), generator=torch.Generator().manual_seed(5))
    cache = orc.new_cache(1, 132)
    t0 = time.perf_counter()
    logits = orc.forward(ids, cache)
    tok = logits[:, -1].argmax(-1)
    for _ in range(4):
        logits = orc.forward(tok.view(1, 1), cache)
        tok = logits[:, -1].argmax(-1)
    secs = time.perf_counter() - t0
    return {"value": round(132 / secs, 2), "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": "1 sequence: 128-token prefill + 4 greedy decode steps through the oracle forward"}



WORKLOADS = {"elementwise": elementwise_workload, "rowreduce": rowreduce_workload, "gemm-sweep": gemm_workload,
             "qwen": None, "gpt2": None}



# ----------------------------------------------------------------------------- headline: int8 GEMM


def headline_config() -> dict:
    """The headline workload as both arms describe it (identical at every N)."""
    return {"workload": f"int8 GEMM C = A @ B, M = N = K = {HEAD_MNK}, int32 accumulate and output, "
                        f"A and B uniform over [-128, 127]; one step = {HEAD_PRODUCTS} products cycling over "
                        f"{HEAD_SETS} resident operand sets",
            "M": HEAD_MNK, "N": HEAD_MNK, "K": HEAD_MNK, "dtype": "int8 -> int32",
            "products_per_step": HEAD_PRODUCTS, "operand_sets": HEAD_SETS,
            "l2": "every operand > 126 MB L2 (A, B 256 MiB, C 1 GiB): no flush needed"}


def _int_checksums_ok(c, a, b) -> bool:
    """Exact check of every element of C = A B (int8 operands, so |C| < 2^28
    and int64 sums are exact): row sums C 1 = A (B 1) and column sums
    1^T C = (1^T A) B, in 2048-row bands to bound the int64 temporaries."""
    M = c.shape[0]
    b_rowsum = b.to(torch.int64).sum(1)
    col_want = torch.zeros(c.shape[1], dtype=torch.int64, device=c.device)
    col_got = torch.zeros_like(col_want)
    a_colsum = a.to(torch.int64).sum(0)
    for r0 in range(0, M, 2048):
        cb = c[r0:r0 + 2048].to(torch.int64)
        if not torch.equal(cb.sum(1), (a[r0:r0 + 2048].to(torch.int64) * b_rowsum).sum(1)):
            return False
        col_got += cb.sum(0)
    for k0 in range(0, a.shape[1], 2048):
        col_want += (a_colsum[k0:k0 + 2048, None] * b[k0:k0 + 2048].to(torch.int64)).sum(0)
    return torch.equal(col_got, col_want)


def _sampled_rows_ok(c, a, b, seed) -> bool:
    """Eight rows against an fp64 product (exact: |partial sums| < 2^28)."""
    rows = torch.randint(0, a.shape[0], (8,), generator=torch.Generator().manual_seed(seed)).to(c.device)
    want = (a[rows].double() @ b.double()).to(torch.int64)
    return torch.equal(c[rows].to(torch.int64), want)


def _gen_set(j, dev, M, N, K):
    g = torch.Generator(device=dev).manual_seed(100 + j)
    a = torch.randint(-128, 128, (M, K), generator=g, device=dev, dtype=torch.int8)
    b = torch.randint(-128, 128, (K, N), generator=g, device=dev, dtype=torch.int8)
    return a, b


def gemm_headline(args, world, rank, local, dev) -> dict:
    from xb200 import ops as X

    M = N = K = HEAD_MNK
    P = args.products
    nsets = min(HEAD_SETS, P)
    stream = torch.cuda.current_stream()
    peaks = _peaks()
    plans = []
    sets = []
    if world == 1:
        for j in range(nsets):
            a, b = _gen_set(j, dev, M, N, K)
            c = torch.empty((M, N), dtype=torch.int32, device=dev)
            sets.append((a, b, c))

        def run(j):
            a, b, c = sets[j]
            X.matmul_i8(a, b, out=c)
            return c
        parallelism = "single GPU"
    else:
        from xb200.dist import ShardedMatmul, shard_columns

        s0, ns = shard_columns(N, world)[rank]
        for j in range(nsets):
            a, b = _gen_set(j, dev, M, N, K)
            sets.append((a, b[:, s0:s0 + ns].contiguous(), None))
            del b
            plans.append(ShardedMatmul(M, N, K, torch.int8))

        def run(j):
            return plans[j].run(sets[j][0], sets[j][1])
        parallelism = (f"N-sharded x{world}: each rank computes {N // world} columns and its GEMM epilogue stores "
                       f"them into every rank's C over NVLink (all-gather fused, no NCCL on the data path)")

    # ---- parity: every rank's full C of every operand set, before timing
    checks = []
    for j in range(nsets):
        c = run(j)
        torch.cuda.synchronize()
        a = sets[j][0]
        _, b_full = _gen_set(j, dev, M, N, K)
        ok = _int_checksums_ok(c, a, b_full) and _sampled_rows_ok(c, a, b_full, j)
        if world > 1:
            ok = ok and torch.equal(c, X.matmul_i8(a, b_full))
            ok = ok and plans[j].status() == 0
        ok = ok and X.device_status() == 0
        checks.append(bool(ok))
        del b_full
        torch.cuda.empty_cache()
    if not all(checks):
        print(json.dumps({"error": "headline GEMM parity check failed", "rank": rank, "checks": checks}),
              file=sys.stderr)
        raise SystemExit(3)

    for i in range(max(3, args.warmup)):
        run(i % nsets)
    torch.cuda.synchronize()

    # ---- timed region: K steps x P products, per-launch CUDA events on the launching stream
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps * P)]
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n0 = X.launch_count()
    _barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        start.record(stream)
        for i in range(args.steps * P):
            evs[i][0].record(stream)
            run(i % nsets)
            evs[i][1].record(stream)
        stop.record(stream)
        torch.cuda.synchronize()
    launches = X.launch_count() - n0
    _barrier(world)
    total_ms = _max_over_ranks(start.elapsed_time(stop), world)
    launch_ms = _max_over_ranks(statistics.mean(e0.elapsed_time(e1) for e0, e1 in evs), world)
    status = [p.status() for p in plans] + [X.device_status()]
    if any(status):
        print(json.dumps({"error": "device status after timing", "rank": rank, "status": status}), file=sys.stderr)
        raise SystemExit(3)
    ms_per_step = total_ms / args.steps
    ops_per_step = P * 2 * M * N * K
    value = ops_per_step / (ms_per_step * 1e-3) / 1e12
    rank_ops = 2 * M * (N // world) * K  # this rank's share of one product
    achieved = rank_ops / (launch_ms * 1e-3) / 1e12
    alg_bytes = M * K + K * (N // world) + 4 * M * N  # A, B shard read once; full C written once per rank

    e2e = None
    if args.e2e_steps > 0:
        e2e = gemm_headline_e2e(args, world, rank, dev, sets, plans)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, threads, desc = gemm_cpu_sample()
        cpu = {"value": round(v, 4), "unit": "TOPS", "cores": threads, "kind": "port", "sample": desc}
    for p in plans:
        p.close()
    del sets, plans
    torch.cuda.empty_cache()
    traffic = HEADLINE_TRAFFIC.get(world)
    return {
        "metric": METRIC, "value": round(value, 1), "unit": "TOPS", "n_gpus": world, "steps": args.steps,
        "warmup": max(3, args.warmup), "ms_per_step": round(ms_per_step, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "int8", "data": "synthetic, uniform int8, seeds 100..103",
        "config": headline_config(), "parallelism": parallelism,
        "parity": {"checked_before_timing": True, "operand_sets": nsets,
                   "checks": "int64 row+column checksums of every element, 8 rows vs fp64"
                             + (", equality with the single-GPU product" if world > 1 else ""),
                   "ok": True},
        "roofline": {"bound": "tensor", "kernel": "gemm_kernel<int8, CTA pairs" + (", peer stores>" if world > 1
                                                                                    else ">"),
                     "achieved": round(achieved, 1), "peak": peaks["i8_tops_sustained"],
                     "peak_source": peaks["i8_tops_sustained_source"] + ": the timed region runs the kernel back "
                                    "to back for about a second",
                     "unit": "TOPS", "frac": round(achieved / peaks["i8_tops_sustained"], 4),
                     "frac_of_burst": round(achieved / peaks["i8_tops"], 4),
                     "frac_of_nominal_4500": round(achieved / peaks["i8_tops_nominal"], 4),
                     "launch_ms": round(launch_ms, 4), "ops_per_launch": rank_ops,
                     "traffic": traffic[0] if traffic else None,
                     "traffic_source": traffic[1] if traffic else None, "algorithmic_bytes": alg_bytes},
        "e2e": e2e, "cpu_baseline": cpu, "clocks": clk.summary(), "gpu_launches": launches,
    }


# ncu dram__bytes_read.sum + dram__bytes_write.sum of one headline launch (per
# rank), keyed by world size; see the named summary under profiles/.
HEADLINE_TRAFFIC = {1: (6011971000 + 1064136000, "profiles/gemm_i8_16384_headline.md")}


def gemm_headline_e2e(args, world, rank, dev, sets, plans) -> dict:
    """The headline through the public API with host buffers, every product
    copying its inputs from pinned host memory and its result back.
    N = 1: `bare_matmul_i8[grid](A, B, C)` on pinned host tensors (the
    launcher uploads B, then pieces of A's rows, and brings C's rows back,
    the copies of consecutive pieces overlapping).  N > 1: every rank uploads
    A and its B shard, runs the sharded GEMM, and brings back its 1/N band of
    C's rows (each rank holds the full C; the bands together are C), so the
    host-side result is spread over the N PCIe links."""
    from xb200 import kernels

    M = N = K = HEAD_MNK
    P = args.products
    a_dev, b_dev, c_dev = sets[0]
    ha = _pinned_copy(a_dev)
    hb = _pinned_copy(b_dev)
    if world == 1:
        hc = torch.empty((M, N), dtype=torch.int32, pin_memory=True)
        grid = (M // 128, N // 64)

        def product(j):
            kernels.bare_matmul_i8[grid](ha, hb, hc, M, N, K, K, 1, N, 1, N, 1, BLOCK_SIZE_M=128, BLOCK_SIZE_N=64,
                                         BLOCK_SIZE_K=K)
        h2d, d2h = P * (M * K + K * N), P * M * N * 4
        api = "xb200.kernels.bare_matmul_i8[grid](pinned host A, B, C, ...)"
    else:
        rows = M // world
        hc = torch.empty((rows, N), dtype=torch.int32, pin_memory=True)

        def product(j):
            a, bs, _ = sets[j]
            a.copy_(ha, non_blocking=True)
            bs.copy_(hb, non_blocking=True)
            c = plans[j].run(a, bs)
            hc.copy_(c[rank * rows:(rank + 1) * rows], non_blocking=True)
        h2d, d2h = world * P * (M * K + K * (N // world)), P * M * N * 4
        api = ("xb200.dist.ShardedMatmul.run with A and the B shard copied from pinned host memory and each "
               "rank's band of C's rows copied back, every rank")
    nsets = len(sets)
    for j in range(2):
        product(j % nsets)
    torch.cuda.synchronize()
    times = []
    for _ in range(args.e2e_steps):
        _barrier(world)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for i in range(P):
            product(i % nsets)
        torch.cuda.synchronize()
        times.append(time.perf_counter() - t0)
    secs = _max_over_ranks(statistics.mean(times), world)
    return {"value": round(P * 2 * M * N * K / secs / 1e12, 1), "unit": "TOPS", "ms_per_step": round(secs * 1e3, 2),
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "api": api}


_CPU_SAMPLE = {}  # seed -> (A rows, B): generated once per process


def gemm_cpu_sample(rows: int = CPU_SAMPLE_ROWS, seed: int = 100):
    """The reference's CPU path for the headline: the example's int32 GEMM
    (restated in plain C, OpenMP over every host thread) on `rows` rows of A
    times a full B of the headline's N and K; TOPS = 2 rows N K / time.
    Inputs from a CPU generator (the same sample in both arms)."""
    from oracle import cgemm

    threads = os.cpu_count() or 1
    if seed not in _CPU_SAMPLE:
        g = torch.Generator().manual_seed(seed)
        b = torch.randint(-128, 128, (HEAD_MNK, HEAD_MNK), generator=g, dtype=torch.int8)
        a = torch.randint(-128, 128, (CPU_SAMPLE_ROWS, HEAD_MNK), generator=g, dtype=torch.int8)
        _CPU_SAMPLE[seed] = (a, b)
    a, b = _CPU_SAMPLE[seed]
    a = a[:rows]
    cgemm.gemm_int(a[:8], b)  # warm-up (and build check)
    t0 = time.perf_counter()
    cgemm.gemm_int(a, b)
    secs = time.perf_counter() - t0
    return (2 * rows * HEAD_MNK * HEAD_MNK / secs / 1e12, threads,
            f"int8 {rows} x {HEAD_MNK} x {HEAD_MNK} (rows of A times the full B of the headline shape) through "
            f"the oracle's C GEMM, {threads} threads")


# ----------------------------------------------------------------------------- GEMM sweep (extras)

SWEEP_EXTRA = [(4096, 4096, 4096), (8192, 8192, 8192), (16384, 16384, 16384), (16, 8192, 8192)]


def gemm_sweep_single(args, dev, sizes, kinds, library: bool) -> dict:
    """Per-GEMM timing on one GPU: L2 flushed (256 MB write) before each
    launch, CUDA events around it, median of the repetitions; cuBLAS bf16 /
    int8 GEMMs timed the same way as reference lines."""
    from xb200 import ops as X

    peaks = _peaks()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()
    ops_list = [o for o in gemm_workload(dev, N28, 0, False)[0]
                if (o.name.split("_")[1] in kinds) and tuple(map(int, o.name.split("_")[2].split("x"))) in sizes]
    if args.only:
        ops_list = [o for o in ops_list if args.only in o.name]
    reps = max(3, min(10, args.steps // 2))
    res = {}

    def timed(fn):
        for _ in range(3):
            fn()
        times = []
        for _ in range(reps):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            fn()
            e1.record(stream)
            torch.cuda.synchronize()
            times.append(e0.elapsed_time(e1))
        return statistics.median(times)

    for op in ops_list:
        fn, keep = op.make()
        ms = timed(fn)
        tops = op.flops / (ms * 1e-3) / 1e12
        res[op.name] = {"ms": round(ms, 4), "tops": round(tops, 1), "frac": round(tops / peaks[op.peak_key], 3),
                        "peak_key": op.peak_key}
        del fn, keep
        torch.cuda.empty_cache()
    if library:  # cuBLAS reference lines (library GEMMs, not the product)
        for n in (8192, 16384):
            a = torch.randn((n, n), device=dev).to(torch.bfloat16)
            b = torch.randn((n, n), device=dev).to(torch.bfloat16)
            ai = torch.randint(-128, 128, (n, n), device=dev, dtype=torch.int8)
            bi = torch.randint(-128, 128, (n, n), device=dev, dtype=torch.int8)
            for name, fn in ((f"cublas_bf16_{n}", lambda: a @ b), (f"cublas_int8_{n}", lambda: torch._int_mm(ai, bi))):
                ms = timed(fn)
                res[name] = {"ms": round(ms, 4), "tops": round(2 * n ** 3 / (ms * 1e-3) / 1e12, 1), "library": True}
            del a, b, ai, bi
            torch.cuda.empty_cache()
    X.device_status()
    return {"unit": "TOPS", "l2": "flushed before every launch", "peaks": {k: peaks[k] for k in
                                                                          ("bf16_tflops", "i8_tops")}, "ops": res}


def gemm_sweep_sharded(args, world, rank, dev, sizes) -> dict:
    """N-sharded GEMMs over the ranks: the fused kernel (epilogue stores into
    every rank's C over NVLink) against the NCCL all-gather baseline, CUDA
    events on every rank, max over ranks; TOPS counts the whole product."""
    from xb200.dist import ShardedMatmul, nccl_sharded_matmul, shard_columns

    peaks = _peaks()
    stream = torch.cuda.current_stream()
    reps = max(3, min(10, args.steps // 2))
    res = {}
    for dt in (torch.int8, torch.bfloat16):
        for (M, N, K) in sizes:
            g = torch.Generator(device=dev).manual_seed(0)
            if dt == torch.int8:
                a = torch.randint(-128, 128, (M, K), generator=g, device=dev, dtype=dt)
                b = torch.randint(-128, 128, (K, N), generator=g, device=dev, dtype=dt)
            else:
                a = torch.randn((M, K), generator=g, device=dev).to(dt)
                b = torch.randn((K, N), generator=g, device=dev).to(dt)
            s0, ns = shard_columns(N, world)[rank]
            bs = b[:, s0:s0 + ns].contiguous()
            del b
            sm = ShardedMatmul(M, N, K, dt)
            tag = "i8" if dt == torch.int8 else "bf16"
            for name, fn in ((f"sharded_fused_{tag}_{M}x{N}x{K}", lambda: sm.run(a, bs)),
                             (f"sharded_nccl_{tag}_{M}x{N}x{K}", lambda: nccl_sharded_matmul(a, bs))):
                for _ in range(3):
                    fn()
                times = []
                for _ in range(reps):
                    _barrier(world)
                    torch.cuda.synchronize()
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record(stream)
                    fn()
                    e1.record(stream)
                    torch.cuda.synchronize()
                    times.append(_max_over_ranks(e0.elapsed_time(e1), world))
                ms = statistics.median(times)
                tops = 2 * M * N * K / (ms * 1e-3) / 1e12
                pk = peaks["i8_tops"] if tag == "i8" else peaks["bf16_tflops"]
                res[name] = {"ms": round(ms, 4), "tops": round(tops, 1), "frac_of_world_peak":
                             round(tops / (pk * world), 3)}
            st = sm.status()
            if st != 0:
                raise RuntimeError(f"sharded GEMM status {st}")
            sm.close()
            del a, bs
            torch.cuda.empty_cache()
    return {"unit": "TOPS", "parallelism": f"N-shard x{world}", "ops": res}


# ----------------------------------------------------------------------------- suites (elementwise, rows)


def time_suite(kind, args, world, rank, local, dev, steps, warmup, with_e2e: bool, cpu_leg: bool) -> dict:
    """Every operator of a suite once per step (weak scaling: every rank runs
    the whole suite on its own data), per-launch CUDA events; the line's
    value is all ranks' algorithmic bytes over the slowest rank's time."""
    ops_list, config, metric, dtype = WORKLOADS[kind](dev, args.elements, rank, with_e2e)
    config["launches_per_step"] = len(ops_list)
    config["parallelism"] = f"weak x{world} (independent replicas, no collective)"
    step_bytes = sum(o.nbytes for o in ops_list)
    config["bytes_per_step"] = step_bytes
    stream = torch.cuda.current_stream()
    for _ in range(warmup):
        for o in ops_list:
            o.run()
    torch.cuda.synchronize()
    evs = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in ops_list]
           for _ in range(steps)]
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    _barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        start.record(stream)
        for s in range(steps):
            for i, o in enumerate(ops_list):
                evs[s][i][0].record(stream)
                o.run()
                evs[s][i][1].record(stream)
        stop.record(stream)
        torch.cuda.synchronize()
    _barrier(world)
    total_ms = _max_over_ranks(start.elapsed_time(stop), world)
    per_op_ms = {o.name: statistics.mean(evs[s][i][0].elapsed_time(evs[s][i][1]) for s in range(steps))
                 for i, o in enumerate(ops_list)}
    ms_per_step = total_ms / steps
    value = step_bytes * world / (ms_per_step * 1e-3) / 1e9
    peaks = _peaks()
    hbm = peaks["hbm_gbs"]
    dom = max(ops_list, key=lambda o: per_op_ms[o.name])
    dom_gbs = dom.nbytes / (per_op_ms[dom.name] * 1e-3) / 1e9
    detail = {o.name: {"ms": round(per_op_ms[o.name], 4), "gbs": round(o.nbytes / (per_op_ms[o.name] * 1e-3) / 1e9, 1),
                       "frac": round(o.nbytes / (per_op_ms[o.name] * 1e-3) / 1e9 / hbm, 3)} for o in ops_list}
    e2e = None
    if with_e2e:
        for o in ops_list:
            o.e2e()
        torch.cuda.synchronize()
        _barrier(world)
        t0 = time.perf_counter()
        for _ in range(args.e2e_steps):
            for o in ops_list:
                o.e2e()
        torch.cuda.synchronize()
        secs = _max_over_ranks((time.perf_counter() - t0) / args.e2e_steps, world)
        e2e = {"value": round(world * step_bytes / secs / 1e9, 3), "unit": "GB/s",
               "h2d_bytes_per_step": world * sum(o.h2d for o in ops_list),
               "d2h_bytes_per_step": world * sum(o.d2h for o in ops_list),
               "ms_per_step": round(secs * 1e3, 2),
               "api": "xb200.kernels.<reference kernel>[grid](pinned host tensors...), every rank"}
    cpu = None
    if cpu_leg:
        gbs, threads, desc = cpu_baseline(kind, 1 << 24)
        cpu = {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port", "sample": desc}
    del ops_list
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return {
        "metric": metric, "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": steps,
        "warmup": warmup, "ms_per_step": round(ms_per_step, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": dtype, "data": "synthetic N(0,1), seed = rank", "config": config,
        "roofline": {"bound": "hbm", "kernel": dom.name, "achieved": round(dom_gbs, 1), "peak": hbm,
                     "peak_source": peaks["source"], "unit": "GB/s", "frac": round(dom_gbs / hbm, 4),
                     "traffic": (round(MEASURED_TRAFFIC_RATIO[dom.name][0] * dom.nbytes)
                                 if dom.name in MEASURED_TRAFFIC_RATIO else None),
                     "traffic_source": MEASURED_TRAFFIC_RATIO.get(dom.name, (None, None))[1],
                     "algorithmic_bytes": dom.nbytes},
        "ops": detail, "e2e": e2e, "cpu_baseline": cpu, "clocks": clk.summary(),
        "gpu_launches": len(detail) * steps,
    }


# ----------------------------------------------------------------------------- clocks


class ClockSampler:
    """SM clock and clock-event (throttle) reasons of the benchmark's GPU, read
    through NVML every 5 ms by a background thread while the timed region
    runs (read-only queries; nothing about the GPU is changed)."""

    REASONS = {
        "hw_slowdown": "nvmlClocksEventReasonHwSlowdown",
        "hw_thermal_slowdown": "nvmlClocksEventReasonHwThermalSlowdown",
        "sw_thermal_slowdown": "nvmlClocksEventReasonSwThermalSlowdown",
        "sw_power_cap": "nvmlClocksEventReasonSwPowerCap",
        "hw_power_brake_slowdown": "nvmlClocksEventReasonHwPowerBrakeSlowdown",
    }

    def __init__(self, cuda_index: int, period_s: float = 0.005):
        self.cuda_index = cuda_index
        self.period = period_s
        self.samples = []
        self.smax = None
        self._stop = None
        self._thr = None
        self.nv = None

    def _handle(self):
        import pynvml as nv

        nv.nvmlInit()
        self.nv = nv
        p = torch.cuda.get_device_properties(self.cuda_index)
        try:
            bus = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
            return nv.nvmlDeviceGetHandleByPciBusId_v2(bus)
        except Exception:
            return nv.nvmlDeviceGetHandleByIndex(self.cuda_index)

    def __enter__(self):
        import threading

        try:
            h = self._handle()
            nv = self.nv
            self.smax = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
            get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons",
                                  getattr(nv, "nvmlDeviceGetCurrentClocksThrottleReasons", None))
        except Exception:
            return self
        self._stop = threading.Event()

        def loop():
            while not self._stop.is_set():
                try:
                    self.samples.append((nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM), int(get_reasons(h))))
                except Exception:
                    pass
                self._stop.wait(self.period)

        self._thr = threading.Thread(target=loop, daemon=True)
        self._thr.start()
        return self

    def __exit__(self, *exc):
        if self._thr is not None:
            self._stop.set()
            self._thr.join(timeout=2)

    def summary(self):
        if not self.samples:
            return None
        reasons = set()
        for _, bits in self.samples:
            for name, attr in self.REASONS.items():
                if bits & getattr(self.nv, attr, 0):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(c for c, _ in self.samples), "sm_max_mhz": self.smax,
                "reasons": sorted(reasons), "samples": len(self.samples), "source": "NVML, 5 ms"}


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



# ----------------------------------------------------------------------------- CPU baseline


def cpu_baseline(workload: str, sample: int, reps: int = 1):
    """Time the oracle (the examples' torch CPU expressions) on a bounded sample
    of the workload with every host thread; returns (GB/s, threads, description)."""
    from oracle import ops as O

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(0)
    cases = []
    if workload == "elementwise":
        for dt in (torch.bfloat16, torch.float32):
            eb = 2 if dt == torch.bfloat16 else 4
            x = torch.randn(sample, generator=g).to(dt)
            y = torch.randn(sample, generator=g).to(dt)
            h = sample // 2
            cases += [
                (lambda x=x, y=y: O.vecadd(x, y), 3 * sample * eb), (lambda x=x, y=y: O.axpy(x, y, 2.5), 3 * sample * eb),
                (lambda x=x: O.relu(x), 2 * sample * eb), (lambda x=x: O.leaky_relu(x, 0.01), 2 * sample * eb),
                (lambda x=x: O.gelu_tanh(x), 2 * sample * eb), (lambda x=x: O.sigmoid(x), 2 * sample * eb),
                (lambda x=x: O.silu(x), 2 * sample * eb), (lambda x=x, y=y: O.swiglu(x[:h], y[:h]), 3 * h * eb),
            ]
        planes = max(1, sample // (224 * 224))
        p = torch.randn((planes, 224, 224), generator=g)
        cases.append((lambda: O.avg_pool2d_2x2(p), p.numel() * 4 * 5 // 4))
        desc = f"every suite operator on {sample} elements ({sample / N28:.4f} of the workload), min of {reps}"
    else:
        rows = max(1, sample // COLS)
        for dt in (torch.bfloat16, torch.float32):
            eb = 2 if dt == torch.bfloat16 else 4
            x = (torch.randn(rows, COLS, generator=g) * 3).to(dt)
            w = (1 + 0.1 * torch.randn(COLS, generator=g)).to(dt)
            nb = 2 * rows * COLS * eb
            cases += [(lambda x=x: O.softmax(x), nb), (lambda x=x, w=w: O.layernorm(x, w, w, 1e-5), nb),
                      (lambda x=x: O.rms_norm(x, 1e-6), nb), (lambda x=x, w=w: O.weighted_rms_norm(x, w, 1e-6), nb)]
        desc = f"every row op on [{rows} x {COLS}] ({rows / ROWS:.4f} of the workload), min of {reps}"
    total_b, total_s = 0, 0.0
    for fn, nb in cases:
        fn()
        best = min(_timeit(fn) for _ in range(reps))
        total_b += nb
        total_s += best
    return total_b / total_s / 1e9, threads, desc



def reference_arm(args, world, warmup):
    """--impl reference: the reference's CPU path of the workload on the host
    cores, with every host thread, printed on the xb200 line's metric, unit
    and config.  The examples' own CPU expressions run in the oracle (the
    reference itself cannot run here: its launch path needs an XDNA NPU)."""
    vals = []
    if args.workload == "gemm":
        gemm_cpu_sample(rows=8)  # warm-up (builds the oracle's C GEMM)
        for _ in range(args.steps):
            v, threads, desc = gemm_cpu_sample()
            vals.append(v)
        metric, unit, dtype, cfg = METRIC, "TOPS", "int8", headline_config()
    elif args.workload in LLM_WORKLOADS:
        if args.workload == "qwen":
            from xb200.qwen import QwenConfig
            cfg_m = QwenConfig()
        else:
            from xb200.gpt2 import GPT2Config
            cfg_m = GPT2Config.variant("gpt2")
        steps = max(1, min(args.steps, 5))
        for i in range(1 + steps):
            r = llm_cpu_baseline(args.workload, cfg_m)
            if i:
                vals.append(r["value"])
        threads, desc = r["cores"], r["sample"]
        metric, unit, dtype = "LLM tokens/s (prefill + decode)", "tokens/s", "bf16"
        cfg = {"workload": f"{LLM_WORKLOADS[args.workload]}: batch {args.qwen_batch} x {args.qwen_prompt} prefill "
                           f"+ {args.qwen_new} greedy decode"}
    elif args.workload in SUITE_METRICS:
        sample = 1 << 24
        for _ in range(warmup):
            cpu_baseline(args.workload, 1 << 16)
        vals = [cpu_baseline(args.workload, sample)[0] for _ in range(args.steps)]
        _, threads, desc = cpu_baseline(args.workload, sample)
        metric, unit, dtype = SUITE_METRICS[args.workload], "GB/s", "bf16+f32"
        cfg = {"workload": suite_workload(args.workload, args.elements)}
    else:
        print(json.dumps({"impl": "reference", "unavailable": f"no CPU arm for workload {args.workload}"}))
        return
    value = statistics.median(vals)
    print(json.dumps({
        "impl": "reference", "metric": metric, "value": round(value, 4), "unit": unit, "n_gpus": world,
        "steps": len(vals), "warmup": warmup, "higher_is_better": True,
        "scaling": "strong" if args.workload == "gemm" else "weak", "vs_baseline": None,
        "dtype": dtype, "data": "synthetic, seeded", "config": cfg,
        "cpu_baseline": {"value": round(value, 4), "unit": unit, "cores": threads, "kind": "port", "sample": desc},
        "e2e": {"value": round(value, 4), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))


def _timeit(fn):
    t0 = time.perf_counter()
    fn()
    return time.perf_counter() - t0


# ----------------------------------------------------------------------------- main


def run_extras(args, world, rank, local, dev) -> dict:
    """The metric's other rows, measured in the same process after the headline."""
    extras = {}
    steps = max(3, min(args.steps, 20))
    warm = 3
    t0 = time.perf_counter()
    if world == 1:
        extras["gemm_sweep"] = gemm_sweep_single(args, dev, SWEEP_EXTRA, ("i8", "i8nt", "i16", "bf16"),
                                                 library=not args.no_library)
    else:
        extras["gemm_sweep_sharded"] = gemm_sweep_sharded(args, world, rank, dev,
                                                          [(8192, 8192, 8192), (16384, 16384, 16384)])
    cpu_leg = rank == 0 and world == 1 and not args.no_cpu_baseline
    extras["rowreduce"] = time_suite("rowreduce", args, world, rank, local, dev, steps, warm, args.e2e_steps > 0,
                                     cpu_leg)
    extras["elementwise"] = time_suite("elementwise", args, world, rank, local, dev, steps, warm, False, cpu_leg)
    extras["qwen"] = llm_bench(args, world, rank, local, dev, "qwen", steps, warm, cpu_leg)
    extras["gpt2"] = llm_bench(args, world, rank, local, dev, "gpt2", steps, warm, cpu_leg)
    extras["wall_s"] = round(time.perf_counter() - t0, 1)
    return extras


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="xb200", choices=["xb200", "reference"])
    ap.add_argument("--workload", default="gemm", choices=["gemm"] + sorted(WORKLOADS))
    ap.add_argument("--products", type=int, default=HEAD_PRODUCTS,
                    help="gemm: products per step (default 16; fewer only for profiling)")
    ap.add_argument("--no-extras", action="store_true", help="gemm: only the headline line's own measurements")
    ap.add_argument("--e2e-steps", type=int, default=2)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--qwen-batch", type=int, default=64)
    ap.add_argument("--qwen-prompt", type=int, default=512)
    ap.add_argument("--qwen-new", type=int, default=128)
    ap.add_argument("--qwen-eager", action="store_true", help="qwen: launch decode steps directly (no CUDA graphs)")
    ap.add_argument("--decode-groups", type=int, default=1,
                    help="LLM decode: sequence groups replaying their graphs concurrently on their own streams")
    ap.add_argument("--only", default=None, help="gemm-sweep: run only ops whose name contains this string")
    ap.add_argument("--no-library", action="store_true", help="gemm sweeps: skip the cuBLAS reference lines")
    ap.add_argument("--elements", type=int, default=N28,
                    help="flat tensor length (default 2^28, the workload); smaller values are for profiling only")
    args = ap.parse_args()
    warmup = max(3, args.warmup)

    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        world = int(os.environ.get("WORLD_SIZE", "1"))
        if rank == 0:
            torch.set_num_threads(os.cpu_count() or 1)
            reference_arm(args, world, warmup)
        return

    world, rank, local = _dist_init()
    from xb200 import _lib

    _lib.load()
    dev = torch.device("cuda", torch.cuda.current_device())
    try:
        if args.workload == "gemm":
            line = gemm_headline(args, world, rank, local, dev)
            if not args.no_extras:
                line["extras"] = run_extras(args, world, rank, local, dev)
        elif args.workload in LLM_WORKLOADS:
            line = llm_bench(args, world, rank, local, dev, args.workload, args.steps, warmup,
                             rank == 0 and world == 1 and not args.no_cpu_baseline)
        elif args.workload == "gemm-sweep":
            if world == 1:
                res = gemm_sweep_single(args, dev, GEMM_SIZES, ("i8", "i8nt", "i16", "bf16"),
                                        library=not args.no_library)
            else:
                res = gemm_sweep_sharded(args, world, rank, dev, [(4096, 4096, 4096), (8192, 8192, 8192),
                                                                  (16384, 16384, 16384), (16, 8192, 8192)])
            line = {"metric": "GEMM sweep TOPS", "n_gpus": world, "steps": args.steps, "warmup": warmup, **res}
        else:
            line = time_suite(args.workload, args, world, rank, local, dev, args.steps, warmup,
                              args.e2e_steps > 0, rank == 0 and world == 1 and not args.no_cpu_baseline)
        if rank == 0:
            print(json.dumps(line))
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
