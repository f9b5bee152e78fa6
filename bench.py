"""Benchmark of the xb200 operator set on B200.

Default workload (N=1): the elementwise / activation suite on flat tensors of
2^28 elements, x, y ~ N(0, 1) from a seed -- vec-add, axpy (alpha 2.5), relu,
leaky_relu (0.01), gelu (tanh form), sigmoid, silu in bf16 and fp32, swiglu
on 2^27 + 2^27, and 2x2 / stride-2 average pooling of a [64, 256, 224, 224]
fp32 tensor.  One step = one pass of every operator over its inputs
(17 kernel launches).  Every input is larger than L2 (126 MB), so no flush is
needed between steps.

Other workloads (``--workload``) measure the remaining operator rows with the
same machinery: ``rowreduce`` (softmax, layernorm, rms_norm,
weighted_rms_norm on [32768, 4096] bf16 and fp32), ``gemm`` (the int8 /
int16 / bf16 GEMM sweep; N-sharded over the ranks when N > 1), ``qwen`` and
``gpt2`` (batch 64 x 512-token prefill + 128 greedy decode steps of the
Qwen2.5-0.5B and GPT-2 124M architectures with random-init weights,
batch-sharded over the ranks; metric tokens/s).

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
import sys
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "triton-xdna_b200"))
sys.path.insert(0, ROOT)

N28 = 1 << 28
POOL_SHAPE = (64, 256, 224, 224)
ROWS, COLS = 32768, 4096


def _peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


# DRAM traffic per launch / algorithmic bytes, from one ncu capture of the
# kernel on a smaller case of the same workload (traffic scales with the
# units processed); see the named summary under profiles/.
MEASURED_TRAFFIC_RATIO = {
    "avg_pool2d_2x2_f32": (1000.5 / 1027.6, "profiles/avg_pool2d_f32_16x256x224x224.md"),
}


def _tag(dt):
    return "bf16" if dt == torch.bfloat16 else "f32"


# ----------------------------------------------------------------------------- workloads
#
# A workload is a list of ops.  Each op has a name, its algorithmic bytes, a
# device launch (closure over device-resident tensors) and, for the headline
# workload, a launch through the public reference-signature API on pinned
# host tensors (for the end-to-end number).


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


def qwen_workload(dev, n: int, seed: int, host: bool):
    return [], {"workload": "Qwen2.5-0.5B architecture, random-init bf16 weights (seed 0): batch 64 x 512-token "
                            "random-id prefill + 128 greedy decode steps, batch-sharded over ranks"}, \
        "LLM tokens/s", "bf16"


WORKLOADS = {"elementwise": elementwise_workload, "rowreduce": rowreduce_workload, "gemm": gemm_workload,
             "qwen": qwen_workload, "gpt2": qwen_workload}


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


def run_llm_bench(args, world, rank, local, dev, kind):
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
    graphs = None if args.qwen_eager else model.decode_graphs(B, S, new)  # decode steps replay CUDA graphs
    cache = model.new_cache(B, S + new) if graphs is None else None

    def step():
        return model.generate(ids, new, cache=cache, graphs=graphs)

    for _ in range(max(1, args.warmup)):
        step()
    peaks = _peaks()
    pre, dec = [], []
    _barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        for _ in range(args.steps):
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
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = llm_cpu_baseline(kind, cfg)
    if rank == 0:
        print(json.dumps({
            "metric": "LLM tokens/s (prefill + decode)", "value": round(total_tps, 1), "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(pre_ms + dec_ms, 2), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic random ids, random-init weights (seed 0)",
            "config": {"workload": f"{LLM_WORKLOADS[kind]}: batch {B_total} x {S} prefill + {new} greedy decode",
                       "global_batch": B_total, "seq_len": S, "new_tokens": new,
                       "parallelism": f"batch-sharded x{world} (replicated weights, no collective)",
                       "l2": "weights re-read every step; decode steps replay CUDA graphs"},
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
                    "api": f"{type(model).__name__}.generate(ids copied from pinned host memory) -> tokens to host"},
            "gpu_launches": launches_per_step * args.steps,
            "cpu_baseline": cpu, "clocks": clk.summary(),
        }))


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


def run_gemm_sharded_bench(args, world, rank, local, dev):
    """N-sharded GEMMs over `world` GPUs: the fused kernel (GEMM epilogue
    stores into every rank's C over NVLink) and the NCCL all-gather baseline,
    each timed with CUDA events on every rank (max over ranks); TOPS counts
    the whole M x N x K product."""
    from xb200.dist import ShardedMatmul, nccl_sharded_matmul, shard_columns

    peaks = _peaks()
    peaks["i8_tops"] = 4500.0
    stream = torch.cuda.current_stream()
    sizes = [(4096, 4096, 4096), (8192, 8192, 8192), (16384, 16384, 16384), (16, 8192, 8192)]
    res = {}
    with ClockSampler(local) as clk:
        for dt in (torch.int8, torch.bfloat16):
            for (M, N, K) in sizes:
                if args.only and args.only not in f"{M}":
                    continue
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
                    for _ in range(max(3, args.warmup)):
                        fn()
                    times = []
                    for _ in range(max(3, args.steps // 3)):
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
                    raise RuntimeError(f"peer wait timed out (status {st})")
                sm.close()
                del a, bs
                torch.cuda.empty_cache()
    big = "sharded_fused_bf16_16384x16384x16384"
    if rank == 0:
        print(json.dumps({
            "metric": "GEMM TOPS (N-sharded, all-gather of C fused into the epilogue)",
            "value": res.get(big, {}).get("tops"), "unit": "TOPS", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "i8/bf16", "data": "synthetic, seed 0",
            "config": {"workload": "GEMM M=N=K in {4096, 8192, 16384} + 16x8192x8192, N-sharded, full C on every rank",
                       "parallelism": f"N-shard x{world}, peer-store all-gather over NVLink (NCCL path timed beside)"},
            "ops": res, "clocks": clk.summary(),
        }))


def run_gemm_bench(args, ops_list, config, world, rank, local, dev):
    """Per-GEMM timing: L2 flush, then CUDA events around each launch; the
    cuBLAS bf16 / int8 GEMMs are timed the same way as reference lines."""
    peaks = _peaks()
    peaks["i8_tops"] = 4500.0  # nominal dense int8 (no measured value in MEASURED_PEAKS.json)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()
    res = {}
    if args.only:
        ops_list = [o for o in ops_list if args.only in o.name]
    from xb200 import ops as X

    launches = 0
    with ClockSampler(local) as clk:
        for op in ops_list:
            fn, keep = op.make()
            for _ in range(max(3, args.warmup)):
                fn()
            times = []
            n0 = X.launch_count()
            for _ in range(max(3, args.steps // 3)):
                flush.zero_()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                fn()
                e1.record(stream)
                torch.cuda.synchronize()
                times.append(e0.elapsed_time(e1))
            launches += X.launch_count() - n0
            ms = statistics.median(times)
            tops = op.flops / (ms * 1e-3) / 1e12
            res[op.name] = {"ms": round(ms, 4), "tops": round(tops, 1),
                            "frac": round(tops / peaks[op.peak_key], 3), "peak_key": op.peak_key}
            del fn, keep
            torch.cuda.empty_cache()
        # cuBLAS reference lines (library GEMMs, not the product)
        ref = {}
        for n in (() if args.no_library else (4096, 8192, 16384)):
            a = torch.randn((n, n), device=dev).to(torch.bfloat16)
            b = torch.randn((n, n), device=dev).to(torch.bfloat16)
            ref[f"torch.matmul_bf16_{n}"] = a @ b
            ai = torch.randint(-128, 128, (n, n), device=dev, dtype=torch.int8)
            bi = torch.randint(-128, 128, (n, n), device=dev, dtype=torch.int8)
            for name, fn, fl in ((f"cublas_bf16_{n}", lambda: a @ b, 2 * n ** 3),
                                 (f"cublas_int8_{n}", lambda: torch._int_mm(ai, bi), 2 * n ** 3)):
                for _ in range(3):
                    fn()
                times = []
                for _ in range(5):
                    flush.zero_()
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record(stream)
                    fn()
                    e1.record(stream)
                    torch.cuda.synchronize()
                    times.append(e0.elapsed_time(e1))
                ms = statistics.median(times)
                res[name] = {"ms": round(ms, 4), "tops": round(fl / (ms * 1e-3) / 1e12, 1), "library": True}
            del a, b, ai, bi
            ref.clear()
            torch.cuda.empty_cache()
    clocks = clk.summary()
    big = "gemm_bf16_8192x8192x8192"
    e2e = gemm_e2e(dev, args.e2e_steps) if (big in res and args.e2e_steps > 0) else None
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, threads, desc = gemm_cpu_baseline()
        cpu = {"value": round(v, 4), "unit": "TOPS", "cores": threads, "kind": "port", "sample": desc}
    line = {
        "metric": "GEMM TOPS", "value": res[big]["tops"] if big in res else None, "unit": "TOPS", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "i8/i16/bf16", "data": "synthetic, seed 0", "config": config,
        "roofline": {"bound": "tensor", "kernel": big, "achieved": res.get(big, {}).get("tops"),
                     "peak": peaks["bf16_tflops"], "peak_source": peaks["source"], "unit": "TFLOP/s",
                     "frac": res.get(big, {}).get("frac"), "traffic": None},
        "ops": res, "clocks": clocks, "gpu_launches": launches, "e2e": e2e, "cpu_baseline": cpu,
    }
    if rank == 0:
        print(json.dumps(line))


def gemm_e2e(dev, steps):
    """bf16 8192^3 through the reference-signature launcher with pinned host
    operands, every step: B uploaded whole, then row pieces of A uploaded,
    multiplied and their rows of C brought back, the copies of consecutive
    pieces overlapping; wall clock around each call (it returns with C in host
    memory)."""
    from xb200 import kernels

    n = 8192
    g = torch.Generator().manual_seed(0)
    ha = torch.randn((n, n), generator=g).to(torch.bfloat16).pin_memory()
    hb = torch.randn((n, n), generator=g).to(torch.bfloat16).pin_memory()
    hc = torch.empty((n, n), dtype=torch.bfloat16).pin_memory()
    grid = (n // 256, n // 256)
    times = []
    for i in range(steps + 1):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        kernels.bare_matmul[grid](ha, hb, hc, n, n, n, n, 1, n, 1, n, 1, 256, 256, 64)
        if i:
            times.append((time.perf_counter() - t0) * 1e3)
    ms = statistics.mean(times)
    return {"value": round(2 * n ** 3 / (ms * 1e-3) / 1e12, 1), "unit": "TOPS", "ms_per_step": round(ms, 3),
            "h2d_bytes_per_step": 2 * n * n * 2, "d2h_bytes_per_step": n * n * 2,
            "api": "xb200.kernels.bare_matmul[grid](pinned host A, B, C, ...) (bf16 8192^3)"}


def gemm_cpu_baseline():
    """The int8 GEMM of the oracle (plain-C int32 accumulation, OpenMP over
    every host thread) on a 2048^3 sample; TOPS = 2 M N K / time."""
    from oracle import cgemm

    threads = os.cpu_count() or 1
    n = 2048
    g = torch.Generator().manual_seed(0)
    a = torch.randint(-128, 128, (n, n), generator=g, dtype=torch.int8)
    b = torch.randint(-128, 128, (n, n), generator=g, dtype=torch.int8)
    cgemm.gemm_int(a[:256], b)  # warm-up (and build check)
    t0 = time.perf_counter()
    cgemm.gemm_int(a, b)
    secs = time.perf_counter() - t0
    return 2 * n ** 3 / secs / 1e12, threads, f"int8 {n}x{n}x{n} through the oracle's C GEMM ({threads} threads)"


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


def reference_arm_other(args, world, warmup):
    """--impl reference for the GEMM and LLM workloads: the oracle's CPU path
    (the examples' torch expressions / the C int GEMM) on bounded samples."""
    vals = []
    if args.workload == "gemm":
        for i in range(warmup + args.steps):
            v, threads, desc = gemm_cpu_baseline()
            if i >= warmup:
                vals.append(v)
        metric, unit, dtype = "GEMM TOPS", "TOPS", "i8"
        cfg = {"workload": "GEMM sweep (CPU sample)", "sample": desc}
    else:
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
        cfg = {"workload": f"{LLM_WORKLOADS[args.workload]} (CPU sample)", "sample": desc}
    value = statistics.median(vals)
    print(json.dumps({
        "impl": "reference", "metric": metric, "value": round(value, 4), "unit": unit, "n_gpus": world,
        "steps": len(vals), "warmup": warmup, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": dtype, "data": "synthetic, seed 0", "config": cfg,
        "cpu_baseline": {"value": round(value, 4), "unit": unit, "cores": threads, "kind": "port", "sample": desc},
        "e2e": {"value": round(value, 4), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))


def _timeit(fn):
    t0 = time.perf_counter()
    fn()
    return time.perf_counter() - t0


# ----------------------------------------------------------------------------- main


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="xb200", choices=["xb200", "reference"])
    ap.add_argument("--workload", default="elementwise", choices=sorted(WORKLOADS))
    ap.add_argument("--e2e-steps", type=int, default=2)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--qwen-batch", type=int, default=64)
    ap.add_argument("--qwen-prompt", type=int, default=512)
    ap.add_argument("--qwen-new", type=int, default=128)
    ap.add_argument("--qwen-eager", action="store_true", help="qwen: launch decode steps directly (no CUDA graphs)")
    ap.add_argument("--only", default=None, help="gemm workload: run only ops whose name contains this string")
    ap.add_argument("--no-library", action="store_true", help="gemm workload: skip the cuBLAS reference lines")
    ap.add_argument("--elements", type=int, default=N28,
                    help="flat tensor length (default 2^28, the workload); smaller values are for profiling only")
    args = ap.parse_args()
    warmup = max(3, args.warmup)

    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        world = int(os.environ.get("WORLD_SIZE", "1"))
        if rank != 0:
            return
        if args.workload in LLM_WORKLOADS or args.workload == "gemm":
            reference_arm_other(args, world, warmup)
            return
        sample = 1 << 22
        for _ in range(warmup):
            cpu_baseline(args.workload, 1 << 16)
        vals = [cpu_baseline(args.workload, sample)[0] for _ in range(args.steps)]
        _, threads, desc = cpu_baseline(args.workload, sample)
        value = statistics.median(vals)
        print(json.dumps({
            "impl": "reference", "metric": SUITE_METRICS[args.workload],
            "value": round(value, 3), "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": warmup,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16+f32",
            "data": "synthetic N(0,1), seed 0",
            "config": {"workload": suite_workload(args.workload, args.elements), "cpu_sample": desc},
            "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                             "sample": desc},
            "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }))
        return

    world, rank, local = _dist_init()
    from xb200 import _lib

    _lib.load()
    dev = torch.device("cuda", torch.cuda.current_device())
    # every rank runs the end-to-end leg (its own pinned host tensors and PCIe
    # link); the job's figure is all ranks' bytes over the slowest rank's time
    want_e2e = args.e2e_steps > 0 and args.workload in ("elementwise", "rowreduce")
    if args.workload in LLM_WORKLOADS:
        run_llm_bench(args, world, rank, local, dev, args.workload)
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
        return
    ops_list, config, metric, dtype = WORKLOADS[args.workload](dev, args.elements, rank, want_e2e)
    if args.workload == "gemm":
        if world > 1:
            run_gemm_sharded_bench(args, world, rank, local, dev)
        else:
            run_gemm_bench(args, ops_list, config, world, rank, local, dev)
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
        return
    config["launches_per_step"] = len(ops_list)
    config["parallelism"] = f"weak x{world} (independent replicas, no collective)"
    step_bytes = sum(o.nbytes for o in ops_list)
    config["bytes_per_step"] = step_bytes
    stream = torch.cuda.current_stream()

    for _ in range(warmup):
        for o in ops_list:
            o.run()
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
                o.run()
                evs[s][i][1].record(stream)
        stop.record(stream)
        torch.cuda.synchronize()
    _barrier(world)
    total_ms = _max_over_ranks(start.elapsed_time(stop), world)
    clocks = clk.summary()

    per_op_ms = {o.name: statistics.mean(evs[s][i][0].elapsed_time(evs[s][i][1]) for s in range(args.steps))
                 for i, o in enumerate(ops_list)}
    ms_per_step = total_ms / args.steps
    value = step_bytes * world / (ms_per_step * 1e-3) / 1e9
    peaks = _peaks()
    hbm = peaks["hbm_gbs"]
    dom = max(ops_list, key=lambda o: per_op_ms[o.name])
    dom_gbs = dom.nbytes / (per_op_ms[dom.name] * 1e-3) / 1e9
    detail = {o.name: {"ms": round(per_op_ms[o.name], 4), "gbs": round(o.nbytes / (per_op_ms[o.name] * 1e-3) / 1e9, 1),
                       "frac": round(o.nbytes / (per_op_ms[o.name] * 1e-3) / 1e9 / hbm, 3)} for o in ops_list}

    e2e = None
    if want_e2e:
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
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        gbs, threads, desc = cpu_baseline(args.workload, 1 << 24)
        cpu = {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port", "sample": desc}

    if rank == 0:
        print(json.dumps({
            "metric": metric, "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": warmup, "ms_per_step": round(ms_per_step, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": dtype, "data": "synthetic N(0,1), seed = rank", "config": config,
            "roofline": {"bound": "hbm", "kernel": dom.name, "achieved": round(dom_gbs, 1), "peak": hbm,
                         "peak_source": peaks["source"], "unit": "GB/s", "frac": round(dom_gbs / hbm, 4),
                         "traffic": (round(MEASURED_TRAFFIC_RATIO[dom.name][0] * dom.nbytes)
                                     if dom.name in MEASURED_TRAFFIC_RATIO else None),
                         "traffic_source": MEASURED_TRAFFIC_RATIO.get(dom.name, (None, None))[1],
                         "algorithmic_bytes": dom.nbytes},
            "ops": detail, "e2e": e2e, "cpu_baseline": cpu, "clocks": clocks,
            "gpu_launches": len(ops_list) * args.steps,
        }))
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


if __name__ == "__main__":
    main()
