"""Parity at the shapes bench.py times, on the B200.

* The int8 example's own sweep (examples/matmul_i8_m128_n64_k64/
  matmul_i8_m128_n64_k64.py:89, 94-98: M in {1024, 2048, 4096} x N in
  {1024, 2048} x K in {256, 512, 1024}, atol = rtol = 0), launched the way the
  example launches (`bare_matmul_i8[grid]` on host tensors) and compared
  exactly with the C oracle.
* The GEMM sweep (M = N = K in {256, 1024, 4096, 8192, 16384} and the
  16 x 8192 x 8192 decode shape) for every entry point the benchmark times:
  int8 with row-major B (`matmul_i8`), int8 linear with W [N, K]
  (`linear_i8`), int16 (`matmul_i16`, wrap-around mod 2^32) and bf16
  (`matmul_bf16`, bf16 out).  Integer products up to 4096^3 are compared with
  the C oracle element by element; at 8192^3 and 16384^3 every element is
  covered by exact int64 row and column checksums reduced mod 2^32
  (C 1 = A (B 1), 1^T C = (1^T A) B, both exact in int64 at these
  magnitudes) plus sampled rows and columns against the C oracle.  bf16 is
  compared with an fp32 product of the same bf16 inputs rounded to bf16
  (whole C up to 1024^3 and the decode shape, sampled rows and columns
  above), within one bf16 rounding of the fp32 accumulation.
* The Qwen2.5 workload shape: a batch of 64 x 512-token prompts through the
  24-layer random-init model, teacher-forced, with two of the 64 sequences
  compared against the oracle forward through the prefill and three decode
  steps.
"""

import math

import pytest
import torch

from oracle import cgemm
from xb200 import kernels, ops

pytestmark = pytest.mark.gpu

SWEEP = [(256, 256, 256), (1024, 1024, 1024), (4096, 4096, 4096), (8192, 8192, 8192), (16384, 16384, 16384),
         (16, 8192, 8192)]
SMALL = [s for s in SWEEP if s[0] * s[1] * s[2] <= 4096 ** 3]
LARGE = [s for s in SWEEP if s[0] * s[1] * s[2] > 4096 ** 3]
MOD = 1 << 32


def _ok():
    assert ops.device_status() == 0


def _free():
    torch.cuda.synchronize()
    torch.cuda.empty_cache()


# ---------------------------------------------------------------- int8 example sweep


@pytest.mark.parametrize("M", [1024, 2048, 4096])
@pytest.mark.parametrize("N", [1024, 2048])
@pytest.mark.parametrize("K", [256, 512, 1024])
def test_int8_example_sweep_exact(M, N, K):
    g = torch.Generator().manual_seed(M + 7 * N + 13 * K)
    a = torch.randint(-128, 128, (M, K), generator=g, dtype=torch.int8)
    b = torch.randint(-128, 128, (K, N), generator=g, dtype=torch.int8)
    c = torch.full((M, N), -1, dtype=torch.int32)
    grid = (triton_cdiv(M, 128), triton_cdiv(N, 64))
    kernels.bare_matmul_i8[grid](a, b, c, M, N, K, a.stride(0), a.stride(1), b.stride(0), b.stride(1), c.stride(0),
                                 c.stride(1), BLOCK_SIZE_M=128, BLOCK_SIZE_N=64, BLOCK_SIZE_K=K)
    assert c.device.type == "cpu"
    torch.testing.assert_close(c, cgemm.gemm_int(a, b), atol=0, rtol=0)  # the example's own check


def triton_cdiv(x, y):
    return (x + y - 1) // y


# ---------------------------------------------------------------- integer GEMM sweep


def _int_operands(kind, M, N, K, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    lo, hi, dt = (-2 ** 15, 2 ** 15, torch.int16) if kind == "i16" else (-128, 128, torch.int8)
    a = torch.randint(lo, hi, (M, K), generator=g, device="cuda", dtype=dt)
    if kind == "i8nt":  # W [N, K]
        b = torch.randint(lo, hi, (N, K), generator=g, device="cuda", dtype=dt)
    else:
        b = torch.randint(lo, hi, (K, N), generator=g, device="cuda", dtype=dt)
    return a, b


def _int_run(kind, a, b):
    if kind == "i8":
        return ops.matmul_i8(a, b)
    if kind == "i8nt":
        return ops.linear_i8(a, b)
    return ops.matmul_i16(a, b)


def _b_rowmajor(kind, b):
    """B as [K, N] row-major (the oracle's layout)."""
    return b.t().contiguous() if kind == "i8nt" else b


@pytest.mark.parametrize("kind", ["i8", "i8nt", "i16"])
@pytest.mark.parametrize("M,N,K", SMALL)
def test_int_sweep_exact(kind, M, N, K):
    a, b = _int_operands(kind, M, N, K, M + N + K)
    c = _int_run(kind, a, b)
    assert torch.equal(c.cpu(), cgemm.gemm_int(a.cpu(), _b_rowmajor(kind, b).cpu()))
    _ok()
    del a, b, c
    _free()


@pytest.mark.parametrize("kind", ["i8", "i8nt", "i16"])
@pytest.mark.parametrize("M,N,K", LARGE)
def test_int_sweep_checksums_and_samples(kind, M, N, K):
    a, b = _int_operands(kind, M, N, K, 3 * M + K)
    c = _int_run(kind, a, b)
    torch.cuda.synchronize()
    _ok()
    bk = _b_rowmajor(kind, b)  # [K, N]
    del b
    # every element: row and column checksums, exact in int64, compared mod 2^32
    b_rowsum = bk.to(torch.int64).sum(1)  # [K]
    want_rows = torch.zeros(M, dtype=torch.int64, device="cuda")
    for r0 in range(0, M, 2048):  # bounded int64 temporaries
        want_rows[r0:r0 + 2048] = (a[r0:r0 + 2048].to(torch.int64) * b_rowsum).sum(1)
    got_rows = c.to(torch.int64).sum(1) if M <= 8192 else torch.cat(
        [c[r0:r0 + 2048].to(torch.int64).sum(1) for r0 in range(0, M, 2048)])
    assert torch.equal(got_rows % MOD, want_rows % MOD), "row checksums differ"
    a_colsum = a.to(torch.int64).sum(0)  # [K]
    want_cols = torch.zeros(N, dtype=torch.int64, device="cuda")
    for k0 in range(0, K, 2048):
        want_cols += (a_colsum[k0:k0 + 2048, None] * bk[k0:k0 + 2048].to(torch.int64)).sum(0)
    got_cols = torch.zeros(N, dtype=torch.int64, device="cuda")
    for r0 in range(0, M, 2048):
        got_cols += c[r0:r0 + 2048].to(torch.int64).sum(0)
    assert torch.equal(got_cols % MOD, want_cols % MOD), "column checksums differ"
    # sampled rows (first, last, random) and columns against the C oracle
    gen = torch.Generator().manual_seed(M + N)
    rows = torch.unique(torch.cat([torch.tensor([0, M - 1]), torch.randint(0, M, (6,), generator=gen)]))
    assert torch.equal(c[rows.cuda()].cpu(), cgemm.gemm_int(a[rows.cuda()].cpu(), bk.cpu()))
    if M >= 256:
        cols = torch.unique(torch.cat([torch.tensor([0, N - 1]), torch.randint(0, N, (6,), generator=gen)]))
        r_blk = slice(M // 2 - 128, M // 2 + 128)  # a 256-row band (C oracle cost bounded)
        want = cgemm.gemm_int(a[r_blk].cpu(), bk[:, cols.cuda()].contiguous().cpu())
        assert torch.equal(c[r_blk][:, cols.cuda()].cpu(), want)
    del a, bk, c
    _free()


# ---------------------------------------------------------------- bf16 GEMM sweep


def _bf16_tol(K):
    return dict(atol=1e-2 * math.sqrt(K) * 0.1, rtol=2 ** -7)


@pytest.mark.parametrize("M,N,K", SWEEP)
def test_bf16_sweep(M, N, K):
    g = torch.Generator(device="cuda").manual_seed(M + 5 * K)
    a = torch.randn((M, K), generator=g, device="cuda").to(torch.bfloat16)
    b = torch.randn((K, N), generator=g, device="cuda").to(torch.bfloat16)
    c = ops.matmul_bf16(a, b, torch.bfloat16)
    torch.cuda.synchronize()
    _ok()
    old = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False  # the reference product in true fp32
    try:
        if M * N * K <= 1024 ** 3 or M <= 64:
            ref = (a.float() @ b.float()).to(torch.bfloat16)
            torch.testing.assert_close(c.float(), ref.float(), **_bf16_tol(K))
        else:
            gen = torch.Generator().manual_seed(N)
            rows = torch.unique(torch.cat([torch.tensor([0, M - 1]), torch.randint(0, M, (14,), generator=gen)]))
            rows = rows.cuda()
            ref = (a[rows].float() @ b.float()).to(torch.bfloat16)
            torch.testing.assert_close(c[rows].float(), ref.float(), **_bf16_tol(K))
            cols = torch.unique(torch.cat([torch.tensor([0, N - 1]), torch.randint(0, N, (6,), generator=gen)]))
            cols = cols.cuda()
            ref = (a.float() @ b[:, cols].float()).to(torch.bfloat16)
            torch.testing.assert_close(c[:, cols].float(), ref.float(), **_bf16_tol(K))
    finally:
        torch.backends.cuda.matmul.allow_tf32 = old
    del a, b, c
    _free()


# ---------------------------------------------------------------- Qwen2.5 workload shape


def test_qwen_workload_shape_two_sequences_match_oracle():
    """Batch 64 x 512 (the benchmark's prefill, tiled GEMMs over 32768 rows),
    then three teacher-forced decode steps at batch 64 (the one-launch decode
    kernels); sequences 0 and 41 against the oracle forward of those two
    sequences alone (sequences are independent)."""
    from oracle.qwen import OracleQwen
    from test_qwen_gpu import _cmp
    from xb200.qwen import Qwen2Model, QwenConfig, random_weights

    cfg = QwenConfig()
    sd = random_weights(cfg, seed=0)
    B, S, steps = 64, 512, 3
    ids = torch.randint(0, cfg.vocab_size, (B, S + steps), generator=torch.Generator().manual_seed(9))
    pick = torch.tensor([0, 41])
    model = Qwen2Model(sd, cfg, rope_len=1024)
    cache = model.new_cache(B, S + steps)
    logits = model.forward(ids[:, :S].cuda(), cache)  # [64, 512, vocab] fp32
    got_pre = logits[pick.cuda()].cpu()
    del logits
    got_dec = [model.forward(ids[:, t:t + 1].cuda(), cache, last_only=True)[pick.cuda()].cpu()
               for t in range(S, S + steps)]
    assert ops.device_status() == 0
    del model, cache
    _free()
    orc = OracleQwen(sd, cfg)
    ocache = orc.new_cache(2, S + steps)
    ref = orc.forward(ids[pick, :S], ocache)
    _cmp(got_pre, ref, cos_min=0.999, rel=0.04)  # the 24-layer bounds of test_qwen_gpu
    for i, t in enumerate(range(S, S + steps)):
        r = orc.forward(ids[pick, t:t + 1], ocache)[:, -1]
        _cmp(got_dec[i], r, cos_min=0.999, rel=0.04)
