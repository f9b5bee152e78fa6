"""tcgen05 GEMMs against the oracle.

int8 / int16 are bit-exact (int32 accumulation, wrap-around mod 2^32 for
int16).  bf16 uses the autotune example's tolerance rule
(examples/autotune-matmul/matmul.py:105-115: atol 1.5e-3 * sqrt(8192 / K),
rtol 1.6e-2, inputs scaled by 1/sqrt(K)) against an fp32 product of the same
bf16 inputs.  Full-size shapes are checked exactly through row and column
checksums (C 1 = A (B 1), 1^T C = (1^T A) B) in float64, which is exact at
these magnitudes.
"""

import math

import pytest
import torch

from oracle import cgemm
from oracle import ops as O
from xb200 import ops

pytestmark = pytest.mark.gpu


def _rand_int(shape, lo, hi, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(lo, hi, shape, generator=g, dtype=dtype)


def _status_ok():
    assert ops.device_status() == 0


I8_SHAPES = [(128, 64, 64), (256, 128, 256), (1024, 1024, 256), (200, 304, 176), (16, 512, 1024), (1, 16, 16),
             (300, 640, 4096), (129, 257 + 15, 48)]


@pytest.mark.parametrize("M,N,K", I8_SHAPES)
def test_matmul_i8_exact(M, N, K):
    if (N % 16) or (K % 16):
        pytest.skip("TMA row pitch must be a multiple of 16 bytes")
    a = _rand_int((M, K), -128, 128, torch.int8, M * 7 + K)
    b = _rand_int((K, N), -128, 128, torch.int8, N * 3 + K)
    c = ops.matmul_i8(a.cuda(), b.cuda())
    assert torch.equal(c.cpu(), cgemm.gemm_int(a, b))
    _status_ok()


def test_matmul_i8_padded_leading_dims_and_guard_bands():
    M, N, K = 130, 272, 96
    a_full = _rand_int((M, K + 32), -128, 128, torch.int8, 1)
    b_full = _rand_int((K, N + 48), -128, 128, torch.int8, 2)
    a, b = a_full[:, :K], b_full[:, :N]
    c_full = torch.full((M + 2, N + 40), 12345, dtype=torch.int32, device="cuda")
    c = c_full[1:M + 1, 8:N + 8]
    ops.matmul_i8(a_full.cuda()[:, :K], b_full.cuda()[:, :N], out=c)
    assert torch.equal(c.cpu(), cgemm.gemm_int(a.contiguous(), b.contiguous()))
    c_cpu = c_full.cpu()
    assert torch.all(c_cpu[0] == 12345) and torch.all(c_cpu[-1] == 12345)
    assert torch.all(c_cpu[:, :8] == 12345) and torch.all(c_cpu[:, N + 8:] == 12345)


I16_SHAPES = [(128, 128, 64), (256, 256, 512), (100, 144, 80), (16, 256, 1024), (384, 128, 1000)]


@pytest.mark.parametrize("M,N,K", I16_SHAPES)
def test_matmul_i16_exact(M, N, K):
    a = _rand_int((M, K), -2**15, 2**15, torch.int16, M + K)
    b = _rand_int((K, N), -2**15, 2**15, torch.int16, N + 2 * K)
    c = ops.matmul_i16(a.cuda(), b.cuda())
    assert torch.equal(c.cpu(), cgemm.gemm_int(a, b))
    _status_ok()


def test_matmul_i16_wraps_mod_2_32():
    # extreme values: every partial product is 2^30, sums leave int32 range
    M, N, K = 128, 128, 4096
    a = torch.full((M, K), -2**15, dtype=torch.int16)
    b = torch.full((K, N), -2**15, dtype=torch.int16)
    a[1::2] = 2**15 - 1
    b[:, ::3] = 12345
    c = ops.matmul_i16(a.cuda(), b.cuda())
    assert torch.equal(c.cpu(), O.matmul_int_exact(a, b))
    _status_ok()


BF16_SHAPES = [(256, 256, 256), (512, 384, 320), (1024, 1024, 1024), (200, 264, 136), (16, 1024, 2048),
               (128, 256, 8192)]


@pytest.mark.parametrize("M,N,K", BF16_SHAPES)
def test_matmul_bf16_f32_out(M, N, K):
    g = torch.Generator().manual_seed(M * N + K)
    s = 1.0 / math.sqrt(K)
    a = (torch.randn((M, K), generator=g) * s).to(torch.bfloat16)
    b = (torch.randn((K, N), generator=g) * s).to(torch.bfloat16)
    c = ops.matmul_bf16(a.cuda(), b.cuda(), torch.float32).cpu()
    ref = O.matmul_bf16_f32acc(a, b)
    atol = 1.5e-3 * math.sqrt(8192 / K)
    torch.testing.assert_close(c, ref, atol=atol, rtol=1.6e-2)
    # much tighter in practice: fp32 accumulation of the same products
    assert float((c - ref).abs().max()) < 1e-4 * max(1.0, float(ref.abs().max()))
    _status_ok()


@pytest.mark.parametrize("M,N,K", [(256, 512, 256), (100, 200, 64), (4096, 4096, 4096)])
def test_matmul_bf16_bf16_out(M, N, K):
    g = torch.Generator().manual_seed(K)
    a = torch.randn((M, K), generator=g).to(torch.bfloat16)
    b = torch.randn((K, N), generator=g).to(torch.bfloat16)
    c = ops.matmul_bf16(a.cuda(), b.cuda(), torch.bfloat16).cpu().float()
    ref = O.matmul_bf16_f32acc(a, b).to(torch.bfloat16).float()
    torch.testing.assert_close(c, ref, atol=1e-2 * math.sqrt(K) * 0.1, rtol=2 ** -7)


@pytest.mark.parametrize("M,N,K", [(64, 896, 896), (512, 1152, 896), (33, 4864, 896), (128, 896, 4864)])
def test_linear_bias(M, N, K):
    g = torch.Generator().manual_seed(N + K)
    x = torch.randn((M, K), generator=g).to(torch.bfloat16)
    w = (torch.randn((N, K), generator=g) * 0.02).to(torch.bfloat16)
    bias = (torch.randn(N, generator=g) * 0.1).to(torch.bfloat16)
    y = ops.linear(x.cuda(), w.cuda(), bias.cuda()).cpu().float()
    ref = (x.float() @ w.float().t() + bias.float()).to(torch.bfloat16).float()
    torch.testing.assert_close(y, ref, atol=2e-3, rtol=2 ** -7)
    y2 = ops.linear(x.cuda(), w.cuda(), None).cpu().float()
    ref2 = (x.float() @ w.float().t()).to(torch.bfloat16).float()
    torch.testing.assert_close(y2, ref2, atol=2e-3, rtol=2 ** -7)


def test_zero_k_gives_zeros():
    a = torch.empty((5, 0), dtype=torch.int8, device="cuda")
    b = torch.empty((0, 7), dtype=torch.int8, device="cuda")
    c = ops.matmul_i8(a, b)
    assert torch.equal(c.cpu(), torch.zeros(5, 7, dtype=torch.int32))


def test_unaligned_pitch_is_rejected():
    from xb200 import XbError

    a = torch.zeros((8, 24), dtype=torch.int8, device="cuda")
    b = torch.zeros((24, 8), dtype=torch.int8, device="cuda")
    with pytest.raises(XbError) as e:
        ops.matmul_i8(a, b)
    assert "16 bytes" in e.value.message


def _checksums_exact(a_dev, b_dev, c_dev):
    af, bf, cf = a_dev.double(), b_dev.double(), c_dev.double()
    row = cf.sum(1)
    col = cf.sum(0)
    assert torch.equal(row, af @ bf.sum(1))
    assert torch.equal(col, af.sum(0) @ bf)


@pytest.mark.parametrize("n", [4096, 8192])
def test_full_size_i8_checksums(n):
    g = torch.Generator(device="cuda").manual_seed(n)
    a = torch.randint(-128, 128, (n, n), generator=g, device="cuda", dtype=torch.int8)
    b = torch.randint(-128, 128, (n, n), generator=g, device="cuda", dtype=torch.int8)
    c = ops.matmul_i8(a, b)
    _checksums_exact(a, b, c)
    # plus an exact spot check of 8 rows against the C oracle
    rows = torch.randperm(n, generator=torch.Generator().manual_seed(1))[:8]
    ref = cgemm.gemm_int(a[rows.cuda()].cpu(), b.cpu())
    assert torch.equal(c[rows.cuda()].cpu(), ref)
    _status_ok()
    del a, b, c
    torch.cuda.empty_cache()


def test_full_size_i16_checksums_mod_2_32():
    n = 4096
    g = torch.Generator(device="cuda").manual_seed(7)
    a = torch.randint(-2**15, 2**15, (n, n), generator=g, device="cuda", dtype=torch.int16)
    b = torch.randint(-2**15, 2**15, (n, n), generator=g, device="cuda", dtype=torch.int16)
    c = ops.matmul_i16(a, b)
    rows = torch.randperm(n, generator=torch.Generator().manual_seed(2))[:4]
    ref = cgemm.gemm_int(a[rows.cuda()].cpu(), b.cpu())
    assert torch.equal(c[rows.cuda()].cpu(), ref)
    _status_ok()


@pytest.mark.parametrize("M,N,K", [(1, 896, 896), (7, 1152, 896), (16, 4864, 896), (64, 896, 4864), (64, 896, 896),
                                   (33, 1000, 200), (64, 151936, 896)])
def test_small_m_linear_matches_tiled_gemm(M, N, K):
    g = torch.Generator().manual_seed(M + N + K)
    x = torch.randn((M, K), generator=g).to(torch.bfloat16).cuda()
    w = (torch.randn((N, K), generator=g) * 0.05).to(torch.bfloat16).cuda()
    b = (torch.randn(N, generator=g) * 0.1).to(torch.bfloat16).cuda()
    ref = (x.float() @ w.float().t() + b.float())
    for dt in (torch.bfloat16, torch.float32):
        y = ops.linear(x, w, b, out_dtype=dt)  # M <= 64: swap-AB split-K path
        torch.testing.assert_close(y.float(), ref, atol=2e-3, rtol=2 ** -7 if dt == torch.bfloat16 else 1e-4)
        y2 = ops.linear(x, w, b, out_dtype=dt)
        assert torch.equal(y, y2)  # fixed-order reduction: bit-repeatable
    _status_ok()


def test_small_m_linear_fuses_residual_like_two_ops():
    M, N, K = 64, 896, 4864
    g = torch.Generator().manual_seed(3)
    x = torch.randn((M, K), generator=g).to(torch.bfloat16).cuda()
    w = (torch.randn((N, K), generator=g) * 0.02).to(torch.bfloat16).cuda()
    r = torch.randn((M, N), generator=g).to(torch.bfloat16).cuda()
    fused = ops.linear(x, w, residual=r)
    lin = ops.linear(x, w)
    two = ops.vecadd(r, lin)  # the same rounding sequence, unfused
    assert torch.equal(fused, two)
    big = torch.randn((100, K), generator=g).to(torch.bfloat16).cuda()  # tiled path: linear then vecadd
    rb = torch.randn((100, N), generator=g).to(torch.bfloat16).cuda()
    assert torch.equal(ops.linear(big, w, residual=rb), ops.vecadd(rb, ops.linear(big, w)))


@pytest.mark.parametrize("M", [1, 8, 64])
def test_small_m_swiglu_equals_unfused(M):
    K, F = 896, 4864
    g = torch.Generator().manual_seed(M)
    x = torch.randn((M, K), generator=g).to(torch.bfloat16).cuda()
    w = (torch.randn((2 * F, K), generator=g) * 0.03).to(torch.bfloat16).cuda()
    fused = ops.linear_swiglu(x, w)
    unfused = ops.silu_mul(ops.linear(x, w[:F]), ops.linear(x, w[F:]))
    # the unfused linears split K differently (N = F vs 2F), so the fp32 sums can
    # differ in the last bits: compare at bf16 level, and exactly where they agree
    torch.testing.assert_close(fused.float(), unfused.float(), atol=1e-3, rtol=2 ** -7)
    assert (fused == unfused).float().mean().item() > 0.95


@pytest.mark.parametrize("M,N,K", [(128, 256, 128), (300, 640, 4096), (16, 8192, 512)])
def test_linear_i8_exact(M, N, K):
    x = _rand_int((M, K), -128, 128, torch.int8, M)
    w = _rand_int((N, K), -128, 128, torch.int8, N)
    y = ops.linear_i8(x.cuda(), w.cuda())
    assert torch.equal(y.cpu(), cgemm.gemm_int(x, w.t().contiguous()))


@pytest.mark.parametrize("M,N,K", [(300, 272, 96), (64, 16, 32)])
def test_four_byte_output_with_unaligned_pitch(M, N, K):
    """C rows whose pitch is not a multiple of 16 bytes cannot be TMA-stored:
    the epilogue falls back to per-thread stores with the same results."""
    a = _rand_int((M, K), -128, 128, torch.int8, 11)
    b = _rand_int((K, N), -128, 128, torch.int8, 12)
    c_full = torch.full((M, N + 1), 777, dtype=torch.int32, device="cuda")
    ops.matmul_i8(a.cuda(), b.cuda(), out=c_full[:, :N])
    assert torch.equal(c_full[:, :N].cpu(), cgemm.gemm_int(a, b))
    assert torch.all(c_full[:, N].cpu() == 777)
    g = torch.Generator().manual_seed(13)
    x = (torch.randn((M, K), generator=g) / 8).to(torch.bfloat16)
    y = (torch.randn((K, N), generator=g) / 8).to(torch.bfloat16)
    f_full = torch.full((M, N + 1), 5.0, dtype=torch.float32, device="cuda")
    ops.matmul_bf16(x.cuda(), y.cuda(), torch.float32, out=f_full[:, :N])
    torch.testing.assert_close(f_full[:, :N].cpu(), O.matmul_bf16_f32acc(x, y), atol=1e-4, rtol=1e-4)
    assert torch.all(f_full[:, N].cpu() == 5.0)
    _status_ok()


@pytest.mark.parametrize("rope", [True, False])
def test_fused_decode_qkv_rope_equals_unfused(rope):
    """linear_rope_kv = linear (fp32 bias, bf16 round) then rope_kv, bit for bit."""
    from oracle.qwen import rope_tables
    B, H, KVH, D, smax, pos, K = 5, 14, 2, 64, 48, 17, 896
    g = torch.Generator().manual_seed(31)
    x = (torch.randn(B, K, generator=g) / 4).to(torch.bfloat16).cuda()
    w = (torch.randn((H + 2 * KVH) * D, K, generator=g) / 16).to(torch.bfloat16).cuda()
    b = (torch.randn((H + 2 * KVH) * D, generator=g) / 4).to(torch.bfloat16).cuda()
    cos, sin = (t.cuda() for t in rope_tables(D, 64, 1e6)) if rope else (None, None)
    outs = []
    for fused in (True, False):
        q = torch.empty((B, H, 1, D), dtype=torch.bfloat16, device="cuda")
        kc = torch.zeros((B, KVH, smax, D), dtype=torch.bfloat16, device="cuda")
        vc = torch.zeros_like(kc)
        if fused:
            ops.linear_rope_kv(x, w, b, cos, sin, q, kc, vc, H, KVH, D, pos)
        else:
            ops.rope_kv(ops.linear(x, w, b), cos, sin, q, kc, vc, B, 1, H, KVH, D, pos)
        outs.append((q.cpu(), kc.cpu(), vc.cpu()))
    for a, c in zip(*outs):
        assert torch.equal(a, c)
    _status_ok()


@pytest.mark.parametrize("kind,N,K,bias", [("rms", 896, 896, False), ("rms", 896, 4864, False),
                                           ("layer", 768, 3072, True), ("layer", 1600, 1600, True)])
def test_fused_decode_residual_norm_equals_unfused(kind, N, K, bias):
    """linear_residual_norm: y bit-identical to linear(residual=...), the norm
    within one bf16 rounding of the row-norm kernel (reduction order)."""
    M = 7
    g = torch.Generator().manual_seed(32)
    x = (torch.randn(M, K, generator=g) / 4).to(torch.bfloat16).cuda()
    w = (torch.randn(N, K, generator=g) / 16).to(torch.bfloat16).cuda()
    bv = (torch.randn(N, generator=g) / 4).to(torch.bfloat16).cuda() if bias else None
    r = torch.randn(M, N, generator=g).to(torch.bfloat16).cuda()
    nw = (1 + 0.1 * torch.randn(N, generator=g)).to(torch.bfloat16).cuda()
    nb = (0.1 * torch.randn(N, generator=g)).to(torch.bfloat16).cuda() if kind == "layer" else None
    y, yn = ops.linear_residual_norm(x, w, bv, r, nw, nb, eps=1e-5, kind=kind)
    y_ref = ops.linear(x, w, bv, residual=r)
    assert torch.equal(y.cpu(), y_ref.cpu())
    yn_ref = ops.rms_norm(y_ref, nw, 1e-5) if kind == "rms" else ops.layernorm(y_ref, nw, nb, 1e-5)
    torch.testing.assert_close(yn.float().cpu(), yn_ref.float().cpu(), atol=2e-2, rtol=8e-3)
    _status_ok()


@pytest.mark.parametrize("M", [100, 300, 1000])
def test_linear_residual_epilogue_equals_linear_then_add(M):
    g = torch.Generator().manual_seed(41)
    x = (torch.randn(M, 896, generator=g) / 4).to(torch.bfloat16).cuda()
    w = (torch.randn(896, 896, generator=g) / 16).to(torch.bfloat16).cuda()
    b = (torch.randn(896, generator=g) / 4).to(torch.bfloat16).cuda()
    r = torch.randn(M, 896, generator=g).to(torch.bfloat16).cuda()
    fused = ops.linear(x, w, b, residual=r)
    unfused = ops.vecadd(ops.linear(x, w, b), r)
    assert torch.equal(fused.cpu(), unfused.cpu())
    _status_ok()


@pytest.mark.parametrize("M", [300, 1000])
def test_linear_residual_epilogue_unaligned_residual(M):
    """A residual whose base is 2 bytes past a 16-byte boundary: the
    whole-line epilogue (16-byte residual pieces) must not take it; the
    per-row path gives the same bits as linear then add."""
    g = torch.Generator().manual_seed(43)
    x = (torch.randn(M, 896, generator=g) / 4).to(torch.bfloat16).cuda()
    w = (torch.randn(896, 896, generator=g) / 16).to(torch.bfloat16).cuda()
    rbig = torch.randn(M * 896 + 8, generator=g).to(torch.bfloat16).cuda()
    r = rbig[1:1 + M * 896].view(M, 896)
    assert r.data_ptr() % 16 == 2
    fused = ops.linear(x, w, None, residual=r)
    unfused = ops.vecadd(ops.linear(x, w, None), r.contiguous())
    assert torch.equal(fused.cpu(), unfused.cpu())
    _status_ok()


@pytest.mark.parametrize("M", [1, 16, 64, 100, 300, 700])
def test_interleaved_swiglu_linear_equals_unfused(M):
    """One GEMM with the SwiGLU in its epilogue (or the small-M split-K form)
    = two linears + silu_mul, bit for bit."""
    g = torch.Generator().manual_seed(42)
    K, F = 896, 4864
    x = (torch.randn(M, K, generator=g) / 4).to(torch.bfloat16).cuda()
    wg = (torch.randn(F, K, generator=g) / 16).to(torch.bfloat16).cuda()
    wu = (torch.randn(F, K, generator=g) / 16).to(torch.bfloat16).cuda()
    w = ops.interleave_gate_up(wg, wu)
    fused = ops.linear_swiglu(x, w, interleaved=True)
    unfused = ops.silu_mul(ops.linear(x, wg), ops.linear(x, wu))
    if M > ops.SMALL_M:  # both run the tiled GEMM: identical accumulation order
        assert torch.equal(fused.cpu(), unfused.cpu())
    else:  # split-K counts differ (N = 2 n_out vs n_out): fp32 sums in another order
        torch.testing.assert_close(fused.float().cpu(), unfused.float().cpu(), atol=1e-3, rtol=2 ** -7)
        assert (fused == unfused).float().mean().item() > 0.95
    _status_ok()


@pytest.mark.parametrize("M", [1, 16, 64, 100, 300])
def test_linear_gelu_epilogue_equals_linear_then_gelu(M):
    g = torch.Generator().manual_seed(43)
    x = (torch.randn(M, 768, generator=g) / 4).to(torch.bfloat16).cuda()
    w = (torch.randn(3072, 768, generator=g) / 8).to(torch.bfloat16).cuda()
    b = (torch.randn(3072, generator=g) / 4).to(torch.bfloat16).cuda()
    fused = ops.linear(x, w, b, act="gelu_tanh")
    unfused = ops.gelu_tanh(ops.linear(x, w, b))
    assert torch.equal(fused.cpu(), unfused.cpu())
    _status_ok()
