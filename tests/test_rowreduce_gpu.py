"""Row reductions (softmax, layernorm, rms_norm, weighted rms_norm, row centering)
and 2x2 average pooling against the oracle on device tensors.

Shapes cover the examples' (256 and 32/64 x 256), the Qwen hidden size (896),
the workload's 4096 columns, the register-path boundaries (many group sizes),
ragged columns and padded row strides (scalar fallback), and the full
[32768, 4096] workload through size-independent properties.
"""

import pytest
import torch

from oracle import ops as O
from xb200 import ops

pytestmark = pytest.mark.gpu

DTYPES = [torch.bfloat16, torch.float32]
SHAPES = [(1, 8), (3, 64), (32, 256), (64, 256), (256, 256), (17, 896), (33, 1000), (64, 4096), (8, 8200),
          (5, 16384), (2, 40000)]


def _x(shape, dtype, seed, scale=3.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=g) * scale).to(dtype)


def _param(n, dtype, seed, mean, std):
    g = torch.Generator().manual_seed(seed)
    return (mean + std * torch.randn(n, generator=g)).to(dtype)


def _close(got, ref):
    got = got.cpu()
    if ref.dtype == torch.bfloat16:
        torch.testing.assert_close(got.float(), ref.float(), atol=2e-6, rtol=2 ** -7)
    else:
        torch.testing.assert_close(got, ref, atol=2e-6, rtol=2e-5)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("shape", SHAPES)
def test_softmax(shape, dtype):
    x = _x(shape, dtype, shape[1])
    _close(ops.softmax(x.cuda()), O.softmax(x))


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("shape", SHAPES)
def test_layernorm_affine(shape, dtype):
    x = _x(shape, dtype, shape[1] + 1)
    gma = _param(shape[1], dtype, 1, 1.0, 0.1)
    bta = _param(shape[1], dtype, 2, 0.0, 0.1)
    got = ops.layernorm(x.cuda(), gma.cuda(), bta.cuda(), 1e-5)
    ref = O.layernorm(x, gma, bta, 1e-5)
    got = got.cpu().float()
    # (x - mean) * rstd differs in its last fp32 bits by summation order; the
    # bf16 rounding can then land one ulp apart.
    tol = dict(atol=1e-2, rtol=1e-2) if dtype == torch.bfloat16 else dict(atol=2e-5, rtol=2e-5)
    torch.testing.assert_close(got, ref.float(), **tol)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("shape", SHAPES)
def test_rms_norm(shape, dtype):
    x = _x(shape, dtype, shape[1] + 2)
    _close(ops.rms_norm(x.cuda(), None, 1e-6), O.rms_norm(x, 1e-6))


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("shape", SHAPES)
def test_weighted_rms_norm(shape, dtype):
    x = _x(shape, dtype, shape[1] + 3)
    w = _param(shape[1], dtype, 3, 1.0, 0.1)
    got = ops.rms_norm(x.cuda(), w.cuda(), 1e-6)
    ref = O.weighted_rms_norm(x, w, 1e-6)
    _close(got, ref)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("shape", SHAPES)
def test_row_center(shape, dtype):
    x = _x(shape, dtype, shape[1] + 4)
    got = ops.row_center(x.cuda()).cpu().float()
    ref = O.row_center(x).float()
    tol = dict(atol=2e-2, rtol=1e-2) if dtype == torch.bfloat16 else dict(atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(got, ref, **tol)


@pytest.mark.parametrize("dtype", DTYPES)
def test_padded_row_stride(dtype):
    base = _x((48, 272), dtype, 9)
    x = base[:, :256]  # row stride 272, not contiguous
    y = torch.full((48, 300), 5.0, dtype=dtype, device="cuda")
    ops.softmax(x.cuda(), out=y[:, :256])
    _close(y[:, :256], O.softmax(x))
    assert torch.all(y[:, 256:] == 5.0)
    ops.rms_norm(x.cuda(), None, 1e-5, out=y[:, 10:266])  # misaligned output rows: scalar path
    _close(y[:, 10:266], O.rms_norm(x, 1e-5))


def test_softmax_extreme_rows():
    x = torch.tensor([[1e4, 0.0, -1e4, 3.0], [-1e30, -1e30, -1e30, -1e30], [0.0, 0.0, 0.0, 0.0]], dtype=torch.float32)
    _close(ops.softmax(x.cuda()), O.softmax(x))


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("shape", [(2, 3, 8, 8), (1, 4, 224, 224), (3, 2, 7, 9), (2, 1, 6, 20)])
def test_avg_pool2d(shape, dtype):
    x = _x(shape, dtype, 11, scale=1.0)
    got = ops.avg_pool2d_2x2(x.cuda())
    ref = O.avg_pool2d_2x2(x)
    assert got.shape == ref.shape
    if dtype == torch.float32:
        assert torch.equal(got.cpu(), ref)
    else:
        _close(got, ref)


def test_full_size_row_properties():
    """[32768, 4096] bf16: rows of softmax sum to 1, rms_norm rows have unit
    mean square, row_center rows have zero mean, layernorm rows zero mean and
    unit variance -- all within bf16 rounding."""
    g = torch.Generator(device="cuda").manual_seed(0)
    x = (torch.randn(32768, 4096, generator=g, device="cuda") * 3).to(torch.bfloat16)
    s = ops.softmax(x).float()
    torch.testing.assert_close(s.sum(-1), torch.ones(32768, device="cuda"), atol=2e-2, rtol=0)
    r = ops.rms_norm(x, None, 1e-6).float()
    torch.testing.assert_close((r * r).mean(-1), torch.ones(32768, device="cuda"), atol=1e-2, rtol=0)
    c = ops.row_center(x).float()
    assert float(c.mean(-1).abs().max()) < 2e-2
    ln = ops.layernorm(x, None, None, 1e-5).float()
    assert float(ln.mean(-1).abs().max()) < 1e-2
    torch.testing.assert_close(ln.var(-1, unbiased=False), torch.ones(32768, device="cuda"), atol=2e-2, rtol=0)
    # spot-check 64 rows against the oracle
    idx = torch.randint(0, 32768, (64,), generator=torch.Generator().manual_seed(1))
    xs = x[idx.cuda()].cpu()
    _close(s[idx.cuda()].to(torch.bfloat16), O.softmax(xs))
    del x, s, r, c, ln
    torch.cuda.empty_cache()
