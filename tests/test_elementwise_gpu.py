"""Elementwise / activation kernels against the oracle on device tensors.

Covers both dtypes, ragged lengths (vector body + scalar tail), buffers that
are not 16-byte aligned (scalar path), empty and one-element inputs, guard
bands around the output (no out-of-bounds writes), and the full 2^28-element
workload through size-independent properties.
"""

import pytest
import torch

from oracle import ops as O
from xb200 import ops

pytestmark = pytest.mark.gpu

DTYPES = [torch.bfloat16, torch.float32]

UNARY = {
    "relu": (ops.relu, O.relu),
    "leaky_relu": (lambda x, out=None: ops.leaky_relu(x, 0.01, out=out), lambda x: O.leaky_relu(x, 0.01)),
    "gelu": (ops.gelu, O.gelu),
    "gelu_tanh": (ops.gelu_tanh, O.gelu_tanh),
    "sigmoid": (ops.sigmoid, O.sigmoid),
    "silu": (ops.silu, O.silu),
}
BINARY = {
    "vecadd": (ops.vecadd, O.vecadd),
    "axpy": (lambda a, b, out=None: ops.axpy(a, b, 2.5, out=out), lambda a, b: O.axpy(a, b, 2.5)),
    "swiglu": (ops.swiglu, O.swiglu),
}
EXACT = {"relu", "leaky_relu", "vecadd", "axpy"}


def _x(n, dtype, seed, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(n, generator=g) * scale).to(dtype)


def _check(name, got, ref):
    if name in EXACT:
        assert torch.equal(got.cpu(), ref), name
    elif ref.dtype == torch.bfloat16:
        torch.testing.assert_close(got.cpu().float(), ref.float(), atol=1e-6, rtol=2 ** -7)
    else:
        torch.testing.assert_close(got.cpu(), ref, atol=1e-6, rtol=3e-6)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("n", [1, 7, 4096, (1 << 20) + 37])
@pytest.mark.parametrize("name", sorted(UNARY))
def test_unary(name, n, dtype):
    fn, ref = UNARY[name]
    x = _x(n, dtype, n, scale=3.0)
    got = fn(x.cuda())
    _check(name, got, ref(x))


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("n", [1, 9, 8192, (1 << 20) + 13])
@pytest.mark.parametrize("name", sorted(BINARY))
def test_binary(name, n, dtype):
    fn, ref = BINARY[name]
    a, b = _x(n, dtype, 2 * n), _x(n, dtype, 2 * n + 1)
    got = fn(a.cuda(), b.cuda())
    _check(name, got, ref(a, b))


@pytest.mark.parametrize("dtype", DTYPES)
def test_unaligned_buffers_take_the_scalar_path(dtype):
    n = 10001
    x = _x(n + 1, dtype, 3, scale=3.0)
    xd = x.cuda()[1:]  # 2 or 4 bytes past a 16-byte boundary
    out = torch.empty(n + 1, dtype=dtype, device="cuda")[1:]
    ops.silu(xd, out=out)
    _check("silu", out, O.silu(x[1:]))
    a, b = _x(n + 1, dtype, 4), _x(n + 1, dtype, 5)
    got = ops.vecadd(a.cuda()[1:], b.cuda()[1:])
    _check("vecadd", got, O.vecadd(a[1:], b[1:]))


@pytest.mark.parametrize("dtype", DTYPES)
def test_guard_bands_untouched(dtype):
    n = 12345
    x = _x(n, dtype, 6)
    buf = torch.full((n + 64,), 7.0, dtype=dtype, device="cuda")
    ops.sigmoid(x.cuda(), out=buf[32:32 + n])
    assert torch.all(buf[:32] == 7.0) and torch.all(buf[32 + n:] == 7.0)


def test_empty_input():
    x = torch.empty(0, dtype=torch.bfloat16, device="cuda")
    assert ops.relu(x).numel() == 0
    assert ops.vecadd(x, x).numel() == 0


def test_special_values():
    x = torch.tensor([0.0, -0.0, float("inf"), float("-inf"), float("nan"), 88.0, -88.0, 1e-30, -1e-30],
                     dtype=torch.float32)
    for name in ("relu", "leaky_relu", "sigmoid", "silu"):
        fn, ref = UNARY[name]
        got = fn(x.cuda()).cpu()
        exp = ref(x)
        assert torch.allclose(got, exp, equal_nan=True, atol=0, rtol=1e-6), (name, got, exp)


def test_full_size_properties_bf16():
    """The 2^28-element workload: properties that hold at any size."""
    n = 1 << 28
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(n, generator=g, device="cuda", dtype=torch.float32).to(torch.bfloat16)
    y = torch.randn(n, generator=g, device="cuda", dtype=torch.float32).to(torch.bfloat16)
    r = ops.relu(x)
    assert torch.equal(ops.relu(r), r)  # idempotent
    assert torch.equal(r, torch.clamp_min(x, 0))
    assert torch.equal(ops.vecadd(x, y), ops.vecadd(y, x))  # commutative
    assert torch.equal(ops.vecadd(x, y), x + y)  # same rounding as torch's bf16 add
    s = ops.sigmoid(x).float()
    assert float(s.min()) >= 0.0 and float(s.max()) <= 1.0
    # silu(x) == x * sigmoid(x) up to one rounding each
    torch.testing.assert_close(ops.silu(x).float(), (x.float() * torch.sigmoid(x.float())), atol=1e-2, rtol=1e-2)
    del x, y, r, s
    torch.cuda.empty_cache()
