"""The reference-signature launchers on pinned host tensors: launches cut into
pieces whose uploads, kernels and downloads overlap on three streams must
give exactly the result of the same operator on device-resident tensors, and
leave the output's unwritten elements as they were."""

import pytest
import torch

from xb200 import kernels, ops

pytestmark = pytest.mark.gpu


@pytest.fixture
def small_pieces(monkeypatch):
    # a few tens of KB per piece, so even modest tensors take many pieces
    monkeypatch.setattr(kernels, "_PIECE_BYTES", 48 << 10)


def _pinned(t):
    return t.contiguous().pin_memory()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("n", [4096 * 7 + 123, 200_000])
def test_elementwise_pieces_match_device_path(small_pieces, dtype, n):
    g = torch.Generator().manual_seed(n)
    x = _pinned(torch.randn(n + 50, generator=g).to(dtype))
    y = _pinned(torch.randn(n + 50, generator=g).to(dtype))
    dx, dy = x.cuda(), y.cuda()
    cases = [
        (kernels.vecadd, (x, y), lambda o: ops.vecadd(dx[:n], dy[:n], out=o), {"BLOCK_SIZE_N": 1024}),
        (kernels.axpy_kernel, (x, y), lambda o: ops.axpy(dx[:n], dy[:n], 2.5, out=o), None),
        (kernels.relu_kernel, (x,), lambda o: ops.relu(dx[:n], out=o), None),
        (kernels.gelu_kernel_gpu, (x,), lambda o: ops.gelu_tanh(dx[:n], out=o), None),
        (kernels.silu_kernel, (x,), lambda o: ops.silu(dx[:n], out=o), None),
        (kernels.swiglu_kernel, (x, y), lambda o: ops.swiglu(dx[:n], dy[:n], out=o), None),
    ]
    for k, ins, dev_fn, kw in cases:
        out = _pinned(torch.full((n + 50,), 7.0, dtype=dtype))
        args = list(ins) + [out]
        if k is kernels.axpy_kernel:
            args.append(2.5)
        args.append(n)
        k[(max(1, n // 1024),)](*args, **(kw or {"BLOCK_SIZE": 1024}))
        want = torch.empty(n, dtype=dtype, device="cuda")
        dev_fn(want)
        assert torch.equal(out[:n], want.cpu()), k.name
        assert torch.all(out[n:] == 7.0), f"{k.name} wrote past n_elements"


def test_in_place_launch_on_pinned_memory(small_pieces):
    n = 100_003
    x = _pinned(torch.randn(n, generator=torch.Generator().manual_seed(1)))
    want = ops.relu(x.cuda()).cpu()
    kernels.relu_kernel[(n // 1024 + 1,)](x, x, n, BLOCK_SIZE=1024)
    assert torch.equal(x, want)


def test_row_kernels_in_pieces(small_pieces):
    g = torch.Generator().manual_seed(2)
    rows, cols, pitch = 1024, 96, 128
    x = _pinned(torch.randn(rows, pitch, generator=g))
    out = _pinned(torch.full((rows, cols), -3.0))
    kernels.softmax_kernel[(rows // 4,)](x, out, pitch, 1, cols, 1, cols, BLOCK_SIZE=4)
    assert torch.equal(out, ops.softmax(x.cuda()[:, :cols]).cpu())

    w = _pinned(torch.randn(cols, generator=g))
    xr = _pinned(torch.randn(rows, cols, generator=g))
    yr = _pinned(torch.zeros(rows, cols))
    kernels.weighted_rms_norm_kernel[(rows // 8,)](xr, w, yr, cols, 1e-6, BLOCK_M=8, BLOCK_N=cols)
    assert torch.equal(yr, ops.rms_norm(xr.cuda(), w.cuda(), 1e-6).cpu())

    planes, H, W = 300, 16, 24
    p = _pinned(torch.randn(planes, H, W, generator=g))
    q = _pinned(torch.zeros(planes, H // 2, W // 2))
    kernels.avg_pool2d_kernel[(planes,)](p, q, planes, H, W, BLOCK=1)
    assert torch.equal(q, ops.avg_pool2d_2x2(p.cuda()).cpu())


def test_gemm_rows_in_pieces(small_pieces):
    g = torch.Generator().manual_seed(3)
    M, N, K = 1000, 256, 512
    a = _pinned(torch.randint(-128, 128, (M, K), generator=g, dtype=torch.int8))
    b = _pinned(torch.randint(-128, 128, (K, N), generator=g, dtype=torch.int8))
    c = _pinned(torch.zeros(M, N, dtype=torch.int32))
    kernels.bare_matmul_i8[(8, 4)](a, b, c, M, N, K, K, 1, N, 1, N, 1, 128, 64, 64)
    assert torch.equal(c, a.int() @ b.int())  # integer products: exact whatever the piece sizes

    ab = _pinned(torch.randn(M, K, generator=g).bfloat16())
    bb = _pinned(torch.randn(K, N, generator=g).bfloat16())
    cb = _pinned(torch.zeros(M, N, dtype=torch.bfloat16))
    kernels.bare_matmul[(8, 4)](ab, bb, cb, M, N, K, K, 1, N, 1, N, 1, 128, 64, 64)
    ref = ab.float() @ bb.float()
    torch.testing.assert_close(cb.float(), ref, atol=0.05, rtol=2 ** -7)


def test_pageable_host_tensors_take_one_piece():
    n = 50_000
    x = torch.randn(n, generator=torch.Generator().manual_seed(4))
    out = torch.full((n + 10,), 5.0)
    kernels.sigmoid_kernel[(n // 1024 + 1,)](x, out, n, BLOCK_SIZE=1024)
    assert torch.equal(out[:n], ops.sigmoid(x.cuda()).cpu())
    assert torch.all(out[n:] == 5.0)
