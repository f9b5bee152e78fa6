"""The allocation-free int16 GEMM entry point, through the C ABI.

xb_matmul_i16_noalloc serves callers that cannot allocate device memory:
plugins whose host framework owns every device allocation through its own
pool, and latency-bound paths where a cudaMalloc may synchronise the device.
Its limb planes live in a scratch array built into the library instead of a
caller workspace.  Its output must equal xb_matmul_i16's exactly (both are
exact int32 products) and the C oracle's int32 (mod 2^32) product, on two
calls in a row that share that scratch array.  This file is named to run
last, so a stop-at-first-failure run has already run every other test.
"""

import ctypes

import pytest
import torch

from xb200 import _lib

pytestmark = pytest.mark.gpu

SCRATCH_MAX = 32 * 1024 * 1024  # XB_I16_NOALLOC_SCRATCH_BYTES


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _with_workspace(a, b):
    M, K = a.shape
    N = b.shape[1]
    need = ctypes.c_size_t(0)
    _lib.call("xb_matmul_i16_workspace_size", M, N, K, ctypes.byref(need))
    ws = torch.empty(need.value, dtype=torch.uint8, device="cuda")
    c = torch.empty((M, N), dtype=torch.int32, device="cuda")
    _lib.call("xb_matmul_i16", a.data_ptr(), b.data_ptr(), c.data_ptr(), M, N, K, K, N, N, ws.data_ptr(),
              need.value, _stream())
    return c


def _no_alloc(a, b):
    M, K = a.shape
    N = b.shape[1]
    c = torch.full((M, N), -7, dtype=torch.int32, device="cuda")
    _lib.call("xb_matmul_i16_noalloc", a.data_ptr(), b.data_ptr(), c.data_ptr(), M, N, K, K, N, N, _stream())
    return c


def _pair(M, N, K, seed):
    g = torch.Generator().manual_seed(seed)
    a = torch.randint(-2**15, 2**15, (M, K), generator=g, dtype=torch.int16).cuda()
    b = torch.randint(-2**15, 2**15, (K, N), generator=g, dtype=torch.int16).cuda()
    return a, b


def test_no_alloc_matches_workspace_entry_point_and_oracle_twice():
    from oracle import cgemm

    # Two different products back to back through the shared scratch array;
    # the second is smaller, so stale limbs of the first are left beyond it.
    for (M, N, K), seed in (((384, 256, 1024), 1), ((130, 144, 272), 2)):
        a, b = _pair(M, N, K, seed)
        got = _no_alloc(a, b)
        ref = _with_workspace(a, b)
        torch.cuda.synchronize()
        assert torch.equal(got, ref), f"{M}x{N}x{K}: no-alloc result differs from xb_matmul_i16"
        assert torch.equal(got.cpu(), cgemm.gemm_int(a.cpu(), b.cpu())), \
            f"{M}x{N}x{K}: no-alloc result differs from the C oracle"
    st = ctypes.c_int(0)
    _lib.call("xb_device_status", _stream(), ctypes.byref(st))
    assert st.value == 0


def test_no_alloc_largest_product_within_the_scratch_array():
    """A product that fills most of the array (K ragged), against the oracle:
    checks the size guard lets through everything it should."""
    from oracle import cgemm

    M, N, K = 2048, 2048, 3000
    need = ctypes.c_size_t(0)
    _lib.call("xb_matmul_i16_workspace_size", M, N, K, ctypes.byref(need))
    assert SCRATCH_MAX // 2 < need.value <= SCRATCH_MAX
    a, b = _pair(M, N, K, 3)
    got = _no_alloc(a, b)
    torch.cuda.synchronize()
    rows = torch.tensor([0, 1, 777, 2047])
    assert torch.equal(got.cpu()[rows], cgemm.gemm_int(a.cpu()[rows], b.cpu()))
    # every element through exact int64 checksums reduced mod 2^32
    a64, b64 = a.cpu().to(torch.int64), b.cpu().to(torch.int64)
    want_rows = (a64 @ b64.sum(1)) % 2**32
    want_cols = (a64.sum(0) @ b64) % 2**32
    g64 = got.cpu().to(torch.int64)
    assert torch.equal(g64.sum(1) % 2**32, want_rows)
    assert torch.equal(g64.sum(0) % 2**32, want_cols)


def test_no_alloc_rejects_products_beyond_the_scratch_array():
    M = N = K = 4096  # needs 64 MiB of limb planes, twice the built-in array
    need = ctypes.c_size_t(0)
    _lib.call("xb_matmul_i16_workspace_size", M, N, K, ctypes.byref(need))
    assert need.value > SCRATCH_MAX
    a = torch.zeros((M, K), dtype=torch.int16, device="cuda")
    b = torch.zeros((K, N), dtype=torch.int16, device="cuda")
    c = torch.zeros((M, N), dtype=torch.int32, device="cuda")
    with pytest.raises(_lib.XbError) as e:
        _lib.call("xb_matmul_i16_noalloc", a.data_ptr(), b.data_ptr(), c.data_ptr(), M, N, K, K, N, N, _stream())
    assert e.value.code == _lib.XB_ERR_UNSUPPORTED
    assert "scratch" in e.value.message
