"""Host logic of the reference-signature launchers, without a GPU.

The launch path is exercised through XbKernel with a recording ``run``; the
real entry points are covered by the gpu tests."""

import pytest
import torch

from xb200 import kernels


def _fake(record):
    def run(A, B, C, n_elements, BLOCK_SIZE_N, grid):
        record.append(dict(A=A, B=B, C=C, n=n_elements, block=BLOCK_SIZE_N, grid=grid))

    return run


def test_binds_like_the_reference_signature():
    rec = []
    k = kernels.XbKernel("vecadd", "xb_vecadd", _fake(rec))
    assert k.params == ["A", "B", "C", "n_elements", "BLOCK_SIZE_N"]
    a = torch.zeros(8, device="meta")
    res = k[lambda META: (META["n_elements"] // META["BLOCK_SIZE_N"],)](a, a, a, 8, BLOCK_SIZE_N=4)
    assert rec[0]["grid"] == (2, 1, 1)
    assert rec[0]["n"] == 8 and rec[0]["block"] == 4
    assert "ttsharedir" in res.asm


def test_missing_and_unexpected_arguments_raise():
    k = kernels.XbKernel("vecadd", "xb_vecadd", _fake([]))
    a = torch.zeros(8, device="meta")
    with pytest.raises(TypeError):
        k[(1,)](a, a, a, 8)
    with pytest.raises(TypeError):
        k[(1,)](a, a, a, 8, BLOCK_SIZE_N=4, BOGUS=1)
    with pytest.raises(TypeError):
        k[(1,)](a, a, a, 8, 4, BLOCK_SIZE_N=4)


def test_host_tensors_without_cuda_fail_loudly():
    if torch.cuda.is_available():
        pytest.skip("has a GPU")
    a = torch.zeros(8, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        kernels.vecadd[(1,)](a, a, a.clone(), 8, BLOCK_SIZE_N=8)


def test_registry_covers_every_example_kernel():
    assert set(kernels.REGISTRY) >= {
        "vecadd", "axpy_kernel", "relu_kernel", "leaky_relu_kernel", "gelu_kernel", "sigmoid_kernel", "silu_kernel",
        "swiglu_kernel", "avg_pool_kernel", "softmax_kernel", "_layer_norm_fwd_fused", "rms_norm_kernel",
        "weighted_rms_norm_kernel"}


def test_rows_view_checks_size():
    t = torch.zeros(100)
    with pytest.raises(ValueError):
        kernels._rows_view(t, 11, 10, 10)
    v = kernels._rows_view(t, 10, 8, 10)
    assert v.shape == (10, 8) and v.stride() == (10, 1)


def _bound(k, *args, **kw):
    b = k._bind(args, kw)
    return b, [n for n in k.params if isinstance(b[n], torch.Tensor)]


def test_plan_copies_only_what_the_kernel_reads_and_writes():
    x, y = torch.zeros(10000), torch.zeros(10000)
    b, ptrs = _bound(kernels.relu_kernel, x, y, 9000, 1024)
    units, pitch, per, pinned = kernels.relu_kernel._plan(b, (9, 1, 1), ptrs, ptrs)
    assert units == 9000 and pitch == {"X": 1, "Y": 1}
    assert not pinned and per == units  # pageable host memory: one piece


def test_plan_rows_and_shared_pointers():
    x, w, y = torch.zeros(64, 32), torch.zeros(32), torch.zeros(64, 32)
    k = kernels.weighted_rms_norm_kernel
    b, ptrs = _bound(k, x, w, y, 32, 1e-6, BLOCK_M=16, BLOCK_N=32)
    units, pitch, per, _ = k._plan(b, (4, 1, 1), ptrs, ptrs)
    assert units == 64 and pitch == {"X": 32, "Y": 32}  # the weight is read whole
    assert k.split.piece(b, (4, 1, 1), 32) == ({}, (2, 1, 1))


def test_plan_falls_back_to_copying_everything():
    k = kernels.relu_kernel
    x = torch.zeros(4096)
    # output partly overlapping the input
    b, ptrs = _bound(k, x[:2048], x[1024:3072], 1024, 1024)
    assert k._plan(b, (1, 1, 1), ptrs, ptrs) is None
    # an exact in-place launch keeps the split path
    b, ptrs = _bound(k, x, x, 4096, 1024)
    assert k._plan(b, (4, 1, 1), ptrs, ptrs) is not None
    # a non-contiguous pointer
    b, ptrs = _bound(k, torch.zeros(64, 64).t(), torch.zeros(64, 64), 4096, 1024)
    assert k._plan(b, (4, 1, 1), ptrs, ptrs) is None
    # fewer elements than the launch covers: the copy-everything path raises the runner's error
    b, ptrs = _bound(k, torch.zeros(100), torch.zeros(100), 200, 1024)
    assert k._plan(b, (1, 1, 1), ptrs, ptrs) is None
    # a row output whose rows leave gaps (row stride above the written columns)
    sm = kernels.softmax_kernel
    b, ptrs = _bound(sm, torch.zeros(8, 16), torch.zeros(8, 16), 16, 1, 16, 1, 8, 1)
    assert sm._plan(b, (8, 1, 1), ptrs, ptrs) is None
    b, ptrs = _bound(sm, torch.zeros(8, 16), torch.zeros(8, 8), 16, 1, 8, 1, 8, 1)
    assert sm._plan(b, (8, 1, 1), ptrs, ptrs)[1] == {"input_ptr": 16, "output_ptr": 8}


def test_plan_piece_sizes():
    k = kernels.vecadd
    n = 100_000_000
    b = {"A": torch.empty(0), "B": torch.empty(0), "C": torch.empty(0), "n_elements": n, "BLOCK_SIZE_N": 1024}
    sp = k.split
    assert sp.units(b, (1, 1, 1)) == n and sp.align(b) == 4096
    # a GEMM divides along whole 128-row tiles of A and C
    g = kernels.bare_matmul.split
    gb = dict(M=1000, N=64, K=32, stride_am=32, stride_ak=1, stride_bk=64, stride_bn=1, stride_cm=64, stride_cn=1)
    assert g.pitch(gb) == {"A": 32, "C": 64} and g.align(gb) == 128 and g.piece(gb, (8, 1, 1), 104)[0] == {"M": 104}
