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
