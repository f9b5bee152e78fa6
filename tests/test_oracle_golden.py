"""The oracle against the reference examples' own expected outputs (CPU only).

Fixtures come from tests/golden/make_golden.py, which ran each reference
example's bench_* function with its launch recorded; ``expected`` is the
tensor the example itself computed as its reference.  Elementwise and row ops
must reproduce it bit for bit (the oracle restates the same expression); the
bf16 GEMM example rounds its reference to bf16 (matmul_bf16_m64_n64_k64.py:58)
while the oracle accumulates in fp32, so that one is held to the example's
own tolerance.
"""

import pytest
import torch

from conftest import golden_index, load_golden, materialize_args, output_name
from oracle import cgemm
from oracle import ops as O

INDEX = golden_index()


def _rows(t, rows, cols, stride):
    return torch.as_strided(t, (rows, cols), (stride, 1))


def oracle_for(entry: dict, blob: dict) -> torch.Tensor:
    a = materialize_args(blob)
    g = blob["grid"]
    k = entry["kernel"]
    if k == "vecadd":
        return O.vecadd(a["A"], a["B"])
    if k == "axpy_kernel":
        return O.axpy(a["X"], a["Y"], a["alpha"])
    if k in ("relu_kernel", "leaky_relu_kernel", "gelu_kernel", "sigmoid_kernel", "silu_kernel"):
        fn = {"relu_kernel": O.relu, "leaky_relu_kernel": O.leaky_relu, "gelu_kernel": O.gelu,
              "sigmoid_kernel": O.sigmoid, "silu_kernel": O.silu}[k]
        return fn(a["X"])
    if k == "swiglu_kernel":
        return O.swiglu(a["GATE"], a["UP"])
    if k == "avg_pool_kernel":
        return O.row_center(_rows(a["X"], g[0] * a["BLOCK_M"], a["BLOCK_N"], a["N"]))
    if k == "softmax_kernel":
        return O.softmax(_rows(a["input_ptr"], g[0] * a["BLOCK_SIZE"], a["n_cols"], a["input_stride_row"]))
    if k == "rms_norm_kernel":
        return O.rms_norm(_rows(a["X"], g[0] * a["BLOCK_M"], a["BLOCK_N"], a["N"]), a["eps"])
    if k == "weighted_rms_norm_kernel":
        return O.weighted_rms_norm(_rows(a["X"], g[0] * a["BLOCK_M"], a["BLOCK_N"], a["N"]), a["W"], a["eps"])
    if k == "bare_matmul_i8":
        return O.matmul_int(a["A"], a["B"])
    if k == "bare_matmul":
        return O.matmul_bf16_f32acc(a["A"], a["B"])
    if k == "padded_matmul_kernel":  # only the M x N corner of C is defined
        return O.matmul_f32_bf16emu(torch.as_strided(a["A"], (a["K"], a["M"]), (a["stride_ak"], 1)),
                                    torch.as_strided(a["B"], (a["K"], a["N"]), (a["stride_bk"], 1)))
    if k == "kernel":  # examples/load_2d_block
        return O.mul(a["x_ptr"], a["y_ptr"])
    if k == "_layer_norm_fwd_fused":
        return O.layernorm(_rows(a["input_ptr"], g[0] * a["BLOCK_SIZE"], a["n_cols"], a["input_stride_row"]),
                           eps=a["eps"])
    raise KeyError(k)


PINNED = sorted(c for c, e in INDEX.items() if e["pinned"] and "pinned_by" not in e)


def sampled_f32_gemm_check(c, a_km, b, M, N, seed_state=None):
    """The f32 GEMM example's own check (matmul_f32_..._atransposed.py:140-186):
    100 random elements plus the boundary tiles, each against an f32 numpy
    dot product of the bf16-rounded inputs, np.isclose(rtol=0.1, atol=10).
    Returns the number of mismatches."""
    import numpy as np
    from ml_dtypes import bfloat16

    a16 = a_km.numpy().astype(bfloat16)
    b16 = b.numpy().astype(bfloat16)
    # the example's own sample positions: the global numpy stream after its
    # seed-42 inputs (L88-95, L149-151)
    rng = np.random.RandomState(42)
    rng.rand(a_km.shape[0], M)
    rng.rand(b.shape[0], N)
    sm = list(rng.randint(0, M, 100))
    sn = list(rng.randint(0, N, 100))
    for bm in sorted({min(M - 1, m) for m in (M - 1, M - 64 + 1, 0) if m >= 0}):
        for bn in sorted({min(N - 1, n) for n in (N - 1, N - 32 + 1, 0) if n >= 0}):
            sm.append(bm)
            sn.append(bn)
    bad = 0
    for m, n in zip(sm, sn):
        exp = np.sum(a16[:, m].astype(np.float32) * b16[:, n].astype(np.float32), dtype=np.float32)
        bad += not np.isclose(float(c[m, n]), exp, rtol=0.1, atol=10.0)
    return bad


def test_f32_gemm_oracle_passes_the_examples_check_and_float64():
    case = "padded_matmul_f32_500x500x1024"
    blob = load_golden(case)
    a = materialize_args(blob)
    got = oracle_for(INDEX[case], blob)
    a_km = torch.as_strided(a["A"], (a["K"], a["M"]), (a["stride_ak"], 1))
    b = torch.as_strided(a["B"], (a["K"], a["N"]), (a["stride_bk"], 1))
    assert sampled_f32_gemm_check(got, a_km, b, a["M"], a["N"]) == 0
    exact = a_km.to(torch.bfloat16).double().t() @ b.to(torch.bfloat16).double()
    torch.testing.assert_close(got.double(), exact, atol=0.0, rtol=2e-5)


@pytest.mark.parametrize("case", PINNED)
def test_oracle_matches_reference_expected(case):
    entry = INDEX[case]
    blob = load_golden(case)
    got = oracle_for(entry, blob)
    exp = blob["expected"]
    assert got.shape == exp.shape and got.dtype == exp.dtype
    if entry["kernel"] == "bare_matmul":
        torch.testing.assert_close(got, exp, atol=entry["atol"], rtol=entry["rtol"])
    else:
        assert torch.equal(got, exp), f"{case}: oracle differs from the reference's expected output"


def test_every_example_operator_has_a_fixture():
    kernels = {e["kernel"] for e in INDEX.values()}
    assert kernels >= {"padded_matmul_kernel", "kernel", "vecadd", "axpy_kernel", "relu_kernel", "leaky_relu_kernel", "gelu_kernel", "sigmoid_kernel",
                       "silu_kernel", "swiglu_kernel", "avg_pool_kernel", "softmax_kernel", "rms_norm_kernel",
                       "weighted_rms_norm_kernel", "bare_matmul_i8", "bare_matmul", "_layer_norm_fwd_fused"}


def test_c_int_gemm_restatement_matches_torch_int32():
    g = torch.Generator().manual_seed(0)
    for dt, lo, hi, k in ((torch.int8, -128, 128, 300), (torch.int16, -2**15, 2**15, 700)):
        a = torch.randint(lo, hi, (37, k), generator=g, dtype=dt)
        b = torch.randint(lo, hi, (k, 29), generator=g, dtype=dt)
        c = cgemm.gemm_int(a, b)
        assert torch.equal(c, O.matmul_int(a, b))
        assert torch.equal(c, O.matmul_int_exact(a, b))


def test_int16_products_wrap_mod_2_32():
    # K large enough that the exact int64 sum leaves the int32 range.
    a = torch.full((1, 4096), -2**15, dtype=torch.int16)
    b = torch.full((4096, 1), -2**15, dtype=torch.int16)
    exact = 4096 * 2**30
    wrapped = ((exact + 2**31) % 2**32) - 2**31
    assert int(cgemm.gemm_int(a, b)[0, 0]) == wrapped
    assert int(O.matmul_int(a, b)[0, 0]) == wrapped


def test_i8_gemm_fixture_is_config_shape():
    # The 128x64x64 int8 GEMM workload, on the example's own inputs.
    blob = load_golden("matmul_i8_128x64x64")
    assert tuple(blob["args"]["A"].shape) == (128, 64) and tuple(blob["args"]["B"].shape) == (64, 64)
    assert output_name(blob) == "C"
