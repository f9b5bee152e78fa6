"""Parity on the reference examples' own inputs, launched the way the examples launch.

Each golden fixture holds the arguments an example passed to its kernel and
the expected tensor the example computed itself.  The test calls the xb200
launcher with the same signature on the same HOST tensors (so the
reference's copy-in / copy-back-the-last-pointer semantics are exercised),
then applies the example's own assertion, and a tighter check against the
oracle.
"""

import pytest
import torch

from conftest import golden_index, load_golden, materialize_args, output_name
from xb200 import kernels

pytestmark = pytest.mark.gpu

INDEX = golden_index()
CASES = sorted(c for c in INDEX if INDEX[c]["kernel"] in kernels.REGISTRY)


def _launch(case):
    entry = INDEX[case]
    blob = load_golden(case)
    args = materialize_args(blob)
    k = kernels.REGISTRY[entry["kernel"]]
    grid = tuple(blob["grid"])
    # positional order of the example's call, as recorded
    k[grid](**args)
    return entry, blob, args[output_name(blob)]


@pytest.mark.parametrize("case", [c for c in CASES if INDEX[c]["pinned"] and "pinned_by" not in INDEX[c]])
def test_example_assertion_holds(case):
    entry, blob, out = _launch(case)
    assert out.device.type == "cpu"  # copied back into the caller's host tensor
    torch.testing.assert_close(out, blob["expected"], atol=entry["atol"], rtol=entry["rtol"])


EXACT = {"vecadd", "axpy_kernel", "relu_kernel", "leaky_relu_kernel", "bare_matmul_i8"}


@pytest.mark.parametrize("case", CASES)
def test_tight_against_oracle(case):
    from test_oracle_golden import oracle_for

    entry, blob, out = _launch(case)
    ref = oracle_for(entry, blob)
    if entry["kernel"] in EXACT:
        assert torch.equal(out, ref)
    elif out.dtype == torch.bfloat16:
        # at most one bf16 ulp away, and nearly all elements identical
        torch.testing.assert_close(out.float(), ref.float(), atol=1e-6, rtol=2 ** -7)
        same = (out == ref).float().mean().item()
        assert same > 0.97, f"only {same:.3f} of elements bit-identical"
    elif entry["kernel"] == "bare_matmul":
        # fp32 accumulation in a different order than the CPU's
        torch.testing.assert_close(out, ref, atol=1e-3, rtol=1e-4)
    elif entry["kernel"] == "padded_matmul_kernel":
        a = blob["args"]
        torch.testing.assert_close(out[:a["M"], :a["N"]], ref, atol=1e-3, rtol=2e-5)
    else:
        torch.testing.assert_close(out, ref, atol=2e-5, rtol=2e-5)


def test_f32_gemm_example_check_on_gpu_output():
    """The f32 GEMM example's own sampled check, on the GPU result of its call."""
    from test_oracle_golden import sampled_f32_gemm_check

    case = "padded_matmul_f32_500x500x1024"
    entry, blob, out = _launch(case)
    args = materialize_args(blob)
    a_km = torch.as_strided(args["A"], (args["K"], args["M"]), (args["stride_ak"], 1))
    b = torch.as_strided(args["B"], (args["K"], args["N"]), (args["stride_bk"], 1))
    assert out.device.type == "cpu"
    assert sampled_f32_gemm_check(out, a_km, b, args["M"], args["N"]) == 0
