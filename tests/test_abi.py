"""The C ABI without a GPU: the library loads, exports exactly what the header
declares, and rejects bad arguments on the host before touching the device."""

import ctypes
import re

import pytest

from xb200 import _lib
from xb200._lib import XbError


def test_library_exports_every_header_symbol():
    sigs = _lib.parse_header()
    assert len(sigs) >= 16
    lib = _lib.load()
    for name in sigs:
        assert hasattr(lib, name), f"{name} declared in xb200.h but not exported"


def test_header_and_library_agree_both_ways():
    import subprocess

    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (xb_\w+)", out))
    declared = set(_lib.parse_header())
    assert exported == declared, f"undeclared exports {exported - declared}, missing {declared - exported}"


def test_every_entry_point_ends_with_the_error_buffer():
    for name, (ret, params) in _lib.parse_header().items():
        assert ret == "int", name
        if name == "xb_abi_version":
            continue
        assert params[-2:] == ["char*", "size_t"], f"{name}: {params}"


def test_abi_version():
    assert _lib.call_int("xb_abi_version") >= 1


@pytest.mark.parametrize("fn", ["xb_relu", "xb_sigmoid", "xb_silu", "xb_gelu", "xb_gelu_tanh"])
def test_unary_rejects_negative_count(fn):
    with pytest.raises(XbError) as e:
        _lib.call(fn, 16, 32, -5, 0, None)
    assert e.value.code == _lib.XB_ERR_INVALID
    assert "negative" in e.value.message


def test_unsupported_dtype_is_reported():
    with pytest.raises(XbError) as e:
        _lib.call("xb_vecadd", 16, 32, 48, 10, 7, None)
    assert e.value.code == _lib.XB_ERR_UNSUPPORTED
    assert "dtype" in e.value.message


def test_null_pointer_is_rejected():
    with pytest.raises(XbError) as e:
        _lib.call("xb_axpy", None, 32, 48, ctypes.c_float(2.0), 10, 0, None)
    assert e.value.code == _lib.XB_ERR_INVALID


def test_zero_length_is_a_no_op():
    _lib.call("xb_vecadd", None, None, None, 0, 0, None)
    _lib.call("xb_softmax", None, None, 0, 8, 8, 8, 1, None)


def test_row_stride_shorter_than_row_is_rejected():
    with pytest.raises(XbError) as e:
        _lib.call("xb_softmax", 16, 32, 4, 128, 64, 128, 0, None)
    assert e.value.code == _lib.XB_ERR_INVALID and "stride" in e.value.message


def test_device_name_without_gpu_reports_cuda_error():
    import torch

    if torch.cuda.is_available():
        pytest.skip("has a GPU")
    buf = ctypes.create_string_buffer(64)
    with pytest.raises(XbError) as e:
        _lib.call("xb_device_name", 0, buf, 64, None)
    assert e.value.code == _lib.XB_ERR_CUDA


def test_error_buffer_is_truncated_safely():
    lib = _lib.load()
    err = ctypes.create_string_buffer(8)
    rc = lib.xb_relu(16, 32, -1, 0, None, err, 8)
    assert rc == _lib.XB_ERR_INVALID
    assert len(err.value) == 7
