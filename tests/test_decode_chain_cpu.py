"""Decode chain host side without a GPU: the ctypes mirror of xb_decode_phase
has the C layout (checked against gcc on the header), the library rejects
bad chains before any CUDA call, and the per-slot scratch buffers and chain
counters stay apart."""

import ctypes
import os
import subprocess

import pytest
import torch

from xb200 import _lib, ops
from xb200._lib import XbError

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_phase_struct_matches_the_c_layout(tmp_path):
    fields = [f[0] for f in ops.DecodePhase._fields_]
    src = tmp_path / "layout.c"
    src.write_text(
        "#include <stdio.h>\n#include <stddef.h>\n#include \"xb200.h\"\nint main(void) {\n"
        '  printf("%zu\\n", sizeof(xb_decode_phase));\n'
        + "".join(f'  printf("%zu\\n", offsetof(xb_decode_phase, {f}));\n' for f in fields)
        + "  return 0;\n}\n")
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    got = [int(v) for v in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]
    assert got[0] == ctypes.sizeof(ops.DecodePhase)
    assert got[1:] == [getattr(ops.DecodePhase, f).offset for f in fields]


def _phase(kind=ops.XB_DECODE_STORE, K=512):
    ph = ops.DecodePhase()
    ph.kind = kind
    ph.x, ph.m, ph.ldx = 1 << 20, 8, K
    ph.w, ph.n, ph.k, ph.ldw = 1 << 24, 256, K, K
    ph.y, ph.ldy = 1 << 28, 256
    return ph


def _call(phases, n=None, sync=1 << 12):
    arr = (ops.DecodePhase * max(1, len(phases)))(*phases)
    _lib.call("xb_decode_chain_bf16", ctypes.addressof(arr), len(phases) if n is None else n, sync, None)


@pytest.mark.parametrize("n", [0, 5, -1])
def test_phase_count_is_checked(n):
    with pytest.raises(XbError) as e:
        _call([_phase()], n=n)
    assert e.value.code == _lib.XB_ERR_INVALID


def test_sync_buffer_is_checked():
    with pytest.raises(XbError) as e:
        _call([_phase()], sync=None)
    assert e.value.code == _lib.XB_ERR_INVALID
    with pytest.raises(XbError) as e:
        _call([_phase()], sync=(1 << 12) + 2)
    assert e.value.code == _lib.XB_ERR_INVALID


def test_bad_kind_and_shapes_are_rejected():
    with pytest.raises(XbError) as e:
        _call([_phase(kind=7)])
    assert e.value.code == _lib.XB_ERR_INVALID and "kind" in e.value.message
    bad = _phase()
    bad.m = 65  # more tokens than a decode step
    with pytest.raises(XbError) as e:
        _call([bad])
    assert e.value.code == _lib.XB_ERR_INVALID
    with pytest.raises(XbError) as e:
        _call([_phase(), _phase(K=8192)])  # ten K blocks per CTA at most
    assert e.value.code == _lib.XB_ERR_UNSUPPORTED and "5120" in e.value.message
    rk = _phase(kind=ops.XB_DECODE_ROPE_KV, K=896)
    rk.n, rk.n_head, rk.n_kv_head, rk.head_dim, rk.max_seq, rk.pos_offset = 1000, 14, 2, 64, 40, 3
    with pytest.raises(XbError) as e:  # n must be (H + 2 KVH) * D
        _call([rk])
    assert e.value.code == _lib.XB_ERR_INVALID
    sw = _phase(kind=ops.XB_DECODE_SWIGLU)
    sw.n = 192  # 2 n_out with n_out % 64 != 0
    with pytest.raises(XbError) as e:
        _call([sw])
    assert e.value.code == _lib.XB_ERR_INVALID


def test_workspace_slots_keep_separate_buffers():
    """Each (device, slot) has its own scratch buffer and chain counters;
    nested slots restore the outer one, and growth stays within its slot."""
    dev = torch.device("cpu", 0)  # an explicit index: no CUDA call needed
    base = ops._workspace(dev, 1024)
    with ops.workspace_slot(7):
        a = ops._workspace(dev, 1024)
        sync_a = ops.decode_chain_sync(dev)
        with ops.workspace_slot(8):
            b = ops._workspace(dev, 1024)
            assert b.data_ptr() != a.data_ptr()
            assert ops.decode_chain_sync(dev).data_ptr() != sync_a.data_ptr()
        assert ops._workspace(dev, 1024).data_ptr() == a.data_ptr()  # slot 7 again
        assert ops.decode_chain_sync(dev) is sync_a
        big = ops._workspace(dev, 8 << 20)  # grows slot 7 only
        assert big.numel() * 4 >= 8 << 20 and big.data_ptr() != a.data_ptr()
    assert a.data_ptr() != base.data_ptr()
    assert ops._workspace(dev, 1024).data_ptr() == base.data_ptr()  # slot 0 untouched
    assert sync_a.dtype == torch.int32 and sync_a.numel() * 4 == 16 and int(sync_a.abs().sum()) == 0
