"""Multi-GPU paths on the B200.

* Bounded cross-GPU wait (1 GPU): a wait on a signal nothing sets runs out
  after its time limit and reports XB_ERR_TIMEOUT -- no fault, no hang, and
  the context stays usable.
* The sharded GEMM's wait for a peer's release of its C (1 GPU, two ranks'
  buffers in one GPU's memory, one kernel): with no release the kernel gives
  up after its limit, stores nothing and withholds its completion signal;
  with the release set by hand the same call goes through.
* N-sharded GEMM (2, 4 and 8 GPUs, spawned NCCL ranks): the fused peer-store
  kernel and the NCCL all-gather baseline both reproduce the single-GPU GEMM
  exactly (each column is computed by the same arithmetic), over successive
  calls with different inputs while one rank reads its C late.
"""

import ctypes
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def test_peer_wait_times_out_and_reports_status():
    from xb200 import _lib, ops

    sig = torch.zeros(3, dtype=torch.int64, device="cuda")  # world 2: rank 1's slot never moves
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    _lib.call("xb_peer_wait", sig.data_ptr(), 2, 0, 1, 50_000_000, stream)  # 50 ms limit
    st = ctypes.c_int(0)
    _lib.call("xb_peer_status", stream, ctypes.byref(st))
    assert st.value == _lib.XB_ERR_TIMEOUT
    _lib.call("xb_peer_status", stream, ctypes.byref(st))
    assert st.value == 0  # cleared by the read
    sig[1] = 1  # now satisfied: returns immediately
    _lib.call("xb_peer_wait", sig.data_ptr(), 2, 0, 1, 50_000_000, stream)
    _lib.call("xb_peer_status", stream, ctypes.byref(st))
    assert st.value == 0
    assert torch.equal(ops.vecadd(torch.ones(8, device="cuda"), torch.ones(8, device="cuda")).cpu(),
                       torch.full((8,), 2.0))  # context still healthy


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_kernels_on_two_devices_in_one_process():
    """Kernel set-up (shared-memory limits, resident cluster counts) is per
    device: one process runs the same GEMMs and attention on device 0, then
    device 1, then device 0 again, each checked exactly against the first."""
    from oracle import cgemm
    from xb200 import ops

    g = torch.Generator().manual_seed(4)
    a = torch.randint(-128, 128, (512, 384), generator=g, dtype=torch.int8)
    b = torch.randint(-128, 128, (384, 640), generator=g, dtype=torch.int8)
    x = torch.randn((300, 896), generator=g).to(torch.bfloat16)
    w = (torch.randn((1152, 896), generator=g) * 0.05).to(torch.bfloat16)
    q = torch.randn((2, 14, 100, 64), generator=g).to(torch.bfloat16)
    kc = torch.randn((2, 2, 128, 64), generator=g).to(torch.bfloat16)
    vc = torch.randn((2, 2, 128, 64), generator=g).to(torch.bfloat16)
    want = cgemm.gemm_int(a, b)
    results = []
    for dev in (0, 1, 0):
        with torch.cuda.device(dev):
            d = torch.device("cuda", dev)
            c = ops.matmul_i8(a.to(d), b.to(d))  # CTA pairs (M >= 256)
            y = ops.linear(x.to(d), w.to(d))
            o = torch.empty((2, 100, 14 * 64), dtype=torch.bfloat16, device=d)
            ops.attention(q.to(d), kc.to(d), vc.to(d), o, 2, 100, 14, 2, 64, 0, 0.125)
            torch.cuda.synchronize(d)
            assert ops.device_status() == 0
            results.append((c.cpu(), y.cpu(), o.cpu()))
    assert torch.equal(results[0][0], want)
    for r in results[1:]:
        for got, ref in zip(r, results[0]):
            assert torch.equal(got, ref)


@pytest.mark.parametrize("m", [512, 200])  # CTA pairs, single CTAs
def test_sharded_gemm_release_wait_times_out_then_proceeds(m):
    from xb200 import _lib, ops

    world, ns, k = 2, 256, 256
    g = torch.Generator(device="cuda").manual_seed(3)
    a = torch.randint(-128, 128, (m, k), generator=g, device="cuda", dtype=torch.int8)
    b = torch.randint(-128, 128, (k, ns), generator=g, device="cuda", dtype=torch.int8)
    cs = [torch.full((m, world * ns), -1, dtype=torch.int32, device="cuda") for _ in range(world)]
    sig = [torch.zeros(2 * world + 1, dtype=torch.int64, device="cuda") for _ in range(world)]
    cp = (ctypes.c_void_p * world)(*[c.data_ptr() for c in cs])
    sp = (ctypes.c_void_p * world)(*[x.data_ptr() for x in sig])
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    def call():  # rank 0 of 2, epoch 1, 50 ms limit
        _lib.call("xb_matmul_sharded", a.data_ptr(), b.data_ptr(), ctypes.cast(cp, ctypes.c_void_p),
                  ctypes.cast(sp, ctypes.c_void_p), world, 0, m, ns, k, k, ns, world * ns, 1, 50_000_000,
                  _lib.XB_DT_I8, stream)
        st = ctypes.c_int(0)
        _lib.call("xb_device_status", stream, ctypes.byref(st))
        return st.value

    assert call() == _lib.XB_ERR_TIMEOUT  # nothing plays rank 1: its release never comes
    s0, s1 = sig[0].cpu(), sig[1].cpu()
    assert s1[world + 1 + 0] == 1  # rank 0's own release reached rank 1's buffer
    assert s1[0] == 0  # no completion signal after the abort
    assert s0[world] == 0  # the CTA counter is back at zero
    assert bool((cs[0] == -1).all()) and bool((cs[1] == -1).all())  # nothing stored anywhere
    sig[0][world + 1 + 1] = 1  # rank 1 releases its C for epoch 1
    assert call() == 0
    s0, s1 = sig[0].cpu(), sig[1].cpu()
    assert s1[0] == 1 and s0[world] == 0
    want = ops.matmul_i8(a, b)
    for c in cs:
        assert torch.equal(c[:, :ns], want)
        assert bool((c[:, ns:] == -1).all())  # rank 1's block is not rank 0's to write


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port):
    import datetime

    from xb200 import ops
    from xb200.dist import ShardedMatmul, nccl_sharded_matmul, shard_columns

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        # ragged rows (300), ragged shard columns (176 int8 / 200 bf16: partial
        # 32-column chunks take the per-thread store path; shard row pitches
        # stay multiples of 16 bytes, as the TMA loads of B require), pairs
        # (M >= 256) and single CTAs
        for dtype, (m, n, k) in ((torch.bfloat16, (512, 1024, 768)), (torch.int8, (300, 64 * world, 256)),
                                 (torch.int8, (300, 176 * world, 128)), (torch.bfloat16, (200, 200 * world, 64)),
                                 (torch.bfloat16, (4096, 4096, 4096)), (torch.int8, (2048, 8192, 2048))):
            s0, ns = shard_columns(n, world)[rank]
            sm = ShardedMatmul(m, n, k, dtype)
            outs, wants = [], []
            for epoch in range(3):  # different inputs every call, C rewritten in place
                g = torch.Generator(device="cuda").manual_seed(10 * epoch + 1)
                if dtype == torch.int8:
                    a = torch.randint(-128, 128, (m, k), generator=g, device="cuda", dtype=torch.int8)
                    b = torch.randint(-128, 128, (k, n), generator=g, device="cuda", dtype=torch.int8)
                    wants.append(ops.matmul_i8(a, b))
                else:
                    a = torch.randn((m, k), generator=g, device="cuda").to(torch.bfloat16)
                    b = torch.randn((k, n), generator=g, device="cuda").to(torch.bfloat16)
                    wants.append(ops.matmul_bf16(a, b, torch.bfloat16))
                b_shard = b[:, s0:s0 + ns].contiguous()
                c = sm.run(a, b_shard)
                if rank == world - 1:
                    torch.cuda._sleep(20_000_000)  # this rank reads its C late: peers must not run ahead
                outs.append(c.clone())  # the reader of this call's C, on the same stream
            torch.cuda.synchronize()
            assert sm.status() == 0
            for e in range(3):
                assert torch.equal(outs[e], wants[e]), f"fused sharded GEMM differs on rank {rank}, call {e}"
            base = nccl_sharded_matmul(a, b_shard)
            assert torch.equal(base, wants[-1])
            sm.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_sharded_gemm_matches_single_gpu(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    mp.spawn(_rank_main, args=(world, _free_port()), nprocs=world, join=True)
