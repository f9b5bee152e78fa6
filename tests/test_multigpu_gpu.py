"""Multi-GPU paths on the B200.

* Bounded cross-GPU wait (1 GPU): a wait on a signal nothing sets runs out
  after its time limit and reports XB_ERR_TIMEOUT -- no fault, no hang, and
  the context stays usable.
* N-sharded GEMM (2+ GPUs, spawned NCCL ranks): the fused peer-store kernel
  and the NCCL all-gather baseline both reproduce the single-GPU GEMM
  exactly (each column is computed by the same arithmetic).
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
        # ragged rows (300), ragged shard columns (176, 200: partial 32-column
        # chunks take the per-thread store path), pairs (M >= 256) and single CTAs
        for dtype, (m, n, k) in ((torch.bfloat16, (512, 1024, 768)), (torch.int8, (300, 512, 256)),
                                 (torch.int8, (300, 352, 128)), (torch.bfloat16, (200, 400, 64)),
                                 (torch.bfloat16, (4096, 4096, 4096))):
            g = torch.Generator(device="cuda").manual_seed(1)
            if dtype == torch.int8:
                a = torch.randint(-128, 128, (m, k), generator=g, device="cuda", dtype=torch.int8)
                b = torch.randint(-128, 128, (k, n), generator=g, device="cuda", dtype=torch.int8)
                full = ops.matmul_i8(a, b)
            else:
                a = torch.randn((m, k), generator=g, device="cuda").to(torch.bfloat16)
                b = torch.randn((k, n), generator=g, device="cuda").to(torch.bfloat16)
                full = ops.matmul_bf16(a, b, torch.bfloat16)
            s0, ns = shard_columns(n, world)[rank]
            b_shard = b[:, s0:s0 + ns].contiguous()
            sm = ShardedMatmul(m, n, k, dtype)
            for _ in range(3):  # repeated calls: epochs advance, C is rewritten in place
                c = sm.run(a, b_shard)
                torch.cuda.synchronize()
                assert sm.status() == 0
                assert torch.equal(c, full), f"fused sharded GEMM differs on rank {rank}"
            base = nccl_sharded_matmul(a, b_shard)
            assert torch.equal(base, full)
            sm.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_sharded_gemm_two_gpus_matches_single_gpu():
    mp.spawn(_rank_main, args=(2, _free_port()), nprocs=2, join=True)
