"""Host logic of the multi-GPU paths on CPU: two gloo ranks (spawned
processes) exercise the column sharding and the re-layout of all-gathered
blocks that the NCCL baseline of the N-sharded GEMM uses, and the batch
sharding of the LLM."""

import ctypes
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from xb200.dist import assemble_gathered, shard_batch, shard_columns


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_columns_and_batch():
    assert shard_columns(1024, 4) == [(0, 256), (256, 256), (512, 256), (768, 256)]
    with pytest.raises(ValueError):
        shard_columns(1000, 3)
    assert [shard_batch(64, 8, r) for r in (0, 7)] == [(0, 8), (56, 8)]
    with pytest.raises(ValueError):
        shard_batch(64, 3, 0)


def _worker(rank, world, port, m, n, k):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(0)
        a = torch.randn(m, k, generator=g)
        b = torch.randn(k, n, generator=g)
        start, size = shard_columns(n, world)[rank]
        c_shard = a @ b[:, start:start + size]
        gathered = [torch.empty_like(c_shard) for _ in range(world)]
        dist.all_gather(gathered, c_shard)
        c = assemble_gathered(torch.stack(gathered))
        assert torch.allclose(c, a @ b, atol=1e-5)
        ids = torch.arange(16)
        s0, sz = shard_batch(16, world, rank)
        parts = [torch.empty(sz, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(parts, ids[s0:s0 + sz].contiguous())
        assert torch.equal(torch.cat(parts), ids)
    finally:
        dist.destroy_process_group()


def test_sharded_gemm_layout_with_two_gloo_ranks():
    mp.spawn(_worker, args=(2, _free_port(), 6, 8, 5), nprocs=2, join=True)


def test_sharded_entry_rejects_bad_world_without_a_gpu():
    from xb200 import _lib

    with pytest.raises(_lib.XbError) as e:  # world 9 > 8
        _lib.call("xb_matmul_sharded", 16, 16, None, None, 9, 0, 8, 8, 8, 8, 8, 64, 1, 10**9, 0, None)
    assert e.value.code == _lib.XB_ERR_INVALID
    cp = (ctypes.c_void_p * 2)(16, 16)
    with pytest.raises(_lib.XbError) as e:  # epoch 0: the first call on a signal buffer is epoch 1
        _lib.call("xb_matmul_sharded", 16, 16, ctypes.cast(cp, ctypes.c_void_p), ctypes.cast(cp, ctypes.c_void_p),
                  2, 0, 8, 8, 8, 8, 8, 16, 0, 10**9, 0, None)
    assert e.value.code == _lib.XB_ERR_INVALID and "epoch" in e.value.message
    with pytest.raises(_lib.XbError):
        _lib.call("xb_peer_wait", None, 2, 0, 1, 1000, None)
