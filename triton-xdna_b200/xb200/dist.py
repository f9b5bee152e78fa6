"""Multi-GPU pieces: the N-sharded GEMM with its all-gather fused into the
epilogue, the NCCL all-gather baseline, and batch sharding of the LLM.

One process per GPU (torchrun), `torch.distributed` for the plumbing
(rendezvous, exchanging CUDA IPC handles, the baseline collective).  The
reference runs on one device; these are the multi-GPU forms of its GEMM
(examples/matmul_*) and of its Qwen forward (examples/qwen2_5/model.py).

N-sharding: rank r holds A [M, K] and B[:, r*Ns : (r+1)*Ns] and produces
C[:, r*Ns : (r+1)*Ns]; every rank ends with the full C [M, N].
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib, ops


def shard_columns(n: int, world: int) -> list[tuple[int, int]]:
    """(start, size) of each rank's column block; N must split evenly (the
    sharded kernel writes equal blocks at rank * N_shard)."""
    if world < 1 or n % world:
        raise ValueError(f"N={n} does not split evenly over {world} ranks")
    ns = n // world
    return [(r * ns, ns) for r in range(world)]


def shard_batch(batch: int, world: int, rank: int) -> tuple[int, int]:
    """(start, size) of this rank's slice of a batch of independent sequences."""
    if batch % world:
        raise ValueError(f"batch {batch} does not split evenly over {world} ranks")
    per = batch // world
    return rank * per, per


def assemble_gathered(gathered: torch.Tensor) -> torch.Tensor:
    """[world, M, Ns] blocks from an all-gather -> C [M, world * Ns]."""
    w, m, ns = gathered.shape
    return gathered.permute(1, 0, 2).reshape(m, w * ns)


class _CudaArray:
    """Minimal __cuda_array_interface__ wrapper to view raw device memory as a torch tensor."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"data": (ptr, False), "shape": tuple(shape), "typestr": typestr,
                                         "version": 3, "strides": None}


_TYPESTR = {torch.int32: "<i4", torch.bfloat16: "<V2", torch.uint64: "<u8", torch.int64: "<i8", torch.float32: "<f4"}


class PeerBuffer:
    """`nbytes` of device memory on every rank, each mapped into every rank's
    address space (CUDA IPC over NVLink).  ptrs[r] is rank r's buffer as seen
    from this process; ptrs[rank] is the local one."""

    def __init__(self, nbytes: int, group=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        local = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(64)
        _lib.call("xb_peer_alloc", nbytes, ctypes.byref(local), handle)
        handles = [None] * self.world
        dist.all_gather_object(handles, handle.raw, group=group)
        self.ptrs = []
        for r, h in enumerate(handles):
            if r == self.rank:
                self.ptrs.append(local.value)
            else:
                p = ctypes.c_void_p()
                _lib.call("xb_peer_open", ctypes.create_string_buffer(h, 64), ctypes.byref(p))
                self.ptrs.append(p.value)
        self.nbytes = nbytes

    def local_tensor(self, shape, dtype) -> torch.Tensor:
        if dtype == torch.bfloat16:  # torch reads bf16 through a 2-byte view
            t = torch.as_tensor(_CudaArray(self.ptrs[self.rank], shape, "<i2"), device="cuda")
            return t.view(torch.bfloat16)
        return torch.as_tensor(_CudaArray(self.ptrs[self.rank], shape, _TYPESTR[dtype]), device="cuda")

    def close(self):
        for r, p in enumerate(self.ptrs):
            if r != self.rank and p:
                _lib.call("xb_peer_close", p)
        if self.ptrs and self.ptrs[self.rank]:
            _lib.call("xb_peer_free", self.ptrs[self.rank])
        self.ptrs = []


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


class ShardedMatmul:
    """C [M, N] = A [M, K] @ B [K, N], N-sharded over the ranks of `group`,
    every rank ending with the full C.

    `run` issues one fused kernel per rank (GEMM tiles stored into every
    rank's C over NVLink, then a completion signal to each peer) and a
    bounded wait for the peers' signals; it returns `out`, this rank's C.
    All ranks call `run` the same number of times.

    Successive calls reuse C and are stream-ordered: a call's kernel first
    tells every peer that this rank's C may be overwritten (every earlier
    kernel on the current stream, e.g. a reader of the previous `out`, has
    completed) and stores into a peer's C only after that peer has done the
    same for this call.  So work that reads `out` before the next `run` must
    be enqueued on the same stream (or ordered before it with an event).
    A wait that runs out is reported by `status()`; the plan must then be
    closed and rebuilt."""

    def __init__(self, m: int, n: int, k: int, dtype=torch.bfloat16, group=None, timeout_s: float = 10.0):
        if dtype not in (torch.bfloat16, torch.int8):
            raise TypeError("sharded GEMM supports bf16 and int8")
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise ValueError("at most 8 ranks")
        self.m, self.n, self.k, self.dtype = m, n, k, dtype
        self.n_shard = shard_columns(n, self.world)[self.rank][1]
        self.out_dtype = torch.int32 if dtype == torch.int8 else torch.bfloat16
        osz = 4 if dtype == torch.int8 else 2
        self.c = PeerBuffer(m * n * osz, group)
        self.sig = PeerBuffer(8 * (2 * self.world + 1), group)
        self.epoch = 0
        self.timeout_ns = int(timeout_s * 1e9)
        self._c_ptrs = (ctypes.c_void_p * self.world)(*self.c.ptrs)
        self._s_ptrs = (ctypes.c_void_p * self.world)(*self.sig.ptrs)
        self.out = self.c.local_tensor((m, n), self.out_dtype)

    def run(self, a: torch.Tensor, b_shard: torch.Tensor) -> torch.Tensor:
        if tuple(a.shape) != (self.m, self.k) or tuple(b_shard.shape) != (self.k, self.n_shard):
            raise ValueError("operand shapes do not match the plan")
        if a.dtype != self.dtype or b_shard.dtype != self.dtype:
            raise TypeError("operand dtype does not match the plan")
        dt = 2 if self.dtype == torch.int8 else 0
        self.epoch += 1
        _lib.call("xb_matmul_sharded", a.data_ptr(), b_shard.data_ptr(), ctypes.cast(self._c_ptrs, ctypes.c_void_p),
                  ctypes.cast(self._s_ptrs, ctypes.c_void_p), self.world, self.rank, self.m, self.n_shard, self.k,
                  a.stride(0), b_shard.stride(0), self.n, self.epoch, self.timeout_ns, dt, _stream())
        _lib.call("xb_peer_wait", self.sig.ptrs[self.rank], self.world, self.rank, self.epoch, self.timeout_ns,
                  _stream())
        return self.out

    def status(self) -> int:
        """0, or the first error recorded since the last call (synchronises the
        stream and clears the status words): XB_ERR_TIMEOUT when a peer's
        completion signal (xb_peer_wait) or its release of C (the GEMM
        kernel) did not come in time."""
        st = ctypes.c_int(0)
        _lib.call("xb_peer_status", _stream(), ctypes.byref(st))
        dev = ctypes.c_int(0)
        _lib.call("xb_device_status", _stream(), ctypes.byref(dev))
        return st.value or dev.value

    def close(self):
        torch.cuda.synchronize()
        dist.barrier(self.c.group)
        self.c.close()
        self.sig.close()


def nccl_sharded_matmul(a: torch.Tensor, b_shard: torch.Tensor, group=None) -> torch.Tensor:
    """Baseline: local GEMM of the shard, then an NCCL all-gather and a
    re-layout of the [world, M, Ns] blocks into C [M, N]."""
    world = dist.get_world_size(group)
    if a.dtype == torch.int8:
        c = ops.matmul_i8(a, b_shard)
    else:
        c = ops.matmul_bf16(a, b_shard, torch.bfloat16)
    gathered = torch.empty((world,) + tuple(c.shape), dtype=c.dtype, device=c.device)
    dist.all_gather_into_tensor(gathered, c, group=group)
    return assemble_gathered(gathered)
