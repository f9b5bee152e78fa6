// Peer memory across the GPUs of one node (one process per GPU) and the
// bounded cross-GPU wait used by the N-sharded GEMM.
//
// The reference has no multi-device path; this is the exchange step of the
// N-sharded GEMM: every rank's GEMM epilogue stores its column block of C
// straight into every peer's C over NVLink (peer pointers from CUDA IPC), and
// signals each peer by incrementing an epoch counter in the peer's signal
// buffer.  A peer then waits -- bounded -- until every rank's counter reaches
// the epoch of the call.
//
// Signal buffer of a rank: uint64 [2 * world + 1]; slot r counts the calls
// whose shard from rank r has fully landed here; slot `world` is the rank's
// own CTA-completion counter (the last CTA of the GEMM grid sends the
// signals); slot world + 1 + r counts the calls rank r has started, i.e. how
// many times rank r has released its C for overwriting (the GEMM waits on
// these before its first store into rank r's C).
#include "common.cuh"

namespace xb {
namespace peer {

__device__ int g_peer_status = 0;

__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint64_t now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Thread r (r != rank) waits until signal[r] >= epoch, for at most timeout_ns.
__global__ void peer_wait_kernel(const uint64_t* __restrict__ signal, int world, int rank, uint64_t epoch,
                                 uint64_t timeout_ns) {
  pdl_wait();
  const int r = threadIdx.x;
  if (r >= world || r == rank) return;
  const uint64_t t0 = now_ns();
  while (ld_acquire_sys(signal + r) < epoch) {
    if (now_ns() - t0 > timeout_ns) {
      atomicExch(&g_peer_status, XB_ERR_TIMEOUT);
      return;
    }
    __nanosleep(200);
  }
}

}  // namespace peer
}  // namespace xb

using xb::set_err;

extern "C" int xb_peer_alloc(size_t bytes, void** ptr, void* ipc_handle, char* err, size_t errlen) {
  if (!ptr || !ipc_handle || bytes == 0) {
    set_err(err, errlen, "xb_peer_alloc: bad arguments");
    return XB_ERR_INVALID;
  }
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e == cudaSuccess) e = cudaMemset(p, 0, bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    if (p) cudaFree(p);
    set_err(err, errlen, "xb_peer_alloc: %s", cudaGetErrorString(e));
    return XB_ERR_CUDA;
  }
  memcpy(ipc_handle, &h, sizeof(h));
  *ptr = p;
  return XB_OK;
}

extern "C" int xb_peer_open(const void* ipc_handle, void** ptr, char* err, size_t errlen) {
  if (!ipc_handle || !ptr) {
    set_err(err, errlen, "xb_peer_open: bad arguments");
    return XB_ERR_INVALID;
  }
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    set_err(err, errlen, "xb_peer_open: %s", cudaGetErrorString(e));
    return XB_ERR_CUDA;
  }
  return XB_OK;
}

extern "C" int xb_peer_close(void* ptr, char* err, size_t errlen) {
  cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) {
    set_err(err, errlen, "xb_peer_close: %s", cudaGetErrorString(e));
    return XB_ERR_CUDA;
  }
  return XB_OK;
}

extern "C" int xb_peer_free(void* ptr, char* err, size_t errlen) {
  cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) {
    set_err(err, errlen, "xb_peer_free: %s", cudaGetErrorString(e));
    return XB_ERR_CUDA;
  }
  return XB_OK;
}

extern "C" int xb_peer_wait(const uint64_t* signal, int world, int rank, uint64_t epoch, uint64_t timeout_ns,
                            void* stream, char* err, size_t errlen) {
  if (!signal || world < 1 || world > 1024 || rank < 0 || rank >= world) {
    set_err(err, errlen, "xb_peer_wait: bad arguments");
    return XB_ERR_INVALID;
  }
  if (world == 1) return XB_OK;
  xb::launch_k(xb::peer::peer_wait_kernel, 1, (unsigned)((world + 31) / 32 * 32), 0, (cudaStream_t)stream, signal,
               world, rank, epoch, timeout_ns);
  return xb::check_launch("xb_peer_wait", err, errlen);
}

extern "C" int xb_peer_status(void* stream, int* status, char* err, size_t errlen) {
  if (!status) {
    set_err(err, errlen, "xb_peer_status: null output");
    return XB_ERR_INVALID;
  }
  cudaStream_t s = (cudaStream_t)stream;
  int zero = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(status, xb::peer::g_peer_status, sizeof(int), 0, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e == cudaSuccess) e = cudaMemcpyToSymbolAsync(xb::peer::g_peer_status, &zero, sizeof(int), 0,
                                                    cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) {
    set_err(err, errlen, "xb_peer_status: %s", cudaGetErrorString(e));
    return XB_ERR_CUDA;
  }
  return XB_OK;
}
