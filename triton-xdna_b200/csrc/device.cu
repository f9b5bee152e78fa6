// Device / library queries of the C ABI.
//
// xb_device_name replaces triton_npu_hsa_agent_name
// (amd_triton_npu/backend/include/HsaRuntime/HsaRuntime.cpp:750-766): the
// reference reports the NPU generation so callers can pick a code path; here
// the caller learns the CUDA device name and its SM count (the kernels size
// their grids in multiples of it).
#include "common.cuh"

extern "C" int xb_abi_version(void) { return 2; }

extern "C" int xb_device_name(int device, char* buf, size_t buf_len, int* sm_count, char* err, size_t errlen) {
  if (!buf || buf_len == 0) {
    xb::set_err(err, errlen, "xb_device_name: null or zero-length output buffer");
    return XB_ERR_INVALID;
  }
  cudaDeviceProp p;
  cudaError_t e = cudaGetDeviceProperties(&p, device);
  if (e != cudaSuccess) {
    xb::set_err(err, errlen, "xb_device_name: device %d: %s", device, cudaGetErrorString(e));
    return XB_ERR_CUDA;
  }
  size_t n = strlen(p.name);
  if (n + 1 > buf_len) {
    xb::set_err(err, errlen, "xb_device_name: name '%s' does not fit in %zu bytes", p.name, buf_len);
    return XB_ERR_INVALID;
  }
  memcpy(buf, p.name, n + 1);
  if (sm_count) *sm_count = p.multiProcessorCount;
  return XB_OK;
}

extern "C" int xb_launch_count(uint64_t* count, char* err, size_t errlen) {
  if (!count) {
    xb::set_err(err, errlen, "xb_launch_count: null output");
    return XB_ERR_INVALID;
  }
  *count = xb::launch_counter().load(std::memory_order_relaxed);
  return XB_OK;
}
