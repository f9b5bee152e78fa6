// Shared helpers for the xb200 CUDA kernels (sm_100a).
//
// Error convention mirrors the reference's native C ABI
// (amd_triton_npu/backend/include/HsaRuntime/HsaRuntime.cpp:740-794):
// every entry point returns 0 on success or a negative status, and on error
// writes a NUL-terminated message into the caller's (err, errlen) buffer.
#pragma once

#include <atomic>
#include <mutex>
#include <vector>

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>
#include <stdarg.h>
#include <stdlib.h>

#include "../../include/xb200.h"

namespace xb {

// Write a printf-style message into the caller's error buffer (may be NULL).
inline void set_err(char* err, size_t errlen, const char* fmt, ...) {
  if (!err || errlen == 0) return;
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(err, errlen, fmt, ap);
  va_end(ap);
}

// Report the first error from an asynchronous launch (launch-configuration
// errors surface here; execution errors surface at the caller's next sync).
inline int check_launch(const char* what, char* err, size_t errlen) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_err(err, errlen, "%s: kernel launch failed: %s", what, cudaGetErrorString(e));
    return XB_ERR_CUDA;
  }
  return XB_OK;
}

inline int sm_count(int* out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  static std::atomic<int> cached[64];  // zero-initialised (static storage)
  if (dev >= 0 && dev < 64) {
    const int c = cached[dev].load(std::memory_order_relaxed);
    if (c > 0) { *out = c; return 0; }
  }
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return -1;
  if (dev >= 0 && dev < 64) cached[dev].store(n, std::memory_order_relaxed);
  *out = n;
  return 0;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline int dtype_size(int dt) {
  switch (dt) {
    case XB_DT_BF16: return 2;
    case XB_DT_F32: return 4;
    case XB_DT_I8: return 1;
    case XB_DT_I16: return 2;
    case XB_DT_I32: return 4;
    default: return 0;
  }
}

// ---- element conversions (fp32 compute, round-to-nearest-even stores) ----
template <typename T> struct Cvt;
template <> struct Cvt<float> {
  static __device__ __forceinline__ float to_f(float v) { return v; }
  static __device__ __forceinline__ float from_f(float v) { return v; }
};
template <> struct Cvt<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};

// Round an fp32 value to the storage type and back (models a store of an
// intermediate in the storage dtype, as the reference's torch expressions do).
template <typename T>
__device__ __forceinline__ float round_to(float v) { return Cvt<T>::to_f(Cvt<T>::from_f(v)); }

// Hardware approximations (one MUFU instruction each, relative error about
// 2^-22, subnormal results flushed to zero).  Used only where the result is
// stored as bf16, whose ulp (2^-8 relative) dwarfs that error.
__device__ __forceinline__ float ex2_approx(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}
__device__ __forceinline__ float rcp_approx(float x) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// silu(x) = x * sigmoid(x) on the MUFU approximations, for values stored as
// bf16 (shared by the elementwise kernels and the fused MLP reduction so both
// round identically).
__device__ __forceinline__ float silu_bf16path(float x) {
  return __fmul_rn(x, rcp_approx(1.0f + ex2_approx(x * -1.4426950408889634f)));
}

// tanh-form GELU for bf16 outputs: 0.5 x (1 + tanh(z)) == x * sigmoid(2 z),
// z = sqrt(2/pi) (x + 0.044715 x^3) (examples/gpt2/kernels/gelu.py:9-12),
// shared by the elementwise kernel and the GEMM epilogues so both round
// identically.
__device__ __forceinline__ float gelu_tanh_bf16path(float x) {
  const float kBeta = 0.7978845608028654f;  // sqrt(2/pi)
  const float kKappa = 0.044715f;
  const float x3 = __fmul_rn(__fmul_rn(x, x), x);
  const float inner = __fmul_rn(kBeta, __fadd_rn(x, __fmul_rn(kKappa, x3)));
  return __fmul_rn(x, rcp_approx(1.0f + ex2_approx(__fmul_rn(2.0f, inner) * -1.4426950408889634f)));
}

// Is (v2, i2) a better argmax candidate than (v1, i1)?  Larger value wins,
// then the smaller index; NaN is larger than every number (torch.argmax);
// an index >= cols is "no candidate".  A total order, so any reduction tree
// gives the first index of the maximum.
__device__ __forceinline__ bool argmax_better(float v1, int64_t i1, float v2, int64_t i2, int64_t cols) {
  if (i2 >= cols) return false;
  if (i1 >= cols) return true;
  const bool n1 = v1 != v1, n2 = v2 != v2;
  if (n1 || n2) return n1 && n2 ? i2 < i1 : n2;
  return v2 > v1 || (v2 == v1 && i2 < i1);
}

// ---- programmatic dependent launch ----------------------------------------
// Every kernel waits for its predecessor on the stream with pdl_wait() before
// touching global memory, then lets its own successor begin launching
// (pdl_trigger).  When a kernel is launched with programmatic stream
// serialisation (launch_k below), its launch and any prologue placed before
// pdl_wait() overlap the tail of the previous kernel; correctness is
// unchanged because griddepcontrol.wait returns only once the prerequisite
// grid has completed and its memory is visible.  Without the attribute both
// instructions are no-ops.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// XB_PDL=0 in the environment turns the overlap off (plain launches).
inline bool pdl_enabled() {
  static int on = -1;
  if (on < 0) {
    const char* v = getenv("XB_PDL");
    on = (v && v[0] == '0') ? 0 : 1;
  }
  return on == 1;
}

// Kernels launched by this library since it was loaded (host-side count of
// launch calls, stream capture included; read with xb_launch_count).
inline std::atomic<unsigned long long>& launch_counter() {
  static std::atomic<unsigned long long> n{0};
  return n;
}

constexpr int kMaxDevices = 64;

// Set-up done once per (kernel, what, device).  Kernel attributes set with
// cudaFuncSetAttribute belong to the device that was current at the call, so
// a process that drives several GPUs must set them on each one.  The registry
// is shared by every translation unit of the library and guarded by a mutex
// (host threads may launch concurrently).
struct OnceEntry {
  const void* key;
  int what, dev, value;
};
struct OnceRegistry {
  std::mutex mu;
  std::vector<OnceEntry> done;
};
inline OnceRegistry& once_registry() {
  static OnceRegistry r;
  return r;
}
enum : int { kOnceCarveout = 0, kOnceSmem = 1, kOnceClusters = 16 };  // kOnceClusters + cluster size

// Runs setup(&value) the first time (key, what) is seen on the current device
// and stores `value`; later calls on that device return the stored value
// through *value.  A failed set-up is not recorded (the next call retries).
template <typename F>
inline cudaError_t once_per_device(const void* key, int what, F&& setup, int* value = nullptr) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  OnceRegistry& r = once_registry();
  std::lock_guard<std::mutex> lock(r.mu);
  for (const OnceEntry& o : r.done)
    if (o.key == key && o.what == what && o.dev == dev) {
      if (value) *value = o.value;
      return cudaSuccess;
    }
  int v = 0;
  e = setup(&v);
  if (e != cudaSuccess) return e;
  r.done.push_back({key, what, dev, v});
  if (value) *value = v;
  return cudaSuccess;
}

// Every kernel of the library prefers the largest shared-memory carveout, so
// consecutive kernels never force an SM to drain and reconfigure its L1 /
// shared split (which would serialise them despite programmatic launch).
inline void prefer_max_smem(const void* fn) {
  once_per_device(fn, kOnceCarveout, [fn](int*) {
    cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout, (int)cudaSharedmemCarveoutMaxShared);
    cudaGetLastError();  // a preference only: a refusal is not an error of the launch
    return cudaSuccess;
  });
}

// kMaxSmem = false keeps the default carveout: the streaming elementwise and
// pooling kernels lose bandwidth with the smallest L1.
template <bool kMaxSmem = true, typename... KArgs, typename... Args>
inline cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                            Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  if (kMaxSmem) prefer_max_smem(reinterpret_cast<const void*>(kernel));
  launch_counter().fetch_add(1, std::memory_order_relaxed);
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// 16-byte vector of T.
template <typename T> struct Vec16 {
  static constexpr int N = 16 / sizeof(T);
  T v[N];
};

template <typename T>
__device__ __forceinline__ Vec16<T> ld16_stream(const T* p) {
  Vec16<T> r;
  int4 raw = __ldcs(reinterpret_cast<const int4*>(p));
  memcpy(&r, &raw, 16);
  return r;
}
template <typename T>
__device__ __forceinline__ Vec16<T> ld16(const T* p) {
  Vec16<T> r;
  int4 raw = __ldg(reinterpret_cast<const int4*>(p));
  memcpy(&r, &raw, 16);
  return r;
}
template <typename T>
__device__ __forceinline__ void st16_stream(T* p, const Vec16<T>& v) {
  int4 raw;
  memcpy(&raw, &v, 16);
  __stcs(reinterpret_cast<int4*>(p), raw);
}
template <typename T>
__device__ __forceinline__ void st16(T* p, const Vec16<T>& v) {
  int4 raw;
  memcpy(&raw, &v, 16);
  *reinterpret_cast<int4*>(p) = raw;
}

}  // namespace xb

// Dispatch on the runtime dtype code to a templated launcher.
#define XB_DISPATCH_FLOAT(dt, T, what, err, errlen, ...)                       \
  do {                                                                         \
    if ((dt) == XB_DT_BF16) {                                                  \
      using T = __nv_bfloat16;                                                 \
      __VA_ARGS__;                                                             \
    } else if ((dt) == XB_DT_F32) {                                            \
      using T = float;                                                         \
      __VA_ARGS__;                                                             \
    } else {                                                                   \
      ::xb::set_err(err, errlen, "%s: unsupported dtype code %d (want bf16=%d or f32=%d)", \
                    what, (int)(dt), XB_DT_BF16, XB_DT_F32);                   \
      return XB_ERR_UNSUPPORTED;                                               \
    }                                                                          \
  } while (0)
