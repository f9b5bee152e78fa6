// Flat elementwise / activation kernels (HBM-bound streaming).
//
// One templated kernel family: each thread moves UNROLL=2 16-byte vectors
// (both loads issued before any math), math in fp32, streaming (evict-first)
// loads/stores because every byte is touched exactly once.  The grid covers
// the whole tensor in one pass ("one-shot": many short-lived CTAs, no
// grid-stride loop in practice): the hardware block scheduler then balances
// the work across the SMs of both dies, which measured ~15% faster on B200
// than an occupancy-sized persistent grid for the same kernel (6.8 vs
// 5.95 TB/s for a 2^28-element bf16 stream).  A scalar instantiation handles
// buffers that are not 16-byte aligned and the ragged tail.
//
// The functors restate the reference examples' torch CPU check expressions
// (the parity oracle), including where those round an intermediate to the
// storage dtype:
//   vecadd      examples/vec-add/vec-add.py:49          torch.add(a, b)
//   axpy        examples/axpy/axpy.py:40                alpha * x + y
//   relu        examples/relu/relu.py:35                torch.relu(x)
//   leaky_relu  examples/leaky_relu/leaky_relu.py:40    F.leaky_relu(x, 0.01)
//   gelu        examples/gelu/gelu.py:40                x * sigmoid(1.702 x.float()).to(dtype)
//   gelu_tanh   examples/gpt2/kernels/gelu.py:25-45     tanh-form GELU
//   sigmoid     examples/sigmoid/sigmoid.py:39          torch.sigmoid(x)
//   silu        examples/silu/silu.py:39                F.silu(x)
//   swiglu      examples/swiglu/swiglu.py:43            F.silu(gate) * up
#include "common.cuh"

namespace xb {
namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 2;

// Explicit _rn intrinsics keep the compiler from contracting a*b+c into an
// FMA: the torch expressions evaluate each operator separately.
//
// exp / reciprocal: for fp32 outputs, expf and the correctly rounded
// reciprocal __frcp_rn (a few ulp of fp32 from torch's results).  For bf16
// outputs the fp32 intermediate only has to be good to well under one bf16
// ulp (2^-8 relative), so the hardware approximations are used directly:
// ex2.approx and rcp.approx (relative error ~2^-22, one MUFU instruction
// each).  A sigmoid is then FMUL, EX2, FADD, RCP -- few enough instructions
// that the bf16 activations stay HBM-bound instead of issue-bound.  Both
// approximations flush subnormals, so a bf16 result below 2^-126 in
// magnitude (sigmoid(x) for x < -87.3) becomes 0.
//
// The bf16 form multiplies the reciprocal by an exact 1.0f (a no-op on every
// value): written without it, the bf16 sigmoid kernel measured 200.7 us on
// 2^28 elements against 176.0 us with it, the same bits out.
template <typename T>
__device__ __forceinline__ float sigmoid_t(float x) {
  if constexpr (sizeof(T) == 2) return __fmul_rn(1.0f, rcp_approx(1.0f + ex2_approx(x * -1.4426950408889634f)));
  else return __frcp_rn(__fadd_rn(1.0f, expf(-x)));
}

template <typename T> struct OpAdd {
  __device__ __forceinline__ float operator()(float a, float b) const { return __fadd_rn(a, b); }
};
template <typename T> struct OpAxpy {
  float alpha;
  __device__ __forceinline__ float operator()(float x, float y) const {
    return __fadd_rn(round_to<T>(__fmul_rn(alpha, x)), y);
  }
};
template <typename T> struct OpRelu {
  // torch.relu is clamp_min(x, 0): -0.0 and NaN pass through unchanged.
  __device__ __forceinline__ float operator()(float x) const { return x < 0.0f ? 0.0f : x; }
};
template <typename T> struct OpLeakyRelu {
  float slope;
  __device__ __forceinline__ float operator()(float x) const { return x > 0.0f ? x : __fmul_rn(x, slope); }
};
template <typename T> struct OpGeluSigmoid {
  __device__ __forceinline__ float operator()(float x) const {
    float s = round_to<T>(sigmoid_t<T>(__fmul_rn(1.702f, x)));
    return __fmul_rn(x, s);
  }
};
template <typename T> struct OpGeluTanh {
  __device__ __forceinline__ float operator()(float x) const {
    if constexpr (sizeof(T) == 2) {
      return gelu_tanh_bf16path(x);
    } else {
      const float kBeta = 0.7978845608028654f;  // sqrt(2/pi)
      const float kKappa = 0.044715f;
      float x3 = __fmul_rn(__fmul_rn(x, x), x);
      float inner = __fmul_rn(kBeta, __fadd_rn(x, __fmul_rn(kKappa, x3)));
      // fp32: the same formula as torch's tanh GELU, so the cancellation in
      // 1 + tanh(z) for negative x rounds the same way.
      return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, tanhf(inner)));
    }
  }
};
template <typename T> struct OpSigmoid {
  __device__ __forceinline__ float operator()(float x) const { return sigmoid_t<T>(x); }
};
template <typename T> struct OpSilu {
  __device__ __forceinline__ float operator()(float x) const {
    if constexpr (sizeof(T) == 2) return silu_bf16path(x);
    else return __fdiv_rn(x, __fadd_rn(1.0f, expf(-x)));
  }
};
template <typename T> struct OpSwiglu {
  __device__ __forceinline__ float operator()(float g, float u) const {
    float s = round_to<T>(OpSilu<T>{}(g));
    return __fmul_rn(s, u);
  }
};

// silu(g) * u in fp32 with a single rounding: the Qwen2.5 MLP form
// (examples/qwen2_5/kernels/swiglu.py:29-50, model.py:781-786), unlike the
// swiglu example, which rounds silu(g) to the storage type first.
template <typename T> struct OpMul {
  __device__ __forceinline__ float operator()(float a, float b) const { return __fmul_rn(a, b); }
};

template <typename T> struct OpSiluMul {
  __device__ __forceinline__ float operator()(float g, float u) const { return __fmul_rn(OpSilu<T>{}(g), u); }
};

template <typename T, typename Op>
__global__ void __launch_bounds__(kThreads) unary_vec_kernel(const T* __restrict__ x, T* __restrict__ y,
                                                             int64_t nvec, Op op) {
  pdl_wait();
  pdl_trigger();
  using V = Vec16<T>;
  const int64_t step = (int64_t)gridDim.x * kThreads * kUnroll;
  for (int64_t base = (int64_t)blockIdx.x * kThreads * kUnroll + threadIdx.x; base < nvec; base += step) {
    V v[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      int64_t i = base + (int64_t)u * kThreads;
      if (i < nvec) v[u] = ld16_stream(x + i * V::N);
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      int64_t i = base + (int64_t)u * kThreads;
      if (i < nvec) {
        V o;
#pragma unroll
        for (int e = 0; e < V::N; ++e) o.v[e] = Cvt<T>::from_f(op(Cvt<T>::to_f(v[u].v[e])));
        st16_stream(y + i * V::N, o);
      }
    }
  }
}

template <typename T, typename Op>
__global__ void __launch_bounds__(kThreads) binary_vec_kernel(const T* __restrict__ a, const T* __restrict__ b,
                                                              T* __restrict__ y, int64_t nvec, Op op) {
  pdl_wait();
  pdl_trigger();
  using V = Vec16<T>;
  const int64_t step = (int64_t)gridDim.x * kThreads * kUnroll;
  for (int64_t base = (int64_t)blockIdx.x * kThreads * kUnroll + threadIdx.x; base < nvec; base += step) {
    V va[kUnroll], vb[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      int64_t i = base + (int64_t)u * kThreads;
      if (i < nvec) {
        va[u] = ld16_stream(a + i * V::N);
        vb[u] = ld16_stream(b + i * V::N);
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      int64_t i = base + (int64_t)u * kThreads;
      if (i < nvec) {
        V o;
#pragma unroll
        for (int e = 0; e < V::N; ++e)
          o.v[e] = Cvt<T>::from_f(op(Cvt<T>::to_f(va[u].v[e]), Cvt<T>::to_f(vb[u].v[e])));
        st16_stream(y + i * V::N, o);
      }
    }
  }
}

// Scalar path: elements [begin, n).  Used for the tail after the vector body
// and for whole buffers that are not 16-byte aligned.
template <typename T, typename Op>
__global__ void unary_scalar_kernel(const T* __restrict__ x, T* __restrict__ y, int64_t begin, int64_t n, Op op) {
  pdl_wait();
  pdl_trigger();
  for (int64_t i = begin + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    y[i] = Cvt<T>::from_f(op(Cvt<T>::to_f(x[i])));
}
template <typename T, typename Op>
__global__ void binary_scalar_kernel(const T* __restrict__ a, const T* __restrict__ b, T* __restrict__ y,
                                     int64_t begin, int64_t n, Op op) {
  pdl_wait();
  pdl_trigger();
  for (int64_t i = begin + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    y[i] = Cvt<T>::from_f(op(Cvt<T>::to_f(a[i]), Cvt<T>::to_f(b[i])));
}

int grid_for(int64_t work_items, int per_block) {
  int sms = 148;
  sm_count(&sms);
  int64_t want = (work_items + per_block - 1) / per_block;
  int64_t cap = (int64_t)sms * 8;
  if (want > cap) want = cap;
  if (want < 1) want = 1;
  return (int)want;
}

// One-shot grid: enough CTAs to cover every vector once (the kernels keep a
// grid-stride loop only for tensors beyond 2^31 CTAs).
int oneshot_grid(int64_t work_items, int per_block) {
  int64_t want = (work_items + per_block - 1) / per_block;
  if (want > 0x7fffffffLL) want = 0x7fffffffLL;
  if (want < 1) want = 1;
  return (int)want;
}

template <typename T, typename Op>
int launch_unary(const void* xv, void* yv, int64_t n, Op op, cudaStream_t s, const char* what, char* err,
                 size_t errlen) {
  if (n < 0) { set_err(err, errlen, "%s: negative element count %lld", what, (long long)n); return XB_ERR_INVALID; }
  if (n == 0) return XB_OK;
  if (!xv || !yv) { set_err(err, errlen, "%s: null pointer", what); return XB_ERR_INVALID; }
  const T* x = static_cast<const T*>(xv);
  T* y = static_cast<T*>(yv);
  constexpr int VN = Vec16<T>::N;
  int64_t nvec = (aligned16(x) && aligned16(y)) ? n / VN : 0;
  if (nvec > 0)
    launch_k<false>(unary_vec_kernel<T, Op>, oneshot_grid(nvec, kThreads * kUnroll), kThreads, 0, s, x, y, nvec, op);
  if (nvec * VN < n)
    launch_k<false>(unary_scalar_kernel<T, Op>, grid_for(n - nvec * VN, kThreads), kThreads, 0, s, x, y, nvec * VN, n, op);
  return check_launch(what, err, errlen);
}

template <typename T, typename Op>
int launch_binary(const void* av, const void* bv, void* yv, int64_t n, Op op, cudaStream_t s, const char* what,
                  char* err, size_t errlen) {
  if (n < 0) { set_err(err, errlen, "%s: negative element count %lld", what, (long long)n); return XB_ERR_INVALID; }
  if (n == 0) return XB_OK;
  if (!av || !bv || !yv) { set_err(err, errlen, "%s: null pointer", what); return XB_ERR_INVALID; }
  const T* a = static_cast<const T*>(av);
  const T* b = static_cast<const T*>(bv);
  T* y = static_cast<T*>(yv);
  constexpr int VN = Vec16<T>::N;
  int64_t nvec = (aligned16(a) && aligned16(b) && aligned16(y)) ? n / VN : 0;
  if (nvec > 0)
    launch_k<false>(binary_vec_kernel<T, Op>, oneshot_grid(nvec, kThreads * kUnroll), kThreads, 0, s, a, b, y, nvec, op);
  if (nvec * VN < n)
    launch_k<false>(binary_scalar_kernel<T, Op>, grid_for(n - nvec * VN, kThreads), kThreads, 0, s, a, b, y, nvec * VN, n,
             op);
  return check_launch(what, err, errlen);
}

}  // namespace
}  // namespace xb

using namespace xb;

#define XB_S(stream) static_cast<cudaStream_t>(stream)

extern "C" int xb_vecadd(const void* a, const void* b, void* c, int64_t n, int dtype, void* stream, char* err,
                         size_t errlen) {
  XB_DISPATCH_FLOAT(dtype, T, "xb_vecadd", err, errlen,
                    return launch_binary<T>(a, b, c, n, OpAdd<T>{}, XB_S(stream), "xb_vecadd", err, errlen));
}

extern "C" int xb_axpy(const void* x, const void* y, void* out, float alpha, int64_t n, int dtype, void* stream,
                       char* err, size_t errlen) {
  XB_DISPATCH_FLOAT(dtype, T, "xb_axpy", err, errlen,
                    return launch_binary<T>(x, y, out, n, OpAxpy<T>{alpha}, XB_S(stream), "xb_axpy", err, errlen));
}

extern "C" int xb_relu(const void* x, void* y, int64_t n, int dtype, void* stream, char* err, size_t errlen) {
  XB_DISPATCH_FLOAT(dtype, T, "xb_relu", err, errlen,
                    return launch_unary<T>(x, y, n, OpRelu<T>{}, XB_S(stream), "xb_relu", err, errlen));
}

extern "C" int xb_leaky_relu(const void* x, void* y, float slope, int64_t n, int dtype, void* stream, char* err,
                             size_t errlen) {
  XB_DISPATCH_FLOAT(dtype, T, "xb_leaky_relu", err, errlen,
                    return launch_unary<T>(x, y, n, OpLeakyRelu<T>{slope}, XB_S(stream), "xb_leaky_relu", err,
                                           errlen));
}

extern "C" int xb_gelu(const void* x, void* y, int64_t n, int dtype, void* stream, char* err, size_t errlen) {
  XB_DISPATCH_FLOAT(dtype, T, "xb_gelu", err, errlen,
                    return launch_unary<T>(x, y, n, OpGeluSigmoid<T>{}, XB_S(stream), "xb_gelu", err, errlen));
}

extern "C" int xb_gelu_tanh(const void* x, void* y, int64_t n, int dtype, void* stream, char* err, size_t errlen) {
  XB_DISPATCH_FLOAT(dtype, T, "xb_gelu_tanh", err, errlen,
                    return launch_unary<T>(x, y, n, OpGeluTanh<T>{}, XB_S(stream), "xb_gelu_tanh", err, errlen));
}

extern "C" int xb_sigmoid(const void* x, void* y, int64_t n, int dtype, void* stream, char* err, size_t errlen) {
  XB_DISPATCH_FLOAT(dtype, T, "xb_sigmoid", err, errlen,
                    return launch_unary<T>(x, y, n, OpSigmoid<T>{}, XB_S(stream), "xb_sigmoid", err, errlen));
}

extern "C" int xb_silu(const void* x, void* y, int64_t n, int dtype, void* stream, char* err, size_t errlen) {
  XB_DISPATCH_FLOAT(dtype, T, "xb_silu", err, errlen,
                    return launch_unary<T>(x, y, n, OpSilu<T>{}, XB_S(stream), "xb_silu", err, errlen));
}

extern "C" int xb_swiglu(const void* gate, const void* up, void* out, int64_t n, int dtype, void* stream, char* err,
                         size_t errlen) {
  XB_DISPATCH_FLOAT(dtype, T, "xb_swiglu", err, errlen,
                    return launch_binary<T>(gate, up, out, n, OpSwiglu<T>{}, XB_S(stream), "xb_swiglu", err,
                                            errlen));
}

extern "C" int xb_mul(const void* a, const void* b, void* c, int64_t n, int dtype, void* stream, char* err,
                      size_t errlen) {
  XB_DISPATCH_FLOAT(dtype, T, "xb_mul", err, errlen,
                    return launch_binary<T>(a, b, c, n, OpMul<T>{}, XB_S(stream), "xb_mul", err, errlen));
}

// z[r, c] = x[r, c] * y[r, c] over a strided 2-D region (rows of `cols`
// elements, pitches in elements): the tiled block-pointer product of
// examples/load_2d_block/test_load_2d_tensor_block.py:27-82.
template <typename T>
__global__ void __launch_bounds__(256) mul2d_kernel(const T* __restrict__ x, const T* __restrict__ y, T* __restrict__ z,
                                                    int64_t rows, int64_t cols, int64_t ldx, int64_t ldy, int64_t ldz) {
  pdl_wait();
  pdl_trigger();
  const int64_t c = (int64_t)blockIdx.x * 256 + threadIdx.x;
  if (c >= cols) return;
  for (int64_t r = blockIdx.y; r < rows; r += gridDim.y)
    z[r * ldz + c] = Cvt<T>::from_f(__fmul_rn(Cvt<T>::to_f(x[r * ldx + c]), Cvt<T>::to_f(y[r * ldy + c])));
}

extern "C" int xb_mul_2d(const void* x, const void* y, void* z, int64_t rows, int64_t cols, int64_t ldx, int64_t ldy,
                         int64_t ldz, int dtype, void* stream, char* err, size_t errlen) {
  if (rows < 0 || cols < 0 || ldx < cols || ldy < cols || ldz < cols) {
    set_err(err, errlen, "xb_mul_2d: bad shape or pitch");
    return XB_ERR_INVALID;
  }
  if (rows == 0 || cols == 0) return XB_OK;
  if (!x || !y || !z) {
    set_err(err, errlen, "xb_mul_2d: null pointer");
    return XB_ERR_INVALID;
  }
  const dim3 grid((unsigned)((cols + 255) / 256), (unsigned)(rows < 65535 ? rows : 65535));
  XB_DISPATCH_FLOAT(dtype, T, "xb_mul_2d", err, errlen, {
    launch_k<false>(mul2d_kernel<T>, grid, 256, 0, XB_S(stream), static_cast<const T*>(x), static_cast<const T*>(y),
                    static_cast<T*>(z), rows, cols, ldx, ldy, ldz);
    return check_launch("xb_mul_2d", err, errlen);
  });
}

extern "C" int xb_silu_mul(const void* gate, const void* up, void* out, int64_t n, int dtype, void* stream, char* err,
                           size_t errlen) {
  XB_DISPATCH_FLOAT(dtype, T, "xb_silu_mul", err, errlen,
                    return launch_binary<T>(gate, up, out, n, OpSiluMul<T>{}, XB_S(stream), "xb_silu_mul", err,
                                            errlen));
}
