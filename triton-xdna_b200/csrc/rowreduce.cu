// Row-reduction kernels: softmax, layernorm, rms_norm / weighted rms_norm and
// row centering (the example called average_pool).  HBM-bound: each row is
// read once into registers with 16-byte loads, reduced with warp shuffles
// (plus one shared-memory exchange when a row spans several warps), and
// written once.  fp32 accumulation throughout.
//
// A "group" of GROUP threads owns one row; each thread holds VPT 16-byte
// vectors of it (slot k of thread t is vector k*GROUP + t, so every load
// instruction of a group is one contiguous span).  GROUP <= 32 packs
// 256/GROUP rows into a 256-thread CTA with shuffle-only reductions; GROUP > 32
// is one row per CTA.  Rows that do not fit in registers, or whose length or
// stride is not a whole number of vectors, take a scalar fallback that walks
// the row from global memory (L2-resident re-reads).
//
// Formulas restate the examples' torch CPU checks:
//   softmax     examples/test_softmax/test_softmax.py:77        torch.softmax(x, 1)
//   layernorm   examples/test_layernorm/test_layernorm.py:36-53 (mean, var, rsqrt), plus gamma/beta
//               as in examples/gpt2/kernels/layernorm.py:21-57
//   rms_norm    examples/rms_norm/rms_norm.py:64-68             x * rsqrt(mean(x^2) + eps)
//   weighted    examples/weighted_rms_norm/weighted_rms_norm.py:68-73   (... ) * w
//   row_center  examples/average_pool/average_pool.py:61-64    x - mean(x)
#include "common.cuh"

namespace xb {
namespace {

enum RowOp { kSoftmax = 0, kLayerNorm = 1, kRmsNorm = 2, kRowCenter = 3 };

struct RowArgs {
  const void* x;
  void* y;
  const void* w;  // layernorm gamma / rms weight (nullable)
  const void* b;  // layernorm beta (nullable)
  int64_t rows, cols, xs, ys;
  float eps;
};

// exp(x - m): for bf16 rows the hardware exp2 (FFMA + one MUFU) keeps the
// kernel HBM-bound; fp32 rows use expf.
template <typename T>
__device__ __forceinline__ float exp_shifted(float x, float m) {
  if constexpr (sizeof(T) == 2) return ex2_approx((x - m) * 1.4426950408889634f);
  else return expf(x - m);
}

template <int GROUP, bool MAX>
__device__ __forceinline__ float group_reduce(float v, float* red) {
  constexpr int W = GROUP < 32 ? GROUP : 32;
#pragma unroll
  for (int o = W / 2; o > 0; o >>= 1) {
    float t = __shfl_xor_sync(0xffffffffu, v, o);
    v = MAX ? fmaxf(v, t) : v + t;
  }
  if constexpr (GROUP > 32) {
    constexpr int NW = GROUP / 32;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();  // previous use of red[] is finished
    if (lane == 0) red[warp] = v;
    __syncthreads();
    v = red[0];
#pragma unroll
    for (int i = 1; i < NW; ++i) v = MAX ? fmaxf(v, red[i]) : v + red[i];
  }
  return v;
}

// DECODE (no effect on the arithmetic) makes a separate copy of the kernel
// for launches of at most 256 rows, which prefers the largest shared-memory
// carveout: a decode step's norm then shares the SMs with the weight
// prefetch of the GEMM after it, while large batches keep the L1 they need.
template <typename T, int GROUP, int VPT, int OP, int DECODE = 0>
__global__ void __launch_bounds__(GROUP > 32 ? GROUP : 256) row_vec_kernel(RowArgs a) {
  pdl_wait();
  pdl_trigger();
  constexpr int VN = Vec16<T>::N;
  constexpr int CTA = GROUP > 32 ? GROUP : 256;
  constexpr int RPC = CTA / GROUP;
  __shared__ float red[GROUP > 32 ? GROUP / 32 : 1];

  const int t = threadIdx.x % GROUP;
  const int64_t row = (int64_t)blockIdx.x * RPC + threadIdx.x / GROUP;
  // Rows past the end still take part in the (whole-CTA) reductions when
  // GROUP > 32; with GROUP <= 32 a whole group is past the end together.
  const bool row_ok = row < a.rows;
  const int64_t nvec = a.cols / VN;
  const T* xr = static_cast<const T*>(a.x) + (row_ok ? row : 0) * a.xs;

  float v[VPT][VN];
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int64_t vi = (int64_t)k * GROUP + t;
    if (row_ok && vi < nvec) {
      Vec16<T> q = ld16_stream(xr + vi * VN);
#pragma unroll
      for (int e = 0; e < VN; ++e) v[k][e] = Cvt<T>::to_f(q.v[e]);
    } else {
#pragma unroll
      for (int e = 0; e < VN; ++e) v[k][e] = 0.0f;
    }
  }
  const float inv_n = 1.0f / (float)a.cols;

  if constexpr (OP == kSoftmax) {
    float m = -INFINITY;
#pragma unroll
    for (int k = 0; k < VPT; ++k)
      if ((int64_t)k * GROUP + t < nvec)
#pragma unroll
        for (int e = 0; e < VN; ++e) m = fmaxf(m, v[k][e]);
    m = group_reduce<GROUP, true>(m, red);
    float s = 0.0f;
#pragma unroll
    for (int k = 0; k < VPT; ++k)
      if ((int64_t)k * GROUP + t < nvec)
#pragma unroll
        for (int e = 0; e < VN; ++e) {
          v[k][e] = exp_shifted<T>(v[k][e], m);
          s += v[k][e];
        }
    s = group_reduce<GROUP, false>(s, red);
    const float r = 1.0f / s;
#pragma unroll
    for (int k = 0; k < VPT; ++k)
#pragma unroll
      for (int e = 0; e < VN; ++e) v[k][e] = v[k][e] * r;
  } else if constexpr (OP == kLayerNorm || OP == kRowCenter) {
    float s = 0.0f;
#pragma unroll
    for (int k = 0; k < VPT; ++k)
#pragma unroll
      for (int e = 0; e < VN; ++e) s += v[k][e];
    const float mean = group_reduce<GROUP, false>(s, red) * inv_n;
    if constexpr (OP == kRowCenter) {
#pragma unroll
      for (int k = 0; k < VPT; ++k)
#pragma unroll
        for (int e = 0; e < VN; ++e) v[k][e] = v[k][e] - mean;
    } else {
      float q = 0.0f;
#pragma unroll
      for (int k = 0; k < VPT; ++k)
        if ((int64_t)k * GROUP + t < nvec)
#pragma unroll
          for (int e = 0; e < VN; ++e) {
            const float d = v[k][e] - mean;
            q += d * d;
          }
      const float var = group_reduce<GROUP, false>(q, red) * inv_n;
      const float rstd = __frsqrt_rn(var + a.eps);
      const T* g = static_cast<const T*>(a.w);
      const T* b = static_cast<const T*>(a.b);
#pragma unroll
      for (int k = 0; k < VPT; ++k) {
        const int64_t vi = (int64_t)k * GROUP + t;
        if (vi < nvec) {
          float gv[VN], bv[VN];
          if (g) { Vec16<T> q2 = ld16(g + vi * VN); for (int e = 0; e < VN; ++e) gv[e] = Cvt<T>::to_f(q2.v[e]); }
          else { for (int e = 0; e < VN; ++e) gv[e] = 1.0f; }
          if (b) { Vec16<T> q2 = ld16(b + vi * VN); for (int e = 0; e < VN; ++e) bv[e] = Cvt<T>::to_f(q2.v[e]); }
          else { for (int e = 0; e < VN; ++e) bv[e] = 0.0f; }
#pragma unroll
          for (int e = 0; e < VN; ++e) v[k][e] = (v[k][e] - mean) * rstd * gv[e] + bv[e];
        }
      }
    }
  } else {  // kRmsNorm
    float q = 0.0f;
#pragma unroll
    for (int k = 0; k < VPT; ++k)
#pragma unroll
      for (int e = 0; e < VN; ++e) q += v[k][e] * v[k][e];
    const float ms = group_reduce<GROUP, false>(q, red) * inv_n;
    const float rstd = __frsqrt_rn(ms + a.eps);
    const T* w = static_cast<const T*>(a.w);
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int64_t vi = (int64_t)k * GROUP + t;
      if (vi < nvec) {
        if (w) {
          Vec16<T> q2 = ld16(w + vi * VN);
#pragma unroll
          for (int e = 0; e < VN; ++e) v[k][e] = __fmul_rn(__fmul_rn(v[k][e], rstd), Cvt<T>::to_f(q2.v[e]));
        } else {
#pragma unroll
          for (int e = 0; e < VN; ++e) v[k][e] = __fmul_rn(v[k][e], rstd);
        }
      }
    }
  }

  if (!row_ok) return;
  T* yr = static_cast<T*>(a.y) + row * a.ys;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int64_t vi = (int64_t)k * GROUP + t;
    if (vi < nvec) {
      Vec16<T> o;
#pragma unroll
      for (int e = 0; e < VN; ++e) o.v[e] = Cvt<T>::from_f(v[k][e]);
      st16_stream(yr + vi * VN, o);
    }
  }
}

// Scalar fallback: one 256-thread CTA per row, statistics accumulated over a
// strided walk of the row, then a second walk writes the output.
template <typename T, int OP>
__global__ void __launch_bounds__(256) row_generic_kernel(RowArgs a) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[8];
  const int64_t row = blockIdx.x;
  const T* xr = static_cast<const T*>(a.x) + row * a.xs;
  T* yr = static_cast<T*>(a.y) + row * a.ys;
  const float inv_n = 1.0f / (float)a.cols;
  float p0 = 0.0f, p1 = 0.0f;
  if constexpr (OP == kSoftmax) {
    float m = -INFINITY;
    for (int64_t c = threadIdx.x; c < a.cols; c += 256) m = fmaxf(m, Cvt<T>::to_f(xr[c]));
    m = group_reduce<256, true>(m, red);
    float s = 0.0f;
    for (int64_t c = threadIdx.x; c < a.cols; c += 256) s += expf(Cvt<T>::to_f(xr[c]) - m);
    s = group_reduce<256, false>(s, red);
    p0 = m;
    p1 = 1.0f / s;
    for (int64_t c = threadIdx.x; c < a.cols; c += 256) yr[c] = Cvt<T>::from_f(expf(Cvt<T>::to_f(xr[c]) - p0) * p1);
  } else if constexpr (OP == kLayerNorm || OP == kRowCenter) {
    float s = 0.0f;
    for (int64_t c = threadIdx.x; c < a.cols; c += 256) s += Cvt<T>::to_f(xr[c]);
    const float mean = group_reduce<256, false>(s, red) * inv_n;
    if constexpr (OP == kRowCenter) {
      for (int64_t c = threadIdx.x; c < a.cols; c += 256) yr[c] = Cvt<T>::from_f(Cvt<T>::to_f(xr[c]) - mean);
    } else {
      float q = 0.0f;
      for (int64_t c = threadIdx.x; c < a.cols; c += 256) {
        const float d = Cvt<T>::to_f(xr[c]) - mean;
        q += d * d;
      }
      const float rstd = __frsqrt_rn(group_reduce<256, false>(q, red) * inv_n + a.eps);
      const T* g = static_cast<const T*>(a.w);
      const T* b = static_cast<const T*>(a.b);
      for (int64_t c = threadIdx.x; c < a.cols; c += 256) {
        const float gv = g ? Cvt<T>::to_f(g[c]) : 1.0f;
        const float bv = b ? Cvt<T>::to_f(b[c]) : 0.0f;
        yr[c] = Cvt<T>::from_f((Cvt<T>::to_f(xr[c]) - mean) * rstd * gv + bv);
      }
    }
  } else {
    float q = 0.0f;
    for (int64_t c = threadIdx.x; c < a.cols; c += 256) {
      const float xv = Cvt<T>::to_f(xr[c]);
      q += xv * xv;
    }
    const float rstd = __frsqrt_rn(group_reduce<256, false>(q, red) * inv_n + a.eps);
    const T* w = static_cast<const T*>(a.w);
    for (int64_t c = threadIdx.x; c < a.cols; c += 256) {
      float o = __fmul_rn(Cvt<T>::to_f(xr[c]), rstd);
      if (w) o = __fmul_rn(o, Cvt<T>::to_f(w[c]));
      yr[c] = Cvt<T>::from_f(o);
    }
  }
}

template <typename T, int GROUP, int VPT, int OP>
void launch_vec(const RowArgs& a, cudaStream_t s) {
  constexpr int CTA = GROUP > 32 ? GROUP : 256;
  constexpr int RPC = CTA / GROUP;
  const int64_t grid = (a.rows + RPC - 1) / RPC;
  if constexpr (GROUP > 32 && GROUP <= 128) {
    if (a.rows <= 256) {
      launch_k<true>(row_vec_kernel<T, GROUP, VPT, OP, 1>, (unsigned)grid, CTA, 0, s, a);
      return;
    }
  }
  launch_k<false>(row_vec_kernel<T, GROUP, VPT, OP>, (unsigned)grid, CTA, 0, s, a);
}

// Pick (GROUP, VPT) for a row of nvec vectors; returns false if the row does
// not fit the register path.
template <typename T, int OP>
bool dispatch_vec(const RowArgs& a, int64_t nvec, cudaStream_t s) {
  constexpr int MAXV = sizeof(T) == 2 ? 4 : 8;  // at most 32 fp32 values per thread
  // The configuration depends on the row length only, never on the row
  // count, so a row is reduced in the same order whatever the batch (batch
  // invariance).  Rows of up to 32 * MAXV vectors (the 768- and 896-wide
  // hidden states of GPT-2 and Qwen2.5-0.5B included) take a warp (or less)
  // each, several 16-byte loads in flight per lane; rows of 129..256 vectors
  // get one row per CTA.
  if (nvec > 32 * MAXV && nvec <= 256) {
    launch_vec<T, 128, 2, OP>(a, s);
    return true;
  }
  if (nvec <= 32 * MAXV) {
    int g = 4;
    while (g * MAXV < nvec) g *= 2;
    int vpt = 1;
    while ((int64_t)g * vpt < nvec) vpt *= 2;
#define XB_CASE(G, V) \
  if (g == G && vpt == V) { launch_vec<T, G, V, OP>(a, s); return true; }
    XB_CASE(4, 1) XB_CASE(4, 2) XB_CASE(4, 4)
    XB_CASE(8, 1) XB_CASE(8, 2) XB_CASE(8, 4)
    XB_CASE(16, 1) XB_CASE(16, 2) XB_CASE(16, 4)
    XB_CASE(32, 1) XB_CASE(32, 2) XB_CASE(32, 4)
    if constexpr (MAXV == 8) {
      XB_CASE(4, 8) XB_CASE(8, 8) XB_CASE(16, 8) XB_CASE(32, 8)
    }
#undef XB_CASE
    return false;
  }
  int g = 64;
  while ((int64_t)g * MAXV < nvec && g < 1024) g *= 2;
  if ((int64_t)g * MAXV < nvec) return false;
  switch (g) {
    case 64: launch_vec<T, 64, MAXV, OP>(a, s); return true;
    case 128: launch_vec<T, 128, MAXV, OP>(a, s); return true;
    case 256: launch_vec<T, 256, MAXV, OP>(a, s); return true;
    case 512: launch_vec<T, 512, MAXV, OP>(a, s); return true;
    case 1024: launch_vec<T, 1024, MAXV, OP>(a, s); return true;
  }
  return false;
}

template <typename T, int OP>
int run_row(const RowArgs& a, cudaStream_t s, const char* what, char* err, size_t errlen) {
  if (a.rows < 0 || a.cols < 0) { set_err(err, errlen, "%s: negative shape", what); return XB_ERR_INVALID; }
  if (a.rows == 0) return XB_OK;
  if (a.cols == 0) { set_err(err, errlen, "%s: rows of zero length", what); return XB_ERR_INVALID; }
  if (!a.x || !a.y) { set_err(err, errlen, "%s: null pointer", what); return XB_ERR_INVALID; }
  if (a.xs < a.cols || a.ys < a.cols) {
    set_err(err, errlen, "%s: row stride (%lld, %lld) shorter than the row (%lld)", what, (long long)a.xs,
            (long long)a.ys, (long long)a.cols);
    return XB_ERR_INVALID;
  }
  if (a.rows > 0x7fffffffLL) { set_err(err, errlen, "%s: too many rows", what); return XB_ERR_UNSUPPORTED; }
  constexpr int VN = Vec16<T>::N;
  const bool vec_ok = a.cols % VN == 0 && a.xs % VN == 0 && a.ys % VN == 0 && aligned16(a.x) && aligned16(a.y) &&
                      (!a.w || aligned16(a.w)) && (!a.b || aligned16(a.b));
  if (!(vec_ok && dispatch_vec<T, OP>(a, a.cols / VN, s)))
    launch_k<false>(row_generic_kernel<T, OP>, (unsigned)a.rows, 256, 0, s, a);
  return check_launch(what, err, errlen);
}

}  // namespace
}  // namespace xb

using namespace xb;

extern "C" int xb_softmax(const void* x, void* y, int64_t rows, int64_t cols, int64_t xs, int64_t ys, int dtype,
                          void* stream, char* err, size_t errlen) {
  RowArgs a{x, y, nullptr, nullptr, rows, cols, xs, ys, 0.0f};
  XB_DISPATCH_FLOAT(dtype, T, "xb_softmax", err, errlen,
                    return run_row<T, kSoftmax>(a, (cudaStream_t)stream, "xb_softmax", err, errlen));
}

extern "C" int xb_layernorm(const void* x, const void* gamma, const void* beta, void* y, int64_t rows, int64_t cols,
                            int64_t xs, int64_t ys, float eps, int dtype, void* stream, char* err, size_t errlen) {
  RowArgs a{x, y, gamma, beta, rows, cols, xs, ys, eps};
  XB_DISPATCH_FLOAT(dtype, T, "xb_layernorm", err, errlen,
                    return run_row<T, kLayerNorm>(a, (cudaStream_t)stream, "xb_layernorm", err, errlen));
}

extern "C" int xb_rms_norm(const void* x, const void* w, void* y, int64_t rows, int64_t cols, int64_t xs, int64_t ys,
                           float eps, int dtype, void* stream, char* err, size_t errlen) {
  RowArgs a{x, y, w, nullptr, rows, cols, xs, ys, eps};
  XB_DISPATCH_FLOAT(dtype, T, "xb_rms_norm", err, errlen,
                    return run_row<T, kRmsNorm>(a, (cudaStream_t)stream, "xb_rms_norm", err, errlen));
}

extern "C" int xb_row_center(const void* x, void* y, int64_t rows, int64_t cols, int64_t xs, int64_t ys, int dtype,
                             void* stream, char* err, size_t errlen) {
  RowArgs a{x, y, nullptr, nullptr, rows, cols, xs, ys, 0.0f};
  XB_DISPATCH_FLOAT(dtype, T, "xb_row_center", err, errlen,
                    return run_row<T, kRowCenter>(a, (cudaStream_t)stream, "xb_row_center", err, errlen));
}
