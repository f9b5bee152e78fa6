// 2x2 / stride-2 average pooling over contiguous NCHW planes (HBM-bound).
//
// Each thread produces one 16-byte output vector (4 fp32 or 8 bf16 outputs)
// from two 32-byte spans of the two input rows that feed it, so input and
// output are both moved with 16-byte accesses and every byte once.  The sum
// order ((x00 + x01) + x10) + x11 then / 4 follows torch's CPU avg_pool2d,
// the oracle for the 2-D pooling workload.  Odd heights / widths drop the last
// row / column (floor mode).
#include "common.cuh"

namespace xb {
namespace {

template <typename T>
__global__ void __launch_bounds__(256) pool_vec_kernel(const T* __restrict__ x, T* __restrict__ y, int64_t planes,
                                                       int64_t h, int64_t w, int64_t oh, int64_t ow) {
  pdl_wait();
  pdl_trigger();
  constexpr int VN = Vec16<T>::N;
  const int64_t ovr = ow / VN;  // output vectors per output row
  const int64_t total = planes * oh * ovr;
  for (int64_t o = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; o < total; o += (int64_t)gridDim.x * blockDim.x) {
    const int64_t j = o % ovr;
    const int64_t r = o / ovr;  // plane * oh + oi
    const int64_t plane = r / oh, oi = r - plane * oh;
    const T* r0 = x + (plane * h + 2 * oi) * w + 2 * j * VN;
    const T* r1 = r0 + w;
    Vec16<T> a0 = ld16_stream(r0), a1 = ld16_stream(r0 + VN);
    Vec16<T> b0 = ld16_stream(r1), b1 = ld16_stream(r1 + VN);
    Vec16<T> out;
#pragma unroll
    for (int e = 0; e < VN; ++e) {
      const int c = 2 * e;
      float x00, x01, x10, x11;
      if (c < VN) {
        x00 = Cvt<T>::to_f(a0.v[c]); x01 = Cvt<T>::to_f(a0.v[c + 1]);
        x10 = Cvt<T>::to_f(b0.v[c]); x11 = Cvt<T>::to_f(b0.v[c + 1]);
      } else {
        x00 = Cvt<T>::to_f(a1.v[c - VN]); x01 = Cvt<T>::to_f(a1.v[c - VN + 1]);
        x10 = Cvt<T>::to_f(b1.v[c - VN]); x11 = Cvt<T>::to_f(b1.v[c - VN + 1]);
      }
      out.v[e] = Cvt<T>::from_f((((x00 + x01) + x10) + x11) / 4.0f);
    }
    st16_stream(y + r * ow + j * VN, out);
  }
}

template <typename T>
__global__ void __launch_bounds__(256) pool_scalar_kernel(const T* __restrict__ x, T* __restrict__ y, int64_t planes,
                                                          int64_t h, int64_t w, int64_t oh, int64_t ow) {
  pdl_wait();
  pdl_trigger();
  const int64_t total = planes * oh * ow;
  for (int64_t o = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; o < total; o += (int64_t)gridDim.x * blockDim.x) {
    const int64_t oj = o % ow;
    const int64_t r = o / ow;
    const int64_t plane = r / oh, oi = r - plane * oh;
    const T* r0 = x + (plane * h + 2 * oi) * w + 2 * oj;
    const T* r1 = r0 + w;
    const float s = ((Cvt<T>::to_f(r0[0]) + Cvt<T>::to_f(r0[1])) + Cvt<T>::to_f(r1[0])) + Cvt<T>::to_f(r1[1]);
    y[o] = Cvt<T>::from_f(s / 4.0f);
  }
}

template <typename T>
int run_pool(const void* xv, void* yv, int64_t planes, int64_t h, int64_t w, cudaStream_t s, char* err,
             size_t errlen) {
  if (planes < 0 || h < 0 || w < 0) { set_err(err, errlen, "xb_avg_pool2d_2x2: negative shape"); return XB_ERR_INVALID; }
  const int64_t oh = h / 2, ow = w / 2;
  if (planes == 0 || oh == 0 || ow == 0) return XB_OK;
  if (!xv || !yv) { set_err(err, errlen, "xb_avg_pool2d_2x2: null pointer"); return XB_ERR_INVALID; }
  const T* x = static_cast<const T*>(xv);
  T* y = static_cast<T*>(yv);
  constexpr int VN = Vec16<T>::N;
  // one-shot grid (one output vector per thread): the block scheduler balances
  // the SMs better than a persistent grid-stride loop for a pure stream
  const int64_t cap = 0x7fffffffLL;
  if (w % (2 * VN) == 0 && ow % VN == 0 && aligned16(x) && aligned16(y)) {
    int64_t total = planes * oh * (ow / VN);
    int64_t grid = (total + 255) / 256;
    launch_k<false>(pool_vec_kernel<T>, (unsigned)(grid < cap ? grid : cap), 256, 0, s, x, y, planes, h, w, oh, ow);
  } else {
    int64_t total = planes * oh * ow;
    int64_t grid = (total + 255) / 256;
    launch_k<false>(pool_scalar_kernel<T>, (unsigned)(grid < cap ? grid : cap), 256, 0, s, x, y, planes, h, w, oh, ow);
  }
  return check_launch("xb_avg_pool2d_2x2", err, errlen);
}

}  // namespace
}  // namespace xb

extern "C" int xb_avg_pool2d_2x2(const void* x, void* y, int64_t planes, int64_t h, int64_t w, int dtype,
                                 void* stream, char* err, size_t errlen) {
  XB_DISPATCH_FLOAT(dtype, T, "xb_avg_pool2d_2x2", err, errlen,
                    return xb::run_pool<T>(x, y, planes, h, w, (cudaStream_t)stream, err, errlen));
}
