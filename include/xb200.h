/*
 * xb200 — C ABI of the B200 (sm_100a) operator library.
 *
 * The reference (amd/Triton-XDNA) launches each example operator through a
 * generated per-signature CPython launcher (amd_triton_npu/backend/driver.py:
 * 1375-1628, 1630-1832) or the HSA runtime C ABI
 * (amd_triton_npu/backend/include/HsaRuntime/HsaRuntime.h:34-71).  This header
 * replaces both with one precompiled entry point per operator.
 *
 * Conventions (shared by every entry point):
 *   - plain device pointers, element counts and strides in ELEMENTS;
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream);
 *     all work is enqueued on it, nothing synchronises;
 *   - the last two arguments are an error buffer and its length; on failure a
 *     NUL-terminated message is written there (as triton_npu_hsa_* do,
 *     HsaRuntime.cpp:740-794);
 *   - return 0 (XB_OK) on success, a negative XB_ERR_* code on failure.
 *     Argument errors are detected on the host before anything is launched.
 *   - dtype codes are the XB_DT_* values below.
 */
#ifndef XB200_H
#define XB200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define XB_API __attribute__((visibility("default")))
#else
#define XB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define XB_OK 0
#define XB_ERR_INVALID (-1)     /* bad argument: null pointer, negative size, ... */
#define XB_ERR_CUDA (-2)        /* a CUDA runtime call or a kernel launch failed */
#define XB_ERR_UNSUPPORTED (-3) /* dtype / layout / shape combination not implemented */
#define XB_ERR_TIMEOUT (-4)     /* a bounded device-side wait ran out */

#define XB_DT_BF16 0
#define XB_DT_F32 1
#define XB_DT_I8 2
#define XB_DT_I16 3
#define XB_DT_I32 4

/* Library ABI version (bumped when a signature changes). */
XB_API int xb_abi_version(void);

/* Name of CUDA device `device` ("NVIDIA B200") and its SM count.
 * Replaces triton_npu_hsa_agent_name (HsaRuntime.h:34-40), which reports the
 * NPU generation so callers can pick a code path. */
XB_API int xb_device_name(int device, char* buf, size_t buf_len, int* sm_count,
                   char* err, size_t errlen);

/* ---------------------------------------------------------------------------
 * Flat elementwise / activation operators.  x, y, out: n contiguous elements of
 * `dtype` (bf16 or f32); math in fp32, one rounding per stored value except
 * where noted (the reference's torch expression rounds an intermediate).
 * ------------------------------------------------------------------------- */

/* c = a + b.  Replaces `vecadd` (examples/vec-add/vec-add.py:16-35). */
XB_API int xb_vecadd(const void* a, const void* b, void* c, int64_t n, int dtype,
              void* stream, char* err, size_t errlen);

/* out = alpha*x + y, with alpha*x rounded to dtype before the add (torch's
 * `alpha * x + y` on a bf16 tensor).  Replaces `axpy_kernel`
 * (examples/axpy/axpy.py:13-29). */
XB_API int xb_axpy(const void* x, const void* y, void* out, float alpha, int64_t n,
            int dtype, void* stream, char* err, size_t errlen);

/* y = max(x, 0).  Replaces `relu_kernel` (examples/relu/relu.py:13-26). */
XB_API int xb_relu(const void* x, void* y, int64_t n, int dtype, void* stream,
            char* err, size_t errlen);

/* y = x >= 0 ? x : slope*x.  Replaces `leaky_relu_kernel`
 * (examples/leaky_relu/leaky_relu.py:15-31; slope 0.01 there). */
XB_API int xb_leaky_relu(const void* x, void* y, float slope, int64_t n, int dtype,
                  void* stream, char* err, size_t errlen);

/* y = x * sigmoid(1.702 x) (sigmoid-approximation GELU).  Replaces
 * `gelu_kernel` (examples/gelu/gelu.py:13-30). */
XB_API int xb_gelu(const void* x, void* y, int64_t n, int dtype, void* stream,
            char* err, size_t errlen);

/* y = 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))) (tanh-form GELU).
 * Replaces `gelu_kernel_gpu` (examples/gpt2/kernels/gelu.py:25-45). */
XB_API int xb_gelu_tanh(const void* x, void* y, int64_t n, int dtype, void* stream,
                 char* err, size_t errlen);

/* y = 1 / (1 + exp(-x)).  Replaces `sigmoid_kernel`
 * (examples/sigmoid/sigmoid.py:13-34). */
XB_API int xb_sigmoid(const void* x, void* y, int64_t n, int dtype, void* stream,
               char* err, size_t errlen);

/* y = x * sigmoid(x).  Replaces `silu_kernel` (examples/silu/silu.py:13-30). */
XB_API int xb_silu(const void* x, void* y, int64_t n, int dtype, void* stream,
            char* err, size_t errlen);

/* out = silu(gate) * up, silu(gate) rounded to dtype before the product.
 * Replaces `swiglu_kernel` (examples/swiglu/swiglu.py:13-33). */
XB_API int xb_swiglu(const void* gate, const void* up, void* out, int64_t n,
              int dtype, void* stream, char* err, size_t errlen);

/* ---------------------------------------------------------------------------
 * Row reductions over a [rows, cols] matrix with row strides (elements) and
 * unit column stride.  fp32 accumulation.
 * ------------------------------------------------------------------------- */

/* y = softmax(x) along each row (max-subtracted).  Replaces `softmax_kernel`
 * (examples/test_softmax/test_softmax.py:13-45). */
XB_API int xb_softmax(const void* x, void* y, int64_t rows, int64_t cols,
               int64_t x_row_stride, int64_t y_row_stride, int dtype,
               void* stream, char* err, size_t errlen);

/* y = (x - mean) * rsqrt(var + eps) * gamma + beta; gamma / beta may be NULL
 * (then 1 / 0, as in the example kernel).  Replaces `_layer_norm_fwd_fused`
 * (examples/test_layernorm/test_layernorm.py:13-60) and the affine GPT-2
 * `layernorm_kernel_gpu` (examples/gpt2/kernels/layernorm.py:21-57). */
XB_API int xb_layernorm(const void* x, const void* gamma, const void* beta, void* y,
                 int64_t rows, int64_t cols, int64_t x_row_stride,
                 int64_t y_row_stride, float eps, int dtype, void* stream,
                 char* err, size_t errlen);

/* y = x * rsqrt(mean(x^2) + eps) [* w]; w may be NULL.  Replaces
 * `rms_norm_kernel` (examples/rms_norm/rms_norm.py:23-55) and
 * `weighted_rms_norm_kernel` (examples/weighted_rms_norm/weighted_rms_norm.py:
 * 21-58). */
XB_API int xb_rms_norm(const void* x, const void* w, void* y, int64_t rows,
                int64_t cols, int64_t x_row_stride, int64_t y_row_stride,
                float eps, int dtype, void* stream, char* err, size_t errlen);

/* y = x - mean(x) along each row.  Replaces `avg_pool_kernel`
 * (examples/average_pool/average_pool.py:24-52). */
XB_API int xb_row_center(const void* x, void* y, int64_t rows, int64_t cols,
                  int64_t x_row_stride, int64_t y_row_stride, int dtype,
                  void* stream, char* err, size_t errlen);

/* 2x2 / stride-2 average pooling of contiguous NCHW x[planes, h, w] into
 * y[planes, h/2, w/2] (floor).  The 2-D pooling form of average_pool. */
XB_API int xb_avg_pool2d_2x2(const void* x, void* y, int64_t planes, int64_t h,
                      int64_t w, int dtype, void* stream, char* err,
                      size_t errlen);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* XB200_H */
