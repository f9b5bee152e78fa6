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

/* c = a * b elementwise (flat, n elements). */
XB_API int xb_mul(const void* a, const void* b, void* c, int64_t n, int dtype,
                  void* stream, char* err, size_t errlen);

/* z[r, c] = x[r, c] * y[r, c] over rows x cols with row pitches ldx, ldy,
 * ldz (elements): the tiled block-pointer product of
 * examples/load_2d_block/test_load_2d_tensor_block.py:27-82 (a 4-D block
 * pointer view of a 2-D tensor; every element of each program's block is
 * loaded, multiplied and stored once). */
XB_API int xb_mul_2d(const void* x, const void* y, void* z, int64_t rows,
                     int64_t cols, int64_t ldx, int64_t ldy, int64_t ldz,
                     int dtype, void* stream, char* err, size_t errlen);

/* out = silu(gate) * up evaluated in fp32 with one rounding (the Qwen2.5
 * MLP form).  Replaces `swiglu_kernel_gpu` (examples/qwen2_5/kernels/
 * swiglu.py:29-50). */
XB_API int xb_silu_mul(const void* gate, const void* up, void* out, int64_t n,
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

/* ---------------------------------------------------------------------------
 * Dense GEMMs on the tcgen05 tensor cores.  Row-major operands, leading
 * dimensions in elements.  A and B (and W) must start on a 16-byte boundary
 * with row pitches that are multiples of 16 bytes (TMA); C needs no alignment
 * beyond its element size.  Ragged M / N / K are handled.
 * ------------------------------------------------------------------------- */

/* C[M,N] (int32) = A[M,K] (int8) @ B[K,N] (int8), exact.  Replaces
 * `bare_matmul_i8` (examples/matmul_i8_m128_n64_k64/matmul_i8_m128_n64_k64.py:
 * 22-52, examples/matmul_i8_m64_n64_k64/matmul_i8_m64_n64_k64.py:21-51). */
XB_API int xb_matmul_i8(const void* A, const void* B, void* C, int64_t M,
                        int64_t N, int64_t K, int64_t lda, int64_t ldb,
                        int64_t ldc, void* stream, char* err, size_t errlen);

/* f32 GEMM with bf16 emulation: C[M,N] (f32) = bf16(A) @ bf16(B) with f32
 * accumulation, the operands rounded to bf16 (nearest even).  a_layout 0: A
 * is [M, K] (row pitch lda); 1: A is stored transposed, [K, M] (row pitch
 * lda).  B is [K, N].  M and N need not be multiples of any tile.  Needs
 * the workspace xb_matmul_f32_bf16emu_workspace_size reports (256-byte
 * aligned).  Replaces `padded_matmul_kernel` of
 * examples/matmul_f32_m64_n32_k16_padded_atransposed/
 * matmul_f32_m64_n32_k16_padded_atransposed.py:53-82 (A transposed, ragged
 * M/N, bf16 emulation, golden L140-161). */
XB_API int xb_matmul_f32_bf16emu_workspace_size(int64_t M, int64_t N,
                                                int64_t K, size_t* bytes,
                                                char* err, size_t errlen);
XB_API int xb_matmul_f32_bf16emu(const float* A, const float* B, float* C,
                                 int64_t M, int64_t N, int64_t K, int64_t lda,
                                 int64_t ldb, int64_t ldc, int a_layout,
                                 void* workspace, size_t workspace_bytes,
                                 void* stream, char* err, size_t errlen);

/* Y[M,N] (int32) = X[M,K] (int8) @ W[N,K]^T (int8), W in nn.Linear layout
 * (K-major): the int8 linear layer; exact.  The reference's int8 GEMM with
 * its B operand given transposed (examples/matmul_i8_m128_n64_k64). */
XB_API int xb_linear_i8(const void* X, const void* W, void* Y, int64_t M,
                        int64_t N, int64_t K, int64_t ldx, int64_t ldw,
                        int64_t ldy, void* stream, char* err, size_t errlen);

/* Bytes of device workspace xb_matmul_i16 needs for an M x N x K product.
 * The reference has int16 GEMM only as a README claim (README.md:21) with an
 * i32 accumulator (amd_triton_npu/backend/matmul_transform.py:62-64). */
XB_API int xb_matmul_i16_workspace_size(int64_t M, int64_t N, int64_t K,
                                        size_t* bytes, char* err,
                                        size_t errlen);

/* C[M,N] (int32) = A[M,K] (int16) @ B[K,N] (int16) with int32 wrap-around
 * (mod 2^32), the semantics of an int32 accumulator.  `workspace` (256-byte
 * aligned, >= xb_matmul_i16_workspace_size bytes) receives the int8 limb
 * planes; it must stay untouched until the call's work on `stream` is done. */
XB_API int xb_matmul_i16(const void* A, const void* B, void* C, int64_t M,
                         int64_t N, int64_t K, int64_t lda, int64_t ldb,
                         int64_t ldc, void* workspace, size_t workspace_bytes,
                         void* stream, char* err, size_t errlen);

/* Size of the scratch array built into the library for xb_matmul_i16_noalloc
 * (held on every GPU that loads the library until the process exits). */
#define XB_I16_NOALLOC_SCRATCH_BYTES (32u * 1024u * 1024u)

/* xb_matmul_i16 for callers that cannot allocate device memory: plugins
 * whose host framework owns every device allocation through its own pool
 * (memory taken behind its back breaks its accounting and limits), and
 * latency-bound paths where a cudaMalloc may synchronise the device and
 * stall.  No counterpart in the reference.  The int8 limb planes go to a fixed XB_I16_NOALLOC_SCRATCH_BYTES
 * array inside the library instead of a caller workspace; a product needing
 * more than that (xb_matmul_i16_workspace_size) is rejected with
 * XB_ERR_UNSUPPORTED.  Nothing is allocated.  The first call on a device looks
 * up the array's device address, so make it before any stream capture.  All
 * calls share the array: calls whose GPU work overlaps race. */
XB_API int xb_matmul_i16_noalloc(const void* A, const void* B, void* C,
                                 int64_t M, int64_t N, int64_t K, int64_t lda,
                                 int64_t ldb, int64_t ldc, void* stream,
                                 char* err, size_t errlen);

/* C[M,N] = A[M,K] (bf16) @ B[K,N] (bf16), fp32 accumulation, C in f32 or bf16
 * (out_dtype XB_DT_F32 / XB_DT_BF16).  Replaces `bare_matmul`
 * (examples/matmul_bf16_m64_n64_k64/matmul_bf16_m64_n64_k64.py:16-46,
 * examples/autotune-matmul/matmul.py:22-53). */
XB_API int xb_matmul_bf16(const void* A, const void* B, void* C, int64_t M,
                          int64_t N, int64_t K, int64_t lda, int64_t ldb,
                          int64_t ldc, int out_dtype, void* stream, char* err,
                          size_t errlen);

/* Y[M,N] = X[M,K] (bf16) @ W[N,K]^T (bf16) (+ bias[N], bf16), W in
 * nn.Linear layout, fp32 accumulation, Y in bf16 or f32 (out_dtype); bias
 * may be NULL.  Replaces `triton_linear` (examples/qwen2_5/kernels/matmul.py:
 * 172-296) and the fp32 LM head of examples/qwen2_5/model.py:1097-1106. */
XB_API int xb_linear_bf16(const void* X, const void* W, const void* bias,
                          void* Y, int64_t M, int64_t N, int64_t K,
                          int64_t ldx, int64_t ldw, int64_t ldy, int out_dtype,
                          void* stream, char* err, size_t errlen);

/* Plan for xb_linear_small_bf16: the K-slice count it picks for an
 * M x N x K product and the fp32 workspace it then needs (0 when it writes
 * straight to Y). */
XB_API int xb_linear_small_plan(int64_t M, int64_t N, int64_t K,
                                int has_residual, int* splits,
                                size_t* workspace_bytes, char* err,
                                size_t errlen);

/* Y = [residual +] (X[M,K] @ W[N,K]^T + bias), for few tokens (decode,
 * M <= 64 is the target): the weight rows fill the 128-row MMA dimension and
 * the tokens a 64-wide tile (swap-AB), K is split over `splits` slices (<= 0:
 * automatic) so the weight streams from HBM on every SM, and a fixed-order
 * reduction adds the slices, the bias and the residual (bf16 [M, N], row
 * pitch ldr, may be NULL).  Needs the workspace xb_linear_small_plan
 * reports.  With bf16 output, M <= 64, N % 4 == 0 and 8-byte aligned bf16
 * vectors the whole linear is one launch of the cluster split-K decode
 * kernel (xb_decode_linear_bf16 / xb_decode_linear_residual_bf16; `splits`
 * and the workspace are then unused).  Replaces
 * `triton_linear` + `triton_add` in the decode step
 * (examples/qwen2_5/model.py:1045-1061). */
XB_API int xb_linear_small_bf16(const void* X, const void* W, const void* bias,
                                const void* residual, void* Y, int64_t M,
                                int64_t N, int64_t K, int64_t ldx, int64_t ldw,
                                int64_t ldr, int64_t ldy, int out_dtype,
                                int splits, void* workspace,
                                size_t workspace_bytes, void* stream,
                                char* err, size_t errlen);

/* The decode MLP front half: Y[M, n_out] = silu(X @ Wg^T) * (X @ Wu^T) with
 * W = [Wg; Wu] ([2*n_out, K], gate rows first), one GEMM over the stacked
 * weight (the small-M kernel) and the silu*up in its split-K reduction, with
 * the roundings of the unfused sequence (two bf16 linears, then
 * xb_silu_mul).  Workspace: the xb_linear_small_plan size for N = 2*n_out.
 * Replaces model.py:1049-1059 (gate / up linears + `triton_swiglu`). */
XB_API int xb_linear_small_swiglu_bf16(const void* X, const void* W, void* Y,
                                       int64_t M, int64_t n_out, int64_t K,
                                       int64_t ldx, int64_t ldw, int64_t ldy,
                                       void* workspace, size_t workspace_bytes,
                                       void* stream, char* err, size_t errlen);

/* The fused QKV projection of a prefill (any number of tokens), finished in
 * the GEMM epilogue: qkv = bf16(X @ W^T + bias) with X [batch * seq, K] and
 * W [(H + 2 KVH) * 64, K], then the rotate-half RoPE of the query and key
 * heads at positions pos_offset + s (cos/sin fp32 [>= pos_offset + seq, 64];
 * both NULL: no rotation, learned positions; rope_dup = 1 promises that
 * every table row's second half repeats its first, as rotate-half RoPE
 * tables do, and only the first half is read) -- the roundings of
 * xb_linear_bf16 followed by xb_rope_kv_bf16 -- written straight to q
 * [batch, H, seq, 64] and the K / V caches [batch, KVH, max_seq, 64] (16-byte
 * aligned).  The qkv activations never reach memory.  Replaces
 * examples/qwen2_5/model.py:836-867 (q/k/v projections + rope) and
 * examples/gpt2/model.py:757-775 (c_attn + head split). */
XB_API int xb_linear_rope_kv_bf16(const void* X, const void* W, const void* bias,
                                  const float* cos_t, const float* sin_t,
                                  int rope_dup, void* q_out, void* k_cache,
                                  void* v_cache,
                                  int64_t batch, int64_t seq, int64_t n_head,
                                  int64_t n_kv_head, int64_t head_dim,
                                  int64_t max_seq, int64_t pos_offset,
                                  int64_t K, int64_t ldx, int64_t ldw,
                                  void* stream, char* err, size_t errlen);

/* Y = residual + bf16(X @ W^T + bias) (bf16, any M): the linear with the
 * residual add fused into the GEMM epilogue (o_proj / down_proj of a
 * prefill; examples/qwen2_5/model.py:1045-1046, 1060-1061).  The residual
 * may have any alignment; a 16-byte aligned base and row pitch take the
 * faster whole-line epilogue. */
XB_API int xb_linear_residual_bf16(const void* X, const void* W, const void* bias,
                                   const void* residual, void* Y, int64_t M,
                                   int64_t N, int64_t K, int64_t ldx,
                                   int64_t ldw, int64_t ldr, int64_t ldy,
                                   void* stream, char* err, size_t errlen);

/* Y = bf16(gelu_tanh(bf16(X @ W^T + bias))) (bf16, any M): the linear with
 * the tanh GELU fused (GPT-2 c_fc + gelu, examples/gpt2/model.py:1046-1051),
 * rounded as a linear followed by the GELU kernel.  M <= 64 uses the cluster
 * split-K decode kernel (N % 4 == 0; the workspace, as xb_linear_small_plan
 * reports, only when pointers or pitches rule that kernel out). */
XB_API int xb_linear_gelu_bf16(const void* X, const void* W, const void* bias,
                               void* Y, int64_t M, int64_t N, int64_t K,
                               int64_t ldx, int64_t ldw, int64_t ldy,
                               void* workspace, size_t workspace_bytes,
                               void* stream, char* err, size_t errlen);

/* Y [M, n_out] = bf16(silu(bf16(X Wg^T)) * bf16(X Wu^T)) with W [2 n_out, K]
 * interleaving 64-row blocks of gate and up rows (block 2b = gate rows
 * 64b..64b+63, block 2b+1 = the up rows of the same features); n_out %
 * 64 == 0.  One GEMM whose epilogue applies the SwiGLU (M > 64), or the
 * cluster split-K decode kernel with the SwiGLU in the same launch (M <= 64;
 * the workspace, as xb_linear_small_plan reports for N = 2 n_out, is used
 * only when pointers or pitches rule that kernel out).  The roundings are those of
 * two linears and the silu*up kernel (examples/qwen2_5/model.py:1047-1059,
 * kernels/swiglu.py:94-160). */
XB_API int xb_linear_swiglu_bf16(const void* X, const void* W, void* Y,
                                 int64_t M, int64_t n_out, int64_t K,
                                 int64_t ldx, int64_t ldw, int64_t ldy,
                                 void* workspace, size_t workspace_bytes,
                                 void* stream, char* err, size_t errlen);

/* Decode-step fusions of the small-M linear (one token per sequence, M =
 * batch <= 65535 rows).  Up to 64 rows xb_linear_small_rope_kv_bf16 is ONE
 * launch of the cluster split-K decode kernel (below) and
 * xb_linear_small_residual_norm_bf16 that kernel plus the row-norm kernel;
 * otherwise a split-K GEMM into `workspace` (the bytes xb_linear_small_plan
 * reports for M, N, K) plus one finishing kernel.
 *
 * xb_linear_small_rope_kv_bf16: the fused QKV projection of a decode token
 * finished into attention inputs: qkv = X @ W^T + bias (W [(H + 2 KVH) * D,
 * K]), rounded to bf16, then RoPE of the query and key heads at position
 * pos_offset (cos/sin fp32 tables [>= pos_offset + 1, D]; both NULL: no
 * rotation, for learned positions) written to q [batch, H, 1, D] and the K /
 * V caches [batch, KVH, max_seq, D] at row pos_offset.  Replaces
 * xb_linear_small_bf16 + xb_rope_kv_bf16 on the decode path
 * (examples/qwen2_5/model.py:836-867; examples/gpt2/model.py:757-775).
 *
 * xb_linear_small_residual_norm_bf16: Y = residual + bf16(X @ W^T + bias)
 * (bf16, the residual stream) and Yn = norm(Y) (bf16): norm_kind 0 is
 * RMSNorm (Y * rsqrt(mean(Y^2) + eps) * norm_w), 1 is LayerNorm ((Y - mean) *
 * rsqrt(var + eps) * norm_w + norm_b).  N % 4 == 0, N <= 4096.  Replaces the
 * o_proj / down_proj linear, the residual add and the following norm
 * (examples/qwen2_5/model.py:1045-1061; examples/gpt2/model.py:1032-1059). */
XB_API int xb_linear_small_rope_kv_bf16(const void* X, const void* W,
                                        const void* bias, const float* cos_t,
                                        const float* sin_t, void* q_out,
                                        void* k_cache, void* v_cache,
                                        int64_t batch, int64_t n_head,
                                        int64_t n_kv_head, int64_t head_dim,
                                        int64_t max_seq, int64_t pos_offset,
                                        int64_t K, int64_t ldx, int64_t ldw,
                                        void* workspace, size_t workspace_bytes,
                                        void* stream, char* err, size_t errlen);
XB_API int xb_linear_small_residual_norm_bf16(
    const void* X, const void* W, const void* bias, const void* residual,
    void* Y, void* Yn, const void* norm_w, const void* norm_b, float eps,
    int norm_kind, int64_t M, int64_t N, int64_t K, int64_t ldx, int64_t ldw,
    int64_t ldr, int64_t ldy, int64_t ldn, void* workspace,
    size_t workspace_bytes, void* stream, char* err, size_t errlen);

/* Decode-step linears, one launch each, M <= 64 tokens (one per sequence):
 * the cluster split-K kernel (a cluster of <= 8 CTAs per 128-row block of W
 * [N, K]; the K slices are summed over distributed shared memory in rank
 * order) with the work that follows the linear in the same kernel.
 *
 * Input X [M, K] bf16 (row pitch ldx) is used as is when x_stats is NULL.
 * Otherwise X carries a pending norm, applied as X is loaded:
 *   x_norm_kind 0  xn = bf16(x * rsqrt(mean(x^2) + eps) * x_norm_w)      (RMSNorm)
 *   x_norm_kind 1  xn = bf16((x - mean) * rsqrt(var + eps) * x_norm_w
 *                            + x_norm_b)                                  (LayerNorm)
 * with the row statistics combined from x_stats, the block statistics that
 * xb_decode_linear_residual_bf16 wrote with the same kind when it produced X
 * (K % 8 == 0; x_norm_w / x_norm_b 16-byte aligned).  This is how a residual
 * add, the norm after it and the next linear take two launches (the
 * residual stream and the norm of examples/qwen2_5/model.py:1045-1061 and
 * examples/gpt2/model.py:1032-1059).
 *
 * xb_decode_linear_bf16: Y = bf16(xn W^T + bias), act 1 = tanh GELU on that
 *   value (GPT-2 c_fc + gelu, examples/gpt2/model.py:1046-1051).
 * xb_decode_linear_rope_kv_bf16: the QKV projection finished into attention
 *   inputs, as xb_linear_small_rope_kv_bf16 (head_dim % 8 == 0, dividing 128).
 * xb_decode_linear_swiglu_bf16: Y [M, n_out] = bf16(silu(bf16(xn Wg^T)) *
 *   bf16(xn Wu^T)), W interleaving 64-row blocks of gate and up rows (the
 *   layout of xb_linear_swiglu_bf16), n_out % 64 == 0.
 * xb_decode_linear_residual_bf16: Y = residual + bf16(xn W^T + bias) and,
 *   when stats_out is not NULL, the statistics of each Y row per 128-column
 *   block for the norm that follows: stats_out holds ceil(N / 128) * 64 float
 *   pairs ([block][token]); stats_kind 0 stores (sum of squares, 0), 1 stores
 *   (block mean, sum of squared deviations from it).
 * The statistics are summed in block order, so every result is bit-
 * repeatable.  Pitches are in elements; outputs and bf16 vectors 8-byte
 * aligned with pitches % 4 == 0; N % 4 == 0. */
/* The LM head and the greedy next token in one pass (examples/qwen2_5/
 * model.py:1134-1179 and examples/gpt2/model.py:1144-1206 take the argmax of
 * the last position's logits): idx[m] = argmax_n (X W^T)[m, n] (int64, first
 * index of the maximum, NaN largest, as torch.argmax) with X [M, K] and
 * W [N, K] bf16, fp32 accumulation -- the same values a fp32-output linear
 * writes, but the logits never leave the chip: each 128-row tile of W keeps
 * its best row per token ({float, int32} per (tile, token) in `workspace`,
 * xb_linear_argmax_workspace_size bytes) and a second kernel reduces the
 * tiles. */
XB_API int xb_linear_argmax_workspace_size(int64_t M, int64_t N, size_t* bytes,
                                           char* err, size_t errlen);
XB_API int xb_linear_argmax_bf16(const void* X, const void* W, int64_t M,
                                 int64_t N, int64_t K, int64_t ldx, int64_t ldw,
                                 int64_t* idx, void* workspace,
                                 size_t workspace_bytes, void* stream,
                                 char* err, size_t errlen);

XB_API int xb_decode_linear_bf16(const void* X, int64_t M, int64_t ldx,
                                 const float* x_stats, const void* x_norm_w,
                                 const void* x_norm_b, float x_eps,
                                 int x_norm_kind, const void* W,
                                 const void* bias, void* Y, int64_t N,
                                 int64_t K, int64_t ldw, int64_t ldy, int act,
                                 void* stream, char* err, size_t errlen);
XB_API int xb_decode_linear_rope_kv_bf16(
    const void* X, int64_t M, int64_t ldx, const float* x_stats,
    const void* x_norm_w, const void* x_norm_b, float x_eps, int x_norm_kind,
    const void* W, const void* bias, const float* cos_t, const float* sin_t,
    void* q_out, void* k_cache, void* v_cache, int64_t n_head,
    int64_t n_kv_head, int64_t head_dim, int64_t max_seq, int64_t pos_offset,
    int64_t K, int64_t ldw, void* stream, char* err, size_t errlen);
XB_API int xb_decode_linear_swiglu_bf16(const void* X, int64_t M, int64_t ldx,
                                        const float* x_stats,
                                        const void* x_norm_w,
                                        const void* x_norm_b, float x_eps,
                                        int x_norm_kind, const void* W, void* Y,
                                        int64_t n_out, int64_t K, int64_t ldw,
                                        int64_t ldy, void* stream, char* err,
                                        size_t errlen);
XB_API int xb_decode_linear_residual_bf16(
    const void* X, int64_t M, int64_t ldx, const float* x_stats,
    const void* x_norm_w, const void* x_norm_b, float x_eps, int x_norm_kind,
    const void* W, const void* bias, const void* residual, void* Y,
    float* stats_out, int stats_kind, int64_t N, int64_t K, int64_t ldw,
    int64_t ldr, int64_t ldy, void* stream, char* err, size_t errlen);

/* A chain of decode-step linears in ONE persistent launch: up to four
 * phases, each one of the four linears above (kind XB_DECODE_*), where a
 * phase may read what an earlier phase of the chain wrote (its X, the
 * statistics of a pending norm, a residual).  The decoder layer's o_proj +
 * residual, gate/up + SwiGLU, down_proj + residual and the next layer's QKV +
 * RoPE + KV write are one call instead of four launches
 * (examples/qwen2_5/model.py:1045-1061 and 836-867, per decode step).
 *
 * The grid is persistent: clusters of 8 CTAs split K (eight slices of
 * ceil(K / 512) 64-wide blocks, summed over distributed shared memory in rank
 * order) and take the 128-row blocks of each phase in turn; the phases are
 * separated by grid-wide barriers on the counters in `sync`, and the weights
 * of every phase stream in from the start of the launch.  The roundings are
 * those of the single-launch entry points; only the K split can differ from
 * theirs (they pick it per shape), which changes the fp32 sums in their last
 * bits.
 *
 * Field meanings follow the single-launch entry points; n is the number of W
 * rows for every kind (XB_DECODE_SWIGLU: 2 n_out, interleaved 64-row blocks;
 * XB_DECODE_ROPE_KV: (n_head + 2 n_kv_head) * head_dim).  Limits: M <= 64,
 * K <= 5120.  `sync`: 16 bytes of device memory, zeroed once before the first
 * call; every launch leaves it zero when it ends, also after a timeout.  One
 * sync buffer serves one stream at a time.  Returns XB_ERR_UNSUPPORTED when a
 * phase is outside the limits or no 8-CTA cluster fits on the device. */
#define XB_DECODE_STORE 0
#define XB_DECODE_ROPE_KV 1
#define XB_DECODE_SWIGLU 2
#define XB_DECODE_RESIDUAL 3
typedef struct xb_decode_phase {
  int32_t kind;             /* XB_DECODE_* */
  int32_t act;              /* XB_DECODE_STORE: 1 = tanh GELU */
  const void* x;            /* X [m, k] bf16 */
  int64_t m, ldx;
  const float* x_stats;     /* pending norm of X, or NULL */
  const void* x_norm_w;
  const void* x_norm_b;
  float x_eps;
  int32_t x_norm_kind;
  const void* w;            /* W [n, k] bf16 */
  int64_t n, k, ldw;
  const void* bias;         /* STORE / ROPE_KV / RESIDUAL, or NULL */
  void* y;                  /* STORE / SWIGLU / RESIDUAL output */
  int64_t ldy;
  const void* residual;     /* RESIDUAL */
  int64_t ldr;
  float* stats_out;         /* RESIDUAL: statistics of Y for the next norm, or NULL */
  int32_t stats_kind;
  int32_t reserved;
  const float* cos_t;       /* ROPE_KV: RoPE tables, or NULL */
  const float* sin_t;
  void* q_out;
  void* k_cache;
  void* v_cache;
  int64_t n_head, n_kv_head, head_dim, max_seq, pos_offset;
} xb_decode_phase;
XB_API int xb_decode_chain_bf16(const xb_decode_phase* phases, int n_phases,
                                void* sync, void* stream, char* err,
                                size_t errlen);

/* ---------------------------------------------------------------------------
 * N-sharded GEMM across the GPUs of one node (one process per GPU).  The
 * reference runs on one device; this is the multi-GPU form of its GEMM
 * (examples/matmul_*), with the all-gather of C fused into the epilogue.
 * ------------------------------------------------------------------------- */

/* cudaMalloc `bytes` (zeroed) and export a 64-byte CUDA IPC handle for it. */
XB_API int xb_peer_alloc(size_t bytes, void** ptr, void* ipc_handle,
                         char* err, size_t errlen);
/* Map a peer's allocation from its IPC handle (NVLink peer access). */
XB_API int xb_peer_open(const void* ipc_handle, void** ptr, char* err,
                        size_t errlen);
XB_API int xb_peer_close(void* ptr, char* err, size_t errlen);
XB_API int xb_peer_free(void* ptr, char* err, size_t errlen);

/* This rank computes C[:, rank*N_shard : (rank+1)*N_shard] = A[M,K] @
 * B_shard[K,N_shard] (int8 -> int32, or bf16 -> bf16 with fp32
 * accumulation) and stores every output tile into the C of EVERY rank
 * (C_ranks[r]: rank r's C [M, ldc] as mapped in this process) with plain
 * stores over NVLink.  Signal buffers (signal_ranks[r]: rank r's uint64
 * [2 * world + 1], zero-initialised peer memory, one per C) hold in slot p
 * the calls whose block from rank p has landed, in slot `world` a CTA
 * counter, in slot world + 1 + p the calls rank p has started.
 *
 * `epoch` is the 1-based number of this call on these buffers (every rank
 * passes the same value).  At its start the kernel adds 1 to slot
 * world + 1 + rank of every peer (this rank's C may be overwritten: every
 * earlier kernel on `stream`, including readers of the previous C, has
 * completed); before its first store into peer p's C it waits, for at most
 * timeout_ns, until p has done the same for this epoch.  So back-to-back
 * calls never overwrite a C that a peer still reads on its stream.  When its
 * grid is done it adds 1 to slot `rank` of every peer; wait for the peers with
 * xb_peer_wait.  A wait that runs out records XB_ERR_TIMEOUT
 * (xb_device_status), skips every store and withholds the completion
 * signal, so the peers' xb_peer_wait times out too; the buffers must then be
 * re-created.  world <= 8. */
XB_API int xb_matmul_sharded(const void* A, const void* B_shard,
                             void* const* C_ranks, void* const* signal_ranks,
                             int world, int rank, int64_t M, int64_t N_shard,
                             int64_t K, int64_t lda, int64_t ldb, int64_t ldc,
                             uint64_t epoch, uint64_t timeout_ns, int dtype,
                             void* stream, char* err, size_t errlen);

/* Enqueue a wait until every other rank's slot in this rank's signal buffer
 * reaches `epoch` (the number of sharded GEMMs issued so far); gives up
 * after timeout_ns and records XB_ERR_TIMEOUT (read with xb_peer_status). */
XB_API int xb_peer_wait(const uint64_t* signal, int world, int rank,
                        uint64_t epoch, uint64_t timeout_ns, void* stream,
                        char* err, size_t errlen);

/* Read (synchronising `stream`) and clear the peer-wait status word. */
XB_API int xb_peer_status(void* stream, int* status, char* err,
                          size_t errlen);

/* ---------------------------------------------------------------------------
 * Qwen2.5 decoder pieces (examples/qwen2_5/model.py:824-1179).
 * ------------------------------------------------------------------------- */

/* out[m, :] = table[ids[m], :] (bf16 rows of `dim`, dim % 8 == 0).  Ids
 * outside [0, vocab) produce zero rows and set the flag xb_token_status
 * reports.  Replaces model.py:911 (`self.embed_tokens[input_ids]`). */
XB_API int xb_embedding_bf16(const void* table, const int64_t* ids, void* out,
                             int64_t rows, int64_t dim, int64_t vocab,
                             void* stream, char* err, size_t errlen);

/* *status = 1 if an embedding kernel met a token id outside its vocabulary
 * since the previous call (then clears the flag), else 0.  Synchronises
 * `stream`.  The reference raises an IndexError on such ids. */
XB_API int xb_token_status(void* stream, int* status, char* err,
                           size_t errlen);

/* out[m, :] = bf16(table[ids[m], :] + pos_table[pos_offset + m % seq, :]):
 * token plus learned position embeddings of `rows` = batch*seq tokens (rows
 * of `seq` consecutive positions).  Ids outside [0, vocab) produce zero rows
 * and set the flag xb_token_status reports.  Replaces
 * examples/gpt2/model.py:866-876 (`self.wte[input_ids] + self.wpe[positions]`). */
XB_API int xb_embedding_pos_bf16(const void* table, const void* pos_table,
                                 const int64_t* ids, void* out, int64_t rows,
                                 int64_t seq, int64_t dim, int64_t vocab,
                                 int64_t n_pos, int64_t pos_offset,
                                 void* stream, char* err, size_t errlen);

/* Rotary embedding of the fused QKV projection plus the KV-cache write.
 * qkv: [batch*seq, (n_head + 2*n_kv_head)*head_dim]; cos/sin: fp32 tables of
 * at least pos_offset+seq rows of head_dim (rope.py:20-35); q_out:
 * [batch, n_head, seq, head_dim]; k_cache / v_cache: [batch, n_kv_head,
 * max_seq, head_dim], rows pos_offset .. pos_offset+seq-1 written.
 * cos_t and sin_t may both be NULL: the query and key heads are then copied
 * unrotated (models with learned positions: the head split, transpose and
 * cache write of examples/gpt2/model.py:757-775).
 * Replaces model.py:851-867 and kernels/rope.py:44-67. */
XB_API int xb_rope_kv_bf16(const void* qkv, const float* cos_t,
                           const float* sin_t, void* q_out, void* k_cache,
                           void* v_cache, int64_t batch, int64_t seq,
                           int64_t n_head, int64_t n_kv_head, int64_t head_dim,
                           int64_t max_seq, int64_t pos_offset, void* stream,
                           char* err, size_t errlen);

/* Causal GQA attention over the KV cache: query row s (position
 * pos_offset+s) attends keys 0 .. pos_offset+s.  q: [batch, n_head, seq,
 * head_dim]; out: [batch, seq, n_head*head_dim]; head_dim 64.  Online
 * softmax in fp32, P rounded to bf16 before P@V.  Replaces
 * `fused_attention_kernel` (examples/qwen2_5/kernels/attention.py:27-122)
 * and the GQA expansion of model.py:868-889 (done natively here). */
XB_API int xb_attention_bf16(const void* q, const void* k_cache,
                             const void* v_cache, void* out, int64_t batch,
                             int64_t seq, int64_t n_head, int64_t n_kv_head,
                             int64_t head_dim, int64_t max_seq,
                             int64_t pos_offset, float scale, void* workspace,
                             size_t workspace_bytes, void* stream, char* err,
                             size_t errlen);

/* Workspace xb_attention_bf16 needs: the per-chunk partial results of
 * single-token (seq == 1) attention, split over 128-key chunks of the
 * context; 0 for seq > 1. */
XB_API int xb_attention_workspace_size(int64_t batch, int64_t seq,
                                       int64_t n_head, int64_t n_kv_head,
                                       int64_t pos_offset, size_t* bytes,
                                       char* err, size_t errlen);

/* idx[r] = first index of the maximum of x[r, 0:cols] (row pitch ld);
 * NaN counts as the maximum.  Replaces `torch.argmax(logits[..., -1, :])`
 * of model.py:1155, 1171. */
XB_API int xb_argmax_f32(const float* x, int64_t rows, int64_t cols,
                         int64_t ld, int64_t* idx, void* stream, char* err,
                         size_t errlen);

/* Read (synchronising `stream`) and clear the device status word that the
 * tensor-core kernels set when a bounded wait runs out: 0 = fine,
 * XB_ERR_TIMEOUT = a kernel gave up and returned early (its output is not
 * valid).  Mirrors the reference runtime's watchdog
 * (amd_triton_npu/backend/include/HsaRuntime/HsaRuntime.h:57-67). */
XB_API int xb_device_status(void* stream, int* status, char* err,
                            size_t errlen);

/* Number of kernels this library has launched since it was loaded (launch
 * calls made on the host, including those recorded into a CUDA graph during
 * stream capture; graph replays are not counted).  No reference counterpart:
 * the benchmark uses it to report how many of its own kernels a step runs. */
XB_API int xb_launch_count(uint64_t* count, char* err, size_t errlen);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* XB200_H */
