// f32 GEMM with bf16 emulation: the f32 operands are rounded to bf16 (round
// to nearest even, as the reference's bf16-emulation lowering and its numpy
// golden do) by a conversion pass, then multiplied on the tensor cores with
// fp32 accumulation by the bf16 GEMM.
//
// Reference: examples/matmul_f32_m64_n32_k16_padded_atransposed/
// matmul_f32_m64_n32_k16_padded_atransposed.py:53-186 (`padded_matmul_kernel`:
// A stored K x M, i.e. transposed, B K x N, C M x N f32; M and N not multiples
// of the tile; golden = bf16(A)^T bf16(B) with f32 accumulation, L140-161).
//
// The conversion writes A' [M, Kp] (K-major, transposed through 32 x 32
// shared-memory tiles when A is stored K x M) and B' [K, Np] (MN-major), with
// Kp, Np rounded up to 8 elements so every row is whole 16-byte TMA boxes;
// the padding columns are zero.
#include "common.cuh"

namespace xb {
namespace cvt {

typedef __nv_bfloat16 bf16;

// dst[r, c] = bf16(src[r, c]) for c < cols, 0 for cols <= c < ldd.
__global__ void __launch_bounds__(256) cvt_rows_kernel(const float* __restrict__ src, int64_t rows, int64_t cols,
                                                       int64_t lds, bf16* __restrict__ dst, int64_t ldd) {
  pdl_wait();
  pdl_trigger();
  const int64_t c = (int64_t)blockIdx.x * 256 + threadIdx.x;
  if (c >= ldd) return;
  for (int64_t r = blockIdx.y; r < rows; r += gridDim.y)
    dst[r * ldd + c] = __float2bfloat16_rn(c < cols ? src[r * lds + c] : 0.0f);
}

// dst[m, k] = bf16(src[k, m]) (src [K, M] with pitch lds), 0 for K <= k < ldd.
__global__ void __launch_bounds__(256) cvt_transpose_kernel(const float* __restrict__ src, int64_t K, int64_t M,
                                                            int64_t lds, bf16* __restrict__ dst, int64_t ldd) {
  pdl_wait();
  pdl_trigger();
  __shared__ float tile[32][33];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8 threads
  const int64_t m0 = (int64_t)blockIdx.x * 32, k0 = (int64_t)blockIdx.y * 32;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t k = k0 + ty + 8 * i, m = m0 + tx;
    tile[ty + 8 * i][tx] = (k < K && m < M) ? src[k * lds + m] : 0.0f;
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t m = m0 + ty + 8 * i, k = k0 + tx;
    if (m < M && k < ldd) dst[m * ldd + k] = __float2bfloat16_rn(tile[tx][ty + 8 * i]);
  }
}

int64_t pad8(int64_t v) { return (v + 7) / 8 * 8; }
size_t a_bytes(int64_t M, int64_t K) { return ((size_t)M * (size_t)pad8(K) * 2 + 255) / 256 * 256; }
size_t b_bytes(int64_t N, int64_t K) { return (size_t)K * (size_t)pad8(N) * 2; }

}  // namespace cvt
}  // namespace xb

using namespace xb::cvt;
using xb::check_launch;
using xb::launch_k;
using xb::set_err;

extern "C" int xb_matmul_f32_bf16emu_workspace_size(int64_t M, int64_t N, int64_t K, size_t* bytes, char* err,
                                                    size_t errlen) {
  if (M < 0 || N < 0 || K < 0 || !bytes) {
    set_err(err, errlen, "xb_matmul_f32_bf16emu_workspace_size: bad arguments");
    return XB_ERR_INVALID;
  }
  *bytes = a_bytes(M, K) + b_bytes(N, K);
  return XB_OK;
}

extern "C" int xb_matmul_f32_bf16emu(const float* A, const float* B, float* C, int64_t M, int64_t N, int64_t K,
                                     int64_t lda, int64_t ldb, int64_t ldc, int a_layout, void* workspace,
                                     size_t workspace_bytes, void* stream, char* err, size_t errlen) {
  const char* what = "xb_matmul_f32_bf16emu";
  cudaStream_t s = (cudaStream_t)stream;
  if (M < 0 || N < 0 || K < 0 || (a_layout != 0 && a_layout != 1)) {
    set_err(err, errlen, "%s: bad shape or A layout (0 = [M, K], 1 = [K, M])", what);
    return XB_ERR_INVALID;
  }
  if (M == 0 || N == 0) return XB_OK;
  if (lda < (a_layout ? M : K) || ldb < N || ldc < N) {
    set_err(err, errlen, "%s: leading dimension shorter than the row", what);
    return XB_ERR_INVALID;
  }
  if (!A || !B || !C) {
    set_err(err, errlen, "%s: null pointer", what);
    return XB_ERR_INVALID;
  }
  if (K == 0) {
    cudaError_t e = cudaMemset2DAsync(C, ldc * 4, 0, N * 4, M, s);
    if (e != cudaSuccess) {
      set_err(err, errlen, "%s: %s", what, cudaGetErrorString(e));
      return XB_ERR_CUDA;
    }
    return XB_OK;
  }
  const size_t need = a_bytes(M, K) + b_bytes(N, K);
  if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255) != 0) {
    set_err(err, errlen, "%s: 256-byte aligned workspace of %zu bytes needed (%zu given)", what, need,
            workspace_bytes);
    return XB_ERR_INVALID;
  }
  const int64_t Kp = pad8(K), Np = pad8(N);
  bf16* a2 = static_cast<bf16*>(workspace);
  bf16* b2 = reinterpret_cast<bf16*>(static_cast<uint8_t*>(workspace) + a_bytes(M, K));
  if (a_layout == 1) {
    const dim3 grid((unsigned)((M + 31) / 32), (unsigned)((Kp + 31) / 32));
    if (grid.y > 65535) {
      set_err(err, errlen, "%s: K too large for the transpose grid", what);
      return XB_ERR_UNSUPPORTED;
    }
    launch_k(cvt_transpose_kernel, grid, 256, 0, s, A, K, M, lda, a2, Kp);
  } else {
    launch_k(cvt_rows_kernel, dim3((unsigned)((Kp + 255) / 256), (unsigned)(M < 65535 ? M : 65535)), 256, 0, s, A,
             M, K, lda, a2, Kp);
  }
  launch_k(cvt_rows_kernel, dim3((unsigned)((Np + 255) / 256), (unsigned)(K < 65535 ? K : 65535)), 256, 0, s, B, K,
           N, ldb, b2, Np);
  int rc = check_launch(what, err, errlen);
  if (rc) return rc;
  return xb_matmul_bf16(a2, b2, C, M, N, K, Kp, Np, ldc, XB_DT_F32, stream, err, errlen);
}
