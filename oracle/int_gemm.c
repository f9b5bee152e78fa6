/*
 * ORACLE (test infrastructure, not product code): plain-C restatement of the
 * integer GEMMs C[M,N] = A[M,K] @ B[K,N] with int32 accumulation.
 *
 * Follows examples/matmul_i8_m128_n64_k64/matmul_i8_m128_n64_k64.py:63
 * (torch.matmul(a.to(int32), b.to(int32))): every product and partial sum is
 * taken modulo 2^32, which is what an int32 accumulator does and what torch's
 * CPU int32 matmul does.  The same routine covers int16 inputs (the
 * reference's accumulator for i8/i16 is i32,
 * amd_triton_npu/backend/matmul_transform.py:62-64).
 *
 * Row-major operands with leading dimensions lda/ldb/ldc in elements.
 * Optional OpenMP over rows.
 */
#include <stdint.h>

void oracle_gemm_i8_i32(const int8_t* A, const int8_t* B, int32_t* C, int64_t M, int64_t N, int64_t K,
                        int64_t lda, int64_t ldb, int64_t ldc) {
#pragma omp parallel for schedule(static)
  for (int64_t m = 0; m < M; ++m) {
    uint32_t* crow = (uint32_t*)(C + m * ldc);
    for (int64_t n = 0; n < N; ++n) crow[n] = 0u;
    for (int64_t k = 0; k < K; ++k) {
      const uint32_t a = (uint32_t)(int32_t)A[m * lda + k];
      const int8_t* brow = B + k * ldb;
      for (int64_t n = 0; n < N; ++n) crow[n] += a * (uint32_t)(int32_t)brow[n];
    }
  }
}

void oracle_gemm_i16_i32(const int16_t* A, const int16_t* B, int32_t* C, int64_t M, int64_t N, int64_t K,
                         int64_t lda, int64_t ldb, int64_t ldc) {
#pragma omp parallel for schedule(static)
  for (int64_t m = 0; m < M; ++m) {
    uint32_t* crow = (uint32_t*)(C + m * ldc);
    for (int64_t n = 0; n < N; ++n) crow[n] = 0u;
    for (int64_t k = 0; k < K; ++k) {
      const uint32_t a = (uint32_t)(int32_t)A[m * lda + k];
      const int16_t* brow = B + k * ldb;
      for (int64_t n = 0; n < N; ++n) crow[n] += a * (uint32_t)(int32_t)brow[n];
    }
  }
}
