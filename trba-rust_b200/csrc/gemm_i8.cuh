// Host-side entry points of the tcgen05 int8 GEMM (gemm_i8.cu).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace trba {

// 2-D int8 tensor map over rows x k (leading dimension ld bytes), boxes of
// 128 bytes of K by box_rows rows, 128-byte swizzle, zero fill outside.
bool make_tmap_i8(CUtensorMap *m, const void *ptr, int rows, int k, int ld, int box_rows);
int pick_bn(int N);
bool gemm_i8_tc(const int8_t *A, const int8_t *B, int32_t *C, int M, int N, int K, int ld,
                cudaStream_t st);
void gemm_i8_simt(const int8_t *A, const int8_t *B, int32_t *C, int M, int N, int K, int ld,
                  cudaStream_t st);

}  // namespace trba
