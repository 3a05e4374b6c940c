// Layout helpers of the implicit-GEMM conv forward (conv_implicit.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace trba {

// int8 NCHW [B, C, HW] -> NHWC [B, HW, C]; C a multiple of 16, out 16-byte
// aligned.
void nhwc_from_nchw_i8(const int8_t *in, int8_t *out, int B, int C, int HW, cudaStream_t st);

}  // namespace trba
