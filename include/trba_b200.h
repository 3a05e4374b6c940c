/*
 * trba_b200.h — entry points of libtrba_b200.so that have no counterpart in
 * the reference's ABI: diagnostics of the tensor-core kernels.  (The fused
 * training-step API lives in trba_qat.h.)
 */
#ifndef TRBA_B200_H
#define TRBA_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* launch_gemm_int8 routed through the CUDA-core (dp4a) kernel that serves
 * operands a tensor map cannot describe (base not 16-byte aligned). */
void trba_gemm_int8_simt(const int8_t *a, const int8_t *b, int32_t *c, int m, int n, int k,
                         void *stream);

/* Device error word of the tensor-core kernels: 1 when a bounded mbarrier
 * wait gave up.  Synchronises the device; clears the word if clear != 0. */
int trba_tc_error_poll(int clear);

#ifdef __cplusplus
}
#endif
#endif
