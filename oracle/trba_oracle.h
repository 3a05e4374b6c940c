/*
 * TEST INFRASTRUCTURE ONLY — the CPU oracle of the TRBA INT8-QAT hot path.
 *
 * A plain-C restatement of the reference's native backend (the C-ABI that
 * trba-rust's src/backend.rs binds), written from the reference's behaviour,
 * not copied.  Every entry point keeps the reference's exact name and
 * signature (`void *stream` last, ignored here, "device" pointers are host
 * pointers), so the host-step oracle (oracle/step_oracle.py) can drive either
 * this library or the reference's own CPU backend built into oracle/_ref/.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load
 * this library, and only as the checker.  The product (trba-rust_b200/) never
 * links it and has no CPU fallback.
 *
 * Pinning: tests/test_oracle_golden.py checks every function here against
 * (a) the golden vectors of the reference's own unit tests (src/tests.rs,
 * reproduced from its det() generator) and (b) the reference's CPU backend
 * compiled from its sources into oracle/_ref/, on the same seeded inputs.
 */
#ifndef TRBA_ORACLE_H
#define TRBA_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* det(i, seed) of the reference's tests (src/tests.rs:39-43). */
float orc_det(unsigned long long i, unsigned long long seed);
void orc_det_fill(float *out, long long n, unsigned long long seed, float mul);
void orc_det_fill_i8(int8_t *out, long long n, unsigned long long seed, float mul);

#ifdef __cplusplus
}
#endif
#endif
