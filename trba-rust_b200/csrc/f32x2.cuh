// Packed f32x2 arithmetic (sm_100a) with IEEE round-to-nearest results that
// equal the scalar multiply and add, operation by operation.
//
// A pair lives in one 64-bit register (f32x2: low half = the element at the
// lower address when the pair is loaded from memory), so accumulators,
// weights loaded as 64-bit words and the packed instructions need no
// register moves between them.
//
// mul.rn.f32x2 followed by add.rn.f32x2 is contracted into one fused
// multiply-add by the code generator, which rounds once instead of twice.
// The product is therefore written as fma.rn.f32x2(a, b, z) with z = (-0, -0)
// built from a value supplied at run time (a kernel argument): a*b + -0 is
// the correctly rounded product for every a, b (including signed zeros,
// infinities and NaN), and the generator cannot fold an addend it does not
// know.
#pragma once

namespace trba {

typedef unsigned long long f32x2;

__device__ __forceinline__ f32x2 pack2(float lo, float hi) {
    f32x2 r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}

__device__ __forceinline__ void unpack2(f32x2 v, float &lo, float &hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}

// Correctly rounded lane-wise product; neg_zero2 = pack2(z, z) with z = -0.0f
// from a run-time value.
__device__ __forceinline__ f32x2 prod2_rn(f32x2 a, f32x2 b, f32x2 neg_zero2) {
    f32x2 r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(neg_zero2));
    return r;
}

__device__ __forceinline__ f32x2 add2_rn(f32x2 a, f32x2 b) {
    f32x2 r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}

}  // namespace trba
