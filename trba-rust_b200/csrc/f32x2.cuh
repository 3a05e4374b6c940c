// Packed f32x2 arithmetic (sm_100a) with IEEE round-to-nearest results that
// equal the scalar multiply and add, operation by operation.
//
// mul.rn.f32x2 followed by add.rn.f32x2 is contracted into one fused
// multiply-add by the code generator, which rounds once instead of twice.
// The product is therefore written as fma.rn.f32x2(a, b, z) with z = -0.0
// supplied at run time (a kernel argument): a*b + -0 is the correctly
// rounded product for every a, b (including signed zeros, infinities and
// NaN), and the generator cannot fold an addend it does not know.
#pragma once

namespace trba {

struct F2 {
    float x, y;
};

__device__ __forceinline__ F2 prod2_rn(F2 a, F2 b, float neg_zero) {
    F2 r;
    asm("{\n\t.reg .b64 a, b, z, d;\n\t"
        "mov.b64 a, {%2, %3};\n\tmov.b64 b, {%4, %5};\n\tmov.b64 z, {%6, %6};\n\t"
        "fma.rn.f32x2 d, a, b, z;\n\tmov.b64 {%0, %1}, d;\n\t}"
        : "=f"(r.x), "=f"(r.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(neg_zero));
    return r;
}

__device__ __forceinline__ F2 add2_rn(F2 a, F2 b) {
    F2 r;
    asm("{\n\t.reg .b64 a, b, d;\n\t"
        "mov.b64 a, {%2, %3};\n\tmov.b64 b, {%4, %5};\n\t"
        "add.rn.f32x2 d, a, b;\n\tmov.b64 {%0, %1}, d;\n\t}"
        : "=f"(r.x), "=f"(r.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return r;
}

}  // namespace trba
