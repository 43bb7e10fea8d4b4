// b2q_numerics.cuh — fp32 element rules shared by every kernel.
//
// Every helper spells out its rounding steps with __f*_rn intrinsics so that
// nvcc cannot contract or reorder them; the CPU checker performs the same
// operations in the same order, so these results are bit-reproducible there.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_fp16.h>

namespace b2q {

// e^x for |x| <= 80: Cody-Waite reduction x = n ln2 + r (ln2 split into the
// 16-bit head 0x3F317200 and its tail) and the degree-8 Taylor polynomial of
// e^r on |r| <= ln2/2, scaled by 2^n through the exponent field.
__device__ __forceinline__ float own_expf(float x) {
    const float n = rintf(__fmul_rn(x, 1.44269504088896340736f));
    float r = __fmaf_rn(n, -0.693145751953125f, x);
    r = __fmaf_rn(n, -1.42860682030941723212e-6f, r);
    float p = 2.48015873015873015873e-5f;
    p = __fmaf_rn(p, r, 1.98412698412698412698e-4f);
    p = __fmaf_rn(p, r, 1.38888888888888888889e-3f);
    p = __fmaf_rn(p, r, 8.33333333333333333333e-3f);
    p = __fmaf_rn(p, r, 4.16666666666666666667e-2f);
    p = __fmaf_rn(p, r, 1.66666666666666666667e-1f);
    p = __fmaf_rn(p, r, 0.5f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    const int32_t ni = static_cast<int32_t>(n);
    return __fmul_rn(p, __int_as_float((ni + 127) << 23));
}

// GELU, the tanh form of src/cuda/siglip2_megakernel.cu:276-280,
// 0.5*x*(1+tanh(y)) with y = sqrt(2/pi)*x*(1+0.044715*x^2), evaluated as the
// equal x / (1 + e^{-2y}): one exponential (own_expf, argument clamped to
// +-80) and one division, branch-free.  The division a/b (b >= 1) is a
// reciprocal seeded from the bit pattern (0x7EF311C7 - bits(b), the "magic
// constant" method, relative error below 1/8), refined by three
// Newton-Raphson steps y += y*(1 - b*y), and one Markstein correction of the
// quotient q = q0 + y*(a - b*q0), q0 = a*y.  gelu2 does two elements with
// packed f32x2 arithmetic; both perform, per element, exactly the operations
// of the CPU checker's orc_gelu.
__device__ __forceinline__ float2 own_div2(float2 a, float2 b) {
    float2 y = make_float2(__int_as_float(0x7EF311C7 - __float_as_int(b.x)),
                           __int_as_float(0x7EF311C7 - __float_as_int(b.y)));
    const float2 nb = make_float2(-b.x, -b.y);
    const float2 one = make_float2(1.0f, 1.0f);
#pragma unroll
    for (int it = 0; it < 3; ++it) y = __ffma2_rn(y, __ffma2_rn(nb, y, one), y);
    const float2 q0 = __fmul2_rn(a, y);
    return __ffma2_rn(__ffma2_rn(nb, q0, a), y, q0);
}

// Round to nearest even of |t| < 2^22 on the fp32 adder: t + 1.5*2^23 lands
// in [2^23, 2^24), where the ulp is 1, so the addition itself rounds t to an
// integer; subtracting the constant again is exact, and the integer is the
// difference of the bit patterns.  Identical to rintf / __float2int_rn on
// that range, without the conversion pipe.
constexpr float kRintMagic = 12582912.0f;   // 1.5 * 2^23, bits 0x4B400000

// a * b per lane, each product rounded on its own.  The scalar __fmul_rn is
// documented never to be merged into a multiply-add; a packed product that
// feeds a packed add can be (measured: the rounding adders below then saw
// the unrounded product and chose the other integer near .5 ties).
__device__ __forceinline__ float2 fmul2_rounded(float2 a, float2 b) {
    return make_float2(__fmul_rn(a.x, b.x), __fmul_rn(a.y, b.y));
}
__device__ __forceinline__ float2 rint2_adder(float2 t, int32_t& n0, int32_t& n1) {
    const float2 tm = __fadd2_rn(t, make_float2(kRintMagic, kRintMagic));
    n0 = __float_as_int(tm.x) - 0x4B400000;
    n1 = __float_as_int(tm.y) - 0x4B400000;
    return __fadd2_rn(tm, make_float2(-kRintMagic, -kRintMagic));
}

__device__ __forceinline__ float2 gelu2(float2 x) {
    const float2 x2 = __fmul2_rn(x, x);
    const float2 inner = __ffma2_rn(make_float2(0.044715f, 0.044715f), x2, make_float2(1.0f, 1.0f));
    const float c = -1.59576912160573071175978423973752f;   // -2*sqrt(2/pi)
    float2 z = __fmul2_rn(__fmul2_rn(make_float2(c, c), x), inner);
    z.x = fminf(fmaxf(z.x, -80.0f), 80.0f);
    z.y = fminf(fmaxf(z.y, -80.0f), 80.0f);
    // e^z, as own_expf
    const float2 t = fmul2_rounded(z, make_float2(1.44269504088896340736f, 1.44269504088896340736f));
    int32_t n0, n1;   // |t| <= 80 * log2(e)
    const float2 n = rint2_adder(t, n0, n1);
    float2 r = __ffma2_rn(n, make_float2(-0.693145751953125f, -0.693145751953125f), z);
    r = __ffma2_rn(n, make_float2(-1.42860682030941723212e-6f, -1.42860682030941723212e-6f), r);
    const float kc[9] = {2.48015873015873015873e-5f, 1.98412698412698412698e-4f, 1.38888888888888888889e-3f,
                         8.33333333333333333333e-3f, 4.16666666666666666667e-2f, 1.66666666666666666667e-1f,
                         0.5f, 1.0f, 1.0f};
    float2 p = make_float2(kc[0], kc[0]);
#pragma unroll
    for (int i = 1; i < 9; ++i) p = __ffma2_rn(p, r, make_float2(kc[i], kc[i]));
    const float2 sc = make_float2(__int_as_float((n0 + 127) << 23), __int_as_float((n1 + 127) << 23));
    // p * 2^n is exact (a normal number scaled by a power of two), so it does
    // not matter whether the product and the add are fused
    const float2 d = __fadd2_rn(make_float2(1.0f, 1.0f), __fmul2_rn(p, sc));
    return own_div2(x, d);
}

__device__ __forceinline__ float gelu(float x) { return gelu2(make_float2(x, x)).x; }

// q8_1 element rule (src/cuda/siglip2_custom_mmq.cu:63-81): given the block
// absmax a, inv = a == 0 ? 0 : 127/a, q = rint(x*inv) clamped to [-128,127].
__device__ __forceinline__ float q8_inv_scale(float amax) { return amax == 0.0f ? 0.0f : __fdiv_rn(127.0f, amax); }
__device__ __forceinline__ float q8_scale(float amax) { return __fdiv_rn(amax, 127.0f); }
__device__ __forceinline__ int q8_round(float x, float inv) {
    int q = __float2int_rn(__fmul_rn(x, inv));
    return q > 127 ? 127 : (q < -128 ? -128 : q);
}

// The same rule for two values of one block whose absmax is a (inv = 127/a
// rounded): |x| <= a bounds |x * inv| by 127 * (1 + 2^-24), below 127.5, so
// the rounded value already lies in [-127, 127] and the clamp never applies.
// Rounding to nearest even is done on the fp32 adder (t + 1.5 * 2^23 rounds
// t to an integer for |t| < 2^22; subtracting the constant back is exact).
// Returns the integers as floats, identical to q8_round's results.
__device__ __forceinline__ float2 q8_round_adder2(float2 x, float inv) {
    const float2 t = fmul2_rounded(x, make_float2(inv, inv));
    const float2 tm = __fadd2_rn(t, make_float2(kRintMagic, kRintMagic));
    return __fadd2_rn(tm, make_float2(-kRintMagic, -kRintMagic));
}

}  // namespace b2q
