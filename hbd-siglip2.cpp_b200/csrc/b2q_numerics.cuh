// b2q_numerics.cuh — fp32 element rules shared by every kernel.
//
// Every helper spells out its rounding steps with __f*_rn intrinsics so that
// nvcc cannot contract or reorder them; the CPU checker performs the same
// operations in the same order, so these results are bit-reproducible there.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace b2q {

// e^x for |x| <= 80: Cody-Waite reduction x = n ln2 + r (ln2 split into the
// 16-bit head 0x3F317200 and its tail) and the degree-8 Taylor polynomial of
// e^r on |r| <= ln2/2, scaled by 2^n through the exponent field.
__device__ __forceinline__ float own_expf(float x) {
    const float n = rintf(__fmul_rn(x, 1.44269504088896340736f));
    float r = __fmaf_rn(-n, 0.693145751953125f, x);
    r = __fmaf_rn(-n, 1.42860682030941723212e-6f, r);
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

// tanh: Maclaurin series to x^19 for |x| < 0.5625, 1 - 2/(e^{2|x|} + 1)
// up to 9, +-1 beyond (within 2 ulp of the correctly rounded value).
__device__ __forceinline__ float own_tanhf(float x) {
    const float ax = fabsf(x);
    if (ax < 0.5625f) {
        const float x2 = __fmul_rn(x, x);
        float q = -2.39129120018333196640e-04f;
        q = __fmaf_rn(q, x2, 5.90027426369488239288e-04f);
        q = __fmaf_rn(q, x2, -1.45583436824381351471e-03f);
        q = __fmaf_rn(q, x2, 3.59212793409824371338e-03f);
        q = __fmaf_rn(q, x2, -8.86323582381010055542e-03f);
        q = __fmaf_rn(q, x2, 2.18694880604743957520e-02f);
        q = __fmaf_rn(q, x2, -5.39682544767856597900e-02f);
        q = __fmaf_rn(q, x2, 1.33333340287208557129e-01f);
        q = __fmaf_rn(q, x2, -3.33333343267440795898e-01f);
        const float x3 = __fmul_rn(x2, x);
        return __fmaf_rn(q, x3, x);
    }
    float y;
    if (ax < 9.0f) {
        const float e = own_expf(__fmul_rn(2.0f, ax));
        y = __fsub_rn(1.0f, __fdiv_rn(2.0f, __fadd_rn(e, 1.0f)));
    } else {
        y = 1.0f;
    }
    return copysignf(y, x);
}

// GELU, tanh form of src/cuda/siglip2_megakernel.cu:276-280, evaluated left
// to right: 0.5*x*(1+tanh(sqrt(2/pi)*x*(1+0.044715*x*x))).
__device__ __forceinline__ float gelu_tanh(float x) {
    const float x2 = __fmul_rn(x, x);
    const float inner = __fadd_rn(1.0f, __fmul_rn(0.044715f, x2));
    const float arg = __fmul_rn(__fmul_rn(0.79788456080286535587989211986876f, x), inner);
    const float t = own_tanhf(arg);
    return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, t));
}

// q8_1 element rule (src/cuda/siglip2_custom_mmq.cu:63-81): given the block
// absmax a, inv = a == 0 ? 0 : 127/a, q = rint(x*inv) clamped to [-128,127].
__device__ __forceinline__ float q8_inv_scale(float amax) { return amax == 0.0f ? 0.0f : __fdiv_rn(127.0f, amax); }
__device__ __forceinline__ float q8_scale(float amax) { return __fdiv_rn(amax, 127.0f); }
__device__ __forceinline__ int q8_round(float x, float inv) {
    int q = __float2int_rn(__fmul_rn(x, inv));
    return q > 127 ? 127 : (q < -128 ? -128 : q);
}

}  // namespace b2q
