// Q8_0 block arithmetic (quant.rs:856-874), shared by the kernels and by the
// exhaustive check in tests/cuda/q8_math_check.cu.  Compiled with -fmad=false;
// the fused multiply-adds below are explicit.
#pragma once
#include <cstdint>

namespace krt {

// d = amax / 127, correctly rounded, for amax >= +0 (a fold of fmaxf from
// +0.0, so never -0 or NaN).  The product with the rounded reciprocal c of 127
// is corrected once by its exact residual r = amax - 127 q0 (computed exactly
// by the fused multiply-add): q1 = q0 + r c (P. Markstein, "Computation of
// elementary functions on the IBM RISC System/6000 processor", IBM J. Res.
// Dev. 34(1), 1990).  +inf passes through.  Checked against the correctly
// rounded division for every non-negative f32.
__device__ __forceinline__ float q8_scale(float amax) {
    const float c = 1.0f / 127.0f;
    const float q0 = __fmul_rn(amax, c);
    const float r = __fmaf_rn(-q0, 127.0f, amax);
    const float q1 = __fmaf_rn(r, c, q0);
    return amax < __int_as_float(0x7f800000) ? q1 : amax;
}

// 1 / d, correctly rounded, for d > 0: the hardware reciprocal approximation
// y0 refined by one Newton-Raphson step y1 = y0 + y0 (1 - d y0) with fused
// multiply-adds (Markstein 1990, as above).  Quotients that overflow
// (d <= 2^-128) or fall into the subnormals (d > 2^126, or +inf) take the
// correctly rounded division; d = amax / 127 never exceeds 2^122 for finite
// amax.  Checked against the correctly rounded division for every positive
// f32.
__device__ __forceinline__ float q8_inv(float d) {
    if (d <= 0x1p-128f || d > 0x1p126f) return __fdiv_rn(1.0f, d);
    float y0;
    asm("rcp.approx.f32 %0, %1;" : "=f"(y0) : "f"(d));
    const float e = __fmaf_rn(-d, y0, 1.0f);
    return __fmaf_rn(e, y0, y0);
}

// quant.rs:871: (v * inv).round().clamp(-127, 127) as i8 -- round half away
// from zero, NaN -> 0.  Half away from zero is sign(v) floor(|v| + 1/2); the
// sum |v| + 1/2 rounded toward zero has the same floor as the exact sum
// (integers below 2^24 are floats, so rounding down never crosses one, and
// above 2^23 the sum is |v| itself), and the conversion's truncation takes
// that floor.  The conversion saturates and maps NaN to 0, so the clamp can
// run on the integer.  Checked against roundf for every f32.
__device__ __forceinline__ int q8_round(float v) {
    const float half = __int_as_float((__float_as_int(v) & (int)0x80000000u) | 0x3f000000);  // copysign(1/2, v)
    return __float2int_rz(__fadd_rz(v, half));
}

__device__ __forceinline__ int8_t q8_code(float v) { return (int8_t)max(-127, min(127, q8_round(v))); }

// When the clamp can be left out.  For a block with amax > 0, d = q8_scale(amax)
// and inv = q8_inv(d), every |v| <= amax gives |v * inv| < 127.5, so
// q8_round(v * inv) is already in [-127, 127], unless d <= 2^-128: then 1/d
// overflows to +inf and the products are +-inf (or NaN).  Proof: d is amax/127
// with relative error below 2^-22 (2^-24 when normal; d > 2^-128 bounds the
// subnormal case), inv is 1/d within 2^-24, so amax * inv <= 127 (1 + 2^-21)
// and the rounded product stays below 127.5.  amax = +inf gives inv = 0.
__device__ __forceinline__ bool q8_needs_clamp(float d) { return d > 0.0f && d <= 0x1p-128f; }

// The reference's `if d > 0 { 1 / d } else { 0 }` (quant.rs:866) for a block
// scale d = q8_scale(amax), without branches: q8_inv's Newton step where it
// applies; 1/d overflows to +inf for 0 < d <= 2^-128; d = +inf gives 0.  A
// finite amax gives d < 2^121, so q8_inv's other division case (d > 2^126)
// is only d = +inf here.
__device__ __forceinline__ float q8_inv_block(float d) {
    float y0;
    asm("rcp.approx.f32 %0, %1;" : "=f"(y0) : "f"(d));
    const float e = __fmaf_rn(-d, y0, 1.0f);
    const float y1 = __fmaf_rn(e, y0, y0);
    return d > 0x1p-128f ? (d <= 0x1p126f ? y1 : 0.0f) : (d > 0.0f ? __int_as_float(0x7f800000) : 0.0f);
}

}  // namespace krt
