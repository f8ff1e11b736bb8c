// Per-token int8 quantisation helpers shared by the quantiser and the fused
// norm/GELU producers.
//
// q = clamp(rint_half_even(fl(x / s)), -127, 127), fl = IEEE fp32 division.
// Fast path: t = fl(x * r) with r = fl(1 / s).  |t - x/s| <= |x/s| * 2^-22.9
// and |fl(x/s) - x/s| <= 2^-18 for |x/s| <= 128, so |t - fl(x/s)| < 2^-15.
// Whenever t is farther than 2^-14 from the half-integer between its two
// neighbouring integers, rint(t) == rint(fl(x/s)); only inside that window
// (about 1 element in 16k for smooth data; the 8 elements of a group are then
// redone together) the exact division is done.  Everything per element runs
// on the FMA/ALU pipes (no conversion-unit op), two elements per fp32
// instruction.
#pragma once

#include "common.cuh"

namespace h3b {

// Round-half-even of |t| < 2^22 on the FMA pipe: adding 1.5 * 2^23 leaves the
// integer in the low mantissa bits (ties to even by the add's own rounding).
// The low byte of the sum's bit pattern is the two's-complement low byte of
// that integer, because 0x4B400000 has a zero low byte.
constexpr float kRoundMagic = 12582912.0f;  // 1.5 * 2^23
constexpr float kNearHalf = 0.5f - 6.103515625e-05f;  // 0.5 - 2^-14

// Packed fp32 pairs (sm_100 f32x2 arithmetic: one instruction per two lanes'
// worth of IEEE round-to-nearest results, identical to the scalar ops).
__device__ __forceinline__ uint64_t f2(float a, float b) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void f2_split(uint64_t r, float& a, float& b) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t sub2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}

// bf16(gelu_tanh(x)) of two elements: PyTorch's GeluCUDAKernelImpl formula in
// fp32, x^3 as (x*x)*x, inner = kBeta * fma(kKappa, x^3, x), 0.5*x*(1+tanhf(inner)),
// each operation rounded once, on fp32 pairs (f32x2 instructions round each
// lane exactly as the scalar ones).
__device__ __forceinline__ uint32_t gelu2(uint32_t v) {
    constexpr float kBeta = (float)(1.41421356237309504880 * 1.12837916709551257390 * 0.5);
    constexpr float kKappa = (float)0.044715;
    const uint64_t x = f2(bf16_lo(v), bf16_hi(v));
    const uint64_t x3 = mul2(mul2(x, x), x);
    const uint64_t inner = mul2(f2(kBeta, kBeta), fma2(f2(kKappa, kKappa), x3, x));
    float i0, i1;
    f2_split(inner, i0, i1);
    const uint64_t t1 = add2(f2(1.0f, 1.0f), f2(tanhf(i0), tanhf(i1)));
    float y0, y1;
    f2_split(mul2(mul2(f2(0.5f, 0.5f), x), t1), y0, y1);
    return pack_bf16x2(y0, y1);
}

// 8 values -> 8 int8 codes packed into two 32-bit words (s == 0 gives zeros).
// Fast path for all 8: t = x * r, m = t + magic (code in m's low byte),
// d = t - (m - magic).  If any |d| is not below 0.5 - 2^-14 (t near a
// half-integer, or NaN: r = inf for a subnormal scale), the 8 elements are
// redone with the exact division.
__device__ __forceinline__ uint2 quant8(const float (&v)[8], float s, float r) {
    if (s == 0.0f) return make_uint2(0u, 0u);
    const uint64_t rr = f2(r, r), mg = f2(kRoundMagic, kRoundMagic);
    uint32_t c[8];
    bool near = false;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const uint64_t t = mul2(f2(v[2 * e], v[2 * e + 1]), rr);
        const uint64_t m = add2(t, mg);
        const uint64_t d = sub2(t, sub2(m, mg));
        float m0, m1, d0, d1;
        f2_split(m, m0, m1);
        f2_split(d, d0, d1);
        c[2 * e] = __float_as_uint(m0);
        c[2 * e + 1] = __float_as_uint(m1);
        near |= !(fabsf(d0) <= kNearHalf) | !(fabsf(d1) <= kNearHalf);
    }
    if (near) {
        // rare: decide every element of the group with the exact quotient
#pragma unroll
        for (int e = 0; e < 8; ++e) c[e] = __float_as_uint(__fadd_rn(__fdiv_rn(v[e], s), kRoundMagic));
    }
    // |fl(x/s)| <= 127 by construction (|x| <= absmax), so the clamp to
    // [-127, 127] of the reference formula never changes a code
    const uint32_t a = __byte_perm(__byte_perm(c[0], c[1], 0x0040), __byte_perm(c[2], c[3], 0x0040), 0x5410);
    const uint32_t b = __byte_perm(__byte_perm(c[4], c[5], 0x0040), __byte_perm(c[6], c[7], 0x0040), 0x5410);
    return make_uint2(a, b);
}

// absmax of 8 bf16 values held as four bf16x2 words, as bf16 bits: for
// non-negative finite bf16 the bit patterns order like the values, so the
// max of |x| is an unsigned 16-bit max of (bits & 0x7FFF).
__device__ __forceinline__ uint32_t absmax_bits8(uint4 v, uint32_t m) {
    m = __vmaxu2(m, v.x & 0x7FFF7FFFu);
    m = __vmaxu2(m, v.y & 0x7FFF7FFFu);
    m = __vmaxu2(m, v.z & 0x7FFF7FFFu);
    m = __vmaxu2(m, v.w & 0x7FFF7FFFu);
    return m;
}

__device__ __forceinline__ float fold_absmax_bits(uint32_t m) {
    const uint32_t b = max(m & 0xFFFFu, m >> 16);
    return __uint_as_float(b << 16);
}

__device__ __forceinline__ void unpack8(uint4 v, float (&f)[8]) {
    f[0] = bf16_lo(v.x); f[1] = bf16_hi(v.x);
    f[2] = bf16_lo(v.y); f[3] = bf16_hi(v.y);
    f[4] = bf16_lo(v.z); f[5] = bf16_hi(v.z);
    f[6] = bf16_lo(v.w); f[7] = bf16_hi(v.w);
}

// scale = absmax / 127 (IEEE) and its correctly rounded reciprocal
__device__ __forceinline__ void row_scale(float amax, float& s, float& r) {
    s = __fdiv_rn(amax, 127.0f);
    r = s != 0.0f ? __frcp_rn(s) : 0.0f;
}

}  // namespace h3b
