// Device helpers shared by the Q4_0 x Q8_0 kernels (mat-vec, token-batched mat-vec).
#pragma once

#include "alb_common.cuh"
#include "alb_internal.h"

namespace alb {

static constexpr int GEMV_WARPS = 8;            // consumer warps per CTA
static constexpr int XREC_INTS = 12;            // 48-byte activation record per block

// ------------------------------------------------------------ quantizer
// One warp per 32-value block; lane j owns element j.  amax is an exact max
// (order-free), d = amax/127 and id = 1/d are IEEE divisions, q = RNE(x*id)
// (vcvtnq_s32_f32), d stored as fp16 (arm.cpp:1834-1851).
__device__ __forceinline__ void q8_block_lane(float v, int8_t & q, uint16_t & dh) {
    const float amax = alb_warp_max(fabsf(v));
    const float d = amax / 127.0f;
    const float id = d != 0.0f ? 1.0f / d : 0.0f;
    q = (int8_t)__float2int_rn(__fmul_rn(v, id));
    dh = alb_f2h(d);
}

// ------------------------------------------------------------ GEMV core
// Exact int32 dot of one Q4_0 block (16 nibble bytes, offset 8) with one Q8_0
// block held as 8 packed ints (elements 4k..4k+3 in qs[k]) and its sum.
__device__ __forceinline__ int q4q8_dot(uint4 w, const int4 a_lo, const int4 a_hi, int asum) {
    int s = 0;
    s = __dp4a((int)(w.x & 0x0F0F0F0Fu), a_lo.x, s);
    s = __dp4a((int)(w.y & 0x0F0F0F0Fu), a_lo.y, s);
    s = __dp4a((int)(w.z & 0x0F0F0F0Fu), a_lo.z, s);
    s = __dp4a((int)(w.w & 0x0F0F0F0Fu), a_lo.w, s);
    s = __dp4a((int)((w.x >> 4) & 0x0F0F0F0Fu), a_hi.x, s);
    s = __dp4a((int)((w.y >> 4) & 0x0F0F0F0Fu), a_hi.y, s);
    s = __dp4a((int)((w.z >> 4) & 0x0F0F0F0Fu), a_hi.z, s);
    s = __dp4a((int)((w.w >> 4) & 0x0F0F0F0Fu), a_hi.w, s);
    return s - 8 * asum;
}

// Same dot with fewer integer operations: the high nibbles enter dp4a in place
// (bytes 16*hi, as unsigned) and the sum is divided by 16 once; exact.
__device__ __forceinline__ int q4q8_dot_fast(uint4 w, const int4 a_lo, const int4 a_hi, int asum) {
    int s = 0, t = 0;
    asm("dp4a.u32.s32 %0, %1, %2, %0;" : "+r"(s) : "r"(w.x & 0x0F0F0F0Fu), "r"(a_lo.x));
    asm("dp4a.u32.s32 %0, %1, %2, %0;" : "+r"(s) : "r"(w.y & 0x0F0F0F0Fu), "r"(a_lo.y));
    asm("dp4a.u32.s32 %0, %1, %2, %0;" : "+r"(s) : "r"(w.z & 0x0F0F0F0Fu), "r"(a_lo.z));
    asm("dp4a.u32.s32 %0, %1, %2, %0;" : "+r"(s) : "r"(w.w & 0x0F0F0F0Fu), "r"(a_lo.w));
    asm("dp4a.u32.s32 %0, %1, %2, %0;" : "+r"(t) : "r"(w.x & 0xF0F0F0F0u), "r"(a_hi.x));
    asm("dp4a.u32.s32 %0, %1, %2, %0;" : "+r"(t) : "r"(w.y & 0xF0F0F0F0u), "r"(a_hi.y));
    asm("dp4a.u32.s32 %0, %1, %2, %0;" : "+r"(t) : "r"(w.z & 0xF0F0F0F0u), "r"(a_hi.z));
    asm("dp4a.u32.s32 %0, %1, %2, %0;" : "+r"(t) : "r"(w.w & 0xF0F0F0F0u), "r"(a_hi.w));
    return s + (t >> 4) - 8 * asum;   // t is 16 * (sum of hi * a): exact division
}
// Exact conversions on the integer / fp32 pipes (no conversion instruction: the
// conversion unit is a fraction of the ALU rate and saturates in the mat-vec).
// int32 with |i| < 2^22 -> float: bits(1.5 * 2^23 + i) - 1.5 * 2^23.
__device__ __forceinline__ float alb_i2f_small(int i) {
    return __fsub_rn(__int_as_float(i + 0x4B400000), 12582912.0f);
}
// fp16 bits -> float for every finite half: exponent and mantissa placed in a
// float (value * 2^-112, a float denormal for a half subnormal), times 2^112.
__device__ __forceinline__ float alb_h2f_bits(uint32_t h) {
    return __fmul_rn(__int_as_float((int)(((h & 0x7FFFu) << 13) | ((h & 0x8000u) << 16))), 0x1p112f);
}

// f32(a) * f32(b) of two fp16 bit patterns, exactly (11 x 11 significand bits
// fit a float, subnormals included): one mixed-precision fma (sm_100) whose -0
// addend leaves the product, and its sign of zero, unchanged.
__device__ __forceinline__ float alb_mul_f16_exact(unsigned short a, unsigned short b) {
    float r;
    asm("fma.rn.f32.f16 %0, %1, %2, %3;" : "=f"(r) : "h"(a), "h"(b), "f"(-0.0f));
    return r;
}

// fma(f32(a), f32(b), c) with one rounding, a and b given as fp16 bits: the
// mixed-precision fma of sm_100 (the fp16 product is exact in fp32, so this is
// the fp32 fma of the converted values, without the conversions).
__device__ __forceinline__ float alb_fma_f16_f32(unsigned short a, unsigned short b, float c) {
    float r;
    asm("fma.rn.f32.f16 %0, %1, %2, %3;" : "=f"(r) : "h"(a), "h"(b), "f"(c));
    return r;
}

// fp16 bits -> the bits of (value * 2^-1008) as a double (see alb_h2d), without
// the final scaling; pairs with an operand pre-scaled by 2^1008.
__device__ __forceinline__ double alb_h2d_bits(uint32_t h) {
    return __hiloint2double((int)(((h & 0x7FFFu) << 10) | ((h & 0x8000u) << 16)), 0);
}

// Exact conversions onto the fp64 pipe (no conversion instruction).
// fp16 bits -> double for every finite half: the half's exponent and mantissa
// bits placed at the top of a double's (value * 2^-1008, a subnormal double
// for a subnormal half), then scaled by 2^1008.
__device__ __forceinline__ double alb_h2d(uint32_t h) {
    const uint32_t hi = ((h & 0x7FFFu) << 10) | ((h & 0x8000u) << 16);
    return __hiloint2double((int)hi, 0) * 0x1p1008;
}
// int32 -> double: (2^52 + (i + 2^31)) - (2^52 + 2^31), all exact.
__device__ __forceinline__ double alb_i2d(int i) {
    return __hiloint2double(0x43300000, i ^ (int)0x80000000) - 4503601774854144.0;
}

// Writes the Q8_0 record of block b from one warp's 32 lane values.
__device__ __forceinline__ void store_xrec(int * xs, int b, int lane, int8_t q, uint16_t dh) {
    const int qi = (int)(uint8_t)q;
    const int b1 = __shfl_down_sync(0xffffffffu, qi, 1);
    const int b2 = __shfl_down_sync(0xffffffffu, qi, 2);
    const int b3 = __shfl_down_sync(0xffffffffu, qi, 3);
    int s = (int)q;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    int * rec = xs + b * XREC_INTS;
    if ((lane & 3) == 0) rec[lane >> 2] = qi | (b1 << 8) | (b2 << 16) | (b3 << 24);
    if (lane == 0) {
        rec[8] = __float_as_int(alb_h2f(dh));
        rec[9] = s;
    }
}


}  // namespace alb
