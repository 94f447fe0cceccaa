// vw_fp8.cuh -- E4M3 KV codec on the device.
//
// Two encoders, selected per pool:
//  * reference codec (default): a bit-exact port of f32_to_fp8_e4m3 in the
//    reference (kernels/norm/rms_norm.bm:98-113): clamp to +-448, rebias the
//    exponent, TRUNCATE the mantissa, exp<=0 -> 0x00, exp>=15 -> sign|0x7F;
//  * OCP mode: the hardware's round-to-nearest-even saturating conversion.
// Scale per token per head = amax / 448 as one IEEE division (amax 0 -> 1),
// and each element is encoded from x / scale, also an IEEE division.
//
// Decode inside the attention gather never materialises f32: a code byte b
// becomes the binary16 bit pattern ((b & 0x80) << 8) | ((b & 0x7F) << 7),
// whose value is exactly decode(b) / 256 for every code the encoders produce
// (in the reference codec that includes 0x7F -> 480/256; for OCP codes also
// the subnormals).  The factor 256 is folded into the per-token scales.  The
// reference decoder (kernels/gemm/gemm_fp8.bm:110-116) gives different values
// only for codes 0x01..0x07 and 0x80..0x87, which the reference encoder never
// writes (it flushes every |x| < 2^-6 to 0x00).
#pragma once
#include <cstdint>

namespace vw {

__device__ __forceinline__ uint32_t fp8_encode_ref(float x) {
    float c = fminf(fmaxf(x, -448.0f), 448.0f);
    uint32_t bits = __float_as_uint(c);
    uint32_t sign = bits >> 31;
    int exp = (int)((bits >> 23) & 0xFFu) - 127 + 7;
    uint32_t mant = (bits >> 20) & 0x7u;
    if (exp <= 0) return 0u;
    if (exp >= 15) return (sign << 7) | 0x7Fu;
    return (sign << 7) | ((uint32_t)exp << 3) | mant;
}

// Two floats -> two OCP E4M3 codes (lo byte from `lo`).
__device__ __forceinline__ uint32_t fp8_encode_ocp2(float lo, float hi) {
    uint16_t r;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
    return r;
}

// Four consecutive floats -> four codes packed little-endian in a u32.
__device__ __forceinline__ uint32_t fp8_encode4(const float (&v)[4], float scale, bool ocp) {
    float a = __fdiv_rn(v[0], scale), b = __fdiv_rn(v[1], scale);
    float c = __fdiv_rn(v[2], scale), d = __fdiv_rn(v[3], scale);
    if (ocp) return fp8_encode_ocp2(a, b) | (fp8_encode_ocp2(c, d) << 16);
    return fp8_encode_ref(a) | (fp8_encode_ref(b) << 8) | (fp8_encode_ref(c) << 16) |
           (fp8_encode_ref(d) << 24);
}

__device__ __forceinline__ float fp8_row_scale(float amax) {
    return amax == 0.0f ? 1.0f : __fdiv_rn(amax, 448.0f);
}

// Codes b0,b1 (bytes 0,1 of w when sel == 0; bytes 2,3 when sel == 1) ->
// binary16 pair holding decode(b) (unscaled), b0 in the low half, by the
// hardware E4M3 conversion.  It reads 0x7F / 0xFF as NaN, where the
// reference decoder has +-480; min(|x|, 480) with x's sign
// (min.xorsign.abs) maps NaN to +-480 and leaves every finite code, whose
// magnitude is at most 448, as it is.  Exact for every code the encoders write.
__device__ __forceinline__ uint32_t fp8x2_to_f16x2_hw(uint32_t w, int sel) {
    const uint16_t pair = (uint16_t)(sel ? (w >> 16) : (w & 0xFFFFu));
    uint32_t h, r;
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h) : "h"(pair));
    asm("min.xorsign.abs.f16x2 %0, %1, %2;" : "=r"(r) : "r"(h), "r"(0x5F805F80u));
    return r;
}

// Codes b0,b1 (bytes 0,1 of w when sel == 0; bytes 2,3 when sel == 1) ->
// binary16 pair holding decode(b)/256, b0 in the low half.
__device__ __forceinline__ uint32_t fp8x2_to_f16x2_scaled(uint32_t w, int sel) {
    // place b0 in bits 8..15 and b1 in bits 24..31
    uint32_t x = __byte_perm(w, 0u, sel ? 0x3424u : 0x1404u);
    return ((x >> 1) & 0x3F803F80u) | (x & 0x80008000u);
}

}  // namespace vw
