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
// binary16 pair holding decode(b)/256, b0 in the low half: a byte permute, a
// shift and one three-input logic op.  (The hardware conversion
// cvt.rn.f16x2.e4m3x2 turns both 0x7F and 0xFF into the same positive NaN, so
// giving them the reference decoder's +-480 needs a min and the code's sign
// put back: four instructions per pair instead of three.)
__device__ __forceinline__ uint32_t fp8x2_to_f16x2_scaled(uint32_t w, int sel) {
    // place b0 in bits 8..15 and b1 in bits 24..31
    uint32_t x = __byte_perm(w, 0u, sel ? 0x3424u : 0x1404u);
    return ((x >> 1) & 0x3F803F80u) | (x & 0x80008000u);
}

// The same expansion without a byte permute where the codes already sit in
// bytes 1 and 3: codes b1,b3 of w -> pair (b1 low, b3 high), a shift and a
// three-input logic op.  Bytes 0 and 2 do not reach the result.
__device__ __forceinline__ uint32_t fp8_pair_odd(uint32_t w) {
    return ((w >> 1) & 0x3F803F80u) | (w & 0x80008000u);
}

// Codes b0,b2 of w -> pair (b0 low, b2 high).
__device__ __forceinline__ uint32_t fp8_pair_even(uint32_t w) {
    return ((w << 7) & 0x3F803F80u) | ((w << 8) & 0x80008000u);
}

// Byte j of wa (low half) and byte j of wb (high half): one permute that puts
// them in bytes 1 and 3, then fp8_pair_odd.
__device__ __forceinline__ uint32_t fp8_pair_cross(uint32_t wa, uint32_t wb, int j) {
    return fp8_pair_odd(__byte_perm(wa, wb, (uint32_t)(((4 + j) << 12) | (j << 4))));
}

}  // namespace vw
