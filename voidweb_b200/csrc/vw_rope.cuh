// vw_rope.cuh -- rotary position embedding of one element pair, shared by the
// decode (query tile and the appended K row) and the prefill (query fragments
// and the chunk append), so that every path rotates bit-identically.
#pragma once

namespace vw {

// Rotary position embedding of one pair (x[d], x[d + D/2]) at position pos,
// kernels/rope/rope.bm:22-52: theta_d = 1 / theta^(2d/D), angle = theta_d * pos,
// (x_r, x_i) -> (x_r cos - x_i sin, x_r sin + x_i cos), all in f32 with no
// fused multiply-adds, the result rounded to the io type by the caller.
__device__ __forceinline__ void rope_pair(float& xr, float& xi, int d, int D, float theta, float pos) {
    const float freq = __fdiv_rn(1.0f, powf(theta, __fdiv_rn(2.0f * (float)d, (float)D)));
    float s, c;
    sincosf(__fmul_rn(freq, pos), &s, &c);
    const float r = __fsub_rn(__fmul_rn(xr, c), __fmul_rn(xi, s));
    const float i = __fadd_rn(__fmul_rn(xr, s), __fmul_rn(xi, c));
    xr = r;
    xi = i;
}

}  // namespace vw
