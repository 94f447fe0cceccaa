// vw_fp8w.cu -- the FP8 weight path that shares the KV codec: RMSNorm with
// E4M3 output and the E4M3 x E4M3 -> bf16 GEMM.
//
// Reference: kernels/norm/rms_norm.bm:62-94 (rms_norm_fp8_out: one warp per
// row, lane-strided sum of squares, butterfly shuffle reduction, the
// truncating encoder of :98-113) and kernels/gemm/gemm_fp8.bm:31-107 (gemm_fp8:
// C = (a_scale * b_scale) * (A . B) + bias with the decoder of :110-116, bf16
// out; tiles 128 x 128 x 64, a scalar dot product per output).
//
//  * rms_norm_fp8_kernel follows the reference's operation order exactly (one
//    warp per row, f32 multiply and add without contraction, the butterfly
//    at distances 16 .. 1, IEEE sqrt and divisions), so its codes are the
//    reference's bit for bit.
//  * gemm_fp8_kernel runs on the tcgen05 tensor cores in kind::f16: the
//    reference decoder differs from the hardware E4M3 format (0x7F / 0xFF
//    decode to +-480 instead of NaN, codes with a zero exponent field to
//    (1 + m/8) 2^-7 instead of subnormals, 0x80 to -2^-7), so the codes are
//    decoded on the CUDA cores into binary16, which holds every reference value
//    exactly: for a code c != 0 the half is (c & 0x80) << 8 | ((c & 0x7F) << 7)
//    + 0x2000, i.e. exponent field e + 8 and mantissa m << 7.  CTA = a 128 x 128
//    tile of C; four warps decode 64-deep slices of A (K-major) and B
//    (MN-major) into 128-B-swizzled f16 stages, one lane issues 4 MMAs
//    (M = 128, N = 128, K = 16) per slice into a tensor-memory accumulator, and
//    the four warps apply the scales and the bias and store bf16 rows.
#include <cuda.h>
#include <cuda_runtime.h>
#include <atomic>
#include <cstdint>

#include "vw_fp8.cuh"
#include "vw_internal.h"
#include "vw_ptx.cuh"
#include "vw_tc.cuh"

namespace vw {

namespace {

// ------------------------------------------------------------------ RMSNorm

__global__ void __launch_bounds__(128) rms_norm_fp8_kernel(const uint16_t* __restrict__ x,
                                                           const uint16_t* __restrict__ w,
                                                           uint8_t* __restrict__ out, uint32_t rows,
                                                           uint32_t hidden, float scale, float eps) {
    const uint32_t row = blockIdx.x * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= rows) return;
    const uint16_t* xr = x + (size_t)row * hidden;
    float sum = 0.0f;
    for (uint32_t d = lane; d < hidden; d += 32) {
        const float v = f16_bits_to_f32(xr[d]);
        sum = __fadd_rn(sum, __fmul_rn(v, v));
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, off));
    const float inv_rms = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, (float)hidden), eps)));
    uint8_t* o = out + (size_t)row * hidden;
    for (uint32_t d = lane; d < hidden; d += 32) {
        const float v = f16_bits_to_f32(xr[d]), wt = f16_bits_to_f32(w[d]);
        o[d] = (uint8_t)fp8_encode_ref(__fmul_rn(__fmul_rn(__fmul_rn(v, inv_rms), wt), scale));
    }
}

// ------------------------------------------------------------------ GEMM

constexpr int kGm = 128, kGn = 128, kGk = 64;   // C tile, K slice
constexpr int kGst = 3;                         // f16 slice stages
constexpr int kGaBytes = kGm * kGk * 2;         // A slice: [128 rows][128 B]
constexpr int kGbBytes = kGk * kGn * 2;         // B slice: [2 columns of 64 n][64 rows][128 B]
constexpr int kGstage = kGaBytes + kGbBytes;
constexpr int kGsmem = 1024 + kGst * kGstage + 2 * kGst * 8 + 8 + 16;
constexpr uint32_t kGidesc = idesc_f16(false, true, kGm, kGn);   // f16, B MN-major

// Codes c0 (bits 0-7) and c1 (bits 16-23) of v -> the f16 pair of their
// reference decodings (c == 0 -> 0).
__device__ __forceinline__ uint32_t dec2(uint32_t v) {
    const uint32_t c = v & 0x00FF00FFu;
    const uint32_t h = ((c & 0x00800080u) << 8) | (((c & 0x007F007Fu) << 7) + 0x20002000u);
    const uint32_t zero = __vcmpeq2(c, 0u);       // 0xFFFF in each half whose code is 0
    return h & ~zero;
}

// 16 codes (one uint4) -> 16 f16 values (two uint4), in order.
__device__ __forceinline__ void dec16(const uint4 v, uint4& lo, uint4& hi) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    uint32_t r[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        r[2 * i] = dec2(__byte_perm(w[i], 0u, 0x4140));       // codes 0, 1
        r[2 * i + 1] = dec2(__byte_perm(w[i], 0u, 0x4342));   // codes 2, 3
    }
    lo = make_uint4(r[0], r[1], r[2], r[3]);
    hi = make_uint4(r[4], r[5], r[6], r[7]);
}

__global__ void __launch_bounds__(160, 1)
gemm_fp8_kernel(const uint8_t* __restrict__ A, const uint8_t* __restrict__ B, uint16_t* __restrict__ C,
                const uint16_t* __restrict__ bias, uint32_t M, uint32_t N, uint32_t K, float scale,
                uint32_t* err) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(base + kGst * kGstage);
    uint64_t* empty = full + kGst;
    uint64_t* done = empty + kGst;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint64_t deadline = cycles() + kWaitDeadlineCycles;
    const uint32_t m0 = blockIdx.x * kGm, n0 = blockIdx.y * kGn;
    const int nk = (int)((K + kGk - 1) / kGk);
    if (threadIdx.x == 0) {
        for (int s = 0; s < kGst; ++s) { mbar_init(&full[s], 4); mbar_init(&empty[s], 1); }
        mbar_init(done, 1);
        fence_mbar_init();
    }
    if (warp == 4) {
        tmem_alloc(tmem_slot, 128);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tmem_slot;
    bool ok = true;

    if (warp == 4) {
        if (lane == 0) {
            for (int kt = 0; kt < nk && ok; ++kt) {
                const int s = kt % kGst;
                if (!mbar_wait(&full[s], (kt / kGst) & 1, deadline)) { ok = false; break; }
                tc_fence_after();
                const uint32_t sa = smem_u32(base + s * kGstage), sb = sa + kGaBytes;
#pragma unroll
                for (int kk = 0; kk < kGk / 16; ++kk) {
                    // A: K-major rows of 128 B; B: MN-major, 64-element columns 8 KB apart
                    const uint64_t ad = smem_desc_sw128(sa + kk * 32, 16, 1024);
                    const uint64_t bd = smem_desc_sw128(sb + kk * 16 * 128, kGk * 128, 1024);
                    tc_mma_ss(tbase, ad, bd, kGidesc, (kt > 0 || kk > 0) ? 1u : 0u);
                }
                tc_commit(&empty[s]);
            }
            if (!ok) atomicOr(err, kDevErrTimeout);
            // every issued MMA completes before the tensor memory is freed; they
            // finish in bounded time, so the wait has a deadline of its own
            tc_commit(done);
            if (!mbar_wait(done, 0, cycles() + kWaitDeadlineCycles)) atomicOr(err, kDevErrTimeout);
        }
    } else {
        // ---- decoders: thread t takes row t of the A slice and half a row of
        // the B slice (row t % 64, columns 64 * (t / 64) .. +63)
        const int t = threadIdx.x;
        const uint32_t am = m0 + t;
        const int bk = t & 63, bc = t >> 6;
        const uint32_t bn = n0 + 64 * bc;
        for (int kt = 0; kt < nk && ok; ++kt) {
            const int s = kt % kGst;
            const uint32_t k0 = (uint32_t)kt * kGk;
            // this lane's codes (zero outside the matrices; K and N are multiples of 16)
            uint4 av[4], bv[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const uint32_t ka = k0 + 16 * u;
                av[u] = (am < M && ka < K) ? __ldg(reinterpret_cast<const uint4*>(A + (size_t)am * K + ka))
                                           : make_uint4(0, 0, 0, 0);
                const uint32_t kb = k0 + bk, nb = bn + 16 * u;
                bv[u] = (kb < K && nb < N) ? __ldg(reinterpret_cast<const uint4*>(B + (size_t)kb * N + nb))
                                           : make_uint4(0, 0, 0, 0);
            }
            if (kt >= kGst && !__all_sync(0xffffffffu, mbar_wait(&empty[s], ((kt / kGst) - 1) & 1, deadline))) {
                ok = false;
                break;
            }
            uint8_t* ar = base + s * kGstage + t * 128;
            uint8_t* br = base + s * kGstage + kGaBytes + bc * (kGk * 128) + bk * 128;
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                uint4 lo, hi;
                dec16(av[u], lo, hi);
                *reinterpret_cast<uint4*>(ar + (((2 * u) ^ (t & 7)) << 4)) = lo;
                *reinterpret_cast<uint4*>(ar + (((2 * u + 1) ^ (t & 7)) << 4)) = hi;
                dec16(bv[u], lo, hi);
                *reinterpret_cast<uint4*>(br + (((2 * u) ^ (bk & 7)) << 4)) = lo;
                *reinterpret_cast<uint4*>(br + (((2 * u + 1) ^ (bk & 7)) << 4)) = hi;
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(&full[s]);
        }
        // ---- epilogue: row t of the tile from tensor memory
        if (ok && __all_sync(0xffffffffu, mbar_wait(done, 0, deadline))) {
            tc_fence_after();
            const uint32_t lanes = (uint32_t)(warp * 32) << 16;
#pragma unroll 1
            for (int c0 = 0; c0 < kGn; c0 += 16) {
                uint32_t r[16];
                tmem_ld16(tbase + lanes + c0, r);
                tmem_wait_ld();
                const uint32_t n = n0 + c0;
                if (am < M && n < N) {
                    uint32_t wv[8];
#pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        const float b0 = bias ? bf16_bits_to_f32(bias[n + 2 * k]) : 0.0f;
                        const float b1 = bias ? bf16_bits_to_f32(bias[n + 2 * k + 1]) : 0.0f;
                        const float v0 = __uint_as_float(r[2 * k]) * scale + b0;
                        const float v1 = __uint_as_float(r[2 * k + 1]) * scale + b1;
                        wv[k] = pack2<true>(v0, v1);
                    }
                    uint8_t* dst = reinterpret_cast<uint8_t*>(C + (size_t)am * N + n);
                    *reinterpret_cast<uint4*>(dst) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
                    *reinterpret_cast<uint4*>(dst + 16) = make_uint4(wv[4], wv[5], wv[6], wv[7]);
                }
            }
        } else if (lane == 0) {
            atomicOr(err, kDevErrTimeout);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 4) {
        tc_fence_after();
        tmem_dealloc(tbase, 128);
    }
}

// Device error word of these kernels (they have no pool): kDevErrTimeout bits.
__device__ uint32_t g_fp8w_err;

}  // namespace

cudaError_t fp8w_error(uint32_t* word, bool clear) {
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return e;
    e = cudaMemcpyFromSymbol(word, g_fp8w_err, sizeof(uint32_t));
    if (e == cudaSuccess && clear) {
        const uint32_t zero = 0;
        e = cudaMemcpyToSymbol(g_fp8w_err, &zero, sizeof(uint32_t));
    }
    return e;
}

cudaError_t launch_rms_norm_fp8(const void* x, const void* w, uint8_t* out, uint32_t rows, uint32_t hidden,
                                float scale, float eps, cudaStream_t s) {
    if (rows == 0) return cudaSuccess;
    rms_norm_fp8_kernel<<<(rows + 3) / 4, 128, 0, s>>>(static_cast<const uint16_t*>(x),
                                                       static_cast<const uint16_t*>(w), out, rows, hidden,
                                                       scale, eps);
    return cudaGetLastError();
}

cudaError_t launch_gemm_fp8(const uint8_t* a, const uint8_t* b, void* c, const void* bias, uint32_t M,
                            uint32_t N, uint32_t K, float a_scale, float b_scale, cudaStream_t s) {
    uint32_t* err = nullptr;
    cudaError_t ge = cudaGetSymbolAddress(reinterpret_cast<void**>(&err), g_fp8w_err);
    if (ge != cudaSuccess) return ge;
    static std::atomic<bool> configured{false};
    if (!configured.load()) {
        cudaError_t e = cudaFuncSetAttribute(gemm_fp8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kGsmem);
        if (e != cudaSuccess) return e;
        configured.store(true);
    }
    const dim3 grid((M + kGm - 1) / kGm, (N + kGn - 1) / kGn);
    gemm_fp8_kernel<<<grid, 160, kGsmem, s>>>(a, b, static_cast<uint16_t*>(c),
                                              static_cast<const uint16_t*>(bias), M, N, K,
                                              a_scale * b_scale, err);
    return cudaGetLastError();
}

}  // namespace vw
