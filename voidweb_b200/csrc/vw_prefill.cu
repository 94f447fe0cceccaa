// vw_prefill.cu -- chunked prefill over the paged pool: the chunk append and
// the prefill attention.
//
// Reference: kernels/attention/flash_attention.bm:31-106 (flash_attention_fwd:
// FlashAttention-2 over contiguous K/V, BLOCK_Q = 64 query tokens per CTA,
// BLOCK_KV = 64 keys per tile, online softmax, no causal mask, block_table
// unused) and its launcher :167-177; the chunking comes from the scheduler
// (scheduler/scheduler.bm:251-266: up to 2048 prompt tokens per step, the
// sequence's block table alongside).  Here the keys are the pool's pages: the
// chunk of sequence b holds positions ctx_start[b] .. ctx_start[b] + n_b - 1,
// its K/V rows are appended into their slots first (prefill_append_kernel),
// then query token i attends to keys 0 .. ctx_start[b] + i (causal, what a
// decoder needs) or to all ctx_start[b] + n_b keys (the reference kernel's
// seq_kv, without a mask).
//
//  * Work split.  CTA (tile, q head): 64 query tokens of one sequence for one
//    query head; four consumer warps own 16 tokens each; the page-heads of the
//    head's KV head stream through a ring of shared-memory stages (one TMA box
//    per page-head, the decode's tensor map) and every warp reads every page.
//  * Math.  Per page (16 keys) and warp: S = Q K^T as 2 x D/16 mma.sync
//    m16n8k16 (query tokens as M, keys as N, K fragments by ldmatrix from the
//    swizzled stage), the causal / length mask, an online softmax in the log2
//    domain, then O += P V with P reused from the S fragments as the A operand
//    (for bf16 pages as a bf16 pair hi + lo) and V fragments by transposing
//    ldmatrix.  f32 accumulation.
//  * Every wait is bounded; on timeout the kernel records kDevErrTimeout,
//    drains its TMA loads and returns.
#include <cuda.h>
#include <cuda_runtime.h>
#include <atomic>
#include <cstdint>

#include "vw_fp8.cuh"
#include "vw_internal.h"
#include "vw_ptx.cuh"
#include "vw_rope.cuh"

namespace vw {

namespace {

constexpr int kPfWarps = 4;                       // consumer warps, 16 query tokens each
constexpr int kPfTile = 16 * kPfWarps;            // query tokens per CTA
constexpr int kPfStages = 8;                      // page-head stages in the ring

constexpr int pf_align(int x, int a) { return (x + a - 1) / a * a; }

template <int D_, int IO_>
struct PfTraits {
    static constexpr int D = D_, IO = IO_;
    static constexpr int W = kPfWarps;
    static constexpr int THREADS = (W + 1) * 32;
    static constexpr int KT = D / 16;             // k-steps of S = Q K^T
    static constexpr int NO = D / 8;              // n-tiles (8 d each) of O
    static constexpr int CHUNKS = D * 2 / 128;    // 128-B columns of a row
    static constexpr int STAGE = 32 * D * 2;      // one page-head: K rows 0-15, V rows 16-31
    static constexpr int S = kPfStages;
    static constexpr int TPFX = pf_align((kMaxBatchPerLaunch + 1) * 4, 128);
    static constexpr int SMEM = 1024 + S * STAGE + TPFX + 2 * S * 8;
    static constexpr bool MMA_BF16 = IO == kBF16;
    static_assert(D == 64 || D == 128, "head_dim 64 or 128");
    static_assert(STAGE % 1024 == 0, "1024-B stage alignment (128-B swizzle)");
};

template <int IO>
__device__ __forceinline__ float pf_io_to_f32(uint32_t h) {
    return IO == kBF16 ? bf16_bits_to_f32(h) : f16_bits_to_f32(h);
}
template <int IO>
__device__ __forceinline__ uint16_t pf_f32_to_io(float f) {
    return IO == kBF16 ? f32_to_bf16_bits(f) : f32_to_f16_bits(f);
}

// Largest b with pfx[b] <= x over b in [0, B).
__device__ __forceinline__ int pf_find(const int* pfx, int B, int x) {
    int lo = 0, hi = B - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (pfx[mid] <= x) lo = mid; else hi = mid - 1;
    }
    return lo;
}

// Largest b with cu_q[b] <= i, reading the offsets from global memory.
__device__ __forceinline__ int pf_find_global(const int32_t* cu_q, int B, int i) {
    int lo = 0, hi = B - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (__ldg(cu_q + mid) <= i) lo = mid; else hi = mid - 1;
    }
    return lo;
}

// ------------------------------------------------------------------ append

// One warp per (token i, KV head h): the K and V rows of the token go to slot
// block_tables[b][p/16]*16 + p%16, p = ctx_start[b] + i - cu_q[b] (the paging
// rule of flash_attention.bm:132-140).  With rope_theta > 0 the K row is rotated
// at position p first (lane l holds elements l*D/32 .. +D/32-1, whose partners
// d +- D/2 lane l ^ 16 holds), rounded to the io type as a separate RoPE pass
// would.  FP8 pools quantise each row with its own scale (the decode's codec).
__global__ void __launch_bounds__(256) prefill_append_kernel(
    PoolGeom g, uint8_t* __restrict__ data, float* __restrict__ scales, uint32_t layer,
    const uint16_t* __restrict__ k_new, const uint16_t* __restrict__ v_new,
    const int32_t* __restrict__ cu_q, const int32_t* __restrict__ ctx_start,
    const uint32_t* __restrict__ block_tables, uint32_t bt_stride, uint32_t B, uint32_t T,
    float rope_theta, uint32_t* err) {
    const uint32_t lane = threadIdx.x & 31;
    const uint64_t w = (uint64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (w >= (uint64_t)T * g.num_kv_heads) return;
    const uint32_t h = (uint32_t)(w % g.num_kv_heads);
    const int i = (int)(w / g.num_kv_heads);
    if (i >= __ldg(cu_q + B)) return;                  // past the last chunk
    const int b = pf_find_global(cu_q, (int)B, i);
    const int p = __ldg(ctx_start + b) + (i - __ldg(cu_q + b));
    if (p < 0 || p >= (int)(bt_stride * kBlockSize)) {
        if (lane == 0) atomicOr(err, kDevErrSeqLen);
        return;
    }
    const uint32_t blk = __ldg(block_tables + (size_t)b * bt_stride + p / kBlockSize);
    if (blk >= g.num_blocks) {
        if (lane == 0) atomicOr(err, kDevErrBlockId);
        return;
    }
    const uint32_t D = g.head_dim, PER = D / 32;       // 2 (D=64) or 4 (D=128) elements per lane
    const float pos = (float)p;
    for (uint32_t kv = 0; kv < 2; ++kv) {
        const uint16_t* src = (kv == 0 ? k_new : v_new) + ((size_t)i * g.num_kv_heads + h) * D + lane * PER;
        uint32_t w2[2] = {0u, 0u};
        w2[0] = *reinterpret_cast<const uint32_t*>(src);
        if (PER == 4) w2[1] = *reinterpret_cast<const uint32_t*>(src + 2);
        if (kv == 0 && rope_theta > 0.0f) {
            const bool lo = lane < 16;
            for (uint32_t k = 0; k < PER / 2; ++k) {
                const uint32_t own = w2[k];
                const uint32_t other = __shfl_xor_sync(0xffffffffu, own, 16);
                const uint32_t rw = lo ? own : other, iw = lo ? other : own;
                float r0 = g.io_kind == kBF16 ? bf16_bits_to_f32(rw & 0xFFFFu) : f16_bits_to_f32(rw & 0xFFFFu);
                float i0 = g.io_kind == kBF16 ? bf16_bits_to_f32(iw & 0xFFFFu) : f16_bits_to_f32(iw & 0xFFFFu);
                float r1 = g.io_kind == kBF16 ? bf16_bits_to_f32(rw >> 16) : f16_bits_to_f32(rw >> 16);
                float i1 = g.io_kind == kBF16 ? bf16_bits_to_f32(iw >> 16) : f16_bits_to_f32(iw >> 16);
                const int d = (int)((lane & 15) * PER + 2 * k);
                rope_pair(r0, i0, d, (int)D, rope_theta, pos);
                rope_pair(r1, i1, d + 1, (int)D, rope_theta, pos);
                const float a0 = lo ? r0 : i0, a1 = lo ? r1 : i1;
                const uint32_t b0 = g.io_kind == kBF16 ? f32_to_bf16_bits(a0) : f32_to_f16_bits(a0);
                const uint32_t b1 = g.io_kind == kBF16 ? f32_to_bf16_bits(a1) : f32_to_f16_bits(a1);
                w2[k] = b0 | (b1 << 16);
            }
        }
        const uint64_t row = ((((uint64_t)layer * g.num_blocks + blk) * g.num_kv_heads + h) * 2 + kv) *
                                 kBlockSize + (uint32_t)p % kBlockSize;
        if (g.kv_kind != kFP8) {
            uint8_t* dst = data + row * D * 2 + lane * PER * 2;
            if (PER == 4) *reinterpret_cast<uint2*>(dst) = make_uint2(w2[0], w2[1]);
            else *reinterpret_cast<uint32_t*>(dst) = w2[0];
        } else {
            // FP8 pools have head_dim 128: four elements per lane
            float v[4];
            for (int e = 0; e < 4; ++e) {
                const uint32_t hbits = (w2[e >> 1] >> (16 * (e & 1))) & 0xFFFFu;
                v[e] = g.io_kind == kBF16 ? bf16_bits_to_f32(hbits) : f16_bits_to_f32(hbits);
            }
            float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
            const float scale = fp8_row_scale(amax);
            *reinterpret_cast<uint32_t*>(data + row * D + lane * 4) = fp8_encode4(v, scale, g.fp8_ocp != 0);
            if (lane == 0) scales[row] = scale;
        }
    }
}

// ------------------------------------------------------------------ attention

// Query fragments (A operand of S = Q K^T) of this warp's 16 tokens, rows
// lane/4 and lane/4 + 8: k-step kt holds elements kt*16 + 2c, +1 (regs 0, 1)
// and kt*16 + 8 + 2c, +1 (regs 2, 3), c = lane % 4.  With rope_theta > 0 each
// row is rotated at its own position (the partner d + D/2 of an element of
// k-step kt < KT/2 is the same register of k-step kt + KT/2).
template <class T>
__device__ __forceinline__ void pf_load_q(const PrefillParams& p, const uint8_t* q0, int row_stride,
                                          bool live0, bool live1, float pos0, float pos1, int lane,
                                          uint32_t (&qa)[T::KT][4]) {
    const int g = lane >> 2, c = lane & 3;
    const uint8_t* r0 = q0 + (size_t)g * row_stride;
    const uint8_t* r1 = q0 + (size_t)(g + 8) * row_stride;
#pragma unroll
    for (int kt = 0; kt < T::KT; ++kt) {
        const int d0 = kt * 16 + 2 * c, d1 = d0 + 8;
        qa[kt][0] = live0 ? __ldg(reinterpret_cast<const uint32_t*>(r0 + d0 * 2)) : 0u;
        qa[kt][1] = live1 ? __ldg(reinterpret_cast<const uint32_t*>(r1 + d0 * 2)) : 0u;
        qa[kt][2] = live0 ? __ldg(reinterpret_cast<const uint32_t*>(r0 + d1 * 2)) : 0u;
        qa[kt][3] = live1 ? __ldg(reinterpret_cast<const uint32_t*>(r1 + d1 * 2)) : 0u;
    }
    if (p.rope_theta > 0.0f) {
#pragma unroll
        for (int kt = 0; kt < T::KT / 2; ++kt)
#pragma unroll
            for (int x = 0; x < 4; ++x) {
                const int d = kt * 16 + (x >> 1) * 8 + 2 * c;
                const float pos = (x & 1) ? pos1 : pos0;
                uint32_t& a = qa[kt][x];
                uint32_t& bb = qa[kt + T::KT / 2][x];
                float ar = pf_io_to_f32<T::IO>(a & 0xFFFFu), ai = pf_io_to_f32<T::IO>(bb & 0xFFFFu);
                float br = pf_io_to_f32<T::IO>(a >> 16), bi = pf_io_to_f32<T::IO>(bb >> 16);
                rope_pair(ar, ai, d, T::D, p.rope_theta, pos);
                rope_pair(br, bi, d + 1, T::D, p.rope_theta, pos);
                a = (uint32_t)pf_f32_to_io<T::IO>(ar) | ((uint32_t)pf_f32_to_io<T::IO>(br) << 16);
                bb = (uint32_t)pf_f32_to_io<T::IO>(ai) | ((uint32_t)pf_f32_to_io<T::IO>(bi) << 16);
            }
    }
}

template <class T>
__global__ void __launch_bounds__(T::THREADS, 2)
prefill_kernel(const __grid_constant__ CUtensorMap tmap, const PrefillParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* stages = base;
    int* tpfx = reinterpret_cast<int*>(base + T::S * T::STAGE);
    uint64_t* full = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(tpfx) + T::TPFX);
    uint64_t* empty = full + T::S;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint64_t deadline = cycles() + kWaitDeadlineCycles;

    if (threadIdx.x == 0) {
        for (int s = 0; s < T::S; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], T::W); }
        fence_mbar_init();
    }
    if (p.flags & kDecodePdl) griddep_wait();     // q, chunk rows and pages from the predecessor
    // query tiles per sequence, prefix over the batch (warp 0)
    if (warp == 0) {
        int run = 0;
        if (lane == 0) tpfx[0] = 0;
        for (int b0 = 0; b0 < (int)p.B; b0 += 32) {
            const int b = b0 + lane;
            int nt = 0;
            if (b < (int)p.B) {
                const int n = __ldg(p.cu_q + b + 1) - __ldg(p.cu_q + b);
                nt = n > 0 ? (n + kPfTile - 1) / kPfTile : 0;
            }
            int incl = nt;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const int v = __shfl_up_sync(0xffffffffu, incl, off);
                if (lane >= off) incl += v;
            }
            if (b < (int)p.B) tpfx[b + 1] = run + incl;
            run += __shfl_sync(0xffffffffu, incl, 31);
        }
    }
    __syncthreads();
    const int x = blockIdx.x;
    if (x >= tpfx[p.B]) return;
    const int b = pf_find(tpfx, (int)p.B, x);
    const int q_off = __ldg(p.cu_q + b);
    const int n = __ldg(p.cu_q + b + 1) - q_off;
    const int cs = __ldg(p.ctx_start + b);
    const int total = cs + n;
    // the offsets come from device memory: a chunk outside q's T rows or past
    // its block-table row is flagged and skipped
    if (q_off < 0 || q_off + n > (int)p.T || cs < 0 || total > (int)(p.bt_stride * kBlockSize)) {
        if (threadIdx.x == 0) atomicOr(p.err, kDevErrSeqLen);
        return;
    }
    const int t0 = (x - tpfx[b]) * kPfTile;
    const int qmax = cs + min(t0 + kPfTile - 1, n - 1);          // last query position of the tile
    const int kend = p.causal ? qmax + 1 : total;                // keys [0, kend)
    const int npages = (kend + kBlockSize - 1) / kBlockSize;
    const int j = blockIdx.y, h = j / (int)p.group;

    if (warp == T::W) {
        // ---- producer: block ids 32 at a time, lane 0 issues one box per page-head
        bool ok = true;
        for (int i0 = 0; i0 < npages && ok; i0 += 32) {
            const int m = min(32, npages - i0);
            uint32_t blk = 0xFFFFFFFFu;
            if (lane < m) blk = __ldg(p.block_tables + (size_t)b * p.bt_stride + i0 + lane);
            for (int jj = 0; jj < m; ++jj) {
                const uint32_t bj = __shfl_sync(0xffffffffu, blk, jj);
                if (lane == 0 && ok) {
                    const int ii = i0 + jj, s = ii % T::S;
                    if (ii >= T::S && !mbar_wait(&empty[s], ((ii / T::S) - 1) & 1, deadline)) {
                        ok = false;
                    } else {
                        int row0 = -32;                  // negative row: TMA zero-fills
                        if (bj < p.num_blocks)
                            row0 = (int)(((p.layer * p.num_blocks + bj) * p.Hkv + (uint32_t)h) * 32u);
                        else
                            atomicOr(p.err, kDevErrBlockId);
                        mbar_arrive_expect_tx(&full[s], T::STAGE);
                        uint8_t* st = stages + s * T::STAGE;
                        if constexpr (T::CHUNKS == 1)
                            tma_load_2d(st, &tmap, &full[s], 0, row0);
                        else
                            tma_load_3d(st, &tmap, &full[s], 0, row0, 0);
                    }
                }
                ok = __shfl_sync(0xffffffffu, ok, 0);
            }
        }
        if (lane == 0) {
            if (!ok) atomicOr(p.err, kDevErrTimeout);
            // drain: no TMA write may land after the CTA has exited
            const int issued = ok ? npages : 0;
            for (int ii = issued > T::S ? issued - T::S : 0; ii < issued; ++ii)
                if (!mbar_wait(&full[ii % T::S], (ii / T::S) & 1, deadline)) {
                    atomicOr(p.err, kDevErrTimeout);
                    break;
                }
        }
        return;
    }

    // ---- consumer warp: query tokens t0 + 16*warp + (lane/4, lane/4 + 8)
    const int g = lane >> 2, c = lane & 3;
    const int tq0 = t0 + 16 * warp + g, tq1 = tq0 + 8;
    const bool live0 = tq0 < n, live1 = tq1 < n;
    const int qp0 = cs + tq0, qp1 = cs + tq1;                    // query positions
    const int kend0 = p.causal ? qp0 + 1 : total, kend1 = p.causal ? qp1 + 1 : total;
    const size_t row_stride = (size_t)p.Hq * T::D * 2;
    const uint8_t* qbase = reinterpret_cast<const uint8_t*>(p.q) +
                           ((size_t)(q_off + t0 + 16 * warp) * p.Hq + j) * T::D * 2;
    uint32_t qa[T::KT][4];
    pf_load_q<T>(p, qbase, (int)row_stride, live0, live1, (float)qp0, (float)qp1, lane, qa);

    float o[T::NO][4];
#pragma unroll
    for (int nt = 0; nt < T::NO; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.0f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;

    // ldmatrix lane geometry (as the decode): K rows feed the B operand of
    // S = Q K^T (keys as N), V rows the B operand of O = P V through the
    // transposing load
    const int mi = lane >> 3;
    const int k_tok = (lane & 7) + ((mi & 1) << 3), k_hs = mi >> 1;
    const int v_tok = (lane & 7) + ((mi >> 1) << 3), v_hs = mi & 1;
    bool alive = true;
    for (int ii = 0; ii < npages && alive; ++ii) {
        const int s = ii % T::S;
        if (!__all_sync(0xffffffffu, mbar_wait(&full[s], (ii / T::S) & 1, deadline))) {
            if (lane == 0) atomicOr(p.err, kDevErrTimeout);
            alive = false;
            break;
        }
        uint8_t* st = stages + s * T::STAGE;
        const int key0 = ii * kBlockSize;
        if (key0 + kBlockSize > total) {
            // keys past the sequence hold whatever the pool has there: zero
            // their V rows (every warp writes the same zeros before reading) so
            // that masked probabilities cannot meet NaN or Inf
            const int valid = total - key0;
            const int per_row = T::CHUNKS * 8;
            for (int k = lane; k < (16 - valid) * per_row; k += 32) {
                const int piece = k % per_row, row = 16 + valid + k / per_row;
                *reinterpret_cast<uint4*>(st + (piece >> 3) * 4096 + row * 128 + ((piece & 7) << 4)) =
                    make_uint4(0, 0, 0, 0);
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
        }
        const uint32_t tbase = smem_u32(st);
        float sa[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
        for (int kt = 0; kt < T::KT; ++kt) {
            uint32_t r0, r1, r2, r3;
            ldsm_x4(tbase + (kt >> 2) * 4096 + k_tok * 128 + ((((kt & 3) * 2 + k_hs) ^ (k_tok & 7)) << 4),
                    r0, r1, r2, r3);
            // r0 / r2: keys 0-7 (d 0-7 / 8-15 of the k-step), r1 / r3: keys 8-15
            mma_16816<T::MMA_BF16>(sa[0], qa[kt][0], qa[kt][1], qa[kt][2], qa[kt][3], r0, r2);
            mma_16816<T::MMA_BF16>(sa[1], qa[kt][0], qa[kt][1], qa[kt][2], qa[kt][3], r1, r3);
        }
        // scores of rows g (sa[.][0..1]) and g+8 (sa[.][2..3]); keys key0 + 8*nh + 2c + e
        float sv[2][4];
        float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
        for (int nh = 0; nh < 2; ++nh)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int key = key0 + nh * 8 + 2 * c + e;
                sv[nh][e] = key < kend0 ? sa[nh][e] * p.scale_log2 : -INFINITY;
                sv[nh][2 + e] = key < kend1 ? sa[nh][2 + e] * p.scale_log2 : -INFINITY;
                mx0 = fmaxf(mx0, sv[nh][e]);
                mx1 = fmaxf(mx1, sv[nh][2 + e]);
            }
#pragma unroll
        for (int off = 1; off < 4; off <<= 1) {
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
            mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
        }
        const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
        // a row with no key yet keeps the reference point 0 (its scores are -inf)
        const float ref0 = mn0 == -INFINITY ? 0.0f : mn0, ref1 = mn1 == -INFINITY ? 0.0f : mn1;
        const float al0 = ex2(m0 - ref0), al1 = ex2(m1 - ref1);
        m0 = mn0;
        m1 = mn1;
        l0 *= al0;
        l1 *= al1;
#pragma unroll
        for (int nt = 0; nt < T::NO; ++nt) {
            o[nt][0] *= al0; o[nt][1] *= al0;
            o[nt][2] *= al1; o[nt][3] *= al1;
        }
        float pr[2][4];
#pragma unroll
        for (int nh = 0; nh < 2; ++nh) {
            pr[nh][0] = ex2(sv[nh][0] - ref0);
            pr[nh][1] = ex2(sv[nh][1] - ref0);
            pr[nh][2] = ex2(sv[nh][2] - ref1);
            pr[nh][3] = ex2(sv[nh][3] - ref1);
            l0 += pr[nh][0] + pr[nh][1];
            l1 += pr[nh][2] + pr[nh][3];
        }
        // P as the A operand (16 tokens x 16 keys): the S fragments in place.
        // A bf16 probability keeps 8 significant bits, too few where a row's
        // output is a near-cancelling sum of a few large V terms; bf16 pages
        // therefore add the rounding residual as a second operand (P = hi + lo,
        // ~2^-18 relative), f16 pages keep P in f16 (11 bits).
        uint32_t ph[4], pl[4] = {0u, 0u, 0u, 0u};
        {
            const float x[4][2] = {{pr[0][0], pr[0][1]}, {pr[0][2], pr[0][3]},
                                   {pr[1][0], pr[1][1]}, {pr[1][2], pr[1][3]}};
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                ph[r] = pack2<T::MMA_BF16>(x[r][0], x[r][1]);
                if constexpr (T::MMA_BF16)
                    pl[r] = pack2<true>(x[r][0] - bf16_bits_to_f32(ph[r] & 0xFFFFu),
                                        x[r][1] - bf16_bits_to_f32(ph[r] >> 16));
            }
        }
#pragma unroll
        for (int mt = 0; mt < T::D / 16; ++mt) {
            uint32_t r0, r1, r2, r3;
            ldsm_x4_t(tbase + (mt >> 2) * 4096 + (16 + v_tok) * 128 +
                          ((((mt & 3) * 2 + v_hs) ^ (v_tok & 7)) << 4),
                      r0, r1, r2, r3);
            // r0 / r2: d 16mt .. +7 for keys 0-7 / 8-15; r1 / r3: d 16mt + 8 .. +15
            mma_16816<T::MMA_BF16>(o[2 * mt], ph[0], ph[1], ph[2], ph[3], r0, r2);
            mma_16816<T::MMA_BF16>(o[2 * mt + 1], ph[0], ph[1], ph[2], ph[3], r1, r3);
            if constexpr (T::MMA_BF16) {
                mma_16816<true>(o[2 * mt], pl[0], pl[1], pl[2], pl[3], r0, r2);
                mma_16816<true>(o[2 * mt + 1], pl[0], pl[1], pl[2], pl[3], r1, r3);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
    if (!alive) return;
#pragma unroll
    for (int off = 1; off < 4; off <<= 1) {
        l0 += __shfl_xor_sync(0xffffffffu, l0, off);
        l1 += __shfl_xor_sync(0xffffffffu, l1, off);
    }
    const float inv0 = 1.0f / l0, inv1 = 1.0f / l1;
    uint8_t* obase = reinterpret_cast<uint8_t*>(p.out) + ((size_t)(q_off + t0 + 16 * warp) * p.Hq + j) * T::D * 2;
#pragma unroll
    for (int nt = 0; nt < T::NO; ++nt) {
        const int d = nt * 8 + 2 * c;
        if (live0)
            *reinterpret_cast<uint32_t*>(obase + (size_t)g * row_stride + d * 2) =
                (uint32_t)pf_f32_to_io<T::IO>(o[nt][0] * inv0) | ((uint32_t)pf_f32_to_io<T::IO>(o[nt][1] * inv0) << 16);
        if (live1)
            *reinterpret_cast<uint32_t*>(obase + (size_t)(g + 8) * row_stride + d * 2) =
                (uint32_t)pf_f32_to_io<T::IO>(o[nt][2] * inv1) | ((uint32_t)pf_f32_to_io<T::IO>(o[nt][3] * inv1) << 16);
    }
}

template <class T>
cudaError_t launch_t(const PrefillLaunch& L) {
    static std::atomic<bool> configured{false};
    if (!configured.load()) {
        cudaError_t e = cudaFuncSetAttribute(prefill_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             T::SMEM);
        if (e != cudaSuccess) return e;
        configured.store(true);
    }
    const PrefillParams& p = L.p;
    // an upper bound on the query tiles: sum over b of ceil(n_b / 64) <= T / 64 + B
    const uint32_t tiles = (p.T + kPfTile - 1) / kPfTile + p.B;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(tiles, p.Hq);
    cfg.blockDim = dim3(T::THREADS);
    cfg.dynamicSmemBytes = T::SMEM;
    cfg.stream = L.stream;
    cudaLaunchAttribute attr[1];
    if (p.flags & kDecodePdl) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    return cudaLaunchKernelEx(&cfg, prefill_kernel<T>, *L.tmap, p);
}

}  // namespace

int prefill_query_tile() { return kPfTile; }

cudaError_t launch_paged_prefill(const PrefillLaunch& L) {
    if (L.kv_kind == kFP8) return cudaErrorNotSupported;
    if (L.head_dim == 128)
        return L.io_kind == kBF16 ? launch_t<PfTraits<128, kBF16>>(L) : launch_t<PfTraits<128, kF16>>(L);
    if (L.head_dim == 64)
        return L.io_kind == kBF16 ? launch_t<PfTraits<64, kBF16>>(L) : launch_t<PfTraits<64, kF16>>(L);
    return cudaErrorNotSupported;
}

cudaError_t launch_prefill_append(const PoolGeom& g, uint8_t* data, float* scales, uint32_t layer,
                                  const void* k_new, const void* v_new, const int32_t* cu_q,
                                  const int32_t* ctx_start, const uint32_t* block_tables,
                                  uint32_t bt_stride, uint32_t B, uint32_t T, float rope_theta,
                                  uint32_t* err, cudaStream_t s) {
    const uint64_t warps = (uint64_t)T * g.num_kv_heads;
    if (warps == 0) return cudaSuccess;
    const uint32_t blocks = (uint32_t)((warps + 7) / 8);
    prefill_append_kernel<<<blocks, 256, 0, s>>>(g, data, scales, layer,
                                                 static_cast<const uint16_t*>(k_new),
                                                 static_cast<const uint16_t*>(v_new), cu_q, ctx_start,
                                                 block_tables, bt_stride, B, T, rope_theta, err);
    return cudaGetLastError();
}

}  // namespace vw
