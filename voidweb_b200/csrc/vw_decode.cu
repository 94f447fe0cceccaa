// vw_decode.cu -- paged decode attention for B200 (sm_100a), optionally fused
// with the KV append of the step's new token.
//
// Reference: kernels/attention/flash_attention.bm:113-162 (paged_attention_decode:
// one CTA per sequence, HEAD_DIM threads, single head, per-token online softmax)
// and its launcher :180-189.  This kernel computes the same function --
// o = softmax(q K^T * scale) V over the sequence's pages found through its
// block table, the last page partial (:132-140) -- re-designed for B200:
//
//  * Work split.  The unit of work is one (sequence, KV head) page: 16 tokens of
//    K and V for one KV head.  All pages of all (sequence, KV head) segments are
//    laid end to end and cut into equal contiguous ranges, one per CTA of a
//    persistent grid sized to the SM count, so every CTA streams the same number
//    of bytes whatever the context lengths (split-K over pages).  A segment cut
//    by a range boundary leaves (o, max, sum) partials; the last CTA to finish a
//    piece of it (an atomic arrival counter, no waiting) merges them.
//  * GQA.  The Hq/Hkv query heads that share a KV head are processed together:
//    each K/V page is read from HBM once per KV head, never once per query head.
//  * Data movement.  One producer warp walks the block table and issues TMA
//    tensor loads of whole K and V page tiles (128-B swizzled) into a ring of
//    shared-memory stages tracked by mbarriers; no multicast.
//  * Math.  Each consumer warp takes every W-th page of the range and runs the
//    per-page micro-tiles on the tensor cores with warp-level mma.sync m16n8k16
//    (tokens as M, query heads as N: S^T = K Q^T, then O^T = V^T P^T), f32
//    accumulation, online softmax in the log2 domain with warp-shuffle maxima.
//    A page gives a 16 x 8 x 128 micro-tile, below the 64-row minimum of a
//    tcgen05 MMA, and the kernel is HBM-bound with tensor pipes mostly idle.
//  * Fused append.  With k_new / v_new given, the warp that owns a segment's last
//    page writes the new token's K/V row (quantised for FP8 pools) to its slot
//    block_table[p/16]*16 + p%16, p = seq_len-1, in HBM and into the staged page.
//  * FP8 pools.  Pages hold E4M3 codes plus one f32 scale per token per head;
//    the consumer warp expands a page into binary16 tiles in shared memory and
//    folds the scales into the scores and the probabilities.
//
// Every wait is bounded (vw_ptx.cuh); on timeout the kernel records
// kDevErrTimeout and unwinds after draining its outstanding TMA loads.
#include <cuda.h>
#include <cuda_runtime.h>
#include <atomic>
#include <cstdint>

#include "vw_fp8.cuh"
#include "vw_internal.h"
#include "vw_ptx.cuh"

namespace vw {

namespace {

constexpr int kConsumerWarps = 4;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kProducerWarp = kConsumerWarps;
constexpr int kSmemBudget = 200 * 1024;

__host__ __device__ constexpr int align_up_c(int x, int a) { return (x + a - 1) / a * a; }

template <int D_, int NT_, int KV_, int IO_>
struct Traits {
    static constexpr int D = D_, NT = NT_, KV = KV_, IO = IO_;
    static constexpr int G = 8 * NT;                         // padded query heads per KV head
    static constexpr int EB = KV == kFP8 ? 1 : 2;            // pool element bytes
    static constexpr int ROW = D * EB;                       // bytes of one token row
    static constexpr int CHUNKS = ROW / 128;                 // 128-B swizzle rows per token
    static constexpr int TILE = 16 * ROW;                    // one K (or V) page tile
    static constexpr int STAGE = align_up_c(2 * TILE + (KV == kFP8 ? 128 : 0), 1024);
    static constexpr bool MMA_BF16 = KV == kBF16;            // FP8 pages compute in f16
    static constexpr int KT = D / 16;                        // k-steps of Q K^T
    static constexpr int MT = D / 16;                        // d-tiles of V^T P^T
    static constexpr int CTILE = KV == kFP8 ? 16 * D * 2 : 0;  // f16 tile per K/V per warp
    static constexpr int MERGE = kConsumerWarps * G * (D + 2) * 4;
    static constexpr int PFX = align_up_c((kMaxBatchPerLaunch + 1) * 4, 128);
    static constexpr int FIXED = kConsumerWarps * 2 * CTILE + align_up_c(MERGE, 1024) + PFX +
                                 1024 /* mbarriers + flags */;
    static constexpr int S = (kSmemBudget - FIXED) / STAGE > 16 ? 16
                                                                 : (kSmemBudget - FIXED) / STAGE;
    static constexpr int SMEM = 1024 /*align slack*/ + S * STAGE + FIXED;
    static_assert(CHUNKS >= 1, "row must be at least 128 bytes");
    static_assert(S >= 4, "too few pipeline stages");
    static_assert(SMEM <= 227 * 1024, "shared memory over the per-CTA limit");
    static_assert((S * STAGE) % 1024 == 0 && (2 * CTILE) % 1024 == 0, "1024-B tile alignment");
};

struct Smem {
    uint8_t* stages;
    uint8_t* ctile;      // FP8 only: [W][2][CTILE]
    float* mo;           // [W][G][D]
    float* mm;           // [W][G]
    float* ml;           // [W][G]
    int* pfx;            // [B+1] exclusive prefix of pages per sequence
    uint64_t* full;      // [S]
    uint64_t* empty;     // [S]
    int* flag;           // scratch word for broadcasts
};

template <class T>
__device__ __forceinline__ Smem carve(uint8_t* base) {
    Smem s;
    uint8_t* p = base;
    s.stages = p; p += T::S * T::STAGE;
    s.ctile = p; p += kConsumerWarps * 2 * T::CTILE;
    s.mo = reinterpret_cast<float*>(p);
    s.mm = s.mo + kConsumerWarps * T::G * T::D;
    s.ml = s.mm + kConsumerWarps * T::G;
    p += align_up_c(T::MERGE, 1024);
    s.pfx = reinterpret_cast<int*>(p); p += T::PFX;               // keeps p 128-B aligned
    s.full = reinterpret_cast<uint64_t*>(p);
    s.empty = s.full + T::S;
    s.flag = reinterpret_cast<int*>(s.empty + T::S);
    return s;
}

// Byte offset of element (t, d) inside a 128-B-swizzled tile of 2-byte rows of D.
__device__ __forceinline__ uint32_t swz16(int t, int d) {
    int byte = d * 2;
    return (uint32_t)((byte >> 7) * 2048 + t * 128 + ((((byte & 127) >> 4) ^ (t & 7)) << 4) +
                      (byte & 15));
}
// Same for 1-byte rows of 128 (FP8, D = 128).
__device__ __forceinline__ uint32_t swz8(int t, int d) {
    return (uint32_t)(t * 128 + ((((d & 127) >> 4) ^ (t & 7)) << 4) + (d & 15));
}

// Largest b with Hkv * pfx[b] <= x (x < Hkv * pfx[B]).
__device__ __forceinline__ int find_seq(const int* pfx, int B, int Hkv, long long x) {
    int lo = 0, hi = B - 1;
    while (lo < hi) {
        int mid = (lo + hi + 1) >> 1;
        if ((long long)Hkv * pfx[mid] <= x) lo = mid; else hi = mid - 1;
    }
    return lo;
}

__device__ __forceinline__ void set_err(uint32_t* err, uint32_t bit) { atomicOr(err, bit); }

template <int IO>
__device__ __forceinline__ float io_to_f32(uint32_t h) {
    return IO == kBF16 ? bf16_bits_to_f32(h) : f16_bits_to_f32(h);
}
template <int IO>
__device__ __forceinline__ uint16_t f32_to_io(float f) {
    return IO == kBF16 ? f32_to_bf16_bits(f) : f32_to_f16_bits(f);
}

// ------------------------------------------------------------------ producer

template <class T>
__device__ void producer(const CUtensorMap* tmap, const DecodeParams& p, const Smem& sm,
                         int begin, int n, uint64_t deadline) {
    const int lane = threadIdx.x & 31;
    const uint64_t pol = policy_evict_first();
    const int Hkv = (int)p.Hkv;
    const int layer_base = (int)(p.layer * p.num_blocks);
    bool ok = true;
    for (int i0 = 0; i0 < n && ok; i0 += 32) {
        // each lane resolves one page of the next 32: segment, page, block id
        int i = i0 + lane;
        int c3 = 0, c4 = -1;
        if (i < n) {
            long long x = (long long)begin + i;
            int b = find_seq(sm.pfx, (int)p.B, Hkv, x);
            int np = sm.pfx[b + 1] - sm.pfx[b];
            int r = (int)(x - (long long)Hkv * sm.pfx[b]);
            int h = r / np, pg = r - h * np;
            uint32_t blk = __ldg(p.block_tables + (size_t)b * p.bt_stride + pg);
            c3 = h;
            if (blk < p.num_blocks) c4 = layer_base + (int)blk;
            else set_err(p.err, kDevErrBlockId);        // c4 = -1: TMA zero-fills the tile
        }
        const int m = min(32, n - i0);
        for (int j = 0; j < m; ++j) {
            const int ii = i0 + j;
            const int h = __shfl_sync(0xffffffffu, c3, j);
            const int row = __shfl_sync(0xffffffffu, c4, j);
            const int s = ii % T::S;
            if (ii >= T::S && !mbar_wait(&sm.empty[s], ((ii / T::S) - 1) & 1, deadline)) {
                ok = false;
                break;
            }
            if (lane == 0) {
                uint8_t* st = sm.stages + s * T::STAGE;
                const bool scales = T::KV == kFP8 && row >= 0;
                if (T::KV == kFP8 && !scales) {
                    // invalid block id: zero scales (plain stores, ordered before the
                    // arrive below, and fenced against this stage's next TMA write)
                    float* dst = reinterpret_cast<float*>(st + 2 * T::TILE);
                    for (int k = 0; k < 32; ++k) dst[k] = 0.0f;
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                }
                mbar_arrive_expect_tx(&sm.full[s], 2 * T::TILE + (scales ? 128 : 0));
                for (int c = 0; c < T::CHUNKS; ++c) {
                    tma_load_5d(st + c * 2048, tmap, &sm.full[s], 0, c, 0, h, row, pol);
                    tma_load_5d(st + T::TILE + c * 2048, tmap, &sm.full[s], 0, c, 0, Hkv + h,
                                row, pol);
                }
                if (scales) {
                    // scales of this page: K then V, 16 f32 each
                    const float* ks = p.kv_scales + ((size_t)row * 2 * Hkv + h) * 16;
                    const float* vs = p.kv_scales + ((size_t)row * 2 * Hkv + Hkv + h) * 16;
                    bulk_load(st + 2 * T::TILE, ks, 64, &sm.full[s], pol);
                    bulk_load(st + 2 * T::TILE + 64, vs, 64, &sm.full[s], pol);
                }
            }
            __syncwarp();
        }
    }
    if (!ok) set_err(p.err, kDevErrTimeout);
    // Drain: never leave the CTA while a TMA load may still write its smem.
    const int first = n > T::S ? n - T::S : 0;
    for (int ii = first; ii < n; ++ii) {
        if (!mbar_wait(&sm.full[ii % T::S], (ii / T::S) & 1, deadline)) {
            set_err(p.err, kDevErrTimeout);
            break;
        }
    }
}

// ------------------------------------------------------------------ consumer

template <class T>
__device__ __forceinline__ void load_q(const DecodeParams& p, int b, int h, int lane,
                                       uint32_t (&qf)[T::NT][T::KT][2]) {
    const uint16_t* q = reinterpret_cast<const uint16_t*>(p.q);
#pragma unroll
    for (int nt = 0; nt < T::NT; ++nt) {
        const int j = nt * 8 + (lane >> 2);
        const bool live = j < (int)p.group;
        const uint16_t* row = q + ((size_t)b * p.Hq + (size_t)h * p.group + (live ? j : 0)) * T::D;
#pragma unroll
        for (int kt = 0; kt < T::KT; ++kt) {
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
                const int d = kt * 16 + hf * 8 + 2 * (lane & 3);
                uint32_t v = live ? __ldg(reinterpret_cast<const uint32_t*>(row + d)) : 0u;
                if constexpr (T::KV == kFP8 && T::IO == kBF16) {
                    // pages compute in f16: convert the bf16 query pair
                    v = pack2<false>(bf16_bits_to_f32(v & 0xFFFFu), bf16_bits_to_f32(v >> 16));
                }
                qf[nt][kt][hf] = v;
            }
        }
    }
}

// Write the new token's row (t = valid-1) of one KV head into HBM and into the
// staged page.  One warp; each lane owns D/32 consecutive elements.
template <class T>
__device__ __forceinline__ void append_row(const DecodeParams& p, uint8_t* stage, int b, int h,
                                           uint32_t blk, int t, int lane) {
    constexpr int PER = T::D / 32;    // 2 (D=64) or 4 (D=128)
    const bool blk_ok = blk < p.num_blocks;
    if (!blk_ok && lane == 0) set_err(p.err, kDevErrBlockId);
#pragma unroll
    for (int kv = 0; kv < 2; ++kv) {
        const uint16_t* src = reinterpret_cast<const uint16_t*>(kv == 0 ? p.k_new : p.v_new) +
                              ((size_t)b * p.Hkv + h) * T::D + lane * PER;
        const size_t row = (((size_t)p.layer * p.num_blocks + blk) * 2 + kv) * p.Hkv + h;
        uint8_t* tile = stage + kv * T::TILE;
        if constexpr (T::KV != kFP8) {
            uint32_t w[PER / 2];
#pragma unroll
            for (int k = 0; k < PER / 2; ++k) w[k] = __ldg(reinterpret_cast<const uint32_t*>(src) + k);
            uint8_t* gdst = p.kv_data + (row * 16 + t) * T::ROW + lane * PER * 2;
            uint8_t* sdst = tile + swz16(t, lane * PER);
            if constexpr (PER == 4) {
                if (blk_ok) *reinterpret_cast<uint2*>(gdst) = make_uint2(w[0], w[1]);
                *reinterpret_cast<uint2*>(sdst) = make_uint2(w[0], w[1]);
            } else {
                if (blk_ok) *reinterpret_cast<uint32_t*>(gdst) = w[0];
                *reinterpret_cast<uint32_t*>(sdst) = w[0];
            }
        } else {
            static_assert(T::D == 128, "FP8 pools need head_dim 128");
            uint2 raw = __ldg(reinterpret_cast<const uint2*>(src));
            float v[4] = {io_to_f32<T::IO>(raw.x & 0xFFFFu), io_to_f32<T::IO>(raw.x >> 16),
                          io_to_f32<T::IO>(raw.y & 0xFFFFu), io_to_f32<T::IO>(raw.y >> 16)};
            float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
            for (int off = 16; off > 0; off >>= 1)
                amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
            const float scale = fp8_row_scale(amax);
            const uint32_t codes = fp8_encode4(v, scale, p.fp8_ocp != 0);
            uint8_t* gdst = p.kv_data + (row * 16 + t) * T::ROW + lane * 4;
            if (blk_ok) *reinterpret_cast<uint32_t*>(gdst) = codes;
            *reinterpret_cast<uint32_t*>(tile + swz8(t, lane * 4)) = codes;
            if (lane == 0) {
                if (blk_ok) p.kv_scales[row * 16 + t] = scale;
                reinterpret_cast<float*>(stage + 2 * T::TILE)[kv * 16 + t] = scale;
            }
        }
    }
}

// Zero V rows [valid, 16) of a staged page so masked tokens cannot inject
// NaN/Inf through 0 * garbage in the P.V product.
template <class T>
__device__ __forceinline__ void zero_tail(uint8_t* stage, int valid, int lane) {
    uint8_t* vt = stage + T::TILE;
    const int per_row = T::ROW / 16;                 // 16-B pieces per row
    const int total = (16 - valid) * per_row;
    for (int k = lane; k < total; k += 32) {
        const int t = valid + k / per_row, piece = k % per_row;
        const int c = piece >> 3, ch = piece & 7;
        *reinterpret_cast<uint4*>(vt + c * 2048 + t * 128 + (ch << 4)) = make_uint4(0, 0, 0, 0);
    }
}

// FP8: expand the staged K and V code tiles into this warp's f16 tiles.
template <class T>
__device__ __forceinline__ void dequant_page(const uint8_t* stage, uint8_t* ctile, int lane) {
#pragma unroll
    for (int kv = 0; kv < 2; ++kv) {
        const uint8_t* src = stage + kv * T::TILE;
        uint8_t* dst = ctile + kv * T::CTILE;
#pragma unroll
        for (int it = 0; it < 4; ++it) {
            const int t = it * 4 + (lane >> 3), c16 = lane & 7;
            const uint4 w = *reinterpret_cast<const uint4*>(src + t * 128 + ((c16 ^ (t & 7)) << 4));
            uint4 lo, hi;
            lo.x = fp8x2_to_f16x2_scaled(w.x, 0); lo.y = fp8x2_to_f16x2_scaled(w.x, 1);
            lo.z = fp8x2_to_f16x2_scaled(w.y, 0); lo.w = fp8x2_to_f16x2_scaled(w.y, 1);
            hi.x = fp8x2_to_f16x2_scaled(w.z, 0); hi.y = fp8x2_to_f16x2_scaled(w.z, 1);
            hi.z = fp8x2_to_f16x2_scaled(w.w, 0); hi.w = fp8x2_to_f16x2_scaled(w.w, 1);
            *reinterpret_cast<uint4*>(dst + swz16(t, c16 * 16)) = lo;
            *reinterpret_cast<uint4*>(dst + swz16(t, c16 * 16 + 8)) = hi;
        }
    }
}

template <class T>
__device__ void consumer(const DecodeParams& p, const Smem& sm, int begin, int end, int per_cta,
                         uint64_t deadline) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ctid = threadIdx.x;                     // 0 .. W*32-1
    const int Hkv = (int)p.Hkv;
    const int W = kConsumerWarps;
    const bool append = p.k_new != nullptr;

    // ldmatrix lane geometry (see the fragment layout notes at the top)
    const int mi = lane >> 3;
    const int k_tok = (lane & 7) + ((mi & 1) << 3), k_hs = mi >> 1;
    const int v_tok = (lane & 7) + ((mi >> 1) << 3), v_hs = mi & 1;
    const int t0 = lane >> 2, t1 = t0 + 8;

    uint8_t* my_ctile = sm.ctile + warp * 2 * T::CTILE;
    bool alive = true;

    for (int x = begin; x < end;) {
        const int b = find_seq(sm.pfx, (int)p.B, Hkv, x);
        const int np = sm.pfx[b + 1] - sm.pfx[b];
        const int seg_start = Hkv * sm.pfx[b] + 0;
        const int r = x - seg_start;
        const int h = r / np, pg0 = r - h * np;
        const int s_begin = seg_start + h * np;       // flat index of this segment's page 0
        const int cnt = min(np - pg0, end - x);
        const bool complete = pg0 == 0 && cnt == np;
        const int i_base = x - begin;
        const int seq_len = (int)__ldg(p.seq_lens + b);

        uint32_t qf[T::NT][T::KT][2];
        load_q<T>(p, b, h, lane, qf);

        float o[T::NT][T::MT][4];
        float mrun[T::NT][2], lrun[T::NT][2];
#pragma unroll
        for (int nt = 0; nt < T::NT; ++nt) {
            mrun[nt][0] = mrun[nt][1] = -INFINITY;
            lrun[nt][0] = lrun[nt][1] = 0.0f;
#pragma unroll
            for (int mt = 0; mt < T::MT; ++mt) o[nt][mt][0] = o[nt][mt][1] = o[nt][mt][2] = o[nt][mt][3] = 0.0f;
        }

        const int first_i = i_base + ((warp - i_base) % W + W) % W;
        for (int i = first_i; i < i_base + cnt && alive; i += W) {
            const int pg = pg0 + (i - i_base);
            const int s = i % T::S;
            uint8_t* st = sm.stages + s * T::STAGE;
            if (!mbar_wait(&sm.full[s], (i / T::S) & 1, deadline)) {
                if (lane == 0) set_err(p.err, kDevErrTimeout);
                alive = false;
                break;
            }
            int valid = 16;
            if (pg == np - 1) {
                valid = seq_len - pg * 16;
                if (append) {
                    const uint32_t blk = __ldg(p.block_tables + (size_t)b * p.bt_stride + pg);
                    append_row<T>(p, st, b, h, blk, valid - 1, lane);
                }
                if (valid < 16) zero_tail<T>(st, valid, lane);
                // plain stores into a TMA-filled stage: order them before the stage's
                // next asynchronous (TMA) write, which follows the empty arrive below
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
            }
            const float* kscale = reinterpret_cast<const float*>(st + 2 * T::TILE);
            float ks0 = 1.0f, ks1 = 1.0f, vs0 = 1.0f, vs1 = 1.0f;
            uint32_t kbase, vbase;
            if constexpr (T::KV == kFP8) {
                ks0 = kscale[t0] * 256.0f; ks1 = kscale[t1] * 256.0f;
                vs0 = kscale[16 + t0] * 256.0f; vs1 = kscale[16 + t1] * 256.0f;
                dequant_page<T>(st, my_ctile, lane);
                __syncwarp();
                if (lane == 0) mbar_arrive(&sm.empty[s]);   // stage no longer needed
                kbase = smem_u32(my_ctile);
                vbase = smem_u32(my_ctile + T::CTILE);
            } else {
                kbase = smem_u32(st);
                vbase = smem_u32(st + T::TILE);
            }

            // ---- S^T = K Q^T  (16 tokens x 8*NT heads)
            float sacc[T::NT][4];
#pragma unroll
            for (int nt = 0; nt < T::NT; ++nt) sacc[nt][0] = sacc[nt][1] = sacc[nt][2] = sacc[nt][3] = 0.0f;
#pragma unroll
            for (int kt = 0; kt < T::KT; ++kt) {
                uint32_t a0, a1, a2, a3;
                const uint32_t addr = kbase + (kt >> 2) * 2048 + k_tok * 128 +
                                      ((((kt & 3) * 2 + k_hs) ^ (k_tok & 7)) << 4);
                ldsm_x4(addr, a0, a1, a2, a3);
#pragma unroll
                for (int nt = 0; nt < T::NT; ++nt)
                    mma_16816<T::MMA_BF16>(sacc[nt], a0, a1, a2, a3, qf[nt][kt][0], qf[nt][kt][1]);
            }

            // ---- online softmax (log2 domain), P^T fragments via movmatrix
            uint32_t pb[T::NT][2];
            const bool v0 = t0 < valid, v1 = t1 < valid;
#pragma unroll
            for (int nt = 0; nt < T::NT; ++nt) {
                float s00 = v0 ? sacc[nt][0] * p.scale_log2 * ks0 : -INFINITY;
                float s01 = v0 ? sacc[nt][1] * p.scale_log2 * ks0 : -INFINITY;
                float s10 = v1 ? sacc[nt][2] * p.scale_log2 * ks1 : -INFINITY;
                float s11 = v1 ? sacc[nt][3] * p.scale_log2 * ks1 : -INFINITY;
                float mx0 = fmaxf(s00, s10), mx1 = fmaxf(s01, s11);
#pragma unroll
                for (int off = 4; off < 32; off <<= 1) {
                    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
                    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
                }
                const float mn0 = fmaxf(mrun[nt][0], mx0), mn1 = fmaxf(mrun[nt][1], mx1);
                const float al0 = ex2(mrun[nt][0] - mn0), al1 = ex2(mrun[nt][1] - mn1);
                mrun[nt][0] = mn0; mrun[nt][1] = mn1;
                const float p00 = ex2(s00 - mn0), p01 = ex2(s01 - mn1);
                const float p10 = ex2(s10 - mn0), p11 = ex2(s11 - mn1);
                lrun[nt][0] = lrun[nt][0] * al0 + (p00 + p10);
                lrun[nt][1] = lrun[nt][1] * al1 + (p01 + p11);
#pragma unroll
                for (int mt = 0; mt < T::MT; ++mt) {
                    o[nt][mt][0] *= al0; o[nt][mt][1] *= al1;
                    o[nt][mt][2] *= al0; o[nt][mt][3] *= al1;
                }
                float q00 = p00, q01 = p01, q10 = p10, q11 = p11;
                if constexpr (T::KV == kFP8) {
                    q00 = v0 ? p00 * vs0 : 0.0f; q01 = v0 ? p01 * vs0 : 0.0f;
                    q10 = v1 ? p10 * vs1 : 0.0f; q11 = v1 ? p11 * vs1 : 0.0f;
                }
                pb[nt][0] = movmatrix_t(pack2<T::MMA_BF16>(q00, q01));
                pb[nt][1] = movmatrix_t(pack2<T::MMA_BF16>(q10, q11));
            }

            // ---- O^T += V^T P^T  (D x 8*NT)
#pragma unroll
            for (int mt = 0; mt < T::MT; ++mt) {
                uint32_t a0, a1, a2, a3;
                const uint32_t addr = vbase + (mt >> 2) * 2048 + v_tok * 128 +
                                      ((((mt & 3) * 2 + v_hs) ^ (v_tok & 7)) << 4);
                ldsm_x4_t(addr, a0, a1, a2, a3);
#pragma unroll
                for (int nt = 0; nt < T::NT; ++nt)
                    mma_16816<T::MMA_BF16>(o[nt][mt], a0, a1, a2, a3, pb[nt][0], pb[nt][1]);
            }
            if constexpr (T::KV != kFP8) {
                __syncwarp();
                if (lane == 0) mbar_arrive(&sm.empty[s]);
            } else {
                __syncwarp();
            }
        }

        // ---- merge the W warps' states for this segment
        if (!alive && lane == 0) sm.flag[1] = 1;  // abort marker, read by all warps below
        float* mo = sm.mo + warp * T::G * T::D;
#pragma unroll
        for (int nt = 0; nt < T::NT; ++nt) {
#pragma unroll
            for (int off = 4; off < 32; off <<= 1) {
                lrun[nt][0] += __shfl_xor_sync(0xffffffffu, lrun[nt][0], off);
                lrun[nt][1] += __shfl_xor_sync(0xffffffffu, lrun[nt][1], off);
            }
            const int j0 = nt * 8 + 2 * (lane & 3);
#pragma unroll
            for (int mt = 0; mt < T::MT; ++mt) {
                const int d = mt * 16 + (lane >> 2);
                mo[j0 * T::D + d] = o[nt][mt][0];
                mo[(j0 + 1) * T::D + d] = o[nt][mt][1];
                mo[j0 * T::D + d + 8] = o[nt][mt][2];
                mo[(j0 + 1) * T::D + d + 8] = o[nt][mt][3];
            }
            if (lane < 4) {
                sm.mm[warp * T::G + j0] = mrun[nt][0];
                sm.mm[warp * T::G + j0 + 1] = mrun[nt][1];
                sm.ml[warp * T::G + j0] = lrun[nt][0];
                sm.ml[warp * T::G + j0 + 1] = lrun[nt][1];
            }
        }
        named_bar_sync(1, W * 32);
        // every consumer warp reads the same marker after the barrier, so all of
        // them leave the segment loop together and no named barrier is orphaned
        const bool abort = sm.flag[1] != 0;

        const int g = (int)p.group;
        const int seg = b * Hkv + h;
        uint16_t* out = reinterpret_cast<uint16_t*>(p.out);
        const int slot = (x == begin) ? 0 : 1;
        float* po = p.part_o + ((size_t)blockIdx.x * 2 + slot) * T::G * T::D;
        float* pml = p.part_ml + ((size_t)blockIdx.x * 2 + slot) * T::G * 2;
        for (int idx = ctid; idx < g * T::D && !abort; idx += W * 32) {
            const int j = idx / T::D, d = idx - j * T::D;
            float M = -INFINITY;
#pragma unroll
            for (int w = 0; w < W; ++w) M = fmaxf(M, sm.mm[w * T::G + j]);
            float Ls = 0.0f, Os = 0.0f;
#pragma unroll
            for (int w = 0; w < W; ++w) {
                const float f = ex2(sm.mm[w * T::G + j] - M);
                Ls += sm.ml[w * T::G + j] * f;
                Os += sm.mo[(w * T::G + j) * T::D + d] * f;
            }
            if (complete) {
                out[((size_t)b * p.Hq + (size_t)h * g + j) * T::D + d] = f32_to_io<T::IO>(Os / Ls);
            } else {
                po[j * T::D + d] = Os;
                if (d == 0) { pml[j * 2] = M; pml[j * 2 + 1] = Ls; }
            }
        }
        if (!complete && !abort) {
            __threadfence();
            named_bar_sync(1, W * 32);
            const int c0 = s_begin / per_cta, c1 = (s_begin + np - 1) / per_cta;
            if (ctid == 0) {
                const uint32_t old = atomicAdd(p.counters + seg, 1u);
                sm.flag[0] = old == (uint32_t)(c1 - c0);
            }
            named_bar_sync(1, W * 32);
            if (sm.flag[0]) {
                __threadfence();
                for (int idx = ctid; idx < g * T::D; idx += W * 32) {
                    const int j = idx / T::D, d = idx - j * T::D;
                    float M = -INFINITY;
                    for (int c = c0; c <= c1; ++c) {
                        const int sl = (c == c0 && s_begin != c0 * per_cta) ? 1 : 0;
                        M = fmaxf(M, __ldcg(p.part_ml + (((size_t)c * 2 + sl) * T::G + j) * 2));
                    }
                    float Ls = 0.0f, Os = 0.0f;
                    for (int c = c0; c <= c1; ++c) {
                        const int sl = (c == c0 && s_begin != c0 * per_cta) ? 1 : 0;
                        const size_t base = ((size_t)c * 2 + sl) * T::G;
                        const float f = ex2(__ldcg(p.part_ml + (base + j) * 2) - M);
                        Ls += __ldcg(p.part_ml + (base + j) * 2 + 1) * f;
                        Os += __ldcg(p.part_o + (base + j) * T::D + d) * f;
                    }
                    out[((size_t)b * p.Hq + (size_t)h * g + j) * T::D + d] =
                        f32_to_io<T::IO>(Os / Ls);
                }
                if (ctid == 0) p.counters[seg] = 0u;
            }
        }
        named_bar_sync(1, W * 32);
        x += cnt;
        if (abort) break;
    }
}

template <class T>
__global__ void __launch_bounds__(kThreads, 1)
decode_kernel(const __grid_constant__ CUtensorMap tmap, const DecodeParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const Smem sm = carve<T>(base);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint64_t deadline = globaltimer() + kWaitDeadlineNs;

    if (threadIdx.x == 0) {
        for (int s = 0; s < T::S; ++s) { mbar_init(&sm.full[s], 1); mbar_init(&sm.empty[s], 1); }
        fence_mbar_init();
        sm.flag[0] = 0;
        sm.flag[1] = 0;
    }
    if (warp == kProducerWarp) {
        if (lane == 0) prefetch_tensormap(&tmap);
        // pages per sequence -> exclusive prefix (one warp, 32 sequences at a time)
        int run = 0;
        if (lane == 0) sm.pfx[0] = 0;
        for (int base_b = 0; base_b < (int)p.B; base_b += 32) {
            const int b = base_b + lane;
            int np = 0;
            if (b < (int)p.B) {
                const int sl = (int)__ldg(p.seq_lens + b);
                np = (sl + 15) >> 4;
                if (sl <= 0 || np > (int)p.bt_stride) {
                    if (blockIdx.x == 0) set_err(p.err, kDevErrSeqLen);
                    np = sl <= 0 ? 0 : (int)p.bt_stride;
                }
            }
            int incl = np;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const int v = __shfl_up_sync(0xffffffffu, incl, off);
                if (lane >= off) incl += v;
            }
            if (b < (int)p.B) sm.pfx[b + 1] = run + incl;
            run += __shfl_sync(0xffffffffu, incl, 31);
        }
    }
    __syncthreads();

    const int total = (int)p.Hkv * sm.pfx[p.B];
    int per_cta = (total + (int)gridDim.x - 1) / (int)gridDim.x;
    if (per_cta < kMinPagesPerCta) per_cta = kMinPagesPerCta;
    const int begin = (int)blockIdx.x * per_cta;
    const int end = min(total, begin + per_cta);
    if (begin >= end) return;

    if (warp == kProducerWarp) producer<T>(&tmap, p, sm, begin, end - begin, deadline);
    else consumer<T>(p, sm, begin, end, per_cta, deadline);
}

template <class T>
cudaError_t launch_t(const DecodeLaunch& L) {
    // the dynamic-smem opt-in is per device; remember it per device ordinal
    static std::atomic<uint64_t> configured{0};
    int dev = 0;
    cudaGetDevice(&dev);
    const uint64_t bit = 1ull << (dev & 63);
    if (!(configured.load() & bit)) {
        cudaError_t e = cudaFuncSetAttribute(decode_kernel<T>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, T::SMEM);
        if (e != cudaSuccess) return e;
        configured.fetch_or(bit);
    }
    decode_kernel<T><<<L.grid, kThreads, T::SMEM, L.stream>>>(*L.tmap, L.p);
    return cudaGetLastError();
}

template <int D, int KV, int IO>
cudaError_t launch_d(const DecodeLaunch& L) {
    if (L.p.group <= 8) return launch_t<Traits<D, 1, KV, IO>>(L);
    return launch_t<Traits<D, 2, KV, IO>>(L);
}

}  // namespace

size_t decode_scratch_floats_o(int grid, int head_dim) { return (size_t)grid * 2 * 16 * head_dim; }
size_t decode_scratch_floats_ml(int grid) { return (size_t)grid * 2 * 16 * 2; }

cudaError_t launch_paged_decode(const DecodeLaunch& L) {
    const uint32_t D = L.head_dim;
    if (L.kv_kind == kFP8) {
        if (D != 128) return cudaErrorInvalidValue;
        return L.io_kind == kBF16 ? launch_d<128, kFP8, kBF16>(L) : launch_d<128, kFP8, kF16>(L);
    }
    if (L.kv_kind == kBF16) {
        return D == 64 ? launch_d<64, kBF16, kBF16>(L) : launch_d<128, kBF16, kBF16>(L);
    }
    return D == 64 ? launch_d<64, kF16, kF16>(L) : launch_d<128, kF16, kF16>(L);
}

}  // namespace vw
