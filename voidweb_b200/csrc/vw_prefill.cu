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
//  * Work split.  CTA (tile, q head): 128 query tokens of one sequence for one
//    query head; the keys of the head's KV head stream through shared memory in
//    rounds of 4 page-heads (64 keys): a ring of K tiles and a ring of V tiles,
//    filled by TMA through a second tensor map of the pool (boxes of 16 rows of
//    one 128-B column), so that a round's keys have a uniform row stride.
//  * Math on the fifth-generation tensor cores (tcgen05): per round, S = Q K^T
//    with M = 128 query rows and N = 64 keys (A = the query tile, B = the K
//    tile, both 128-B-swizzled K-major shared-memory operands), accumulated in
//    tensor memory; four softmax warps (one query row per thread, no shuffles)
//    read S, apply the causal / length mask and an online softmax with a
//    lazily raised maximum, and write P back to tensor memory over S; then
//    O += P V per page-head with P from tensor memory and the V tile as an
//    MN-major operand (M = 128, N = head_dim, K = 16 keys).  O stays in tensor
//    memory until the epilogue.  bf16 probabilities are written as a bf16 pair
//    hi + lo (two PV MMAs) so that P keeps ~2^-18 relative precision.
//  * FP8 pools: decoder warps expand the codes into the same f16 tiles; the
//    softmax applies the per-token K and V scales.
//  * Every wait is bounded; on timeout the kernel records kDevErrTimeout,
//    drains its TMA loads and returns.

// The prefill's barrier waits keep the hardware's own suspend limit: with a
// 200 ns hint the FP8 prefill measured 332 against 339 TFLOP/s and the bf16
// one 590 against 593 (the decode gains from the hint).
#define VW_MBAR_SUSPEND_HINT_NS 0
#include <cuda.h>
#include <cuda_runtime.h>
#include <atomic>
#include <cstdint>

#include "vw_fp8.cuh"
#include "vw_internal.h"
#include "vw_ptx.cuh"
#include "vw_rope.cuh"
#include "vw_tc.cuh"

namespace vw {

namespace {

constexpr int pf_align(int x, int a) { return (x + a - 1) / a * a; }

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

// Largest b in [0, B) with cu_q[b] <= i (cu_q non-decreasing, cu_q[0] <= i),
// by the whole warp: each round the 32 lanes probe 32 evenly spaced offsets of
// the remaining range at once and keep the bracket the last true probe starts,
// so B <= 32 takes one round of loads and B <= 1024 two (a binary search by
// one lane is a chain of log2(B) dependent loads).  Every lane gets the result.
__device__ __forceinline__ int pf_find_warp(const int32_t* cu_q, int B, int i, int lane) {
    int lo = 0, n = B;
    while (n > 1) {
        const int step = (n + 31) / 32;
        const int idx = lo + lane * step;
        const bool ok = idx < lo + n && __ldg(cu_q + idx) <= i;
        const uint32_t m = __ballot_sync(0xffffffffu, ok);      // lanes 0 .. k (monotone)
        const int k = 31 - __clz((int)m);                         // lane 0 is always true
        const int nlo = lo + k * step;
        n = min(step, lo + n - nlo);
        lo = nlo;
    }
    return lo;
}

// ------------------------------------------------------------------ append

// One warp per token i: its K and V rows of every KV head go to slot
// block_tables[b][p/16]*16 + p%16, p = ctx_start[b] + i - cu_q[b] (the paging
// rule of flash_attention.bm:132-140).  The token's sequence, position and
// block are resolved once for all its heads, and the rows of four heads are
// loaded before any is stored, so a warp keeps eight rows in flight behind one
// chain of dependent lookups.  With rope_theta > 0 the K row is rotated at
// position p first (lane l holds elements l*D/32 .. +D/32-1, whose partners
// d +- D/2 lane l ^ 16 holds), rounded to the io type as a separate RoPE pass
// would.  FP8 pools quantise each row with its own scale (the decode's codec).
constexpr uint32_t kAppendHeadGroup = 4;

__global__ void __launch_bounds__(256) prefill_append_kernel(
    PoolGeom g, uint8_t* __restrict__ data, float* __restrict__ scales, uint32_t layer,
    const uint16_t* __restrict__ k_new, const uint16_t* __restrict__ v_new,
    const int32_t* __restrict__ cu_q, const int32_t* __restrict__ ctx_start,
    const uint32_t* __restrict__ block_tables, uint32_t bt_stride, uint32_t B, uint32_t T,
    float rope_theta, uint32_t* err) {
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t i = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);   // token (T <= 2^24)
    if (i >= T || (int)i >= __ldg(cu_q + B)) return;      // past the last chunk
    const int b = pf_find_warp(cu_q, (int)B, (int)i, (int)lane);
    const int p = __ldg(ctx_start + b) + ((int)i - __ldg(cu_q + b));
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
    const uint32_t Hkv = g.num_kv_heads;
    const float pos = (float)p;
    for (uint32_t h0 = 0; h0 < Hkv; h0 += kAppendHeadGroup) {
        uint32_t w[kAppendHeadGroup][2][2];
#pragma unroll
        for (uint32_t hh = 0; hh < kAppendHeadGroup; ++hh)
#pragma unroll
            for (uint32_t kv = 0; kv < 2; ++kv) {
                w[hh][kv][0] = w[hh][kv][1] = 0u;
                if (h0 + hh >= Hkv) continue;
                const uint16_t* src = (kv == 0 ? k_new : v_new) + ((size_t)i * Hkv + h0 + hh) * D + lane * PER;
                w[hh][kv][0] = __ldg(reinterpret_cast<const uint32_t*>(src));
                if (PER == 4) w[hh][kv][1] = __ldg(reinterpret_cast<const uint32_t*>(src + 2));
            }
#pragma unroll
        for (uint32_t hh = 0; hh < kAppendHeadGroup; ++hh) {
            const uint32_t h = h0 + hh;
            if (h >= Hkv) break;
#pragma unroll
            for (uint32_t kv = 0; kv < 2; ++kv) {
                uint32_t* w2 = w[hh][kv];
                if (kv == 0 && rope_theta > 0.0f) {
                    const bool lo = lane < 16;
#pragma unroll
                    for (uint32_t k = 0; k < 2; ++k) {        // PER / 2 words (static indices)
                        if (k >= PER / 2) break;
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
                const uint64_t row = ((((uint64_t)layer * g.num_blocks + blk) * Hkv + h) * 2 + kv) *
                                         kBlockSize + (uint32_t)p % kBlockSize;
                if (g.kv_kind != kFP8) {
                    uint8_t* dst = data + row * D * 2 + lane * PER * 2;
                    if (PER == 4) *reinterpret_cast<uint2*>(dst) = make_uint2(w2[0], w2[1]);
                    else *reinterpret_cast<uint32_t*>(dst) = w2[0];
                } else {
                    // FP8 pools have head_dim 128: four elements per lane
                    float v[4];
#pragma unroll
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
    }
}

// ------------------------------------------------------------------ attention

constexpr int kTcRows = 128;                      // query tokens per CTA: the MMA's M
constexpr int kTcPages = 4;                       // page-heads per round (16 keys each)
constexpr float kTcRescale = 8.0f;                // log2 units: p <= 2^8 against a stale max

template <int D_, int IO_, int KV_>
struct TcTraits {
    static constexpr int D = D_, IO = IO_;
    static constexpr bool BF = IO == kBF16;
    // FP8 pools: decoder warps expand the codes into f16 tiles (code b -> the
    // binary16 value decode(b)/256, exact), so the MMAs run in f16 whatever the
    // io type; the factor 256 returns through the K scales and the output
    static constexpr bool FP8 = KV_ == kFP8;
    static constexpr bool MBF = BF && !FP8;           // the MMAs' operand type is bf16
    // P as a pair hi + lo of the MMA type (two PV MMAs): bf16 pages, and FP8
    // pages whose f16 P carries the V scales
    static constexpr bool PSPLIT = BF || FP8;
    static constexpr float VFOLD = FP8 ? 256.0f : 1.0f;
    static constexpr int NDEC = FP8 ? 2 : 0;          // decoder warps (FP8 pools)
    static constexpr int CH = D * 2 / 128;            // 128-B columns of a row
    static constexpr int R = kTcPages;                // page-heads per round
    static constexpr int KEYS = 16 * R;               // keys per round: the N of S = Q K^T
    // round stages: the K rows and the V rows of a round's page-heads, each a tile
    // [CH][KEYS rows][128 B] (128-B swizzled), in a ring of NSTK K tiles and a
    // ring of NSTV V tiles.  A K tile frees when S of its round completes, two
    // rounds before the V tile of that round: with f16/bf16 pages at head_dim
    // 128 the K ring is one deeper, which is what shared memory holds with two
    // CTAs per SM (what tensor memory allows); head_dim 64 keeps 4 + 4.
    static constexpr int NST = D == 128 ? 2 : 4;
    static constexpr int NSTK = (D == 128 && !FP8) ? 3 : NST;
    static constexpr int NSTV = NST;
    static constexpr int TILE = CH * KEYS * 128;      // bytes of one K (or V) tile
    static constexpr int HALF_BOX = 16 * 128;         // one TMA box: 16 rows of one column
    static constexpr int QBYTES = kTcRows * D * 2;    // query tile [CH][128 rows][128 B]
    static constexpr int KSTEPS = D / 16;             // MMAs of S = Q K^T per round
    // tensor memory: O in columns [0, D); two S buffers of KEYS f32 columns.  P
    // (bf16/f16 pairs: KEYS/2 columns, then KEYS/2 for the low part of bf16
    // probabilities) is written over the S buffer it was computed from.
    static constexpr int COL_S = D;
    static constexpr uint32_t TMEM_COLS = 256u;       // two CTAs per SM share the 512 columns
    // the query tiles' prefix over the batch, read only in the prologue: it
    // lives in the last V tile, which nothing writes before the prologue ends
    static constexpr int TPFX = pf_align((kMaxBatchPerLaunch + 1) * 4, 128);
    // FP8 pools: per stage the round's K scales (x256), then its V scales
    static constexpr int SCL = FP8 ? NST * 2 * KEYS * 4 : 0;
    // full_k, empty_k per K tile, full_v, empty_v per V tile; s_full/p_full/p_free
    // x2; done
    static constexpr int NBAR = 2 * NSTK + 2 * NSTV + 7;
    // the dynamic shared memory starts 1024-B aligned on B200 (checked at run
    // time: the kernel flags kDevErrLaunch and returns otherwise)
    static constexpr int SMEM = QBYTES + (NSTK + NSTV) * TILE + SCL + NBAR * 8 + 16;
    // 4 softmax warps, 1 MMA warp, then 2 TMA producer warps (K tiles, V tiles)
    // or NDEC decoder warps
    static constexpr int THREADS = (FP8 ? 5 + NDEC : 7) * 32;
    static constexpr uint32_t IDESC_S = idesc_f16(MBF, false, kTcRows, KEYS);
    static constexpr uint32_t IDESC_PV = idesc_f16(MBF, true, kTcRows, D);
    static_assert(D == 64 || D == 128, "head_dim 64 or 128");
    static_assert(!FP8 || D == 128, "FP8 pools have head_dim 128");
    static_assert(!FP8 || NDEC * 32 == KEYS, "one decoder thread per key of a round (scales)");
    static_assert(!FP8 || NSTK == NSTV, "FP8 decoders fill a round's K and V tiles together");
    static_assert(TPFX <= TILE, "the tile prefix fits in a V tile");
    static_assert(COL_S + 2 * KEYS <= (int)TMEM_COLS, "tensor-memory columns");
    static_assert(QBYTES % 1024 == 0 && TILE % 1024 == 0, "1024-B alignment");
    static_assert(2 * (SMEM + 1024) <= 233472, "two CTAs per SM");
    static_assert(3 * (SMEM + 1024) > 233472, "at most two CTAs per SM (tensor memory)");
};

// FP8 pools: the decoder warps' part of round t, in two halves so that the
// global loads of a round are in flight while the decoders wait for its stage.
// Thread dt (0 .. 63) loads 16 chunks of 16 codes (chunk i: K rows for i < 8,
// V rows after; page-head (i & 7) / 2, row (i & 1) * 8 + dt / 8, elements
// (dt % 8) * 16 ..), a warp reading 512 contiguous bytes per load, and key dt's
// K scale (x256) and V scale; then, once the stage is free, writes each chunk as
// two 16-B f16 units into the tile layout the TMA gives an f16 pool: [column]
// [KEYS rows][128 B], unit u of key row k at (u ^ (k % 8)) * 16.  Keys past the
// sequence's end, in page-heads past npages or in an out-of-range block
// (flagged) are zero rows with zero scales, so that masked probabilities meet
// no NaN.
struct Fp8RoundRegs {
    uint4 w[16];
    float ks, vs;
};

template <class T>
__device__ __forceinline__ void fp8_round_ids(const uint32_t* bt, int t, int npages, uint32_t (&blk)[T::R]) {
#pragma unroll
    for (int pg = 0; pg < T::R; ++pg) blk[pg] = t * T::R + pg < npages ? __ldg(bt + t * T::R + pg) : 0xFFFFFFFFu;
}

template <class T>
__device__ __forceinline__ void fp8_load_round(const PrefillParams& p, const uint32_t (&blk)[T::R], int t, int h,
                                               int total, int npages, int dt, Fp8RoundRegs& r) {
    if (dt == 0)
#pragma unroll
        for (int pg = 0; pg < T::R; ++pg)
            if (t * T::R + pg < npages && blk[pg] >= p.num_blocks) atomicOr(p.err, kDevErrBlockId);
    auto head_row = [&](uint32_t bj, int kv) -> size_t {   // first row of the K (kv 0) or V half
        return ((((size_t)p.layer * p.num_blocks + bj) * p.Hkv + (uint32_t)h) * 2 + kv) * kBlockSize;
    };
    const int e0 = (dt & 7) * 16;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        const int pg = (i & 7) >> 1, rr = (i & 1) * 8 + (dt >> 3);
        const bool valid = blk[pg] < p.num_blocks && t * T::KEYS + pg * 16 + rr < total;
        r.w[i] = valid ? __ldg(reinterpret_cast<const uint4*>(p.kv_data + (head_row(blk[pg], i >> 3) + rr) * T::D + e0))
                       : make_uint4(0, 0, 0, 0);
    }
    const int pg = dt >> 4, rr = dt & 15;
    const bool valid = blk[pg] < p.num_blocks && t * T::KEYS + dt < total;
    r.ks = valid ? __ldg(p.kv_scales + head_row(blk[pg], 0) + rr) * 256.0f : 0.0f;
    r.vs = valid ? __ldg(p.kv_scales + head_row(blk[pg], 1) + rr) : 0.0f;
}

template <class T>
__device__ __forceinline__ void fp8_store_round(uint8_t* kt, uint8_t* vt, float* scl, int dt,
                                                const Fp8RoundRegs& r) {
    scl[dt] = r.ks;
    scl[T::KEYS + dt] = r.vs;
    const int e0 = (dt & 7) * 16, c = e0 >> 6, ua = (e0 & 63) >> 3;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        const int key = ((i & 7) >> 1) * 16 + (i & 1) * 8 + (dt >> 3);
        uint8_t* row = (i >> 3 ? vt : kt) + c * (T::KEYS * 128) + key * 128;
        const uint4 a = make_uint4(fp8x2_to_f16x2_scaled(r.w[i].x, 0), fp8x2_to_f16x2_scaled(r.w[i].x, 1),
                                   fp8x2_to_f16x2_scaled(r.w[i].y, 0), fp8x2_to_f16x2_scaled(r.w[i].y, 1));
        const uint4 bq = make_uint4(fp8x2_to_f16x2_scaled(r.w[i].z, 0), fp8x2_to_f16x2_scaled(r.w[i].z, 1),
                                    fp8x2_to_f16x2_scaled(r.w[i].w, 0), fp8x2_to_f16x2_scaled(r.w[i].w, 1));
        *reinterpret_cast<uint4*>(row + ((ua ^ (key & 7)) << 4)) = a;
        *reinterpret_cast<uint4*>(row + (((ua + 1) ^ (key & 7)) << 4)) = bq;
    }
    // generic-proxy writes, read next by the tensor cores (async proxy)
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// CTA (tile, q head): 128 query tokens of one sequence for one query head.
//  * FP8 pools: warps 5-6 (decoders) instead of the producers: per round the
//    code rows of the R page-heads, expanded to f16 tiles (fp8_decode_round),
//    and the round's scales; the softmax scales S by the K scales and P by the
//    V scales, and the output by 256.
//  * warps 5 and 6 (producers): per round of R page-heads, warp 5 loads one TMA
//    box per 128-B column of each page-head's 16 K rows into the round's K
//    tile, warp 6 its 16 V rows into the V tile, so that the keys of the round
//    are R*16 rows with a uniform stride in both tiles.  K tiles and V tiles
//    are separate rings with their own barriers: a K tile is refilled as soon
//    as S of its round completes, rounds before the V tile of that round frees.
//  * warp 4: allocates tensor memory; one lane issues per round t
//    S_t = Q K_t^T (D/16 MMAs, M = 128, N = R*16 keys, K = 16; both operands
//    128-B-swizzled K-major shared-memory tiles) into S buffer t%2, then
//    O += P_{t-1} V_{t-1} (per page-head: M = 128, N = D, K = 16 keys; A = P
//    from tensor memory, B = the V tile rows as an MN-major operand).  S_t is
//    issued only after P_{t-2}'s MMAs completed, since P_{t-2} occupies the
//    buffer.  Commits release the round's K tile (after S), its V tile and
//    the P buffer (after P V), and last the epilogue.
//  * warps 0-3 (thread r = query row r = tensor-memory lane r): load and
//    (RoPE-)rotate the query rows into the swizzled K-major tile; per round read
//    S, mask, run the online softmax with a lazily raised maximum (O in tensor
//    memory is rescaled only when a row's maximum grows by more than 2^8) and
//    write P over S; finally read O, divide by the row sum and store the rows.
template <class T>
__global__ void __launch_bounds__(T::THREADS, 2)
prefill_kernel(const __grid_constant__ CUtensorMap tmap, const PrefillParams p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // the 128-B-swizzled tiles need 1024-B alignment; the layout has no slack
    if (smem_u32(smem_raw) & 1023u) {
        if (threadIdx.x == 0) atomicOr(p.err, kDevErrLaunch);
        return;
    }
    uint8_t* qs = smem_raw;
    uint8_t* ktiles = qs + T::QBYTES;                 // ring of NSTK K tiles
    uint8_t* vtiles = ktiles + T::NSTK * T::TILE;     // ring of NSTV V tiles
    float* scl = reinterpret_cast<float*>(vtiles + T::NSTV * T::TILE);   // FP8 scales
    int* tpfx = reinterpret_cast<int*>(vtiles + (T::NSTV - 1) * T::TILE);   // prologue only
    // K tiles and V tiles fill and drain separately: a K tile is free once
    // S = Q K^T of its round completes, a V tile only after P V
    uint64_t* full_k = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(scl) + T::SCL);
    uint64_t* empty_k = full_k + T::NSTK;
    uint64_t* full_v = empty_k + T::NSTK;
    uint64_t* empty_v = full_v + T::NSTV;
    uint64_t* s_full = empty_v + T::NSTV;
    uint64_t* p_full = s_full + 2;
    uint64_t* p_free = p_full + 2;
    uint64_t* done = p_free + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint64_t deadline = cycles() + (p.wait_cycles ? p.wait_cycles : kWaitDeadlineCycles);
    // test hook (vw_debug_set_wait_limit): no K/V tile is filled, so the MMA
    // issuer's and the softmax warps' first waits run out
    const bool withhold = p.wait_cycles != 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < T::NSTK; ++s) {
            mbar_init(&full_k[s], T::FP8 ? T::NDEC : 1);  // decoder warps, or the TMA transaction
            mbar_init(&empty_k[s], 1);
        }
        for (int s = 0; s < T::NSTV; ++s) {
            mbar_init(&full_v[s], T::FP8 ? T::NDEC : 1);
            mbar_init(&empty_v[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&s_full[b], 1);
            mbar_init(&p_full[b], 4);
            mbar_init(&p_free[b], 1);
        }
        mbar_init(done, 1);
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
                nt = n > 0 ? (n + kTcRows - 1) / kTcRows : 0;
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
    const int t0 = (x - tpfx[b]) * kTcRows;
    const int qmax = cs + min(t0 + kTcRows - 1, n - 1);          // last query position of the tile
    const int kend = p.causal ? qmax + 1 : total;                // keys [0, kend)
    const int npages = (kend + kBlockSize - 1) / kBlockSize;
    const int nrounds = (npages + T::R - 1) / T::R;
    const int j = blockIdx.y, h = j / (int)p.group;

    if (warp == 4) {
        tmem_alloc(tmem_slot, T::TMEM_COLS);
        tmem_relinquish();
    }
    if (warp < 4) {
        // query row r into the swizzled K-major tile: 16-B unit u of the row goes
        // to column u / 8, unit (u % 8) ^ (r % 8)
        const int r = threadIdx.x, tq = t0 + r;
        const bool live = tq < n;
        const uint8_t* src = reinterpret_cast<const uint8_t*>(p.q) + ((size_t)(q_off + tq) * p.Hq + j) * T::D * 2;
        constexpr int U = T::D / 8, HALF = U / 2;
#pragma unroll
        for (int u = 0; u < HALF; ++u) {
            uint4 lo = make_uint4(0, 0, 0, 0), hi = make_uint4(0, 0, 0, 0);
            if (live) {
                lo = __ldg(reinterpret_cast<const uint4*>(src + u * 16));
                hi = __ldg(reinterpret_cast<const uint4*>(src + (u + HALF) * 16));
            }
            if (p.rope_theta > 0.0f && live) {
                // pairs (d, d + D/2): element e of unit u with element e of unit u + D/16
                uint32_t a[4] = {lo.x, lo.y, lo.z, lo.w}, c[4] = {hi.x, hi.y, hi.z, hi.w};
                const float pos = (float)(cs + tq);
#pragma unroll
                for (int w = 0; w < 4; ++w) {
                    float ar = pf_io_to_f32<T::IO>(a[w] & 0xFFFFu), ai = pf_io_to_f32<T::IO>(c[w] & 0xFFFFu);
                    float br = pf_io_to_f32<T::IO>(a[w] >> 16), bi = pf_io_to_f32<T::IO>(c[w] >> 16);
                    const int d = u * 8 + 2 * w;
                    rope_pair(ar, ai, d, T::D, p.rope_theta, pos);
                    rope_pair(br, bi, d + 1, T::D, p.rope_theta, pos);
                    a[w] = (uint32_t)pf_f32_to_io<T::IO>(ar) | ((uint32_t)pf_f32_to_io<T::IO>(br) << 16);
                    c[w] = (uint32_t)pf_f32_to_io<T::IO>(ai) | ((uint32_t)pf_f32_to_io<T::IO>(bi) << 16);
                }
                lo = make_uint4(a[0], a[1], a[2], a[3]);
                hi = make_uint4(c[0], c[1], c[2], c[3]);
            }
            if constexpr (T::FP8 && T::BF) {           // FP8 pages compute in f16
                auto cv = [](uint32_t x) {
                    return pack2<false>(bf16_bits_to_f32(x & 0xFFFFu), bf16_bits_to_f32(x >> 16));
                };
                lo = make_uint4(cv(lo.x), cv(lo.y), cv(lo.z), cv(lo.w));
                hi = make_uint4(cv(hi.x), cv(hi.y), cv(hi.z), cv(hi.w));
            }
            const int u2 = u + HALF;
            *reinterpret_cast<uint4*>(qs + (u >> 3) * (kTcRows * 128) + r * 128 + (((u & 7) ^ (r & 7)) << 4)) = lo;
            *reinterpret_cast<uint4*>(qs + (u2 >> 3) * (kTcRows * 128) + r * 128 + (((u2 & 7) ^ (r & 7)) << 4)) = hi;
        }
        // generic-proxy writes, read next by the tensor cores (async proxy)
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tmem_slot;

    if (T::FP8 && warp >= 5) {
        // ---- decoders: round t into stage t % NST
        const int dt = threadIdx.x - 5 * 32;
        const uint32_t* bt = p.block_tables + (size_t)b * p.bt_stride;
        bool ok = true;
        uint32_t nblk[T::R];
        fp8_round_ids<T>(bt, 0, npages, nblk);
        for (int t = 0; t < nrounds && !withhold; ++t) {
            const int st_i = t % T::NST;
            uint32_t blk[T::R];
#pragma unroll
            for (int pg = 0; pg < T::R; ++pg) blk[pg] = nblk[pg];
            Fp8RoundRegs r;
            fp8_load_round<T>(p, blk, t, h, total, npages, dt, r);   // in flight during the wait
            fp8_round_ids<T>(bt, t + 1, npages, nblk);
            // the V tile's release follows the K tile's (P V is committed after S)
            if (t >= T::NST &&
                !__all_sync(0xffffffffu, mbar_wait(&empty_v[st_i], ((t / T::NST) - 1) & 1, deadline))) {
                ok = false;
                break;
            }
            fp8_store_round<T>(ktiles + st_i * T::TILE, vtiles + st_i * T::TILE, scl + st_i * 2 * T::KEYS, dt, r);
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&full_k[st_i]);
                mbar_arrive(&full_v[st_i]);
            }
        }
        if (!ok && lane == 0) atomicOr(p.err, kDevErrTimeout);
    } else if (warp >= 5) {
        // ---- producers: warp 5 streams the rounds' K tiles into the K ring, warp 6
        // their V tiles into the V ring, each as soon as the tile it refills is
        // free (a K tile after S of its round, a V tile only after P V).  Separate
        // warps, so that each sleeps in its own barrier wait.  The block ids come
        // in windows of 32 pages (8 rounds), one per lane; the next window is
        // loaded when the current one starts, so no copy waits for its id.
        const int kv = warp - 5;
        const int ns = kv ? T::NSTV : T::NSTK;
        uint64_t* fbar = kv ? full_v : full_k;
        uint64_t* ebar = kv ? empty_v : empty_k;
        uint8_t* tiles = kv ? vtiles : ktiles;
        const uint32_t* bt = p.block_tables + (size_t)b * p.bt_stride;
        if (lane == 0) prefetch_tensormap(&tmap);
        constexpr int WIN = 32 / T::R;                // rounds per id window
        uint32_t win = lane < npages ? __ldg(bt + lane) : 0xFFFFFFFFu;
        uint32_t nwin = 32 + lane < npages ? __ldg(bt + 32 + lane) : 0xFFFFFFFFu;
        bool ok = true;
        int issued = 0;
        for (int t = 0; t < nrounds && !withhold; ++t) {
            const int st_i = t % ns;
            if (t > 0 && t % WIN == 0) {
                win = nwin;
                const int pn = (t / WIN + 1) * 32 + lane;
                nwin = pn < npages ? __ldg(bt + pn) : 0xFFFFFFFFu;
            }
            if (t >= ns && !__all_sync(0xffffffffu, mbar_wait(&ebar[st_i], ((t / ns) - 1) & 1, deadline))) {
                ok = false;
                break;
            }
            uint64_t* fb = &fbar[st_i];
            const int pg0 = t * T::R, m = min(T::R, npages - pg0);
            if (lane == 0) mbar_arrive_expect_tx(fb, (uint32_t)(m * T::CH * T::HALF_BOX));
            __syncwarp();
            // one box per lane: lane l copies column l % CH of page-head l / CH
            // (the producers share their schedulers with the softmax warps, so
            // the round's copies go out as one warp instruction)
            const int pg = lane / T::CH, c = lane % T::CH;
            const uint32_t bj = __shfl_sync(0xffffffffu, win, (t % WIN) * T::R + (pg < T::R ? pg : 0));
            if (pg < m) {
                int row0 = -32;                          // negative rows: TMA zero-fills
                if (bj < p.num_blocks)
                    row0 = (int)(((p.layer * p.num_blocks + bj) * p.Hkv + (uint32_t)h) * 32u) + 16 * kv;
                else if (kv == 0 && c == 0)
                    atomicOr(p.err, kDevErrBlockId);
                tma_load_2d(tiles + st_i * T::TILE + c * (T::KEYS * 128) + pg * T::HALF_BOX, &tmap, fb, c * 64,
                            row0);
            }
            issued = t + 1;
        }
        if (lane == 0) {
            if (!ok) atomicOr(p.err, kDevErrTimeout);
            // drain: no TMA write may land after the CTA has exited.  The copies
            // still in flight are this warp's last ns rounds; they land in bounded
            // time, so the drain has a deadline of its own (the kernel's may have
            // run out already)
            const uint64_t drain_deadline = cycles() + kWaitDeadlineCycles;
            for (int t = issued > ns ? issued - ns : 0; t < issued; ++t)
                if (!mbar_wait(&fbar[t % ns], (t / ns) & 1, drain_deadline)) {
                    atomicOr(p.err, kDevErrTimeout);
                    break;
                }
        }
    } else if (warp == 4) {
        // ---- MMA issuer
        if (lane == 0) {
            bool ok = true;
            // descriptors: the query tile's per k-step (fixed), and per stage a base
            // to which a k-step adds (kk / 4) * column + (kk % 4) * 32 bytes (>> 4 in
            // the address field, which never carries: shared memory ends below 256 KB)
            uint64_t qdesc[T::KSTEPS];
#pragma unroll
            for (int kk = 0; kk < T::KSTEPS; ++kk)
                qdesc[kk] = smem_desc_sw128(smem_u32(qs) + (kk >> 2) * (kTcRows * 128) + (kk & 3) * 32, 16, 1024);
            // K tile: K-major, 8-key groups 1024 B apart; V tile: MN-major, 64-element
            // columns KEYS*128 B apart, 8-key groups 1024 B apart
            const uint64_t kdesc0 = smem_desc_sw128(smem_u32(ktiles), 16, 1024);
            const uint64_t vdesc0 = smem_desc_sw128(smem_u32(vtiles), T::KEYS * 128, 1024);
            auto issue_pv = [&](int t) -> bool {
                const int bb = t & 1, st_i = t % T::NSTV;
                if (!mbar_wait(&p_full[bb], (t >> 1) & 1, deadline)) return false;
                if (!mbar_wait(&full_v[st_i], (t / T::NSTV) & 1, deadline)) return false;
                const int keyl = total - t * T::KEYS;   // keys of the round inside the sequence
                if (!T::FP8 && keyl < T::KEYS && keyl > 0 && (keyl & 15)) {
                    // the page-head holding the sequence's last key: its V rows past
                    // the end hold whatever the pool has there; zero them so that
                    // masked probabilities cannot meet NaN or Inf
                    uint8_t* vt = vtiles + st_i * T::TILE;
                    for (int c = 0; c < T::CH; ++c)
                        for (int row = keyl; row < ((keyl + 15) & ~15); ++row)
                            for (int u = 0; u < 8; ++u)
                                *reinterpret_cast<uint4*>(vt + c * (T::KEYS * 128) + row * 128 + u * 16) =
                                    make_uint4(0, 0, 0, 0);
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                }
                tc_fence_after();
                const uint32_t pcol = tbase + T::COL_S + T::KEYS * bb;
                const uint64_t vst = vdesc0 + (uint64_t)((st_i * T::TILE) >> 4);
                for (int pg = 0; pg < T::R && t * T::R + pg < npages; ++pg) {
                    const uint64_t vdesc = vst + (uint64_t)((pg * T::HALF_BOX) >> 4);
                    tc_mma_ts(tbase, pcol + 8 * pg, vdesc, T::IDESC_PV, (t > 0 || pg > 0) ? 1u : 0u);
                    if constexpr (T::PSPLIT) tc_mma_ts(tbase, pcol + T::KEYS / 2 + 8 * pg, vdesc, T::IDESC_PV, 1u);
                }
                tc_commit(&empty_v[st_i]);
                tc_commit(&p_free[bb]);
                return true;
            };
            for (int t = 0; t < nrounds && ok; ++t) {
                const int bb = t & 1, st_i = t % T::NSTK;
                if (!mbar_wait(&full_k[st_i], (t / T::NSTK) & 1, deadline)) { ok = false; break; }
                // buffer bb holds P_{t-2} until its MMAs complete
                if (t >= 2 && !mbar_wait(&p_free[bb], ((t - 2) >> 1) & 1, deadline)) { ok = false; break; }
                tc_fence_after();
                const uint64_t kst = kdesc0 + (uint64_t)((st_i * T::TILE) >> 4);
                const uint32_t dcol = tbase + T::COL_S + T::KEYS * bb;
#pragma unroll
                for (int kk = 0; kk < T::KSTEPS; ++kk)
                    tc_mma_ss(dcol, qdesc[kk], kst + (uint64_t)(((kk >> 2) * (T::KEYS * 128) + (kk & 3) * 32) >> 4),
                              T::IDESC_S, kk > 0 ? 1u : 0u);
                tc_commit(&empty_k[st_i]);
                tc_commit(&s_full[bb]);
                if (t >= 1 && !issue_pv(t - 1)) { ok = false; break; }
            }
            if (ok && nrounds > 0) ok = issue_pv(nrounds - 1);
            if (!ok) atomicOr(p.err, kDevErrTimeout);
            // every MMA issued here completes before the epilogue reads O and
            // before the tensor memory is freed: the issued MMAs finish in bounded
            // time, so this wait has a deadline of its own (after a timeout the
            // kernel's may have run out)
            tc_commit(done);
            if (!mbar_wait(done, 0, cycles() + kWaitDeadlineCycles)) atomicOr(p.err, kDevErrTimeout);
        }
    } else {
        // ---- softmax warps: thread r owns query row r
        const int r = threadIdx.x, tq = t0 + r;
        const bool live = tq < n;
        const int kend_r = live ? (p.causal ? cs + tq + 1 : total) : 0;
        const uint32_t lanes = (uint32_t)(warp * 32) << 16;
        float m_ref = -INFINITY, l = 0.0f;
        bool ok = true;
        for (int t = 0; t < nrounds; ++t) {
            const int bb = t & 1;
            if (!__all_sync(0xffffffffu, mbar_wait(&s_full[bb], (t >> 1) & 1, deadline))) { ok = false; break; }
            const int st_i = t % T::NST;
            // FP8: the decoders' scales of the round (their writes precede the
            // K tile's full barrier; FP8 rings have NSTK == NSTV == NST)
            if (T::FP8 && !__all_sync(0xffffffffu, mbar_wait(&full_k[st_i], (t / T::NST) & 1, deadline))) {
                ok = false;
                break;
            }
            const float* ksc = scl + st_i * 2 * T::KEYS;
            tc_fence_after();
            float xs[T::KEYS];
            {
                uint32_t sr[16];
#pragma unroll
                for (int c16 = 0; c16 < T::KEYS / 16; ++c16) {
                    tmem_ld16(tbase + lanes + T::COL_S + T::KEYS * bb + 16 * c16, sr);
                    tmem_wait_ld();
#pragma unroll
                    for (int k = 0; k < 16; ++k) xs[16 * c16 + k] = __uint_as_float(sr[k]);
                }
            }
            if constexpr (T::FP8) {
#pragma unroll
                for (int k4 = 0; k4 < T::KEYS / 4; ++k4) {
                    const float4 f = *reinterpret_cast<const float4*>(ksc + 4 * k4);
                    xs[4 * k4] *= f.x; xs[4 * k4 + 1] *= f.y; xs[4 * k4 + 2] *= f.z; xs[4 * k4 + 3] *= f.w;
                }
            }
            // keys of page-heads past npages are stale rows; they lie past kend_r.
            // Scores stay unscaled here (scale > 0 keeps the order); the scale is
            // folded into the exponent below.
            const int key0 = t * T::KEYS;
            float tmax = -INFINITY;
            if (__all_sync(0xffffffffu, key0 + T::KEYS <= kend_r)) {
#pragma unroll
                for (int k = 0; k < T::KEYS; ++k) tmax = fmaxf(tmax, xs[k]);
            } else {
#pragma unroll
                for (int k = 0; k < T::KEYS; ++k) {
                    xs[k] = key0 + k < kend_r ? xs[k] : -INFINITY;
                    tmax = fmaxf(tmax, xs[k]);
                }
            }
            tmax *= p.scale_log2;
            const bool need = tmax > m_ref + kTcRescale;
            float alpha = 1.0f;
            if (need) {
                alpha = ex2(m_ref - tmax);      // 0 while the row had no key
                m_ref = tmax;
            }
            if (__any_sync(0xffffffffu, need && t > 0)) {
                // rescale O: after PV(t-1) (whose phase is the next of its buffer:
                // S_t was issued after PV(t-2) completed), before PV(t)
                if (!__all_sync(0xffffffffu, mbar_wait(&p_free[bb ^ 1], ((t - 1) >> 1) & 1, deadline))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
#pragma unroll 1
                for (int c0 = 0; c0 < T::D; c0 += 16) {
                    uint32_t o16[16];
                    tmem_ld16(tbase + lanes + c0, o16);
                    tmem_wait_ld();
#pragma unroll
                    for (int k = 0; k < 16; ++k) o16[k] = __float_as_uint(__uint_as_float(o16[k]) * alpha);
                    tmem_st16(tbase + lanes + c0, o16);
                }
            }
            l *= alpha;
            const float mu = m_ref == -INFINITY ? 0.0f : m_ref;
            float ls = 0.0f;
#pragma unroll
            for (int c8 = 0; c8 < T::KEYS / 16; ++c8) {
                uint32_t ph[8], pl[8];
                float vsc[16];
                if constexpr (T::FP8) {                 // P carries the V scales (f16 P V)
#pragma unroll
                    for (int k4 = 0; k4 < 4; ++k4) {
                        const float4 f = *reinterpret_cast<const float4*>(ksc + T::KEYS + 16 * c8 + 4 * k4);
                        vsc[4 * k4] = f.x; vsc[4 * k4 + 1] = f.y; vsc[4 * k4 + 2] = f.z; vsc[4 * k4 + 3] = f.w;
                    }
                }
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    const float p0 = ex2(fmaf(xs[16 * c8 + 2 * k], p.scale_log2, -mu));
                    const float p1 = ex2(fmaf(xs[16 * c8 + 2 * k + 1], p.scale_log2, -mu));
                    ls += p0 + p1;
                    if constexpr (T::FP8) {
                        const float a0 = p0 * vsc[2 * k], a1 = p1 * vsc[2 * k + 1];
                        ph[k] = pack2<false>(a0, a1);
                        pl[k] = pack2<false>(a0 - f16_bits_to_f32(ph[k] & 0xFFFFu), a1 - f16_bits_to_f32(ph[k] >> 16));
                    } else {
                        ph[k] = pack2<T::BF>(p0, p1);
                        pl[k] = T::BF ? pack2<true>(p0 - bf16_bits_to_f32(ph[k] & 0xFFFFu),
                                                    p1 - bf16_bits_to_f32(ph[k] >> 16))
                                      : 0u;
                    }
                }
                tmem_st8(tbase + lanes + T::COL_S + T::KEYS * bb + 8 * c8, ph);
                if constexpr (T::PSPLIT) tmem_st8(tbase + lanes + T::COL_S + T::KEYS * bb + T::KEYS / 2 + 8 * c8, pl);
            }
            l += ls;
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[bb]);
        }
        // epilogue: O / l, after the last PV
        if (ok && __all_sync(0xffffffffu, mbar_wait(done, 0, deadline))) {
            tc_fence_after();
            const float inv = l > 0.0f ? T::VFOLD / l : 0.0f;
            uint8_t* dst = reinterpret_cast<uint8_t*>(p.out) + ((size_t)(q_off + tq) * p.Hq + j) * T::D * 2;
#pragma unroll 1
            for (int c0 = 0; c0 < T::D; c0 += 16) {
                uint32_t o16[16];
                tmem_ld16(tbase + lanes + c0, o16);
                tmem_wait_ld();
                uint32_t w[8];
#pragma unroll
                for (int k = 0; k < 8; ++k)
                    w[k] = (uint32_t)pf_f32_to_io<T::IO>(__uint_as_float(o16[2 * k]) * inv) |
                           ((uint32_t)pf_f32_to_io<T::IO>(__uint_as_float(o16[2 * k + 1]) * inv) << 16);
                if (live) {
                    *reinterpret_cast<uint4*>(dst + c0 * 2) = make_uint4(w[0], w[1], w[2], w[3]);
                    *reinterpret_cast<uint4*>(dst + c0 * 2 + 16) = make_uint4(w[4], w[5], w[6], w[7]);
                }
            }
        } else if (lane == 0) {
            atomicOr(p.err, kDevErrTimeout);
        }
    }
    // tensor memory is freed by the warp that allocated it, after every use
    tc_fence_before();
    __syncthreads();
    if (warp == 4) {
        tc_fence_after();
        tmem_dealloc(tbase, T::TMEM_COLS);
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
    // an upper bound on the query tiles: sum over b of ceil(n_b / 128) <= T / 128 + B
    const uint32_t tiles = (p.T + kTcRows - 1) / kTcRows + p.B;
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

int prefill_query_tile() { return kTcRows; }

cudaError_t launch_paged_prefill(const PrefillLaunch& L) {
    if (L.kv_kind == kFP8) {
        if (L.head_dim != 128) return cudaErrorNotSupported;
        return L.io_kind == kBF16 ? launch_t<TcTraits<128, kBF16, kFP8>>(L)
                                  : launch_t<TcTraits<128, kF16, kFP8>>(L);
    }
    if (L.head_dim == 128)
        return L.io_kind == kBF16 ? launch_t<TcTraits<128, kBF16, kBF16>>(L)
                                  : launch_t<TcTraits<128, kF16, kF16>>(L);
    if (L.head_dim == 64)
        return L.io_kind == kBF16 ? launch_t<TcTraits<64, kBF16, kBF16>>(L) : launch_t<TcTraits<64, kF16, kF16>>(L);
    return cudaErrorNotSupported;
}

cudaError_t launch_prefill_append(const PoolGeom& g, uint8_t* data, float* scales, uint32_t layer,
                                  const void* k_new, const void* v_new, const int32_t* cu_q,
                                  const int32_t* ctx_start, const uint32_t* block_tables,
                                  uint32_t bt_stride, uint32_t B, uint32_t T, float rope_theta,
                                  uint32_t* err, cudaStream_t s) {
    if (T == 0) return cudaSuccess;
    const uint32_t blocks = (T + 7) / 8;                // one warp per token
    prefill_append_kernel<<<blocks, 256, 0, s>>>(g, data, scales, layer,
                                                 static_cast<const uint16_t*>(k_new),
                                                 static_cast<const uint16_t*>(v_new), cu_q, ctx_start,
                                                 block_tables, bt_stride, B, T, rope_theta, err);
    return cudaGetLastError();
}

}  // namespace vw
