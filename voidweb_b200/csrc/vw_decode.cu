// vw_decode.cu -- paged decode attention for B200 (sm_100a), optionally fused
// with the KV append of the step's new token.
//
// Reference: kernels/attention/flash_attention.bm:113-162 (paged_attention_decode:
// one CTA per sequence, HEAD_DIM threads, single head, per-token online softmax)
// and its launcher :180-189.  This kernel computes the same function --
// o = softmax(q K^T * scale) V over the sequence's pages found through its
// block table, the last page partial (:132-140) -- re-designed for B200:
//
//  * Work split.  The unit of work is one page-head: 16 tokens of K and V of one
//    KV head, 8 KB contiguous in the pool ([L][NB][Hkv][2][16][D]).  All
//    page-heads of all (sequence, KV head) segments are laid end to end and cut
//    into equal contiguous ranges, one per CTA of a persistent grid of two CTAs
//    per SM, so every CTA streams the same number of bytes whatever the context
//    lengths (split-K over pages).  A segment cut by a range boundary leaves
//    (o, max, sum) partials, which a small combine grid launched right behind
//    the decode (programmatic dependent launch) merges; the decode CTAs
//    themselves never wait for one another or take an atomic.
//  * GQA.  The Hq/Hkv query heads that share a KV head are processed together:
//    each page is read from HBM once per KV head, never once per query head.
//  * Data movement.  A producer warp resolves block ids 32 pages at a time, one
//    batch ahead, and four of its lanes issue TMA tensor loads in parallel: one
//    or two boxes of 32 rows x 128 B (128-B swizzled) bring a page-head's K and
//    V into a ring of shared-memory stages tracked by mbarriers, plus one bulk
//    copy of each segment's query tile into a small ring.  A single issuing
//    thread serialises on the TMA round trip, which is why several lanes issue.
//    No multicast and no L2 eviction hints (an evict-first hint measurably
//    lowered throughput).
//  * Math.  Each of the W consumer warps takes every W-th page of the range and
//    runs the per-page micro-tiles on the tensor cores with warp-level mma.sync
//    m16n8k16 (tokens as M, query heads as N: S^T = K Q^T, then O^T = V^T P^T),
//    f32 accumulation, online softmax in the log2 domain.  The running maximum
//    is only raised (with a warp-shuffle reduction and a rescale of O) when some
//    score exceeds it by more than 2^8; otherwise probabilities up to 256 are
//    accumulated against the stale maximum, which changes no result but takes
//    the reduction off the per-page critical path.  A page gives a 16 x 8 x 128
//    micro-tile, below the 64-row minimum of a tcgen05 MMA; the kernel is
//    HBM-bound with the tensor pipes mostly idle.
//  * Fused append.  With k_new / v_new given, the warp that owns a segment's last
//    page writes the new token's K/V row (quantised for FP8 pools) to its slot
//    block_table[p/16]*16 + p%16, p = seq_len-1, in HBM and into the staged page.
//  * FP8 pools.  Pages hold E4M3 codes plus one f32 scale per token per head;
//    each lane of a consumer warp reads its share of the page's codes from the
//    stage into registers and expands them into binary16 MMA fragments (the
//    d order permuted so that a lane's fragments come from four 16-B loads
//    per K or V half and need no transpose); the scales fold into the scores
//    and the probabilities.
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
#include "vw_rope.cuh"

#ifndef VW_DECODE_WARPS
#define VW_DECODE_WARPS 4
#endif
#ifndef VW_DECODE_FP8_WARPS
#define VW_DECODE_FP8_WARPS 4
#endif
#ifndef VW_DECODE_CTAS_PER_SM
#define VW_DECODE_CTAS_PER_SM 2
#endif
// decode CTAs per SM in a launch's grid (at most the resident count above; a
// smaller grid leaves slots free for the next launch's CTAs)
#ifndef VW_DECODE_GRID_PER_SM
#define VW_DECODE_GRID_PER_SM VW_DECODE_CTAS_PER_SM
#endif
// register bound of the 2-byte-page, one-tile decode: the threads of this many
// CTAs per SM (3: 128 registers)
#ifndef VW_DECODE_MIN_CTAS_2B
#define VW_DECODE_MIN_CTAS_2B 3
#endif
#ifndef VW_DECODE_ISSUERS
#define VW_DECODE_ISSUERS 4
#endif
#ifndef VW_DECODE_FP8_PRODUCERS
#define VW_DECODE_FP8_PRODUCERS 2
#endif
#ifndef VW_DECODE_FP8_ISSUERS
#define VW_DECODE_FP8_ISSUERS 1
#endif
#ifndef VW_DECODE_MAX_STAGES
#define VW_DECODE_MAX_STAGES 16
#endif

namespace vw {

#ifdef VW_DECODE_TRACE
// Optional per-CTA phase timeline (build with -DVW_DECODE_TRACE): %globaltimer
// stamps of [start, prologue done, first load issued, first page ready, last
// load issued, last page done, merges done, exit] and combines done, for the
// most recent launch; read back with vw_debug_trace().
// Rows [layer & 1][blockIdx.x]: decode CTAs use slots 0-8, combine CTAs
// 12-14 (start, partials visible, done), so two consecutive layers' decode and
// combine grids can be read back together.
__device__ unsigned long long g_vw_trace[2 * 1024 * 16];
#define VW_TRACE(slot, val) \
    (g_vw_trace[(((p.layer & 1u) * 1024u) + blockIdx.x) * 16 + (slot)] = (val))
#else
#define VW_TRACE(slot, val) ((void)0)
#endif

namespace {

constexpr int kConsumerWarps = VW_DECODE_WARPS;
constexpr int kFp8ConsumerWarps = VW_DECODE_FP8_WARPS;
constexpr int kCtasPerSm = VW_DECODE_CTAS_PER_SM;
// Issuing lanes per producer warp, and producer warps.  The lanes of one warp
// that issue copies with different operands run them one after another, so an
// FP8 page-head (a tensor copy and a scale copy) issues faster from one lane in
// each of two warps than from four lanes of one warp.
constexpr int kIssuers = VW_DECODE_ISSUERS;
constexpr int kFp8ProducerWarps = VW_DECODE_FP8_PRODUCERS;
constexpr int kFp8Issuers = VW_DECODE_FP8_ISSUERS;
constexpr int kMaxStages = VW_DECODE_MAX_STAGES;
// per-CTA shared memory: an SM holds 228 KB and reserves 1 KB per resident CTA
__host__ __device__ constexpr int smem_per_cta(int ctas) { return 233472 / ctas - 1024; }
// 2-byte pages feed ldmatrix in place from the stage, [CHUNKS][32 rows][128 B]
// (column stride 4096 B); FP8 pages are read as codes straight into registers
constexpr int kStageColumn = 4096;
constexpr float kRescaleThreshold = 8.0f;             // log2 units: p <= 2^8 vs a stale max

// E4M3 codes -> f16 pairs for the MMA fragments hold value / 256; the 256 is
// folded into the K scales and the output.
constexpr float kFp8Fold = 256.0f;

__host__ __device__ constexpr int align_up_c(int x, int a) { return (x + a - 1) / a * a; }
__host__ __device__ constexpr int gcd_c(int a, int b) { return b == 0 ? a : gcd_c(b, a % b); }

template <int D_, int NT_, int KV_, int IO_>
struct Traits {
    static constexpr int D = D_, NT = NT_, KV = KV_, IO = IO_;
    // FP8 pages with one query-head tile: more consumer warps (the E4M3
    // expansion makes the consumers, not the copies, set the pace)
    static constexpr int W = (KV_ == kFP8 && NT_ == 1) ? kFp8ConsumerWarps : kConsumerWarps;
    static constexpr int PW = KV_ == kFP8 ? kFp8ProducerWarps : 1;   // producer warps W..W+PW-1
    static constexpr int IPW = KV_ == kFP8 ? kFp8Issuers : kIssuers;  // issuing lanes per producer warp
    static constexpr int NI = PW * IPW;                               // issuers in all
    static constexpr int THREADS = (W + PW) * 32;
    static constexpr int G = 8 * NT;                         // padded query heads per KV head
    static constexpr int EB = KV == kFP8 ? 1 : 2;            // pool element bytes
    static constexpr int ROW = D * EB;                       // bytes of one token row
    static constexpr int CHUNKS = ROW / 128;                 // 128-B swizzle columns per row
    static constexpr int STAGE = 32 * ROW;                   // one page-head: K rows 0-15, V 16-31
    static constexpr int SCAL = KV == kFP8 ? 128 : 0;        // K and V scales of a page-head
    static constexpr bool MMA_BF16 = KV == kBF16;            // FP8 pages compute in f16
    // P as a pair hi + lo of the MMA type, two P V MMAs: a single bf16 (2^-9)
    // or f16 x V-scale (2^-11) probability puts outputs whose few large V terms
    // cancel outside max-abs 2e-3 / rel 1e-2; f16 pools keep a single f16 P
    static constexpr bool PSPLIT = KV == kBF16 || KV == kFP8;
    // FP8 pages: the V codes are read after the softmax (not with the K codes)
    // when registers are short -- two query-head tiles, or more than four
    // consumer warps -- so that the K and V codes are never live together
    static constexpr bool LATE_V = KV == kFP8 && (NT != 1 || W > 4);
    static constexpr int KT = D / 16;                        // k-steps of Q K^T
    static constexpr int MT = D / 16;                        // d-tiles of V^T P^T
    // FP8 merge rows of D + 4 floats: a warp's stores of its O^T fragments
    // (lanes 4g+c hold query heads 2c, 2c+1, d values 32 apart) then fall on 32
    // different banks.  2-byte pages keep rows of D (a 4-way conflict measured
    // cheaper than the padded rows).
    static constexpr int MROW = KV == kFP8 ? D + 4 : D;
    // the warp states are merged one 8-head tile at a time: [W][8] rows of
    // MROW + 2 floats (o, max, sum), then [W + 2][8] weights, max and sum
    static constexpr int MERGE = W * 8 * (MROW + 2) * 4 + (W + 2) * 8 * 4;
    static constexpr int QTILE = G * D * 2;
    static constexpr int QSLOT = QTILE + 2 * D * 2;          // + the new token's K and V rows
    // query tiles in flight (one per segment); two with two query-head tiles,
    // whose larger slots would otherwise cost pipeline stages
    static constexpr int QS = NT == 1 ? 4 : 2;
    // prefixes of pages and of sequences with pages [B+1] each, and the seq_lens [B]
    static constexpr int PFX = align_up_c((3 * kMaxBatchPerLaunch + 2) * 4, 128);
    static constexpr int FIXED = align_up_c(MERGE, 1024) +
                                 align_up_c(QS * QSLOT, 1024) + PFX + PW * 1024 + 1024;
    // resident CTAs per SM the shared memory is sized for: FP8 pages and two
    // query-head tiles need the larger stages and registers of two
    static constexpr int RES = (NT == 1 && KV != kFP8) ? kCtasPerSm : 2;
    static constexpr int SMEM_CAP = smem_per_cta(RES);
    static constexpr int BUDGET = SMEM_CAP - 1024 /* base alignment slack */ -
                                  (SCAL ? 1024 : 0) /* scale ring alignment */;
    // Stage count: as many as fit, rounded down to a multiple of the consumer
    // warps and of the issuers.  Page i lives in stage i % S, is issued by
    // issuer i % NI (lane k / PW of producer warp k % PW) and consumed by warp
    // i % W; with S a multiple of both, every stage is filled by one lane and
    // drained by one warp, each in page order.  That is what the mbarrier parity
    // waits require: a parity wait can only tell the current phase from the one
    // before it, so no waiter may ever run two phases ahead of a barrier.
    static constexpr int LCM_WI = W * NI / gcd_c(W, NI);
    static constexpr int S_FIT = (BUDGET - FIXED) / (STAGE + SCAL) > kMaxStages
                                     ? kMaxStages : (BUDGET - FIXED) / (STAGE + SCAL);
    static constexpr int S = S_FIT / LCM_WI * LCM_WI;
    static constexpr int SMEM = 1024 + S * STAGE + align_up_c(S * SCAL, 1024) + FIXED;
    // FP8: probabilities carry the V scale but not the 1/256 of the f16 code
    // expansion; the output is multiplied back by 256
    static constexpr float VFOLD = KV == kFP8 ? kFp8Fold : 1.0f;
    // Register budget: the f16/bf16 kernels with one query-head tile fit in 128
    // registers (the bound of 3 CTAs' worth of threads), which leaves every SM
    // sub-partition room for the single-warp combine CTAs that wait beside the
    // decode CTAs; the others keep 168 (2 CTAs' worth) to avoid spills.
    static constexpr int MIN_CTAS = (NT == 1 && KV != kFP8) ? VW_DECODE_MIN_CTAS_2B : 2;
    static_assert(CHUNKS >= 1, "row must be at least 128 bytes");
    static_assert(S >= 4, "too few pipeline stages");
    static_assert(S % W == 0 && S % NI == 0, "stage ownership needs S % W == S % issuers == 0");
    static_assert(32 % NI == 0 && IPW <= 32, "issuers must divide the 32-page batch");
    static_assert(SMEM <= SMEM_CAP, "shared memory over the per-CTA limit");
    static_assert(STAGE % 1024 == 0, "1024-B tile alignment");
};

// Page as the producer publishes it to its issuing lanes: TMA row of its first
// K row (negative for an invalid block id: TMA zero-fills), and when the page
// starts a segment of this CTA's range (else qseg = -1) the segment ordinal,
// its first query row, and the row b*Hkv+h of the new K/V token when this CTA
// also holds the segment's last page and appends it (else kvrow = -1).
struct PageInfo {
    int kvrow, row0, qseg, qrow;
};

struct Smem {
    uint8_t* stages;     // [S][STAGE]
    float* scal;         // [S][32] FP8 scales (K 16, V 16)
    float* mo;           // [W][8][MROW] one 8-head tile of the warp states
    float* mm;           // [W][8]
    float* ml;           // [W][8]
    float* mf;           // [W][8] warp weights, then [8] max, [8] sum
    uint8_t* qring;      // [QS][QSLOT]: [G][D] query rows, then new K, new V rows (io dtype)
    int* pfx;            // [B+1] exclusive prefix of pages per sequence
    int* nzp;            // [B+1] exclusive prefix of sequences with pages
    int* slen;           // [B] seq_lens as the prologue read them
    PageInfo* pinfo;     // [PW][2][32] producer batches, one pair per producer warp
    uint64_t* full;      // [S]
    uint64_t* empty;     // [S]
    uint64_t* qfull;     // [QS]
    uint64_t* qempty;    // [QS]
    int* flag;           // [1] abort marker, [2..4] planned begin, end, first ordinal
};

template <class T>
__device__ __forceinline__ Smem carve(uint8_t* base) {
    Smem s;
    uint8_t* p = base;
    s.stages = p; p += T::S * T::STAGE;
    s.scal = reinterpret_cast<float*>(p); p += align_up_c(T::S * T::SCAL, 1024);
    s.mo = reinterpret_cast<float*>(p);
    s.mm = s.mo + T::W * 8 * T::MROW;
    s.ml = s.mm + T::W * 8;
    s.mf = s.ml + T::W * 8;
    p += align_up_c(T::MERGE, 1024);
    s.qring = p; p += align_up_c(T::QS * T::QSLOT, 1024);
    s.pfx = reinterpret_cast<int*>(p);
    s.nzp = s.pfx + (kMaxBatchPerLaunch + 1);
    s.slen = s.nzp + (kMaxBatchPerLaunch + 1);
    p += T::PFX;
    s.pinfo = reinterpret_cast<PageInfo*>(p); p += T::PW * 1024;
    s.full = reinterpret_cast<uint64_t*>(p);
    s.empty = s.full + T::S;
    s.qfull = s.empty + T::S;
    s.qempty = s.qfull + T::QS;
    s.flag = reinterpret_cast<int*>(s.qempty + T::QS);
    return s;
}

// Byte offset of element d of row `row` (0..31) inside a page-head tile of
// 2-byte elements stored as [CHUNKS][32 rows][128 B], 128-B swizzled.
__device__ __forceinline__ uint32_t swz16(int row, int d) {
    const int byte = d * 2;
    return (uint32_t)((byte >> 7) * 4096 + row * 128 + ((((byte & 127) >> 4) ^ (row & 7)) << 4) +
                      (byte & 15));
}
// Same for 1-byte rows of 128 (FP8, D = 128): [32 rows][128 B].
__device__ __forceinline__ uint32_t swz8(int row, int d) {
    return (uint32_t)(row * 128 + ((((d & 127) >> 4) ^ (row & 7)) << 4) + (d & 15));
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

// Page ranges of the decode CTAs.  The (sequence b, KV head h) segments,
// ordered by (b, h), lie end to end.  A CTA that crosses a segment boundary
// pays for a second query tile, a merge of its warps' states and a partial
// write, and it is the one that finishes last; so each segment is followed by
// a gap of `cost` virtual pages (DecodeParams::seg_cost) and the virtual line
// is cut into equal lengths vper.  Page x of the segment with ordinal k (among
// segments with pages) sits at v(x) = x + cost * k; CTA c takes the pages
// whose v falls in [c * vper, (c + 1) * vper), so the CTA holding page x is
// v(x) / vper.  With cost 0 this is the plain equal split.  The decode, its
// combine grid and the plan all cut with the launch's cost.

// Virtual positions stay far below 2^31: a launch covers fewer than 2^26 pages
// (the pool's rows are checked against 2^31 at creation) plus at most
// kMaxSegmentCost per segment.
__host__ __device__ __forceinline__ int virtual_total(int total_pages, int segments, int cost) {
    return total_pages + cost * segments;
}
__host__ __device__ __forceinline__ int virtual_per_cta(int vtotal, int grid) {
    const int v = (vtotal + grid - 1) / grid;
    return v < kMinPagesPerCta ? kMinPagesPerCta : v;
}

// First page x with v(x) >= t (total when there is none), from the exclusive
// prefixes of pages (pfx) and of sequences with pages (nzp) over B sequences.
__device__ __forceinline__ int range_start(const int* pfx, const int* nzp, int B, int Hkv, int cost, int t) {
    const int total = Hkv * pfx[B];
    if (t >= virtual_total(total, Hkv * nzp[B], cost)) return total;
    // largest b whose first virtual position is <= t (always a sequence with pages)
    int lo = 0, hi = B - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (virtual_total(Hkv * pfx[mid], Hkv * nzp[mid], cost) <= t) lo = mid; else hi = mid - 1;
    }
    const int np = pfx[lo + 1] - pfx[lo];
    const int r = t - virtual_total(Hkv * pfx[lo], Hkv * nzp[lo], cost);
    const int h = r / (np + cost);
    const int off = r - h * (np + cost);
    // inside the gap after segment h: the range starts at the next segment
    return Hkv * pfx[lo] + h * np + (off < np ? off : np);
}

__device__ __forceinline__ void set_err(uint32_t* err, uint32_t bit) { atomicOr(err, bit); }

// Pages per sequence -> exclusive prefixes of pages (pfx) and of sequences with
// pages (nzp), by one warp, 32 sequences at a time, keeping each seq_len in
// slen when given.  A seq_len of 0 gives no pages and one longer than its
// block-table row is clamped to the row; both are flagged when `report`.
__device__ __forceinline__ void warp_prefixes(const uint32_t* seq_lens, int B, int bt_stride,
                                              uint32_t* err, bool report, int* pfx, int* nzp,
                                              int* slen, int lane) {
    int run = 0, run_nz = 0;
    if (lane == 0) { pfx[0] = 0; nzp[0] = 0; }
    for (int base_b = 0; base_b < B; base_b += 32) {
        const int b = base_b + lane;
        int np = 0;
        if (b < B) {
            const int sl = (int)__ldg(seq_lens + b);
            if (slen) slen[b] = sl;
            np = (sl + 15) >> 4;
            if (sl <= 0 || np > bt_stride) {
                if (report) set_err(err, kDevErrSeqLen);
                np = sl <= 0 ? 0 : bt_stride;
            }
        }
        int incl = np, incl_nz = np > 0 ? 1 : 0;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, incl, off);
            const int vz = __shfl_up_sync(0xffffffffu, incl_nz, off);
            if (lane >= off) { incl += v; incl_nz += vz; }
        }
        if (b < B) { pfx[b + 1] = run + incl; nzp[b + 1] = run_nz + incl_nz; }
        run += __shfl_sync(0xffffffffu, incl, 31);
        run_nz += __shfl_sync(0xffffffffu, incl_nz, 31);
    }
}

template <int IO>
__device__ __forceinline__ float io_to_f32(uint32_t h) {
    return IO == kBF16 ? bf16_bits_to_f32(h) : f16_bits_to_f32(h);
}
template <int IO>
__device__ __forceinline__ uint16_t f32_to_io(float f) {
    return IO == kBF16 ? f32_to_bf16_bits(f) : f32_to_f16_bits(f);
}

// ------------------------------------------------------------------ producer

struct Resolved {
    int h, qseg, qrow, kvrow;
    uint32_t blk;
    bool live;
};

// Lane-parallel resolution of CTA-relative page i: its segment, KV head and
// block id (the block-table load is consumed one batch later).
__device__ __forceinline__ Resolved resolve_page(const DecodeParams& p, const Smem& sm, int begin,
                                                 int first_ord, int i, int n) {
    Resolved r{0, -1, -1, -1, 0xFFFFFFFFu, false};
    if (i < n) {
        const long long x = (long long)begin + i;
        const int b = find_seq(sm.pfx, (int)p.B, (int)p.Hkv, x);
        const int np = sm.pfx[b + 1] - sm.pfx[b];
        const int rr = (int)(x - (long long)p.Hkv * sm.pfx[b]);
        const int h = rr / np, pg = rr - h * np;
        r.h = h;
        r.live = true;
        r.blk = __ldg(p.block_tables + (size_t)b * p.bt_stride + pg);
        if (i == 0 || pg == 0) {
            r.qseg = sm.nzp[b] * (int)p.Hkv + h - first_ord;
            r.qrow = (int)(b * p.Hq + h * p.group);
            // the segment's last page is page i + np-1-pg of this range
            if (p.k_new != nullptr && i + (np - 1 - pg) < n) r.kvrow = (int)(b * p.Hkv + h);
        }
    }
    return r;
}

// Producer warp pw (0 .. PW-1): resolves every page of the range into its own
// record buffer, and its lanes 0 .. IPW-1 issue the pages of issuers
// lane * PW + pw.  Lane 0 of warp 0 also issues the query tiles, in segment
// order.
template <class T>
__device__ void producer(const CUtensorMap* tmap, const DecodeParams& p, const Smem& sm,
                         int begin, int n, int first_ord, int pw, uint64_t deadline) {
    const int lane = threadIdx.x & 31;
    PageInfo* const mine = sm.pinfo + pw * 64;
    const int k_me = lane * T::PW + pw;             // issuer number (lane < IPW)
    const bool qlane = pw == 0 && lane == 0;         // issues the query tiles
    const uint32_t Hkv = p.Hkv;
    const uint32_t qbytes = p.group * T::D * 2;
    const uint8_t* qbase = reinterpret_cast<const uint8_t*>(p.q);
    const uint8_t* kbase = reinterpret_cast<const uint8_t*>(p.k_new);
    const uint8_t* vbase = reinterpret_cast<const uint8_t*>(p.v_new);
    int segs_issued = 0;                             // highest segment ordinal issued + 1
    int issued_hi = -1;                              // last page this lane issued
    bool ok = true;

    auto publish = [&](const Resolved& r, int buf) {
        PageInfo pi;
        pi.kvrow = r.kvrow;
        pi.qseg = r.qseg;
        pi.qrow = r.qrow;
        pi.row0 = -32;
        if (r.live) {
            if (r.blk < p.num_blocks)
                pi.row0 = (int)(((p.layer * p.num_blocks + r.blk) * Hkv + (uint32_t)r.h) * 32u);
            else
                set_err(p.err, kDevErrBlockId);     // negative row: TMA zero-fills the tile
        }
        mine[buf * 32 + lane] = pi;
    };

    // Issue page ii (this lane owns its stage) into stage ii % S.
    auto issue_page = [&](int ii, const PageInfo& pi) -> bool {
        const int s = ii % T::S;
        if (ii >= T::S && !mbar_wait(&sm.empty[s], ((ii / T::S) - 1) & 1, deadline)) return false;
        if (ii == 0) VW_TRACE(2, globaltimer());
        if (ii == n - 1) VW_TRACE(4, globaltimer());
        uint8_t* st = sm.stages + s * T::STAGE;
        if constexpr (T::KV == kFP8) {
            float* sc = sm.scal + s * 32;
            if (pi.row0 >= 0) {
                // the page-head's K and V scales: 32 consecutive f32
                mbar_arrive_expect_tx(&sm.full[s], T::STAGE + 128);
                bulk_load(sc, p.kv_scales + pi.row0, 128, &sm.full[s]);
            } else {
                // invalid block id: zero scales with plain stores, ordered before
                // the arrive and fenced against this slot's next bulk write
                for (int k = 0; k < 32; ++k) sc[k] = 0.0f;
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                mbar_arrive_expect_tx(&sm.full[s], T::STAGE);
            }
        } else {
            mbar_arrive_expect_tx(&sm.full[s], T::STAGE);
        }
        // one tensor copy per page-head: rows of one 128-B column, then the next
        // column (the map's third dimension) when a row is 256 B
        if constexpr (T::CHUNKS == 1)
            tma_load_2d(st, tmap, &sm.full[s], 0, pi.row0);
        else
            tma_load_3d(st, tmap, &sm.full[s], 0, pi.row0, 0);
        issued_hi = ii;
        return true;
    };

    if (lane == 0) VW_TRACE(10, globaltimer());
    if (p.plan == nullptr) {                        // else batch 0 came with the plan
        Resolved cur = resolve_page(p, sm, begin, first_ord, lane, n);
        publish(cur, 0);
    }
    __syncwarp();
    if (lane == 0) VW_TRACE(11, globaltimer());
    // Early pages: the first S pages fill every stage once and need no empty
    // wait.  With kDecodeEarlyPages they are issued before the predecessor
    // grid has finished (the caller vouches that it writes neither the tables
    // nor these pages); the query tiles wait for it.
    // (at most the first batch: only its 32 page records are published yet)
    const int early_n = (p.flags & kDecodeEarlyPages) ? min(min(T::S, 32), n) : 0;
    if (lane < T::IPW)
        for (int j = k_me; j < early_n; j += T::NI) issue_page(j, mine[j]);
    if (early_n > 0 && pw == 0) {
        // warm L2 with the query tiles (and new K/V rows) of the first batch's
        // segments: the predecessor may still write them, but L2 is where that
        // write lands, so the bulk copies after the wait find them there anyway
        const PageInfo pi = mine[lane];
        if (lane < n && pi.qseg >= 0) {
            bulk_prefetch_l2(qbase + (size_t)pi.qrow * T::D * 2, qbytes);
            if (pi.kvrow >= 0) {
                bulk_prefetch_l2(kbase + (size_t)pi.kvrow * T::D * 2, T::D * 2);
                bulk_prefetch_l2(vbase + (size_t)pi.kvrow * T::D * 2, T::D * 2);
            }
        }
    }
    if (p.flags & kDecodePdl) griddep_wait();
    int buf = 0;
    for (int i0 = 0; i0 < n; i0 += 32) {
        const Resolved nxt = resolve_page(p, sm, begin, first_ord, i0 + 32 + lane, n);
        const int m = min(32, n - i0);
        if (lane < T::IPW) {
            // the query lane scans every page of the batch for segment starts so
            // that query tiles are issued in segment order by one thread (the query
            // ring's parity waits need that); each issuer issues the pages of its
            // own stages
            for (int j = qlane ? 0 : k_me; j < m && ok; j += qlane ? 1 : T::NI) {
                const int ii = i0 + j;
                const PageInfo pi = mine[buf * 32 + j];
                if (qlane && pi.qseg >= 0 && !(p.flags & kDecodeWithholdQ)) {
                    // a new segment starts here: its query tile
                    const int k = pi.qseg, qs = k % T::QS;
                    if (k >= T::QS &&
                        !mbar_wait(&sm.qempty[qs], ((k / T::QS) - 1) & 1, deadline)) {
                        ok = false;
                        break;
                    }
                    uint8_t* slot = sm.qring + qs * T::QSLOT;
                    const bool nkv = pi.kvrow >= 0;
                    if (k == 0 && (p.flags & kDecodeDirectQ)) {
                        // the consumers load this segment's rows themselves; the
                        // slot's phase still completes, so the ring stays in step
                        mbar_arrive(&sm.qfull[qs]);
                    } else {
                        mbar_arrive_expect_tx(&sm.qfull[qs], qbytes + (nkv ? 4 * T::D : 0));
                        bulk_load(slot, qbase + (size_t)pi.qrow * T::D * 2, qbytes, &sm.qfull[qs]);
                        if (nkv) {
                            bulk_load(slot + T::QTILE, kbase + (size_t)pi.kvrow * T::D * 2, T::D * 2,
                                      &sm.qfull[qs]);
                            bulk_load(slot + T::QTILE + T::D * 2, vbase + (size_t)pi.kvrow * T::D * 2,
                                      T::D * 2, &sm.qfull[qs]);
                        }
                    }
                    segs_issued = k + 1;
                }
                if ((j % T::NI) != k_me || ii < early_n) continue;   // another issuer's stage
                if (!issue_page(ii, pi)) {
                    ok = false;
                    break;
                }
            }
        }
        if (__any_sync(0xffffffffu, !ok)) { ok = false; break; }
        __syncwarp();
        buf ^= 1;
        publish(nxt, buf);
        __syncwarp();
    }
    if (!ok) set_err(p.err, kDevErrTimeout);
    // Drain: never leave the CTA while a TMA or bulk load may still write its
    // shared memory.  A lane issues the pages of its own stages in page order
    // and stops at its first failed wait, so its copies still in flight are at
    // most the last S / NI pages it issued (an older page's stage has been
    // refilled, so that page was consumed); the query lane likewise waits for
    // its last QS query tiles.  The drain has a deadline of its own: after
    // a timeout the kernel's deadline has passed, and giving up at once would
    // leave copies writing into a CTA that has exited.
    const uint64_t drain_deadline = cycles() + kWaitDeadlineCycles;
    if (lane < T::IPW) {
        for (int ii = issued_hi; ii >= 0 && ii > issued_hi - T::S; ii -= T::NI) {
            if (!mbar_wait(&sm.full[ii % T::S], (ii / T::S) & 1, drain_deadline)) {
                set_err(p.err, kDevErrTimeout);
                break;
            }
        }
    }
    for (int k = segs_issued > T::QS ? segs_issued - T::QS : 0; qlane && k < segs_issued; ++k) {
        if (!mbar_wait(&sm.qfull[k % T::QS], (k / T::QS) & 1, drain_deadline)) {
            set_err(p.err, kDevErrTimeout);
            break;
        }
    }
}

// Merge of the split-K pieces of one segment (b, h) for query head j and
// output elements d..d+3: the pieces (o, max, sum) left by decode CTAs
// c0..c0+n-1 (CTA c0 in slot slot0, the others in slot 0) are weighted by
// 2^(max_c - max), the online-softmax rule of flash_attention.bm:149-157
// applied across pieces; up to kCombineBatch pieces per memory round trip.
constexpr int kCombineBatch = 8;

template <int D, int G, int IO>
__device__ __forceinline__ void merge_unit(const DecodeParams& p, int b, int h, int j, int d, int c0,
                                           int n, int slot0, float vfold) {
    uint16_t* out = reinterpret_cast<uint16_t*>(p.out);
    const int g = (int)p.group;
    float M = -INFINITY, Ls = 0.0f, a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
    for (int k0 = 0; k0 < n; k0 += kCombineBatch) {
        float2 ml[kCombineBatch];
        float4 o[kCombineBatch];
#pragma unroll
        for (int k = 0; k < kCombineBatch; ++k) {
            ml[k] = make_float2(-INFINITY, 0.0f);
            o[k] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if (k0 + k < n) {
                const int c = c0 + k0 + k;
                const size_t piece = (size_t)c * 2 + (c == c0 ? slot0 : 0);
                ml[k] = __ldcg(reinterpret_cast<const float2*>(p.part_ml + (piece * G + j) * 2));
                o[k] = __ldcg(reinterpret_cast<const float4*>(p.part_o + (piece * G + j) * D + d));
            }
        }
        float Mn = M;
#pragma unroll
        for (int k = 0; k < kCombineBatch; ++k) Mn = fmaxf(Mn, ml[k].x);
        const float r = M > -INFINITY ? ex2(M - Mn) : 0.0f;
        Ls *= r; a0 *= r; a1 *= r; a2 *= r; a3 *= r;
#pragma unroll
        for (int k = 0; k < kCombineBatch; ++k) {
            const float w = ml[k].x > -INFINITY ? ex2(ml[k].x - Mn) : 0.0f;
            Ls += ml[k].y * w;
            a0 += o[k].x * w; a1 += o[k].y * w; a2 += o[k].z * w; a3 += o[k].w * w;
        }
        M = Mn;
    }
    const float r = vfold / Ls;
    const uint32_t lo = (uint32_t)f32_to_io<IO>(a0 * r) | ((uint32_t)f32_to_io<IO>(a1 * r) << 16);
    const uint32_t hi = (uint32_t)f32_to_io<IO>(a2 * r) | ((uint32_t)f32_to_io<IO>(a3 * r) << 16);
    *reinterpret_cast<uint2*>(out + ((size_t)b * p.Hq + (size_t)h * g + j) * D + d) = make_uint2(lo, hi);
}

// ------------------------------------------------------------------ consumer

// Query fragments (B operand of S^T = K Q^T) from the staged query tile.
// 2-byte pages: a lane's fragments hold elements d and d + D/2 (k-steps kt and
// kt + KT/2), so with rope_theta > 0 the rotation of the query heads at
// position pos happens here in registers, rounded to the io type as a separate
// RoPE pass would.  FP8 pages: k-step kt of lane c = lane%4 holds elements
// 32c+4kt .. 32c+4kt+3 (the order of the K fragments, see Fp8Codes), so the
// RoPE partner d +- D/2 of an element is in lane c ^ 2; the rotation runs
// before the pairs are put in fragment order.
template <class T>
__device__ __forceinline__ void load_q(const DecodeParams& p, const uint8_t* qtile, int lane,
                                       float pos, uint32_t (&qf)[T::NT][T::KT][2]) {
#pragma unroll
    for (int nt = 0; nt < T::NT; ++nt) {
        const int j = nt * 8 + (lane >> 2);
        const bool live = j < (int)p.group;
        const uint8_t* row = qtile + (live ? j : 0) * T::D * 2;
        if constexpr (T::KV == kFP8) {
            const int c = lane & 3;
            uint32_t w[16];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const uint4 v = live ? *reinterpret_cast<const uint4*>(row + c * 64 + u * 16)
                                     : make_uint4(0, 0, 0, 0);
                w[4 * u] = v.x; w[4 * u + 1] = v.y; w[4 * u + 2] = v.z; w[4 * u + 3] = v.w;
            }
            if (p.rope_theta > 0.0f) {
                const bool lo = c < 2;                  // elements below D/2
#pragma unroll
                for (int m = 0; m < 16; ++m) {
                    const uint32_t other = __shfl_xor_sync(0xffffffffu, w[m], 2);
                    const uint32_t rw = lo ? w[m] : other, iw = lo ? other : w[m];
                    float r0 = io_to_f32<T::IO>(rw & 0xFFFFu), i0 = io_to_f32<T::IO>(iw & 0xFFFFu);
                    float r1 = io_to_f32<T::IO>(rw >> 16), i1 = io_to_f32<T::IO>(iw >> 16);
                    const int d = (c & 1) * 32 + 2 * m;   // index of the lower element
                    rope_pair(r0, i0, d, T::D, p.rope_theta, pos);
                    rope_pair(r1, i1, d + 1, T::D, p.rope_theta, pos);
                    w[m] = lo ? ((uint32_t)f32_to_io<T::IO>(r0) | ((uint32_t)f32_to_io<T::IO>(r1) << 16))
                              : ((uint32_t)f32_to_io<T::IO>(i0) | ((uint32_t)f32_to_io<T::IO>(i1) << 16));
                }
            }
#pragma unroll
            for (int m = 0; m < 16; ++m) {
                if constexpr (T::IO == kBF16)       // pages compute in f16
                    w[m] = pack2<false>(bf16_bits_to_f32(w[m] & 0xFFFFu), bf16_bits_to_f32(w[m] >> 16));
            }
            // k-step kt: elements 32c+4kt+1, +3 first, then +0, +2 (the K pairs)
#pragma unroll
            for (int kt = 0; kt < T::KT; ++kt) {
                qf[nt][kt][0] = __byte_perm(w[2 * kt], w[2 * kt + 1], 0x7632u);
                qf[nt][kt][1] = __byte_perm(w[2 * kt], w[2 * kt + 1], 0x5410u);
            }
        } else {
#pragma unroll
            for (int kt = 0; kt < T::KT; ++kt)
#pragma unroll
                for (int hf = 0; hf < 2; ++hf) {
                    const int d = kt * 16 + hf * 8 + 2 * (lane & 3);
                    qf[nt][kt][hf] = live ? *reinterpret_cast<const uint32_t*>(row + d * 2) : 0u;
                }
            if (p.rope_theta > 0.0f) {
#pragma unroll
                for (int kt = 0; kt < T::KT / 2; ++kt)
#pragma unroll
                    for (int hf = 0; hf < 2; ++hf) {
                        const int d = kt * 16 + hf * 8 + 2 * (lane & 3);
                        uint32_t& a = qf[nt][kt][hf];
                        uint32_t& b = qf[nt][kt + T::KT / 2][hf];
                        float ar = io_to_f32<T::IO>(a & 0xFFFFu), ai = io_to_f32<T::IO>(b & 0xFFFFu);
                        float br = io_to_f32<T::IO>(a >> 16), bi = io_to_f32<T::IO>(b >> 16);
                        rope_pair(ar, ai, d, T::D, p.rope_theta, pos);
                        rope_pair(br, bi, d + 1, T::D, p.rope_theta, pos);
                        a = (uint32_t)f32_to_io<T::IO>(ar) | ((uint32_t)f32_to_io<T::IO>(br) << 16);
                        b = (uint32_t)f32_to_io<T::IO>(ai) | ((uint32_t)f32_to_io<T::IO>(bi) << 16);
                    }
            }
        }
    }
}

// Write the new token's row (t = valid-1) of one KV head into HBM and into the
// staged page-head (K at row t, V at row 16+t).  One warp; each lane owns D/32
// consecutive elements, given in nkv[kv] (the rows the producer staged with the
// segment's query tile).
template <class T>
__device__ __forceinline__ void append_row(const DecodeParams& p, uint8_t* stage, float* scal,
                                           int h, uint32_t blk, int t, int lane,
                                           const uint32_t (&nkv)[2][2]) {
    constexpr int PER = T::D / 32;    // 2 (D=64) or 4 (D=128)
    const bool blk_ok = blk < p.num_blocks;
    if (!blk_ok && lane == 0) set_err(p.err, kDevErrBlockId);
#pragma unroll
    for (int kv = 0; kv < 2; ++kv) {
        // pool row of (layer, block, head, kv, t) in [L][NB][Hkv][2][16]
        const size_t prow = ((((size_t)p.layer * p.num_blocks + blk) * p.Hkv + h) * 2 + kv) * 16 + t;
        const int srow = kv * 16 + t;
        if constexpr (T::KV != kFP8) {
            const uint32_t* w = nkv[kv];
            uint8_t* gdst = p.kv_data + prow * T::ROW + lane * PER * 2;
            uint8_t* sdst = stage + swz16(srow, lane * PER);
            if constexpr (PER == 4) {
                if (blk_ok) *reinterpret_cast<uint2*>(gdst) = make_uint2(w[0], w[1]);
                *reinterpret_cast<uint2*>(sdst) = make_uint2(w[0], w[1]);
            } else {
                if (blk_ok) *reinterpret_cast<uint32_t*>(gdst) = w[0];
                *reinterpret_cast<uint32_t*>(sdst) = w[0];
            }
        } else {
            static_assert(T::D == 128, "FP8 pools need head_dim 128");
            const uint2 raw = make_uint2(nkv[kv][0], nkv[kv][1]);
            float v[4] = {io_to_f32<T::IO>(raw.x & 0xFFFFu), io_to_f32<T::IO>(raw.x >> 16),
                          io_to_f32<T::IO>(raw.y & 0xFFFFu), io_to_f32<T::IO>(raw.y >> 16)};
            float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
            for (int off = 16; off > 0; off >>= 1)
                amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
            const float scale = fp8_row_scale(amax);
            const uint32_t codes = fp8_encode4(v, scale, p.fp8_ocp != 0);
            uint8_t* gdst = p.kv_data + prow * T::ROW + lane * 4;
            if (blk_ok) *reinterpret_cast<uint32_t*>(gdst) = codes;
            *reinterpret_cast<uint32_t*>(stage + swz8(srow, lane * 4)) = codes;
            if (lane == 0) {
                if (blk_ok) p.kv_scales[prow] = scale;
                scal[srow] = scale;
            }
        }
    }
}

// Zero V rows [valid, 16) of a staged page-head so masked tokens cannot inject
// NaN/Inf through 0 * garbage in the P.V product.
template <class T>
__device__ __forceinline__ void zero_tail(uint8_t* stage, int valid, int lane) {
    const int per_row = T::CHUNKS * 8;                   // 16-B pieces per row
    const int total = (16 - valid) * per_row;
    for (int k = lane; k < total; k += 32) {
        const int piece = k % per_row, row = 16 + valid + k / per_row;
        const int c = piece >> 3, ch = piece & 7;
        *reinterpret_cast<uint4*>(stage + c * 4096 + row * 128 + (ch << 4)) = make_uint4(0, 0, 0, 0);
    }
}

// FP8 page-head fragments, read as codes straight from the stage (128-B
// swizzled rows, 16-B unit u of stage row r at (u ^ (r & 7)) * 16).
//  * K: lane (g = lane/4, c = lane%4) takes the 32 codes 32c .. 32c+31 of token
//    rows g and g+8, two 16-B units per row.  The order of the reduction over
//    d inside a k-step of S^T = K Q^T is free, so k-step kt uses word kt of
//    each lane's run (codes 32c+4kt .. +3): fragment columns 2c, 2c+1 hold its
//    odd bytes (d = 32c+4kt+1, +3), columns 2c+8, 2c+9 its even bytes
//    (d = 32c+4kt, +2), which the expansion reaches without a byte permute;
//    load_q orders the query pairs the same way.
//  * V: for O^T = V^T P^T the A fragment of lane (g, c) holds tokens 2c, 2c+1,
//    2c+8, 2c+9 (the k index is the token, as in the P fragments); the output
//    rows of each d-tile are free, so row r of d-tile mt is
//    d = 16*(r%8) + 8*(r/8) + mt (fp8_out_d) and the lane reads 16-B unit g of
//    its four token rows: every fragment pair is one byte of two of them, with
//    no transpose.
struct Fp8Codes {
    uint4 k[2][2];     // [token row g, g+8][16-B unit 2c, 2c+1]
    uint4 v[4];        // unit g of token rows 2c, 2c+1, 2c+8, 2c+9
};

// kv = 0: the K rows (stage rows 0-15) into f.k; kv = 1: the V rows into f.v.
// Both are conflict-free: the 8 lanes of a 16-B load phase read 8 different
// units.
__device__ __forceinline__ void load_fp8_codes(const uint8_t* st, int lane, int kv, Fp8Codes& f) {
    const int g = lane >> 2, c = lane & 3;
    if (kv == 0) {
#pragma unroll
        for (int rr = 0; rr < 2; ++rr)
#pragma unroll
            for (int hh = 0; hh < 2; ++hh)
                f.k[rr][hh] = *reinterpret_cast<const uint4*>(st + (g + 8 * rr) * 128 + (((2 * c + hh) ^ g) << 4));
    } else {
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int tok = 2 * c + (r & 1) + 8 * (r >> 1);
            f.v[r] = *reinterpret_cast<const uint4*>(st + (16 + tok) * 128 + ((g ^ (tok & 7)) << 4));
        }
    }
}

__device__ __forceinline__ uint32_t word_of(const uint4& h, int k) {
    return k == 0 ? h.x : k == 1 ? h.y : k == 2 ? h.z : h.w;
}

// Word i (0..7) of a lane's 32-byte run held as two uint4.
__device__ __forceinline__ uint32_t run_word(const uint4 (&u)[2], int i) { return word_of(u[i >> 2], i & 3); }

__host__ __device__ __forceinline__ int fp8_out_d(int r, int mt) {
    return 16 * (r & 7) + 8 * (r >> 3) + mt;
}

// Column of output element d in a merge row.  The FP8 fragments put d values
// 16 apart in one store (lanes g = 0..7); flipping bits 0-2 of d by bits 4-6
// spreads them over the banks, and with the rows of D + 4 floats of the four
// query-head pairs a store's 32 lanes meet 32 different banks (a permutation
// inside each block of 16).
template <class T>
__device__ __forceinline__ int merge_col(int d) {
    return T::KV == kFP8 ? d ^ ((d >> 4) & 7) : d;
}

template <class T>
__device__ void consumer(const DecodeParams& p, const Smem& sm, int begin, int end,
                         uint64_t deadline) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ctid = threadIdx.x;                     // 0 .. W*32-1
    const int Hkv = (int)p.Hkv;
    constexpr int W = T::W;
    constexpr int NTH = W * 32;
    const bool append = p.k_new != nullptr;

    // ldmatrix lane geometry: K rows feed A = K (tokens x d), V rows (16..31)
    // feed A = V^T (d x tokens) through the transposing load
    const int mi = lane >> 3;
    const int k_tok = (lane & 7) + ((mi & 1) << 3), k_hs = mi >> 1;
    const int v_tok = (lane & 7) + ((mi >> 1) << 3), v_hs = mi & 1;
    const int t0 = lane >> 2, t1 = t0 + 8;

    bool alive = true;
    int seg_k = 0;

    for (int x = begin; x < end;) {
        const int b = find_seq(sm.pfx, (int)p.B, Hkv, x);
        const int np = sm.pfx[b + 1] - sm.pfx[b];
        const int seg_start = Hkv * sm.pfx[b];
        const int r = x - seg_start;
        const int h = r / np, pg0 = r - h * np;
        const int cnt = min(np - pg0, end - x);
        const bool complete = pg0 == 0 && cnt == np;
        const int i_base = x - begin;
        const int seq_len = sm.slen[b];     // read in the prologue: no load after the release

        // query tile of this segment (staged by the producer)
        uint32_t qf[T::NT][T::KT][2];
        uint32_t nkv[2][2] = {{0u, 0u}, {0u, 0u}};
        {
            const int qs = seg_k % T::QS;
            // The first segment's rows come straight from global memory (L2, where
            // the producer prefetched them) when kDecodeDirectQ is set; the others
            // from the query ring.  Every lane waits, then the warp agrees (and
            // reconverges) before the warp-collective fragment loads that follow.
            const bool direct = seg_k == 0 && (p.flags & kDecodeDirectQ);
            const bool got = !alive || direct ||
                             mbar_wait(&sm.qfull[qs], (seg_k / T::QS) & 1, deadline);
            if (!__all_sync(0xffffffffu, got)) {
                if (lane == 0) set_err(p.err, kDevErrTimeout);
                alive = false;
            }
            const uint8_t* qsrc = direct ? reinterpret_cast<const uint8_t*>(p.q) +
                                               (size_t)(b * p.Hq + h * p.group) * T::D * 2
                                         : sm.qring + qs * T::QSLOT;
            load_q<T>(p, qsrc, lane, (float)(seq_len - 1), qf);
            if (append && pg0 + cnt == np) {
                // this range holds the segment's last page: keep the staged new
                // K/V row pieces of this lane for the append
                const size_t kvoff = (size_t)(b * Hkv + h) * T::D * 2 + lane * (T::D / 32) * 2;
                const uint8_t* krow = direct ? reinterpret_cast<const uint8_t*>(p.k_new) + kvoff
                                             : sm.qring + qs * T::QSLOT + T::QTILE + lane * (T::D / 32) * 2;
                const uint8_t* vrow = direct ? reinterpret_cast<const uint8_t*>(p.v_new) + kvoff
                                             : krow + T::D * 2;
#pragma unroll
                for (int k = 0; k < T::D / 64; ++k) {
                    nkv[0][k] = reinterpret_cast<const uint32_t*>(krow)[k];
                    nkv[1][k] = reinterpret_cast<const uint32_t*>(vrow)[k];
                }
                if (p.rope_theta > 0.0f) {
                    // the new K row at position seq_len-1: lane l holds elements
                    // l*D/32 .. +D/32-1, whose partners (d +- D/2) lane l ^ 16 holds
                    const bool lo = lane < 16;
                    const float pos = (float)(seq_len - 1);
#pragma unroll
                    for (int k = 0; k < T::D / 64; ++k) {
                        const uint32_t own = nkv[0][k];
                        const uint32_t other = __shfl_xor_sync(0xffffffffu, own, 16);
                        const uint32_t rw = lo ? own : other, iw = lo ? other : own;
                        float r0 = io_to_f32<T::IO>(rw & 0xFFFFu), i0 = io_to_f32<T::IO>(iw & 0xFFFFu);
                        float r1 = io_to_f32<T::IO>(rw >> 16), i1 = io_to_f32<T::IO>(iw >> 16);
                        const int d = (lane & 15) * (T::D / 32) + 2 * k;
                        rope_pair(r0, i0, d, T::D, p.rope_theta, pos);
                        rope_pair(r1, i1, d + 1, T::D, p.rope_theta, pos);
                        nkv[0][k] = lo ? ((uint32_t)f32_to_io<T::IO>(r0) | ((uint32_t)f32_to_io<T::IO>(r1) << 16))
                                       : ((uint32_t)f32_to_io<T::IO>(i0) | ((uint32_t)f32_to_io<T::IO>(i1) << 16));
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.qempty[qs]);
            ++seg_k;
        }

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
            float* sc = sm.scal + s * 32;
            // warp-uniform wait: ldmatrix / mma.sync below need the whole warp
            if (!__all_sync(0xffffffffu, mbar_wait(&sm.full[s], (i / T::S) & 1, deadline))) {
                if (lane == 0) set_err(p.err, kDevErrTimeout);
                alive = false;
                break;
            }
            if (i == 0 && lane == 0) VW_TRACE(3, globaltimer());
            int valid = 16;
            if (pg == np - 1) {
                // a seq_len beyond the table (flagged in the prologue) reads its
                // pages as full and appends nothing
                valid = seq_len - pg * 16;
                const bool in_page = valid <= 16;
                if (!in_page) valid = 16;
                if (append && in_page) {
                    const uint32_t blk = __ldg(p.block_tables + (size_t)b * p.bt_stride + pg);
                    append_row<T>(p, st, sc, h, blk, valid - 1, lane, nkv);
                }
                if (valid < 16) zero_tail<T>(st, valid, lane);
                // plain stores into a TMA-filled stage: order them before the stage's
                // next asynchronous (TMA) write, which follows the empty arrive below
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
            }
            float ks0 = 1.0f, ks1 = 1.0f, vs0 = 1.0f, vs1 = 1.0f;
            const uint32_t tbase = smem_u32(st);
            Fp8Codes fc;
            if constexpr (T::KV == kFP8) {
                // this lane's codes and scales are all the page-head it needs:
                // the stage goes back to the producer before any math, or, with
                // LATE_V, after the V codes are read following the softmax
                ks0 = sc[t0] * kFp8Fold; ks1 = sc[t1] * kFp8Fold;
                vs0 = sc[16 + t0]; vs1 = sc[16 + t1];
                load_fp8_codes(st, lane, 0, fc);
                if constexpr (!T::LATE_V) {
                    load_fp8_codes(st, lane, 1, fc);
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&sm.empty[s]);
                }
            }

            // ---- S^T = K Q^T  (16 tokens x 8*NT heads), two independent chains
            float sa[T::NT][4], sb[T::NT][4];
#pragma unroll
            for (int nt = 0; nt < T::NT; ++nt)
#pragma unroll
                for (int k = 0; k < 4; ++k) sa[nt][k] = sb[nt][k] = 0.0f;
#pragma unroll
            for (int kt = 0; kt < T::KT; ++kt) {
                uint32_t a0, a1, a2, a3;
                if constexpr (T::KV == kFP8) {
                    const uint32_t w0 = run_word(fc.k[0], kt), w1 = run_word(fc.k[1], kt);
                    a0 = fp8_pair_odd(w0); a1 = fp8_pair_odd(w1);
                    a2 = fp8_pair_even(w0); a3 = fp8_pair_even(w1);
                } else {
                    const uint32_t addr = tbase + (kt >> 2) * kStageColumn + k_tok * 128 +
                                          ((((kt & 3) * 2 + k_hs) ^ (k_tok & 7)) << 4);
                    ldsm_x4(addr, a0, a1, a2, a3);
                }
#pragma unroll
                for (int nt = 0; nt < T::NT; ++nt) {
                    if (kt & 1) mma_16816<T::MMA_BF16>(sb[nt], a0, a1, a2, a3, qf[nt][kt][0], qf[nt][kt][1]);
                    else mma_16816<T::MMA_BF16>(sa[nt], a0, a1, a2, a3, qf[nt][kt][0], qf[nt][kt][1]);
                }
            }


            // ---- online softmax (log2 domain) with a lazily raised maximum
            const bool v0 = t0 < valid, v1 = t1 < valid;
            float sv[T::NT][4];
            bool need = false;
#pragma unroll
            for (int nt = 0; nt < T::NT; ++nt) {
                sv[nt][0] = v0 ? (sa[nt][0] + sb[nt][0]) * p.scale_log2 * ks0 : -INFINITY;
                sv[nt][1] = v0 ? (sa[nt][1] + sb[nt][1]) * p.scale_log2 * ks0 : -INFINITY;
                sv[nt][2] = v1 ? (sa[nt][2] + sb[nt][2]) * p.scale_log2 * ks1 : -INFINITY;
                sv[nt][3] = v1 ? (sa[nt][3] + sb[nt][3]) * p.scale_log2 * ks1 : -INFINITY;
                need |= fmaxf(sv[nt][0], sv[nt][2]) > mrun[nt][0] + kRescaleThreshold;
                need |= fmaxf(sv[nt][1], sv[nt][3]) > mrun[nt][1] + kRescaleThreshold;
            }
            if (__any_sync(0xffffffffu, need)) {
#pragma unroll
                for (int nt = 0; nt < T::NT; ++nt) {
                    float mx0 = fmaxf(sv[nt][0], sv[nt][2]), mx1 = fmaxf(sv[nt][1], sv[nt][3]);
#pragma unroll
                    for (int off = 4; off < 32; off <<= 1) {
                        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
                        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
                    }
                    const float mn0 = fmaxf(mrun[nt][0], mx0), mn1 = fmaxf(mrun[nt][1], mx1);
                    const float al0 = ex2(mrun[nt][0] - mn0), al1 = ex2(mrun[nt][1] - mn1);
                    mrun[nt][0] = mn0; mrun[nt][1] = mn1;
                    lrun[nt][0] *= al0; lrun[nt][1] *= al1;
#pragma unroll
                    for (int mt = 0; mt < T::MT; ++mt) {
                        o[nt][mt][0] *= al0; o[nt][mt][1] *= al1;
                        o[nt][mt][2] *= al0; o[nt][mt][3] *= al1;
                    }
                }
            }
            uint32_t pb[T::NT][2], pl[T::NT][2];
#pragma unroll
            for (int nt = 0; nt < T::NT; ++nt) {
                const float p00 = ex2(sv[nt][0] - mrun[nt][0]), p01 = ex2(sv[nt][1] - mrun[nt][1]);
                const float p10 = ex2(sv[nt][2] - mrun[nt][0]), p11 = ex2(sv[nt][3] - mrun[nt][1]);
                lrun[nt][0] += p00 + p10;
                lrun[nt][1] += p01 + p11;
                float q00 = p00, q01 = p01, q10 = p10, q11 = p11;
                if constexpr (T::KV == kFP8) {
                    q00 = v0 ? p00 * vs0 : 0.0f; q01 = v0 ? p01 * vs0 : 0.0f;
                    q10 = v1 ? p10 * vs1 : 0.0f; q11 = v1 ? p11 * vs1 : 0.0f;
                }
                if constexpr (T::MMA_BF16) {
                    // hi = q truncated to bf16 (its top 16 bits), lo = q - hi (exact
                    // in f32) rounded to bf16
                    const uint32_t h00 = __float_as_uint(q00) & 0xFFFF0000u, h01 = __float_as_uint(q01) & 0xFFFF0000u;
                    const uint32_t h10 = __float_as_uint(q10) & 0xFFFF0000u, h11 = __float_as_uint(q11) & 0xFFFF0000u;
                    pb[nt][0] = movmatrix_t(__byte_perm(h00, h01, 0x7632));
                    pb[nt][1] = movmatrix_t(__byte_perm(h10, h11, 0x7632));
                    pl[nt][0] = movmatrix_t(pack2<true>(q00 - __uint_as_float(h00), q01 - __uint_as_float(h01)));
                    pl[nt][1] = movmatrix_t(pack2<true>(q10 - __uint_as_float(h10), q11 - __uint_as_float(h11)));
                } else {
                    const uint32_t a = pack2<false>(q00, q01), c = pack2<false>(q10, q11);
                    pb[nt][0] = movmatrix_t(a);
                    pb[nt][1] = movmatrix_t(c);
                    if constexpr (T::PSPLIT) {
                        pl[nt][0] = movmatrix_t(pack2<false>(q00 - f16_bits_to_f32(a & 0xFFFFu),
                                                             q01 - f16_bits_to_f32(a >> 16)));
                        pl[nt][1] = movmatrix_t(pack2<false>(q10 - f16_bits_to_f32(c & 0xFFFFu),
                                                             q11 - f16_bits_to_f32(c >> 16)));
                    }
                }
            }

            // ---- O^T += V^T P^T  (D x 8*NT); V is stage rows 16-31
            if constexpr (T::LATE_V) {
                load_fp8_codes(st, lane, 1, fc);
                __syncwarp();
                if (lane == 0) mbar_arrive(&sm.empty[s]);
            }
#pragma unroll
            for (int mt = 0; mt < T::MT; ++mt) {
                uint32_t a0, a1, a2, a3;
                if constexpr (T::KV == kFP8) {
                    // byte mt of unit g: d = 16g + mt (rows g) and 16g + 8 + mt (rows g + 8)
                    const int lo = mt >> 2, hi = 2 + (mt >> 2), j = mt & 3;
                    a0 = fp8_pair_cross(word_of(fc.v[0], lo), word_of(fc.v[1], lo), j);
                    a1 = fp8_pair_cross(word_of(fc.v[0], hi), word_of(fc.v[1], hi), j);
                    a2 = fp8_pair_cross(word_of(fc.v[2], lo), word_of(fc.v[3], lo), j);
                    a3 = fp8_pair_cross(word_of(fc.v[2], hi), word_of(fc.v[3], hi), j);
                } else {
                    const uint32_t addr = tbase + (mt >> 2) * kStageColumn + (16 + v_tok) * 128 +
                                          ((((mt & 3) * 2 + v_hs) ^ (v_tok & 7)) << 4);
                    ldsm_x4_t(addr, a0, a1, a2, a3);
                }
#pragma unroll
                for (int nt = 0; nt < T::NT; ++nt) {
                    mma_16816<T::MMA_BF16>(o[nt][mt], a0, a1, a2, a3, pb[nt][0], pb[nt][1]);
                    if constexpr (T::PSPLIT) mma_16816<T::MMA_BF16>(o[nt][mt], a0, a1, a2, a3, pl[nt][0], pl[nt][1]);
                }
            }
            __syncwarp();
            if constexpr (T::KV != kFP8) {
                if (lane == 0) mbar_arrive(&sm.empty[s]);
            }
        }

        // ---- merge the W warps' states for this segment, one 8-head tile at a
        // time (three barriers per tile)
        if (ctid == 0 && x + cnt >= end) VW_TRACE(5, globaltimer());
        if (!alive && lane == 0) sm.flag[1] = 1;  // abort marker, read by all warps below
        float* mo = sm.mo + warp * 8 * T::MROW;
        const int g = (int)p.group;
        // A segment wholly inside this range is written out here; a piece of a
        // segment split across ranges leaves (o, max, sum) for the combine kernel.
        uint16_t* out = reinterpret_cast<uint16_t*>(p.out);
        const int slot = (x == begin) ? 0 : 1;
        float* po = p.part_o + ((size_t)blockIdx.x * 2 + slot) * T::G * T::D;
        float* pml = p.part_ml + ((size_t)blockIdx.x * 2 + slot) * T::G * 2;
        bool abort = false;
#pragma unroll
        for (int nt = 0; nt < T::NT; ++nt) {
#pragma unroll
            for (int off = 4; off < 32; off <<= 1) {
                lrun[nt][0] += __shfl_xor_sync(0xffffffffu, lrun[nt][0], off);
                lrun[nt][1] += __shfl_xor_sync(0xffffffffu, lrun[nt][1], off);
            }
            const int jl = 2 * (lane & 3);        // this lane's heads in the tile: jl, jl + 1
#pragma unroll
            for (int mt = 0; mt < T::MT; ++mt) {
                // O^T rows lane/4 and lane/4 + 8 of d-tile mt
                const int dA = T::KV == kFP8 ? fp8_out_d(lane >> 2, mt) : mt * 16 + (lane >> 2);
                const int dB = T::KV == kFP8 ? fp8_out_d((lane >> 2) + 8, mt) : dA + 8;
                mo[jl * T::MROW + merge_col<T>(dA)] = o[nt][mt][0];
                mo[(jl + 1) * T::MROW + merge_col<T>(dA)] = o[nt][mt][1];
                mo[jl * T::MROW + merge_col<T>(dB)] = o[nt][mt][2];
                mo[(jl + 1) * T::MROW + merge_col<T>(dB)] = o[nt][mt][3];
            }
            if (lane < 4) {
                sm.mm[warp * 8 + jl] = mrun[nt][0];
                sm.mm[warp * 8 + jl + 1] = mrun[nt][1];
                sm.ml[warp * 8 + jl] = lrun[nt][0];
                sm.ml[warp * 8 + jl + 1] = lrun[nt][1];
            }
            named_bar_sync(1, NTH);
            // every consumer warp reads the same marker after the barrier, so all
            // of them leave the segment loop together and no named barrier is
            // orphaned
            abort = sm.flag[1] != 0;
            const int jn = min(8, g - nt * 8);    // live query heads of the tile
            // per-head weights of the W warp states: max, sum, and one factor per
            // warp (warps without pages in this segment carry -inf and get 0)
            if (ctid < jn) {
                const int j = ctid;
                float M = -INFINITY;
#pragma unroll
                for (int w = 0; w < W; ++w) M = fmaxf(M, sm.mm[w * 8 + j]);
                float Ls = 0.0f;
#pragma unroll
                for (int w = 0; w < W; ++w) {
                    const float mw = sm.mm[w * 8 + j];
                    const float f = mw > -INFINITY ? ex2(mw - M) : 0.0f;
                    Ls += sm.ml[w * 8 + j] * f;
                    sm.mf[w * 8 + j] = f;
                }
                sm.mf[W * 8 + j] = M;
                sm.mf[(W + 1) * 8 + j] = Ls;
            }
            named_bar_sync(1, NTH);
            for (int idx = ctid; idx < jn * T::D && !abort; idx += NTH) {
                const int jt = idx / T::D, d = idx - jt * T::D, j = nt * 8 + jt;
                float Os = 0.0f;
#pragma unroll
                for (int w = 0; w < W; ++w)
                    Os += sm.mo[(w * 8 + jt) * T::MROW + merge_col<T>(d)] * sm.mf[w * 8 + jt];
                if (complete) {
                    out[((size_t)b * p.Hq + (size_t)h * g + j) * T::D + d] =
                        f32_to_io<T::IO>(Os / sm.mf[(W + 1) * 8 + jt] * T::VFOLD);
                } else {
                    po[j * T::D + d] = Os;
                    if (d == 0) { pml[j * 2] = sm.mf[W * 8 + jt]; pml[j * 2 + 1] = sm.mf[(W + 1) * 8 + jt]; }
                }
            }
            named_bar_sync(1, NTH);
        }
        x += cnt;
        if (abort) break;
    }
    if (ctid == 0) VW_TRACE(6, globaltimer());
}

template <class T>
__global__ void __launch_bounds__(T::THREADS, T::MIN_CTAS)
decode_kernel(const __grid_constant__ CUtensorMap tmap, const DecodeParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const Smem sm = carve<T>(base);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint64_t deadline = cycles() + (p.wait_cycles ? p.wait_cycles : kWaitDeadlineCycles);
    if (threadIdx.x == 0) VW_TRACE(0, globaltimer());
#ifdef VW_DECODE_TRACE
    if (threadIdx.x == 0) {
        uint32_t smid;
        asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
        VW_TRACE(9, smid);
    }
#endif

    if (threadIdx.x == 0) {
        for (int s = 0; s < T::S; ++s) { mbar_init(&sm.full[s], 1); mbar_init(&sm.empty[s], 1); }
        for (int s = 0; s < T::QS; ++s) { mbar_init(&sm.qfull[s], 1); mbar_init(&sm.qempty[s], T::W); }
        fence_mbar_init();
        sm.flag[0] = 0;
        sm.flag[1] = 0;
    }
    // Programmatic dependent launch: without early pages everything waits for
    // the predecessor before the first global read.  The successor, this
    // launch's combine grid, may launch at once: its single-warp CTAs wait in
    // griddepcontrol.wait and fit beside two decode CTAs, and its own early
    // signal lets the next layer's decode launch and stream its first pages
    // while this grid drains.  Three grids can be in flight (this decode, its
    // combine, the next decode); the next decode writes partials only after
    // its own wait, when this grid and its combine are complete, so two
    // alternating partial sets suffice.
    const bool pdl = (p.flags & kDecodePdl) != 0;
    const bool early = pdl && (p.flags & kDecodeEarlyPages) != 0;
    if (pdl && !early) griddep_wait();
    griddep_launch_dependents();
    // The page assignment: from the plan (one round trip for the prefixes,
    // this CTA's range and its first 32 page records), or computed here.
    const bool planned = p.plan != nullptr;
    if (planned) {
        const int* entry = p.plan + kPlanCta + (size_t)blockIdx.x * kPlanCtaInts;
        // (L2 reads: the plan is rewritten by later plan launches)
        for (int i = threadIdx.x; i <= (int)p.B; i += T::THREADS) {
            sm.pfx[i] = __ldcg(p.plan + kPlanPfx + i);
            sm.nzp[i] = __ldcg(p.plan + kPlanNzp + i);
            if (i < (int)p.B) sm.slen[i] = (int)__ldg(p.seq_lens + i);
        }
        if (warp >= T::W) {
            // every producer warp takes the first batch into its own buffer
            if (lane == 0) prefetch_tensormap(&tmap);
            if (warp == T::W && lane < 3) sm.flag[2 + lane] = __ldcg(entry + lane);
            const int4 rec = __ldcg(reinterpret_cast<const int4*>(entry + 4) + lane);
            PageInfo pi;
            pi.kvrow = p.k_new != nullptr ? rec.x : -1;
            pi.row0 = rec.y >= 0 ? rec.y + (int)(p.layer * p.num_blocks * p.Hkv * 32u) : rec.y;
            pi.qseg = rec.z;
            pi.qrow = rec.w;
            sm.pinfo[(warp - T::W) * 64 + lane] = pi;
        }
    } else if (warp == T::W) {
        if (lane == 0) prefetch_tensormap(&tmap);
        warp_prefixes(p.seq_lens, (int)p.B, (int)p.bt_stride, p.err, blockIdx.x == 0, sm.pfx, sm.nzp,
                      sm.slen, lane);
    }
    __syncthreads();
    if (threadIdx.x == 0) VW_TRACE(1, globaltimer());

    int begin, end;
    if (planned) {
        begin = sm.flag[2];
        end = sm.flag[3];
    } else {
        const int total = (int)p.Hkv * sm.pfx[p.B];
        const int cost = (int)p.seg_cost;
        const int vper = virtual_per_cta(virtual_total(total, (int)p.Hkv * sm.nzp[p.B], cost), (int)gridDim.x);
        begin = range_start(sm.pfx, sm.nzp, (int)p.B, (int)p.Hkv, cost, (int)blockIdx.x * vper);
        end = range_start(sm.pfx, sm.nzp, (int)p.B, (int)p.Hkv, cost, ((int)blockIdx.x + 1) * vper);
    }
    if (begin >= end) return;

    if (warp >= T::W) {
        if (warp == T::W && lane == 0) VW_TRACE(15, globaltimer());
        // ordinal of the first segment of this range among non-empty segments
        int first_ord;
        if (planned) {
            first_ord = sm.flag[4];
        } else {
            const int b0 = find_seq(sm.pfx, (int)p.B, (int)p.Hkv, begin);
            const int h0 = (begin - (int)p.Hkv * sm.pfx[b0]) / (sm.pfx[b0 + 1] - sm.pfx[b0]);
            first_ord = sm.nzp[b0] * (int)p.Hkv + h0;
        }
        DecodeParams pp = p;
        if (!early) pp.flags &= ~(kDecodePdl | kDecodeEarlyPages);   // already waited above
        producer<T>(&tmap, pp, sm, begin, end - begin, first_ord, T::PW == 1 ? 0 : warp - T::W,
                    deadline);
    } else {
        if (early) {
            griddep_wait();            // q, k_new, v_new may come from the predecessor
            if (threadIdx.x == 0) VW_TRACE(8, globaltimer());
        }
        consumer<T>(p, sm, begin, end, deadline);
    }
    if (threadIdx.x == 0) VW_TRACE(7, globaltimer());
}

// ------------------------------------------------------------------ combine

// The combine grid is resident next to the decode grids of this layer and the
// next one (it launches before the decode grid ends and waits in
// griddepcontrol.wait), so its CTAs must fit beside two decode CTAs.  The
// register file is split over the SM's four sub-partitions (16,384 each); ten
// 128-register decode warps leave 4,096 in a sub-partition holding three of
// them, so a combine CTA is a single warp of at most 80 registers (2,560),
// and it runs with the decode's shared-memory carveout.  CTA (segment, j) merges query head j of the
// segment, four output elements per lane.
constexpr int kCombineWarps = 1;
constexpr int kCombineThreads = kCombineWarps * 32;
constexpr int kCombineMinBlocks = 25;  // 65,536 / (32 x 25) -> a cap of 80 registers

// Merge of the split-K partials, one CTA per (sequence, KV head) segment.  The
// CTA recomputes the decode grid's page ranges from seq_lens (same clamping,
// same per-CTA quantum), returns at once for a segment that one decode CTA
// finished, and otherwise merges the pieces (o, max, sum) left by decode CTAs
// c0..c1 with weights 2^(max_c - max) -- the merge rule of the online softmax
// in flash_attention.bm:149-157, applied across pieces instead of tokens.
// Launched as a programmatic dependent of its decode grid: the geometry is
// computed while the decode still runs, the partials are read after
// griddepcontrol.wait.  Each thread produces four consecutive output elements.
template <int D, int G, int IO>
__global__ void __launch_bounds__(kCombineThreads, kCombineMinBlocks) combine_kernel(const DecodeParams p, int dec_grid,
                                                                  float vfold) {
    __shared__ int red[kCombineThreads / 32][4];
    if (threadIdx.x == 0) VW_TRACE(12, globaltimer());
    // the next grid (the following layer's decode) may start its prologue now;
    // it waits for this whole grid before it writes anything this grid reads
    griddep_launch_dependents();
    const int Hkv = (int)p.Hkv;
    const int b = (int)blockIdx.x / Hkv, h = (int)blockIdx.x - b * Hkv;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    auto pages = [&](int i) {
        const int sl = (int)__ldcg(p.seq_lens + i);
        const int np = (sl + 15) >> 4;
        return sl <= 0 ? 0 : min(np, (int)p.bt_stride);
    };
    // pages and sequences with pages, before b and in all (the decode's prefixes)
    int before = 0, all = 0, nz_before = 0, nz_all = 0;
    for (int i = threadIdx.x; i < (int)p.B; i += kCombineThreads) {
        const int np = pages(i);
        all += np;
        nz_all += np > 0;
        if (i < b) { before += np; nz_before += np > 0; }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        before += __shfl_xor_sync(0xffffffffu, before, off);
        all += __shfl_xor_sync(0xffffffffu, all, off);
        nz_before += __shfl_xor_sync(0xffffffffu, nz_before, off);
        nz_all += __shfl_xor_sync(0xffffffffu, nz_all, off);
    }
    if (lane == 0) { red[warp][0] = before; red[warp][1] = all; red[warp][2] = nz_before; red[warp][3] = nz_all; }
    __syncthreads();
    before = all = nz_before = nz_all = 0;
#pragma unroll
    for (int w = 0; w < kCombineThreads / 32; ++w) {
        before += red[w][0]; all += red[w][1]; nz_before += red[w][2]; nz_all += red[w][3];
    }
    const int np = pages(b);
    if (np == 0) return;
    const int cost = (int)p.seg_cost;
    const int vper = virtual_per_cta(virtual_total(Hkv * all, Hkv * nz_all, cost), dec_grid);
    const int s_begin = Hkv * before + h * np;
    const int k = Hkv * nz_before + h;        // segment ordinal
    const int v0 = s_begin + cost * k;
    const int c0 = v0 / vper, c1 = (v0 + np - 1) / vper;
    if (c0 == c1) return;                      // written out by the decode CTA itself
    // CTA c0 holds this segment in slot 0 when the segment starts its range
    // (the page before it, of segment k-1, lies in an earlier CTA), else in
    // slot 1 (its last segment); every later CTA starts inside it
    const int slot0 = (k == 0 || (s_begin - 1) + cost * (k - 1) < c0 * vper) ? 0 : 1;
    griddep_wait();
    if (threadIdx.x == 0) VW_TRACE(13, globaltimer());
    const int g = (int)p.group;
    const int n = c1 - c0 + 1;
    const int j = (int)blockIdx.y * kCombineWarps + warp, d = lane * 4;
    if (j < g && d < D) merge_unit<D, G, IO>(p, b, h, j, d, c0, n, slot0, vfold);
    if (threadIdx.x == 0) VW_TRACE(14, globaltimer());
}


// ------------------------------------------------------------------ plan

// One warp per decode CTA: the same prefixes, range and first-batch page
// records the decode prologue computes, written once for all the layers of a
// step.  Page records are resolved as for an appending decode (kvrow set when
// the range holds the segment's last page); a decode without new rows ignores
// kvrow.
__global__ void __launch_bounds__(32) plan_kernel(const DecodeParams p, int* plan) {
    __shared__ int pfx[kMaxBatchPerLaunch + 1], nzp[kMaxBatchPerLaunch + 1];
    const int lane = threadIdx.x;
    const int B = (int)p.B, Hkv = (int)p.Hkv;
    warp_prefixes(p.seq_lens, B, (int)p.bt_stride, p.err, blockIdx.x == 0, pfx, nzp, nullptr, lane);
    __syncwarp();
    if (blockIdx.x == 0) {
        if (lane == 0) {
            plan[0] = B; plan[1] = (int)p.bt_stride; plan[2] = (int)gridDim.x; plan[3] = Hkv;
        }
        for (int i = lane; i <= B; i += 32) { plan[kPlanPfx + i] = pfx[i]; plan[kPlanNzp + i] = nzp[i]; }
    }
    const int total = Hkv * pfx[B];
    const int cost = (int)p.seg_cost;
    const int vper = virtual_per_cta(virtual_total(total, Hkv * nzp[B], cost), (int)gridDim.x);
    const int begin = range_start(pfx, nzp, B, Hkv, cost, (int)blockIdx.x * vper);
    const int end = range_start(pfx, nzp, B, Hkv, cost, ((int)blockIdx.x + 1) * vper);
    int* entry = plan + kPlanCta + (size_t)blockIdx.x * kPlanCtaInts;
    int first_ord = 0;
    if (begin < end) {
        const int b0 = find_seq(pfx, B, Hkv, begin);
        const int h0 = (begin - Hkv * pfx[b0]) / (pfx[b0 + 1] - pfx[b0]);
        first_ord = nzp[b0] * Hkv + h0;
    }
    if (lane == 0) { entry[0] = begin; entry[1] = end; entry[2] = first_ord; entry[3] = 0; }
    int4 rec = make_int4(-1, -32, -1, -1);
    const int n = end - begin, i = lane;
    if (i < n) {
        const int x = begin + i;
        const int b = find_seq(pfx, B, Hkv, x);
        const int np = pfx[b + 1] - pfx[b];
        const int rr = x - Hkv * pfx[b];
        const int h = rr / np, pg = rr - h * np;
        const uint32_t blk = __ldg(p.block_tables + (size_t)b * p.bt_stride + pg);
        if (blk < p.num_blocks) rec.y = (int)((blk * (uint32_t)Hkv + (uint32_t)h) * 32u);
        else set_err(p.err, kDevErrBlockId);
        if (i == 0 || pg == 0) {
            rec.z = nzp[b] * Hkv + h - first_ord;
            rec.w = (int)(b * p.Hq + h * p.group);
            if (i + (np - 1 - pg) < n) rec.x = b * Hkv + h;
        }
    }
    reinterpret_cast<int4*>(entry + 4)[lane] = rec;
}

}  // namespace

cudaError_t launch_decode_plan(const DecodeParams& p, int grid, int* plan, cudaStream_t s) {
    plan_kernel<<<grid, 32, 0, s>>>(p, plan);
    return cudaGetLastError();
}

namespace {

template <class T>
cudaError_t launch_combine(const DecodeLaunch& L) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(L.p.B * L.p.Hkv, (L.p.group + kCombineWarps - 1) / kCombineWarps);
    cfg.blockDim = dim3(kCombineThreads);
    cfg.stream = L.stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, combine_kernel<T::D, T::G, T::IO>, L.p, L.grid, T::VFOLD);
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
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(decode_kernel<T>, cudaFuncAttributePreferredSharedMemoryCarveout,
                                     (int)cudaSharedmemCarveoutMaxShared);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(combine_kernel<T::D, T::G, T::IO>,
                                     cudaFuncAttributePreferredSharedMemoryCarveout,
                                     (int)cudaSharedmemCarveoutMaxShared);
        if (e != cudaSuccess) return e;
        configured.fetch_or(bit);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(L.grid);
    cfg.blockDim = dim3(T::THREADS);
    cfg.dynamicSmemBytes = T::SMEM;
    cfg.stream = L.stream;
    cudaLaunchAttribute attr[1];
    if (L.p.flags & kDecodePdl) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    cudaError_t e = cudaLaunchKernelEx(&cfg, decode_kernel<T>, *L.tmap, L.p);
    if (e != cudaSuccess) return e;
    return launch_combine<T>(L);
}

template <int D, int KV, int IO>
cudaError_t launch_d(const DecodeLaunch& L) {
    if (L.p.group <= 8) return launch_t<Traits<D, 1, KV, IO>>(L);
    return launch_t<Traits<D, 2, KV, IO>>(L);
}

}  // namespace

static_assert(VW_DECODE_GRID_PER_SM >= 1 && VW_DECODE_GRID_PER_SM <= VW_DECODE_CTAS_PER_SM,
              "grid CTAs per SM must be resident together");
int decode_ctas_per_sm() { return VW_DECODE_GRID_PER_SM; }
size_t decode_scratch_floats_o(int grid, int head_dim) { return (size_t)grid * 2 * 16 * head_dim; }
size_t decode_scratch_floats_ml(int grid) { return (size_t)grid * 2 * 16 * 2; }

#ifdef VW_DECODE_TRACE
extern "C" __attribute__((visibility("default"))) int vw_debug_trace(void* host, int reset) {
    cudaMemcpyFromSymbol(host, g_vw_trace, sizeof(g_vw_trace));
    if (reset) {
        static unsigned long long zeros[2 * 1024 * 16];
        cudaMemcpyToSymbol(g_vw_trace, zeros, sizeof(zeros));
    }
    return (int)cudaGetLastError();
}
#endif

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
