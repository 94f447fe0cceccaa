// vw_internal.h -- structures shared by the kernels (.cu) and the C-ABI layer.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace vw {

enum KvKind : uint32_t { kF16 = 0, kBF16 = 1, kFP8 = 2 };

constexpr int kBlockSize = 16;          // tokens per page (engine/engine.bm:102)
constexpr int kMaxBatchPerLaunch = 1024; // sequences per decode launch (prefix tables in smem)
constexpr int kMinPagesPerCta = 8;      // work quantum when the batch is tiny
constexpr int kMaxSegmentCost = 64;     // bound of DecodeParams::seg_cost

// Everything a decode launch needs besides the tensor map.
struct DecodeParams {
    const void* q;              // [B][Hq][D] io dtype
    void* out;                  // [B][Hq][D] io dtype
    const void* k_new;          // [B][Hkv][D] io dtype, or null (decode only)
    const void* v_new;
    const uint32_t* block_tables;   // [B][bt_stride]
    const uint32_t* seq_lens;       // [B], context length including the new token
    uint8_t* kv_data;           // pool pages (append writes)
    float* kv_scales;           // FP8 scales [L][NB][Hkv][2][16]
    float* part_o;              // [grid][2][G][D] split-K partial outputs
    float* part_ml;             // [grid][2][G][2] (running max, sum)
    uint32_t* err;              // device error word
    const int* plan;            // page assignment written by the plan kernel (kDecodePlanned)
    uint32_t B, Hq, Hkv, group, num_blocks, layer, bt_stride, fp8_ocp;
    float scale_log2;           // softmax scale * log2(e)
    float rope_theta;           // > 0: rotate q and the new K row (RoPE) at position seq_len-1
    uint32_t flags;             // kDecodePdl | kDecodeEarlyPages | kDecodePlanned
    uint32_t seg_cost;          // virtual pages per segment boundary in the CTA split (<= kMaxSegmentCost)
    uint64_t wait_cycles;       // bound of the device waits in SM cycles (0: kWaitDeadlineCycles)
};

constexpr uint32_t kDecodePdl = 0x1u;
constexpr uint32_t kDecodeEarlyPages = 0x2u;
constexpr uint32_t kDecodePlanned = 0x4u;
// The consumer warps read the first segment's query rows (and new K/V rows)
// straight from global memory after the dependency wait, instead of waiting
// for the producer's bulk copy of them into the query ring.
constexpr uint32_t kDecodeDirectQ = 0x200u;
// Test hook (vw_debug_set_wait_limit): the producer withholds the query-tile
// copies, so the consumers' first wait is one that nothing completes and runs
// out at the (shortened) deadline.
constexpr uint32_t kDecodeWithholdQ = 0x400u;

// Decode plan (int32 words): a header {B, bt_stride, grid, Hkv}, the exclusive
// prefixes of pages and of sequences with pages over the batch, then one entry
// per decode CTA: {begin, end, first segment ordinal, 0} and the 32 page records
// of its first batch ({kvrow, row0 without the layer offset, qseg, qrow}).
constexpr int kPlanPfx = 4;
constexpr int kPlanNzp = kPlanPfx + kMaxBatchPerLaunch + 1;
constexpr int kPlanCta = (kPlanNzp + kMaxBatchPerLaunch + 1 + 3) / 4 * 4;
constexpr int kPlanCtaInts = 4 + 32 * 4;
inline size_t plan_ints(int grid) { return (size_t)kPlanCta + (size_t)grid * kPlanCtaInts; }
// p carries the batch (B, Hq, Hkv, group, bt_stride, num_blocks, tables,
// seq_lens, err); plan receives plan_ints(grid) words.
cudaError_t launch_decode_plan(const DecodeParams& p, int grid, int* plan, cudaStream_t s);

struct DecodeLaunch {
    DecodeParams p;
    const CUtensorMap* tmap;    // host copy, passed by value as a __grid_constant__
    uint32_t head_dim, kv_kind, io_kind;
    int grid;
    cudaStream_t stream;
};

// Returns cudaSuccess or the launch error.  Unsupported shapes must have been
// rejected by the caller.
cudaError_t launch_paged_decode(const DecodeLaunch& L);
int decode_ctas_per_sm();
size_t decode_scratch_floats_o(int grid, int head_dim);
size_t decode_scratch_floats_ml(int grid);

// Paged prefill (chunked prefill over the pool): sequence b's chunk of
// n_b = cu_q[b+1] - cu_q[b] tokens sits at positions ctx_start[b] + i.
struct PrefillParams {
    const void* q;              // [T][Hq][D] io dtype (packed chunk tokens of all sequences)
    void* out;                  // [T][Hq][D] io dtype
    const int32_t* cu_q;        // [B+1] token offsets of the chunks
    const int32_t* ctx_start;   // [B] tokens cached before each chunk
    const uint32_t* block_tables;   // [B][bt_stride]
    const uint8_t* kv_data;     // pool pages (FP8 pools: the codes the decoder warps read)
    const float* kv_scales;     // FP8 scales [L][NB][Hkv][2][16]
    uint32_t* err;              // device error word
    uint32_t B, T, Hq, Hkv, group, num_blocks, layer, bt_stride, causal, flags;
    float scale_log2;           // softmax scale * log2(e)
    float rope_theta;           // > 0: rotate q at its position (RoPE)
    // bound of the device waits in SM cycles (0: kWaitDeadlineCycles); when set
    // (vw_debug_set_wait_limit) the K/V tiles are withheld, so the first waits
    // are ones that nothing completes and run out
    uint64_t wait_cycles;
};

struct PrefillLaunch {
    PrefillParams p;
    const CUtensorMap* tmap;    // the pool's 16-row half-page-head map
    uint32_t head_dim, kv_kind, io_kind;
    cudaStream_t stream;
};

// Returns cudaSuccess or the launch error; shapes were validated by the caller.
cudaError_t launch_paged_prefill(const PrefillLaunch& L);
int prefill_query_tile();

struct PoolGeom {
    uint32_t num_layers, num_kv_heads, head_dim, num_blocks, kv_kind, io_kind, fp8_ocp;
};

cudaError_t launch_kv_append(const PoolGeom& g, uint8_t* data, float* scales, uint32_t layer,
                             const void* k_new, const void* v_new, const int64_t* slots,
                             uint32_t n, uint32_t* err, cudaStream_t s);
cudaError_t launch_block_copy(const PoolGeom& g, uint8_t* data, float* scales,
                              const uint32_t* pairs, uint32_t n, uint32_t* err, cudaStream_t s);
// Chunk append of a prefill: token i of sequence b (cu_q[b] <= i < cu_q[b+1]) at
// position ctx_start[b] + i - cu_q[b] goes to slot
// block_tables[b][p/16] * 16 + p % 16; K rows rotated first when rope_theta > 0.
cudaError_t launch_prefill_append(const PoolGeom& g, uint8_t* data, float* scales, uint32_t layer,
                                  const void* k_new, const void* v_new, const int32_t* cu_q,
                                  const int32_t* ctx_start, const uint32_t* block_tables,
                                  uint32_t bt_stride, uint32_t B, uint32_t T, float rope_theta,
                                  uint32_t* err, cudaStream_t s);
// FP8 weight path (vw_fp8w.cu): RMSNorm with E4M3 output and the E4M3 GEMM.
cudaError_t launch_rms_norm_fp8(const void* x, const void* w, uint8_t* out, uint32_t rows, uint32_t hidden,
                                float scale, float eps, cudaStream_t s);
cudaError_t launch_gemm_fp8(const uint8_t* a, const uint8_t* b, void* c, const void* bias, uint32_t M,
                            uint32_t N, uint32_t K, float a_scale, float b_scale, cudaStream_t s);
cudaError_t fp8w_error(uint32_t* word, bool clear);
cudaError_t launch_kv_gather(const PoolGeom& g, const uint8_t* data, const float* scales,
                             uint32_t layer, const uint32_t* block_table, uint32_t seq_len,
                             void* out_k, void* out_v, float* out_ks, float* out_vs,
                             uint32_t* err, cudaStream_t s);

#ifdef __CUDACC__
__host__ __device__
#endif
inline size_t elem_bytes(uint32_t kv_kind) { return kv_kind == kFP8 ? 1 : 2; }

}  // namespace vw
