// vw_kv_ops.cu -- byte-moving kernels of the paged KV pool: reshape-and-cache
// append, copy-on-write / compaction block copies, and the block-table gather.
//
// All three are HBM-bound copies: a warp moves whole token rows of one KV head
// (D elements) with 8-B or 16-B vector accesses, so it touches whole 32-B
// sectors, and keeps several rows' loads in flight before it stores them.  Pool layout:
//   data  [L][NB][Hkv][2][16][D]   (2 = K, V; element f16/bf16 or an E4M3 code)
//   scale [L][NB][Hkv][2][16]      (FP8 pools only)
// Bounds: every block id and slot is checked against the pool before it is
// used; a bad one sets a bit in the pool's device error word and the row is
// skipped, so no kernel here can write outside the pool.
#include <cuda_runtime.h>
#include <cstdint>

#include "vw_fp8.cuh"
#include "vw_internal.h"
#include "vw_ptx.cuh"

namespace vw {

namespace {

__device__ __forceinline__ float io_f32(uint32_t h, uint32_t io) {
    return io == kBF16 ? bf16_bits_to_f32(h) : f16_bits_to_f32(h);
}

// Row w of a launch over n tokens -> (token i, K or V, KV head h), with w in
// the order [token][K, V][head].  Index math is 32-bit (the host keeps the row
// count below 2^31): a 64-bit division costs ~100 instructions per warp, which
// bounded these short copies by issue rather than by memory.
struct RowIdx {
    uint32_t i, kv, h;
};
__device__ __forceinline__ RowIdx row_index(uint32_t w, uint32_t Hkv) {
    const uint32_t q = w / Hkv;
    return RowIdx{q >> 1, q & 1u, w - q * Hkv};
}

// Pool row (token slot t of block blk, head h, K or V) of a layer.
__device__ __forceinline__ uint64_t pool_row(const PoolGeom& g, uint32_t layer, uint32_t blk, uint32_t h,
                                             uint32_t kv, uint32_t t) {
    return ((((uint64_t)layer * g.num_blocks + blk) * g.num_kv_heads + h) * 2 + kv) * kBlockSize + t;
}

constexpr uint32_t kRowsPerWarp = 4;     // a warp's loads of 4 rows are in flight together

// Reshape-and-cache.  The reference has no append kernel; its paging rule
// (kernels/attention/flash_attention.bm:132-140: token p lives in logical block
// p/16 at slot p%16) defines slot = block_table[p/16]*16 + p%16.  Warp w of the
// grid handles rows 4w .. 4w+3 (token i, kv, head h); negative slots are
// padding and skipped.  16-bit pools: every lane loads its piece of the four
// rows before it stores any; FP8 pools quantise row by row.
__global__ void __launch_bounds__(256) kv_append_kernel(PoolGeom g, uint8_t* __restrict__ data,
                                                        float* __restrict__ scales, uint32_t layer,
                                                        const uint16_t* __restrict__ k_new,
                                                        const uint16_t* __restrict__ v_new,
                                                        const int64_t* __restrict__ slots,
                                                        uint32_t n, uint32_t* err) {
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t w0 = (blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * kRowsPerWarp;
    const uint32_t rows = n * 2u * g.num_kv_heads;
    const uint32_t D = g.head_dim;
    if (g.kv_kind != kFP8) {
        // D 16-bit elements = D/4 u64 words per row: one word per lane (D 128) or
        // one per lane of the first half-warp (D 64)
        const bool active = lane < D / 4;
        uint64_t v[kRowsPerWarp];
        uint64_t* dst[kRowsPerWarp];
#pragma unroll
        for (uint32_t r = 0; r < kRowsPerWarp; ++r) {
            dst[r] = nullptr;
            const uint32_t w = w0 + r;
            if (w >= rows) continue;
            const RowIdx x = row_index(w, g.num_kv_heads);
            const int64_t slot = __ldg(slots + x.i);
            if (slot < 0) continue;
            if (slot >= (int64_t)g.num_blocks * kBlockSize) {
                if (lane == 0) atomicOr(err, kDevErrSlot);
                continue;
            }
            const uint16_t* src = (x.kv == 0 ? k_new : v_new) + ((size_t)x.i * g.num_kv_heads + x.h) * D;
            if (active) v[r] = __ldg(reinterpret_cast<const uint64_t*>(src) + lane);
            dst[r] = reinterpret_cast<uint64_t*>(
                data + pool_row(g, layer, (uint32_t)(slot / kBlockSize), x.h, x.kv,
                                (uint32_t)(slot % kBlockSize)) * D * 2);
        }
#pragma unroll
        for (uint32_t r = 0; r < kRowsPerWarp; ++r)
            if (dst[r] && active) dst[r][lane] = v[r];
        return;
    }
    // FP8: 4 elements per lane (head_dim 128), one row at a time (the row's
    // scale needs the whole row's maximum)
    for (uint32_t r = 0; r < kRowsPerWarp; ++r) {
        const uint32_t w = w0 + r;
        if (w >= rows) return;
        const RowIdx x = row_index(w, g.num_kv_heads);
        const int64_t slot = __ldg(slots + x.i);
        if (slot < 0) continue;
        if (slot >= (int64_t)g.num_blocks * kBlockSize) {
            if (lane == 0) atomicOr(err, kDevErrSlot);
            continue;
        }
        const uint16_t* src = (x.kv == 0 ? k_new : v_new) + ((size_t)x.i * g.num_kv_heads + x.h) * D;
        const uint64_t row = pool_row(g, layer, (uint32_t)(slot / kBlockSize), x.h, x.kv,
                                      (uint32_t)(slot % kBlockSize));
        const uint2 raw = __ldg(reinterpret_cast<const uint2*>(src) + lane);
        float v[4] = {io_f32(raw.x & 0xFFFFu, g.io_kind), io_f32(raw.x >> 16, g.io_kind),
                      io_f32(raw.y & 0xFFFFu, g.io_kind), io_f32(raw.y >> 16, g.io_kind)};
        float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
        const float scale = fp8_row_scale(amax);
        *reinterpret_cast<uint32_t*>(data + row * D + lane * 4) = fp8_encode4(v, scale, g.fp8_ocp != 0);
        if (lane == 0) scales[row] = scale;
    }
}

// Block copy for copy-on-write and compaction moves (no reference counterpart;
// the decision point is the ref-count in engine/kv_cache.bm:94-113).  CTA
// (pair, layer) copies that layer's K and V rows of every head, plus the FP8
// scales, from block src to block dst with 16-B accesses, eight loads in
// flight per thread before their stores.  Pairs must have distinct
// destinations that are not sources in the same call.
constexpr uint32_t kCopyUnroll = 8;

__global__ void __launch_bounds__(256) block_copy_kernel(PoolGeom g, uint8_t* __restrict__ data,
                                                         float* __restrict__ scales,
                                                         const uint32_t* __restrict__ pairs,
                                                         uint32_t n, uint32_t* err) {
    const uint32_t pi = blockIdx.x, layer = blockIdx.y;
    if (pi >= n) return;
    const uint32_t src = __ldg(pairs + 2 * pi), dst = __ldg(pairs + 2 * pi + 1);
    if (src >= g.num_blocks || dst >= g.num_blocks) {
        if (threadIdx.x == 0) atomicOr(err, kDevErrBlockId);
        return;
    }
    const uint32_t bytes = 2u * g.num_kv_heads * kBlockSize * g.head_dim * (uint32_t)elem_bytes(g.kv_kind);
    const uint4* s = reinterpret_cast<const uint4*>(data + ((uint64_t)layer * g.num_blocks + src) * bytes);
    uint4* d = reinterpret_cast<uint4*>(data + ((uint64_t)layer * g.num_blocks + dst) * bytes);
    const uint32_t n16 = bytes / 16;
    for (uint32_t k0 = threadIdx.x; k0 < n16; k0 += blockDim.x * kCopyUnroll) {
        uint4 v[kCopyUnroll];
#pragma unroll
        for (uint32_t j = 0; j < kCopyUnroll; ++j) {
            const uint32_t k = k0 + j * blockDim.x;
            if (k < n16) v[j] = __ldg(s + k);
        }
#pragma unroll
        for (uint32_t j = 0; j < kCopyUnroll; ++j) {
            const uint32_t k = k0 + j * blockDim.x;
            if (k < n16) d[k] = v[j];
        }
    }
    if (g.kv_kind == kFP8) {
        const uint32_t ns = 2u * g.num_kv_heads * kBlockSize;
        const float* ss = scales + ((uint64_t)layer * g.num_blocks + src) * ns;
        float* ds = scales + ((uint64_t)layer * g.num_blocks + dst) * ns;
        for (uint32_t k = threadIdx.x; k < ns; k += blockDim.x) ds[k] = __ldg(ss + k);
    }
}

// Block-table gather of one sequence: raw rows into out_k/out_v
// [Hkv][seq_len][D] and, for FP8, their scales [Hkv][seq_len].  Follows the
// paging walk of kernels/attention/flash_attention.bm:132-140.  Warp w moves
// rows 4w .. 4w+3 ([position][K, V][head] order), all four loads in flight
// before the stores.
__global__ void __launch_bounds__(256) kv_gather_kernel(PoolGeom g, const uint8_t* __restrict__ data,
                                                        const float* __restrict__ scales,
                                                        uint32_t layer,
                                                        const uint32_t* __restrict__ block_table,
                                                        uint32_t seq_len, uint8_t* __restrict__ out_k,
                                                        uint8_t* __restrict__ out_v,
                                                        float* __restrict__ out_ks,
                                                        float* __restrict__ out_vs, uint32_t* err) {
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t w0 = (blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * kRowsPerWarp;
    const uint32_t rows = seq_len * 2u * g.num_kv_heads;
    const uint32_t rb = g.head_dim * (uint32_t)elem_bytes(g.kv_kind);   // 64, 128 or 256 B
    const uint32_t words = rb / 8;                                       // u64 words per row
    const bool active = lane < words;
    uint64_t v[kRowsPerWarp];
    uint64_t* dst[kRowsPerWarp];
#pragma unroll
    for (uint32_t r = 0; r < kRowsPerWarp; ++r) {
        dst[r] = nullptr;
        const uint32_t w = w0 + r;
        if (w >= rows) continue;
        const RowIdx x = row_index(w, g.num_kv_heads);      // x.i = the position p
        const uint32_t blk = __ldg(block_table + x.i / kBlockSize);
        if (blk >= g.num_blocks) {
            if (lane == 0) atomicOr(err, kDevErrBlockId);
            continue;
        }
        const uint64_t row = pool_row(g, layer, blk, x.h, x.kv, x.i % kBlockSize);
        const uint64_t o = (uint64_t)x.h * seq_len + x.i;
        if (active) v[r] = __ldg(reinterpret_cast<const uint64_t*>(data + row * rb) + lane);
        dst[r] = reinterpret_cast<uint64_t*>((x.kv == 0 ? out_k : out_v) + o * rb);
        if (g.kv_kind == kFP8 && lane == 0) (x.kv == 0 ? out_ks : out_vs)[o] = __ldg(scales + row);
    }
#pragma unroll
    for (uint32_t r = 0; r < kRowsPerWarp; ++r)
        if (dst[r] && active) dst[r][lane] = v[r];
}

}  // namespace

cudaError_t launch_kv_append(const PoolGeom& g, uint8_t* data, float* scales, uint32_t layer,
                             const void* k_new, const void* v_new, const int64_t* slots,
                             uint32_t n, uint32_t* err, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    const uint64_t rows = (uint64_t)n * 2 * g.num_kv_heads;
    const unsigned grid = (unsigned)((rows + 8 * kRowsPerWarp - 1) / (8 * kRowsPerWarp));
    kv_append_kernel<<<grid, 256, 0, s>>>(g, data, scales, layer,
                                          static_cast<const uint16_t*>(k_new),
                                          static_cast<const uint16_t*>(v_new), slots, n, err);
    return cudaGetLastError();
}

cudaError_t launch_block_copy(const PoolGeom& g, uint8_t* data, float* scales,
                              const uint32_t* pairs, uint32_t n, uint32_t* err, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    block_copy_kernel<<<dim3(n, g.num_layers), 256, 0, s>>>(g, data, scales, pairs, n, err);
    return cudaGetLastError();
}

cudaError_t launch_kv_gather(const PoolGeom& g, const uint8_t* data, const float* scales,
                             uint32_t layer, const uint32_t* block_table, uint32_t seq_len,
                             void* out_k, void* out_v, float* out_ks, float* out_vs,
                             uint32_t* err, cudaStream_t s) {
    if (seq_len == 0) return cudaSuccess;
    const uint64_t rows = (uint64_t)seq_len * 2 * g.num_kv_heads;
    const unsigned grid = (unsigned)((rows + 8 * kRowsPerWarp - 1) / (8 * kRowsPerWarp));
    kv_gather_kernel<<<grid, 256, 0, s>>>(g, data, scales, layer, block_table, seq_len,
                                          static_cast<uint8_t*>(out_k), static_cast<uint8_t*>(out_v),
                                          out_ks, out_vs, err);
    return cudaGetLastError();
}

}  // namespace vw
