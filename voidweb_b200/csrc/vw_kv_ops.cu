// vw_kv_ops.cu -- byte-moving kernels of the paged KV pool: reshape-and-cache
// append, copy-on-write / compaction block copies, and the block-table gather.
//
// All three are HBM-bound copies: one warp moves one token row of one KV head
// (D elements) with 16-B (or 8-B) vector accesses, so a warp touches whole 32-B
// sectors and consecutive warps walk consecutive rows.  Pool layout:
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

// Reshape-and-cache.  The reference has no append kernel; its paging rule
// (kernels/attention/flash_attention.bm:132-140: token p lives in logical block
// p/16 at slot p%16) defines slot = block_table[p/16]*16 + p%16.  Warp w of the
// grid handles row (token i, kv, head h); negative slots are padding and skipped.
__global__ void __launch_bounds__(256) kv_append_kernel(PoolGeom g, uint8_t* __restrict__ data,
                                                        float* __restrict__ scales, uint32_t layer,
                                                        const uint16_t* __restrict__ k_new,
                                                        const uint16_t* __restrict__ v_new,
                                                        const int64_t* __restrict__ slots,
                                                        uint32_t n, uint32_t* err) {
    const uint32_t lane = threadIdx.x & 31;
    const uint64_t w = (uint64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const uint64_t rows = (uint64_t)n * 2 * g.num_kv_heads;
    if (w >= rows) return;
    const uint32_t h = (uint32_t)(w % g.num_kv_heads);
    const uint32_t kv = (uint32_t)((w / g.num_kv_heads) & 1);
    const uint32_t i = (uint32_t)(w / (2ull * g.num_kv_heads));
    const int64_t slot = slots[i];
    if (slot < 0) return;
    if (slot >= (int64_t)g.num_blocks * kBlockSize) {
        if (lane == 0) atomicOr(err, kDevErrSlot);
        return;
    }
    const uint64_t blk = (uint64_t)slot / kBlockSize, t = (uint64_t)slot % kBlockSize;
    const uint64_t row = ((((uint64_t)layer * g.num_blocks + blk) * g.num_kv_heads + h) * 2 + kv) *
                             kBlockSize + t;
    const uint16_t* src = (kv == 0 ? k_new : v_new) + ((uint64_t)i * g.num_kv_heads + h) * g.head_dim;
    if (g.kv_kind != kFP8) {
        // bit copy of D 16-bit elements: D*2/8 u64 words, lane-strided
        const uint64_t* s64 = reinterpret_cast<const uint64_t*>(src);
        uint64_t* d64 = reinterpret_cast<uint64_t*>(data + row * g.head_dim * 2);
        for (uint32_t k = lane; k < g.head_dim / 4; k += 32) d64[k] = s64[k];
        return;
    }
    // FP8: 4 elements per lane per step (head_dim 128 -> exactly one step)
    float amax = 0.0f;
    for (uint32_t d = lane * 4; d < g.head_dim; d += 128) {
        const uint2 raw = *reinterpret_cast<const uint2*>(src + d);
        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(io_f32(raw.x & 0xFFFFu, g.io_kind)),
                                       fabsf(io_f32(raw.x >> 16, g.io_kind))),
                                 fmaxf(fabsf(io_f32(raw.y & 0xFFFFu, g.io_kind)),
                                       fabsf(io_f32(raw.y >> 16, g.io_kind)))));
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    const float scale = fp8_row_scale(amax);
    for (uint32_t d = lane * 4; d < g.head_dim; d += 128) {
        const uint2 raw = *reinterpret_cast<const uint2*>(src + d);
        float v[4] = {io_f32(raw.x & 0xFFFFu, g.io_kind), io_f32(raw.x >> 16, g.io_kind),
                      io_f32(raw.y & 0xFFFFu, g.io_kind), io_f32(raw.y >> 16, g.io_kind)};
        *reinterpret_cast<uint32_t*>(data + row * g.head_dim + d) = fp8_encode4(v, scale, g.fp8_ocp != 0);
    }
    if (lane == 0) scales[row] = scale;
}

// Block copy for copy-on-write and compaction moves (no reference counterpart;
// the decision point is the ref-count in engine/kv_cache.bm:94-113).  CTA
// (pair, layer) copies that layer's K and V rows of every head, plus the FP8
// scales, from block src to block dst with 16-B accesses.  Pairs must have
// distinct destinations that are not sources in the same call.
__global__ void __launch_bounds__(256) block_copy_kernel(PoolGeom g, uint8_t* __restrict__ data,
                                                         float* __restrict__ scales,
                                                         const uint32_t* __restrict__ pairs,
                                                         uint32_t n, uint32_t* err) {
    const uint32_t pi = blockIdx.x, layer = blockIdx.y;
    if (pi >= n) return;
    const uint32_t src = pairs[2 * pi], dst = pairs[2 * pi + 1];
    if (src >= g.num_blocks || dst >= g.num_blocks) {
        if (threadIdx.x == 0) atomicOr(err, kDevErrBlockId);
        return;
    }
    const uint64_t bytes = 2ull * g.num_kv_heads * kBlockSize * g.head_dim * elem_bytes(g.kv_kind);
    const uint4* s = reinterpret_cast<const uint4*>(data + ((uint64_t)layer * g.num_blocks + src) * bytes);
    uint4* d = reinterpret_cast<uint4*>(data + ((uint64_t)layer * g.num_blocks + dst) * bytes);
    const uint64_t n16 = bytes / 16;
    for (uint64_t k = threadIdx.x; k < n16; k += blockDim.x) d[k] = s[k];
    if (g.kv_kind == kFP8) {
        const uint64_t ns = 2ull * g.num_kv_heads * kBlockSize;
        const float* ss = scales + ((uint64_t)layer * g.num_blocks + src) * ns;
        float* ds = scales + ((uint64_t)layer * g.num_blocks + dst) * ns;
        for (uint64_t k = threadIdx.x; k < ns; k += blockDim.x) ds[k] = ss[k];
    }
}

// Block-table gather of one sequence: raw rows into out_k/out_v
// [Hkv][seq_len][D] and, for FP8, their scales [Hkv][seq_len].  Follows the
// paging walk of kernels/attention/flash_attention.bm:132-140.
__global__ void __launch_bounds__(256) kv_gather_kernel(PoolGeom g, const uint8_t* __restrict__ data,
                                                        const float* __restrict__ scales,
                                                        uint32_t layer,
                                                        const uint32_t* __restrict__ block_table,
                                                        uint32_t seq_len, uint8_t* __restrict__ out_k,
                                                        uint8_t* __restrict__ out_v,
                                                        float* __restrict__ out_ks,
                                                        float* __restrict__ out_vs, uint32_t* err) {
    const uint32_t lane = threadIdx.x & 31;
    const uint64_t w = (uint64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const uint64_t rows = (uint64_t)seq_len * 2 * g.num_kv_heads;
    if (w >= rows) return;
    const uint32_t h = (uint32_t)(w % g.num_kv_heads);
    const uint32_t kv = (uint32_t)((w / g.num_kv_heads) & 1);
    const uint32_t p = (uint32_t)(w / (2ull * g.num_kv_heads));
    const uint32_t blk = block_table[p / kBlockSize];
    if (blk >= g.num_blocks) {
        if (lane == 0) atomicOr(err, kDevErrBlockId);
        return;
    }
    const uint64_t row = ((((uint64_t)layer * g.num_blocks + blk) * g.num_kv_heads + h) * 2 + kv) *
                             kBlockSize + p % kBlockSize;
    const uint64_t rb = (uint64_t)g.head_dim * elem_bytes(g.kv_kind);
    const uint64_t o = (uint64_t)h * seq_len + p;
    const uint64_t* s = reinterpret_cast<const uint64_t*>(data + row * rb);
    uint64_t* d = reinterpret_cast<uint64_t*>((kv == 0 ? out_k : out_v) + o * rb);
    for (uint32_t k = lane; k < rb / 8; k += 32) d[k] = s[k];
    if (g.kv_kind == kFP8 && lane == 0) (kv == 0 ? out_ks : out_vs)[o] = scales[row];
}

}  // namespace

cudaError_t launch_kv_append(const PoolGeom& g, uint8_t* data, float* scales, uint32_t layer,
                             const void* k_new, const void* v_new, const int64_t* slots,
                             uint32_t n, uint32_t* err, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    const uint64_t rows = (uint64_t)n * 2 * g.num_kv_heads;
    const unsigned grid = (unsigned)((rows + 7) / 8);
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
    const unsigned grid = (unsigned)((rows + 7) / 8);
    kv_gather_kernel<<<grid, 256, 0, s>>>(g, data, scales, layer, block_table, seq_len,
                                          static_cast<uint8_t*>(out_k), static_cast<uint8_t*>(out_v),
                                          out_ks, out_vs, err);
    return cudaGetLastError();
}

}  // namespace vw
