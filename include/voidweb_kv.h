/* voidweb_kv.h -- C ABI of the B200 paged KV-cache library (libvoidweb_kv.so).
 *
 * Drop-in boundary for VOIDWEB's paged KV-cache hot path.  The engine binds
 * exactly one symbol of its kernel library, voidweb_forward_pass, through
 * dlopen/dlsym (engine/ffi.bm:61-77) with the packed ForwardArgs /
 * SeqDescriptor structs (engine/ffi.bm:15-40); that symbol is declared at the
 * end of this header.  The op-level entry points below are the library-side
 * surface behind it: the reference's launcher
 * launch_paged_attn_decode(q, kv_cache, block_table, seq_lens, o)
 * (kernels/attention/flash_attention.bm:180-189) plus the append, block-copy,
 * gather and FP8 operations the engine's block manager and radix tree need
 * (engine/kv_cache.bm, radix_cache/radix_cache.bm), and the host block manager
 * and radix tree themselves.
 *
 * Conventions (engine/ffi.bm:112-118): every function returns int32_t, 0 on
 * success, a nonzero vw_status otherwise; vw_last_error() returns a message
 * for the calling thread.  Device pointers are plain CUDA device addresses;
 * `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 * Nothing here throws across the boundary.
 *
 * Pool layout in HBM (a block id addresses 16 token slots in every layer,
 * engine/engine.bm:170-182):
 *   data  [num_layers][num_blocks][num_kv_heads][2][16][head_dim]
 *         (2 = K, V; element = f16, bf16, or one E4M3 code byte), i.e. the
 *         reference's per-head page kv_cache[block][2][16][HEAD_DIM]
 *         (kernels/attention/flash_attention.bm:116) stacked over heads,
 *         blocks and layers; one head's K and V page is contiguous
 *   scale [num_layers][num_blocks][num_kv_heads][2][16]  f32, FP8 pools only
 */
#ifndef VOIDWEB_KV_H
#define VOIDWEB_KV_H

#include <stdint.h>

#if defined(__GNUC__)
#define VW_API __attribute__((visibility("default")))
#else
#define VW_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define VW_BLOCK_SIZE 16

typedef enum {
    VW_OK = 0,
    VW_ERR_INVALID_ARG = 1,   /* a size, pointer or alignment was rejected before launch */
    VW_ERR_UNSUPPORTED = 2,   /* a valid but unimplemented shape (e.g. head_dim 96) */
    VW_ERR_CUDA = 3,          /* a CUDA runtime call failed */
    VW_ERR_OOM = 4,           /* device or block-pool allocation failed */
    VW_ERR_DEVICE_CHECK = 5   /* a kernel's bounds check tripped (vw_pool_check) */
} vw_status;

typedef enum { VW_F16 = 0, VW_BF16 = 1, VW_FP8_E4M3 = 2 } vw_dtype;

/* FP8 codec: the reference's truncating encoder (kernels/norm/rms_norm.bm:98-113)
 * is the default; OCP E4M3FN round-to-nearest-even saturating is optional. */
typedef enum { VW_FP8_REFERENCE = 0, VW_FP8_OCP = 1 } vw_fp8_mode;

/* Device error word bits returned by vw_pool_check. */
#define VW_DEV_ERR_BLOCK_ID 0x1u  /* a block id >= num_blocks was seen and skipped */
#define VW_DEV_ERR_SEQ_LEN 0x2u   /* seq_len == 0 or longer than its block-table row */
#define VW_DEV_ERR_TIMEOUT 0x4u   /* a bounded device wait gave up */
#define VW_DEV_ERR_SLOT 0x8u      /* an append slot was outside the pool */
#define VW_DEV_ERR_LAUNCH 0x10u   /* a kernel found its launch unusable and did nothing */

typedef struct vw_pool vw_pool;

typedef struct {
    uint32_t num_layers;
    uint32_t num_kv_heads;
    uint32_t head_dim;       /* 64 or 128 (FP8 pools: 128) */
    uint32_t num_blocks;     /* pool size in 16-token blocks, shared by all layers */
    uint32_t kv_dtype;       /* vw_dtype of the pages */
    uint32_t io_dtype;       /* VW_F16 or VW_BF16: q, new K/V rows, outputs; equals
                                kv_dtype unless the pool is FP8 */
    uint32_t fp8_mode;       /* vw_fp8_mode */
    uint32_t max_batch;      /* most sequences one decode call may carry (<= 1024) */
    int32_t device;          /* CUDA device ordinal */
    uint32_t reserved;       /* must be 0 */
    void* kv_data;           /* optional caller-owned device buffer (NULL: allocate) */
    void* kv_scales;         /* optional caller-owned FP8 scale buffer (NULL: allocate) */
} vw_pool_config;

/* Replaces: the pool the engine sizes in Engine::load (engine/engine.bm:98-104)
 * and keeps implicitly behind voidweb_forward_pass.  Allocates the pages
 * (unless given), the split-K scratch and the device error word. */
VW_API int32_t vw_pool_create(const vw_pool_config* cfg, vw_pool** out);
VW_API int32_t vw_pool_destroy(vw_pool* pool);
/* Device addresses and byte sizes of the page and scale buffers. */
VW_API int32_t vw_pool_info(const vw_pool* pool, void** kv_data, void** kv_scales,
                     uint64_t* data_bytes, uint64_t* scale_bytes);
/* Synchronises the device, returns the device error word in *device_error and
 * clears it.  Returns VW_ERR_DEVICE_CHECK when the word was nonzero. */
VW_API int32_t vw_pool_check(vw_pool* pool, uint32_t* device_error);

/* Reshape-and-cache (no reference kernel; paging rule of
 * flash_attention.bm:132-140).  k_new, v_new: [num_tokens][num_kv_heads][head_dim]
 * io dtype; slot_mapping: [num_tokens] int64, slot = block*16 + offset, a
 * negative slot skips the token.  FP8 pools quantise each row on the way in. */
VW_API int32_t vw_kv_append(vw_pool* pool, uint32_t layer, const void* k_new, const void* v_new,
                     const int64_t* slot_mapping, uint32_t num_tokens, void* stream);

typedef struct {
    uint32_t layer;
    uint32_t num_seqs;
    uint32_t num_q_heads;          /* multiple of num_kv_heads; group <= 16 */
    uint32_t block_table_stride;   /* entries per block-table row */
    const void* q;                 /* [num_seqs][num_q_heads][head_dim] io dtype */
    const uint32_t* block_tables;  /* [num_seqs][block_table_stride] physical block ids */
    const uint32_t* seq_lens;      /* [num_seqs] context length, including the new token */
    void* out;                     /* [num_seqs][num_q_heads][head_dim] io dtype */
    const void* k_new;             /* optional fused append: [num_seqs][num_kv_heads][head_dim] */
    const void* v_new;             /*   written at position seq_len-1 before attending */
    float scale;                   /* softmax scale; 0 means 1/sqrt(head_dim) (flash_attention.bm:187) */
    uint32_t flags;                /* VW_DECODE_* bits below, 0 for a plain launch */
    float rope_theta;              /* with VW_DECODE_ROPE: the RoPE base (ModelConfig rope_theta) */
    uint32_t reserved;             /* must be 0 */
} vw_decode_args;

/* Rotary position embedding fused into the decode (kernels/rope/rope.bm:22-52,
 * rotate-half pairs (d, d + head_dim/2), theta_d = rope_theta^(-2d/head_dim)):
 * q of every query head and the new K row (with k_new) are rotated to position
 * seq_len-1 and rounded to the io type before use, as a separate RoPE pass
 * over q and k would leave them; the pool stores rotated K.  V is unchanged. */
#define VW_DECODE_ROPE 0x8u

/* Launch as a programmatic dependent of the previous kernel on the stream: the
 * kernel may start while its predecessor drains and waits for it before
 * reading q, k_new, v_new (and, without VW_DECODE_EARLY_PAGES, anything).
 * Each call is a decode grid followed by a small combine grid on the same
 * stream; consecutive calls on one stream may overlap and stay correct. */
#define VW_DECODE_PDL 0x1u
/* With VW_DECODE_PDL: the caller guarantees that the preceding kernel writes
 * neither the block tables, nor seq_lens, nor this layer's pages, so the
 * kernel starts streaming pages before the predecessor finishes. */
#define VW_DECODE_EARLY_PAGES 0x2u

/* With a plan (vw_decode_plan) of the same block tables, seq_lens, num_seqs,
 * stride and query heads: the launch takes its page assignment from the plan
 * instead of computing it.  With VW_DECODE_EARLY_PAGES the plan is read before
 * the predecessor finishes, so the predecessor must not be the plan launch
 * itself (launch the step's first layer without VW_DECODE_EARLY_PAGES). */
#define VW_DECODE_PLANNED 0x4u

/* Replaces: launch_paged_attn_decode (kernels/attention/flash_attention.bm:180-189,
 * kernel :113-162), generalised to GQA and split-K; with k_new/v_new set it is
 * also the append of the step's token (one launch per layer).  Device pointers;
 * all of them 16-byte aligned.  Calls on one stream are ordered; calls of one
 * pool on different streams must not run at the same time (they share the
 * pool's split-K scratch). */
VW_API int32_t vw_paged_decode(vw_pool* pool, const vw_decode_args* args, void* stream);

/* Page assignment of a decode batch, computed once and reused by every layer's
 * vw_paged_decode with VW_DECODE_PLANNED (no counterpart in the reference,
 * whose decode has one CTA per sequence): each decode CTA's range of pages, its
 * first page records and the batch prefixes, in pool memory.  block_tables and
 * seq_lens are the device arrays the decodes will pass; their contents must not
 * change until the next plan.  One plan per pool: a new plan replaces it, in
 * stream order.  On the 28-layer Qwen2.5-7B batch-16 step the plan launch
 * costs more than it saves (early page streaming already hides the decode's
 * own prologue behind the previous layer), so it is an option, not a default. */
VW_API int32_t vw_decode_plan(vw_pool* pool, const uint32_t* block_tables, const uint32_t* seq_lens,
                              uint32_t num_seqs, uint32_t block_table_stride, uint32_t num_q_heads,
                              void* stream);

/* vw_paged_decode with its split-K scratch in a fixed array compiled into this
 * library instead of in memory the pool allocated.  No counterpart in the
 * reference: its single-CTA-per-sequence decode keeps no partials at all.
 *
 * For callers that cannot allocate device memory where they decode -- a
 * serving loop that has handed all free HBM to its own caching allocator, or
 * code that must not call cudaMalloc because it synchronises the device --
 * and that want the decode to touch no library-allocated scratch: neither
 * this call nor its one-time setup allocates anything.  Same arguments,
 * results and flags as vw_paged_decode.
 *
 * Limit: the array holds the partials of a 296-CTA decode grid (148 SMs x 2,
 * a B200) at head_dim <= 128 and up to 16 query heads per KV head, 4.9 MB per
 * device; a pool whose grid needs more gets VW_ERR_UNSUPPORTED and should use
 * vw_paged_decode.  The first call on each device looks the array's address
 * up (cudaGetSymbolAddress); make that first call before any stream capture.
 * There is one array per device, shared by every pool on it: calls on one
 * stream are ordered and safe, but two calls whose kernels can run at the same
 * time (different streams, or different pools on the same device) race. */
VW_API int32_t vw_paged_decode_static(vw_pool* pool, const vw_decode_args* args, void* stream);

/* Copy-on-write block copy / compaction move (no reference counterpart; the
 * decision point is the ref-count in engine/kv_cache.bm:94-113).  pairs:
 * device [num_pairs][2] uint32 (src, dst); every layer's K, V and scales of
 * src are copied to dst.  Destinations must be distinct and not also sources. */
VW_API int32_t vw_block_copy(vw_pool* pool, const uint32_t* pairs, uint32_t num_pairs, void* stream);

/* Block-table gather of one sequence (paging walk of flash_attention.bm:132-140):
 * raw rows out_k, out_v [num_kv_heads][seq_len][head_dim] in the page element
 * type; FP8 pools also write out_k_scales, out_v_scales [num_kv_heads][seq_len]. */
VW_API int32_t vw_kv_gather(vw_pool* pool, uint32_t layer, const uint32_t* block_table,
                     uint32_t seq_len, void* out_k, void* out_v, float* out_k_scales,
                     float* out_v_scales, void* stream);

/* One decode step over every layer with HOST buffers (the end-to-end path):
 * copies the step's inputs host->device, runs append + decode per layer, and
 * copies the attention outputs device->host before returning (the call
 * synchronises with `stream`).  The second call with the same arguments and
 * buffers (same host pointers, sizes, scale and rope_theta) records the step
 * as a CUDA graph, which later identical calls replay: uploads of 1, 1, 2, 4,
 * ... layers ahead of the layers that read them, each layer's outputs read
 * back as soon as it ends.  Calls with other buffers run directly on the
 * stream; buffers that cannot be recorded (e.g. pageable host memory) stay on
 * the direct path.  Pinned host buffers reused across steps are the fast
 * case.  Not for use inside the caller's own stream capture. */
typedef struct {
    uint32_t num_seqs;
    uint32_t num_q_heads;
    uint32_t block_table_stride;
    uint32_t reserved;
    const void* q;                 /* host [L][num_seqs][num_q_heads][head_dim] io dtype */
    const void* k_new;             /* host [L][num_seqs][num_kv_heads][head_dim] */
    const void* v_new;             /* host [L][num_seqs][num_kv_heads][head_dim] */
    const uint32_t* block_tables;  /* host [num_seqs][block_table_stride] */
    const uint32_t* seq_lens;      /* host [num_seqs] (including the new token) */
    void* out;                     /* host [L][num_seqs][num_q_heads][head_dim] */
    float scale;
    float rope_theta;              /* > 0: fused RoPE on q and the new K rows (VW_DECODE_ROPE) */
} vw_step_host_args;
VW_API int32_t vw_decode_step_host(vw_pool* pool, const vw_step_host_args* args, void* stream);

/* ---- Chunked prefill over the pool ------------------------------------------
 * Replaces: launch_flash_attn_prefill (kernels/attention/flash_attention.bm:167-177,
 * kernel flash_attention_fwd :31-106), which attends over contiguous K/V and
 * ignores its block table.  Here the chunk of sequence b is the query tokens
 * cu_seqlens[b] .. cu_seqlens[b+1]-1 at positions ctx_start[b] + i (the tokens
 * before ctx_start[b] are already cached, e.g. a radix-matched prefix or an
 * earlier chunk; scheduler/scheduler.bm:251-266 cuts prompts into chunks of
 * up to 2048 tokens).  With k_new / v_new the chunk's own K/V rows are first
 * appended to slots block_tables[b][p/16]*16 + p%16 (FP8 pools quantise them);
 * then token i attends to keys 0 .. ctx_start[b]+i with VW_PREFILL_CAUSAL, or
 * to all ctx_start[b] + n_b keys without it (the reference kernel has no mask).
 * Every pool kind: f16 / bf16 pages (head_dim 64 or 128) and FP8 E4M3 pages
 * (head_dim 128; attention over the dequantised codes).  Device pointers,
 * 16-byte aligned (the int arrays 4-byte). */
typedef struct {
    uint32_t layer;
    uint32_t num_seqs;             /* B, at most the pool's max_batch */
    uint32_t num_tokens;           /* T = cu_seqlens[B]: rows of q, k_new, v_new, out */
    uint32_t num_q_heads;          /* multiple of num_kv_heads */
    uint32_t block_table_stride;
    uint32_t flags;                /* VW_PREFILL_* */
    const void* q;                 /* [T][num_q_heads][head_dim] io dtype */
    const void* k_new;             /* [T][num_kv_heads][head_dim] chunk rows, or NULL when the */
    const void* v_new;             /*   pages already hold them */
    const int32_t* cu_seqlens;     /* [B+1] chunk offsets, cu_seqlens[0] = 0, non-decreasing */
    const int32_t* ctx_start;      /* [B] tokens cached before each chunk */
    const uint32_t* block_tables;  /* [B][block_table_stride] */
    void* out;                     /* [T][num_q_heads][head_dim] io dtype */
    float scale;                   /* softmax scale; 0 means 1/sqrt(head_dim) (flash_attention.bm:174) */
    float rope_theta;              /* with VW_PREFILL_ROPE: q and the chunk's K rows are rotated */
} vw_prefill_args;

#define VW_PREFILL_CAUSAL 0x1u     /* token i attends to keys 0 .. its own position */
#define VW_PREFILL_ROPE 0x2u       /* RoPE (kernels/rope/rope.bm:22-52) at each token's position */
#define VW_PREFILL_PDL 0x4u        /* launch as a programmatic dependent of the previous kernel */

VW_API int32_t vw_paged_prefill(vw_pool* pool, const vw_prefill_args* args, void* stream);

/* ---- FP8 weight path sharing the KV codec ---------------------------------------
 * rms_norm_fp8_out (kernels/norm/rms_norm.bm:62-94): x, weight f16
 * [rows][hidden] / [hidden] -> out E4M3 codes [rows][hidden] of
 * ((x * inv_rms) * w) * scale through the reference encoder, in the reference's
 * operation order (codes bit-exact). */
VW_API int32_t vw_rms_norm_fp8_out(const void* x, const void* weight, uint8_t* out, uint32_t rows,
                                   uint32_t hidden, float scale, float eps, void* stream);
/* gemm_fp8 (kernels/gemm/gemm_fp8.bm:31-107): C [M][N] bf16 = (a_scale *
 * b_scale) * (A . B) + bias, A [M][K] and B [K][N] E4M3 codes row-major decoded
 * as the reference decoder does (gemm_fp8.bm:110-116), bias bf16 [N] or NULL.
 * N and K multiples of 16; a, b, c 16-byte aligned.  tcgen05 tensor cores. */
VW_API int32_t vw_gemm_fp8(const uint8_t* a, const uint8_t* b, void* c, const void* bias, uint32_t M,
                           uint32_t N, uint32_t K, float a_scale, float b_scale, void* stream);
/* Synchronises, returns and clears the device error word of the two calls above
 * (VW_DEV_ERR_TIMEOUT); VW_ERR_DEVICE_CHECK when it was nonzero. */
VW_API int32_t vw_fp8_weight_check(uint32_t* device_error);

/* ---- Host block manager (engine/kv_cache.bm:29-164, C++ implementation) ---- */
typedef struct vw_block_manager vw_block_manager;
/* kv_cache.bm:41-58: free list 0..max_blocks, the next alloc pops the last. */
VW_API int32_t vw_bm_create(uint32_t block_size, uint32_t max_blocks, vw_block_manager** out);
VW_API int32_t vw_bm_destroy(vw_block_manager* bm);
VW_API uint32_t vw_bm_capacity(const vw_block_manager* bm);                 /* kv_cache.bm:60-62 */
VW_API uint32_t vw_bm_free_count(const vw_block_manager* bm);               /* kv_cache.bm:64-66 */
/* kv_cache.bm:69-78: LIFO pop, ref_count 1; *out = id.  VW_ERR_OOM when empty. */
VW_API int32_t vw_bm_alloc(vw_block_manager* bm, uint32_t* out);
/* kv_cache.bm:81-91: all-or-nothing, VW_ERR_OOM when fewer than n are free. */
VW_API int32_t vw_bm_alloc_seq(vw_block_manager* bm, uint32_t n, uint32_t* out);
VW_API void vw_bm_incref(vw_block_manager* bm, uint32_t id);                /* kv_cache.bm:94-98 */
VW_API void vw_bm_decref(vw_block_manager* bm, uint32_t id);                /* kv_cache.bm:101-113 */
VW_API void vw_bm_free_seq(vw_block_manager* bm, const uint32_t* table, uint32_t n); /* :116-120 */
VW_API uint32_t vw_bm_ref_count(const vw_block_manager* bm, uint32_t id);   /* 0 when free */
/* kv_cache.bm:127-138; returns the number of ids (written up to cap). */
VW_API uint32_t vw_bm_prefix_lookup(const vw_block_manager* bm, const uint32_t* tokens, uint32_t n,
                             uint32_t* out, uint32_t cap);
/* kv_cache.bm:142-151 */
VW_API void vw_bm_register_prefix_block(vw_block_manager* bm, uint32_t id, uint64_t token_hash);
/* kv_cache.bm:157-164 */
VW_API uint64_t vw_rolling_hash(uint64_t prev, const uint32_t* tokens, uint32_t n);
/* Snapshot of the free list in pop order reversed (the last entry pops next). */
VW_API uint32_t vw_bm_free_list(const vw_block_manager* bm, uint32_t* out, uint32_t cap);
/* Copy-on-write before appending into table[index] (no reference counterpart):
 * when that block's ref_count > 1, allocate a fresh block, decref the old one,
 * store the new id in table[index] and return the (src, dst) pair in
 * *pair_out, setting *copied = 1; otherwise *copied = 0.  VW_ERR_OOM if no
 * block is free. */
VW_API int32_t vw_bm_cow(vw_block_manager* bm, uint32_t* table, uint32_t index, uint32_t* pair_out,
                  uint32_t* copied);
/* Compaction plan: moves every used block with id >= used_count to the lowest
 * free id below used_count (ascending), returning the (src, dst) pairs and
 * updating the manager (ids, free list back to new()'s order over the tail).
 * Callers remap their block tables with the same pairs.  Returns the number of
 * pairs (written up to cap). */
VW_API uint32_t vw_bm_compact(vw_block_manager* bm, uint32_t* pairs_out, uint32_t cap);

/* ---- Host radix prefix tree (radix_cache/radix_cache.bm:27-285) ---- */
typedef struct vw_radix vw_radix;
VW_API int32_t vw_radix_create(uint32_t block_size, uint32_t max_blocks, vw_radix** out);
VW_API int32_t vw_radix_destroy(vw_radix* r);
/* radix_cache.bm:77-108 (reuse blocks of a partial edge match included). */
VW_API uint32_t vw_radix_lookup(vw_radix* r, const uint32_t* tokens, uint32_t n, uint32_t* matched_len,
                         uint32_t* out, uint32_t cap);
/* radix_cache.bm:111-179 + :222-228; ids freed by the over-budget eviction are
 * written to freed_out (up to cap) and counted in the return value. */
VW_API uint32_t vw_radix_insert(vw_radix* r, const uint32_t* tokens, uint32_t n, const uint32_t* blocks,
                         uint32_t nb, uint32_t* freed_out, uint32_t cap);
/* radix_cache.bm:231-240 with the leaf walk done edge by edge; returns ids freed. */
VW_API uint32_t vw_radix_evict_lru(vw_radix* r, uint32_t target, uint32_t* freed_out, uint32_t cap);
VW_API uint32_t vw_radix_total_blocks(const vw_radix* r);                   /* radix_cache.bm:242-244 */
/* Pin / unpin every node on the matched path (ref_count of radix_cache.bm:32). */
VW_API void vw_radix_lock(vw_radix* r, const uint32_t* tokens, uint32_t n);
VW_API void vw_radix_unlock(vw_radix* r, const uint32_t* tokens, uint32_t n);
/* Rename block ids after a compaction: every id equal to pairs[i].src becomes pairs[i].dst. */
VW_API void vw_radix_remap(vw_radix* r, const uint32_t* pairs, uint32_t num_pairs);

/* ---- Continuous-batching scheduler wired to the block manager ---------------
 * scheduler/scheduler.bm:186-293 (FCFS waiting queue, running set, a prefill
 * token budget per step, chunks of at most max_chunk prompt tokens, one decode
 * token per running sequence; engine/engine.bm:127-146 runs schedule -> forward
 * -> sample -> commit) with the KV bookkeeping the reference leaves out: block
 * tables allocated from the block manager, prefix reuse of full 16-token pages
 * through the chained prefix hash (kv_cache.bm:127-164; the index holds one
 * reference per kept page and releases the least recently used ones when the
 * pool runs out), copy-on-write pairs for shared pages a step writes,
 * preemption (recompute) of the youngest request when a decode cannot get a
 * page, and continuation of prompts longer than one chunk.  The block
 * manager is the caller's (one per pool); the scheduler only calls it. */
typedef struct vw_sched vw_sched;
typedef struct {
    uint32_t max_batch_tokens;     /* prefill tokens per step (engine.bm:115 uses 8192) */
    uint32_t max_running_seqs;     /* engine.bm:116 uses 256 */
    uint32_t max_chunk;            /* scheduler.bm:255 uses 2048 */
    uint32_t max_seq_len;          /* prompt + new tokens of one request */
    uint32_t prefix_cache;         /* 1: reuse and keep full pages by prefix hash */
    uint32_t reserved;             /* must be 0 */
} vw_sched_config;
typedef struct {                   /* one sequence of a step, in descriptor order */
    uint64_t seq_id;
    uint32_t is_prefill;           /* 1: a prompt chunk, 0: a decode (1 token) */
    uint32_t num_tokens;           /* tokens appended this step */
    uint32_t ctx_start;            /* tokens already cached = the first token's position */
    uint32_t samples;              /* 1: commit the token sampled from this step's last row */
    uint32_t token_offset;         /* index of the first token in the batch's tokens[] */
    uint32_t reserved;
} vw_sched_seq;
typedef struct {                   /* arrays owned by the scheduler, valid until its next call */
    uint32_t num_seqs;
    uint32_t table_stride;
    const vw_sched_seq* seqs;      /* prefill chunks first, then decodes */
    const uint32_t* tokens;        /* the step's input tokens */
    const uint32_t* block_tables;  /* [num_seqs][table_stride], covering ctx_start + num_tokens */
    uint32_t num_copies;
    uint32_t reserved;
    const uint32_t* copies;        /* [num_copies][2] (src, dst): vw_block_copy before the step */
} vw_sched_batch;
typedef struct {
    uint32_t waiting, running, finished;
    uint32_t cached_pages;         /* pages the prefix index keeps (one reference each) */
    uint32_t table_refs;           /* block-table entries of the running requests */
    uint32_t free_blocks;
    uint32_t preemptions;
    uint32_t reserved;
} vw_sched_stat;
VW_API int32_t vw_sched_create(const vw_sched_config* cfg, vw_block_manager* bm, vw_sched** out);
VW_API int32_t vw_sched_destroy(vw_sched* s);     /* releases every page it holds */
/* scheduler.bm:230-235; stop_token < 0: none (Request::is_done, scheduler.bm:85-95) */
VW_API int32_t vw_sched_add_request(vw_sched* s, const uint32_t* prompt, uint32_t n,
                                    uint32_t max_new_tokens, int64_t stop_token, uint64_t* id_out);
/* scheduler.bm:241-293 plus the bookkeeping above */
VW_API int32_t vw_sched_schedule(vw_sched* s, vw_sched_batch* out);
/* scheduler.bm:296-319: every scheduled sequence's tokens are cached; (ids[i],
 * tokens[i]) are the tokens sampled for the sequences with samples = 1. */
VW_API int32_t vw_sched_commit(vw_sched* s, const uint64_t* ids, const uint32_t* tokens, uint32_t n);
/* scheduler.bm:322-326, one request at a time: its id and output tokens (up to
 * cap); VW_ERR_INVALID_ARG when none is finished. */
VW_API int32_t vw_sched_take_finished(vw_sched* s, uint64_t* id, uint32_t* out_tokens, uint32_t cap,
                                      uint32_t* num_out);
VW_API int32_t vw_sched_stats(const vw_sched* s, vw_sched_stat* st);

/* Message for the last failure on this thread ("" if none). */
VW_API const char* vw_last_error(void);

/* ---- Failure injection for tests of a caller's error handling ----------------
 * The engine turns any nonzero status of voidweb_forward_pass into a failed
 * step (engine/ffi.bm:112-118) and an exhausted block pool into an allocation
 * error (engine/kv_cache.bm:82-85).  vw_fault_inject arms `count` failures of
 * one kind (count 0 disarms); each later call of an entry point that can fail
 * that way consumes one and returns the status at once, before touching the
 * device or the bookkeeping:
 *   VW_FAULT_OOM         -> VW_ERR_OOM: vw_pool_create, vw_decode_step_host,
 *                           voidweb_forward_pass, vw_bm_alloc, vw_bm_alloc_seq, vw_bm_cow
 *   VW_FAULT_INVALID_ARG -> VW_ERR_INVALID_ARG and
 *   VW_FAULT_CUDA        -> VW_ERR_CUDA: vw_pool_create, vw_kv_append,
 *                           vw_paged_decode, vw_paged_decode_static, vw_decode_plan,
 *                           vw_block_copy, vw_kv_gather, vw_paged_prefill,
 *                           vw_decode_step_host, voidweb_forward_pass,
 *                           vw_rms_norm_fp8_out, vw_gemm_fp8
 * The environment variable VOIDWEB_KV_FAULT ("oom:N,invalid:N,cuda:N") arms
 * the same counts when the library is loaded.  No counterpart in the reference. */
#define VW_FAULT_OOM 1u
#define VW_FAULT_INVALID_ARG 2u
#define VW_FAULT_CUDA 3u
VW_API int32_t vw_fault_inject(uint32_t kind, uint32_t count);
/* Failures of `kind` still armed. */
VW_API uint32_t vw_fault_pending(uint32_t kind);

/* Test hook for the bounded device waits: the decode and prefill launches of
 * this pool give up every wait for a copy or a consumer after `cycles` SM
 * clock cycles from the kernel's start (0 restores the default, about 2 s and
 * the normal launch), and they withhold copies -- the decode its query tiles,
 * the prefill its K/V tiles -- so that their first waits are ones that nothing
 * satisfies.  Such a launch records VW_DEV_ERR_TIMEOUT, waits (under the
 * default limit) for the copies and tensor-core operations it has in flight,
 * frees its tensor memory, and returns; its outputs are undefined (a prefill's
 * chunk append still runs).  vw_pool_check clears the word, after which the
 * pool runs normally.  No counterpart in the reference. */
VW_API int32_t vw_debug_set_wait_limit(vw_pool* pool, uint64_t cycles);

/* Number of device (cudaMalloc) and pinned host (cudaHostAlloc) allocations this
 * library has made since it was loaded: a test can check that a call allocates
 * nothing by reading it before and after.  No counterpart in the reference. */
VW_API uint64_t vw_debug_alloc_count(void);

/* ---- The symbol the engine dlopens (engine/ffi.bm:15-40, :68, :113) ---- */
#pragma pack(push, 1)
typedef struct {
    uint64_t seq_id;
    uint64_t token_ptr;    /* host uint32_t[num_tokens] */
    uint32_t num_tokens;
    uint64_t block_ptr;    /* host uint32_t[num_blocks] physical block ids */
    uint32_t num_blocks;
    uint8_t is_prefill;
} SeqDescriptor;

typedef struct {
    const SeqDescriptor* seqs;
    uint32_t num_seqs;
    uint32_t hidden_size;
    uint32_t num_heads;
    uint32_t num_kv_heads;
    uint32_t num_layers;
    uint32_t vocab_size;
    uint32_t head_dim;
    float rope_theta;
    uint32_t quant_type;   /* QuantScheme ordinal (quantization/quantization.bm:13-19) */
    float* logits_out;     /* host [num_seqs][vocab_size] */
} ForwardArgs;
#pragma pack(pop)

/* Host-side I/O of the attention slice: the transformer layers around
 * attention (embedding, QKV/O projections, MLP, LM head) are outside this
 * library, so the caller binds the pool and the per-layer q / new K / new V
 * rows and the attention output buffer that voidweb_forward_pass reads and
 * writes (host, [L][rows][heads][head_dim] in the io dtype, one row per token
 * of each descriptor, in descriptor order).  The binding is process-wide.
 * With pinned buffers (cudaHostAlloc / cudaHostRegister) the decode part of a
 * forward pass is the fast path of vw_decode_step_host: the library keeps each
 * step's block tables and lengths in pinned buffers of its own, reused from
 * step to step, so from the second step of the same batch size and table
 * stride every forward pass replays one recorded CUDA graph (uploads,
 * append + decode of every layer, read-back).  Binding a NULL pool releases
 * those buffers. */
VW_API int32_t vw_forward_bind(vw_pool* pool, const void* q, const void* k_new, const void* v_new,
                        void* attn_out);
/* Number of tokens already cached for seq_id (e.g. after a prefill done
 * elsewhere; unseen sequences start at 0).  voidweb_forward_pass advances it
 * by one per decode step; vw_forward_release forgets the sequence. */
VW_API int32_t vw_forward_set_seq_len(uint64_t seq_id, uint32_t len);
VW_API int32_t vw_forward_release(uint64_t seq_id);

/* engine/ffi.bm:68,113: returns 0 on success.  Descriptor i owns num_tokens
 * consecutive rows of the bound buffers (rows in descriptor order:
 * [L][sum of num_tokens][heads][head_dim]).  A decode descriptor
 * (is_prefill == 0, num_tokens == 1) puts its token at position len(seq_id)
 * and attends over len(seq_id)+1 tokens; a prefill descriptor (is_prefill ==
 * 1, the scheduler's chunk, scheduler/scheduler.bm:251-266) puts its
 * num_tokens tokens at positions len(seq_id) .. len(seq_id)+num_tokens-1 and
 * each attends causally over the cached tokens and the chunk up to itself.
 * The host block list (block_ptr, num_blocks) is the block table; len(seq_id)
 * then grows by num_tokens.  logits_out is not written (no LM head in this
 * library). */
VW_API int32_t voidweb_forward_pass(const ForwardArgs* args);

#ifdef __cplusplus
}
#endif

#endif /* VOIDWEB_KV_H */
