// vw_capi.cu -- the C ABI of libvoidweb_kv.so (declared in include/voidweb_kv.h):
// pool lifetime, argument validation, TMA descriptor encoding, kernel dispatch,
// the host-buffer decode step, and the voidweb_forward_pass shim the engine
// dlopens (engine/ffi.bm:61-77, :113).
//
// Every entry point validates its arguments on the host before any launch and
// reports failure through an int32 status plus a thread-local message, as the
// engine expects (engine/ffi.bm:112-118); nothing throws across the boundary.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/voidweb_kv.h"
#include "vw_fault.h"
#include "vw_internal.h"

using namespace vw;

namespace {

thread_local std::string g_last_error;

int32_t fail(int32_t code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

int32_t cuda_fail(cudaError_t e, const char* what) {
    return fail(VW_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Every device and pinned-host allocation of this library goes through these
// two, so that vw_debug_alloc_count can tell a caller whether a call allocated.
std::atomic<uint64_t> g_alloc_calls{0};
template <class T>
cudaError_t dev_alloc(T** p, size_t bytes) {
    g_alloc_calls.fetch_add(1);
    return cudaMalloc(reinterpret_cast<void**>(p), bytes);
}
cudaError_t pinned_alloc(void** p, size_t bytes) {
    g_alloc_calls.fetch_add(1);
    return cudaHostAlloc(p, bytes, cudaHostAllocPortable);
}

// An armed injected failure (vw_fault_inject) of one of `kinds` ends the call
// here, before anything else happens.
#define VW_FAULT_POINT(kinds, name)                                                   \
    do {                                                                              \
        const char* what_ = "";                                                       \
        const int32_t rc_ = vw::fault_take((kinds), &what_);                          \
        if (rc_ != VW_OK) return fail(rc_, "%s: injected fault (%s)", (name), what_); \
    } while (0)
constexpr uint32_t kFaultAll = vw::kCanOom | vw::kCanInvalid | vw::kCanCuda;
constexpr uint32_t kFaultLaunch = vw::kCanInvalid | vw::kCanCuda;

// RAII-free device scope switch: the library never leaves the caller's
// current device changed.
struct DeviceScope {
    int prev = -1;
    bool ok = true;
    explicit DeviceScope(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) ok = cudaSetDevice(dev) == cudaSuccess;
    }
    ~DeviceScope() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

}  // namespace

// Everything a recorded host-buffer step depends on.
struct StepKey {
    uint32_t B, Hq, stride, scale_bits, theta_bits;
    const void *q, *k, *v, *bt, *sl, *out;
    const uint8_t* stage;
    bool operator==(const StepKey& o) const {
        return B == o.B && Hq == o.Hq && stride == o.stride && scale_bits == o.scale_bits &&
               theta_bits == o.theta_bits && q == o.q && k == o.k && v == o.v && bt == o.bt &&
               sl == o.sl && out == o.out && stage == o.stage;
    }
};

struct vw_pool {
    vw_pool_config cfg{};
    PoolGeom geom{};
    uint8_t* data = nullptr;
    float* scales = nullptr;
    bool own_data = false, own_scales = false;
    uint64_t data_bytes = 0, scale_bytes = 0;
    alignas(64) CUtensorMap tmap;       // page-head boxes (decode)
    alignas(64) CUtensorMap tmap_half;  // 16-row boxes of one 128-B column (prefill)
    float* part_o = nullptr;
    float* part_ml = nullptr;
    uint32_t* err = nullptr;
    int grid = 0;
    // split-K scratch: two sets, alternated per decode launch so that two
    // overlapping launches (programmatic dependent launch) never share one
    size_t scratch_o = 0, scratch_ml = 0;
    uint64_t launches = 0;
    uint64_t wait_cycles = 0;           // vw_debug_set_wait_limit (0: the default bound)
    // decode plan (vw_decode_plan) and the batch it was made for
    int* plan = nullptr;
    bool plan_ready = false;
    const void* plan_tables = nullptr;
    const void* plan_lens = nullptr;
    uint32_t plan_seqs = 0, plan_stride = 0, plan_q_heads = 0;
    // staging for vw_decode_step_host and for the forward pass's prefill (grow-only)
    uint8_t* stage = nullptr;
    size_t stage_bytes = 0;
    uint8_t* pstage = nullptr;
    size_t pstage_bytes = 0;
    cudaStream_t s_h2d = nullptr, s_d2h = nullptr, s_cap = nullptr;
    std::vector<cudaEvent_t> ev_in, ev_done;
    cudaEvent_t ev_entry = nullptr, ev_exit = nullptr;
    // vw_decode_step_host: the step recorded as a CUDA graph for one set of
    // arguments (host buffers included), made on the second call with them
    StepKey step_key{}, step_seen{}, step_bad{};
    cudaGraphExec_t step_exec = nullptr;
};

namespace {

void pool_free_all(vw_pool* p) {
    if (p->own_data && p->data) cudaFree(p->data);
    if (p->own_scales && p->scales) cudaFree(p->scales);
    if (p->part_o) cudaFree(p->part_o);
    if (p->part_ml) cudaFree(p->part_ml);
    if (p->plan) cudaFree(p->plan);
    if (p->err) cudaFree(p->err);
    if (p->stage) cudaFree(p->stage);
    if (p->pstage) cudaFree(p->pstage);
    if (p->step_exec) cudaGraphExecDestroy(p->step_exec);
    if (p->s_h2d) cudaStreamDestroy(p->s_h2d);
    if (p->s_d2h) cudaStreamDestroy(p->s_d2h);
    if (p->s_cap) cudaStreamDestroy(p->s_cap);
    for (auto e : p->ev_in) cudaEventDestroy(e);
    for (auto e : p->ev_done) cudaEventDestroy(e);
    if (p->ev_entry) cudaEventDestroy(p->ev_entry);
    if (p->ev_exit) cudaEventDestroy(p->ev_exit);
}

int32_t encode_pool_map(vw_pool* p) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return fail(VW_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    const PoolGeom& g = p->geom;
    const uint64_t eb = elem_bytes(g.kv_kind);
    const uint64_t row = (uint64_t)g.head_dim * eb;
    // View of the pool as 128-B columns of token rows: dimension 0 = the 128 bytes
    // of one column, 1 = token rows (stride one row), 2 = the row's columns
    // (stride 128 B; present when a row is 256 B).  One box = a whole page-head,
    // its 32 rows (K rows then V rows) of every column, landing in smem as
    // [column][32 rows][128 B] with the 128-B swizzle.
    const uint64_t rows = (uint64_t)g.num_layers * g.num_blocks * g.num_kv_heads * 32;
    const uint32_t cols = (uint32_t)(row / 128);
    cuuint64_t dims[3] = {128 / eb, rows, cols};
    cuuint64_t strides[2] = {row, 128};
    cuuint32_t box[3] = {(cuuint32_t)(128 / eb), 32, cols};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(&p->tmap, eb == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_UINT16,
                    cols > 1 ? 3 : 2, p->data, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(VW_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    // Second view for the prefill: token rows of head_dim elements; one box =
    // 16 rows (the K or the V half of a page-head) of one 128-B column, so that
    // the K rows of consecutive page-heads land 16 rows apart in one tile.
    cuuint64_t dims2[2] = {(cuuint64_t)g.head_dim, rows};
    cuuint64_t strides2[1] = {row};
    cuuint32_t box2[2] = {(cuuint32_t)(128 / eb), 16};
    r = fn(&p->tmap_half, eb == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_UINT16, 2,
           p->data, dims2, strides2, box2, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(VW_ERR_CUDA, "cuTensorMapEncodeTiled (half) failed (%d)", (int)r);
    return VW_OK;
}

}  // namespace

extern "C" {

const char* vw_last_error(void) { return g_last_error.c_str(); }

int32_t vw_pool_create(const vw_pool_config* cfg, vw_pool** out) {
    VW_FAULT_POINT(kFaultAll, "vw_pool_create");
    if (!cfg || !out) return fail(VW_ERR_INVALID_ARG, "vw_pool_create: null argument");
    *out = nullptr;
    const vw_pool_config& c = *cfg;
    if (c.reserved != 0) return fail(VW_ERR_INVALID_ARG, "vw_pool_create: reserved must be 0");
    if (c.num_layers == 0 || c.num_kv_heads == 0 || c.num_blocks == 0)
        return fail(VW_ERR_INVALID_ARG, "vw_pool_create: layers, kv heads and blocks must be > 0");
    if (c.kv_dtype > VW_FP8_E4M3 || (c.io_dtype != VW_F16 && c.io_dtype != VW_BF16))
        return fail(VW_ERR_INVALID_ARG, "vw_pool_create: bad kv_dtype %u / io_dtype %u",
                    c.kv_dtype, c.io_dtype);
    if (c.kv_dtype != VW_FP8_E4M3 && c.kv_dtype != c.io_dtype)
        return fail(VW_ERR_INVALID_ARG, "vw_pool_create: f16/bf16 pools need io_dtype == kv_dtype");
    if (c.fp8_mode > VW_FP8_OCP) return fail(VW_ERR_INVALID_ARG, "vw_pool_create: bad fp8_mode");
    if (c.head_dim != 64 && c.head_dim != 128)
        return fail(VW_ERR_UNSUPPORTED, "vw_pool_create: head_dim %u (64 or 128)", c.head_dim);
    if (c.kv_dtype == VW_FP8_E4M3 && c.head_dim != 128)
        return fail(VW_ERR_UNSUPPORTED, "vw_pool_create: FP8 pools need head_dim 128");
    if (c.max_batch == 0 || c.max_batch > (uint32_t)kMaxBatchPerLaunch)
        return fail(VW_ERR_INVALID_ARG, "vw_pool_create: max_batch must be 1..%d", kMaxBatchPerLaunch);
    if ((uint64_t)c.num_layers * c.num_blocks * c.num_kv_heads * 32 > 0x7FFFFFFFull)
        return fail(VW_ERR_INVALID_ARG,
                    "vw_pool_create: layers * blocks * kv_heads * 32 rows exceed 2^31-1");
    if (c.kv_data && !aligned(c.kv_data, 256))
        return fail(VW_ERR_INVALID_ARG, "vw_pool_create: kv_data must be 256-byte aligned");
    if (c.kv_scales && !aligned(c.kv_scales, 256))
        return fail(VW_ERR_INVALID_ARG, "vw_pool_create: kv_scales must be 256-byte aligned");
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || c.device < 0 || c.device >= ndev)
        return fail(VW_ERR_INVALID_ARG, "vw_pool_create: device %d not available", c.device);
    DeviceScope ds(c.device);
    if (!ds.ok) return fail(VW_ERR_CUDA, "vw_pool_create: cudaSetDevice failed");

    vw_pool* p = new vw_pool();
    p->cfg = c;
    p->geom = PoolGeom{c.num_layers, c.num_kv_heads, c.head_dim, c.num_blocks, c.kv_dtype,
                       c.io_dtype, c.fp8_mode};
    const uint64_t eb = elem_bytes(c.kv_dtype);
    const uint64_t rows = (uint64_t)c.num_layers * c.num_blocks * 2 * c.num_kv_heads * 16;
    p->data_bytes = rows * c.head_dim * eb;
    p->scale_bytes = c.kv_dtype == VW_FP8_E4M3 ? rows * 4 : 0;
    cudaError_t e;
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, c.device);
    p->grid = (sms > 0 ? sms : 148) * decode_ctas_per_sm();
    if (c.kv_data) {
        p->data = static_cast<uint8_t*>(c.kv_data);
    } else {
        if ((e = dev_alloc(&p->data, p->data_bytes)) != cudaSuccess) {
            const unsigned long long bytes = p->data_bytes;
            delete p;
            return fail(VW_ERR_OOM, "vw_pool_create: %llu bytes of pages: %s", bytes, cudaGetErrorString(e));
        }
        p->own_data = true;
    }
    if (p->scale_bytes) {
        if (c.kv_scales) {
            p->scales = static_cast<float*>(c.kv_scales);
        } else if ((e = dev_alloc(&p->scales, p->scale_bytes)) == cudaSuccess) {
            p->own_scales = true;
        } else {
            pool_free_all(p);
            delete p;
            return fail(VW_ERR_OOM, "vw_pool_create: scales: %s", cudaGetErrorString(e));
        }
    }
    const size_t n_o = decode_scratch_floats_o(p->grid, c.head_dim);
    const size_t n_ml = decode_scratch_floats_ml(p->grid);
    p->scratch_o = n_o;
    p->scratch_ml = n_ml;
    if ((e = dev_alloc(&p->part_o, 2 * n_o * 4)) != cudaSuccess ||
        (e = dev_alloc(&p->part_ml, 2 * n_ml * 4)) != cudaSuccess ||
        (e = dev_alloc(&p->plan, plan_ints(p->grid) * 4)) != cudaSuccess ||
        (e = dev_alloc(&p->err, 4)) != cudaSuccess) {
        pool_free_all(p);
        delete p;
        return fail(VW_ERR_OOM, "vw_pool_create: scratch: %s", cudaGetErrorString(e));
    }
    if ((e = cudaMemset(p->err, 0, 4)) != cudaSuccess ||
        (e = cudaDeviceSynchronize()) != cudaSuccess) {
        pool_free_all(p);
        delete p;
        return cuda_fail(e, "vw_pool_create: memset");
    }
    int32_t rc = encode_pool_map(p);
    if (rc != VW_OK) {
        pool_free_all(p);
        delete p;
        return rc;
    }
    *out = p;
    return VW_OK;
}

int32_t vw_pool_destroy(vw_pool* pool) {
    if (!pool) return VW_OK;
    DeviceScope ds(pool->cfg.device);
    cudaDeviceSynchronize();
    pool_free_all(pool);
    delete pool;
    return VW_OK;
}

int32_t vw_pool_info(const vw_pool* pool, void** kv_data, void** kv_scales, uint64_t* data_bytes,
                     uint64_t* scale_bytes) {
    if (!pool) return fail(VW_ERR_INVALID_ARG, "vw_pool_info: null pool");
    if (kv_data) *kv_data = pool->data;
    if (kv_scales) *kv_scales = pool->scales;
    if (data_bytes) *data_bytes = pool->data_bytes;
    if (scale_bytes) *scale_bytes = pool->scale_bytes;
    return VW_OK;
}

uint64_t vw_debug_alloc_count(void) { return g_alloc_calls.load(); }

int32_t vw_debug_set_wait_limit(vw_pool* pool, uint64_t cycles) {
    if (!pool) return fail(VW_ERR_INVALID_ARG, "vw_debug_set_wait_limit: null pool");
    pool->wait_cycles = cycles;
    return VW_OK;
}

int32_t vw_pool_check(vw_pool* pool, uint32_t* device_error) {
    if (!pool) return fail(VW_ERR_INVALID_ARG, "vw_pool_check: null pool");
    DeviceScope ds(pool->cfg.device);
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return cuda_fail(e, "vw_pool_check: synchronize");
    uint32_t w = 0;
    if ((e = cudaMemcpy(&w, pool->err, 4, cudaMemcpyDeviceToHost)) != cudaSuccess)
        return cuda_fail(e, "vw_pool_check: read");
    if ((e = cudaMemset(pool->err, 0, 4)) != cudaSuccess) return cuda_fail(e, "vw_pool_check: clear");
    if (device_error) *device_error = w;
    if (w) return fail(VW_ERR_DEVICE_CHECK, "device bounds check flags 0x%x", w);
    return VW_OK;
}

int32_t vw_kv_append(vw_pool* pool, uint32_t layer, const void* k_new, const void* v_new,
                     const int64_t* slot_mapping, uint32_t num_tokens, void* stream) {
    VW_FAULT_POINT(kFaultLaunch, "vw_kv_append");
    if (!pool) return fail(VW_ERR_INVALID_ARG, "vw_kv_append: null pool");
    if (layer >= pool->geom.num_layers)
        return fail(VW_ERR_INVALID_ARG, "vw_kv_append: layer %u >= %u", layer, pool->geom.num_layers);
    if (num_tokens == 0) return VW_OK;
    if ((uint64_t)num_tokens * 2 * pool->geom.num_kv_heads >= (1ull << 31))
        return fail(VW_ERR_INVALID_ARG, "vw_kv_append: num_tokens %u too large", num_tokens);
    if (!k_new || !v_new || !slot_mapping)
        return fail(VW_ERR_INVALID_ARG, "vw_kv_append: null device pointer");
    if (!aligned(k_new, 16) || !aligned(v_new, 16) || !aligned(slot_mapping, 8))
        return fail(VW_ERR_INVALID_ARG, "vw_kv_append: k_new/v_new must be 16-byte aligned");
    DeviceScope ds(pool->cfg.device);
    cudaError_t e = launch_kv_append(pool->geom, pool->data, pool->scales, layer, k_new, v_new,
                                     slot_mapping, num_tokens, pool->err,
                                     static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? VW_OK : cuda_fail(e, "vw_kv_append launch");
}

static int32_t decode_validate(const vw_pool* pool, const vw_decode_args* a) {
    if (!pool || !a) return fail(VW_ERR_INVALID_ARG, "vw_paged_decode: null argument");
    const PoolGeom& g = pool->geom;
    if (a->flags & ~(uint32_t)(VW_DECODE_PDL | VW_DECODE_EARLY_PAGES | VW_DECODE_PLANNED | VW_DECODE_ROPE))
        return fail(VW_ERR_INVALID_ARG, "vw_paged_decode: unknown flags 0x%x", a->flags);
    if (a->reserved != 0) return fail(VW_ERR_INVALID_ARG, "vw_paged_decode: reserved must be 0");
    if ((a->flags & VW_DECODE_ROPE) && !(a->rope_theta > 1.0f && std::isfinite(a->rope_theta)))
        return fail(VW_ERR_INVALID_ARG, "vw_paged_decode: VW_DECODE_ROPE needs a finite rope_theta > 1");
    if ((a->flags & VW_DECODE_PLANNED) &&
        (!pool->plan_ready || pool->plan_tables != a->block_tables || pool->plan_lens != a->seq_lens ||
         pool->plan_seqs != a->num_seqs || pool->plan_stride != a->block_table_stride ||
         pool->plan_q_heads != a->num_q_heads))
        return fail(VW_ERR_INVALID_ARG,
                    "vw_paged_decode: VW_DECODE_PLANNED without a vw_decode_plan of the same "
                    "block tables, seq_lens, num_seqs, stride and query heads");
    if ((a->flags & VW_DECODE_EARLY_PAGES) && !(a->flags & VW_DECODE_PDL))
        return fail(VW_ERR_INVALID_ARG, "vw_paged_decode: VW_DECODE_EARLY_PAGES needs VW_DECODE_PDL");
    if (a->layer >= g.num_layers)
        return fail(VW_ERR_INVALID_ARG, "vw_paged_decode: layer %u >= %u", a->layer, g.num_layers);
    if (a->num_seqs > pool->cfg.max_batch)
        return fail(VW_ERR_INVALID_ARG, "vw_paged_decode: num_seqs %u > max_batch %u", a->num_seqs,
                    pool->cfg.max_batch);
    if (a->num_q_heads == 0 || a->num_q_heads % g.num_kv_heads != 0)
        return fail(VW_ERR_INVALID_ARG, "vw_paged_decode: num_q_heads %u not a multiple of %u",
                    a->num_q_heads, g.num_kv_heads);
    if (a->num_q_heads / g.num_kv_heads > 16)
        return fail(VW_ERR_UNSUPPORTED, "vw_paged_decode: GQA group %u > 16",
                    a->num_q_heads / g.num_kv_heads);
    if (a->block_table_stride == 0)
        return fail(VW_ERR_INVALID_ARG, "vw_paged_decode: block_table_stride must be > 0");
    if (!a->q || !a->block_tables || !a->seq_lens || !a->out)
        return fail(VW_ERR_INVALID_ARG, "vw_paged_decode: null device pointer");
    if ((a->k_new == nullptr) != (a->v_new == nullptr))
        return fail(VW_ERR_INVALID_ARG, "vw_paged_decode: k_new and v_new go together");
    if (!aligned(a->q, 16) || !aligned(a->out, 16) || !aligned(a->block_tables, 4) ||
        !aligned(a->seq_lens, 4) || (a->k_new && (!aligned(a->k_new, 16) || !aligned(a->v_new, 16))))
        return fail(VW_ERR_INVALID_ARG, "vw_paged_decode: misaligned pointer");
    if (!(a->scale >= 0.0f) || std::isinf(a->scale))
        return fail(VW_ERR_INVALID_ARG, "vw_paged_decode: bad scale");
    return VW_OK;
}

// Split-K scratch given to a decode launch in place of the pool's own.
struct DecodeScratch {
    float* o;
    float* ml;
};

// Decode launch options fixed for the process, from the environment:
//  VOIDWEB_KV_DIRECT_Q=1|0          the first segment's query rows read straight
//                                   from global memory by the consumer warps
//                                   (default 1: 4455 -> 4503 GB/s on the Qwen step)
uint32_t env_decode_flags() {
    static const uint32_t v = [] {
        uint32_t f = 0;
        const char* q = std::getenv("VOIDWEB_KV_DIRECT_Q");
        if (!(q && std::strcmp(q, "0") == 0)) f |= kDecodeDirectQ;
        return f;
    }();
    return v;
}

// Virtual pages charged per segment boundary when the decode CTAs split a
// batch (the gap of the split in vw_decode.cu).  Measured on B200s: 2-byte
// pages 18 (the Qwen2.5-7B batch-16 step 4658 GB/s against 4531 at 12, 4665
// at 21, 4609 at 24, 4032 at 6; the Llama-3-70B one-KV-head batch 6265
// against 6290 at 12 and 6244 at 24), FP8 pages 12 (the Llama-3-8B batch 4062
// against 3995 at 0, 4081 at 6, 3996 at 18).
// VOIDWEB_KV_SEGMENT_COST=n overrides it (at most kMaxSegmentCost).
uint32_t segment_cost(const PoolGeom& g) {
    static const long env = [] {
        const char* e = std::getenv("VOIDWEB_KV_SEGMENT_COST");
        return e ? std::strtol(e, nullptr, 10) : -1L;
    }();
    if (env >= 0) return (uint32_t)std::min<long>(env, kMaxSegmentCost);
    return g.kv_kind == kFP8 ? 12u : 18u;
}

static int32_t decode_launch(vw_pool* pool, const vw_decode_args* a, cudaStream_t s,
                             const DecodeScratch* fixed = nullptr) {
    const PoolGeom& g = pool->geom;
    DecodeLaunch L{};
    DecodeParams& p = L.p;
    p.q = a->q;
    p.out = a->out;
    p.k_new = a->k_new;
    p.v_new = a->v_new;
    p.block_tables = a->block_tables;
    p.seq_lens = a->seq_lens;
    p.kv_data = pool->data;
    p.kv_scales = pool->scales;
    if (fixed) {
        p.part_o = fixed->o;
        p.part_ml = fixed->ml;
    } else {
        const uint64_t set = pool->launches++ & 1;
        p.part_o = pool->part_o + set * pool->scratch_o;
        p.part_ml = pool->part_ml + set * pool->scratch_ml;
    }
    p.flags = a->flags | env_decode_flags();
    p.seg_cost = segment_cost(g);
    p.plan = (a->flags & VW_DECODE_PLANNED) ? pool->plan : nullptr;
    p.err = pool->err;
    p.B = a->num_seqs;
    p.Hq = a->num_q_heads;
    p.Hkv = g.num_kv_heads;
    p.group = a->num_q_heads / g.num_kv_heads;
    p.num_blocks = g.num_blocks;
    p.layer = a->layer;
    p.bt_stride = a->block_table_stride;
    p.fp8_ocp = g.fp8_ocp;
    // reference scale: 1.0 / (HEAD_DIM as f32).sqrt() (flash_attention.bm:187)
    const float scale = a->scale > 0.0f ? a->scale : 1.0f / std::sqrt((float)g.head_dim);
    p.scale_log2 = scale * 1.4426950408889634f;
    p.rope_theta = (a->flags & VW_DECODE_ROPE) ? a->rope_theta : 0.0f;
    p.wait_cycles = pool->wait_cycles;
    if (pool->wait_cycles) {
        // the bounded-wait test hook: the query tiles are withheld (and read only
        // from the ring), so the first wait of every consumer warp runs out
        p.flags = (p.flags | kDecodeWithholdQ) & ~kDecodeDirectQ;
    }
    L.tmap = &pool->tmap;
    L.head_dim = g.head_dim;
    L.kv_kind = g.kv_kind;
    L.io_kind = g.io_kind;
    L.grid = pool->grid;
    L.stream = s;
    cudaError_t e = launch_paged_decode(L);
    return e == cudaSuccess ? VW_OK : cuda_fail(e, "vw_paged_decode launch");
}

int32_t vw_paged_decode(vw_pool* pool, const vw_decode_args* args, void* stream) {
    VW_FAULT_POINT(kFaultLaunch, "vw_paged_decode");
    int32_t rc = decode_validate(pool, args);
    if (rc != VW_OK) return rc;
    if (args->num_seqs == 0) return VW_OK;
    DeviceScope ds(pool->cfg.device);
    return decode_launch(pool, args, static_cast<cudaStream_t>(stream));
}

// ---------------------------------------------------------------------------
// Chunked prefill: launch_flash_attn_prefill (kernels/attention/flash_attention.bm:167-177)
// over the pool's pages.
// ---------------------------------------------------------------------------

static int32_t prefill_validate(const vw_pool* pool, const vw_prefill_args* a) {
    if (!pool || !a) return fail(VW_ERR_INVALID_ARG, "vw_paged_prefill: null argument");
    const PoolGeom& g = pool->geom;
    if (a->flags & ~(uint32_t)(VW_PREFILL_CAUSAL | VW_PREFILL_ROPE | VW_PREFILL_PDL))
        return fail(VW_ERR_INVALID_ARG, "vw_paged_prefill: unknown flags 0x%x", a->flags);
    if ((a->flags & VW_PREFILL_ROPE) && !(a->rope_theta > 1.0f && std::isfinite(a->rope_theta)))
        return fail(VW_ERR_INVALID_ARG, "vw_paged_prefill: VW_PREFILL_ROPE needs a finite rope_theta > 1");
    if (a->layer >= g.num_layers)
        return fail(VW_ERR_INVALID_ARG, "vw_paged_prefill: layer %u >= %u", a->layer, g.num_layers);
    if (a->num_seqs > pool->cfg.max_batch || a->num_seqs > (uint32_t)kMaxBatchPerLaunch)
        return fail(VW_ERR_INVALID_ARG, "vw_paged_prefill: num_seqs %u > max_batch %u", a->num_seqs,
                    pool->cfg.max_batch);
    if (a->num_q_heads == 0 || a->num_q_heads % g.num_kv_heads != 0 || a->num_q_heads > 65535)
        return fail(VW_ERR_INVALID_ARG, "vw_paged_prefill: num_q_heads %u not a multiple of %u",
                    a->num_q_heads, g.num_kv_heads);
    if (a->block_table_stride == 0)
        return fail(VW_ERR_INVALID_ARG, "vw_paged_prefill: block_table_stride must be > 0");
    if (a->num_tokens > (1u << 24) || (uint64_t)a->num_tokens * g.num_kv_heads >= (1ull << 31))
        return fail(VW_ERR_INVALID_ARG, "vw_paged_prefill: num_tokens %u too large", a->num_tokens);
    if (!a->q || !a->cu_seqlens || !a->ctx_start || !a->block_tables || !a->out)
        return fail(VW_ERR_INVALID_ARG, "vw_paged_prefill: null device pointer");
    if ((a->k_new == nullptr) != (a->v_new == nullptr))
        return fail(VW_ERR_INVALID_ARG, "vw_paged_prefill: k_new and v_new go together");
    if (!aligned(a->q, 16) || !aligned(a->out, 16) || !aligned(a->cu_seqlens, 4) ||
        !aligned(a->ctx_start, 4) || !aligned(a->block_tables, 4) ||
        (a->k_new && (!aligned(a->k_new, 16) || !aligned(a->v_new, 16))))
        return fail(VW_ERR_INVALID_ARG, "vw_paged_prefill: misaligned pointer");
    if (!(a->scale >= 0.0f) || std::isinf(a->scale))
        return fail(VW_ERR_INVALID_ARG, "vw_paged_prefill: bad scale");
    return VW_OK;
}

int32_t vw_paged_prefill(vw_pool* pool, const vw_prefill_args* a, void* stream) {
    VW_FAULT_POINT(kFaultLaunch, "vw_paged_prefill");
    int32_t rc = prefill_validate(pool, a);
    if (rc != VW_OK) return rc;
    if (a->num_seqs == 0 || a->num_tokens == 0) return VW_OK;
    DeviceScope ds(pool->cfg.device);
    const PoolGeom& g = pool->geom;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e;
    const float theta = (a->flags & VW_PREFILL_ROPE) ? a->rope_theta : 0.0f;
    if (a->k_new) {
        e = launch_prefill_append(g, pool->data, pool->scales, a->layer, a->k_new, a->v_new,
                                  a->cu_seqlens, a->ctx_start, a->block_tables, a->block_table_stride,
                                  a->num_seqs, a->num_tokens, theta, pool->err, s);
        if (e != cudaSuccess) return cuda_fail(e, "vw_paged_prefill: append launch");
    }
    PrefillLaunch L{};
    PrefillParams& p = L.p;
    p.q = a->q;
    p.out = a->out;
    p.cu_q = a->cu_seqlens;
    p.ctx_start = a->ctx_start;
    p.block_tables = a->block_tables;
    p.kv_data = pool->data;
    p.kv_scales = pool->scales;
    p.err = pool->err;
    p.B = a->num_seqs;
    p.T = a->num_tokens;
    p.Hq = a->num_q_heads;
    p.Hkv = g.num_kv_heads;
    p.group = a->num_q_heads / g.num_kv_heads;
    p.num_blocks = g.num_blocks;
    p.layer = a->layer;
    p.bt_stride = a->block_table_stride;
    p.causal = (a->flags & VW_PREFILL_CAUSAL) ? 1u : 0u;
    // the attention of a chunk waits for its append (same stream); the PDL flag
    // lets the first launch of the two overlap its predecessor
    p.flags = (a->flags & VW_PREFILL_PDL) && !a->k_new ? kDecodePdl : 0u;
    const float scale = a->scale > 0.0f ? a->scale : 1.0f / std::sqrt((float)g.head_dim);
    p.scale_log2 = scale * 1.4426950408889634f;
    p.rope_theta = theta;
    p.wait_cycles = pool->wait_cycles;
    L.tmap = &pool->tmap_half;
    L.head_dim = g.head_dim;
    L.kv_kind = g.kv_kind;
    L.io_kind = g.io_kind;
    L.stream = s;
    e = launch_paged_prefill(L);
    if (e != cudaSuccess) return cuda_fail(e, "vw_paged_prefill: launch");
    return VW_OK;
}

// ---------------------------------------------------------------------------
// FP8 weight path: rms_norm_fp8_out (kernels/norm/rms_norm.bm:62-94) and
// gemm_fp8 (kernels/gemm/gemm_fp8.bm:31-107).
// ---------------------------------------------------------------------------

int32_t vw_rms_norm_fp8_out(const void* x, const void* weight, uint8_t* out, uint32_t rows, uint32_t hidden,
                            float scale, float eps, void* stream) {
    VW_FAULT_POINT(kFaultLaunch, "vw_rms_norm_fp8_out");
    if (!x || !weight || !out) return fail(VW_ERR_INVALID_ARG, "vw_rms_norm_fp8_out: null pointer");
    if (hidden == 0) return fail(VW_ERR_INVALID_ARG, "vw_rms_norm_fp8_out: hidden must be > 0");
    if (!aligned(x, 2) || !aligned(weight, 2))
        return fail(VW_ERR_INVALID_ARG, "vw_rms_norm_fp8_out: misaligned pointer");
    if (!std::isfinite(scale) || !(eps >= 0.0f) || !std::isfinite(eps))
        return fail(VW_ERR_INVALID_ARG, "vw_rms_norm_fp8_out: bad scale / eps");
    cudaError_t e = launch_rms_norm_fp8(x, weight, out, rows, hidden, scale, eps, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? VW_OK : cuda_fail(e, "vw_rms_norm_fp8_out");
}

int32_t vw_gemm_fp8(const uint8_t* a, const uint8_t* b, void* c, const void* bias, uint32_t M, uint32_t N,
                    uint32_t K, float a_scale, float b_scale, void* stream) {
    VW_FAULT_POINT(kFaultLaunch, "vw_gemm_fp8");
    if (!a || !b || !c) return fail(VW_ERR_INVALID_ARG, "vw_gemm_fp8: null pointer");
    if (M == 0 || N == 0 || K == 0) return fail(VW_ERR_INVALID_ARG, "vw_gemm_fp8: empty shape");
    if (N % 16 || K % 16) return fail(VW_ERR_UNSUPPORTED, "vw_gemm_fp8: N and K must be multiples of 16");
    if ((uint64_t)M * K >= (1ull << 40) || (uint64_t)K * N >= (1ull << 40))
        return fail(VW_ERR_INVALID_ARG, "vw_gemm_fp8: too large");
    if (!aligned(a, 16) || !aligned(b, 16) || !aligned(c, 16) || (bias && !aligned(bias, 2)))
        return fail(VW_ERR_INVALID_ARG, "vw_gemm_fp8: misaligned pointer");
    if (!std::isfinite(a_scale) || !std::isfinite(b_scale))
        return fail(VW_ERR_INVALID_ARG, "vw_gemm_fp8: bad scale");
    cudaError_t e = launch_gemm_fp8(a, b, c, bias, M, N, K, a_scale, b_scale, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? VW_OK : cuda_fail(e, "vw_gemm_fp8");
}

int32_t vw_fp8_weight_check(uint32_t* device_error) {
    uint32_t w = 0;
    cudaError_t e = fp8w_error(&w, true);
    if (device_error) *device_error = w;
    if (e != cudaSuccess) return cuda_fail(e, "vw_fp8_weight_check");
    return w ? VW_ERR_DEVICE_CHECK : VW_OK;
}

int32_t vw_decode_plan(vw_pool* pool, const uint32_t* block_tables, const uint32_t* seq_lens,
                       uint32_t num_seqs, uint32_t block_table_stride, uint32_t num_q_heads,
                       void* stream) {
    VW_FAULT_POINT(kFaultLaunch, "vw_decode_plan");
    if (!pool) return fail(VW_ERR_INVALID_ARG, "vw_decode_plan: null pool");
    const PoolGeom& g = pool->geom;
    if (num_seqs == 0 || num_seqs > pool->cfg.max_batch)
        return fail(VW_ERR_INVALID_ARG, "vw_decode_plan: num_seqs %u not in 1..%u", num_seqs,
                    pool->cfg.max_batch);
    if (!block_tables || !seq_lens || !aligned(block_tables, 4) || !aligned(seq_lens, 4))
        return fail(VW_ERR_INVALID_ARG, "vw_decode_plan: bad block_tables / seq_lens pointer");
    if (block_table_stride == 0)
        return fail(VW_ERR_INVALID_ARG, "vw_decode_plan: block_table_stride must be > 0");
    if (num_q_heads == 0 || num_q_heads % g.num_kv_heads != 0 || num_q_heads / g.num_kv_heads > 16)
        return fail(VW_ERR_INVALID_ARG, "vw_decode_plan: num_q_heads %u does not fit %u KV heads",
                    num_q_heads, g.num_kv_heads);
    DeviceScope ds(pool->cfg.device);
    DecodeParams p{};
    p.block_tables = block_tables;
    p.seq_lens = seq_lens;
    p.err = pool->err;
    p.B = num_seqs;
    p.Hq = num_q_heads;
    p.Hkv = g.num_kv_heads;
    p.group = num_q_heads / g.num_kv_heads;
    p.num_blocks = g.num_blocks;
    p.bt_stride = block_table_stride;
    p.seg_cost = segment_cost(g);
    cudaError_t e = launch_decode_plan(p, pool->grid, pool->plan, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "vw_decode_plan launch");
    pool->plan_ready = true;
    pool->plan_tables = block_tables;
    pool->plan_lens = seq_lens;
    pool->plan_seqs = num_seqs;
    pool->plan_stride = block_table_stride;
    pool->plan_q_heads = num_q_heads;
    return VW_OK;
}

int32_t vw_block_copy(vw_pool* pool, const uint32_t* pairs, uint32_t num_pairs, void* stream) {
    VW_FAULT_POINT(kFaultLaunch, "vw_block_copy");
    if (!pool) return fail(VW_ERR_INVALID_ARG, "vw_block_copy: null pool");
    if (num_pairs == 0) return VW_OK;
    if (!pairs || !aligned(pairs, 8)) return fail(VW_ERR_INVALID_ARG, "vw_block_copy: bad pairs");
    DeviceScope ds(pool->cfg.device);
    cudaError_t e = launch_block_copy(pool->geom, pool->data, pool->scales, pairs, num_pairs,
                                      pool->err, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? VW_OK : cuda_fail(e, "vw_block_copy launch");
}

int32_t vw_kv_gather(vw_pool* pool, uint32_t layer, const uint32_t* block_table, uint32_t seq_len,
                     void* out_k, void* out_v, float* out_k_scales, float* out_v_scales,
                     void* stream) {
    VW_FAULT_POINT(kFaultLaunch, "vw_kv_gather");
    if (!pool) return fail(VW_ERR_INVALID_ARG, "vw_kv_gather: null pool");
    if (layer >= pool->geom.num_layers) return fail(VW_ERR_INVALID_ARG, "vw_kv_gather: bad layer");
    if (seq_len == 0) return VW_OK;
    if ((uint64_t)seq_len * 2 * pool->geom.num_kv_heads >= (1ull << 31))
        return fail(VW_ERR_INVALID_ARG, "vw_kv_gather: seq_len %u too large", seq_len);
    if (!block_table || !out_k || !out_v || !aligned(out_k, 16) || !aligned(out_v, 16))
        return fail(VW_ERR_INVALID_ARG, "vw_kv_gather: bad output pointers");
    if (pool->geom.kv_kind == kFP8 && (!out_k_scales || !out_v_scales))
        return fail(VW_ERR_INVALID_ARG, "vw_kv_gather: FP8 pools need scale outputs");
    DeviceScope ds(pool->cfg.device);
    cudaError_t e = launch_kv_gather(pool->geom, pool->data, pool->scales, layer, block_table,
                                     seq_len, out_k, out_v, out_k_scales, out_v_scales, pool->err,
                                     static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? VW_OK : cuda_fail(e, "vw_kv_gather launch");
}

// ---------------------------------------------------------------------------
// Host-buffer step: H2D of the step's inputs, append + decode on every layer,
// D2H of the outputs, the copies overlapping the kernels.
//  * Directly on the stream: layers in 4 chunks; the uploads of chunk c+1 and
//    the read-back of chunk c-1 overlap the kernels of chunk c.  The first
//    launch of a chunk follows a cross-stream wait, so it does not overlap its
//    predecessor (programmatic dependent launch needs the kernel just before).
//  * Recorded as a CUDA graph on the second call with the same arguments and
//    buffers, and replayed from then on: in a graph the uploads are plain
//    dependencies, so every launch after the first keeps its overlap with the
//    one before, the uploads can be fine at the start (layers 1, 1, 2, 4, ...:
//    the first decode waits for one layer's rows) and each layer's outputs go
//    back as soon as its combine ends (only the last layer's read-back remains
//    after the kernels); one graph launch replaces the 2 L kernel launches.
// ---------------------------------------------------------------------------

static int32_t enqueue_step_host(vw_pool* pool, const vw_step_host_args* a, cudaStream_t cs, bool graph) {
    const PoolGeom& g = pool->geom;
    const uint32_t B = a->num_seqs, Hq = a->num_q_heads, L = g.num_layers, D = g.head_dim;
    const size_t qb = (size_t)B * Hq * D * 2, kb = (size_t)B * g.num_kv_heads * D * 2;
    const size_t btb = (size_t)B * a->block_table_stride * 4, slb = (size_t)B * 4;
    auto up = [](size_t x) { return (x + 255) & ~size_t(255); };
    uint8_t* d_q = pool->stage;
    uint8_t* d_out = d_q + up(qb * L);
    uint8_t* d_k = d_out + up(qb * L);
    uint8_t* d_v = d_k + up(kb * L);
    uint32_t* d_bt = reinterpret_cast<uint32_t*>(d_v + up(kb * L));
    uint32_t* d_sl = reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(d_bt) + up(btb));
    // upload chunks [cut[c], cut[c+1]) and read-back groups [back[r], back[r+1])
    std::vector<uint32_t> cut{0}, back{0};
    if (graph) {
        for (uint32_t n = 1; cut.back() < L; n = cut.size() <= 2 ? 1 : n * 2)
            cut.push_back(std::min(L, cut.back() + n));
        // every layer's outputs go back as soon as it ends (measured against
        // groups of 4 layers and one read-back after the last layer: 3867,
        // 3835 and 3553 GB/s end to end on the Qwen step)
        for (uint32_t l = 1; l <= L; ++l) back.push_back(l);
    } else {
        const uint32_t chunks = L < 4 ? L : 4;
        for (uint32_t c = 1; c <= chunks; ++c) cut.push_back(L * c / chunks);
        back = cut;
    }
    const size_t nev = std::max(cut.size(), back.size());
    while (pool->ev_in.size() < nev) {
        cudaEvent_t x, y;
        if (cudaEventCreateWithFlags(&x, cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&y, cudaEventDisableTiming) != cudaSuccess)
            return fail(VW_ERR_CUDA, "vw_decode_step_host: event creation failed");
        pool->ev_in.push_back(x);
        pool->ev_done.push_back(y);
    }
    const uint8_t* hq = static_cast<const uint8_t*>(a->q);
    const uint8_t* hk = static_cast<const uint8_t*>(a->k_new);
    const uint8_t* hv = static_cast<const uint8_t*>(a->v_new);
    uint8_t* ho = static_cast<uint8_t*>(a->out);
    cudaEventRecord(pool->ev_entry, cs);
    cudaStreamWaitEvent(pool->s_h2d, pool->ev_entry, 0);
    cudaStreamWaitEvent(pool->s_d2h, pool->ev_entry, 0);
    // the tables go up on the read-back stream (idle until the first layer
    // ends), beside the first layer's rows on the upload stream
    cudaMemcpyAsync(d_bt, a->block_tables, btb, cudaMemcpyHostToDevice, pool->s_d2h);
    cudaMemcpyAsync(d_sl, a->seq_lens, slb, cudaMemcpyHostToDevice, pool->s_d2h);
    cudaEventRecord(pool->ev_exit, pool->s_d2h);
    cudaStreamWaitEvent(cs, pool->ev_exit, 0);
    for (size_t c = 0; c + 1 < cut.size(); ++c) {
        const uint32_t l0 = cut[c], nl = cut[c + 1] - cut[c];
        cudaMemcpyAsync(d_q + l0 * qb, hq + l0 * qb, nl * qb, cudaMemcpyHostToDevice, pool->s_h2d);
        cudaMemcpyAsync(d_k + l0 * kb, hk + l0 * kb, nl * kb, cudaMemcpyHostToDevice, pool->s_h2d);
        cudaMemcpyAsync(d_v + l0 * kb, hv + l0 * kb, nl * kb, cudaMemcpyHostToDevice, pool->s_h2d);
        cudaEventRecord(pool->ev_in[c], pool->s_h2d);
    }
    int32_t rc = VW_OK;
    size_t c = 0, r = 0;
    for (uint32_t l = 0; l < L && rc == VW_OK; ++l) {
        bool waited = false;
        if (l == cut[c]) {                               // the chunk's rows are on the device
            cudaStreamWaitEvent(cs, pool->ev_in[c++], 0);
            waited = true;
        }
        vw_decode_args da{};
        da.layer = l;
        da.num_seqs = B;
        da.num_q_heads = Hq;
        da.block_table_stride = a->block_table_stride;
        da.q = d_q + l * qb;
        da.block_tables = d_bt;
        da.seq_lens = d_sl;
        da.out = d_out + l * qb;
        da.k_new = d_k + l * kb;
        da.v_new = d_v + l * kb;
        da.scale = a->scale;
        // the previous launch writes only its own layer's pages and outputs, so
        // this one may start early and stream its pages
        if (l > 0 && (graph || !waited)) da.flags = VW_DECODE_PDL | VW_DECODE_EARLY_PAGES;
        if (a->rope_theta > 0.0f) {
            da.flags |= VW_DECODE_ROPE;
            da.rope_theta = a->rope_theta;
        }
        rc = decode_validate(pool, &da);
        if (rc == VW_OK) rc = decode_launch(pool, &da, cs);
        if (rc == VW_OK && l + 1 == back[r + 1]) {       // read back a finished group
            const uint32_t l0 = back[r];
            cudaEventRecord(pool->ev_done[r], cs);
            cudaStreamWaitEvent(pool->s_d2h, pool->ev_done[r], 0);
            cudaMemcpyAsync(ho + l0 * qb, d_out + l0 * qb, (l + 1 - l0) * qb, cudaMemcpyDeviceToHost,
                            pool->s_d2h);
            ++r;
        }
    }
    // join both side streams back into cs (a recorded graph must end joined)
    cudaEventRecord(pool->ev_exit, pool->s_d2h);
    cudaStreamWaitEvent(cs, pool->ev_exit, 0);
    if (c < cut.size() - 1) cudaStreamWaitEvent(cs, pool->ev_in[cut.size() - 2], 0);
    return rc;
}

int32_t vw_decode_step_host(vw_pool* pool, const vw_step_host_args* a, void* stream) {
    VW_FAULT_POINT(kFaultAll, "vw_decode_step_host");
    if (!pool || !a) return fail(VW_ERR_INVALID_ARG, "vw_decode_step_host: null argument");
    if (a->reserved) return fail(VW_ERR_INVALID_ARG, "vw_decode_step_host: reserved");
    if (a->rope_theta != 0.0f && !(a->rope_theta > 1.0f && std::isfinite(a->rope_theta)))
        return fail(VW_ERR_INVALID_ARG, "vw_decode_step_host: rope_theta must be 0 or a finite value > 1");
    const PoolGeom& g = pool->geom;
    const uint32_t B = a->num_seqs, Hq = a->num_q_heads, L = g.num_layers, D = g.head_dim;
    if (B == 0) return VW_OK;
    if (!a->q || !a->k_new || !a->v_new || !a->block_tables || !a->seq_lens || !a->out)
        return fail(VW_ERR_INVALID_ARG, "vw_decode_step_host: null host pointer");
    const size_t qb = (size_t)B * Hq * D * 2, kb = (size_t)B * g.num_kv_heads * D * 2;
    const size_t btb = (size_t)B * a->block_table_stride * 4, slb = (size_t)B * 4;
    auto up = [](size_t x) { return (x + 255) & ~size_t(255); };
    const size_t need = up(qb * L) * 2 + up(kb * L) * 2 + up(btb) + up(slb);
    DeviceScope ds(pool->cfg.device);
    cudaError_t e;
    if (pool->stage_bytes < need) {
        if (pool->stage) cudaFree(pool->stage);
        pool->stage = nullptr;
        pool->stage_bytes = 0;
        if ((e = dev_alloc(&pool->stage, need)) != cudaSuccess)
            return fail(VW_ERR_OOM, "vw_decode_step_host: staging: %s", cudaGetErrorString(e));
        pool->stage_bytes = need;
    }
    if (!pool->s_h2d) {
        if (cudaStreamCreateWithFlags(&pool->s_h2d, cudaStreamNonBlocking) != cudaSuccess ||
            cudaStreamCreateWithFlags(&pool->s_d2h, cudaStreamNonBlocking) != cudaSuccess ||
            cudaStreamCreateWithFlags(&pool->s_cap, cudaStreamNonBlocking) != cudaSuccess ||
            cudaEventCreateWithFlags(&pool->ev_entry, cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&pool->ev_exit, cudaEventDisableTiming) != cudaSuccess)
            return fail(VW_ERR_CUDA, "vw_decode_step_host: stream/event creation failed");
    }
    cudaStream_t cs = static_cast<cudaStream_t>(stream);
    uint32_t sb, tb;
    std::memcpy(&sb, &a->scale, 4);
    std::memcpy(&tb, &a->rope_theta, 4);
    const StepKey key{B, Hq, a->block_table_stride, sb, tb, a->q, a->k_new, a->v_new,
                      a->block_tables, a->seq_lens, a->out, pool->stage};
    if (!(pool->step_exec && key == pool->step_key) && key == pool->step_seen && !(key == pool->step_bad)) {
        // second call with these arguments: record the step once
        if (pool->step_exec) cudaGraphExecDestroy(pool->step_exec);
        pool->step_exec = nullptr;
        int32_t rc = VW_ERR_CUDA;
        cudaGraph_t graph = nullptr;
        if (cudaStreamBeginCapture(pool->s_cap, cudaStreamCaptureModeThreadLocal) == cudaSuccess) {
            rc = enqueue_step_host(pool, a, pool->s_cap, true);
            if (cudaStreamEndCapture(pool->s_cap, &graph) != cudaSuccess) rc = VW_ERR_CUDA;
        }
        if (rc == VW_OK && graph &&
            cudaGraphInstantiateWithFlags(&pool->step_exec, graph, 0) == cudaSuccess)
            pool->step_key = key;
        else {
            pool->step_exec = nullptr;            // not recordable (e.g. pageable host buffers):
            pool->step_bad = key;                 // these arguments stay on the direct path
        }
        if (graph) cudaGraphDestroy(graph);
        (void)cudaGetLastError();
    }
    if (pool->step_exec && key == pool->step_key) {
        if ((e = cudaGraphLaunch(pool->step_exec, cs)) != cudaSuccess)
            return cuda_fail(e, "vw_decode_step_host: graph launch");
        if ((e = cudaStreamSynchronize(cs)) != cudaSuccess) return cuda_fail(e, "vw_decode_step_host");
        return VW_OK;
    }
    pool->step_seen = key;
    int32_t rc = enqueue_step_host(pool, a, cs, false);
    e = cudaStreamSynchronize(cs);
    if (rc != VW_OK) return rc;
    if (e != cudaSuccess) return cuda_fail(e, "vw_decode_step_host");
    e = cudaGetLastError();
    return e == cudaSuccess ? VW_OK : cuda_fail(e, "vw_decode_step_host");
}

// ---------------------------------------------------------------------------
// voidweb_forward_pass: the symbol KernelLib::open binds (engine/ffi.bm:68).
// ---------------------------------------------------------------------------

namespace {
// Pinned host memory kept across forward passes (grow-only): the step's block
// tables and lengths, and the gathered decode rows of a mixed batch.  Reusing
// the same pinned buffers keeps vw_decode_step_host's arguments identical from
// one engine step to the next, so its recorded step graph is replayed instead
// of the copies and launches being issued one by one.
struct PinnedBuf {
    void* p = nullptr;
    size_t cap = 0;
    void* get(size_t bytes) {
        if (bytes <= cap) return p;
        if (p) cudaFreeHost(p);
        p = nullptr;
        cap = 0;
        if (pinned_alloc(&p, bytes) != cudaSuccess) {
            p = nullptr;
            (void)cudaGetLastError();
            return nullptr;
        }
        cap = bytes;
        return p;
    }
    void release() {
        if (p) cudaFreeHost(p);
        p = nullptr;
        cap = 0;
    }
};

struct ForwardState {
    std::mutex mu;
    vw_pool* pool = nullptr;
    const void* q = nullptr;
    const void* k = nullptr;
    const void* v = nullptr;
    void* out = nullptr;
    std::unordered_map<uint64_t, uint32_t> seq_len;   // tokens cached per sequence
    PinnedBuf table, lens, dq, dk, dv, dout;
};
ForwardState& fwd() {
    static ForwardState s;
    return s;
}
}  // namespace

int32_t vw_forward_bind(vw_pool* pool, const void* q, const void* k_new, const void* v_new,
                        void* attn_out) {
    ForwardState& s = fwd();
    std::lock_guard<std::mutex> lk(s.mu);
    if (!pool && s.pool) {          // unbinding: the pinned staging goes with the pool
        DeviceScope ds(s.pool->cfg.device);
        for (PinnedBuf* b : {&s.table, &s.lens, &s.dq, &s.dk, &s.dv, &s.dout}) b->release();
    }
    s.pool = pool;
    s.q = q;
    s.k = k_new;
    s.v = v_new;
    s.out = attn_out;
    return VW_OK;
}

int32_t vw_forward_set_seq_len(uint64_t seq_id, uint32_t len) {
    ForwardState& s = fwd();
    std::lock_guard<std::mutex> lk(s.mu);
    s.seq_len[seq_id] = len;
    return VW_OK;
}

int32_t vw_forward_release(uint64_t seq_id) {
    ForwardState& s = fwd();
    std::lock_guard<std::mutex> lk(s.mu);
    s.seq_len.erase(seq_id);
    return VW_OK;
}

// The prefill descriptors of a forward pass (rows gathered from the bound
// buffers into [L][Tp][...] host arrays): per layer, chunk append + causal
// prefill attention, with the outputs copied back to `out` [L][Tp][Hq][D].
static int32_t forward_prefill(vw_pool* pool, uint32_t L, uint32_t Hq, uint32_t Bp, uint32_t Tp,
                               const std::vector<uint8_t>& q, const std::vector<uint8_t>& k,
                               const std::vector<uint8_t>& v, const std::vector<int32_t>& cu,
                               const std::vector<int32_t>& ctx, const std::vector<uint32_t>& bt,
                               uint32_t stride, float rope_theta, std::vector<uint8_t>& out) {
    const PoolGeom& g = pool->geom;
    const size_t qb = (size_t)Tp * Hq * g.head_dim * 2, kb = (size_t)Tp * g.num_kv_heads * g.head_dim * 2;
    auto up = [](size_t x) { return (x + 255) & ~size_t(255); };
    const size_t need = up(qb) * 2 * L + up(kb) * 2 * L + up(cu.size() * 4) + up(ctx.size() * 4) +
                        up(bt.size() * 4);
    DeviceScope ds(pool->cfg.device);
    cudaError_t e;
    if (pool->pstage_bytes < need) {
        if (pool->pstage) cudaFree(pool->pstage);
        pool->pstage = nullptr;
        pool->pstage_bytes = 0;
        if ((e = dev_alloc(&pool->pstage, need)) != cudaSuccess)
            return fail(VW_ERR_OOM, "voidweb_forward_pass: prefill staging: %s", cudaGetErrorString(e));
        pool->pstage_bytes = need;
    }
    uint8_t* d_q = pool->pstage;
    uint8_t* d_out = d_q + up(qb) * L;
    uint8_t* d_k = d_out + up(qb) * L;
    uint8_t* d_v = d_k + up(kb) * L;
    int32_t* d_cu = reinterpret_cast<int32_t*>(d_v + up(kb) * L);
    int32_t* d_ctx = reinterpret_cast<int32_t*>(reinterpret_cast<uint8_t*>(d_cu) + up(cu.size() * 4));
    uint32_t* d_bt = reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(d_ctx) + up(ctx.size() * 4));
    bool ok = cudaMemcpy(d_cu, cu.data(), cu.size() * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
              cudaMemcpy(d_ctx, ctx.data(), ctx.size() * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
              cudaMemcpy(d_bt, bt.data(), bt.size() * 4, cudaMemcpyHostToDevice) == cudaSuccess;
    for (uint32_t l = 0; l < L && ok; ++l)
        ok = cudaMemcpy(d_q + l * up(qb), q.data() + l * qb, qb, cudaMemcpyHostToDevice) == cudaSuccess &&
             cudaMemcpy(d_k + l * up(kb), k.data() + l * kb, kb, cudaMemcpyHostToDevice) == cudaSuccess &&
             cudaMemcpy(d_v + l * up(kb), v.data() + l * kb, kb, cudaMemcpyHostToDevice) == cudaSuccess;
    if (!ok) return fail(VW_ERR_CUDA, "voidweb_forward_pass: prefill upload");
    for (uint32_t l = 0; l < L; ++l) {
        vw_prefill_args pa{};
        pa.layer = l;
        pa.num_seqs = Bp;
        pa.num_tokens = Tp;
        pa.num_q_heads = Hq;
        pa.block_table_stride = stride;
        pa.flags = VW_PREFILL_CAUSAL | (rope_theta > 0.0f ? VW_PREFILL_ROPE : 0u);
        pa.q = d_q + l * up(qb);
        pa.k_new = d_k + l * up(kb);
        pa.v_new = d_v + l * up(kb);
        pa.cu_seqlens = d_cu;
        pa.ctx_start = d_ctx;
        pa.block_tables = d_bt;
        pa.out = d_out + l * up(qb);
        pa.scale = 0.0f;
        pa.rope_theta = rope_theta;
        int32_t rc = vw_paged_prefill(pool, &pa, nullptr);
        if (rc != VW_OK) return rc;
    }
    out.resize(qb * L);
    for (uint32_t l = 0; l < L; ++l)
        if ((e = cudaMemcpy(out.data() + l * qb, d_out + l * up(qb), qb, cudaMemcpyDeviceToHost)) != cudaSuccess)
            return cuda_fail(e, "voidweb_forward_pass: prefill download");
    return VW_OK;
}

int32_t voidweb_forward_pass(const ForwardArgs* args) {
    VW_FAULT_POINT(kFaultAll, "voidweb_forward_pass");
    if (!args) return fail(VW_ERR_INVALID_ARG, "voidweb_forward_pass: null args");
    ForwardState& s = fwd();
    std::lock_guard<std::mutex> lk(s.mu);
    if (!s.pool || !s.q || !s.k || !s.v || !s.out)
        return fail(VW_ERR_INVALID_ARG, "voidweb_forward_pass: no pool / attention I/O bound");
    ForwardArgs a;
    std::memcpy(&a, args, sizeof a);     // packed struct: copy out before reading fields
    const PoolGeom& g = s.pool->geom;
    if (a.num_kv_heads != g.num_kv_heads || a.head_dim != g.head_dim || a.num_layers != g.num_layers)
        return fail(VW_ERR_INVALID_ARG, "voidweb_forward_pass: model shape does not match the pool");
    if (a.num_seqs == 0) return VW_OK;
    if (!a.seqs) return fail(VW_ERR_INVALID_ARG, "voidweb_forward_pass: null seqs");
    if (a.num_heads == 0 || a.num_heads % g.num_kv_heads != 0)
        return fail(VW_ERR_INVALID_ARG, "voidweb_forward_pass: num_heads %u does not fit %u KV heads",
                    a.num_heads, g.num_kv_heads);
    std::vector<SeqDescriptor> d(a.num_seqs);
    std::memcpy(d.data(), a.seqs, sizeof(SeqDescriptor) * a.num_seqs);
    const uint32_t L = g.num_layers, Hq = a.num_heads, D = g.head_dim, Hkv = g.num_kv_heads;
    // rows of descriptor i: [row0[i], row0[i] + num_tokens)
    std::vector<uint32_t> row0(a.num_seqs), pos(a.num_seqs), pf, dc;
    uint64_t T = 0;
    uint32_t stride = 1;
    std::unordered_map<uint64_t, uint32_t> seen;
    for (uint32_t i = 0; i < a.num_seqs; ++i) {
        const SeqDescriptor& sd = d[i];
        if (sd.num_tokens == 0 || (!sd.is_prefill && sd.num_tokens != 1))
            return fail(VW_ERR_INVALID_ARG, "voidweb_forward_pass: seq %llu has %u tokens",
                        (unsigned long long)sd.seq_id, sd.num_tokens);
        if (seen.count(sd.seq_id))
            return fail(VW_ERR_INVALID_ARG, "voidweb_forward_pass: seq %llu appears twice",
                        (unsigned long long)sd.seq_id);
        seen[sd.seq_id] = i;
        row0[i] = (uint32_t)T;
        T += sd.num_tokens;
        pos[i] = s.seq_len.count(sd.seq_id) ? s.seq_len[sd.seq_id] : 0;
        if ((uint64_t)pos[i] + sd.num_tokens > (uint64_t)sd.num_blocks * 16)
            return fail(VW_ERR_INVALID_ARG, "voidweb_forward_pass: seq %llu needs %llu blocks, has %u",
                        (unsigned long long)sd.seq_id,
                        (unsigned long long)(((uint64_t)pos[i] + sd.num_tokens + 15) / 16), sd.num_blocks);
        if (sd.num_blocks && !sd.block_ptr)
            return fail(VW_ERR_INVALID_ARG, "voidweb_forward_pass: null block_ptr");
        if (sd.num_blocks > stride) stride = sd.num_blocks;
        (sd.is_prefill ? pf : dc).push_back(i);
    }
    if (T > (1u << 24)) return fail(VW_ERR_INVALID_ARG, "voidweb_forward_pass: too many tokens");
    const float theta = a.rope_theta > 1.0f ? a.rope_theta : 0.0f;
    const size_t qrow = (size_t)Hq * D * 2, krow = (size_t)Hkv * D * 2;
    const uint8_t* hq = static_cast<const uint8_t*>(s.q);
    const uint8_t* hk = static_cast<const uint8_t*>(s.k);
    const uint8_t* hv = static_cast<const uint8_t*>(s.v);
    uint8_t* ho = static_cast<uint8_t*>(s.out);
    auto table_of = [&](uint32_t i, uint32_t* dst) {
        std::memcpy(dst, reinterpret_cast<const void*>(d[i].block_ptr), (size_t)d[i].num_blocks * 4);
    };

    if (!pf.empty()) {
        const uint32_t Bp = (uint32_t)pf.size();
        uint32_t Tp = 0;
        std::vector<int32_t> cu(Bp + 1, 0), ctx(Bp);
        std::vector<uint32_t> bt((size_t)Bp * stride, 0);
        for (uint32_t k = 0; k < Bp; ++k) {
            cu[k] = (int32_t)Tp;
            Tp += d[pf[k]].num_tokens;
            ctx[k] = (int32_t)pos[pf[k]];
            table_of(pf[k], &bt[(size_t)k * stride]);
        }
        cu[Bp] = (int32_t)Tp;
        std::vector<uint8_t> q((size_t)L * Tp * qrow), kk((size_t)L * Tp * krow), vv((size_t)L * Tp * krow), o;
        for (uint32_t l = 0; l < L; ++l)
            for (uint32_t k = 0; k < Bp; ++k) {
                const size_t n = d[pf[k]].num_tokens, src = (size_t)l * T + row0[pf[k]], dst = (size_t)l * Tp + cu[k];
                std::memcpy(&q[dst * qrow], hq + src * qrow, n * qrow);
                std::memcpy(&kk[dst * krow], hk + src * krow, n * krow);
                std::memcpy(&vv[dst * krow], hv + src * krow, n * krow);
            }
        int32_t rc = forward_prefill(s.pool, L, Hq, Bp, Tp, q, kk, vv, cu, ctx, bt, stride, theta, o);
        if (rc != VW_OK) return rc;
        for (uint32_t l = 0; l < L; ++l)
            for (uint32_t k = 0; k < Bp; ++k) {
                const size_t n = d[pf[k]].num_tokens, dst = (size_t)l * T + row0[pf[k]], src = (size_t)l * Tp + cu[k];
                std::memcpy(ho + dst * qrow, &o[src * qrow], n * qrow);
            }
    }

    if (!dc.empty()) {
        const uint32_t Bd = (uint32_t)dc.size();
        DeviceScope ds(s.pool->cfg.device);
        uint32_t* table = static_cast<uint32_t*>(s.table.get((size_t)Bd * stride * 4));
        uint32_t* lens = static_cast<uint32_t*>(s.lens.get((size_t)Bd * 4));
        if (!table || !lens) return fail(VW_ERR_OOM, "voidweb_forward_pass: pinned staging");
        std::memset(table, 0, (size_t)Bd * stride * 4);
        for (uint32_t k = 0; k < Bd; ++k) {
            table_of(dc[k], &table[(size_t)k * stride]);
            lens[k] = pos[dc[k]] + 1;
        }
        // an all-decode batch uses the bound buffers in place; otherwise the
        // decode rows are gathered into [L][Bd][...] pinned arrays first
        const bool direct = pf.empty();
        uint8_t *q = nullptr, *kk = nullptr, *vv = nullptr, *o = nullptr;
        if (!direct) {
            q = static_cast<uint8_t*>(s.dq.get((size_t)L * Bd * qrow));
            kk = static_cast<uint8_t*>(s.dk.get((size_t)L * Bd * krow));
            vv = static_cast<uint8_t*>(s.dv.get((size_t)L * Bd * krow));
            o = static_cast<uint8_t*>(s.dout.get((size_t)L * Bd * qrow));
            if (!q || !kk || !vv || !o) return fail(VW_ERR_OOM, "voidweb_forward_pass: pinned staging");
            for (uint32_t l = 0; l < L; ++l)
                for (uint32_t k = 0; k < Bd; ++k) {
                    const size_t src = (size_t)l * T + row0[dc[k]], dst = (size_t)l * Bd + k;
                    std::memcpy(&q[dst * qrow], hq + src * qrow, qrow);
                    std::memcpy(&kk[dst * krow], hk + src * krow, krow);
                    std::memcpy(&vv[dst * krow], hv + src * krow, krow);
                }
        }
        vw_step_host_args st{};
        st.num_seqs = Bd;
        st.num_q_heads = Hq;
        st.block_table_stride = stride;
        st.q = direct ? s.q : q;
        st.k_new = direct ? s.k : kk;
        st.v_new = direct ? s.v : vv;
        st.block_tables = table;
        st.seq_lens = lens;
        st.out = direct ? s.out : o;
        st.scale = 0.0f;
        // ModelConfig.rope_theta (engine/ffi.bm:37): q and the new K rows are rotated
        // in the decode, as the engine's own kernels would before attention
        st.rope_theta = theta;
        int32_t rc = vw_decode_step_host(s.pool, &st, nullptr);
        if (rc != VW_OK) return rc;
        if (!direct)
            for (uint32_t l = 0; l < L; ++l)
                for (uint32_t k = 0; k < Bd; ++k)
                    std::memcpy(ho + ((size_t)l * T + row0[dc[k]]) * qrow, o + ((size_t)l * Bd + k) * qrow, qrow);
    }
    for (uint32_t i = 0; i < a.num_seqs; ++i) s.seq_len[d[i].seq_id] = pos[i] + d[i].num_tokens;
    return VW_OK;
}

}  // extern "C"

// ------------------------------------------------------------ static scratch
//
// vw_paged_decode_static: the decode of vw_paged_decode with its split-K
// partials in a fixed array compiled into this library instead of the pool's
// scratch.  The array is sized for the decode grid of a B200 (148 SMs x 2 CTAs
// = 296 CTAs), head_dim up to 128 and up to 16 query heads per KV head:
// 296 * 2 * 16 * 128 f32 of partial outputs (4.85 MB) plus 296 * 2 * 16 * 2
// f32 of (max, sum) (74 KB), one copy per device.  A launch whose grid needs
// more is rejected.  The decode writes every partial that its combine grid
// reads within the same call, so nothing in the array has to start at zero.

namespace {

constexpr size_t kStaticCtas = 296;
constexpr size_t kStaticFloatsO = kStaticCtas * 2 * 16 * 128;
constexpr size_t kStaticFloatsMl = kStaticCtas * 2 * 16 * 2;
constexpr int kStaticMaxDevices = 64;

static __device__ __align__(256) float g_static_part_o[kStaticFloatsO];
static __device__ __align__(256) float g_static_part_ml[kStaticFloatsMl];

struct StaticScratch {
    float* o = nullptr;
    float* ml = nullptr;
};

// Device addresses of the two arrays, looked up once per device with that
// device current (the caller's DeviceScope).
int32_t static_scratch(int dev, StaticScratch* out) {
    static std::mutex mu;
    static StaticScratch addr[kStaticMaxDevices];
    static bool ready[kStaticMaxDevices] = {};
    if (dev < 0 || dev >= kStaticMaxDevices)
        return fail(VW_ERR_UNSUPPORTED, "vw_paged_decode_static: device ordinal %d out of range", dev);
    std::lock_guard<std::mutex> lock(mu);
    if (!ready[dev]) {
        void* po = nullptr;
        void* pml = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&po, g_static_part_o);
        if (e != cudaSuccess) return cuda_fail(e, "vw_paged_decode_static: cudaGetSymbolAddress (o)");
        e = cudaGetSymbolAddress(&pml, g_static_part_ml);
        if (e != cudaSuccess) return cuda_fail(e, "vw_paged_decode_static: cudaGetSymbolAddress (ml)");
        addr[dev].o = static_cast<float*>(po);
        addr[dev].ml = static_cast<float*>(pml);
        ready[dev] = true;
    }
    *out = addr[dev];
    return VW_OK;
}

}  // namespace

extern "C" {

int32_t vw_paged_decode_static(vw_pool* pool, const vw_decode_args* a, void* stream) {
    VW_FAULT_POINT(kFaultLaunch, "vw_paged_decode_static");
    int32_t rc = decode_validate(pool, a);
    if (rc != VW_OK) return rc;
    const PoolGeom& g = pool->geom;
    const size_t need_o = decode_scratch_floats_o(pool->grid, g.head_dim);
    const size_t need_ml = decode_scratch_floats_ml(pool->grid);
    if (need_o > kStaticFloatsO || need_ml > kStaticFloatsMl)
        return fail(VW_ERR_UNSUPPORTED,
                    "vw_paged_decode_static: a %d-CTA decode grid at head_dim %u needs %zu + %zu "
                    "floats of split-K scratch; the static array holds %zu + %zu (%zu CTAs at "
                    "head_dim 128); use vw_paged_decode",
                    pool->grid, g.head_dim, need_o, need_ml, kStaticFloatsO, kStaticFloatsMl,
                    kStaticCtas);
    if (a->num_seqs == 0) return VW_OK;
    DeviceScope ds(pool->cfg.device);
    if (!ds.ok) return fail(VW_ERR_CUDA, "vw_paged_decode_static: cannot select device %d", pool->cfg.device);
    StaticScratch sc;
    rc = static_scratch(pool->cfg.device, &sc);
    if (rc != VW_OK) return rc;
    // the same launch as vw_paged_decode (flags, plan, wait bound) with the
    // static array in place of the pool's scratch
    const DecodeScratch fixed{sc.o, sc.ml};
    return decode_launch(pool, a, static_cast<cudaStream_t>(stream), &fixed);
}

}  // extern "C"
