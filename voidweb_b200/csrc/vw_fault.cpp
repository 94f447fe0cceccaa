// vw_fault.cpp -- host-side fault injection for the engine's error paths.
//
// The engine treats any nonzero status of voidweb_forward_pass as a failed
// step (engine/ffi.bm:112-118) and an exhausted block pool as an allocation
// error (engine/kv_cache.bm:82-85).  To test those paths without faulting a
// GPU, a caller (or the environment) can arm a number of failures of one kind;
// the next entry points that can fail that way consume them, one per call,
// and return the status before they touch the device or the bookkeeping.
//
//   vw_fault_inject(VW_FAULT_OOM, 2)         the next two allocating calls fail
//   VOIDWEB_KV_FAULT="oom:2,invalid:1,cuda:1" the same, armed when the library loads
#include <atomic>
#include <cstdint>
#include <cstdlib>
#include <cstring>

#include "../../include/voidweb_kv.h"
#include "vw_fault.h"

namespace {

constexpr int kKinds = 4;    // index = VW_FAULT_* (0 unused)
std::atomic<uint32_t> g_pending[kKinds];

int32_t status_of(uint32_t kind) {
    switch (kind) {
        case VW_FAULT_OOM: return VW_ERR_OOM;
        case VW_FAULT_INVALID_ARG: return VW_ERR_INVALID_ARG;
        case VW_FAULT_CUDA: return VW_ERR_CUDA;
        default: return VW_OK;
    }
}

// VOIDWEB_KV_FAULT: comma-separated kind:count pairs, kinds oom / invalid / cuda.
struct EnvArm {
    EnvArm() {
        const char* s = std::getenv("VOIDWEB_KV_FAULT");
        if (!s) return;
        while (*s) {
            const char* colon = std::strchr(s, ':');
            if (!colon) break;
            const size_t len = (size_t)(colon - s);
            uint32_t kind = 0;
            if (len == 3 && std::strncmp(s, "oom", 3) == 0) kind = VW_FAULT_OOM;
            else if (len == 7 && std::strncmp(s, "invalid", 7) == 0) kind = VW_FAULT_INVALID_ARG;
            else if (len == 4 && std::strncmp(s, "cuda", 4) == 0) kind = VW_FAULT_CUDA;
            char* end = nullptr;
            const unsigned long n = std::strtoul(colon + 1, &end, 10);
            if (kind) g_pending[kind].store((uint32_t)n);
            s = end;
            while (*s == ',' || *s == ' ') ++s;
            if (end == colon + 1) break;
        }
    }
};
const EnvArm g_env_arm;

}  // namespace

namespace vw {

int32_t fault_take(uint32_t kinds, const char** what) {
    for (uint32_t k = 1; k < kKinds; ++k) {
        if (!(kinds & (1u << k))) continue;
        uint32_t n = g_pending[k].load();
        while (n > 0 && !g_pending[k].compare_exchange_weak(n, n - 1)) {
        }
        if (n > 0) {
            if (what) *what = k == VW_FAULT_OOM ? "out of memory" : k == VW_FAULT_INVALID_ARG
                                                                        ? "invalid argument"
                                                                        : "CUDA launch failure";
            return status_of(k);
        }
    }
    return VW_OK;
}

}  // namespace vw

extern "C" {

int32_t vw_fault_inject(uint32_t kind, uint32_t count) {
    if (kind == 0 || kind >= (uint32_t)kKinds) return VW_ERR_INVALID_ARG;
    g_pending[kind].store(count);
    return VW_OK;
}

uint32_t vw_fault_pending(uint32_t kind) {
    if (kind == 0 || kind >= (uint32_t)kKinds) return 0;
    return g_pending[kind].load();
}

}  // extern "C"
