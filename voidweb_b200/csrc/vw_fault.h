// vw_fault.h -- host-side fault injection shared by the C-ABI entry points.
#pragma once
#include <cstdint>

namespace vw {

// Bit mask of VW_FAULT_* kinds an entry point can fail with.
constexpr uint32_t kCanOom = 1u << 1;      // VW_FAULT_OOM
constexpr uint32_t kCanInvalid = 1u << 2;  // VW_FAULT_INVALID_ARG
constexpr uint32_t kCanCuda = 1u << 3;     // VW_FAULT_CUDA

// Consumes one armed failure of the first kind in `kinds` that has one and
// returns its status (VW_ERR_OOM / VW_ERR_INVALID_ARG / VW_ERR_CUDA), with a
// short description in *what; VW_OK when none is armed.
int32_t fault_take(uint32_t kinds, const char** what);

}  // namespace vw
