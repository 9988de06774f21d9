// Host-side helpers shared by the library's translation units.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include "mxg.h"

namespace mxg {

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline int cuda_status(cudaError_t e) { return e == cudaSuccess ? MXG_OK : MXG_ERR_CUDA; }

// Longest a single mbarrier wait of a kernel may take before it gives up
// with MXG_ERR_DEVICE_TIMEOUT.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

// Current device is an sm_100-class GPU (cached per device ordinal).
int check_device();
// SM count of the current device (cached).
int num_sms();
// Device address of the per-device error word (set up once per device).
int* device_error_word();
// Stall-injection limit armed by mxg_debug_inject_stall (consumed by the next launch).
int64_t take_injected_stall();
// SMs the persistent GEMMs may use (0: all), set by mxg_set_gemm_sm_limit.
int gemm_sm_limit();
// The driver's cuTensorMapEncodeTiled (null when unavailable), looked up once.
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();

}  // namespace mxg
