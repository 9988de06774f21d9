// C-ABI support: device checks, the per-device error word, status strings.
#include <cuda_runtime.h>

#include <atomic>
#include <mutex>

#include "mxg.h"
#include "mxg_internal.h"

// Error word written by kernels (first error wins); one instance per device
// that loads the library.
__device__ int g_mxg_error = 0;

namespace mxg {

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_mu;
int g_sms[kMaxDevices] = {0};
int g_ok[kMaxDevices] = {0};  // 0 unknown, 1 supported, -1 unsupported
int* g_err_ptr[kMaxDevices] = {nullptr};
std::atomic<int64_t> g_stall_ns{0};

int current_device() {
  int d = -1;
  if (cudaGetDevice(&d) != cudaSuccess) return -1;
  return (d >= 0 && d < kMaxDevices) ? d : -1;
}
}  // namespace

int check_device() {
  const int d = current_device();
  if (d < 0) return MXG_ERR_CUDA;
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_ok[d] == 0) {
    cudaDeviceProp p;
    if (cudaGetDeviceProperties(&p, d) != cudaSuccess) return MXG_ERR_CUDA;
    g_ok[d] = (p.major == 10 && p.minor == 0) ? 1 : -1;
    g_sms[d] = p.multiProcessorCount;
  }
  return g_ok[d] == 1 ? MXG_OK : MXG_ERR_UNSUPPORTED_DEVICE;
}

int num_sms() {
  const int d = current_device();
  if (d < 0) return 1;
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_sms[d] == 0) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, d);
    g_sms[d] = v > 0 ? v : 1;
  }
  return g_sms[d];
}

int* device_error_word() {
  const int d = current_device();
  if (d < 0) return nullptr;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_err_ptr[d]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_mxg_error) != cudaSuccess) return nullptr;
    g_err_ptr[d] = reinterpret_cast<int*>(p);
  }
  return g_err_ptr[d];
}

int64_t take_injected_stall() { return g_stall_ns.exchange(0); }

static std::atomic<int> g_gemm_sm_limit{0};
int gemm_sm_limit() { return g_gemm_sm_limit.load(); }

}  // namespace mxg

extern "C" const char* mxg_error_string(int code) {
  switch (code) {
    case MXG_OK: return "ok";
    case MXG_ERR_INVALID_ARGUMENT: return "invalid argument";
    case MXG_ERR_BAD_SHAPE: return "unsupported shape";
    case MXG_ERR_MISALIGNED: return "pointer not 16-byte aligned";
    case MXG_ERR_WORKSPACE_TOO_SMALL: return "workspace too small";
    case MXG_ERR_CUDA: return "CUDA error";
    case MXG_ERR_DEVICE_TIMEOUT: return "device-side wait timed out";
    case MXG_ERR_BAD_OFFSETS: return "inconsistent group offsets";
    case MXG_ERR_UNSUPPORTED_DEVICE: return "device is not an sm_100 GPU";
    case MXG_ERR_TOO_MANY_GROUPS: return "too many groups";
    default: return "unknown error";
  }
}

extern "C" int mxg_version(void) { return 100; }

extern "C" int mxg_get_device_error(int* code, int clear) {
  if (!code) return MXG_ERR_INVALID_ARGUMENT;
  int* p = mxg::device_error_word();
  if (!p) return MXG_ERR_CUDA;
  if (cudaDeviceSynchronize() != cudaSuccess) return MXG_ERR_CUDA;
  int v = 0;
  if (cudaMemcpy(&v, p, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return MXG_ERR_CUDA;
  *code = v;
  if (clear && v != 0) {
    const int zero = 0;
    if (cudaMemcpy(p, &zero, sizeof(int), cudaMemcpyHostToDevice) != cudaSuccess) return MXG_ERR_CUDA;
  }
  return MXG_OK;
}

extern "C" int mxg_set_gemm_sm_limit(int sms) {
  if (sms < 0) return MXG_ERR_INVALID_ARGUMENT;
  mxg::g_gemm_sm_limit.store(sms);
  return MXG_OK;
}

extern "C" int mxg_get_gemm_sm_limit(void) { return mxg::g_gemm_sm_limit.load(); }

extern "C" int mxg_debug_inject_stall(int64_t timeout_ns) {
  if (timeout_ns < 0) return MXG_ERR_INVALID_ARGUMENT;
  mxg::g_stall_ns.store(timeout_ns);
  return MXG_OK;
}
