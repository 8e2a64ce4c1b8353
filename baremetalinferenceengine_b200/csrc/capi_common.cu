// C ABI plumbing: status strings, the thread-local error message, device status
// read-back and per-device SM counts.
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include <map>
#include <mutex>
#include <utility>

#include "bm_host.h"

namespace bm {

namespace {
thread_local char g_message[512] = {0};
constexpr int kMaxDevices = 64;
int g_sm_count[kMaxDevices] = {0};  // 0 = not yet queried; benign race (same value)
}  // namespace

int fail(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_message, sizeof(g_message), fmt, ap);
  va_end(ap);
  return status;
}

void clear_error() { g_message[0] = '\0'; }

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("BM_PDL");
    return v == nullptr || std::strcmp(v, "0") != 0;
  }();
  return on;
}

int check_launch(const char* what) {
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) {
    return fail(BM_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(err));
  }
  return BM_OK;
}

int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return 148;
  if (dev < kMaxDevices && g_sm_count[dev] > 0) return g_sm_count[dev];
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
  if (dev < kMaxDevices) g_sm_count[dev] = n;
  return n;
}

int allow_dynamic_smem(const void* kernel, int bytes, const char* what) {
  static std::mutex mu;
  static std::map<std::pair<int, const void*>, int> granted;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) dev = -1;
  std::lock_guard<std::mutex> lock(mu);
  auto it = granted.find({dev, kernel});
  if (it != granted.end() && it->second >= bytes) return BM_OK;
  cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (err != cudaSuccess) return fail(BM_ERR_CUDA, "%s: %s", what, cudaGetErrorString(err));
  granted[{dev, kernel}] = bytes;
  return BM_OK;
}

}  // namespace bm

extern "C" {

const char* bm_status_string(int status) {
  switch (status) {
    case BM_OK:
      return "BM_OK";
    case BM_ERR_INVALID_ARGUMENT:
      return "BM_ERR_INVALID_ARGUMENT";
    case BM_ERR_CUDA:
      return "BM_ERR_CUDA";
    case BM_ERR_DEVICE:
      return "BM_ERR_DEVICE";
    default:
      return "BM_ERR_UNKNOWN";
  }
}

int bm_abi_version(void) { return BM_ABI_VERSION; }

const char* bm_last_error_message(void) { return bm::g_message; }

int bm_status_read(int32_t* d_status, int32_t* flags_out, void* stream) {
  if (d_status == nullptr || flags_out == nullptr) {
    return bm::fail(BM_ERR_INVALID_ARGUMENT, "bm_status_read: NULL pointer");
  }
  cudaStream_t s = bm::as_stream(stream);
  int32_t host = 0;
  cudaError_t err = cudaMemcpyAsync(&host, d_status, sizeof(int32_t), cudaMemcpyDeviceToHost, s);
  if (err == cudaSuccess) err = cudaMemsetAsync(d_status, 0, sizeof(int32_t), s);
  if (err == cudaSuccess) err = cudaStreamSynchronize(s);
  if (err != cudaSuccess) {
    return bm::fail(BM_ERR_CUDA, "bm_status_read: %s", cudaGetErrorString(err));
  }
  *flags_out = host;
  if (host != 0) {
    return bm::fail(BM_ERR_DEVICE, "device status bits 0x%x%s%s%s", host,
                    (host & BM_DEVERR_BAD_ID) ? " bad-token-id" : "",
                    (host & BM_DEVERR_BAD_POSITION) ? " bad-position" : "",
                    (host & BM_DEVERR_BAD_SEQUENCE) ? " bad-sequence" : "");
  }
  bm::clear_error();
  return BM_OK;
}

}  // extern "C"
