// Error reporting, version and device queries of the C ABI.
#include "mqc_host.h"

#include <cstdio>
#include <cstring>
#include <mutex>

namespace mqc {

namespace {
thread_local char g_detail[512] = {0};
constexpr int kMaxDevices = 64;
int g_sm_count[kMaxDevices] = {0};  // written once per device; benign if raced
}  // namespace

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_detail, sizeof(g_detail), fmt, ap);
  va_end(ap);
  return code;
}

void clear_error() { g_detail[0] = '\0'; }

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    return fail(MQC_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
  }
  return MQC_OK;
}

int num_sms() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
  if (g_sm_count[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    g_sm_count[dev] = n;
  }
  return g_sm_count[dev];
}

namespace {
std::mutex g_pool_mu;
cudaMemPool_t g_pool[kMaxDevices] = {};

cudaError_t scratch_pool(cudaMemPool_t* out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_pool_mu);
  if (g_pool[dev] == nullptr) {
    cudaMemPoolProps props = {};
    props.allocType = cudaMemAllocationTypePinned;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = dev;
    cudaMemPool_t pool = nullptr;
    e = cudaMemPoolCreate(&pool, &props);
    if (e != cudaSuccess) return e;
    uint64_t keep = kScratchKeepBytes;
    e = cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
    if (e != cudaSuccess) {
      cudaMemPoolDestroy(pool);
      return e;
    }
    g_pool[dev] = pool;
  }
  *out = g_pool[dev];
  return cudaSuccess;
}
}  // namespace

cudaError_t scratch_alloc(void** p, size_t bytes, cudaStream_t st) {
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  cudaError_t e = cudaStreamIsCapturing(st, &cap);
  if (e != cudaSuccess) return e;
  if (cap != cudaStreamCaptureStatusNone) return cudaMallocAsync(p, bytes, st);
  cudaMemPool_t pool = nullptr;
  e = scratch_pool(&pool);
  if (e != cudaSuccess) return e;
  return cudaMallocFromPoolAsync(p, bytes, pool, st);
}

cudaError_t scratch_free(void* p, cudaStream_t st) { return cudaFreeAsync(p, st); }

}  // namespace mqc

extern "C" {

const char* mqc_version(void) { return "0.1.0"; }

const char* mqc_status_string(int status) {
  switch (status) {
    case MQC_OK: return "success";
    case MQC_ERR_INVALID_VALUE: return "invalid argument value";
    case MQC_ERR_MISALIGNED: return "pointer misaligned for vector access";
    case MQC_ERR_UNSUPPORTED: return "unsupported configuration";
    case MQC_ERR_CUDA: return "CUDA runtime error";
    case MQC_ERR_DEVICE_TIMEOUT: return "bounded device-side wait timed out";
    default: return "unknown status";
  }
}

const char* mqc_last_error(void) { return mqc::g_detail; }

}  // extern "C"
