// Host-side helpers shared by the C-ABI entry points: argument checks that set
// the per-thread error detail, and launch-error translation.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>

#include "mambaqc_b200.h"

namespace mqc {

// Records a formatted detail for mqc_last_error() and returns `code`.
int fail(int code, const char* fmt, ...);
// Clears the detail (called on entry of every C-ABI function).
void clear_error();
// Translates cudaGetLastError() after a launch into MQC_OK / MQC_ERR_CUDA.
int check_launch(const char* what);
// Number of SMs of the current device (cached per device).
int num_sms();
// Stream-ordered scratch for the entry points that need it (current device).
// Memory comes from a pool private to the library, one per device, that keeps
// up to kScratchKeepBytes cached across synchronisations instead of handing it
// back to the driver after every synchronize (what the default pool does), so
// repeated calls do not re-map their scratch. While `st` is being captured into
// a CUDA graph the default pool is used (the allocation becomes a graph node).
constexpr uint64_t kScratchKeepBytes = uint64_t(8) << 30;
cudaError_t scratch_alloc(void** p, size_t bytes, cudaStream_t st);
cudaError_t scratch_free(void* p, cudaStream_t st);

// Row statistics of the quaternion LayerNorm (layer_norm.cu): mean and 1/std of
// the norms of each row, exactly as mqc_qln_fwd computes them.
int qln_row_stats(const void* q, float* mean, float* rstd, int64_t rows, int64_t d_model,
                  float eps, int dtype, cudaStream_t st);

inline bool aligned(const void* p, uintptr_t a) {
  return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0;
}

inline int dtype_size(int dtype) { return dtype == MQC_DTYPE_BF16 ? 2 : 4; }

inline bool dtype_ok(int dtype) { return dtype == MQC_DTYPE_F32 || dtype == MQC_DTYPE_BF16; }

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

}  // namespace mqc

#define MQC_REQUIRE(cond, code, ...)                     \
  do {                                                   \
    if (!(cond)) return ::mqc::fail((code), __VA_ARGS__); \
  } while (0)
