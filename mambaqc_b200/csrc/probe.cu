// FP32 FMA throughput probe: the denominator of the FP32-issue roofline of the
// scan kernels (no counterpart in the reference). Every thread runs 8 independent
// FMA chains for `iters` iterations; one launch does
// grid * block * 8 * iters FMAs = 2x that many FLOPs.
#include "mqc_common.cuh"
#include "mqc_host.h"

namespace mqc {
namespace {

__global__ void __launch_bounds__(256) fma_probe_kernel(float* out, int64_t iters, float s) {
  float a0 = threadIdx.x * 1e-7f, a1 = a0 + 1e-7f, a2 = a0 + 2e-7f, a3 = a0 + 3e-7f;
  float a4 = a0 + 4e-7f, a5 = a0 + 5e-7f, a6 = a0 + 6e-7f, a7 = a0 + 7e-7f;
  const float m = 0.9999999f;
  for (int64_t i = 0; i < iters; ++i) {
#pragma unroll
    for (int u = 0; u < 16; ++u) {
      a0 = fmaf(a0, m, s); a1 = fmaf(a1, m, s); a2 = fmaf(a2, m, s); a3 = fmaf(a3, m, s);
      a4 = fmaf(a4, m, s); a5 = fmaf(a5, m, s); a6 = fmaf(a6, m, s); a7 = fmaf(a7, m, s);
    }
  }
  const float r = ((a0 + a1) + (a2 + a3)) + ((a4 + a5) + (a6 + a7));
  if (r == 12345.f) out[0] = r;  // keeps the chains alive; never true in practice
}

}  // namespace
}  // namespace mqc

extern "C" int mqc_probe_fp32_fma(float* out, int64_t iters, int64_t* fmas_per_launch,
                                  void* stream) {
  using namespace mqc;
  clear_error();
  MQC_REQUIRE(out != nullptr && iters > 0, MQC_ERR_INVALID_VALUE, "mqc_probe_fp32_fma: bad args");
  const int grid = num_sms() * 8;
  fma_probe_kernel<<<grid, 256, 0, as_stream(stream)>>>(out, iters, 1e-9f);
  if (fmas_per_launch) *fmas_per_launch = int64_t(grid) * 256 * 8 * 16 * iters;
  return check_launch("mqc_probe_fp32_fma");
}
