// Quaternion LayerNorm fused into the operand load of the output projection:
//   out[m, :] = LN(y)[m, :] @ W^T (+ bias),  y [M, Dq, 4], W [N, 4 Dq], bf16.
//
// The reference block runs `self.out_proj(self.norm(y_quat))`
// (mambaqc/models/quaternion_mamba2_block.py:154-157): the LayerNorm writes
// the normalised activations (M x 4Dq, the widest tensor after the scan) and
// the projection reads them back. Here the LayerNorm is the prologue of a
// hand-written sm_100a GEMM and its output never reaches global memory:
//   1. qln_row_stats (layer_norm.cu) reads y once and writes the mean and
//      1/std of the quaternion norms of every row (8 bytes per row);
//   2. the GEMM streams raw y tiles into shared memory with TMA, normalises
//      them in place (per quaternion: n = sqrt(|q|^2 + eps),
//      out = gamma * (n - mean) * rstd * q / (n + eps) + beta, with gamma and
//      beta staged in shared memory once per CTA and the reciprocal Newton-
//      refined), and feeds them to tcgen05.mma with the fp32 accumulator in
//      tensor memory.
//
// One CTA computes a BM x BN = 128 x 384 tile of out, walking K in BK = 64
// blocks through a shared-memory ring of up to four stages. Warp roles:
//   warp 0      TMA producer (one thread): raw y tile + W tile per stage;
//   warp 1      tensor-memory allocation and the MMA issuer (one thread);
//   warps 2..17 transform each landed y tile in place (a row per four
//               threads), fence it for the tensor core, signal the MMA issuer;
//               after the last K block, the epilogue (tcgen05.ld -> bf16 ->
//               global).
// Every mbarrier wait is bounded: on timeout the CTA raises its abort flag and
// the status word, stops issuing work, lets what was issued finish (bounded),
// frees its tensor memory and returns. Plain TMA loads only (no multicast);
// every tensor map covers this GPU's memory.
#include <cuda.h>

#include <mutex>

#include "tc_common.cuh"

namespace mqc {
namespace {

// A CTA covers BN = 384 output columns as two MMAs (N = 256 and N = 128), so a
// y tile is normalised once per 384 columns and the config-4 output projection
// (768 columns) runs as 2 x 64 CTAs, one wave.
constexpr int BM = 128, BN1 = 256, BN2 = 128, BN = BN1 + BN2, BK = 64;
constexpr int kMaxStages = 4;
constexpr int kXformWarps = 16;
constexpr int kThreads = 32 * (2 + kXformWarps);
constexpr uint32_t kABytes = BM * BK * 2;  // 16 KB
constexpr uint32_t kB1Bytes = BN1 * BK * 2;  // 32 KB
constexpr uint32_t kBBytes = BN * BK * 2;    // 48 KB
constexpr uint32_t kStageBytes = kABytes + kBBytes;
constexpr uint32_t kTmemCols = 512;        // fp32 accumulators: 256 + 128 columns
constexpr long long kPollLimit = 1ll << 26;
constexpr size_t kSmemMax = 232448;        // dynamic shared memory of one CTA (227 KB)

struct SmemCtl {
  uint64_t full[kMaxStages], ready[kMaxStages], empty[kMaxStages], accum;
  uint32_t tmem_base;
  int abort;
  float mean[BM], rstd[BM];
};

// Shared memory: the stage ring, the control block, then gamma [Dq] and beta
// [Dq][4] (staged once per CTA). As many stages as fit, at most 4.
inline size_t gb_bytes(int Dq) { return size_t((Dq + 3) & ~3) * 4 + size_t(Dq) * 16; }
inline int ring_stages(int Dq) {
  const size_t fixed = 1024 + sizeof(SmemCtl) + gb_bytes(Dq);
  const size_t n = (kSmemMax - fixed) / kStageBytes;
  return n >= size_t(kMaxStages) ? kMaxStages : int(n);
}
inline size_t smem_bytes(int Dq) {
  return 1024 + size_t(ring_stages(Dq)) * kStageBytes + sizeof(SmemCtl) + gb_bytes(Dq);
}

__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity,
                                              volatile int* abort_flag, int* status) {
  return tc::wait_or_abort(bar, parity, abort_flag, status, kPollLimit);
}

using tc::fence_async_smem;
using tc::mbar_arrive_plain;
using tc::mma_commit;
using tc::pack_bf16x2;
using tc::tc_fence_after;
using tc::tc_fence_before;
using tc::tma_load_2d;
using tc::tmem_ld32;

__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) { return tc::kmajor_desc<128>(saddr); }

constexpr uint32_t kIdesc1 = tc::idesc_bf16(BM, BN1);
constexpr uint32_t kIdesc2 = tc::idesc_bf16(BM, BN2);

// The LayerNorm of one bf16 quaternion: qln_fwd_kernel's formula, with the
// square root and the reciprocal 1 / (n + eps) taken as hardware
// approximations (the reciprocal Newton-refined) instead of correctly rounded
// operations: an ulp or two of fp32, far below the bf16 rounding of the result.
__device__ __forceinline__ float4 qln_point(float4 v, float mu, float rsd, float gm, float4 bt,
                                            float eps) {
  float nrm;
  asm("sqrt.approx.ftz.f32 %0, %1;"
      : "=f"(nrm)
      : "f"(fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, v.w * v.w))) + eps));
  const float nh = (nrm - mu) * rsd;
  const float g = gm * nh * rcp_nr(nrm + eps);
  return make_float4(fmaf(g, v.x, bt.x), fmaf(g, v.y, bt.y), fmaf(g, v.z, bt.z),
                     fmaf(g, v.w, bt.w));
}

struct QlnLinParams {
  const float* mean;
  const float* rstd;
  const float* gamma;
  const float* beta;
  const __nv_bfloat16* bias;
  __nv_bfloat16* out;
  int M, N, K;  // K = 4 * Dq
  float eps;
  int* status;
  int stages;   // ring depth (<= kMaxStages)
};

__global__ void __launch_bounds__(kThreads, 1)
    qln_linear_kernel(const __grid_constant__ CUtensorMap tmY,
                      const __grid_constant__ CUtensorMap tmW1,
                      const __grid_constant__ CUtensorMap tmW2, const QlnLinParams p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // 1024-byte aligned stage ring (the 128-byte swizzle atoms), control block after it
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int kStages = p.stages;
  SmemCtl* ctl = reinterpret_cast<SmemCtl*>(base + size_t(kStages) * kStageBytes);
  float* sgamma = reinterpret_cast<float*>(ctl + 1);
  float4* sbeta = reinterpret_cast<float4*>(sgamma + ((p.K / 4 + 3) & ~3));
  volatile int* abort_flag = &ctl->abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  const int nkb = p.K / BK;
  for (int d = threadIdx.x; d < p.K / 4; d += blockDim.x) {
    sgamma[d] = __ldg(p.gamma + d);
    sbeta[d] = QIO<float>::ld(p.beta + d * 4);
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&ctl->full[s], 1);
      mbar_init(&ctl->ready[s], 32 * kXformWarps);
      mbar_init(&ctl->empty[s], 1);
    }
    mbar_init(&ctl->accum, 1);
    ctl->abort = 0;
    fence_mbar_init();
  }
  if (threadIdx.x < BM) {
    const int m = m0 + threadIdx.x;
    ctl->mean[threadIdx.x] = m < p.M ? p.mean[m] : 0.f;
    ctl->rstd[threadIdx.x] = m < p.M ? p.rstd[m] : 0.f;
  }
  if (warp == 1) {  // tensor memory for the accumulator (whole warp)
    tc::tmem_alloc(&ctl->tmem_base, kTmemCols);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int issued = 0;
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % kStages;
        if (kb >= kStages &&
            !wait_or_abort(&ctl->empty[s], uint32_t(((kb / kStages) - 1) & 1), abort_flag,
                           p.status))
          break;
        if (*abort_flag) break;
        unsigned char* st = base + size_t(s) * kStageBytes;
        mbar_arrive_expect_tx(&ctl->full[s], kStageBytes);
        tma_load_2d(st, &tmY, kb * BK, m0, &ctl->full[s]);
        tma_load_2d(st + kABytes, &tmW1, kb * BK, n0, &ctl->full[s]);
        tma_load_2d(st + kABytes + kB1Bytes, &tmW2, kb * BK, n0 + BN1, &ctl->full[s]);
        issued = kb + 1;
      }
      // the CTA must outlive its copies: wait (bounded) for the last ones issued
      for (int kb = issued > kStages ? issued - kStages : 0; kb < issued; ++kb)
        mbar_wait_bounded(&ctl->full[kb % kStages], uint32_t((kb / kStages) & 1), kDrainPollLimit);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int issued = 0;
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % kStages;
        if (!wait_or_abort(&ctl->ready[s], uint32_t((kb / kStages) & 1), abort_flag, p.status))
          break;
        tc_fence_after();
        const uint32_t sa = smem_addr(base + size_t(s) * kStageBytes);
        const uint32_t sb = sa + kABytes;
#pragma unroll
        for (int k = 0; k < BK / 16; ++k) {  // 16 bf16 = 32 bytes per MMA along K
          const uint32_t acc = (kb > 0 || k > 0) ? 1u : 0u;
          const uint64_t ad = sw128_desc(sa + 32 * k);
          tc::mma_bf16<kIdesc1>(tmem, ad, sw128_desc(sb + 32 * k), acc);
          tc::mma_bf16<kIdesc2>(tmem + uint32_t(BN1), ad, sw128_desc(sb + kB1Bytes + 32 * k), acc);
        }
        mma_commit(&ctl->empty[s]);  // frees the stage once these MMAs have read it
        issued = kb + 1;
      }
      if (issued == nkb) {
        mma_commit(&ctl->accum);
      } else if (issued > 0) {
        // aborted: wait (bounded) until the MMAs already issued are done
        const int kb = issued - 1;
        mbar_wait_bounded(&ctl->empty[kb % kStages], uint32_t((kb / kStages) & 1),
                          kDrainPollLimit);
      }
    }
  } else {
    // ------------------------------------------------------------ transform
    const int xt = threadIdx.x - 64;  // 0 .. 511
    const int r = xt >> 2;            // tile row
    const int c_lo = (xt & 3) * 2;    // first of this thread's 2 16-byte chunks
    const float mu = ctl->mean[r], rsd = ctl->rstd[r];
    bool ok = true;
    for (int kb = 0; kb < nkb && ok; ++kb) {
      const int s = kb % kStages;
      ok = wait_or_abort(&ctl->full[s], uint32_t((kb / kStages) & 1), abort_flag, p.status);
      if (!ok) break;
      unsigned char* rowp = base + size_t(s) * kStageBytes + r * 128;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int c = c_lo + j;                           // logical 16-byte chunk of the row
        uint4* cp = reinterpret_cast<uint4*>(rowp + ((c ^ (r & 7)) << 4));
        const uint4 raw = *cp;
        const int d0 = kb * (BK / 4) + 2 * c;             // quaternion index of the chunk
        const float4 q0 = QIO<__nv_bfloat16>::unpack(make_uint2(raw.x, raw.y));
        const float4 q1 = QIO<__nv_bfloat16>::unpack(make_uint2(raw.z, raw.w));
        const float4 o0 = qln_point(q0, mu, rsd, sgamma[d0], sbeta[d0], p.eps);
        const float4 o1 = qln_point(q1, mu, rsd, sgamma[d0 + 1], sbeta[d0 + 1], p.eps);
        *cp = make_uint4(pack_bf16x2(o0.x, o0.y), pack_bf16x2(o0.z, o0.w),
                         pack_bf16x2(o1.x, o1.y), pack_bf16x2(o1.z, o1.w));
      }
      fence_async_smem();  // generic-proxy writes -> visible to the tensor core
      mbar_arrive_plain(&ctl->ready[s]);
    }
    // ------------------------------------------------------------ epilogue
    // (tcgen05.ld is warp-collective: the whole warp takes the same branch)
    bool go = ok && wait_or_abort(&ctl->accum, 0u, abort_flag, p.status);
    go = __all_sync(0xffffffffu, go);
    if (go) {
      tc_fence_after();
      const int ew = warp - 2;        // 0 .. 15
      const int quarter = warp & 3;   // tensor-memory lanes 32*quarter .. +31
      const int part = ew >> 2;       // columns 96*part .. +95
      const int row = quarter * 32 + lane;
      const int m = m0 + row;
#pragma unroll 1
      for (int cb = 0; cb < 3; ++cb) {
        const int col0 = part * 96 + cb * 32;
        float v[32];
        tmem_ld32(tmem + (uint32_t(quarter * 32) << 16) + uint32_t(col0), v);
        const int n = n0 + col0;
        if (m < p.M) {
          if (p.bias != nullptr) {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (n + i < p.N) v[i] += __bfloat162float(p.bias[n + i]);
          }
          __nv_bfloat16* dst = p.out + int64_t(m) * p.N + n;
          if (n + 32 <= p.N && (p.N & 7) == 0) {
#pragma unroll
            for (int i = 0; i < 32; i += 8)
              *reinterpret_cast<uint4*>(dst + i) =
                  make_uint4(pack_bf16x2(v[i], v[i + 1]), pack_bf16x2(v[i + 2], v[i + 3]),
                             pack_bf16x2(v[i + 4], v[i + 5]), pack_bf16x2(v[i + 6], v[i + 7]));
          } else {
            for (int i = 0; i < 32 && n + i < p.N; ++i) dst[i] = __float2bfloat16_rn(v[i]);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tc::tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// against the driver library).
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
static std::mutex g_encode_mutex;
static EncodeTiledFn g_encode = nullptr;

int make_map_bf16_2d(CUtensorMap* map, const void* ptr, uint64_t rows, uint64_t cols,
                     uint32_t box_rows, uint32_t box_cols, int row_bytes, const char* who) {
  {
    std::lock_guard<std::mutex> lock(g_encode_mutex);
    if (g_encode == nullptr) {
      void* f = nullptr;
      cudaDriverEntryPointQueryResult q{};
      if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) !=
              cudaSuccess ||
          f == nullptr)
        return fail(MQC_ERR_CUDA, "%s: cuTensorMapEncodeTiled unavailable", who);
      g_encode = reinterpret_cast<EncodeTiledFn>(f);
    }
  }
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * 2};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = g_encode(
      map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
      CU_TENSOR_MAP_INTERLEAVE_NONE,
      row_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(MQC_ERR_CUDA, "%s: cuTensorMapEncodeTiled failed (%d)", who, int(r));
  return MQC_OK;
}

}  // namespace mqc

using namespace mqc;

extern "C" int mqc_qln_linear_fwd(const void* q, const float* gamma, const float* beta,
                                  const void* weight, const void* bias, void* out, float* mean,
                                  float* rstd, int64_t rows, int64_t d_model,
                                  int64_t out_features, float eps, int* status, void* stream) {
  clear_error();
  const char* name = "mqc_qln_linear_fwd";
  MQC_REQUIRE(rows >= 0 && d_model >= 0 && out_features >= 0, MQC_ERR_INVALID_VALUE,
              "%s: negative size", name);
  if (rows == 0 || out_features == 0) return MQC_OK;
  MQC_REQUIRE(q && gamma && beta && weight && out && mean && rstd, MQC_ERR_INVALID_VALUE,
              "%s: null pointer", name);
  MQC_REQUIRE(d_model >= 16 && d_model % 16 == 0 && d_model <= 4096, MQC_ERR_UNSUPPORTED,
              "%s: d_model must be a multiple of 16 in [16, 4096] (K = 4 d_model in blocks of %d)",
              name, BK);
  MQC_REQUIRE(rows <= 0x7fffffff && out_features <= 0x7fffffff, MQC_ERR_UNSUPPORTED,
              "%s: size out of range", name);
  MQC_REQUIRE(aligned(q, 16) && aligned(weight, 16) && aligned(beta, 16) && aligned(out, 2),
              MQC_ERR_MISALIGNED, "%s: q, weight and beta must be 16-byte aligned", name);
  cudaStream_t st = as_stream(stream);
  int rc = qln_row_stats(q, mean, rstd, rows, d_model, eps, MQC_DTYPE_BF16, st);
  if (rc != MQC_OK) return rc;
  const int64_t K = 4 * d_model;
  CUtensorMap tmY, tmW1, tmW2;
  rc = make_map_bf16_2d(&tmY, q, uint64_t(rows), uint64_t(K), BM, BK, 128, name);
  if (rc == MQC_OK)
    rc = make_map_bf16_2d(&tmW1, weight, uint64_t(out_features), uint64_t(K), BN1, BK, 128, name);
  if (rc == MQC_OK)
    rc = make_map_bf16_2d(&tmW2, weight, uint64_t(out_features), uint64_t(K), BN2, BK, 128, name);
  if (rc != MQC_OK) return rc;
  const size_t smem = smem_bytes(int(d_model));
  cudaError_t e = cudaFuncSetAttribute(qln_linear_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess)
    return fail(MQC_ERR_CUDA, "%s: smem attribute: %s", name, cudaGetErrorString(e));
  QlnLinParams p{mean, rstd, gamma, beta, static_cast<const __nv_bfloat16*>(bias),
                 static_cast<__nv_bfloat16*>(out), int(rows), int(out_features), int(K), eps,
                 status, ring_stages(int(d_model))};
  dim3 grid{unsigned((out_features + BN - 1) / BN), unsigned((rows + BM - 1) / BM), 1u};
  MQC_REQUIRE(grid.y <= 65535, MQC_ERR_UNSUPPORTED, "%s: too many rows", name);
  qln_linear_kernel<<<grid, kThreads, smem, st>>>(tmY, tmW1, tmW2, p);
  return check_launch(name);
}
