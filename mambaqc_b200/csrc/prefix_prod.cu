// Cumulative left product over time: out[b,t,l] = q[b,t,l] (x) out[b,t-1,l].
//
// Reference: parallel_scan_quaternion / parallel_scan_quaternion_reference,
// mambaqc/kernels/parallel_scan.py:171-295. The reference runs a Brent-Kung tree
// with one kernel launch per tree node; here one launch (or two for short,
// narrow problems) does it: every lane (b, l) is an independent sequential chain,
// so with enough lanes the kernel is a pure HBM stream (read q once, write out
// once) and the chain latency hides behind UNROLL independent loads per thread.
//
// When lanes are too few to fill the GPU, time is cut into chunks:
//   pass 1: P[b,c,l] = q[end_c] (x) ... (x) q[start_c]        (reads q)
//   pass 2: carry = P[c-1] (x) ... (x) P[0]; run chunk c from carry (reads q, writes out)
// Products are combined later (x) earlier, preserving the non-commutative order.
#include <mutex>

#include "mqc_common.cuh"
#include "mqc_host.h"

namespace mqc {
namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 8;

// Runs steps [t0, t1) of lane (b, l) starting from `acc`; optionally stores each
// prefix to `out`, returns the final accumulator. Loads are double-buffered: the
// next kUnroll steps are requested before the current ones are multiplied and
// stored, so every thread always has loads in flight.
template <typename T, bool STORE>
__device__ __forceinline__ float4 run_chain(const T* __restrict__ q, T* __restrict__ out,
                                            int64_t row_stride, int64_t off, int64_t t0,
                                            int64_t t1, float4 acc) {
  int64_t t = t0;
  if (t + kUnroll <= t1) {
    float4 cur[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) cur[u] = QIO<T>::ld_stream(q + off + (t + u) * row_stride);
    for (; t + kUnroll <= t1; t += kUnroll) {
      float4 nxt[kUnroll];
      const bool more = t + 2 * kUnroll <= t1;
#pragma unroll
      for (int u = 0; u < kUnroll; ++u)
        nxt[u] = more ? QIO<T>::ld_stream(q + off + (t + kUnroll + u) * row_stride) : cur[u];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        acc = qmul(cur[u], acc);
        if (STORE) QIO<T>::st_stream(out + off + (t + u) * row_stride, acc);
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) cur[u] = nxt[u];
    }
  }
  for (; t < t1; ++t) {
    acc = qmul(QIO<T>::ld_stream(q + off + t * row_stride), acc);
    if (STORE) QIO<T>::st_stream(out + off + t * row_stride, acc);
  }
  return acc;
}

// grid: (ceil(lanes / kThreads), batch)
template <typename T>
__global__ void __launch_bounds__(kThreads) prefix_seq_kernel(const T* __restrict__ q,
                                                              T* __restrict__ out,
                                                              int64_t seq_len, int64_t lanes) {
  const int64_t l = int64_t(blockIdx.x) * kThreads + threadIdx.x;
  if (l >= lanes) return;
  const int64_t b = blockIdx.y;
  const int64_t row = lanes * 4;
  const int64_t off = b * seq_len * row + l * 4;
  run_chain<T, true>(q, out, row, off, 0, seq_len, make_float4(1.f, 0.f, 0.f, 0.f));
}

// pass 1 -- grid: (ceil(lanes / kThreads), nchunks, batch); P: [batch, nchunks, lanes, 4] fp32
template <typename T>
__global__ void __launch_bounds__(kThreads) prefix_chunk_total_kernel(
    const T* __restrict__ q, float* __restrict__ P, int64_t seq_len, int64_t lanes,
    int64_t chunk) {
  const int64_t l = int64_t(blockIdx.x) * kThreads + threadIdx.x;
  if (l >= lanes) return;
  const int64_t c = blockIdx.y, b = blockIdx.z, nchunks = gridDim.y;
  const int64_t row = lanes * 4;
  const int64_t t0 = c * chunk;
  const int64_t t1 = t0 + chunk < seq_len ? t0 + chunk : seq_len;
  const float4 tot = run_chain<T, false>(q, nullptr, row, b * seq_len * row + l * 4, t0, t1,
                                         make_float4(1.f, 0.f, 0.f, 0.f));
  QIO<float>::st(P + ((b * nchunks + c) * lanes + l) * 4, tot);
}

// pass 2 -- same grid as pass 1
template <typename T>
__global__ void __launch_bounds__(kThreads) prefix_chunk_apply_kernel(
    const T* __restrict__ q, const float* __restrict__ P, T* __restrict__ out, int64_t seq_len,
    int64_t lanes, int64_t chunk) {
  const int64_t l = int64_t(blockIdx.x) * kThreads + threadIdx.x;
  if (l >= lanes) return;
  const int64_t c = blockIdx.y, b = blockIdx.z, nchunks = gridDim.y;
  const int64_t row = lanes * 4;
  float4 carry = make_float4(1.f, 0.f, 0.f, 0.f);
  for (int64_t k = 0; k < c; ++k) carry = qmul(QIO<float>::ld(P + ((b * nchunks + k) * lanes + l) * 4), carry);
  const int64_t t0 = c * chunk;
  const int64_t t1 = t0 + chunk < seq_len ? t0 + chunk : seq_len;
  run_chain<T, true>(q, out, row, b * seq_len * row + l * 4, t0, t1, carry);
}

template <typename T>
int launch(const void* qv, void* outv, int64_t batch, int64_t seq_len, int64_t lanes,
           cudaStream_t st) {
  const T* q = static_cast<const T*>(qv);
  T* out = static_cast<T*>(outv);
  const int64_t lane_blocks = (lanes + kThreads - 1) / kThreads;
  // a single streaming pass needs only a few hundred threads per SM (each keeps
  // 2 x kUnroll loads in flight); chunk time only below that
  const int64_t want_threads = int64_t(num_sms()) * 256;
  const int64_t have = batch * lanes;
  int64_t nchunks = 1;
  if (have < want_threads && seq_len >= 64) {
    nchunks = (want_threads + have - 1) / have;
    const int64_t max_chunks = seq_len / 32;  // keep >= 32 steps per chunk
    if (nchunks > max_chunks) nchunks = max_chunks;
    if (nchunks > 1024) nchunks = 1024;
  }
  MQC_REQUIRE(lane_blocks <= 0x7fffffff && batch <= 65535, MQC_ERR_UNSUPPORTED,
              "mqc_prefix_prod: grid too large (batch=%lld lanes=%lld)", (long long)batch,
              (long long)lanes);
  if (nchunks <= 1) {
    dim3 grid{unsigned(lane_blocks), unsigned(batch), 1u};
    prefix_seq_kernel<T><<<grid, kThreads, 0, st>>>(q, out, seq_len, lanes);
    return check_launch("mqc_prefix_prod");
  }
  const int64_t chunk = (seq_len + nchunks - 1) / nchunks;
  nchunks = (seq_len + chunk - 1) / chunk;
  // Chunk totals live in a stream-ordered scratch allocation (freed on the same
  // stream right after pass 2, so the memory pool recycles it).
  float* P = nullptr;
  const size_t bytes = size_t(batch) * size_t(nchunks) * size_t(lanes) * 16;
  cudaError_t e = scratch_alloc(reinterpret_cast<void**>(&P), bytes, st);
  if (e != cudaSuccess)
    return fail(MQC_ERR_CUDA, "mqc_prefix_prod: scratch allocation of %zu bytes: %s", bytes,
                cudaGetErrorString(e));
  dim3 grid{unsigned(lane_blocks), unsigned(nchunks), unsigned(batch)};
  prefix_chunk_total_kernel<T><<<grid, kThreads, 0, st>>>(q, P, seq_len, lanes, chunk);
  prefix_chunk_apply_kernel<T><<<grid, kThreads, 0, st>>>(q, P, out, seq_len, lanes, chunk);
  int rc = check_launch("mqc_prefix_prod(chunked)");
  scratch_free(P, st);
  return rc;
}

}  // namespace
}  // namespace mqc

extern "C" int mqc_prefix_prod(const void* q, void* out, int64_t batch, int64_t seq_len,
                               int64_t lanes, int dtype, void* stream) {
  using namespace mqc;
  clear_error();
  MQC_REQUIRE(dtype_ok(dtype), MQC_ERR_INVALID_VALUE, "mqc_prefix_prod: unknown dtype %d", dtype);
  MQC_REQUIRE(batch >= 0 && seq_len >= 0 && lanes >= 0, MQC_ERR_INVALID_VALUE,
              "mqc_prefix_prod: negative size");
  if (batch == 0 || seq_len == 0 || lanes == 0) return MQC_OK;
  MQC_REQUIRE(q != nullptr && out != nullptr, MQC_ERR_INVALID_VALUE,
              "mqc_prefix_prod: null pointer");
  const uintptr_t al = dtype == MQC_DTYPE_F32 ? 16 : 8;
  MQC_REQUIRE(aligned(q, al) && aligned(out, al), MQC_ERR_MISALIGNED,
              "mqc_prefix_prod: pointers must be %d-byte aligned", int(al));
  if (dtype == MQC_DTYPE_F32) return launch<float>(q, out, batch, seq_len, lanes, as_stream(stream));
  return launch<__nv_bfloat16>(q, out, batch, seq_len, lanes, as_stream(stream));
}

// ---------------------------------------------------------------------------
// Allocation-free variant (mqc_prefix_prod_noalloc)
//
// Some callers cannot allocate device memory while they run: a server that
// hands all device memory to its own allocator at start-up, or a process with a
// fixed device-memory budget in which an allocation failing mid-run is not
// acceptable. For them the chunked path takes its chunk products from this
// fixed file-scope array instead of cudaMallocAsync. Every GPU that loads the
// library holds the array (4 MiB) until the process exits.
// ---------------------------------------------------------------------------

namespace mqc {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;  // 4 MiB = 262144 chunk products
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchBytes / sizeof(float)];

// Device address of g_noalloc_scratch in the current context. In host code the
// array's name is only a host-side stand-in, so the address is looked up with
// cudaGetSymbolAddress, with the device current, the first time a context calls
// this entry point, and cached under that context's process-unique id
// (cuCtxGetId). A context created later on the same device -- after
// cudaDeviceReset, or a driver-API context -- has a new id and gets its own
// lookup, so a cached address never outlives the context it belongs to.
using CtxGetCurrentFn = int (*)(void**);
using CtxGetIdFn = int (*)(void*, unsigned long long*);

constexpr int kNoAllocCacheSlots = 64;
struct NoAllocSlot {
  unsigned long long ctx_id;
  float* ptr;
};
std::mutex g_noalloc_mutex;
NoAllocSlot g_noalloc_cache[kNoAllocCacheSlots] = {};
int g_noalloc_next = 0;
CtxGetCurrentFn g_ctx_get_current = nullptr;
CtxGetIdFn g_ctx_get_id = nullptr;

int noalloc_scratch(float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess)
    return fail(MQC_ERR_CUDA, "mqc_prefix_prod_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (g_ctx_get_current == nullptr || g_ctx_get_id == nullptr) {
    void* f1 = nullptr;
    void* f2 = nullptr;
    cudaDriverEntryPointQueryResult q1{}, q2{};
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f1, cudaEnableDefault, &q1) != cudaSuccess ||
        cudaGetDriverEntryPoint("cuCtxGetId", &f2, cudaEnableDefault, &q2) != cudaSuccess ||
        f1 == nullptr || f2 == nullptr)
      return fail(MQC_ERR_CUDA, "mqc_prefix_prod_noalloc: driver entry points "
                                "cuCtxGetCurrent/cuCtxGetId unavailable");
    g_ctx_get_current = reinterpret_cast<CtxGetCurrentFn>(f1);
    g_ctx_get_id = reinterpret_cast<CtxGetIdFn>(f2);
  }
  void* ctx = nullptr;
  unsigned long long id = 0;
  if (g_ctx_get_current(&ctx) == 0 && ctx == nullptr) {
    // the runtime has not bound a context to this thread yet: cudaSetDevice
    // initialises the device's primary context and makes it current
    e = cudaSetDevice(dev);
    if (e != cudaSuccess)
      return fail(MQC_ERR_CUDA, "mqc_prefix_prod_noalloc: cudaSetDevice: %s",
                  cudaGetErrorString(e));
  }
  if (g_ctx_get_current(&ctx) != 0 || ctx == nullptr || g_ctx_get_id(ctx, &id) != 0)
    return fail(MQC_ERR_CUDA, "mqc_prefix_prod_noalloc: cannot identify the current context");
  for (const NoAllocSlot& s : g_noalloc_cache) {
    if (s.ptr != nullptr && s.ctx_id == id) {
      *out = s.ptr;
      return MQC_OK;
    }
  }
  void* p = nullptr;
  e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess || p == nullptr)
    return fail(MQC_ERR_CUDA, "mqc_prefix_prod_noalloc: cudaGetSymbolAddress: %s",
                cudaGetErrorString(e));
  g_noalloc_cache[g_noalloc_next] = NoAllocSlot{id, static_cast<float*>(p)};
  g_noalloc_next = (g_noalloc_next + 1) % kNoAllocCacheSlots;
  *out = static_cast<float*>(p);
  return MQC_OK;
}

template <typename T>
int launch_noalloc(const void* qv, void* outv, int64_t batch, int64_t seq_len, int64_t lanes,
                   cudaStream_t st) {
  const T* q = static_cast<const T*>(qv);
  T* out = static_cast<T*>(outv);
  const int64_t lane_blocks = (lanes + kThreads - 1) / kThreads;
  MQC_REQUIRE(lane_blocks <= 0x7fffffff && batch <= 65535, MQC_ERR_UNSUPPORTED,
              "mqc_prefix_prod_noalloc: grid too large (batch=%lld lanes=%lld)", (long long)batch,
              (long long)lanes);
  // Same chunking rule as mqc_prefix_prod, with the chunk count further capped
  // so that the chunk products (batch * chunks * lanes * 16 bytes) fit in the
  // static array; when not even two chunks fit, the single pass runs, which
  // needs no scratch. Every size mqc_prefix_prod accepts is therefore served.
  const int64_t want_threads = int64_t(num_sms()) * 256;
  const int64_t have = batch * lanes;
  int64_t nchunks = 1;
  if (have < want_threads && seq_len >= 64) {
    nchunks = (want_threads + have - 1) / have;
    const int64_t max_chunks = seq_len / 32;
    if (nchunks > max_chunks) nchunks = max_chunks;
    if (nchunks > 1024) nchunks = 1024;
    const int64_t fit = int64_t(kNoAllocScratchBytes / (size_t(have) * 16));
    if (nchunks > fit) nchunks = fit;
  }
  if (nchunks > 1) {
    const int64_t chunk = (seq_len + nchunks - 1) / nchunks;
    nchunks = (seq_len + chunk - 1) / chunk;
  }
  if (nchunks <= 1) {
    dim3 grid{unsigned(lane_blocks), unsigned(batch), 1u};
    prefix_seq_kernel<T><<<grid, kThreads, 0, st>>>(q, out, seq_len, lanes);
    return check_launch("mqc_prefix_prod_noalloc");
  }
  const int64_t chunk = (seq_len + nchunks - 1) / nchunks;
  const size_t need = size_t(batch) * size_t(nchunks) * size_t(lanes) * 16;
  // unreachable by construction of nchunks; kept as the array's hard guard
  MQC_REQUIRE(need <= kNoAllocScratchBytes, MQC_ERR_UNSUPPORTED,
              "mqc_prefix_prod_noalloc: %zu bytes of chunk scratch exceed the static maximum "
              "of %zu bytes", need, kNoAllocScratchBytes);
  float* P = nullptr;
  int rc = noalloc_scratch(&P);
  if (rc != MQC_OK) return rc;
  // Pass 1 writes every chunk product that pass 2 reads, so nothing left in the
  // array by an earlier call is ever read and nothing needs clearing.
  dim3 grid{unsigned(lane_blocks), unsigned(nchunks), unsigned(batch)};
  prefix_chunk_total_kernel<T><<<grid, kThreads, 0, st>>>(q, P, seq_len, lanes, chunk);
  prefix_chunk_apply_kernel<T><<<grid, kThreads, 0, st>>>(q, P, out, seq_len, lanes, chunk);
  return check_launch("mqc_prefix_prod_noalloc(chunked)");
}

}  // namespace
}  // namespace mqc

extern "C" int mqc_prefix_prod_noalloc(const void* q, void* out, int64_t batch, int64_t seq_len,
                                       int64_t lanes, int dtype, void* stream) {
  using namespace mqc;
  clear_error();
  MQC_REQUIRE(dtype_ok(dtype), MQC_ERR_INVALID_VALUE, "mqc_prefix_prod_noalloc: unknown dtype %d",
              dtype);
  MQC_REQUIRE(batch >= 0 && seq_len >= 0 && lanes >= 0, MQC_ERR_INVALID_VALUE,
              "mqc_prefix_prod_noalloc: negative size");
  if (batch == 0 || seq_len == 0 || lanes == 0) return MQC_OK;
  MQC_REQUIRE(q != nullptr && out != nullptr, MQC_ERR_INVALID_VALUE,
              "mqc_prefix_prod_noalloc: null pointer");
  const uintptr_t al = dtype == MQC_DTYPE_F32 ? 16 : 8;
  MQC_REQUIRE(aligned(q, al) && aligned(out, al), MQC_ERR_MISALIGNED,
              "mqc_prefix_prod_noalloc: pointers must be %d-byte aligned", int(al));
  if (dtype == MQC_DTYPE_F32)
    return launch_noalloc<float>(q, out, batch, seq_len, lanes, as_stream(stream));
  return launch_noalloc<__nv_bfloat16>(q, out, batch, seq_len, lanes, as_stream(stream));
}
