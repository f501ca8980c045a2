// Peer-memory exchange between the ranks of one node (one process per GPU,
// NVLink / NVSwitch), for the channel-sharded long-sequence scan.
//
// No counterpart in the reference (it has no multi-GPU code). The channel-
// sharded scan gives rank r channels [r*Dl, (r+1)*Dl) of every step, and every
// rank wants the whole output y [B, T, G*Dl, 4]. A collective library gathers
// contiguous per-rank blocks, which leaves a [G][B][T][Dl] layout to permute
// afterwards (a full extra pass over y). Here every rank instead owns one
// output buffer that the other ranks can address (CUDA IPC), and a push kernel
// writes the rank's freshly scanned time segment straight into its channel
// columns of every rank's buffer over NVLink -- the final layout, no permute --
// while the next segment is being scanned.
//
// Buffers come from cudaMalloc (IPC needs a whole allocation) and are shared
// with cudaIpcGetMemHandle / cudaIpcOpenMemHandle; no multicast object and no
// TMA is involved, only plain stores from SMs to peer memory.
#include <cstring>

#include "mqc_common.cuh"
#include "mqc_host.h"

namespace mqc {
namespace {

constexpr int kMaxPeers = 8;
constexpr int kPushThreads = 256;

struct PushDst {
  void* p[kMaxPeers];
};

// Copies `chunks` 16-byte (V = uint4) or 8-byte (V = uint2) pieces per row of the
// source segment [batch, seg_len, row_chunks] into row (b, t_off + t) at column
// chunk ch_off of every destination [batch, seq_total, dst_row_chunks].
template <typename V>
__global__ void __launch_bounds__(kPushThreads) channel_push_kernel(
    const V* __restrict__ src, PushDst dst, int ndst, int64_t batch, int64_t seg_len,
    int64_t row_chunks, int64_t dst_row_chunks, int64_t ch_off, int64_t t_off,
    int64_t seq_total) {
  const int64_t n = batch * seg_len * row_chunks;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
    const int64_t row = i / row_chunks, k = i - row * row_chunks;
    const int64_t b = row / seg_len, t = row - b * seg_len;
    const int64_t o = (b * seq_total + t_off + t) * dst_row_chunks + ch_off + k;
    const V v = __ldcs(src + i);
#pragma unroll
    for (int r = 0; r < kMaxPeers; ++r)
      if (r < ndst) __stcs(static_cast<V*>(dst.p[r]) + o, v);
  }
  // make this thread's stores to peer memory visible system-wide before the
  // kernel is seen as complete by the ranks that synchronise with it
  __threadfence_system();
}

}  // namespace
}  // namespace mqc

using namespace mqc;

extern "C" int mqc_peer_alloc(size_t bytes, void** ptr, void* handle) {
  clear_error();
  MQC_REQUIRE(ptr != nullptr && handle != nullptr, MQC_ERR_INVALID_VALUE,
              "mqc_peer_alloc: null pointer");
  MQC_REQUIRE(bytes > 0, MQC_ERR_INVALID_VALUE, "mqc_peer_alloc: zero bytes");
  *ptr = nullptr;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess)
    return fail(MQC_ERR_CUDA, "mqc_peer_alloc: cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
  cudaIpcMemHandle_t h;
  e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return fail(MQC_ERR_CUDA, "mqc_peer_alloc: cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == MQC_PEER_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle, &h, sizeof(h));
  *ptr = p;
  return MQC_OK;
}

extern "C" int mqc_peer_free(void* ptr) {
  clear_error();
  if (ptr == nullptr) return MQC_OK;
  cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess)
    return fail(MQC_ERR_CUDA, "mqc_peer_free: %s", cudaGetErrorString(e));
  return MQC_OK;
}

extern "C" int mqc_peer_open(const void* handle, void** ptr) {
  clear_error();
  MQC_REQUIRE(ptr != nullptr && handle != nullptr, MQC_ERR_INVALID_VALUE,
              "mqc_peer_open: null pointer");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  *ptr = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess)
    return fail(MQC_ERR_CUDA, "mqc_peer_open: cudaIpcOpenMemHandle: %s", cudaGetErrorString(e));
  return MQC_OK;
}

extern "C" int mqc_peer_close(void* ptr) {
  clear_error();
  if (ptr == nullptr) return MQC_OK;
  cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess)
    return fail(MQC_ERR_CUDA, "mqc_peer_close: %s", cudaGetErrorString(e));
  return MQC_OK;
}

extern "C" int mqc_channel_push(const void* src, void* const* dsts, int ndst, int64_t batch,
                                int64_t seg_len, int64_t ch_local, int64_t ch_total,
                                int64_t ch_off, int64_t t_off, int64_t seq_total, int dtype,
                                void* stream) {
  clear_error();
  const char* name = "mqc_channel_push";
  MQC_REQUIRE(dtype_ok(dtype), MQC_ERR_INVALID_VALUE, "%s: unknown dtype %d", name, dtype);
  MQC_REQUIRE(ndst >= 1 && ndst <= kMaxPeers, MQC_ERR_INVALID_VALUE,
              "%s: 1 to %d destinations, got %d", name, kMaxPeers, ndst);
  MQC_REQUIRE(batch >= 0 && seg_len >= 0 && ch_local >= 0 && ch_off >= 0 && t_off >= 0,
              MQC_ERR_INVALID_VALUE, "%s: negative size", name);
  MQC_REQUIRE(ch_off + ch_local <= ch_total && t_off + seg_len <= seq_total,
              MQC_ERR_INVALID_VALUE, "%s: segment [%lld, +%lld) x channels [%lld, +%lld) outside "
              "[%lld steps x %lld channels]", name, (long long)t_off, (long long)seg_len,
              (long long)ch_off, (long long)ch_local, (long long)seq_total, (long long)ch_total);
  if (batch == 0 || seg_len == 0 || ch_local == 0) return MQC_OK;
  MQC_REQUIRE(src != nullptr && dsts != nullptr, MQC_ERR_INVALID_VALUE, "%s: null pointer", name);
  PushDst d{};
  for (int r = 0; r < ndst; ++r) {
    MQC_REQUIRE(dsts[r] != nullptr, MQC_ERR_INVALID_VALUE, "%s: null destination %d", name, r);
    d.p[r] = dsts[r];
  }
  const int64_t qbytes = dtype == MQC_DTYPE_F32 ? 16 : 8;  // one quaternion
  bool wide = true;  // 16-byte pieces
  wide = wide && aligned(src, 16) && (ch_local * qbytes) % 16 == 0 && (ch_total * qbytes) % 16 == 0 &&
         (ch_off * qbytes) % 16 == 0;
  for (int r = 0; r < ndst; ++r) wide = wide && aligned(dsts[r], 16);
  MQC_REQUIRE(aligned(src, 8), MQC_ERR_MISALIGNED, "%s: source must be 8-byte aligned", name);
  for (int r = 0; r < ndst; ++r)
    MQC_REQUIRE(aligned(dsts[r], 8), MQC_ERR_MISALIGNED, "%s: destinations must be 8-byte aligned",
                name);
  const int64_t piece = wide ? 16 : 8;
  const int64_t row_chunks = ch_local * qbytes / piece;
  const int64_t dst_row_chunks = ch_total * qbytes / piece;
  const int64_t off_chunks = ch_off * qbytes / piece;
  const int64_t n = batch * seg_len * row_chunks;
  int64_t blocks = (n + kPushThreads - 1) / kPushThreads;
  const int64_t cap = int64_t(num_sms()) * 8;
  if (blocks > cap) blocks = cap;
  cudaStream_t st = as_stream(stream);
  if (wide)
    channel_push_kernel<uint4><<<unsigned(blocks), kPushThreads, 0, st>>>(
        static_cast<const uint4*>(src), d, ndst, batch, seg_len, row_chunks, dst_row_chunks,
        off_chunks, t_off, seq_total);
  else
    channel_push_kernel<uint2><<<unsigned(blocks), kPushThreads, 0, st>>>(
        static_cast<const uint2*>(src), d, ndst, batch, seg_len, row_chunks, dst_row_chunks,
        off_chunks, t_off, seq_total);
  return check_launch(name);
}
