// Fused Cayley + scan forward on HOST buffers: the host-facing form of
// mqc_ssm_scan_fwd for callers whose tensors live in (pinned) host memory. It is
// the fused QuaternionMamba2Block._ssm_forward
// (mambaqc/models/quaternion_mamba2_block.py:214-228) with the host <-> device
// transfers made part of the call.
//
// The sequence is cut into time segments, each holding every batch row. Three
// streams form a pipeline:
//   * the copy-in stream moves segment k's delta, s, B, C into one of two device
//     slots, one strided 2-D copy per tensor (rows = batch);
//   * the caller's stream scans segment k with the regular entry point, all
//     batch rows at once (so the scan fills the GPU), starting from segment
//     k-1's final state;
//   * the copy-out stream moves segment k's y back into the host y.
// PCIe transfers in both directions therefore overlap each other and the
// kernels. Device memory comes from the library's stream-ordered scratch pool;
// nothing is allocated by the caller.
#include <cstring>
#include <mutex>

#include "ssm_scan_common.cuh"

namespace mqc {
namespace {

constexpr int kMaxDevices = 64;
struct HostPipe {
  cudaStream_t in = nullptr, out = nullptr;
  cudaEvent_t ev[8] = {};  // [0,1] in done, [2,3] scan done, [4,5] out done, [6] start, [7] end
};
std::mutex g_pipe_mu;
HostPipe g_pipe[kMaxDevices];

int host_pipe(HostPipe** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return fail(MQC_ERR_CUDA, "mqc_ssm_scan_fwd_host: no current device");
  std::lock_guard<std::mutex> lock(g_pipe_mu);
  HostPipe& p = g_pipe[dev];
  if (p.in == nullptr) {
    if (cudaStreamCreateWithFlags(&p.in, cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreateWithFlags(&p.out, cudaStreamNonBlocking) != cudaSuccess)
      return fail(MQC_ERR_CUDA, "mqc_ssm_scan_fwd_host: stream creation failed");
    for (auto& e : p.ev)
      if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess)
        return fail(MQC_ERR_CUDA, "mqc_ssm_scan_fwd_host: event creation failed");
  }
  *out = &p;
  return MQC_OK;
}

int ck(cudaError_t e, const char* what) {
  return e == cudaSuccess ? MQC_OK
                          : fail(MQC_ERR_CUDA, "mqc_ssm_scan_fwd_host: %s: %s", what,
                                 cudaGetErrorString(e));
}

}  // namespace
}  // namespace mqc

using namespace mqc;
using mqc::scan::align_up;

extern "C" int mqc_ssm_scan_fwd_host(const mqc_ssm_scan_args* a, int64_t segments,
                                     void* stream) {
  clear_error();
  const char* name = "mqc_ssm_scan_fwd_host";
  MQC_REQUIRE(a != nullptr, MQC_ERR_INVALID_VALUE, "%s: null args", name);
  MQC_REQUIRE(dtype_ok(a->dtype), MQC_ERR_INVALID_VALUE, "%s: unknown dtype %d", name, a->dtype);
  MQC_REQUIRE(!(a->flags & MQC_SSM_Q_GIVEN) && a->ckpt == nullptr, MQC_ERR_UNSUPPORTED,
              "%s: fused form only (no explicit q, no checkpoints)", name);
  MQC_REQUIRE(a->batch >= 0 && a->seq_len >= 0 && a->channels >= 0 && a->d_state >= 1,
              MQC_ERR_INVALID_VALUE, "%s: bad sizes", name);
  if (a->batch == 0 || a->seq_len == 0 || a->channels == 0) return MQC_OK;
  MQC_REQUIRE(segments >= 1 && a->seq_len % segments == 0, MQC_ERR_INVALID_VALUE,
              "%s: seq_len %lld does not split into %lld segments", name,
              (long long)a->seq_len, (long long)segments);
  MQC_REQUIRE(segments <= 4096, MQC_ERR_UNSUPPORTED, "%s: at most 4096 segments", name);
  MQC_REQUIRE(a->dskip_sb == 0 && a->dskip_st == 0, MQC_ERR_UNSUPPORTED,
              "%s: the skip weight must be per channel ([D])", name);
  MQC_REQUIRE(a->delta && a->lambda_ && a->Bm && a->Cm && a->s && a->dskip && a->y,
              MQC_ERR_INVALID_VALUE, "%s: null pointer", name);

  const int64_t Bn = a->batch, T = a->seq_len, D = a->channels, N = a->d_state;
  // pieces: [seg/2, seg x (segments-1), seg/2] when seg = T/segments is even
  // (halving the pipeline's fill and drain: the first copy-in and the last
  // scan + copy-out), else `segments` pieces of seg steps
  const int64_t seg = T / segments;
  const bool halves = segments >= 2 && seg % 2 == 0;
  const int64_t pieces = halves ? segments + 1 : segments;
  auto piece_start = [&](int64_t k) -> int64_t {
    if (!halves) return k * seg;
    return k == 0 ? 0 : seg / 2 + (k - 1) * seg;
  };
  auto piece_len = [&](int64_t k) -> int64_t {
    if (!halves) return seg;
    return (k == 0 || k == pieces - 1) ? seg / 2 : seg;
  };
  const size_t es = size_t(dtype_size(a->dtype));
  const bool shared = a->flags & MQC_SSM_BC_SHARED;
  const int64_t sw = (a->flags & MQC_SSM_S_REAL) ? 1 : 4;
  // bytes per (batch row, time step) of each streamed tensor
  const size_t row_d = size_t(D) * es, row_s = size_t(D * sw) * es,
               row_bc = size_t(shared ? N * 4 : D * N * 4) * es, row_y = size_t(D) * 4 * es;
  const size_t slot_bytes = align_up(size_t(Bn * seg) * row_d, 256) +
                            align_up(size_t(Bn * seg) * row_s, 256) +
                            2 * align_up(size_t(Bn * seg) * row_bc, 256) +
                            align_up(size_t(Bn * seg) * row_y, 256);
  const size_t lam_bytes = align_up(size_t(D * N) * 16, 256);
  const size_t dsk_bytes = align_up(size_t(D) * 4, 256);
  const size_t h_bytes = align_up(size_t(Bn * D * N) * 16, 256);
  const size_t total = 2 * slot_bytes + lam_bytes + dsk_bytes + 2 * h_bytes;

  HostPipe* hp = nullptr;
  int rc = host_pipe(&hp);
  if (rc != MQC_OK) return rc;
  cudaStream_t st = as_stream(stream);
  unsigned char* ws = nullptr;
  rc = ck(scratch_alloc(reinterpret_cast<void**>(&ws), total, st), "scratch allocation");
  if (rc != MQC_OK) return rc;
  unsigned char* slot[2] = {ws, ws + slot_bytes};
  float* lam_d = reinterpret_cast<float*>(ws + 2 * slot_bytes);
  float* dsk_d = reinterpret_cast<float*>(ws + 2 * slot_bytes + lam_bytes);
  float* hbuf[2] = {reinterpret_cast<float*>(ws + 2 * slot_bytes + lam_bytes + dsk_bytes),
                    reinterpret_cast<float*>(ws + 2 * slot_bytes + lam_bytes + dsk_bytes +
                                             h_bytes)};
  auto part = [&](unsigned char* base, int k) -> unsigned char* {
    size_t off = 0;
    const size_t sizes[5] = {size_t(Bn * seg) * row_d, size_t(Bn * seg) * row_s,
                             size_t(Bn * seg) * row_bc, size_t(Bn * seg) * row_bc,
                             size_t(Bn * seg) * row_y};
    for (int i = 0; i < k; ++i) off += align_up(sizes[i], 256);
    return base + off;
  };
  // one strided copy: rows = batch, each row `width` bytes at host stride T*row
  auto copy_in = [&](unsigned char* dst, const void* src, size_t row, int64_t k) {
    const int64_t t0 = piece_start(k), len = piece_len(k);
    return cudaMemcpy2DAsync(dst, size_t(len) * row,
                             static_cast<const unsigned char*>(src) + size_t(t0) * row,
                             size_t(T) * row, size_t(len) * row, size_t(Bn),
                             cudaMemcpyHostToDevice, hp->in);
  };

  // parameters and the start state on the caller's stream, then fork
  rc = ck(cudaMemcpyAsync(lam_d, a->lambda_, size_t(D * N) * 16, cudaMemcpyHostToDevice, st),
          "Lambda copy");
  if (rc == MQC_OK)
    rc = ck(cudaMemcpyAsync(dsk_d, a->dskip, size_t(D) * 4, cudaMemcpyHostToDevice, st),
            "skip copy");
  if (rc == MQC_OK && a->h0 != nullptr)
    rc = ck(cudaMemcpyAsync(hbuf[0], a->h0, size_t(Bn * D * N) * 16, cudaMemcpyHostToDevice, st),
            "h0 copy");
  if (rc == MQC_OK) rc = ck(cudaEventRecord(hp->ev[6], st), "event");
  if (rc == MQC_OK) rc = ck(cudaStreamWaitEvent(hp->in, hp->ev[6], 0), "wait");
  if (rc == MQC_OK) rc = ck(cudaStreamWaitEvent(hp->out, hp->ev[6], 0), "wait");

  for (int64_t k = 0; k < pieces && rc == MQC_OK; ++k) {
    const int j = int(k & 1);
    unsigned char* sl = slot[j];
    // copy in (slot j is free once the scan of segment k-2 is done)
    if (k >= 2) rc = ck(cudaStreamWaitEvent(hp->in, hp->ev[2 + j], 0), "wait");
    if (rc == MQC_OK) rc = ck(copy_in(part(sl, 0), a->delta, row_d, k), "delta copy");
    if (rc == MQC_OK) rc = ck(copy_in(part(sl, 1), a->s, row_s, k), "s copy");
    if (rc == MQC_OK) rc = ck(copy_in(part(sl, 2), a->Bm, row_bc, k), "B copy");
    if (rc == MQC_OK) rc = ck(copy_in(part(sl, 3), a->Cm, row_bc, k), "C copy");
    if (rc == MQC_OK) rc = ck(cudaEventRecord(hp->ev[j], hp->in), "event");
    // scan on the caller's stream (y slot j is free once segment k-2 is copied out)
    if (rc == MQC_OK) rc = ck(cudaStreamWaitEvent(st, hp->ev[j], 0), "wait");
    if (rc == MQC_OK && k >= 2) rc = ck(cudaStreamWaitEvent(st, hp->ev[4 + j], 0), "wait");
    if (rc == MQC_OK) {
      mqc_ssm_scan_args s = *a;
      s.batch = Bn;
      s.seq_len = piece_len(k);
      s.delta = part(sl, 0);
      s.s = part(sl, 1);
      s.Bm = part(sl, 2);
      s.Cm = part(sl, 3);
      s.y = part(sl, 4);
      s.lambda_ = lam_d;
      s.dskip = dsk_d;
      s.h0 = (k == 0 && a->h0 == nullptr) ? nullptr : hbuf[k & 1];
      s.hT = hbuf[(k + 1) & 1];
      rc = mqc_ssm_scan_fwd(&s, stream);
    }
    if (rc == MQC_OK) rc = ck(cudaEventRecord(hp->ev[2 + j], st), "event");
    // copy out
    if (rc == MQC_OK) rc = ck(cudaStreamWaitEvent(hp->out, hp->ev[2 + j], 0), "wait");
    if (rc == MQC_OK)
      rc = ck(cudaMemcpy2DAsync(
                  static_cast<unsigned char*>(a->y) + size_t(piece_start(k)) * row_y,
                  size_t(T) * row_y, part(sl, 4), size_t(piece_len(k)) * row_y,
                  size_t(piece_len(k)) * row_y, size_t(Bn), cudaMemcpyDeviceToHost, hp->out),
              "y copy");
    if (rc == MQC_OK) rc = ck(cudaEventRecord(hp->ev[4 + j], hp->out), "event");
  }
  // join: the caller's stream waits for every copy; final state; scratch freed
  if (rc == MQC_OK) rc = ck(cudaEventRecord(hp->ev[7], hp->out), "event");
  if (rc == MQC_OK) rc = ck(cudaStreamWaitEvent(st, hp->ev[7], 0), "wait");
  if (rc == MQC_OK) rc = ck(cudaEventRecord(hp->ev[6], hp->in), "event");
  if (rc == MQC_OK) rc = ck(cudaStreamWaitEvent(st, hp->ev[6], 0), "wait");
  if (rc == MQC_OK && a->hT != nullptr)
    rc = ck(cudaMemcpyAsync(a->hT, hbuf[pieces & 1], size_t(Bn * D * N) * 16,
                            cudaMemcpyDeviceToHost, st),
            "hT copy");
  scratch_free(ws, st);
  return rc;
}
