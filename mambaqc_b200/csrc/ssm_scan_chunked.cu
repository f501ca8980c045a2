// Time-chunked (time-parallel) selective scan forward.
//
// For long sequences with few (b, d, n) lanes -- one channel shard of a long
// sequence per GPU -- the sequential scan cannot fill the GPU. The scan
// h_t = q_t (x) h_{t-1} + u_t is affine in h, and affine maps compose in order
// (later (x) earlier): over a chunk of steps it is h -> P (x) h + h_loc with
// P = q_last (x) ... (x) q_first and h_loc the chunk's final state from h = 0.
// So with T cut into nc equal chunks (the chunk index folded into the batch:
// [B, T, ...] is viewed as [B*nc, T/nc, ...], no copies):
//   pass 1  state-only scan of every chunk from zero -> (P_c, h_loc_c)
//   carry   H_{-1} = h0, H_c = P_c (x) H_{c-1} + h_loc_c   (sequential over c, per lane)
//   pass 2  the regular fused scan of every chunk from H_{c-1} -> y
// Pass 2 is the same kernel as the unchunked scan; the extra work is pass 1
// (a scan without readout) and the carry (3 x 16 B per chunk and lane).
#include <cstdlib>

#include "ssm_scan_common.cuh"

namespace mqc {
namespace scan {
namespace {

constexpr int kCarryThreads = 256;

// grid (ceil(lanes / 256), batch); P, hloc, hin: [batch, nc, lanes, 4]; h0, hT: [batch, lanes, 4]
__global__ void __launch_bounds__(kCarryThreads)
    chunk_carry_kernel(const float* __restrict__ P, const float* __restrict__ hloc,
                       const float* __restrict__ h0, float* __restrict__ hin,
                       float* __restrict__ hT, int nc, int64_t lanes) {
  const int64_t l = int64_t(blockIdx.x) * kCarryThreads + threadIdx.x;
  if (l >= lanes) return;
  const int64_t b = blockIdx.y;
  float4 H = h0 != nullptr ? QIO<float>::ld(h0 + (b * lanes + l) * 4) : f4_zero();
  for (int c = 0; c < nc; ++c) {
    const int64_t idx = ((b * nc + c) * lanes + l) * 4;
    QIO<float>::st(hin + idx, H);
    H = qmul_acc(QIO<float>::ld(P + idx), H, QIO<float>::ld(hloc + idx));
  }
  if (hT != nullptr) QIO<float>::st(hT + (b * lanes + l) * 4, H);
}

// Composition of chunk summaries into one: over c = 0 .. nc-1,
// Q <- P_c (x) Q (Q = 1 at first), E <- P_c (x) E + hloc_c (E = 0 at first).
// grid (ceil(lanes / 256), batch); P, hloc: [batch, nc, lanes, 4]; Pout, Eout: [batch, lanes, 4]
__global__ void __launch_bounds__(kCarryThreads)
    chunk_compose_kernel(const float* __restrict__ P, const float* __restrict__ hloc,
                         float* __restrict__ Pout, float* __restrict__ Eout, int nc,
                         int64_t lanes) {
  const int64_t l = int64_t(blockIdx.x) * kCarryThreads + threadIdx.x;
  if (l >= lanes) return;
  const int64_t b = blockIdx.y;
  float4 Q = make_float4(1.f, 0.f, 0.f, 0.f);
  float4 E = f4_zero();
  for (int c = 0; c < nc; ++c) {
    const int64_t idx = ((b * nc + c) * lanes + l) * 4;
    const float4 Pc = QIO<float>::ld(P + idx);
    E = qmul_acc(Pc, E, QIO<float>::ld(hloc + idx));
    Q = qmul(Pc, Q);
  }
  QIO<float>::st(Pout + (b * lanes + l) * 4, Q);
  QIO<float>::st(Eout + (b * lanes + l) * 4, E);
}

// Start states of consecutive time segments from their summaries:
// H_0 = h0 (or 0), H_{s+1} = P_s (x) H_s + E_s; hin[s] = H_s, hT = H_S.
// grid (ceil(lanes / 256), batch); P, E, hin: [segments, batch, lanes, 4]
__global__ void __launch_bounds__(kCarryThreads)
    segment_carry_kernel(const float* __restrict__ P, const float* __restrict__ E,
                         const float* __restrict__ h0, float* __restrict__ hin,
                         float* __restrict__ hT, int segments, int batch, int64_t lanes) {
  const int64_t l = int64_t(blockIdx.x) * kCarryThreads + threadIdx.x;
  if (l >= lanes) return;
  const int64_t b = blockIdx.y;
  float4 H = h0 != nullptr ? QIO<float>::ld(h0 + (b * lanes + l) * 4) : f4_zero();
  for (int sg = 0; sg < segments; ++sg) {
    const int64_t idx = ((int64_t(sg) * batch + b) * lanes + l) * 4;
    if (hin != nullptr) QIO<float>::st(hin + idx, H);
    H = qmul_acc(QIO<float>::ld(P + idx), H, QIO<float>::ld(E + idx));
  }
  if (hT != nullptr) QIO<float>::st(hT + (b * lanes + l) * 4, H);
}

size_t chunked_workspace(int64_t batch, int64_t nchunks, int64_t lanes) {
  return size_t(3) * size_t(batch) * size_t(nchunks) * size_t(lanes) * 16;
}

}  // namespace
}  // namespace scan
}  // namespace mqc

using namespace mqc;
using namespace mqc::scan;

namespace {

// Peer outputs of the channel-sharded scan (mqc_ssm_scan_fwd_chunked_peer).
struct PeerSpec {
  void* const* ptrs;
  int n;
  int64_t ch_total, ch_off;
  bool mc;  // ptrs[0] is a multicast address (n == 1)
};

// Pass 2 (or the whole scan when nchunks == 1): mqc_ssm_scan_fwd, or with peer
// outputs the packed kernel writing y into every peer buffer.
int scan_pass(const mqc_ssm_scan_args* a2, const PeerSpec* peer, void* stream) {
  if (peer == nullptr) return mqc_ssm_scan_fwd(a2, stream);
  FwdParams p{};
  int rc = validate_and_fill(a2, &p, "mqc_ssm_scan_fwd_chunked_peer");
  if (rc != MQC_OK || p.T == 0 || p.B == 0 || p.D == 0) return rc;
  p.npeer = peer->n;
  for (int r = 0; r < peer->n; ++r) p.ypeer[r] = peer->ptrs[r];
  p.y_ld = peer->ch_total * 4;
  p.y_coff = peer->ch_off * 4;
  p.peer_mc = peer->mc ? 1 : 0;
  return dispatch_shared_packed(p, a2->dtype, (a2->flags & MQC_SSM_S_REAL) != 0,
                                as_stream(stream));
}

// Carry (start state of every chunk from the chunk summaries P, hloc and h0, and
// the final state) followed by pass 2: the regular scan of every chunk from its
// start state, chunks folded into the batch.
int carry_and_rescan(const mqc_ssm_scan_args* a, const FwdParams& p, int64_t nchunks,
                     const float* Pbuf, const float* hloc, float* hin, const PeerSpec* peer,
                     void* stream) {
  const int64_t lanes = int64_t(p.D) * p.N;
  cudaStream_t st = as_stream(stream);
  dim3 grid{unsigned((lanes + kCarryThreads - 1) / kCarryThreads), unsigned(p.B), 1u};
  chunk_carry_kernel<<<grid, kCarryThreads, 0, st>>>(Pbuf, hloc, p.h0, hin, p.hT, int(nchunks),
                                                     lanes);
  int rc = check_launch("mqc_ssm_scan_fwd_chunked(carry)");
  if (rc != MQC_OK) return rc;
  mqc_ssm_scan_args a2 = *a;
  a2.batch = int64_t(p.B) * nchunks;
  a2.seq_len = p.T / nchunks;
  a2.h0 = hin;
  a2.hT = nullptr;
  return scan_pass(&a2, peer, stream);
}

int chunked_impl(const mqc_ssm_scan_args* a, int64_t nchunks, void* workspace,
                 size_t workspace_bytes, const PeerSpec* peer, void* stream);

}  // namespace

extern "C" size_t mqc_ssm_scan_fwd_chunked_workspace_size(int64_t batch, int64_t channels,
                                                          int64_t d_state, int64_t nchunks) {
  if (batch <= 0 || channels <= 0 || d_state <= 0 || nchunks <= 0) return 0;
  return chunked_workspace(batch, nchunks, channels * d_state);
}

extern "C" int mqc_ssm_scan_fwd_chunked(const mqc_ssm_scan_args* a, int64_t nchunks,
                                        void* workspace, size_t workspace_bytes,
                                        void* stream) {
  clear_error();
  return chunked_impl(a, nchunks, workspace, workspace_bytes, nullptr, stream);
}

extern "C" int mqc_ssm_scan_fwd_chunked_peer(const mqc_ssm_scan_args* a, int64_t nchunks,
                                             void* workspace, size_t workspace_bytes,
                                             void* const* ypeer, int npeer, int64_t ch_total,
                                             int64_t ch_off, void* stream) {
  clear_error();
  const char* name = "mqc_ssm_scan_fwd_chunked_peer";
  MQC_REQUIRE(a != nullptr && ypeer != nullptr, MQC_ERR_INVALID_VALUE, "%s: null pointer", name);
  MQC_REQUIRE(npeer >= 1 && npeer <= kMaxPeerOutputs, MQC_ERR_INVALID_VALUE,
              "%s: 1 to %d outputs, got %d", name, kMaxPeerOutputs, npeer);
  MQC_REQUIRE((a->flags & MQC_SSM_BC_SHARED) && !(a->flags & MQC_SSM_Q_GIVEN), MQC_ERR_UNSUPPORTED,
              "%s: channel-shared B/C and the fused Cayley form only", name);
  const char* impl = getenv("MQC_SCAN_IMPL");
  MQC_REQUIRE(impl == nullptr || impl[0] == '\0', MQC_ERR_UNSUPPORTED,
              "%s: needs the packed kernel (MQC_SCAN_IMPL is set)", name);
  MQC_REQUIRE(a->ckpt == nullptr && a->dskip_sb == 0 && a->dskip_st == 0, MQC_ERR_UNSUPPORTED,
              "%s: no checkpoints, per-channel skip weight only", name);
  MQC_REQUIRE(nchunks >= 1 && a->seq_len % nchunks == 0 && a->seq_len / nchunks > kShortScan,
              MQC_ERR_UNSUPPORTED, "%s: seq_len / nchunks must be an integer above %d", name,
              kShortScan);
  MQC_REQUIRE(ch_off >= 0 && ch_off + a->channels <= ch_total, MQC_ERR_INVALID_VALUE,
              "%s: channels [%lld, +%lld) outside %lld", name, (long long)ch_off,
              (long long)a->channels, (long long)ch_total);
  const uintptr_t qa = a->dtype == MQC_DTYPE_F32 ? 16 : 8;
  for (int r = 0; r < npeer; ++r)
    MQC_REQUIRE(ypeer[r] != nullptr && aligned(ypeer[r], qa), MQC_ERR_MISALIGNED,
                "%s: output %d null or not %d-byte aligned", name, r, int(qa));
  mqc_ssm_scan_args a1 = *a;
  a1.y = ypeer[0];  // validated like y; the kernel writes every ypeer[r]
  const PeerSpec peer{ypeer, npeer, ch_total, ch_off, false};
  return chunked_impl(&a1, nchunks, workspace, workspace_bytes, &peer, stream);
}

extern "C" int mqc_ssm_scan_fwd_chunked_multicast(const mqc_ssm_scan_args* a, int64_t nchunks,
                                                  void* workspace, size_t workspace_bytes,
                                                  void* ymc, int64_t ch_total, int64_t ch_off,
                                                  void* stream) {
  clear_error();
  const char* name = "mqc_ssm_scan_fwd_chunked_multicast";
  MQC_REQUIRE(a != nullptr && ymc != nullptr, MQC_ERR_INVALID_VALUE, "%s: null pointer", name);
  MQC_REQUIRE((a->flags & MQC_SSM_BC_SHARED) && !(a->flags & MQC_SSM_Q_GIVEN), MQC_ERR_UNSUPPORTED,
              "%s: channel-shared B/C and the fused Cayley form only", name);
  // the packed kernel gathers a quaternion from four lanes of its channel: at
  // least four lanes per channel, i.e. d_state above 16
  MQC_REQUIRE(a->d_state > 16 && a->d_state <= 256, MQC_ERR_UNSUPPORTED,
              "%s: d_state must be in (16, 256] (got %lld)", name, (long long)a->d_state);
  const char* impl = getenv("MQC_SCAN_IMPL");
  MQC_REQUIRE(impl == nullptr || impl[0] == '\0', MQC_ERR_UNSUPPORTED,
              "%s: needs the packed kernel (MQC_SCAN_IMPL is set)", name);
  MQC_REQUIRE(a->ckpt == nullptr && a->dskip_sb == 0 && a->dskip_st == 0, MQC_ERR_UNSUPPORTED,
              "%s: no checkpoints, per-channel skip weight only", name);
  MQC_REQUIRE(nchunks >= 1 && a->seq_len % nchunks == 0 && a->seq_len / nchunks > kShortScan,
              MQC_ERR_UNSUPPORTED, "%s: seq_len / nchunks must be an integer above %d", name,
              kShortScan);
  MQC_REQUIRE(ch_off >= 0 && ch_off + a->channels <= ch_total, MQC_ERR_INVALID_VALUE,
              "%s: channels [%lld, +%lld) outside %lld", name, (long long)ch_off,
              (long long)a->channels, (long long)ch_total);
  const uintptr_t qa = a->dtype == MQC_DTYPE_F32 ? 16 : 8;
  MQC_REQUIRE(aligned(ymc, qa), MQC_ERR_MISALIGNED, "%s: output not %d-byte aligned", name,
              int(qa));
  mqc_ssm_scan_args a1 = *a;
  a1.y = ymc;  // validated like y; the kernel writes it only with multimem stores
  void* const ptrs[1] = {ymc};
  const PeerSpec peer{ptrs, 1, ch_total, ch_off, true};
  return chunked_impl(&a1, nchunks, workspace, workspace_bytes, &peer, stream);
}

namespace {

int chunked_impl(const mqc_ssm_scan_args* a, int64_t nchunks, void* workspace,
                 size_t workspace_bytes, const PeerSpec* peer, void* stream) {
  const char* name = peer ? "mqc_ssm_scan_fwd_chunked_peer" : "mqc_ssm_scan_fwd_chunked";
  MQC_REQUIRE(a != nullptr, MQC_ERR_INVALID_VALUE, "%s: null args", name);
  MQC_REQUIRE(!(a->flags & MQC_SSM_Q_GIVEN), MQC_ERR_UNSUPPORTED,
              "%s: explicit q is not supported (use the fused form)", name);
  MQC_REQUIRE(a->ckpt == nullptr, MQC_ERR_UNSUPPORTED, "%s: no checkpoints (forward only)", name);
  MQC_REQUIRE(nchunks >= 1, MQC_ERR_INVALID_VALUE, "%s: nchunks must be >= 1", name);
  FwdParams p{};
  int rc = validate_and_fill(a, &p, name);
  if (rc != MQC_OK || p.T == 0 || p.B == 0 || p.D == 0) return rc;
  if (nchunks == 1) return scan_pass(a, peer, stream);
  MQC_REQUIRE(p.T % nchunks == 0, MQC_ERR_INVALID_VALUE, "%s: seq_len %d not divisible by %lld",
              name, p.T, (long long)nchunks);
  // chunks are folded into the batch, so the skip weight may vary over channels only
  MQC_REQUIRE(a->dskip_sb == 0 && a->dskip_st == 0, MQC_ERR_UNSUPPORTED,
              "%s: the skip weight must be per channel ([D], strides 0 over batch and time)", name);
  MQC_REQUIRE(int64_t(p.B) * nchunks <= 65535, MQC_ERR_UNSUPPORTED,
              "%s: batch * nchunks must be <= 65535", name);
  const int64_t lanes = int64_t(p.D) * p.N;
  const size_t need = chunked_workspace(p.B, nchunks, lanes);
  MQC_REQUIRE(workspace != nullptr && workspace_bytes >= need && aligned(workspace, 16),
              MQC_ERR_INVALID_VALUE, "%s: 16-byte aligned workspace of %zu bytes required", name,
              need);
  float* Pbuf = static_cast<float*>(workspace);
  float* hloc = Pbuf + size_t(p.B) * nchunks * lanes * 4;
  float* hin = hloc + size_t(p.B) * nchunks * lanes * 4;
  cudaStream_t st = as_stream(stream);
  const bool s_real = a->flags & MQC_SSM_S_REAL;
  const bool shared = a->flags & MQC_SSM_BC_SHARED;

  // pass 1: state-only scan of each chunk from zero, chunks folded into the batch.
  // With one batch row the last chunk's summary is never read (the final state
  // comes out of pass 2), so pass 1 stops one chunk short.
  const bool skip_last = p.B == 1;
  FwdParams p1 = p;
  p1.B = skip_last ? int(nchunks - 1) : int(int64_t(p.B) * nchunks);
  p1.T = int(p.T / nchunks);
  p1.h0 = nullptr;
  p1.hT = hloc;
  p1.pout = Pbuf;
  p1.y = nullptr;
  p1.ckpt = nullptr;
  p1.nck = 0;
  const char* impl = getenv("MQC_SCAN_IMPL");
  const bool packed = shared && (impl == nullptr || impl[0] == '\0');
  rc = packed ? dispatch_state_only_packed(p1, a->dtype, s_real, st)
              : dispatch_state_only(p1, a->dtype, s_real, shared, st);
  if (rc != MQC_OK) return rc;
  if (!skip_last) return carry_and_rescan(a, p, nchunks, Pbuf, hloc, hin, peer, stream);

  // one batch row: carry over the first nc-1 summaries gives every chunk's start
  // state (the last one written as the carry's final state); pass 2 then writes
  // each chunk's final state into hloc (free by then) and the last one is hT
  dim3 grid{unsigned((lanes + kCarryThreads - 1) / kCarryThreads), 1u, 1u};
  chunk_carry_kernel<<<grid, kCarryThreads, 0, st>>>(Pbuf, hloc, p.h0, hin,
                                                     hin + size_t(nchunks - 1) * lanes * 4,
                                                     int(nchunks - 1), lanes);
  rc = check_launch("mqc_ssm_scan_fwd_chunked(carry)");
  if (rc != MQC_OK) return rc;
  mqc_ssm_scan_args a2 = *a;
  a2.batch = nchunks;
  a2.seq_len = p.T / nchunks;
  a2.h0 = hin;
  a2.hT = p.hT != nullptr ? hloc : nullptr;
  rc = scan_pass(&a2, peer, stream);
  if (rc != MQC_OK || p.hT == nullptr) return rc;
  const cudaError_t e = cudaMemcpyAsync(p.hT, hloc + size_t(nchunks - 1) * lanes * 4,
                                        size_t(lanes) * 16, cudaMemcpyDeviceToDevice, st);
  return e == cudaSuccess ? MQC_OK
                          : fail(MQC_ERR_CUDA, "%s: final state copy: %s", name,
                                 cudaGetErrorString(e));
}

}  // namespace

extern "C" size_t mqc_ssm_scan_fwd_summary_workspace_size(int64_t batch, int64_t channels,
                                                          int64_t d_state, int64_t nchunks) {
  // the chunk summaries plus room for the chunk start states, so that the same
  // workspace can be handed to mqc_ssm_scan_fwd_chunked_resume
  if (batch <= 0 || channels <= 0 || d_state <= 0 || nchunks <= 1) return 0;
  return chunked_workspace(batch, nchunks, channels * d_state);
}

extern "C" int mqc_ssm_scan_fwd_summary(const mqc_ssm_scan_args* a, int64_t nchunks, float* P,
                                        float* E, void* workspace, size_t workspace_bytes,
                                        void* stream) {
  clear_error();
  const char* name = "mqc_ssm_scan_fwd_summary";
  MQC_REQUIRE(a != nullptr, MQC_ERR_INVALID_VALUE, "%s: null args", name);
  MQC_REQUIRE(!(a->flags & MQC_SSM_Q_GIVEN), MQC_ERR_UNSUPPORTED,
              "%s: explicit q is not supported (use the fused form)", name);
  MQC_REQUIRE(a->ckpt == nullptr && a->h0 == nullptr && a->hT == nullptr,
              MQC_ERR_INVALID_VALUE, "%s: h0, hT and ckpt must be NULL (the summary is the map "
              "from the zero state)", name);
  MQC_REQUIRE(nchunks >= 1, MQC_ERR_INVALID_VALUE, "%s: nchunks must be >= 1", name);
  MQC_REQUIRE(P != nullptr && E != nullptr && aligned(P, 16) && aligned(E, 16),
              MQC_ERR_INVALID_VALUE, "%s: P and E must be 16-byte aligned device buffers", name);
  // y is not written; the caller's y (or P, when it has none) only passes the checks
  mqc_ssm_scan_args av = *a;
  if (av.y == nullptr) av.y = P;
  FwdParams p{};
  int rc = validate_and_fill(&av, &p, name);
  if (rc != MQC_OK || p.B == 0 || p.D == 0) return rc;
  cudaStream_t st = as_stream(stream);
  const int64_t lanes = int64_t(p.D) * p.N;
  if (p.T == 0) {
    // empty sequence: the identity map
    dim3 grid{unsigned((lanes + kCarryThreads - 1) / kCarryThreads), unsigned(p.B), 1u};
    chunk_compose_kernel<<<grid, kCarryThreads, 0, st>>>(P, E, P, E, 0, lanes);
    return check_launch(name);
  }
  MQC_REQUIRE(p.T % nchunks == 0, MQC_ERR_INVALID_VALUE, "%s: seq_len %d not divisible by %lld",
              name, p.T, (long long)nchunks);
  MQC_REQUIRE(int64_t(p.B) * nchunks <= 65535, MQC_ERR_UNSUPPORTED,
              "%s: batch * nchunks must be <= 65535", name);
  const bool s_real = a->flags & MQC_SSM_S_REAL;
  const bool shared = a->flags & MQC_SSM_BC_SHARED;
  float* Pc = P;
  float* Ec = E;
  if (nchunks > 1) {
    const size_t need = mqc_ssm_scan_fwd_summary_workspace_size(p.B, p.D, p.N, nchunks);
    MQC_REQUIRE(workspace != nullptr && workspace_bytes >= need && aligned(workspace, 16),
                MQC_ERR_INVALID_VALUE, "%s: 16-byte aligned workspace of %zu bytes required",
                name, need);
    Pc = static_cast<float*>(workspace);
    Ec = Pc + size_t(p.B) * nchunks * lanes * 4;
  }
  FwdParams p1 = p;
  p1.B = int(int64_t(p.B) * nchunks);
  p1.T = int(p.T / nchunks);
  p1.h0 = nullptr;
  p1.hT = Ec;
  p1.pout = Pc;
  p1.y = nullptr;
  p1.ckpt = nullptr;
  p1.nck = 0;
  const char* impl = getenv("MQC_SCAN_IMPL");
  const bool packed = shared && (impl == nullptr || impl[0] == '\0');
  rc = packed ? dispatch_state_only_packed(p1, a->dtype, s_real, st)
              : dispatch_state_only(p1, a->dtype, s_real, shared, st);
  if (rc != MQC_OK || nchunks == 1) return rc;
  dim3 grid{unsigned((lanes + kCarryThreads - 1) / kCarryThreads), unsigned(p.B), 1u};
  chunk_compose_kernel<<<grid, kCarryThreads, 0, st>>>(Pc, Ec, P, E, int(nchunks), lanes);
  return check_launch(name);
}

extern "C" int mqc_ssm_scan_carry(const float* P, const float* E, const float* h0, float* hin,
                                  float* hT, int64_t segments, int64_t batch, int64_t lanes,
                                  void* stream) {
  clear_error();
  const char* name = "mqc_ssm_scan_carry";
  MQC_REQUIRE(segments >= 0 && batch >= 0 && lanes >= 0, MQC_ERR_INVALID_VALUE,
              "%s: negative size", name);
  MQC_REQUIRE(segments <= INT32_MAX && batch <= 65535, MQC_ERR_UNSUPPORTED,
              "%s: sizes too large", name);
  if (batch == 0 || lanes == 0) return MQC_OK;
  MQC_REQUIRE(segments == 0 || (P != nullptr && E != nullptr), MQC_ERR_INVALID_VALUE,
              "%s: null P or E", name);
  MQC_REQUIRE((P == nullptr || aligned(P, 16)) && (E == nullptr || aligned(E, 16)) &&
                  (h0 == nullptr || aligned(h0, 16)) && (hin == nullptr || aligned(hin, 16)) &&
                  (hT == nullptr || aligned(hT, 16)),
              MQC_ERR_MISALIGNED, "%s: buffers must be 16-byte aligned", name);
  dim3 grid{unsigned((lanes + kCarryThreads - 1) / kCarryThreads), unsigned(batch), 1u};
  segment_carry_kernel<<<grid, kCarryThreads, 0, as_stream(stream)>>>(
      P, E, h0, hin, hT, int(segments), int(batch), lanes);
  return check_launch(name);
}

extern "C" int mqc_ssm_scan_fwd_chunked_resume(const mqc_ssm_scan_args* a, int64_t nchunks,
                                               void* workspace, size_t workspace_bytes,
                                               void* stream) {
  clear_error();
  const char* name = "mqc_ssm_scan_fwd_chunked_resume";
  MQC_REQUIRE(a != nullptr, MQC_ERR_INVALID_VALUE, "%s: null args", name);
  MQC_REQUIRE(!(a->flags & MQC_SSM_Q_GIVEN), MQC_ERR_UNSUPPORTED,
              "%s: explicit q is not supported (use the fused form)", name);
  MQC_REQUIRE(a->ckpt == nullptr, MQC_ERR_UNSUPPORTED, "%s: no checkpoints (forward only)", name);
  MQC_REQUIRE(nchunks >= 1, MQC_ERR_INVALID_VALUE, "%s: nchunks must be >= 1", name);
  FwdParams p{};
  int rc = validate_and_fill(a, &p, name);
  if (rc != MQC_OK || p.T == 0 || p.B == 0 || p.D == 0) return rc;
  if (nchunks == 1) return mqc_ssm_scan_fwd(a, stream);
  MQC_REQUIRE(p.T % nchunks == 0, MQC_ERR_INVALID_VALUE, "%s: seq_len %d not divisible by %lld",
              name, p.T, (long long)nchunks);
  MQC_REQUIRE(a->dskip_sb == 0 && a->dskip_st == 0, MQC_ERR_UNSUPPORTED,
              "%s: the skip weight must be per channel ([D], strides 0 over batch and time)", name);
  MQC_REQUIRE(int64_t(p.B) * nchunks <= 65535, MQC_ERR_UNSUPPORTED,
              "%s: batch * nchunks must be <= 65535", name);
  const int64_t lanes = int64_t(p.D) * p.N;
  const size_t need = chunked_workspace(p.B, nchunks, lanes);
  MQC_REQUIRE(workspace != nullptr && workspace_bytes >= need && aligned(workspace, 16),
              MQC_ERR_INVALID_VALUE, "%s: 16-byte aligned workspace of %zu bytes required", name,
              need);
  const float* Pbuf = static_cast<const float*>(workspace);
  const float* hloc = Pbuf + size_t(p.B) * nchunks * lanes * 4;
  float* hin = static_cast<float*>(workspace) + size_t(2) * p.B * nchunks * lanes * 4;
  return carry_and_rescan(a, p, nchunks, Pbuf, hloc, hin, nullptr, stream);
}
