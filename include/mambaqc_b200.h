/*
 * mambaqc_b200 -- C ABI of the B200 (sm_100a) quaternion SSM hot path.
 *
 * Every entry point takes raw device pointers, sizes in elements and a CUDA
 * stream (cudaStream_t passed as void*; NULL = legacy default stream), launches
 * asynchronously on that stream and never synchronises. Entry points allocate no
 * device memory, except where a declaration below says otherwise.
 * Tensors are dense and row-major (C order) unless a stride is given; a
 * quaternion is the last axis of 4 scalars (r, i, j, k), the layout of the
 * reference's [..., 4] tensors. Return value: MQC_OK or an mqc_status code; on
 * failure mqc_last_error() gives a human-readable message for the calling host
 * thread.
 *
 * Each declaration cites the reference (polux06/mambaqc) Python function it
 * replaces, as path:line inside that project.
 */
#ifndef MAMBAQC_B200_H_
#define MAMBAQC_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define MQC_API __attribute__((visibility("default")))
#else
#define MQC_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Storage type of floating-point tensor arguments. Arithmetic is fp32. */
typedef enum mqc_dtype {
  MQC_DTYPE_F32 = 0,
  MQC_DTYPE_BF16 = 1
} mqc_dtype;

typedef enum mqc_status {
  MQC_OK = 0,
  MQC_ERR_INVALID_VALUE = 1, /* bad size, null pointer, unknown flag         */
  MQC_ERR_MISALIGNED = 2,    /* pointer not aligned to its vector width      */
  MQC_ERR_UNSUPPORTED = 3,   /* valid but not implemented (e.g. d_state>256) */
  MQC_ERR_CUDA = 4,          /* CUDA runtime error at launch                 */
  MQC_ERR_DEVICE_TIMEOUT = 5 /* a bounded device-side wait gave up           */
} mqc_status;

/* Bits a kernel ORs into a caller-provided device status word (int32). */
#define MQC_DEVICE_STATUS_TIMEOUT 0x1

/* Library version, "major.minor.patch". */
MQC_API const char* mqc_version(void);
/* Static description of an mqc_status code. */
MQC_API const char* mqc_status_string(int status);
/* Detail of the last failing call on this host thread ("" if none). */
MQC_API const char* mqc_last_error(void);

/* ---- quaternion algebra: mambaqc/kernels/quaternion_ops.py ---------------- */

/* out[i] = p[i] (x) q[i] (Hamilton product), i < n quaternions.
 * Replaces quaternion_multiply(p, q), quaternion_ops.py:259-303, and
 * quaternion_multiply_batched, quaternion_ops.py:306-357 (dense case). */
MQC_API int mqc_qmul(const void* p, const void* q, void* out, int64_t n, int dtype, void* stream);

/* out[i0,i1,i2,i3] = p[i0,i1,i2,i3] (x) q[i0,i1,i2,i3] over the index space
 * shape[0..3] = [batch, seq_len, d_model, d_state], p and q read through element
 * strides per axis (non-negative multiples of 4; 0 broadcasts; the quaternion
 * axis itself contiguous), out dense [shape..., 4]. shape[0]*shape[1] and
 * shape[2]*shape[3] below 2^31. Replaces quaternion_multiply_batched with its
 * stride arguments, quaternion_ops.py:306-357 (kernel :77-160), without a copy
 * of non-contiguous inputs. */
MQC_API int mqc_qmul_strided(const void* p, const void* q, void* out, const int64_t* shape,
                             const int64_t* p_strides, const int64_t* q_strides, int dtype,
                             void* stream);

/* out[i] = conj(q[i]). Replaces quaternion_conjugate, quaternion_ops.py:360-391. */
MQC_API int mqc_qconj(const void* q, void* out, int64_t n, int dtype, void* stream);

/* out[i] = conj(q[i]) / max(|q[i]|^2, eps).
 * Replaces quaternion_inverse(q, eps), quaternion_ops.py:394-428. */
MQC_API int mqc_qinv(const void* q, void* out, int64_t n, float eps, int dtype, void* stream);

/* out[i] = |q[i]| (one scalar per quaternion, same dtype).
 * Replaces quaternion_norm, quaternion_ops.py:431-461. */
MQC_API int mqc_qnorm(const void* q, void* out, int64_t n, int dtype, void* stream);

/* q[i] = (1 - z[i]/2)^-1 (x) (1 + z[i]/2), |1 - z/2|^2 clamped below by eps.
 * Replaces cayley_discretization_fused(z, eps), cayley_transform.py:132-195. */
MQC_API int mqc_cayley(const void* z, void* q, int64_t n, float eps, int dtype, void* stream);

/* dz[i] = (dq/dz[i])^T dq[i]: the vector-Jacobian product of mqc_cayley, with the
 * eps clamp treated as a constant where active. The reference has no GPU
 * backward (its Cayley kernel, cayley_transform.py:24-129, is not
 * differentiable); this is the gradient of cayley_discretization_reference,
 * cayley_transform.py:199-223, as torch autograd computes it on the CPU. */
MQC_API int mqc_cayley_bwd(const void* z, const void* dq, void* dz, int64_t n, float eps, int dtype,
                   void* stream);

/* ---- prefix product: mambaqc/kernels/parallel_scan.py --------------------- */

/* For q, out of shape [batch, seq_len, lanes, 4] (lanes = d_model * d_state):
 * out[b,t,l] = q[b,t,l] (x) out[b,t-1,l], out[b,-1,l] = 1.
 * When batch*lanes is too small to fill the GPU, time is split into chunks and
 * the chunk products go to scratch taken with cudaMallocAsync on `stream` and
 * released with cudaFreeAsync on the same stream (batch*chunks*lanes*16 bytes).
 * Replaces parallel_scan_quaternion(q_sequence), parallel_scan.py:171-264. */
MQC_API int mqc_prefix_prod(const void* q, void* out, int64_t batch, int64_t seq_len, int64_t lanes,
                    int dtype, void* stream);

/* Same result as mqc_prefix_prod, allocating nothing. No counterpart in the
 * reference. For callers that cannot allocate device memory while they run --
 * e.g. a server that gives all device memory to its own allocator at start-up,
 * or a process on a fixed device-memory budget where an allocation failing
 * mid-run is not acceptable. When time is split into chunks, the chunk products
 * live in a fixed 4 MiB static device array that every GPU loading this library
 * holds until exit. The chunk count follows mqc_prefix_prod's rule, capped so
 * that the products (batch * chunks * lanes * 16 bytes) fit in the array; a size
 * where not even two chunks fit runs as one pass over time, which needs no
 * scratch. So every size mqc_prefix_prod accepts is served (bit for bit equal
 * where the cap does not bind, equal up to rounding where it does), and the only
 * rejections are mqc_prefix_prod's own (MQC_ERR_UNSUPPORTED for a grid beyond
 * batch 65535). The first call in each device context looks up the array's
 * device address (set-up, once per context, with that device current); make
 * that first call before any stream capture. All calls share the one array:
 * calls that overlap on the GPU (e.g. on two streams of one device) race.
 * Nothing in the array needs clearing between calls: each call writes every
 * entry it reads. */
MQC_API int mqc_prefix_prod_noalloc(const void* q, void* out, int64_t batch, int64_t seq_len,
                                    int64_t lanes, int dtype, void* stream);

/* ---- selective scan: mambaqc/kernels/ssm_fused.py + block._ssm_forward ------ */

/* Flags of mqc_ssm_scan_args.flags */
#define MQC_SSM_Q_GIVEN 0x1   /* q is given explicitly (else formed from delta, Lambda) */
#define MQC_SSM_BC_SHARED 0x2 /* B, C are [B,T,N,4] shared by all channels           */
#define MQC_SSM_S_REAL 0x4    /* s is a real signal x [B,T,D], S = (x, 0, 0, 0)      */

/*
 * Arguments of one selective scan over time, per (batch b, channel d, state n):
 *
 *   q_t   = Q_GIVEN ? q[b,t,d,n] : cayley(delta[b,t,d] * Lambda[d,n], eps)
 *   h_t   = q_t (x) h_{t-1} + B_t (x) S_t,            h_{-1} = h0 or 0
 *   y_t   = sum_n C_t (x) h_t + D[b,t,d] * S_t
 *
 * Shapes (B batch, T seq_len, D channels, N d_state):
 *   delta [B,T,D] dtype           Lambda [D,N,4] fp32        q [B,T,D,N,4] dtype
 *   Bm, Cm [B,T,N,4] (BC_SHARED) or [B,T,D,N,4], dtype
 *   s  x [B,T,D] (S_REAL) or S [B,T,D,4], dtype
 *   dskip fp32, element (b,t,d) at dskip[b*dskip_sb + t*dskip_st + d*dskip_sd]
 *   h0 [B,D,N,4] fp32 or NULL (zero state); y [B,T,D,4] dtype; hT [B,D,N,4] fp32 or NULL
 *   status: device int32 the kernel ORs MQC_DEVICE_STATUS_* into, or NULL.
 *   wait_poll_limit: polls of a bounded device wait before giving up; <0 = default.
 */
typedef struct mqc_ssm_scan_args {
  int64_t batch, seq_len, channels, d_state;
  int32_t dtype;
  int32_t flags;
  float eps;
  int32_t reserved0;
  const void* delta;
  const float* lambda_;
  const void* q;
  const void* Bm;
  const void* Cm;
  const void* s;
  const float* dskip;
  int64_t dskip_sb, dskip_st, dskip_sd;
  const float* h0;
  void* y;
  float* hT;
  int32_t* status;
  int64_t wait_poll_limit;
  /* Optional state checkpoints for the backward: with ckpt != NULL and
   * ckpt_every = MQC_SSM_CKPT_EVERY, the state after steps K-1, 2K-1, ... (K =
   * ckpt_every, all < T-1) is written to ckpt [B, ceil(T/K)-1, D, N, 4] fp32. */
  float* ckpt;
  int64_t ckpt_every;
} mqc_ssm_scan_args;

/* The checkpoint interval the backward expects. */
#define MQC_SSM_CKPT_EVERY 8

/* Full scan over T. With MQC_SSM_Q_GIVEN this replaces
 * ssm_forward_fused(q, B, S, C, D), ssm_fused.py:340-401; without it, it is the
 * fused form of QuaternionMamba2Block._ssm_forward lines
 * models/quaternion_mamba2_block.py:214-228 (z = Delta*Lambda, Cayley, scan)
 * that never materialises z or q. */
MQC_API int mqc_ssm_scan_fwd(const mqc_ssm_scan_args* args, void* stream);

/* Time-parallel form of mqc_ssm_scan_fwd (fused Cayley, no Q_GIVEN, no
 * checkpoints) for long sequences with few channels: T is cut into nchunks equal
 * chunks (seq_len % nchunks == 0); every chunk is scanned from zero for its end
 * state and operator product, the chunks are chained on the device, and every
 * chunk is rescanned from its true start state. Same outputs as
 * mqc_ssm_scan_fwd (y, optional hT; h0 honoured). The skip weight must be per
 * channel (dskip_sb = dskip_st = 0). `workspace` (16-byte aligned, caller-owned)
 * must hold mqc_ssm_scan_fwd_chunked_workspace_size(...) bytes. The reference's
 * only time-parallel primitive is parallel_scan_quaternion (parallel_scan.py:171),
 * which the model never calls; this is the scan of ssm_forward_fused
 * (ssm_fused.py:340-401) made time-parallel. */
/* mqc_ssm_scan_fwd (fused Cayley form, no checkpoints) on HOST buffers:
 * delta, Lambda, Bm, Cm, s, dskip, h0 (optional) are read from host memory and
 * y, hT (optional) are written to host memory; `status` stays a device pointer
 * or NULL. The skip weight must be per channel (dskip_sb = dskip_st = 0). The
 * sequence is cut into time segments (seq_len % segments == 0; with
 * s = seq_len / segments even and segments >= 2 the pieces are s/2, s, ..., s,
 * s/2, which halves the pipeline's fill and drain), each holding every batch
 * row; segment k is copied in on an internal stream
 * while segment k-1 is scanned on `stream` (from segment k-2's final state) and
 * segment k-2's y is copied out on a second internal stream. Pinned host memory
 * makes the copies asynchronous. Returns once everything is enqueued; the host
 * y and hT are complete when `stream` is. Calls on one device share the two
 * internal streams: do not overlap two calls on one device. This is the
 * host-facing form of QuaternionMamba2Block._ssm_forward lines
 * models/quaternion_mamba2_block.py:214-228, with the transfers inside the call. */
MQC_API int mqc_ssm_scan_fwd_host(const mqc_ssm_scan_args* args, int64_t segments, void* stream);

/*
 * The block's B/C projections fused into its per-channel scan (forward):
 *
 *   B[b,t,d,n,:] = sum_k x[b,t,k] w_b[(d*N + n)*4 + :, k]   (C likewise with w_c)
 *   h_t = cayley(delta[b,t,d] Lambda[d,n]) (x) h_{t-1} + B_t s[b,t,d]
 *   y[b,t,d] = sum_n C_t (x) h_t + dskip[d] (s[b,t,d], 0, 0, 0)
 *
 * with B and C rounded to bf16 (the projection's output in the reference's bf16
 * autocast) and never written to memory: the tensor cores produce each
 * channel's B/C tile on chip and the scan consumes it from shared memory.
 * Shapes: x [batch*seq_len, in_features] bf16 (the block's activated inner
 * signal, row-major); w_b, w_c [channels*d_state*4, in_features] bf16 (the
 * B_proj/C_proj weights as stored); delta, s [batch, seq_len, channels] and
 * y [batch, seq_len, channels, 4] in `dtype`; Lambda [channels, d_state, 4],
 * h0/hT [batch, channels, d_state, 4] fp32 (optional); skip weight of channel d
 * at dskip[d*dskip_sd]. d_state 16, 32 or 64; in_features a multiple of 64.
 * Replaces B_proj(x), C_proj(x) and the scan of
 * QuaternionMamba2Block._ssm_forward, models/quaternion_mamba2_block.py:186-191
 * and 214-228 (the projections: layers/quaternion_linear.py:145-161).
 */
typedef struct mqc_bc_proj_scan_args {
  int64_t batch, seq_len, channels, d_state, in_features;
  int32_t dtype;
  float eps;
  const void* x;
  const void* w_b;
  const void* w_c;
  const void* delta;
  const void* s;
  const float* lambda_;
  const float* dskip;
  int64_t dskip_sd;
  const float* h0;
  float* hT;
  void* y;
  int32_t* status;
  int64_t wait_poll_limit;
} mqc_bc_proj_scan_args;

MQC_API int mqc_bc_proj_scan_fwd(const mqc_bc_proj_scan_args* args, void* stream);

MQC_API size_t mqc_ssm_scan_fwd_chunked_workspace_size(int64_t batch, int64_t channels,
                                                       int64_t d_state, int64_t nchunks);
MQC_API int mqc_ssm_scan_fwd_chunked(const mqc_ssm_scan_args* args, int64_t nchunks,
                                     void* workspace, size_t workspace_bytes, void* stream);

/* Summary of a time range for a time-sharded scan. The scan is affine in the
 * state, so over the steps in `args` it is h -> P (x) h + E, where
 *   P = q_{T-1} (x) ... (x) q_0 (the step operators, later on the left);
 *   E = the final state reached from h = 0.
 * Writes P and E [B, D, N, 4] fp32 and no y. args->h0, hT and ckpt must be NULL;
 * args->y is ignored. With nchunks > 1 the range is scanned in nchunks
 * time-parallel chunks whose summaries are then composed; that needs a
 * caller-owned workspace of mqc_ssm_scan_fwd_summary_workspace_size(...)
 * bytes. No counterpart in the reference, which has no multi-GPU path; it is
 * the exchange step of the time-sharded scan of QuaternionMamba2Block._ssm_forward
 * (models/quaternion_mamba2_block.py:214-228). */
MQC_API size_t mqc_ssm_scan_fwd_summary_workspace_size(int64_t batch, int64_t channels,
                                                       int64_t d_state, int64_t nchunks);
MQC_API int mqc_ssm_scan_fwd_summary(const mqc_ssm_scan_args* args, int64_t nchunks, float* P,
                                     float* E, void* workspace, size_t workspace_bytes,
                                     void* stream);

/* The scan of a range whose chunk summaries are already in `workspace`: a
 * mqc_ssm_scan_fwd_summary call with the same inputs and nchunks filled it.
 * Runs only the carry from args->h0 and the full pass, so a time-sharded rank
 * scans its range with one state-only pass in total, not two. Same arguments
 * and results as mqc_ssm_scan_fwd_chunked. No counterpart in the reference. */
MQC_API int mqc_ssm_scan_fwd_chunked_resume(const mqc_ssm_scan_args* args, int64_t nchunks,
                                            void* workspace, size_t workspace_bytes,
                                            void* stream);

/* Start states of consecutive time segments from their summaries
 * (mqc_ssm_scan_fwd_summary):
 *   H_0 = h0 (zero if NULL);  H_{s+1} = P_s (x) H_s + E_s;
 *   hin[s] = H_s;  hT = H_segments.
 * P, E, hin [segments, batch, lanes, 4] fp32 (segment-major, as an all-gather
 * of per-rank summaries lays them out); h0, hT [batch, lanes, 4] fp32; hin or
 * hT may be NULL. No counterpart in the reference. */
MQC_API int mqc_ssm_scan_carry(const float* P, const float* E, const float* h0, float* hin,
                               float* hT, int64_t segments, int64_t batch, int64_t lanes,
                               void* stream);

/* ---- peer-memory exchange between the ranks of one node ------------------- */
/* No counterpart in the reference, which has no multi-GPU code. Used by the
 * channel-sharded scan to write each rank's output channels straight into every
 * rank's full output over NVLink (plain stores to peer memory; no multicast). */

#define MQC_PEER_HANDLE_BYTES 64

/* cudaMalloc(bytes) on the current device, with the 64-byte IPC handle another
 * process of this node passes to mqc_peer_open to address the same memory. */
MQC_API int mqc_peer_alloc(size_t bytes, void** ptr, void* handle);
MQC_API int mqc_peer_free(void* ptr);
/* Maps a peer's buffer (from its mqc_peer_alloc handle) into this process. */
MQC_API int mqc_peer_open(const void* handle, void** ptr);
MQC_API int mqc_peer_close(void* ptr);

/* mqc_ssm_scan_fwd_chunked for one channel shard of a sequence split over the
 * ranks by channel, with the exchange of y fused into the scan: the kernel that
 * produces y stores every value into each of the npeer (<= 8) outputs
 * ypeer[r] [batch, seq_len, ch_total, 4] (dtype; this GPU's and the other
 * ranks' buffers from mqc_peer_alloc / mqc_peer_open) at channels ch_off ..
 * ch_off + channels - 1, so y crosses NVLink while the scan runs and lands in
 * its final layout. args->y is ignored. Channel-shared B/C, the fused Cayley
 * form, a per-channel skip weight, seq_len / nchunks > 8. The kernel ends with
 * a system-scope fence; ranks that synchronise with its completion (e.g. a
 * collective ordered after it) see the data. */
MQC_API int mqc_ssm_scan_fwd_chunked_peer(const mqc_ssm_scan_args* args, int64_t nchunks,
                                          void* workspace, size_t workspace_bytes,
                                          void* const* ypeer, int npeer, int64_t ch_total,
                                          int64_t ch_off, void* stream);

/* mqc_ssm_scan_fwd_chunked_peer with one multicast output: ymc is the multicast
 * address of a [batch, seq_len, ch_total, 4] buffer (dtype) bound on every rank
 * (an NVLink SHARP multicast object, e.g. the multicast_ptr of a torch
 * symmetric-memory tensor). The kernel gathers each y quaternion on one lane and
 * stores it once with multimem.st; NVSwitch writes it into every rank's buffer,
 * so one store replaces one per rank. d_state in (16, 256]; the other rules are
 * those of mqc_ssm_scan_fwd_chunked_peer. No counterpart in the reference, which
 * has no multi-GPU code. */
MQC_API int mqc_ssm_scan_fwd_chunked_multicast(const mqc_ssm_scan_args* args, int64_t nchunks,
                                               void* workspace, size_t workspace_bytes,
                                               void* ymc, int64_t ch_total, int64_t ch_off,
                                               void* stream);

/* Copies a time segment of this rank's channel shard, src [batch, seg_len,
 * ch_local, 4] (dtype, contiguous), into rows t_off .. t_off+seg_len-1 and
 * channels ch_off .. ch_off+ch_local-1 of each of the ndst (<= 8) outputs
 * dsts[r] [batch, seq_total, ch_total, 4] -- local or peer memory. Ends with a
 * system-scope fence, so a rank that synchronises with this kernel's
 * completion (e.g. through a collective ordered after it) sees the data. */
MQC_API int mqc_channel_push(const void* src, void* const* dsts, int ndst, int64_t batch,
                             int64_t seg_len, int64_t ch_local, int64_t ch_total, int64_t ch_off,
                             int64_t t_off, int64_t seq_total, int dtype, void* stream);

/*
 * Backward of mqc_ssm_scan_fwd without Q_GIVEN (the fused Cayley form). The
 * reference has no GPU backward (its Triton kernels are not differentiable);
 * this computes the gradients torch autograd takes through the reference's CPU
 * composition (block._ssm_forward lines 214-228 with cayley_discretization_reference
 * and the ssm_step_reference loop). Per (b, d, n), in reverse time:
 *   lambda_t = conj(C_t) (x) dy_t + conj(q_{t+1}) (x) lambda_{t+1}   (+ dhT at t = T-1)
 *   dq_t = lambda_t (x) conj(h_{t-1});  dz_t = (dq/dz)^T dq_t;  z_t = delta_t Lambda
 *   ddelta_t = sum_n <dz_t, Lambda>;     dLambda += delta_t dz_t
 *   dB_t = lambda_t (x) conj(S_t);       dS_t = sum_n conj(B_t) (x) lambda_t + D dy_t
 *   dC_t = dy_t (x) conj(h_t);           dh0 = conj(q_0) (x) lambda_0
 * States are recomputed from the forward's checkpoints (MQC_SSM_CKPT_EVERY).
 * Inputs as in mqc_ssm_scan_args; dy [B,T,D,4] dtype; dhT [B,D,N,4] fp32 or NULL.
 * Outputs: ddelta [B,T,D] dtype; dlambda_part [B,D,N,4] fp32 (per-batch partial
 * sums, to be summed over B); ds like s (dtype); dh0 [B,D,N,4] fp32 or NULL;
 * dBm/dCm: with BC_SHARED fp32 [B,T,N,4] accumulators the caller zero-fills,
 * otherwise dtype [B,T,D,N,4]. The gradient of the skip weight D is
 * sum <dy, S>, which needs no scan. Shared dB/dC are summed over channels with
 * float atomics, so their low bits can vary from run to run.
 */
typedef struct mqc_ssm_scan_bwd_args {
  int64_t batch, seq_len, channels, d_state;
  int32_t dtype;
  int32_t flags; /* MQC_SSM_BC_SHARED, MQC_SSM_S_REAL */
  float eps;
  int32_t ckpt_every;
  const void* delta;
  const float* lambda_;
  const void* Bm;
  const void* Cm;
  const void* s;
  const float* dskip;
  int64_t dskip_sb, dskip_st, dskip_sd;
  const float* h0;
  const float* ckpt;
  const void* dy;
  const float* dhT;
  void* ddelta;
  float* dlambda_part;
  void* dBm;
  void* dCm;
  void* ds;
  float* dh0;
} mqc_ssm_scan_bwd_args;

MQC_API int mqc_ssm_scan_bwd(const mqc_ssm_scan_bwd_args* args, void* stream);

/* One step with explicit q: h_new = q (x) h_prev + B (x) S, y = sum_n C (x) h_new + D*S.
 * q, Bm, Cm, h_prev, h_new [B,D,N,4]; S [B,D,4]; dskip [B,D] fp32; y [B,D,4].
 * q, Bm, Cm, S, y in dtype; h_prev, h_new fp32.
 * Replaces ssm_step_fused(q, B, S, C, D, h_prev), ssm_fused.py:258-337. */
MQC_API int mqc_ssm_step(const void* q, const void* Bm, const void* S, const void* Cm,
                 const float* dskip, const float* h_prev, float* h_new, void* y, int64_t batch,
                 int64_t channels, int64_t d_state, int dtype, void* stream);

/* ---- quaternion LayerNorm: mambaqc/kernels/quaternion_norm.py -------------- */

#define MQC_QLN_PADDED_COMPAT 0x1 /* reproduce the reference Triton kernel's padded lanes */

/* Row-wise norm LayerNorm over d_model quaternions for `rows` rows:
 *   n = sqrt(|q|^2 + eps); mu, var = mean, biased variance of n over the row;
 *   out = gamma * (n - mu)/sqrt(var + eps) * q/(n + eps) + beta.
 * q, out [rows, d_model, 4] dtype; gamma [d_model], beta [d_model, 4] fp32;
 * mean, rstd [rows] fp32 (saved for the backward) or NULL.
 * Replaces quaternion_layer_norm_fused, quaternion_norm.py:119-174 (and the
 * forward of QuaternionLayerNorm, :177-215). */
MQC_API int mqc_qln_fwd(const void* q, const float* gamma, const float* beta, void* out, float* mean,
                float* rstd, int64_t rows, int64_t d_model, float eps, int flags, int dtype,
                void* stream);

/* LayerNorm fused into the output projection that follows it in the block:
 *   out[r, :] = LN(q)[r, :] @ weight^T (+ bias)
 * with LN as mqc_qln_fwd (exact form). q [rows, d_model, 4], weight
 * [out_features, 4 d_model], bias [out_features] or NULL, out [rows,
 * out_features]: bf16; gamma [d_model], beta [d_model, 4] fp32; mean, rstd
 * [rows] fp32 receive the row statistics (for the backward). The normalised
 * activations are never written: one pass reads q for the row statistics, then
 * a tcgen05 GEMM normalises each q tile in shared memory as its operand.
 * d_model a multiple of 16 (<= 4096); q, weight, beta 16-byte aligned. `status`
 * (device int, may be NULL) receives MQC_DEVICE_STATUS_TIMEOUT if a bounded
 * wait gives up. Replaces self.out_proj(self.norm(y_quat)),
 * models/quaternion_mamba2_block.py:154-157. */
MQC_API int mqc_qln_linear_fwd(const void* q, const float* gamma, const float* beta,
                               const void* weight, const void* bias, void* out, float* mean,
                               float* rstd, int64_t rows, int64_t d_model, int64_t out_features,
                               float eps, int* status, void* stream);

/* Bytes of workspace mqc_qln_bwd needs for `rows` x `d_model` (0 if nothing to do). */
MQC_API size_t mqc_qln_bwd_workspace_size(int64_t rows, int64_t d_model);

/* Backward of mqc_qln_fwd (exact form, not the padded-compat one): from q, gamma,
 * dout = dL/dout and the saved mean/rstd, writes dq [rows, d_model, 4] (dtype) and
 * the parameter gradients dgamma [d_model], dbeta [d_model, 4] (fp32, summed over
 * rows in a fixed order). `workspace` (16-byte aligned, caller-owned) holds
 * per-CTA partial sums. The reference has no GPU backward; this is the gradient
 * torch autograd takes through quaternion_layer_norm_reference,
 * quaternion_norm.py:219-245. */
MQC_API int mqc_qln_bwd(const void* q, const float* gamma, const void* dout, const float* mean,
                const float* rstd, void* dq, float* dgamma, float* dbeta, void* workspace,
                size_t workspace_bytes, int64_t rows, int64_t d_model, float eps, int dtype,
                void* stream);

/* ---- block glue around the scan: models/quaternion_mamba2_block.py --------- */

/* Causal depthwise conv + bias + SiLU of the block's inner signal, in one pass:
 *   a[b,t,d] = bias[d] + sum_k weight[d,k] * x[b, t-(K-1)+k, d]   (x = 0 before t = 0)
 *   out[b,t,d] = a * sigmoid(a)
 * x rows of `channels` elements at a row stride of `x_row_stride` elements (the
 * first half of the in_proj output [B,T,2*d_inner] is read in place); out
 * [B,T,channels] contiguous, same dtype. weight [channels, K] fp32 (the
 * nn.Conv1d weight [channels,1,K]), bias [channels] fp32 or NULL; 1 <= K <= 8.
 * Replaces CausalConv1d.forward (layers/causal_conv1d.py:68-91) followed by
 * F.silu, block lines models/quaternion_mamba2_block.py:140-144. */
MQC_API int mqc_conv_silu_fwd(const void* x, int64_t x_row_stride, const float* weight,
                              const float* bias, void* out, int64_t batch, int64_t seq_len,
                              int64_t channels, int64_t kernel_size, int dtype, void* stream);

/* Bytes of workspace mqc_conv_silu_bwd needs (per-block partial sums of the
 * weight and bias gradients; 0 if nothing to do). */
MQC_API size_t mqc_conv_silu_bwd_workspace_size(int64_t batch, int64_t seq_len, int64_t channels,
                                                int64_t kernel_size);

/* Backward of mqc_conv_silu_fwd (the pre-activation is recomputed from x):
 * dx [B,T,channels] contiguous (dtype); dweight [channels,K] and dbias
 * [channels] fp32, summed over (b,t) in a fixed order (dbias may be NULL).
 * `workspace`: caller-owned, 16-byte aligned. The reference has no GPU backward;
 * this is the gradient autograd takes through conv1d + silu. */
MQC_API int mqc_conv_silu_bwd(const void* x, int64_t x_row_stride, const float* weight,
                              const float* bias, const void* dout, void* dx, float* dweight,
                              float* dbias, int64_t batch, int64_t seq_len, int64_t channels,
                              int64_t kernel_size, int dtype, void* workspace,
                              size_t workspace_bytes, void* stream);

/* The scan's inputs from the dt_proj and gate_proj outputs, in one pass:
 *   delta = softplus(u)  (torch's threshold 20: u above it passes through)
 *   s     = sigmoid(gate) * x
 * u, gate: `rows` rows of `channels` at their own row strides (elements); x, delta,
 * s [rows, channels] contiguous; one dtype. Replaces block lines
 * models/quaternion_mamba2_block.py:183 and 197-198. */
MQC_API int mqc_scan_inputs_fwd(const void* u, int64_t u_row_stride, const void* gate,
                                int64_t gate_row_stride, const void* x, void* delta, void* s,
                                int64_t rows, int64_t channels, int dtype, void* stream);

/* Backward of mqc_scan_inputs_fwd: du = ddelta * sigmoid(u) (ddelta where u > 20),
 * dgate = ds * x * sigmoid(gate) * (1 - sigmoid(gate)), dx = ds * sigmoid(gate).
 * ddelta or ds may be NULL (no gradient: zero). du, dgate, dx [rows, channels]
 * contiguous. */
MQC_API int mqc_scan_inputs_bwd(const void* u, int64_t u_row_stride, const void* gate,
                                int64_t gate_row_stride, const void* x, const void* ddelta,
                                const void* ds, void* du, void* dgate, void* dx, int64_t rows,
                                int64_t channels, int dtype, void* stream);

/* Output gate and residual of the block: out = x + sigmoid(z) * y.
 * x, y, out [rows, cols] contiguous; z `cols` elements per row at a row stride of
 * `z_row_stride` elements (the second half of the in_proj output, read in place);
 * one dtype. Replaces block lines models/quaternion_mamba2_block.py:154-164. */
MQC_API int mqc_gate_residual_fwd(const void* x, const void* z, int64_t z_row_stride,
                                  const void* y, void* out, int64_t rows, int64_t cols, int dtype,
                                  void* stream);

/* Backward of mqc_gate_residual_fwd: dz = dout * y * sigmoid(z) * (1 - sigmoid(z)),
 * dy = dout * sigmoid(z) (dx = dout needs no kernel). dz, dy [rows, cols] contiguous. */
MQC_API int mqc_gate_residual_bwd(const void* z, int64_t z_row_stride, const void* y,
                                  const void* dout, void* dz, void* dy, int64_t rows, int64_t cols,
                                  int dtype, void* stream);

/* ---- diagnostics ---------------------------------------------------------- */

/* Launches a pure FP32 FMA-chain kernel (no memory traffic) that keeps every SM's
 * FP32 pipes busy for `iters` iterations and stores the number of FMAs it issues
 * in *fmas_per_launch. Timing it gives the FP32 peak that the scan kernels'
 * FP32-issue roofline is measured against. No counterpart in the reference.
 * `out`: one device float, written only in a case that never occurs. */
MQC_API int mqc_probe_fp32_fma(float* out, int64_t iters, int64_t* fmas_per_launch, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MAMBAQC_B200_H_ */
