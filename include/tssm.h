/*
 * tssm_b200 — C ABI of the B200 (sm_100a) selective-SSM hot path.
 *
 * Drop-in replacement for the kernels of Triton-SSM.  Every entry point takes
 * plain device pointers, element counts and element strides (the last
 * dimension of every tensor is contiguous, as the reference assumes), a dtype
 * code and a CUDA stream, launches asynchronously on that stream, and returns
 * a tssm_status.  Nothing here allocates device memory; outputs are
 * caller-owned, exactly as the reference's kernels write into caller-owned
 * tensors.  Entry points are stateless and may be called from several host
 * threads on different streams.
 *
 * Each declaration names the reference interface it replaces (file:line in
 * the Triton-SSM sources).
 */
#ifndef TSSM_H_
#define TSSM_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* tssm_stream_t; /* == cudaStream_t */

enum tssm_dtype {
  TSSM_F32 = 0,
  TSSM_BF16 = 1,
  TSSM_F16 = 2,
  TSSM_U8 = 3
};

enum tssm_status {
  TSSM_OK = 0,
  TSSM_ERR_INVALID = 1,     /* bad shape / stride / dtype / alignment argument */
  TSSM_ERR_UNSUPPORTED = 2, /* a valid configuration this build does not handle */
  TSSM_ERR_CUDA = 3,        /* a CUDA runtime error (launch failure, ...) */
  TSSM_ERR_TIMEOUT = 4      /* a bounded device-side wait gave up */
};

/* Library version (major*10000 + minor*100 + patch). */
int tssm_version(void);
/* Static text for a status code. */
const char* tssm_status_string(int status);
/* Detail message of the last failing call on this host thread ("" if none). */
const char* tssm_last_error(void);

/*
 * ZOH discretisation.  Replaces zoh_discretize_diag_kernel
 * (discretize_kernel.py:15-57) for io_dtype = TSSM_F32 and
 * zoh_discretize_diag_bf16_kernel (discretize_kernel.py:60-94) for
 * io_dtype = TSSM_BF16.
 *   A_log [H] f32 (log(-a)); B [Bsz,T,H] io; dt [Bsz,T] f32;
 *   Abar, Bbar [Bsz,T,H] io.
 *   Abar = exp(dt*a), Bbar = expm1*(dt*a)/(a+1e-12)*B with a = -exp(A_log).
 * Strides are in elements; the H stride is 1.
 */
int tssm_zoh_discretize(const void* A_log, const void* B, const void* dt, void* Abar, void* Bbar,
                        int64_t Bsz, int64_t T, int64_t H,
                        int64_t stride_Bb, int64_t stride_Bt,
                        int64_t stride_db, int64_t stride_dt,
                        int64_t stride_ab, int64_t stride_at,
                        int64_t stride_bb, int64_t stride_bt,
                        int io_dtype, tssm_stream_t stream);

/*
 * Diagonal selective scan.  Replaces ssm_forward (ssm_scan.py:239-264), i.e.
 * its four launches ssm_fwd_local_kernel / ssm_carry_scan_kernel /
 * ssm_fwd_apply_kernel / ssm_output_kernel (ssm_scan.py:17-124), with one
 * launch and no intermediate buffers.
 *   u, A, B, C [Bsz,L,H] contiguous (dtype); D [H] (dtype);
 *   y [Bsz,L,H] (dtype); h [Bsz,L,H] (dtype) or NULL to skip storing states.
 *   h_t = A_t*h_{t-1} + B_t*u_t, y_t = C_t*h_t + D*u_t; math in f32.
 * dtype: TSSM_F32 or TSSM_BF16.
 */
int tssm_ssm_forward(const void* u, const void* A, const void* B, const void* C, const void* D,
                     void* y, void* h, int64_t Bsz, int64_t L, int64_t H,
                     int dtype, tssm_stream_t stream);

/*
 * The diagonal scan with the mean-pooled logit head fused into its epilogue:
 * the composition ssm_forward (ssm_scan.py:239-264) -> mean_pool_logit_kernel
 * (streaming_inference_kernel.py:159-194) applied to y, without re-reading y.
 *   Arguments as tssm_ssm_forward, plus poolW [H] f32, pool_bias [1] f32 and
 *   pool_out [Bsz] f32: pool_out[b] = sum_{t,h} poolW[h] y[b,t,h] / (L*H + 1e-9)
 *   + pool_bias[0] (y as stored, in dtype).  pool_out is summed with float
 *   atomics, so its last bits may vary between runs.
 */
int tssm_ssm_forward_pool(const void* u, const void* A, const void* B, const void* C, const void* D,
                          void* y, void* h, const void* poolW, const void* pool_bias, void* pool_out,
                          int64_t Bsz, int64_t L, int64_t H, int dtype, tssm_stream_t stream);

/*
 * Mean-pooled logit head.  Replaces mean_pool_logit_kernel
 * (streaming_inference_kernel.py:159-194).
 *   x [Bsz,T,H] (dtype TSSM_F32 or TSSM_BF16), W [H] f32, bias [1] f32 ->
 *   out [Bsz] f32 = sum_{t,h} W[h] x[b,t,h] / (T*H + 1e-9) + bias[0].
 *   Contiguous.  Summed with float atomics (last bits may vary between runs).
 */
int tssm_mean_pool_logit(const void* x, const void* W, const void* bias, void* out,
                         int64_t Bsz, int64_t T, int64_t H, int dtype, tssm_stream_t stream);

/*
 * Backward of the diagonal scan.  Replaces ssm_backward (ssm_scan.py:267-289),
 * i.e. ssm_bwd_local_kernel / ssm_bwd_carry_scan_kernel / ssm_bwd_apply_kernel
 * (ssm_scan.py:127-231), with one launch and no intermediate buffers.
 *   u, A, B, C, h (forward states), dY [Bsz,L,H] contiguous (dtype);
 *   du, dA, dB, dC [Bsz,L,H] (dtype), written.
 *   dH_t = C_t*dY_t + A_{t+1}*dH_{t+1}; du = B*dH, dA = h_{t-1}*dH,
 *   dB = u*dH, dC = dY*h.  As in the reference, D is a constant: no dD and
 *   no D*dY term in du.  Math in f32.  dtype: TSSM_F32 or TSSM_BF16.
 */
int tssm_ssm_backward(const void* u, const void* A, const void* B, const void* C, const void* h,
                      const void* dY, void* du, void* dA, void* dB, void* dC,
                      int64_t Bsz, int64_t L, int64_t H, int dtype, tssm_stream_t stream);

/*
 * Backward of the ZOH discretisation.  Replaces zoh_discretize_bwd_kernel
 * (discretize_kernel.py:97-162).
 *   A_log [H]; B, Abar, dAbar, dBbar [Bsz,T,H]; dt [Bsz,T]; all f32, contiguous.
 *   dA_log [H], dB [Bsz,T,H], ddt [Bsz,T] f32, written.
 *   ddt is the full sum over H (the reference's per-block store/atomic mix at
 *   :159-162 races); dA_log is overwritten with the sum over (b, t) -- the
 *   reference accumulates into a buffer its caller must zero.  dA_log is
 *   summed with float atomics, so its last bits may vary between runs.
 */
int tssm_zoh_discretize_bwd(const void* A_log, const void* B, const void* dt, const void* Abar,
                            const void* dAbar, const void* dBbar, void* dA_log, void* dB, void* ddt,
                            int64_t Bsz, int64_t T, int64_t H, tssm_stream_t stream);

/*
 * Delta-t projection.  Replaces dt_project_softplus_kernel
 * (discretize_kernel.py:165-213), which does not compile in the reference.
 *   dt_raw [Bsz,T,R] f32, W [R,H] f32, bias [H] f32 -> dt_out [Bsz,T,H] f32:
 *   dt = clamp(log(1 + exp(dt_raw.W + bias)), dt_min, dt_max).  R <= 256.
 */
int tssm_dt_project_softplus(const void* dt_raw, const void* W, const void* bias, void* dt_out,
                             int64_t Bsz, int64_t T, int64_t H, int64_t R, double dt_min, double dt_max,
                             tssm_stream_t stream);

/*
 * The delta-t projection fused into the ZOH discretisation with one dt per
 * (b, t, h): no reference counterpart as one kernel; it composes
 * dt_project_softplus_kernel (discretize_kernel.py:165-213) with the
 * arithmetic of zoh_discretize_diag_kernel (:38-54) at a per-channel dt.
 *   A_log [H], B [Bsz,T,H], dt_raw [Bsz,T,R], W [R,H], bias [H]; all f32.
 *   Abar, Bbar [Bsz,T,H] f32 out; dt_out [Bsz,T,H] f32 or NULL (not stored).
 */
int tssm_zoh_discretize_dtproj(const void* A_log, const void* B, const void* dt_raw, const void* W,
                               const void* bias, void* Abar, void* Bbar, void* dt_out,
                               int64_t Bsz, int64_t T, int64_t H, int64_t R, double dt_min, double dt_max,
                               tssm_stream_t stream);

/*
 * Fused ZOH discretisation + diagonal scan + readout over an N-wide state per
 * channel: the composition zoh_discretize_diag_kernel (discretize_kernel.py:
 * 15-57) -> ssm_forward (ssm_scan.py:239-264) over H' = D*N channels with the
 * readout summed over N, in one launch without the [Bsz,L,D*N] intermediates.
 *   x [Bsz,L,Dm] f32; dt [Bsz,L] f32; A_log [Dm,N] f32; B, C [Bsz,L,N] f32;
 *   Dskip [Dm] f32; y [Bsz,L,Dm] f32; h_last [Bsz,Dm,N] f32 or NULL.
 * All contiguous.  N <= 32.
 */
int tssm_selective_scan(const void* x, const void* dt, const void* A_log, const void* B,
                        const void* C, const void* Dskip, void* y, void* h_last,
                        int64_t Bsz, int64_t L, int64_t Dm, int64_t N, tssm_stream_t stream);

/*
 * Streaming in-place step with parameters shared by all rows.  Replaces
 * streaming_ssm_inplace_kernel (streaming_inference_kernel.py:6-37) for
 * dtype TSSM_F32 and streaming_ssm_inplace_bf16_kernel (:40-71) for
 * TSSM_BF16 (state stored back in bf16, as there).
 *   vhat, h, C, y [Bsz,H] (row strides given); Abar, Bbar, D [H].
 *   h <- Abar*h + Bbar*vhat (in place); y = C*h + D*vhat.
 */
int tssm_streaming_inplace(const void* vhat, void* h, const void* Abar, const void* Bbar,
                           const void* C, const void* D, void* y, int64_t Bsz, int64_t H,
                           int64_t stride_vb, int64_t stride_hb, int64_t stride_cb,
                           int dtype, tssm_stream_t stream);

/*
 * Streaming single step with a per-stream dt and an outer-product f32 state
 * resident in HBM: the composition zoh_discretize_diag_kernel
 * (discretize_kernel.py:15-57) -> streaming_ssm_inplace_kernel
 * (streaming_inference_kernel.py:6-37) over H*P*N channels with the readout
 * summed over N, in one pass over the state.
 *   x [S,Hh,P] io; dt [S] f32; h [S,Hh,P,N] f32 (in place); A_log [Hh] f32;
 *   B, C [S,Hh,N] io; Dskip [Hh,P] f32; y [S,Hh,P] io.  All contiguous.
 *   io_dtype: TSSM_BF16 or TSSM_F32.  N a power of two in [4, 128].
 */
int tssm_streaming_step(const void* x, const void* dt, void* h, const void* A_log,
                        const void* B, const void* C, const void* Dskip, void* y,
                        int64_t S, int64_t Hh, int64_t P, int64_t N,
                        int io_dtype, tssm_stream_t stream);

/*
 * Streaming ring-buffer ingest + forward fill + one step.  Replaces
 * streaming_interp_then_ssm_kernel (streaming_inference_kernel.py:74-156),
 * without its ring_head race (:115-117): one CTA owns each stream.
 *   ring_V, ring_M [Bsz,K+1,H] f32, ring_tau [Bsz,K+1] f32, ring_head [Bsz]
 *   int32 (all updated in place); v_new, m_new [Bsz,H] f32; tau_new [Bsz];
 *   h [Bsz,H] f32 in place; Abar, Bbar, Dskip [H]; C [Bsz,H]; y [Bsz,H] out.
 * The event goes to slot (head+1) % (K+1); per block_h-wide feature tile the
 * nearest older slot whose mask sum exceeds 0.5 supplies vhat when the
 * event's own tile mask sum is below 0.5; then h <- Abar h + Bbar vhat,
 * y = C h + Dskip vhat.  All contiguous.  K+1 <= 64.
 */
int tssm_ring_ingest_step(void* ring_V, void* ring_M, void* ring_tau, void* ring_head,
                          const void* v_new, const void* m_new, const void* tau_new, void* h,
                          const void* Abar, const void* Bbar, const void* C, const void* Dskip,
                          void* y, int64_t Bsz, int64_t H, int64_t K, int64_t block_h,
                          tssm_stream_t stream);

/*
 * Multi-head chunked scan with an outer-product state h[b,h,p,n] on tcgen05
 * tensor cores.  Replaces the multi-head chunked associative scan
 * multihead_ssm_fwd_local_kernel / multihead_ssm_carry_scan_kernel /
 * multihead_ssm_output_kernel (multihead_ssm_kernel.py:19-187) for the
 * B*L*H*P*N-state workload, in one launch:
 *   h_t = exp(dt_t*A_h) h_{t-1} + beta_t x_t (x) B_t ;  y_t[p] = sum_n C_t[n] h_t[p,n] + D[p] x_t[p]
 *   beta_t = dt_t (bdisc 0, Euler, multihead_ssm_kernel.py:73) or
 *            expm1*(dt_t*a)/(a+1e-12) (bdisc 1, ZOH, discretize_kernel.py:50-54), a = -exp(A_log[h]).
 *   x [Bsz,L,H*P] bf16; dt [Bsz,L,H] f32; A_log [H] f32; B, C [Bsz,L,H,N] bf16;
 *   Dskip [H*P] f32; y [Bsz,L,H*P] bf16; h0 [Bsz,H,P,N] f32 or NULL (zero
 *   initial state); h_last [Bsz,H,P,N] f32 or NULL; decay_log2 [Bsz,H] f32 or
 *   NULL: log2 of the whole-sequence decay, sum_t dt_t*A_h*log2(e) (used to
 *   chain sequence slices, see tssm_ssd_carry_fixup).
 * P = 64 and N in {64, 128}; all tensors contiguous; x, B, C, y 16-byte
 * aligned.  Device-side waits are bounded: a wait that gives up is reported
 * by tssm_check_device_status.
 */
int tssm_multihead_ssd(const void* x, const void* dt, const void* A_log, const void* B,
                       const void* C, const void* Dskip, void* y, const void* h0, void* h_last,
                       void* decay_log2, int64_t Bsz, int64_t L, int64_t H, int64_t P, int64_t N,
                       int bdisc, tssm_stream_t stream);

/*
 * Time-aware interpolation of irregular observations.  Replaces
 * fused_time_aware_interp_kernel (fused_interp_kernel.py:9-100) for v_dtype
 * TSSM_F32, fused_interp_bf16_kernel (:103-181) for TSSM_BF16 and
 * fused_interp_fp16_kernel (:186-257) for TSSM_F16, with the same
 * neighbour search (per tile of FTILE features, K candidates each way), weights
 * and priority.
 *   V, Vhat [Bsz,T,F] (v_dtype); M [Bsz,T,F] (m_dtype TSSM_U8 or TSSM_F32,
 *   observed where the value is > 0.5); tau [Bsz,T] f32 (t contiguous).
 *   K in [1,64]; FTILE in [1,4096].
 */
int tssm_time_aware_interp(const void* V, const void* M, const void* tau, void* Vhat, int64_t Bsz,
                           int64_t T, int64_t F, int64_t stride_vb, int64_t stride_vt,
                           int64_t stride_mb, int64_t stride_mt, int64_t stride_tb,
                           int64_t stride_ob, int64_t stride_ot, int64_t K, int64_t FTILE,
                           int v_dtype, int m_dtype, tssm_stream_t stream);

/*
 * Interpolation at one time index fused with one SSM step.  Replaces
 * fused_interp_ssm_step_kernel (fused_ssm_interp.py:11-101):
 *   Vhat[:, t_cur] = interp(...);  h_out = Abar*h_in + Bbar*vhat.
 *   V, Vhat [Bsz,T,F] f32 (Vhat may be NULL); M [Bsz,T,F] (m_dtype);
 *   tau [Bsz,T] f32; Abar, Bbar [F] f32; h_in, h_out [Bsz,F] f32.
 */
int tssm_interp_ssm_step(const void* V, const void* M, const void* tau, const void* Abar,
                         const void* Bbar, const void* h_in, void* Vhat, void* h_out, int64_t Bsz,
                         int64_t T, int64_t F, int64_t stride_vb, int64_t stride_vt, int64_t stride_mb,
                         int64_t stride_mt, int64_t stride_tb, int64_t stride_ob, int64_t stride_ot,
                         int64_t stride_hib, int64_t stride_hob, int64_t t_cur, int64_t K,
                         int64_t FTILE, int m_dtype, tssm_stream_t stream);

/* Bytes of device workspace tssm_interp_ssm needs (tile flags + neighbour
 * table): 0 for an empty problem, -1 for sizes outside what tssm_interp_ssm
 * accepts (Bsz <= 65535, T <= 8192, Lq and Dm < 2^30, and a workspace below
 * 2^56 bytes). */
int64_t tssm_interp_ssm_workspace_size(int64_t Bsz, int64_t T, int64_t Dm, int64_t Lq, int64_t FTILE);

/*
 * Interpolation of irregular observations onto query times fused with an
 * N-state diagonal scan, all queries in one pass: the composition of
 * fused_time_aware_interp_kernel (fused_interp_kernel.py:9-100) and the step
 * of fused_interp_ssm_step_kernel (fused_ssm_interp.py:95-101) applied at
 * every query, with ZOH parameters per (b, d, n) (discretize_kernel.py:38-54)
 * and the readout y = sum_n C*h (+ D*vhat).  The interpolated values never
 * round-trip through HBM.
 *   V [Bsz,T,Dm] f32; M [Bsz,T,Dm] (m_dtype); tau [Bsz,T] f32 sorted;
 *   q [Bsz,Lq] f32 sorted query times, or NULL for index mode (queries are
 *   the observations themselves, Lq == T: the reference's own semantics);
 *   A_log, B, C [Dm,N] f32; Dskip [Dm] f32 or NULL; dt [Bsz] f32 (one
 *   discretisation step per row, e.g. the query spacing);
 *   y [Bsz,Lq,Dm] f32; h_last [Bsz,Dm,N] f32 or NULL; vhat [Bsz,Lq,Dm] or NULL.
 *   workspace: >= tssm_interp_ssm_workspace_size(...) bytes, 256-byte aligned.
 *   All contiguous.  N <= 64, T <= 8192.
 */
int tssm_interp_ssm(const void* V, const void* M, const void* tau, const void* q, const void* A_log,
                    const void* B, const void* C, const void* Dskip, const void* dt, void* y,
                    void* h_last, void* vhat, void* workspace, int64_t workspace_bytes, int64_t Bsz,
                    int64_t T, int64_t Dm, int64_t N, int64_t Lq, int64_t K, int64_t FTILE,
                    int m_dtype, tssm_stream_t stream);

/*
 * tssm_interp_ssm for callers that cannot allocate device memory when they
 * call in (for example a backend running inside another runtime's fixed
 * memory budget, or a latency-critical streaming loop that must not call
 * cudaMalloc): the same computation and arguments without `workspace`; the
 * scratch comes from an 8 MiB array compiled into the library, which every
 * GPU that loads the library holds until the process exits.  No counterpart
 * in the reference (the reference always allocates through PyTorch).
 *   Returns TSSM_ERR_INVALID, with a message, when the problem needs more than
 *   8 MiB of scratch (tssm_interp_ssm_workspace_size tells how much).
 *   The first call on a device looks up the array's device address; make that
 *   first call before any stream capture.
 *   All calls share the one array: calls that overlap on the GPU (other
 *   streams, other host threads) race on it and must be serialised by the
 *   caller.  Nothing in it needs clearing between calls.
 */
int tssm_interp_ssm_static_scratch(const void* V, const void* M, const void* tau, const void* q,
                                   const void* A_log, const void* B, const void* C, const void* Dskip,
                                   const void* dt, void* y, void* h_last, void* vhat, int64_t Bsz,
                                   int64_t T, int64_t Dm, int64_t N, int64_t Lq, int64_t K, int64_t FTILE,
                                   int m_dtype, tssm_stream_t stream);

/*
 * Sequence-parallel chaining of multi-head scan slices (config 4).  The
 * block-level carry scan of ssm_scan.py:53-98 (ssm_carry_scan_kernel +
 * ssm_fwd_apply_kernel) lifted from blocks of one GPU to slices of the sequence
 * held by different ranks: given every rank's final state S_all [nranks,Bsz,H,P,N]
 * f32 and whole-slice decay decay_log2_all [nranks,Bsz,H] f32 (both from
 * tssm_multihead_ssd with a zero initial state, gathered over ranks), rank
 * `rank` forms carry = sum_{j<rank} (prod_{j<k<rank} 2^d_k) S_j and adds its
 * effect, exp(A_h*cumdt(t)) * sum_n C[t,n] carry[p,n], to its own outputs
 * y [Bsz,L,H*P] bf16 (in place), for the leading tokens whose decay is not
 * exactly zero in f32.  C [Bsz,L,H,N] bf16 and dt [Bsz,L,H] f32 are the
 * rank's own slice.  P = 64, N in {64, 128}.  No-op on rank 0.
 */
int tssm_ssd_carry_fixup(const void* S_all, const void* decay_log2_all, int64_t rank, int64_t nranks,
                         const void* C, const void* dt, const void* A_log, void* y, int64_t Bsz,
                         int64_t L, int64_t H, int64_t P, int64_t N, tssm_stream_t stream);

/*
 * The same chaining for `pieces` equal in-device pieces of each sequence
 * (the block-level carry of ssm_scan.py:53-65 and :68-98 applied to pieces
 * rather than ranks).  Piece k of sequence b is sequence b*pieces + k of the
 * views x [Bsz*pieces, L/pieces, H*P] ... that one tssm_multihead_ssd call
 * scanned from zero states:
 *   S [Bsz*pieces,H,P,N] f32, decay_log2 [Bsz*pieces,H] f32: its outputs;
 *   C [Bsz,L,H,N] bf16, dt [Bsz,L,H] f32, A_log [H] f32: the whole sequences;
 *   y [Bsz,L,H*P] bf16: fixed in place for pieces 1 .. pieces-1.
 * L % pieces == 0; P = 64, N in {64, 128}.
 */
int tssm_ssd_carry_fixup_pieces(const void* S, const void* decay_log2, int64_t pieces, const void* C,
                                const void* dt, const void* A_log, void* y, int64_t Bsz, int64_t L, int64_t H,
                                int64_t P, int64_t N, tssm_stream_t stream);

/*
 * tssm_ssd_carry_fixup reading every rank's slice carry from the one packed
 * buffer that a single all-gather of each rank's [state | decay] produces
 * (the exchange step of the reference's carry scan, ssm_scan.py:53-65, done
 * across ranks):
 *   packed [nranks, Bsz*H*P*N + Bsz*H] f32: rank j's final state [Bsz,H,P,N]
 *   starts at packed + j*(Bsz*H*P*N + Bsz*H) and its decay_log2 [Bsz,H]
 *   follows it.
 * Otherwise as tssm_ssd_carry_fixup.  No-op on rank 0.
 */
int tssm_ssd_carry_fixup_packed(const void* packed, int64_t rank, int64_t nranks, const void* C,
                                const void* dt, const void* A_log, void* y, int64_t Bsz, int64_t L,
                                int64_t H, int64_t P, int64_t N, tssm_stream_t stream);

/*
 * Final state and decay of sequences scanned as `pieces` in-device pieces
 * (the carry scan of ssm_scan.py:53-65 over the pieces): with S, decay_log2
 * as in tssm_ssd_carry_fixup_pieces,
 *   state_out [Bsz,H,P,N] f32 = the pieces' states chained in order,
 *     c <- 2^{d_k} c + S_k for k = 0 .. pieces-1;
 *   decay_out [Bsz,H] f32 = sum_k d_k.
 * Either output may be NULL.  P*N a multiple of 4; S and state_out 16-byte
 * aligned.
 */
int tssm_ssd_pieces_final_state(const void* S, const void* decay_log2, int64_t pieces, void* state_out,
                                void* decay_out, int64_t Bsz, int64_t H, int64_t P, int64_t N,
                                tssm_stream_t stream);

/*
 * Multi-head scan with the reference's own diagonal state h[b,head,p].
 * Replaces multihead_ssm_fwd_local_kernel / multihead_ssm_carry_scan_kernel /
 * multihead_ssm_output_kernel (multihead_ssm_kernel.py:19-187, with the
 * scalar-index and item-assignment errors at :101 and :151 read as their
 * evident intent), in one launch:
 *   Abar = exp(dt[b,t,head]*a[head,p]), a = -exp(A_log[head,p]);
 *   h = Abar*h + (beta*B[b,t,head,p])*u[b,t,head*hd+p], beta = dt (bdisc 0) or
 *   the ZOH factor (bdisc 1);  y_head[t] = sum_p C*h + sum_p D*u, written to
 *   every position of the head's slice of y (:182-187).
 *   u, y [Bsz,L,n_heads*head_dim] (dtype f32 or bf16); A_log [n_heads,head_dim]
 *   f32; B, C [Bsz,L,n_heads,head_dim] (dtype); dt [Bsz,L,n_heads] f32;
 *   Dskip [n_heads*head_dim] f32.  All contiguous, head_dim <= 128.
 */
int tssm_multihead_diag(const void* u, const void* A_log, const void* B, const void* C, const void* dt,
                        const void* Dskip, void* y, int64_t Bsz, int64_t L, int64_t n_heads,
                        int64_t head_dim, int bdisc, int dtype, tssm_stream_t stream);

/*
 * The reference's blocked scans launch for launch, for callers that drive its
 * kernels individually (the fused entry points above are the fast path).
 * Intermediates keep the reference's layouts: loc_a, loc_x [Bsz,L,H] and
 * carry [2, rows, NBLK] (a-part first, then x-part; rows = Bsz*H), with
 * NBLK*BLK >= L; blocks past L hold the identity (1, 0).  f32, contiguous.
 *
 * tssm_ssm_fwd_local: ssm_fwd_local_kernel (ssm_scan.py:17-50).
 * tssm_ssm_bwd_local: ssm_bwd_local_kernel (ssm_scan.py:135-170), A_{t+1}
 *   and C*dY walked from the end of each block.
 * tssm_blocked_carry_scan: ssm_carry_scan_kernel (ssm_scan.py:53-65),
 *   multihead_ssm_carry_scan_kernel (multihead_ssm_kernel.py:105-117) with
 *   reverse = 0, ssm_bwd_carry_scan_kernel (ssm_scan.py:173-185) with
 *   reverse = 1: inclusive scan of each row's block carries in place.
 * tssm_ssm_fwd_apply: ssm_fwd_apply_kernel (ssm_scan.py:68-98).
 * tssm_ssm_output: ssm_output_kernel (ssm_scan.py:101-124), y = C*h + D*u.
 * tssm_ssm_bwd_apply: ssm_bwd_apply_kernel (ssm_scan.py:188-231).
 */
int tssm_ssm_fwd_local(const void* u, const void* A, const void* B, void* loc_a, void* loc_x, void* carry,
                       int64_t Bsz, int64_t L, int64_t H, int64_t BLK, int64_t NBLK, tssm_stream_t stream);
int tssm_ssm_bwd_local(const void* A, const void* C, const void* dY, void* loc_a, void* loc_dh, void* carry,
                       int64_t Bsz, int64_t L, int64_t H, int64_t BLK, int64_t NBLK, tssm_stream_t stream);
int tssm_blocked_carry_scan(void* carry, int64_t rows, int64_t NBLK, int reverse, tssm_stream_t stream);
int tssm_ssm_fwd_apply(const void* loc_a, const void* loc_x, const void* carry, void* h, int64_t Bsz,
                       int64_t L, int64_t H, int64_t BLK, int64_t NBLK, tssm_stream_t stream);
int tssm_ssm_output(const void* h, const void* C, const void* D, const void* u, void* y, int64_t Bsz,
                    int64_t L, int64_t H, tssm_stream_t stream);
int tssm_ssm_bwd_apply(const void* loc_a, const void* loc_dh, const void* carry, const void* u,
                       const void* A, const void* B, const void* h, const void* dY, void* du, void* dA,
                       void* dB, void* dC, int64_t Bsz, int64_t L, int64_t H, int64_t BLK, int64_t NBLK,
                       tssm_stream_t stream);

/*
 * The multi-head scan's own launches (multihead_ssm_kernel.py:19-187), read
 * with the intent of its scalar-index lines, for callers that drive them one
 * at a time:
 * tssm_mh_fwd_local: multihead_ssm_fwd_local_kernel (:19-102).  u
 *   [Bsz,L,n_heads*head_dim], B [Bsz,L,n_heads,head_dim] (dtype f32 or bf16,
 *   element strides as the reference passes them); A_log [n_heads,head_dim]
 *   f32 (row stride stride_alh); dt [Bsz,L,n_heads] f32.  Per row
 *   (b, head, p) and block: Abar = exp(dt*a), a = -exp(A_log), bx = (dt*B)*u;
 *   loc_a, loc_x [Bsz,L,n_heads,head_dim] f32; carry [2, Bsz*n_heads*head_dim,
 *   NBLK] f32.
 * tssm_mh_output: multihead_ssm_output_kernel (:120-187).  h = loc_a * x
 *   prefix + loc_x; y_head = sum_p C*h + sum_p D*u written to every position
 *   of the head's slice of y [Bsz,L,n_heads*head_dim] (dtype); D f32.
 * The carry scan between them is tssm_blocked_carry_scan (reverse = 0).
 */
int tssm_mh_fwd_local(const void* u, const void* A_log, const void* B, const void* dt, void* loc_a,
                      void* loc_x, void* carry, int64_t Bsz, int64_t L, int64_t n_heads, int64_t head_dim,
                      int64_t stride_ub, int64_t stride_ul, int64_t stride_alh, int64_t stride_Bb,
                      int64_t stride_Bl, int64_t stride_Bh, int64_t stride_db, int64_t stride_dl,
                      int64_t stride_dh, int64_t BLK, int64_t NBLK, int dtype, tssm_stream_t stream);
int tssm_mh_output(const void* loc_a, const void* loc_x, const void* carry, const void* C, const void* D,
                   const void* u, void* y, int64_t Bsz, int64_t L, int64_t n_heads, int64_t head_dim,
                   int64_t stride_ub, int64_t stride_ul, int64_t stride_Cb, int64_t stride_Cl,
                   int64_t stride_Ch, int64_t BLK, int64_t NBLK, int dtype, tssm_stream_t stream);

/*
 * Synchronise `stream` and report (then clear) this device's status word:
 * TSSM_ERR_TIMEOUT if a kernel's bounded device-side wait gave up since the
 * last check, else TSSM_OK.  No reference counterpart (the reference has no
 * device-side waits).
 */
int tssm_check_device_status(tssm_stream_t stream);

/*
 * Self-test of the failure path: launches one thread that waits, with the
 * bounded wait the pipelined kernels use, on an mbarrier phase that nothing
 * completes; after `timeout_ns` (at most 2 s) it gives up and sets the status
 * word, so the next tssm_check_device_status returns TSSM_ERR_TIMEOUT and the
 * context stays usable.  No reference counterpart.
 */
int tssm_selftest_wait_timeout(int64_t timeout_ns, tssm_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* TSSM_H_ */
