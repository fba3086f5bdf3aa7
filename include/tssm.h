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
 *   initial state); h_last [Bsz,H,P,N] f32 or NULL.
 * P = 64 and N in {64, 128}; all tensors contiguous; x, B, C, y 16-byte
 * aligned.  Device-side waits are bounded: a wait that gives up is reported
 * by tssm_check_device_status.
 */
int tssm_multihead_ssd(const void* x, const void* dt, const void* A_log, const void* B,
                       const void* C, const void* Dskip, void* y, const void* h0, void* h_last,
                       int64_t Bsz, int64_t L, int64_t H, int64_t P, int64_t N, int bdisc,
                       tssm_stream_t stream);

/*
 * Synchronise `stream` and report (then clear) this device's status word:
 * TSSM_ERR_TIMEOUT if a kernel's bounded device-side wait gave up since the
 * last check, else TSSM_OK.  No reference counterpart (the reference has no
 * device-side waits).
 */
int tssm_check_device_status(tssm_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* TSSM_H_ */
