// Single-step streaming updates (replaces streaming_inference_kernel.py:6-71).
//
// streaming_step is a pure HBM stream over the f32 state [S,H,P,N]: each
// thread owns 4 consecutive n of one (s,h,p) row (one 128-bit evict-first
// load + store of state), N/4 threads cover a row, and the readout sum over
// n is a shuffle reduction inside that group.  Every thread handles two rows
// to keep two 128-bit state loads in flight.
#include "common.cuh"

namespace tssm {
namespace {

template <typename T>
__global__ void __launch_bounds__(256) streaming_inplace_kernel(
    const T* __restrict__ vhat, T* __restrict__ h, const T* __restrict__ Abar,
    const T* __restrict__ Bbar, const T* __restrict__ C, const T* __restrict__ D,
    T* __restrict__ y, int64_t Bsz, int64_t H, int64_t svb, int64_t shb, int64_t scb) {
  const int64_t n = Bsz * H;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const int64_t b = i / H;
    const int64_t k = i - b * H;
    const float v = ldf(vhat + b * svb + k);
    const float hp = ldf(h + b * shb + k);
    const float hn = ldf(Abar + k) * hp + ldf(Bbar + k) * v;          // :33
    const float yt = ldf(C + b * scb + k) * hn + ldf(D + k) * v;      // :34
    stf(h + b * shb + k, hn);
    stf(y + b * svb + k, yt);                                         // y uses vhat's strides (:37)
  }
}

template <typename T> struct quad;
template <> struct quad<__nv_bfloat16> {
  __device__ __forceinline__ static void load(const __nv_bfloat16* p, float (&f)[4]) {
    const uint2 v = __ldg(reinterpret_cast<const uint2*>(p));
    const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&v.x);
    const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&v.y);
    f[0] = __low2float(a); f[1] = __high2float(a); f[2] = __low2float(b); f[3] = __high2float(b);
  }
};
template <> struct quad<float> {
  __device__ __forceinline__ static void load(const float* p, float (&f)[4]) {
    const float4 v = __ldg(reinterpret_cast<const float4*>(p));
    f[0] = v.x; f[1] = v.y; f[2] = v.z; f[3] = v.w;
  }
};

// SAME: P is a multiple of the rows a block covers, so every row of a thread
// (and of its block) belongs to one (s, h) pair: the decay, the input
// coefficient and the B, C quads are computed once per thread, not per row.
template <typename IO, int TPR, int RPT, bool SAME>
__global__ void __launch_bounds__(256) streaming_step_kernel(
    const IO* __restrict__ x, const float* __restrict__ dt, float* __restrict__ h,
    const float* __restrict__ A_log, const IO* __restrict__ B, const IO* __restrict__ C,
    const float* __restrict__ Dskip, IO* __restrict__ y, int64_t rows, int Hh, int P) {
  constexpr int RPB = 256 / TPR;               // rows per pass of the block
  constexpr int N = 4 * TPR;
  const int q = threadIdx.x % TPR;             // which 4-wide n group
  const int64_t row0 = (int64_t)blockIdx.x * (RPB * RPT) + threadIdx.x / TPR;
  // the state quads of all RPT rows go out first (evict-first: touched once)
  float4 hv[RPT];
  bool ok[RPT];
#pragma unroll
  for (int r = 0; r < RPT; ++r) {
    const int64_t row = row0 + (int64_t)r * RPB;
    ok[r] = row < rows;
    hv[r] = ok[r] ? ld_stream_f4(reinterpret_cast<const float4*>(h + row * N) + q) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  if constexpr (SAME) {
    const int64_t sh = row0 / P;                 // (s, h) pair of all this thread's rows
    const int s = (int)(sh / Hh), hh = (int)(sh - (int64_t)s * Hh);
    const float a = -expf(__ldg(A_log + hh));
    const float xx = __ldg(dt + s) * a;
    const float e = expf(xx);
    const float coef = zoh_coeff(xx, e, a);
    float bq[4], cq[4], cb[4];
    quad<IO>::load(B + sh * N + 4 * q, bq);
    quad<IO>::load(C + sh * N + 4 * q, cq);
#pragma unroll
    for (int k = 0; k < 4; ++k) cb[k] = coef * bq[k];
    const float* dskr = Dskip + (int64_t)hh * P;
#pragma unroll
    for (int r = 0; r < RPT; ++r) {
      const int64_t row = row0 + (int64_t)r * RPB;
      const float xv = ok[r] ? ldf(x + row) : 0.f;
      float hs[4] = {hv[r].x, hv[r].y, hv[r].z, hv[r].w};
      float part = 0.f;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        hs[k] = e * hs[k] + cb[k] * xv;
        part += cq[k] * hs[k];
      }
#pragma unroll
      for (int off = TPR >> 1; off > 0; off >>= 1) part += __shfl_xor_sync(0xffffffffu, part, off, TPR);
      if (ok[r]) {
        st_stream_f4(reinterpret_cast<float4*>(h + row * N) + q, make_float4(hs[0], hs[1], hs[2], hs[3]));
        if (q == 0) stf(y + row, part + __ldg(dskr + (row - sh * P)) * xv);
      }
    }
  } else {
  // per-row scalars (indices, decay, input coefficient, x, skip) computed once per
  // row by the group's first lane and broadcast to its TPR lanes
#pragma unroll
  for (int r = 0; r < RPT; ++r) {
    const int64_t row = ok[r] ? row0 + (int64_t)r * RPB : 0;
    int sh = 0;
    float e = 0.f, coef = 0.f, xv = 0.f, dsk = 0.f;
    if (q == 0) {
      sh = (int)(row / P);                     // (s, h) pair; S*H < 2^31 (host-checked)
      const int p = (int)(row - (int64_t)sh * P);
      const int s = sh / Hh;
      const int hh = sh - s * Hh;
      const float a = -expf(__ldg(A_log + hh));
      const float xx = __ldg(dt + s) * a;
      e = expf(xx);
      coef = zoh_coeff(xx, e, a);
      xv = ldf(x + row);
      dsk = __ldg(Dskip + (int64_t)hh * P + p);
    }
    sh = __shfl_sync(0xffffffffu, sh, 0, TPR);
    e = __shfl_sync(0xffffffffu, e, 0, TPR);
    coef = __shfl_sync(0xffffffffu, coef, 0, TPR);
    xv = __shfl_sync(0xffffffffu, xv, 0, TPR);
    float bq[4], cq[4];
    quad<IO>::load(B + (int64_t)sh * N + 4 * q, bq);
    quad<IO>::load(C + (int64_t)sh * N + 4 * q, cq);
    float hs[4] = {hv[r].x, hv[r].y, hv[r].z, hv[r].w};
    float part = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      hs[k] = e * hs[k] + (coef * bq[k]) * xv;
      part += cq[k] * hs[k];
    }
#pragma unroll
    for (int off = TPR >> 1; off > 0; off >>= 1) part += __shfl_xor_sync(0xffffffffu, part, off, TPR);
    if (ok[r]) {
      st_stream_f4(reinterpret_cast<float4*>(h + row * N) + q, make_float4(hs[0], hs[1], hs[2], hs[3]));
      if (q == 0) stf(y + row, part + dsk * xv);
    }
  }
  }
}

// Any N (and any alignment): one thread per (s,h,p) row, scalar accesses.
template <typename IO>
__global__ void __launch_bounds__(256) streaming_step_generic_kernel(
    const IO* __restrict__ x, const float* __restrict__ dt, float* __restrict__ h,
    const float* __restrict__ A_log, const IO* __restrict__ B, const IO* __restrict__ C,
    const float* __restrict__ Dskip, IO* __restrict__ y, int64_t rows, int Hh, int P, int N) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t row = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; row < rows; row += stride) {
    const int64_t sh = row / P;
    const int p = (int)(row - sh * P);
    const int64_t s = sh / Hh;
    const int hh = (int)(sh - s * Hh);
    const float a = -expf(__ldg(A_log + hh));
    const float xx = __ldg(dt + s) * a;
    const float e = expf(xx);
    const float coef = zoh_coeff(xx, e, a);
    const float xv = ldf(x + row);
    float acc = 0.f;
    for (int n = 0; n < N; ++n) {
      const float hn = e * h[row * N + n] + (coef * ldf(B + sh * N + n)) * xv;
      h[row * N + n] = hn;
      acc += ldf(C + sh * N + n) * hn;
    }
    stf(y + row, acc + __ldg(Dskip + (int64_t)hh * P + p) * xv);
  }
}

template <typename IO, int TPR>
int launch_step(const void* x, const void* dt, void* h, const void* A_log, const void* B,
                const void* C, const void* Dskip, void* y, int64_t rows, int Hh, int P,
                cudaStream_t st) {
  constexpr int RPT = 4;
  constexpr int RPB = 256 / TPR;
  const int64_t blocks = cdiv(rows, RPB * RPT);
  auto kern = P % (RPB * RPT) == 0 ? streaming_step_kernel<IO, TPR, RPT, true>
                                   : streaming_step_kernel<IO, TPR, RPT, false>;
  kern<<<(unsigned)blocks, 256, 0, st>>>((const IO*)x, (const float*)dt, (float*)h, (const float*)A_log,
                                         (const IO*)B, (const IO*)C, (const float*)Dskip, (IO*)y, rows, Hh, P);
  return check_launch("streaming_step");
}

template <typename IO>
int dispatch_step(int64_t N, bool vec_ok, const void* x, const void* dt, void* h, const void* A_log,
                  const void* B, const void* C, const void* Dskip, void* y, int64_t rows, int Hh,
                  int P, cudaStream_t st) {
  switch (vec_ok ? N : 0) {
    case 4: return launch_step<IO, 1>(x, dt, h, A_log, B, C, Dskip, y, rows, Hh, P, st);
    case 8: return launch_step<IO, 2>(x, dt, h, A_log, B, C, Dskip, y, rows, Hh, P, st);
    case 16: return launch_step<IO, 4>(x, dt, h, A_log, B, C, Dskip, y, rows, Hh, P, st);
    case 32: return launch_step<IO, 8>(x, dt, h, A_log, B, C, Dskip, y, rows, Hh, P, st);
    case 64: return launch_step<IO, 16>(x, dt, h, A_log, B, C, Dskip, y, rows, Hh, P, st);
    case 128: return launch_step<IO, 32>(x, dt, h, A_log, B, C, Dskip, y, rows, Hh, P, st);
  }
  const int64_t blocks = std::min<int64_t>(cdiv(rows, 256), (int64_t)kNumSMs * 32);
  streaming_step_generic_kernel<IO><<<(unsigned)blocks, 256, 0, st>>>(
      (const IO*)x, (const float*)dt, (float*)h, (const float*)A_log, (const IO*)B, (const IO*)C,
      (const float*)Dskip, (IO*)y, rows, Hh, P, (int)N);
  return check_launch("streaming_step");
}

}  // namespace
}  // namespace tssm

extern "C" int tssm_streaming_inplace(const void* vhat, void* h, const void* Abar, const void* Bbar,
                                      const void* C, const void* D, void* y, int64_t Bsz,
                                      int64_t H, int64_t stride_vb, int64_t stride_hb,
                                      int64_t stride_cb, int dtype, tssm_stream_t stream) {
  using namespace tssm;
  TSSM_REQUIRE(Bsz >= 0 && H >= 0, "streaming_inplace: negative size");
  if (Bsz * H == 0) return TSSM_OK;
  TSSM_REQUIRE(vhat && h && Abar && Bbar && C && D && y, "streaming_inplace: null pointer");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int64_t blocks = std::min<int64_t>(cdiv(Bsz * H, 256), (int64_t)kNumSMs * 16);
  if (dtype == TSSM_F32) {
    streaming_inplace_kernel<float><<<(unsigned)blocks, 256, 0, st>>>(
        (const float*)vhat, (float*)h, (const float*)Abar, (const float*)Bbar, (const float*)C,
        (const float*)D, (float*)y, Bsz, H, stride_vb, stride_hb, stride_cb);
  } else if (dtype == TSSM_BF16) {
    using bf = __nv_bfloat16;
    streaming_inplace_kernel<bf><<<(unsigned)blocks, 256, 0, st>>>(
        (const bf*)vhat, (bf*)h, (const bf*)Abar, (const bf*)Bbar, (const bf*)C, (const bf*)D,
        (bf*)y, Bsz, H, stride_vb, stride_hb, stride_cb);
  } else {
    set_error("streaming_inplace: dtype must be f32 or bf16 (got %d)", dtype);
    return TSSM_ERR_INVALID;
  }
  return check_launch("streaming_inplace");
}

extern "C" int tssm_streaming_step(const void* x, const void* dt, void* h, const void* A_log,
                                   const void* B, const void* C, const void* Dskip, void* y,
                                   int64_t S, int64_t Hh, int64_t P, int64_t N, int io_dtype,
                                   tssm_stream_t stream) {
  using namespace tssm;
  TSSM_REQUIRE(S >= 0 && Hh >= 0 && P >= 0 && N >= 0, "streaming_step: negative size");
  if (S * Hh * P * N == 0) return TSSM_OK;
  TSSM_REQUIRE(x && dt && h && A_log && B && C && Dskip && y, "streaming_step: null pointer");
  const int isz = io_dtype == TSSM_BF16 ? 2 : 4;
  // The vector path needs 16-byte state rows and 4-element aligned B, C rows.
  const bool vec_ok = aligned16(h) && (reinterpret_cast<uintptr_t>(B) % (4 * isz)) == 0 &&
                      (reinterpret_cast<uintptr_t>(C) % (4 * isz)) == 0;
  TSSM_REQUIRE(Hh < (1 << 30) && P < (1 << 30) && S * Hh < (int64_t(1) << 31), "streaming_step: S, H or P too large");
  const int64_t rows = S * Hh * P;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (io_dtype == TSSM_BF16)
    return dispatch_step<__nv_bfloat16>(N, vec_ok, x, dt, h, A_log, B, C, Dskip, y, rows, (int)Hh, (int)P, st);
  if (io_dtype == TSSM_F32)
    return dispatch_step<float>(N, vec_ok, x, dt, h, A_log, B, C, Dskip, y, rows, (int)Hh, (int)P, st);
  set_error("streaming_step: io_dtype must be bf16 or f32 (got %d)", io_dtype);
  return TSSM_ERR_INVALID;
}
