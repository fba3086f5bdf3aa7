// Diagonal selective scans in one pass (replaces ssm_scan.py:17-124 / :239-264).
//
// Layout [Bsz, L, H] with H contiguous.  A CTA owns 32 consecutive channels
// (one per lane, so every time step is one coalesced 128-byte row segment per
// warp) of one batch row and walks the sequence in super-segments of NW*S
// steps: warp w holds steps [w*S, (w+1)*S) of the super-segment in registers,
// (1) folds them into an (a, x) aggregate, (2) after one barrier folds the
// aggregates of the warps before it onto the carry entering the super-segment
// and (3) replays its steps from that exclusive prefix, writing h and y.  All
// inputs are read from HBM once; there are no intermediate buffers and no
// inter-CTA communication.
#include "common.cuh"

namespace tssm {
namespace {

template <typename T, int S, int NW>
__global__ void __launch_bounds__(NW * 32, 1) ssm_forward_kernel(
    const T* __restrict__ u, const T* __restrict__ A, const T* __restrict__ B,
    const T* __restrict__ C, const T* __restrict__ D, T* __restrict__ y, T* __restrict__ h,
    int64_t L, int64_t H) {
  __shared__ float s_a[NW][32];
  __shared__ float s_x[NW][32];
  __shared__ float s_carry[32];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int64_t ch = (int64_t)blockIdx.x * 32 + lane;
  const bool valid = ch < H;
  // One 64-bit base per CTA; offsets inside a batch row fit in 32 bits (host-checked).
  const int64_t base = (int64_t)blockIdx.y * L * H + ch;
  const T* __restrict__ ub = u + base;
  const T* __restrict__ Ab = A + base;
  const T* __restrict__ Bb = B + base;
  const T* __restrict__ Cb = C + base;
  T* __restrict__ yb = y + base;
  T* __restrict__ hb = h ? h + base : nullptr;
  const int Hi = (int)H;
  const int Li = (int)L;
  const float dv = valid ? ldf(D + ch) : 0.f;
  float carry = 0.f;
  for (int t0 = 0; t0 < Li; t0 += NW * S) {
    const int ts = t0 + warp * S;
    float a[S], bu[S], uu[S];
#pragma unroll
    for (int i = 0; i < S; ++i) {
      const int t = ts + i;
      if (valid && t < Li) {
        const int off = t * Hi;
        a[i] = ldf(Ab + off);
        uu[i] = ldf(ub + off);
        bu[i] = ldf(Bb + off) * uu[i];
      } else {
        a[i] = 1.f;
        bu[i] = 0.f;
        uu[i] = 0.f;
      }
    }
    float ag_a = 1.f, ag_x = 0.f;
#pragma unroll
    for (int i = 0; i < S; ++i) {
      ag_x = a[i] * ag_x + bu[i];
      ag_a *= a[i];
    }
    s_a[warp][lane] = ag_a;
    s_x[warp][lane] = ag_x;
    __syncthreads();
    float hs = carry;
    for (int w = 0; w < warp; ++w) hs = s_a[w][lane] * hs + s_x[w][lane];
#pragma unroll
    for (int i = 0; i < S; ++i) {
      hs = a[i] * hs + bu[i];
      const int t = ts + i;
      if (valid && t < Li) {
        const int off = t * Hi;
        if (hb) stf(hb + off, hs);
        stf(yb + off, ldf(Cb + off) * hs + dv * uu[i]);
      }
    }
    if (warp == NW - 1) s_carry[lane] = hs;
    __syncthreads();
    carry = s_carry[lane];
  }
}

// Fused discretize + scan + readout over an N-wide state per channel.
// Lanes are (d, n) pairs: NP = pow2 >= N lanes per d, 32/NP d per warp; the
// readout sum over n is a shuffle reduction inside each NP-lane group.
template <int S, int NW>
__global__ void __launch_bounds__(NW * 32) selective_scan_kernel(
    const float* __restrict__ x, const float* __restrict__ dt, const float* __restrict__ A_log,
    const float* __restrict__ B, const float* __restrict__ C, const float* __restrict__ Dskip,
    float* __restrict__ y, float* __restrict__ h_last, int64_t L, int64_t Dm, int N, int NP) {
  __shared__ float s_a[NW][32];
  __shared__ float s_x[NW][32];
  __shared__ float s_carry[32];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int dpw = 32 / NP;
  const int64_t d = (int64_t)blockIdx.x * dpw + lane / NP;
  const int n = lane % NP;
  const bool valid = d < Dm && n < N;
  const int64_t b = blockIdx.y;
  const float a = valid ? -expf(A_log[d * N + n]) : -1.f;
  const float dsk = (d < Dm) ? Dskip[d] : 0.f;
  const float* xb = x + b * L * Dm;
  const float* dtb = dt + b * L;
  const float* Bb = B + b * L * N;
  const float* Cb = C + b * L * N;
  float carry = 0.f;
  for (int64_t t0 = 0; t0 < L; t0 += NW * S) {
    const int64_t ts = t0 + (int64_t)warp * S;
    float ab[S], bu[S], xv[S];
#pragma unroll
    for (int i = 0; i < S; ++i) {
      const int64_t t = ts + i;
      if (valid && t < L) {
        const float xx = dtb[t] * a;
        const float e = expf(xx);
        ab[i] = e;
        xv[i] = xb[t * Dm + d];
        bu[i] = (expm1_guard_f32(xx, e) / (a + 1e-12f) * Bb[t * N + n]) * xv[i];
      } else {
        ab[i] = 1.f;
        bu[i] = 0.f;
        xv[i] = (d < Dm && t < L) ? xb[t * Dm + d] : 0.f;
      }
    }
    float ag_a = 1.f, ag_x = 0.f;
#pragma unroll
    for (int i = 0; i < S; ++i) {
      ag_x = ab[i] * ag_x + bu[i];
      ag_a *= ab[i];
    }
    s_a[warp][lane] = ag_a;
    s_x[warp][lane] = ag_x;
    __syncthreads();
    float hs = carry;
    for (int w = 0; w < warp; ++w) hs = s_a[w][lane] * hs + s_x[w][lane];
#pragma unroll
    for (int i = 0; i < S; ++i) {
      hs = ab[i] * hs + bu[i];
      const int64_t t = ts + i;
      float part = (valid && t < L) ? Cb[t * N + n] * hs : 0.f;
      for (int off = NP >> 1; off > 0; off >>= 1) part += __shfl_xor_sync(0xffffffffu, part, off);
      if (n == 0 && d < Dm && t < L) y[(b * L + t) * Dm + d] = part + dsk * xv[i];
    }
    if (warp == NW - 1) s_carry[lane] = hs;
    __syncthreads();
    carry = s_carry[lane];
  }
  if (h_last && warp == 0 && valid) h_last[(b * Dm + d) * N + n] = carry;
}

}  // namespace
}  // namespace tssm

extern "C" int tssm_ssm_forward(const void* u, const void* A, const void* B, const void* C,
                                const void* D, void* y, void* h, int64_t Bsz, int64_t L,
                                int64_t H, int dtype, tssm_stream_t stream) {
  using namespace tssm;
  TSSM_REQUIRE(Bsz >= 0 && L >= 0 && H >= 0, "ssm_forward: negative size");
  if (Bsz * L * H == 0) return TSSM_OK;
  TSSM_REQUIRE(u && A && B && C && D && y, "ssm_forward: null pointer");
  TSSM_REQUIRE(Bsz <= 65535, "ssm_forward: batch %lld exceeds 65535", (long long)Bsz);
  TSSM_REQUIRE(L * H < (int64_t(1) << 31), "ssm_forward: L*H must be < 2^31 per batch row");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  constexpr int S = 16, NW = 16;
  dim3 grid((unsigned)cdiv(H, 32), (unsigned)Bsz);
  if (dtype == TSSM_F32) {
    ssm_forward_kernel<float, S, NW><<<grid, NW * 32, 0, st>>>(
        (const float*)u, (const float*)A, (const float*)B, (const float*)C, (const float*)D,
        (float*)y, (float*)h, L, H);
  } else if (dtype == TSSM_BF16) {
    using bf = __nv_bfloat16;
    ssm_forward_kernel<bf, S, NW><<<grid, NW * 32, 0, st>>>(
        (const bf*)u, (const bf*)A, (const bf*)B, (const bf*)C, (const bf*)D, (bf*)y, (bf*)h, L, H);
  } else {
    set_error("ssm_forward: dtype must be f32 or bf16 (got %d)", dtype);
    return TSSM_ERR_INVALID;
  }
  return check_launch("ssm_forward");
}

extern "C" int tssm_selective_scan(const void* x, const void* dt, const void* A_log, const void* B,
                                   const void* C, const void* Dskip, void* y, void* h_last,
                                   int64_t Bsz, int64_t L, int64_t Dm, int64_t N,
                                   tssm_stream_t stream) {
  using namespace tssm;
  TSSM_REQUIRE(Bsz >= 0 && L >= 0 && Dm >= 0 && N >= 1, "selective_scan: bad size");
  TSSM_REQUIRE(N <= 32, "selective_scan: N=%lld > 32 is not supported", (long long)N);
  if (Bsz * L * Dm == 0) return TSSM_OK;
  TSSM_REQUIRE(x && dt && A_log && B && C && Dskip && y, "selective_scan: null pointer");
  TSSM_REQUIRE(Bsz <= 65535, "selective_scan: batch %lld exceeds 65535", (long long)Bsz);
  int NP = 1;
  while (NP < N) NP <<= 1;
  constexpr int S = 16, NW = 16;
  dim3 grid((unsigned)cdiv(Dm, 32 / NP), (unsigned)Bsz);
  selective_scan_kernel<S, NW><<<grid, NW * 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      (const float*)x, (const float*)dt, (const float*)A_log, (const float*)B, (const float*)C,
      (const float*)Dskip, (float*)y, (float*)h_last, L, Dm, (int)N, NP);
  return check_launch("selective_scan");
}
