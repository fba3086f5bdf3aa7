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

// Optional fused mean-pool head (POOL): every CTA adds
// sum_{t, its channels} poolW[ch] * y[b,t,ch] * pool_inv to pool_out[b] (plus the
// bias once per batch row), the composition ssm_forward -> mean_pool_logit_kernel
// (streaming_inference_kernel.py:159-194) over y without re-reading it.
template <typename T, int S, int NW, bool POOL>
__global__ void __launch_bounds__(NW * 32, 1) ssm_forward_kernel(
    const T* __restrict__ u, const T* __restrict__ A, const T* __restrict__ B,
    const T* __restrict__ C, const T* __restrict__ D, T* __restrict__ y, T* __restrict__ h,
    int64_t L, int64_t H, const float* __restrict__ poolW, const float* __restrict__ pool_bias,
    float* __restrict__ pool_out, float pool_inv) {
  __shared__ float s_a[NW][32];
  __shared__ float s_x[NW][32];
  __shared__ float s_carry[32];
  __shared__ float s_pool[NW];
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
  const float pw = (POOL && valid) ? poolW[ch] : 0.f;
  float pacc = 0.f;
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
        const float yv = ldf(Cb + off) * hs + dv * uu[i];
        stf(yb + off, yv);
        if (POOL) pacc += pw * io_round<T>(yv);
      }
    }
    if (warp == NW - 1) s_carry[lane] = hs;
    __syncthreads();
    carry = s_carry[lane];
  }
  if (POOL) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) pacc += __shfl_xor_sync(0xffffffffu, pacc, o);
    if (lane == 0) s_pool[warp] = pacc;
    __syncthreads();
    if (threadIdx.x == 0) {
      float s2 = 0.f;
      for (int w = 0; w < NW; ++w) s2 += s_pool[w];
      atomicAdd(pool_out + blockIdx.y, s2 * pool_inv + (blockIdx.x == 0 ? pool_bias[0] : 0.f));
    }
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


// Diagonal multi-head scan with the reference's readout (multihead_ssm_kernel.py:
// 19-187, its compile errors read as their intent): per (b, head, p)
//   Abar = exp(dt[b,t,head] * a[head,p]),  h = Abar*h + (beta*B[b,t,head,p])*u[b,t,head*hd+p]
//   y_head[t] = sum_p C*h + sum_p D*u, written to every position of the head slice.
// CTA = (head, b).  Thread (lane, pg, seg): p = 32*pg + lane, seg = time segment
// of a super-segment of NSEG*S steps (fold / prefix / replay as in
// ssm_forward_kernel); the per-step head sum is a warp reduction plus a sum of
// the PG group partials through shared memory.
template <typename T, int S, int NSEG, int PG, bool ZOH>
__global__ void __launch_bounds__(32 * PG * NSEG, 1) multihead_diag_kernel(
    const T* __restrict__ u, const float* __restrict__ A_log, const T* __restrict__ Bm, const T* __restrict__ Cm,
    const float* __restrict__ dt, const float* __restrict__ Dskip, T* __restrict__ y, int L, int nh, int hd) {
  __shared__ float s_a[NSEG][PG][32];
  __shared__ float s_x[NSEG][PG][32];
  __shared__ float s_carry[PG][32];
  __shared__ float s_part[NSEG][S][PG];
  const int lane = threadIdx.x & 31;
  const int w = threadIdx.x >> 5;
  const int pg = w % PG, seg = w / PG;
  const int head = blockIdx.x, b = blockIdx.y;
  const int p = pg * 32 + lane;
  const bool valid = p < hd;
  const int H = nh * hd;
  const float a = valid ? -expf(A_log[head * hd + p]) : -1.f;
  const float dsk = valid ? Dskip[head * hd + p] : 0.f;
  const T* ub = u + (int64_t)b * L * H + head * hd + p;
  const T* Bb = Bm + (int64_t)b * L * H + head * hd + p;   // [B,L,nh,hd] == [B,L,H]
  const T* Cb = Cm + (int64_t)b * L * H + head * hd + p;
  const float* dtb = dt + (int64_t)b * L * nh + head;
  T* yb = y + (int64_t)b * L * H + head * hd + p;
  float carry = 0.f;
  for (int t0 = 0; t0 < L; t0 += NSEG * S) {
    const int ts = t0 + seg * S;
    float ab[S], bu[S], uu[S];
#pragma unroll
    for (int i = 0; i < S; ++i) {
      const int t = ts + i;
      ab[i] = 1.f;
      bu[i] = 0.f;
      uu[i] = 0.f;
      if (t < L) {
        const float dv = __ldg(dtb + (int64_t)t * nh);
        const float x = dv * a;
        const float e = expf(x);
        if (valid) {
          ab[i] = e;
          uu[i] = ldf(ub + (int64_t)t * H);
          const float beta = ZOH ? zoh_coeff(x, e, a) : dv;
          bu[i] = (beta * ldf(Bb + (int64_t)t * H)) * uu[i];
        }
      }
    }
    float ag_a = 1.f, ag_x = 0.f;
#pragma unroll
    for (int i = 0; i < S; ++i) {
      ag_x = ab[i] * ag_x + bu[i];
      ag_a *= ab[i];
    }
    s_a[seg][pg][lane] = ag_a;
    s_x[seg][pg][lane] = ag_x;
    __syncthreads();
    float hs = carry;
    for (int q = 0; q < seg; ++q) hs = s_a[q][pg][lane] * hs + s_x[q][pg][lane];
#pragma unroll
    for (int i = 0; i < S; ++i) {
      hs = ab[i] * hs + bu[i];
      const int t = ts + i;
      float part = (valid && t < L) ? ldf(Cb + (int64_t)t * H) * hs + dsk * uu[i] : 0.f;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
      if (lane == 0) s_part[seg][i][pg] = part;
    }
    if (seg == NSEG - 1) s_carry[pg][lane] = hs;
    __syncthreads();
#pragma unroll
    for (int i = 0; i < S; ++i) {
      const int t = ts + i;
      if (valid && t < L) {
        float tot = 0.f;
#pragma unroll
        for (int g = 0; g < PG; ++g) tot += s_part[seg][i][g];
        stf(yb + (int64_t)t * H, tot);
      }
    }
    carry = s_carry[pg][lane];
    __syncthreads();
  }
}

template <typename T, int PG>
int launch_diag(const void* u, const void* A_log, const void* B, const void* C, const void* dt, const void* D,
                void* y, int64_t Bsz, int64_t L, int64_t nh, int64_t hd, bool zoh, cudaStream_t st) {
  constexpr int S = 8, NSEG = PG == 1 ? 16 : (PG == 2 ? 8 : 4);
  dim3 grid((unsigned)nh, (unsigned)Bsz);
  if (zoh)
    multihead_diag_kernel<T, S, NSEG, PG, true><<<grid, 32 * PG * NSEG, 0, st>>>(
        (const T*)u, (const float*)A_log, (const T*)B, (const T*)C, (const float*)dt, (const float*)D, (T*)y,
        (int)L, (int)nh, (int)hd);
  else
    multihead_diag_kernel<T, S, NSEG, PG, false><<<grid, 32 * PG * NSEG, 0, st>>>(
        (const T*)u, (const float*)A_log, (const T*)B, (const T*)C, (const float*)dt, (const float*)D, (T*)y,
        (int)L, (int)nh, (int)hd);
  return check_launch("multihead_diag");
}

template <typename T>
int dispatch_diag(const void* u, const void* A_log, const void* B, const void* C, const void* dt, const void* D,
                  void* y, int64_t Bsz, int64_t L, int64_t nh, int64_t hd, bool zoh, cudaStream_t st) {
  if (hd <= 32) return launch_diag<T, 1>(u, A_log, B, C, dt, D, y, Bsz, L, nh, hd, zoh, st);
  if (hd <= 64) return launch_diag<T, 2>(u, A_log, B, C, dt, D, y, Bsz, L, nh, hd, zoh, st);
  return launch_diag<T, 4>(u, A_log, B, C, dt, D, y, Bsz, L, nh, hd, zoh, st);
}

}  // namespace
}  // namespace tssm

namespace tssm {
int ssm_forward_impl(const void* u, const void* A, const void* B, const void* C, const void* D, void* y, void* h,
                     const void* poolW, const void* pool_bias, void* pool_out, int64_t Bsz, int64_t L, int64_t H,
                     int dtype, tssm_stream_t stream) {
  TSSM_REQUIRE(Bsz >= 0 && L >= 0 && H >= 0, "ssm_forward: negative size");
  if (Bsz * L * H == 0) return TSSM_OK;
  TSSM_REQUIRE(u && A && B && C && D && y, "ssm_forward: null pointer");
  TSSM_REQUIRE(Bsz <= 65535, "ssm_forward: batch %lld exceeds 65535", (long long)Bsz);
  TSSM_REQUIRE(L * H < (int64_t(1) << 31), "ssm_forward: L*H must be < 2^31 per batch row");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  constexpr int S = 16, NW = 16;
  dim3 grid((unsigned)cdiv(H, 32), (unsigned)Bsz);
  const float pool_inv = (float)(1.0 / ((double)L * (double)H + 1e-9));
  // With the pooled head the kernel walks shorter per-warp runs (S=8) with twice
  // the warps: at S=16 the extra accumulator leaves too few registers for the
  // loads in flight (measured: +18 us against +6 us at config-1 size).
  const bool pool = pool_out != nullptr;
  const int nthr = pool ? 32 * 32 : NW * 32;
  if (dtype == TSSM_F32) {
    auto kern = pool ? ssm_forward_kernel<float, 8, 32, true> : ssm_forward_kernel<float, S, NW, false>;
    kern<<<grid, nthr, 0, st>>>((const float*)u, (const float*)A, (const float*)B, (const float*)C,
                                (const float*)D, (float*)y, (float*)h, L, H, (const float*)poolW,
                                (const float*)pool_bias, (float*)pool_out, pool_inv);
  } else if (dtype == TSSM_BF16) {
    using bf = __nv_bfloat16;
    auto kern = pool ? ssm_forward_kernel<bf, 8, 32, true> : ssm_forward_kernel<bf, S, NW, false>;
    kern<<<grid, nthr, 0, st>>>((const bf*)u, (const bf*)A, (const bf*)B, (const bf*)C, (const bf*)D, (bf*)y,
                                (bf*)h, L, H, (const float*)poolW, (const float*)pool_bias, (float*)pool_out,
                                pool_inv);
  } else {
    set_error("ssm_forward: dtype must be f32 or bf16 (got %d)", dtype);
    return TSSM_ERR_INVALID;
  }
  return check_launch("ssm_forward");
}
}  // namespace tssm

extern "C" int tssm_ssm_forward(const void* u, const void* A, const void* B, const void* C,
                                const void* D, void* y, void* h, int64_t Bsz, int64_t L,
                                int64_t H, int dtype, tssm_stream_t stream) {
  return tssm::ssm_forward_impl(u, A, B, C, D, y, h, nullptr, nullptr, nullptr, Bsz, L, H, dtype, stream);
}

extern "C" int tssm_ssm_forward_pool(const void* u, const void* A, const void* B, const void* C, const void* D,
                                     void* y, void* h, const void* poolW, const void* pool_bias, void* pool_out,
                                     int64_t Bsz, int64_t L, int64_t H, int dtype, tssm_stream_t stream) {
  using namespace tssm;
  TSSM_REQUIRE(Bsz >= 0 && L >= 0 && H >= 0, "ssm_forward_pool: negative size");
  TSSM_REQUIRE(poolW && pool_bias && pool_out, "ssm_forward_pool: null pool pointer");
  if (Bsz == 0) return TSSM_OK;
  if (L * H == 0)   // nothing to pool: the logit is the bias
    return tssm_mean_pool_logit(nullptr, poolW, pool_bias, pool_out, Bsz, L, H, TSSM_F32, stream);
  if (cudaMemsetAsync(pool_out, 0, (size_t)Bsz * sizeof(float), reinterpret_cast<cudaStream_t>(stream)) != cudaSuccess)
    return check_launch("ssm_forward_pool: clear pool_out");
  return ssm_forward_impl(u, A, B, C, D, y, h, poolW, pool_bias, pool_out, Bsz, L, H, dtype, stream);
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

extern "C" int tssm_multihead_diag(const void* u, const void* A_log, const void* B, const void* C, const void* dt,
                                   const void* Dskip, void* y, int64_t Bsz, int64_t L, int64_t n_heads,
                                   int64_t head_dim, int bdisc, int dtype, tssm_stream_t stream) {
  using namespace tssm;
  TSSM_REQUIRE(Bsz >= 0 && L >= 0 && n_heads >= 0 && head_dim >= 0, "multihead_diag: negative size");
  if (Bsz * L * n_heads * head_dim == 0) return TSSM_OK;
  TSSM_REQUIRE(u && A_log && B && C && dt && Dskip && y, "multihead_diag: null pointer");
  TSSM_REQUIRE(head_dim <= 128, "multihead_diag: head_dim=%lld > 128 is not supported", (long long)head_dim);
  TSSM_REQUIRE(bdisc == 0 || bdisc == 1, "multihead_diag: bdisc must be 0 (euler) or 1 (zoh)");
  TSSM_REQUIRE(Bsz <= 65535 && n_heads <= 65535 && L < (int64_t(1) << 31), "multihead_diag: size out of range");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == TSSM_F32) return dispatch_diag<float>(u, A_log, B, C, dt, Dskip, y, Bsz, L, n_heads, head_dim, bdisc == 1, st);
  if (dtype == TSSM_BF16)
    return dispatch_diag<__nv_bfloat16>(u, A_log, B, C, dt, Dskip, y, Bsz, L, n_heads, head_dim, bdisc == 1, st);
  set_error("multihead_diag: dtype must be f32 or bf16 (got %d)", dtype);
  return TSSM_ERR_INVALID;
}
