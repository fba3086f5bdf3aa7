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
//
// When the rows are TMA-addressable (16-byte aligned bases and row pitch), the
// same scan runs with its inputs staged by TMA (ssm_forward_tma_kernel): a
// producer warp keeps a ring of 128-step x 32-channel tiles of A, u, B and C in
// flight while 16 compute warps scan the previous tile out of shared memory,
// so the HBM latency is hidden instead of being paid once per super-segment.
#include <cudaTypedefs.h>

#include "common.cuh"
#include "tcgen05.cuh"
#include "tmap.cuh"

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
  const float ra = 1.0f / (a + 1e-12f);   // ZOH coefficient as a product (within an ulp of the quotient)
  const float dsk = (d < Dm) ? Dskip[d] : 0.f;
  const float* xb = x + b * L * Dm;
  const float* dtb = dt + b * L;
  const float* Bb = B + b * L * N;
  const float* Cb = C + b * L * N;
  float carry = 0.f;
  for (int64_t t0 = 0; t0 < L; t0 += NW * S) {
    const int64_t ts = t0 + (int64_t)warp * S;
    // every load of the run (C included) goes out before the first use: the replay
    // below has no global load between its dependent readout reductions
    float ab[S], bu[S], xv[S], cv[S];
#pragma unroll
    for (int i = 0; i < S; ++i) {
      const int64_t t = ts + i;
      if (valid && t < L) {
        const float xx = dtb[t] * a;
        const float e = expf(xx);
        ab[i] = e;
        xv[i] = xb[t * Dm + d];
        bu[i] = (expm1_guard_f32(xx, e) * ra * Bb[t * N + n]) * xv[i];
        cv[i] = Cb[t * N + n];
      } else {
        ab[i] = 1.f;
        bu[i] = 0.f;
        xv[i] = (d < Dm && t < L) ? xb[t * Dm + d] : 0.f;
        cv[i] = 0.f;
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
      float part = cv[i] * hs;
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


// ---------------------------------------------------------------- TMA-staged ssm_forward
constexpr int FT_CH = 128;            // steps per staged tile
constexpr int FT_NW = 16;             // compute warps
constexpr int FT_S = FT_CH / FT_NW;   // steps per compute warp and tile
constexpr uint32_t FT_BAR = 1;        // named barrier of the compute warps

template <typename T>
struct FtLayout {
  static constexpr int STAGES = sizeof(T) == 4 ? 3 : 6;
  static constexpr int TILE = FT_CH * 32 * (int)sizeof(T);   // one array's [FT_CH][32] tile
  static constexpr int STAGE = 4 * TILE;                      // A, u, B, C
  static constexpr int OFF_AGG = STAGES * STAGE;              // [2][2][FT_NW][32] f32 aggregates
  static constexpr int OFF_BAR = OFF_AGG + 2 * 2 * FT_NW * 32 * 4;
  static constexpr int OFF_MISC = OFF_BAR + 2 * STAGES * 8;   // abort flag, issued, consumed
  static constexpr int OFF_POOL = OFF_MISC + 16;              // [FT_NW] per-warp pooled sums
  static constexpr int BYTES = OFF_POOL + FT_NW * 4 + 128;    // + slack to align the base to 128
  static_assert(BYTES <= 232448, "ssm_forward_tma shared-memory layout exceeds the per-CTA limit");
};

// CTA = (32 channels, one batch row); warp FT_NW is the TMA producer.  Tiles are
// [FT_CH steps][32 channels] boxes of the [Bsz][L][H] tensors; steps past L and
// channels past H read as zero from the tensor map and are masked here.  POOL adds
// the fused mean-pooled logit head, as in ssm_forward_kernel.
template <typename T, bool POOL>
__global__ void __launch_bounds__((FT_NW + 1) * 32, 1) ssm_forward_tma_kernel(
    const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmU,
    const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmC,
    const T* __restrict__ D, T* __restrict__ y, T* __restrict__ h, int L, int H, const float* __restrict__ poolW,
    const float* __restrict__ pool_bias, float* __restrict__ pool_out, float pool_inv, int* __restrict__ status) {
  using LY = FtLayout<T>;
  constexpr int ST = LY::STAGES;
  extern __shared__ uint8_t ft_raw[];
  uint8_t* smem = ft_raw + ((128u - (sm100::smem_u32(ft_raw) & 127u)) & 127u);
  float* agg = reinterpret_cast<float*>(smem + LY::OFF_AGG);   // [buf][a|x][warp][lane]
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + LY::OFF_BAR);
  uint64_t* empty = full + ST;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + LY::OFF_MISC);
  int* issued = reinterpret_cast<int*>(smem + LY::OFF_MISC + 4);
  int* consumed = reinterpret_cast<int*>(smem + LY::OFF_MISC + 8);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int ch0 = blockIdx.x * 32, b = blockIdx.y;
  const int nt = (L + FT_CH - 1) / FT_CH;
  if (threadIdx.x == 0) {
    for (int i = 0; i < ST; ++i) {
      sm100::mbar_init(&full[i], 1);
      sm100::mbar_init(&empty[i], FT_NW);
    }
    *abort_flag = 0;
    *issued = 0;
    *consumed = 0;
    sm100::fence_mbar_init();
  }
  __syncthreads();

  if (warp == FT_NW) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      sm100::prefetch_tmap(&tmA);
      sm100::prefetch_tmap(&tmU);
      sm100::prefetch_tmap(&tmB);
      sm100::prefetch_tmap(&tmC);
      int k = 0;
      for (; k < nt; ++k) {
        const int s = k % ST;
        if (k >= ST && !sm100::mbar_wait(&empty[s], ((k / ST) - 1) & 1, abort_flag)) {
          if (!*abort_flag) {
            *abort_flag = 1;
            atomicExch(status, 2001);
          }
          break;
        }
        uint8_t* st = smem + s * LY::STAGE;
        sm100::mbar_arrive_expect_tx(&full[s], LY::STAGE);
        sm100::tma_load_3d(st, &tmA, ch0, k * FT_CH, b, &full[s]);
        sm100::tma_load_3d(st + LY::TILE, &tmU, ch0, k * FT_CH, b, &full[s]);
        sm100::tma_load_3d(st + 2 * LY::TILE, &tmB, ch0, k * FT_CH, b, &full[s]);
        sm100::tma_load_3d(st + 3 * LY::TILE, &tmC, ch0, k * FT_CH, b, &full[s]);
      }
      *issued = k;
    }
  } else {
    // ------------------------------------------------------------ compute warps
    const int ch = ch0 + lane;
    const bool valid = ch < H;
    const float dv = valid ? ldf(D + ch) : 0.f;
    const float pw = (POOL && valid) ? poolW[ch] : 0.f;
    float pacc = 0.f;
    const int64_t base = (int64_t)b * L * H + ch;
    float carry = 0.f;
    int k = 0;
    for (; k < nt; ++k) {
      const int s = k % ST, pb = k & 1;
      const bool bad = !sm100::mbar_wait(&full[s], (k / ST) & 1, abort_flag);
      const T* tA = reinterpret_cast<const T*>(smem + s * LY::STAGE);
      const T* tU = tA + FT_CH * 32;
      const T* tB = tU + FT_CH * 32;
      const T* tC = tB + FT_CH * 32;
      const int r0 = warp * FT_S;            // this warp's rows of the tile
      const int t0 = k * FT_CH + r0;         // and their first step
      float a[FT_S], bu[FT_S], uu[FT_S];
      float ag_a = 1.f, ag_x = 0.f;
      if (!bad) {
#pragma unroll
        for (int i = 0; i < FT_S; ++i) {
          const int r = (r0 + i) * 32 + lane;
          if (valid && t0 + i < L) {
            a[i] = ldf(tA + r);
            uu[i] = ldf(tU + r);
            bu[i] = ldf(tB + r) * uu[i];
          } else {
            a[i] = 1.f;
            bu[i] = 0.f;
            uu[i] = 0.f;
          }
        }
#pragma unroll
        for (int i = 0; i < FT_S; ++i) {
          ag_x = a[i] * ag_x + bu[i];
          ag_a *= a[i];
        }
        agg[((pb * 2 + 0) * FT_NW + warp) * 32 + lane] = ag_a;
        agg[((pb * 2 + 1) * FT_NW + warp) * 32 + lane] = ag_x;
      } else if (!*abort_flag) {
        *abort_flag = 1;
        atomicExch(status, 2002);
      }
      // one barrier per tile: the aggregates are double-buffered by tile parity, and a
      // warp writes buffer pb again only after every warp has passed tile k+1's barrier
      if (sm100::named_bar_or(FT_BAR, FT_NW * 32, bad)) break;
      // exclusive prefix for this warp and the carry into the next tile, folded in
      // registers from all warps' aggregates (loaded at once)
      float wa[FT_NW], wx[FT_NW];
#pragma unroll
      for (int w = 0; w < FT_NW; ++w) {
        wa[w] = agg[((pb * 2 + 0) * FT_NW + w) * 32 + lane];
        wx[w] = agg[((pb * 2 + 1) * FT_NW + w) * 32 + lane];
      }
      float hs = carry, nxt = carry;
#pragma unroll
      for (int w = 0; w < FT_NW; ++w) {
        if (w == warp) hs = nxt;
        nxt = wa[w] * nxt + wx[w];
      }
      carry = nxt;
#pragma unroll
      for (int i = 0; i < FT_S; ++i) {
        hs = a[i] * hs + bu[i];
        const int t = t0 + i;
        if (valid && t < L) {
          const int64_t off = base + (int64_t)t * H;
          if (h) stf(h + off, hs);
          const float yv = ldf(tC + (r0 + i) * 32 + lane) * hs + dv * uu[i];
          stf(y + off, yv);
          if (POOL) pacc += pw * io_round<T>(yv);
        }
      }
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(&empty[s]);   // this warp is done with stage s
    }
    if (threadIdx.x == 0) *consumed = k;
    if (POOL && k == nt) {   // every tile scanned (k < nt only after an abort, uniformly)
      float* spool = reinterpret_cast<float*>(smem + LY::OFF_POOL);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) pacc += __shfl_xor_sync(0xffffffffu, pacc, o);
      if (lane == 0) spool[warp] = pacc;
      sm100::named_bar_sync(FT_BAR, FT_NW * 32);
      if (threadIdx.x == 0) {
        float s2 = 0.f;
        for (int w = 0; w < FT_NW; ++w) s2 += spool[w];
        atomicAdd(pool_out + b, s2 * pool_inv + (blockIdx.x == 0 ? pool_bias[0] : 0.f));
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0 && *abort_flag) {
    // loads issued but never consumed must land before the CTA exits
    for (int c = *consumed; c < *issued; ++c) sm100::mbar_wait(&full[c % ST], (c / ST) & 1, nullptr, 100000000ull);
  }
}

// 3-D map over [Bsz][L][H] (H contiguous), box {32 channels, FT_CH steps, 1}, no swizzle.
inline bool ft_map(CUtensorMap* m, const void* base, CUtensorMapDataType dt, int esize, int64_t Bsz, int64_t L,
                   int64_t H) {
  auto fn = tmap_encode_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {(cuuint64_t)H, (cuuint64_t)L, (cuuint64_t)Bsz};
  cuuint64_t strides[2] = {(cuuint64_t)(H * esize), (cuuint64_t)(L * H * esize)};
  cuuint32_t box[3] = {32, FT_CH, 1};
  cuuint32_t es[3] = {1, 1, 1};
  return fn(m, dt, 3, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Launches the TMA-staged scan when the tensors are TMA-addressable; returns
// TSSM_ERR_UNSUPPORTED (nothing launched) otherwise, so the caller falls back.
template <typename T>
int launch_ssm_forward_tma(const void* u, const void* A, const void* B, const void* C, const void* D, void* y,
                           void* h, const void* poolW, const void* pool_bias, void* pool_out, float pool_inv,
                           int64_t Bsz, int64_t L, int64_t H, cudaStream_t st) {
  constexpr int es = (int)sizeof(T);
  if (!aligned16(u) || !aligned16(A) || !aligned16(B) || !aligned16(C) || (H * es) % 16 != 0 ||
      L >= (int64_t(1) << 31) || H >= (int64_t(1) << 31))
    return TSSM_ERR_UNSUPPORTED;
  const CUtensorMapDataType dt = es == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUtensorMap mA, mU, mB, mC;
  if (!ft_map(&mA, A, dt, es, Bsz, L, H) || !ft_map(&mU, u, dt, es, Bsz, L, H) || !ft_map(&mB, B, dt, es, Bsz, L, H) ||
      !ft_map(&mC, C, dt, es, Bsz, L, H))
    return TSSM_ERR_UNSUPPORTED;
  int* status = device_status_ptr();
  if (!status) return TSSM_ERR_UNSUPPORTED;
  constexpr int bytes = FtLayout<T>::BYTES;
  auto kern = pool_out ? ssm_forward_tma_kernel<T, true> : ssm_forward_tma_kernel<T, false>;
  // The dynamic shared-memory opt-in is per device; it is cheap, so set it on every launch.
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess)
    return check_launch("ssm_forward_tma: set smem attribute");
  dim3 grid((unsigned)cdiv(H, 32), (unsigned)Bsz);
  kern<<<grid, (FT_NW + 1) * 32, bytes, st>>>(mA, mU, mB, mC, (const T*)D, (T*)y, (T*)h, (int)L, (int)H,
                                              (const float*)poolW, (const float*)pool_bias, (float*)pool_out,
                                              pool_inv, status);
  return check_launch("ssm_forward_tma");
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
  // Register-staged fallback: with the pooled head it walks shorter per-warp runs
  // (S=8) with twice the warps: at S=16 the extra accumulator leaves too few
  // registers for the loads in flight (measured: +18 us against +6 us at config-1 size).
  const bool pool = pool_out != nullptr;
  const int nthr = pool ? 32 * 32 : NW * 32;
  if (dtype == TSSM_F32 || dtype == TSSM_BF16) {
    const int r = dtype == TSSM_F32
                      ? launch_ssm_forward_tma<float>(u, A, B, C, D, y, h, poolW, pool_bias, pool_out, pool_inv, Bsz,
                                                      L, H, st)
                      : launch_ssm_forward_tma<__nv_bfloat16>(u, A, B, C, D, y, h, poolW, pool_bias, pool_out,
                                                              pool_inv, Bsz, L, H, st);
    if (r != TSSM_ERR_UNSUPPORTED) return r;   // launched (or failed): otherwise the register-staged kernel
  }
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
  constexpr int S = 8, NW = 32;
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
