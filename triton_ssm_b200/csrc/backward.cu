// Backward passes of the diagonal scan and of the ZOH discretisation.
//
// ssm_backward (replaces ssm_scan.py:127-231 / :267-289): for the forward
//     h_t = A_t h_{t-1} + B_t u_t ,  y_t = C_t h_t + D u_t
// the reference propagates only the state path (D is a constant there):
//     dH_t = C_t dY_t + A_{t+1} dH_{t+1}      (dH_{L-1} = C_{L-1} dY_{L-1})
//     du = B dH,  dA = h_{t-1} dH,  dB = u dH,  dC = dY h.
// One pass, same shape as the forward kernel but walking the sequence from the
// end: a CTA owns 32 consecutive channels of one batch row (one lane each, so
// every step is one coalesced 128-byte row segment per warp); warp w holds
// steps [w*S, (w+1)*S) of a super-segment of NW*S steps, folds them into a
// reverse (a, x) aggregate, takes the carry from the warps after it, and
// replays its steps writing du, dA, dB, dC.  Every input is read from HBM once
// (A_{t+1} and h_{t-1} at a run's edge come from the neighbouring run's rows,
// which the cache holds).  When the rows are TMA-addressable the same reverse
// scan runs with its inputs staged by TMA (ssm_backward_tma_kernel): a producer
// warp keeps 64-step tiles of A (shifted one step), u, B, C, dY and a 65-row h
// tile (from t0-1) in flight while 16 compute warps work on the tile after it.
//
// zoh_discretize_bwd (replaces discretize_kernel.py:97-162): per (b, t, h)
//     a = -exp(A_log), x = dt a, e = exp(x), em1 = guarded exp(x)-1 (bf16 form, :134)
//     ddt   += dAbar a Abar + dBbar e B                       (summed over h)
//     dA_log += (dAbar dt Abar + dBbar (e dt a - em1)/(a^2+1e-18) B) (-(-a))  (summed over b, t)
//     dB     = dBbar em1 / (a + 1e-12)
// A CTA owns a block of (b, t) rows and all of H, so each row's ddt is reduced
// inside the CTA (no store/atomic race as in :159-162); dA_log gets one atomic
// add per (CTA, h).
#include <cudaTypedefs.h>

#include "common.cuh"
#include "tcgen05.cuh"
#include "tmap.cuh"

namespace tssm {
namespace {

template <typename T, int S, int NW>
__global__ void __launch_bounds__(NW * 32, 1) ssm_backward_kernel(
    const T* __restrict__ u, const T* __restrict__ A, const T* __restrict__ B, const T* __restrict__ C,
    const T* __restrict__ h, const T* __restrict__ dY, T* __restrict__ du, T* __restrict__ dA,
    T* __restrict__ dB, T* __restrict__ dC, int64_t L, int64_t H) {
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
  const T* __restrict__ hb = h + base;
  const T* __restrict__ dYb = dY + base;
  T* __restrict__ dub = du + base;
  T* __restrict__ dAb = dA + base;
  T* __restrict__ dBb = dB + base;
  T* __restrict__ dCb = dC + base;
  const int Hi = (int)H;
  const int Li = (int)L;
  constexpr int SEG = NW * S;
  float carry = 0.f;   // dH at the first step after the current super-segment (0 past the end)
  for (int t0 = ((Li - 1) / SEG) * SEG; t0 >= 0; t0 -= SEG) {
    const int ts = t0 + warp * S;
    // coefficient A_{t+1} and input C_t dY_t of the reverse recurrence dH_t = A_{t+1} dH_{t+1} + C_t dY_t;
    // the replay's B, u, h are loaded here too, so all of a run's loads are in flight together
    float a[S], x[S], dy[S], bb[S], uu[S], hh[S];
#pragma unroll
    for (int i = 0; i < S; ++i) {
      const int t = ts + i;
      if (valid && t < Li) {
        const int off = t * Hi;
        a[i] = t + 1 < Li ? ldf(Ab + off + Hi) : 0.f;
        dy[i] = ldf(dYb + off);
        x[i] = ldf(Cb + off) * dy[i];
        bb[i] = ldf(Bb + off);
        uu[i] = ldf(ub + off);
        hh[i] = ldf(hb + off);
      } else {
        a[i] = 1.f;
        x[i] = 0.f;
        dy[i] = 0.f;
        bb[i] = uu[i] = hh[i] = 0.f;
      }
    }
    // h_{ts-1}, the state before this run (for dA of its first step)
    const float hbefore = (valid && ts >= 1 && ts - 1 < Li) ? ldf(hb + (ts - 1) * Hi) : 0.f;
    float ag_a = 1.f, ag_x = 0.f;   // dH_ts = ag_a * dH_{ts+S} + ag_x
#pragma unroll
    for (int i = S - 1; i >= 0; --i) {
      ag_x = a[i] * ag_x + x[i];
      ag_a *= a[i];
    }
    s_a[warp][lane] = ag_a;
    s_x[warp][lane] = ag_x;
    __syncthreads();
    float dh = carry;
    for (int w = NW - 1; w > warp; --w) dh = s_a[w][lane] * dh + s_x[w][lane];
    // replay from the end of this warp's steps
#pragma unroll
    for (int i = S - 1; i >= 0; --i) {
      const int t = ts + i;
      dh = a[i] * dh + x[i];
      const float hprev = i > 0 ? hh[i - 1] : hbefore;
      if (valid && t < Li) {
        const int off = t * Hi;
        stf(dub + off, bb[i] * dh);
        stf(dBb + off, uu[i] * dh);
        stf(dCb + off, dy[i] * hh[i]);
        stf(dAb + off, hprev * dh);
      }
    }
    if (warp == 0) s_carry[lane] = dh;   // dH at step t0
    __syncthreads();
    carry = s_carry[lane];
  }
}


// ---------------------------------------------------------------- TMA-staged ssm_backward
constexpr int BT_CH = 64;             // steps per staged tile
constexpr int BT_NW = 16;             // compute warps
constexpr int BT_S = BT_CH / BT_NW;   // steps per compute warp and tile
constexpr uint32_t BT_BAR = 1;        // named barrier of the compute warps

template <typename T>
struct BtLayout {
  static constexpr int STAGES = sizeof(T) == 4 ? 4 : 8;
  static constexpr int TILE = BT_CH * 32 * (int)sizeof(T);                      // [BT_CH][32] tile
  static constexpr int HTILE = ((BT_CH + 1) * 32 * (int)sizeof(T) + 127) / 128 * 128;   // h: rows t0-1 .. t0+63
  static constexpr int STAGE = 5 * TILE + HTILE;                                // A(+1), u, B, C, dY, h
  static constexpr int OFF_AGG = STAGES * STAGE;                                // [2][2][BT_NW][32] f32
  static constexpr int OFF_BAR = OFF_AGG + 2 * 2 * BT_NW * 32 * 4;
  static constexpr int OFF_MISC = OFF_BAR + 2 * STAGES * 8;                     // abort flag, issued, consumed
  static constexpr int BYTES = OFF_MISC + 16 + 128;
  static_assert(BYTES <= 232448, "ssm_backward_tma shared-memory layout exceeds the per-CTA limit");
};

// CTA = (32 channels, one batch row), walking the tiles from the end of the
// sequence; warp BT_NW is the TMA producer.  A is loaded one step ahead (row r
// of the tile is A_{t+1}; A_L reads as zero) and h one step behind (row r is
// h_{t-1}, row r+1 is h_t; h_{-1} reads as zero).
template <typename T>
__global__ void __launch_bounds__((BT_NW + 1) * 32, 1) ssm_backward_tma_kernel(
    const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmU,
    const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmC,
    const __grid_constant__ CUtensorMap tmY, const __grid_constant__ CUtensorMap tmH, T* __restrict__ du,
    T* __restrict__ dA, T* __restrict__ dB, T* __restrict__ dC, int L, int H, int* __restrict__ status) {
  using LY = BtLayout<T>;
  constexpr int ST = LY::STAGES;
  extern __shared__ uint8_t bt_raw[];
  uint8_t* smem = bt_raw + ((128u - (sm100::smem_u32(bt_raw) & 127u)) & 127u);
  float* agg = reinterpret_cast<float*>(smem + LY::OFF_AGG);   // [buf][a|x][warp][lane]
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + LY::OFF_BAR);
  uint64_t* empty = full + ST;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + LY::OFF_MISC);
  int* issued = reinterpret_cast<int*>(smem + LY::OFF_MISC + 4);
  int* consumed = reinterpret_cast<int*>(smem + LY::OFF_MISC + 8);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int ch0 = blockIdx.x * 32, b = blockIdx.y;
  const int nt = (L + BT_CH - 1) / BT_CH;
  if (threadIdx.x == 0) {
    for (int i = 0; i < ST; ++i) {
      sm100::mbar_init(&full[i], 1);
      sm100::mbar_init(&empty[i], BT_NW);
    }
    *abort_flag = 0;
    *issued = 0;
    *consumed = 0;
    sm100::fence_mbar_init();
  }
  __syncthreads();

  if (warp == BT_NW) {
    // ------------------------------------------------------------ producer (last tile first)
    if (lane == 0) {
      sm100::prefetch_tmap(&tmA);
      sm100::prefetch_tmap(&tmU);
      sm100::prefetch_tmap(&tmB);
      sm100::prefetch_tmap(&tmC);
      sm100::prefetch_tmap(&tmY);
      sm100::prefetch_tmap(&tmH);
      int k = 0;
      for (; k < nt; ++k) {
        const int s = k % ST;
        const int t0 = (nt - 1 - k) * BT_CH;
        if (k >= ST && !sm100::mbar_wait(&empty[s], ((k / ST) - 1) & 1, abort_flag)) {
          if (!*abort_flag) {
            *abort_flag = 1;
            atomicExch(status, 2101);
          }
          break;
        }
        uint8_t* st = smem + s * LY::STAGE;
        sm100::mbar_arrive_expect_tx(&full[s], 5 * LY::TILE + (BT_CH + 1) * 32 * (int)sizeof(T));
        sm100::tma_load_3d(st, &tmA, ch0, t0 + 1, b, &full[s]);
        sm100::tma_load_3d(st + LY::TILE, &tmU, ch0, t0, b, &full[s]);
        sm100::tma_load_3d(st + 2 * LY::TILE, &tmB, ch0, t0, b, &full[s]);
        sm100::tma_load_3d(st + 3 * LY::TILE, &tmC, ch0, t0, b, &full[s]);
        sm100::tma_load_3d(st + 4 * LY::TILE, &tmY, ch0, t0, b, &full[s]);
        sm100::tma_load_3d(st + 5 * LY::TILE, &tmH, ch0, t0 - 1, b, &full[s]);
      }
      *issued = k;
    }
  } else {
    // ------------------------------------------------------------ compute warps
    const int ch = ch0 + lane;
    const bool valid = ch < H;
    const int64_t base = (int64_t)b * L * H + ch;
    float carry = 0.f;   // dH at the first step after the current tile (0 past the end)
    int k = 0;
    for (; k < nt; ++k) {
      const int s = k % ST, pb = k & 1;
      const int t0 = (nt - 1 - k) * BT_CH;
      const bool bad = !sm100::mbar_wait(&full[s], (k / ST) & 1, abort_flag);
      const T* tA = reinterpret_cast<const T*>(smem + s * LY::STAGE);   // A_{t+1}
      const T* tU = tA + BT_CH * 32;
      const T* tB = tU + BT_CH * 32;
      const T* tC = tB + BT_CH * 32;
      const T* tY = tC + BT_CH * 32;
      const T* tH = tY + BT_CH * 32;                                      // row r: h_{t-1}, row r+1: h_t
      const int r0 = warp * BT_S;
      float a[BT_S], x[BT_S];
      float ag_a = 1.f, ag_x = 0.f;   // dH at this warp's first step = ag_a * dH after its steps + ag_x
      if (!bad) {
#pragma unroll
        for (int i = 0; i < BT_S; ++i) {
          const int r = (r0 + i) * 32 + lane;
          if (valid && t0 + r0 + i < L) {
            a[i] = ldf(tA + r);
            x[i] = ldf(tC + r) * ldf(tY + r);
          } else {
            a[i] = 1.f;
            x[i] = 0.f;
          }
        }
#pragma unroll
        for (int i = BT_S - 1; i >= 0; --i) {
          ag_x = a[i] * ag_x + x[i];
          ag_a *= a[i];
        }
        agg[((pb * 2 + 0) * BT_NW + warp) * 32 + lane] = ag_a;
        agg[((pb * 2 + 1) * BT_NW + warp) * 32 + lane] = ag_x;
      } else if (!*abort_flag) {
        *abort_flag = 1;
        atomicExch(status, 2102);
      }
      if (sm100::named_bar_or(BT_BAR, BT_NW * 32, bad)) break;
      // dH after this warp's steps (folded over the warps after it) and the carry into
      // the previous tile, from all warps' aggregates
      float wa[BT_NW], wx[BT_NW];
#pragma unroll
      for (int w = 0; w < BT_NW; ++w) {
        wa[w] = agg[((pb * 2 + 0) * BT_NW + w) * 32 + lane];
        wx[w] = agg[((pb * 2 + 1) * BT_NW + w) * 32 + lane];
      }
      float dh = carry, nxt = carry;
#pragma unroll
      for (int w = BT_NW - 1; w >= 0; --w) {
        if (w == warp) dh = nxt;
        nxt = wa[w] * nxt + wx[w];
      }
      carry = nxt;
#pragma unroll
      for (int i = BT_S - 1; i >= 0; --i) {
        dh = a[i] * dh + x[i];
        const int t = t0 + r0 + i;
        if (valid && t < L) {
          const int r = (r0 + i) * 32 + lane;
          const int64_t off = base + (int64_t)t * H;
          stf(du + off, ldf(tB + r) * dh);
          stf(dB + off, ldf(tU + r) * dh);
          stf(dC + off, ldf(tY + r) * ldf(tH + r + 32));
          stf(dA + off, ldf(tH + r) * dh);
        }
      }
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(&empty[s]);
    }
    if (threadIdx.x == 0) *consumed = k;
  }
  __syncthreads();
  if (threadIdx.x == 0 && *abort_flag) {
    for (int c = *consumed; c < *issued; ++c) sm100::mbar_wait(&full[c % ST], (c / ST) & 1, nullptr, 100000000ull);
  }
}

// 3-D map over [Bsz][L][H] (H contiguous), box {32 channels, rows steps, 1}, no swizzle.
inline bool bt_map(CUtensorMap* m, const void* base, CUtensorMapDataType dt, int esize, int64_t Bsz, int64_t L,
                   int64_t H, uint32_t rows) {
  auto fn = tmap_encode_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {(cuuint64_t)H, (cuuint64_t)L, (cuuint64_t)Bsz};
  cuuint64_t strides[2] = {(cuuint64_t)(H * esize), (cuuint64_t)(L * H * esize)};
  cuuint32_t box[3] = {32, rows, 1};
  cuuint32_t es[3] = {1, 1, 1};
  return fn(m, dt, 3, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Launches the TMA-staged backward when the tensors are TMA-addressable; returns
// TSSM_ERR_UNSUPPORTED (nothing launched) otherwise.
template <typename T>
int launch_ssm_backward_tma(const void* u, const void* A, const void* B, const void* C, const void* h, const void* dY,
                            void* du, void* dA, void* dB, void* dC, int64_t Bsz, int64_t L, int64_t H,
                            cudaStream_t st) {
  constexpr int es = (int)sizeof(T);
  if (!aligned16(u) || !aligned16(A) || !aligned16(B) || !aligned16(C) || !aligned16(h) || !aligned16(dY) ||
      (H * es) % 16 != 0 || L >= (int64_t(1) << 31) - BT_CH || H >= (int64_t(1) << 31))
    return TSSM_ERR_UNSUPPORTED;
  const CUtensorMapDataType dt = es == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUtensorMap mA, mU, mB, mC, mY, mH;
  if (!bt_map(&mA, A, dt, es, Bsz, L, H, BT_CH) || !bt_map(&mU, u, dt, es, Bsz, L, H, BT_CH) ||
      !bt_map(&mB, B, dt, es, Bsz, L, H, BT_CH) || !bt_map(&mC, C, dt, es, Bsz, L, H, BT_CH) ||
      !bt_map(&mY, dY, dt, es, Bsz, L, H, BT_CH) || !bt_map(&mH, h, dt, es, Bsz, L, H, BT_CH + 1))
    return TSSM_ERR_UNSUPPORTED;
  int* status = device_status_ptr();
  if (!status) return TSSM_ERR_UNSUPPORTED;
  constexpr int bytes = BtLayout<T>::BYTES;
  auto kern = ssm_backward_tma_kernel<T>;
  // The dynamic shared-memory opt-in is per device; it is cheap, so set it on every launch.
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess)
    return check_launch("ssm_backward_tma: set smem attribute");
  dim3 grid((unsigned)cdiv(H, 32), (unsigned)Bsz);
  kern<<<grid, (BT_NW + 1) * 32, bytes, st>>>(mA, mU, mB, mC, mY, mH, (T*)du, (T*)dA, (T*)dB, (T*)dC, (int)L,
                                              (int)H, status);
  return check_launch("ssm_backward_tma");
}

constexpr int DBWD_THREADS = 256;
constexpr int DBWD_ROWS = 64;   // at most this many (b, t) rows per CTA

// VEC: H % 4 == 0 and 16-byte aligned rows, four channels per thread per pass.
template <bool VEC>
__global__ void __launch_bounds__(DBWD_THREADS) zoh_discretize_bwd_kernel(
    const float* __restrict__ A_log, const float* __restrict__ B, const float* __restrict__ dt,
    const float* __restrict__ Abar, const float* __restrict__ dAbar, const float* __restrict__ dBbar,
    float* __restrict__ dA_log, float* __restrict__ dB, float* __restrict__ ddt, int64_t R, int64_t H) {
  constexpr int NWARP = DBWD_THREADS / 32;
  constexpr int PER = VEC ? 4 : 1;
  __shared__ float s_ddt[DBWD_ROWS][NWARP];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // an even split of the rows over the grid (a whole number of CTAs per SM, so
  // every SM streams the same bytes)
  const int64_t r0 = R * blockIdx.x / gridDim.x;
  const int nrows = (int)(R * (blockIdx.x + 1) / gridDim.x - r0);
  for (int i = tid; i < DBWD_ROWS * NWARP; i += DBWD_THREADS) (&s_ddt[0][0])[i] = 0.f;
  __syncthreads();
  // Chunks of DBWD_THREADS*PER channels; every thread runs every chunk (the ddt
  // shuffle reduction needs whole warps), channels past H contribute nothing.
  for (int64_t hc = 0; hc < H; hc += DBWD_THREADS * PER) {
    const int64_t h0 = hc + (int64_t)tid * PER;
    const bool act = h0 < H;   // VEC: H % 4 == 0, so all PER channels exist
    // per channel: a, and the reciprocals 1/(a^2+1e-18), 1/(a+1e-12) that replace a
    // division per element (within an ulp of the quotients)
    float a[PER], na[PER], acc[PER], r2[PER], r1[PER];
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      na[k] = act ? expf(A_log[h0 + k]) : 1.f;
      a[k] = -na[k];
      acc[k] = 0.f;
      r2[k] = 1.0f / (a[k] * a[k] + 1e-18f);
      r1[k] = 1.0f / (a[k] + 1e-12f);
    }
    // four rows per step: their loads go out together, then four independent reductions
    for (int r4 = 0; r4 < nrows; r4 += 4) {
      float vb[4][PER], vab[4][PER], vda[4][PER], vdb[4][PER], dtv[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int r = r4 + j < nrows ? r4 + j : nrows - 1;   // duplicate rows are computed, not used
        const int64_t row = r0 + r;
        dtv[j] = dt[row];
        if (act) {
          const int64_t off = row * H + h0;
          if (VEC) {
            const float4 q0 = *reinterpret_cast<const float4*>(B + off);
            const float4 q1 = *reinterpret_cast<const float4*>(Abar + off);
            const float4 q2 = *reinterpret_cast<const float4*>(dAbar + off);
            const float4 q3 = *reinterpret_cast<const float4*>(dBbar + off);
            const float t0[4] = {q0.x, q0.y, q0.z, q0.w}, t1[4] = {q1.x, q1.y, q1.z, q1.w};
            const float t2[4] = {q2.x, q2.y, q2.z, q2.w}, t3[4] = {q3.x, q3.y, q3.z, q3.w};
#pragma unroll
            for (int k = 0; k < PER; ++k) {
              vb[j][k] = t0[k];
              vab[j][k] = t1[k];
              vda[j][k] = t2[k];
              vdb[j][k] = t3[k];
            }
          } else {
            vb[j][0] = B[off];
            vab[j][0] = Abar[off];
            vda[j][0] = dAbar[off];
            vdb[j][0] = dBbar[off];
          }
        } else {
#pragma unroll
          for (int k = 0; k < PER; ++k) vb[j][k] = vab[j][k] = vda[j][k] = vdb[j][k] = 0.f;
        }
      }
      float part[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        part[j] = 0.f;
        const bool use = act && r4 + j < nrows;
        float out[PER];
#pragma unroll
        for (int k = 0; k < PER; ++k) {
          const float x = dtv[j] * a[k];
          const float e = expf(x);
          const float em1 = expm1_guard_bf16(x, e);
          part[j] += vda[j][k] * a[k] * vab[j][k] + vdb[j][k] * e * vb[j][k];
          const float num = (e * dtv[j] * a[k] - em1) * r2[k];
          const float da = vda[j][k] * dtv[j] * vab[j][k] + vdb[j][k] * num * vb[j][k];
          if (use) acc[k] += da * (-na[k]);
          out[k] = vdb[j][k] * em1 * r1[k];
        }
        if (!use) part[j] = 0.f;
        if (use) {
          const int64_t off = (r0 + r4 + j) * H + h0;
          if (VEC)
            *reinterpret_cast<float4*>(dB + off) = make_float4(out[0], out[1], out[2], out[3]);
          else
            dB[off] = out[0];
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
        for (int j = 0; j < 4; ++j) part[j] += __shfl_xor_sync(0xffffffffu, part[j], o);
      }
      if (lane == 0) {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (r4 + j < nrows) s_ddt[r4 + j][warp] += part[j];
      }
    }
    if (act) {
#pragma unroll
      for (int k = 0; k < PER; ++k) atomicAdd(dA_log + h0 + k, acc[k]);
    }
  }
  __syncthreads();
  if (tid < nrows) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < NWARP; ++w) s += s_ddt[tid][w];
    ddt[r0 + tid] = s;
  }
}

}  // namespace
}  // namespace tssm

extern "C" int tssm_ssm_backward(const void* u, const void* A, const void* B, const void* C, const void* h,
                                 const void* dY, void* du, void* dA, void* dB, void* dC, int64_t Bsz,
                                 int64_t L, int64_t H, int dtype, tssm_stream_t stream) {
  using namespace tssm;
  TSSM_REQUIRE(Bsz >= 0 && L >= 0 && H >= 0, "ssm_backward: negative size");
  if (Bsz * L * H == 0) return TSSM_OK;
  TSSM_REQUIRE(u && A && B && C && h && dY && du && dA && dB && dC, "ssm_backward: null pointer");
  TSSM_REQUIRE(Bsz <= 65535, "ssm_backward: batch %lld exceeds 65535", (long long)Bsz);
  TSSM_REQUIRE(L * H < (int64_t(1) << 31), "ssm_backward: L*H must be < 2^31 per batch row");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == TSSM_F32 || dtype == TSSM_BF16) {
    const int r = dtype == TSSM_F32
                      ? launch_ssm_backward_tma<float>(u, A, B, C, h, dY, du, dA, dB, dC, Bsz, L, H, st)
                      : launch_ssm_backward_tma<__nv_bfloat16>(u, A, B, C, h, dY, du, dA, dB, dC, Bsz, L, H, st);
    if (r != TSSM_ERR_UNSUPPORTED) return r;   // launched (or failed): otherwise the register-staged kernel
  }
  // runs of 4 steps, 32 warps: the six inputs of a run are loaded before its replay
  constexpr int S = 4, NW = 32;
  dim3 grid((unsigned)cdiv(H, 32), (unsigned)Bsz);
  if (dtype == TSSM_F32) {
    ssm_backward_kernel<float, S, NW><<<grid, NW * 32, 0, st>>>(
        (const float*)u, (const float*)A, (const float*)B, (const float*)C, (const float*)h, (const float*)dY,
        (float*)du, (float*)dA, (float*)dB, (float*)dC, L, H);
  } else if (dtype == TSSM_BF16) {
    using bf = __nv_bfloat16;
    ssm_backward_kernel<bf, S, NW><<<grid, NW * 32, 0, st>>>(
        (const bf*)u, (const bf*)A, (const bf*)B, (const bf*)C, (const bf*)h, (const bf*)dY, (bf*)du, (bf*)dA,
        (bf*)dB, (bf*)dC, L, H);
  } else {
    set_error("ssm_backward: dtype must be f32 or bf16 (got %d)", dtype);
    return TSSM_ERR_INVALID;
  }
  return check_launch("ssm_backward");
}

extern "C" int tssm_zoh_discretize_bwd(const void* A_log, const void* B, const void* dt, const void* Abar,
                                       const void* dAbar, const void* dBbar, void* dA_log, void* dB, void* ddt,
                                       int64_t Bsz, int64_t T, int64_t H, tssm_stream_t stream) {
  using namespace tssm;
  TSSM_REQUIRE(Bsz >= 0 && T >= 0 && H >= 0, "zoh_discretize_bwd: negative size");
  TSSM_REQUIRE(!(H > 0 && !dA_log), "zoh_discretize_bwd: null dA_log");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // dA_log is a fresh gradient (the reference accumulates into a caller-zeroed buffer)
  if (H > 0 && cudaMemsetAsync(dA_log, 0, (size_t)H * sizeof(float), st) != cudaSuccess)
    return check_launch("zoh_discretize_bwd: clear dA_log");
  const int64_t R = Bsz * T;
  if (R == 0) return TSSM_OK;
  TSSM_REQUIRE(A_log && B && dt && Abar && dAbar && dBbar && dB && ddt, "zoh_discretize_bwd: null pointer");
  if (H == 0) return cudaMemsetAsync(ddt, 0, (size_t)R * sizeof(float), st) == cudaSuccess
                         ? TSSM_OK
                         : check_launch("zoh_discretize_bwd: clear ddt");
  const bool vec = (H % 4 == 0) && aligned16(B) && aligned16(Abar) && aligned16(dAbar) && aligned16(dBbar) &&
                   aligned16(dB);
  // two CTAs per SM, or more when that would put over DBWD_ROWS rows in one CTA
  const int64_t nct = std::min<int64_t>(R, std::max<int64_t>(2 * num_sms(), cdiv(R, DBWD_ROWS)));
  TSSM_REQUIRE(nct < (int64_t(1) << 31), "zoh_discretize_bwd: too many rows");
  const unsigned grid = (unsigned)nct;
  if (vec)
    zoh_discretize_bwd_kernel<true><<<grid, DBWD_THREADS, 0, st>>>(
        (const float*)A_log, (const float*)B, (const float*)dt, (const float*)Abar, (const float*)dAbar,
        (const float*)dBbar, (float*)dA_log, (float*)dB, (float*)ddt, R, H);
  else
    zoh_discretize_bwd_kernel<false><<<grid, DBWD_THREADS, 0, st>>>(
        (const float*)A_log, (const float*)B, (const float*)dt, (const float*)Abar, (const float*)dAbar,
        (const float*)dBbar, (float*)dA_log, (float*)dB, (float*)ddt, R, H);
  return check_launch("zoh_discretize_bwd");
}
