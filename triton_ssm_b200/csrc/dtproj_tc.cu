// Delta-t projection on tcgen05 tensor cores, alone (dt_project_softplus_kernel,
// discretize_kernel.py:165-213) and fused into the ZOH discretisation with one
// dt per (b, t, h) (discretize_kernel.py:38-54).
//
//   acc = dt_raw W + bias,  dt = clamp(log(1 + exp(acc)), dt_min, dt_max)
//   Abar = exp(dt a), Bbar = expm1*(dt a) / (a + 1e-12) B,  a = -exp(A_log[h])
//
// The contraction dt_raw [rows x R] . W [R x H] (R <= 64) is a dense GEMM: it
// runs as [128 rows x 64 channels] tiles of kind::tf32 MMAs with f32
// accumulators in TMEM, the dt_raw operand read from TMEM.  tf32 keeps 11 bits of each operand, so every operand
// is split exactly into hi = tf32(x) and lo = x - hi, and the tile is the sum of
// the three products hi.hi + hi.lo + lo.hi (the dropped lo.lo term is below
// 2^-22 of each product: f32-accurate, as the 1e-4 parity bar needs).
//
// Persistent CTAs (one per SM) walk a contiguous range of tiles, channels
// fastest, so a 128-row block of dt_raw is loaded and split once per 16
// channel tiles.  Roles:
//   warp 16, one thread: TMA loads of the dt_raw block, the W slab and (fused
//     form) the B tile two tiles ahead (three buffers), and the 24 MMAs of each
//     tile into one of two TMEM accumulators;
//   warps 0-15 (one thread per tile row and 16-channel quarter): the hi/lo split of
//     each newly loaded operand (dt_raw into TMEM columns, W transposed to
//     K-major shared-memory tiles), then the
//     epilogue of the tile's MMAs -- bias, softplus, clamp, the ZOH arithmetic
//     against the swizzled B tile -- into 128B-swizzled staging tiles that TMA
//     stores write out.
// Every mbarrier wait is bounded; a wait that gives up sets the device status
// word and every role leaves its loop; the CTA drains its MMAs, loads and
// stores (bounded) and frees TMEM before it exits.
#include <cudaTypedefs.h>

#include "common.cuh"
#include "tcgen05.cuh"
#include "tmap.cuh"

namespace tssm {
#ifdef TSSM_DTPROJ_TRACE
// Debug-only phase timestamps (globaltimer, ns) of CTA 0: [tile][event].
__device__ unsigned long long g_dtp_trace[64 * 16];
#define DTP_TRACE(tile, ev)                                                                   \
  do {                                                                                        \
    if (blockIdx.x == 0 && (tile) < 64) g_dtp_trace[(tile) * 16 + (ev)] = globaltimer_ns();   \
  } while (0)
#else
#define DTP_TRACE(tile, ev) \
  do {                      \
  } while (0)
#endif
namespace {
using namespace sm100;

constexpr int TM = 128;                     // rows per tile (the MMA's M)
constexpr int TN = 64;                      // channels per tile (the MMA's N)
constexpr int KM = 64;                      // largest dt_rank on this path
constexpr int NEPI = 512;                   // epilogue threads: one per (tile row, 16-channel quarter)
constexpr int NTHR = NEPI + 32;             // + the load / MMA warp
constexpr int NBB = 3;                      // B-tile buffers (loads run two tiles ahead)
constexpr uint32_t A_RAW = TM * KM * 4;     // 32 KB: the dt_raw block as landed, two [128 x 128 B] K atoms
constexpr uint32_t W_PART = KM * TN * 4;    // 16 KB: two [64 rows x 128 B] tiles (landed: per 32 channels; split: per 32 K)
constexpr uint32_t HALF = TM * 32 * 4;      // 16 KB: one [128 x 32] f32 tile, 128B swizzle
constexpr uint32_t OFF_A = 0;
constexpr uint32_t OFF_WHI = OFF_A + A_RAW;
constexpr uint32_t OFF_WLO = OFF_WHI + W_PART;
constexpr uint32_t OFF_B = OFF_WLO + W_PART;         // [NBB buffers][2 halves] of the B tile
constexpr uint32_t OFF_O = OFF_B + NBB * 2 * HALF;   // staging: [2 halves][out0, out1]
constexpr uint32_t OFF_COL = OFF_O + 4 * HALF;       // [2][3][TN]: bias, a, 1/(a + 1e-12)
constexpr uint32_t OFF_BAR = OFF_COL + 2 * 3 * TN * 4;
constexpr int NBAR = 14;
constexpr uint32_t OFF_MISC = OFF_BAR + NBAR * 8;
constexpr uint32_t SMEM_BYTES = OFF_MISC + 16 + 1024;   // + slack to align the base to 1024
static_assert(SMEM_BYTES <= 232448, "dt-projection shared-memory layout exceeds the per-CTA limit");
// TMEM columns: two f32 accumulators, then the dt_raw block's hi and lo parts (A operand)
constexpr uint32_t TM_D = 0, TM_AHI = 2 * TN, TM_ALO = TM_AHI + KM;
constexpr uint32_t TMEM_COLS = 256;

// Nearest tf32 (the low 13 mantissa bits cleared); x - tf32(x) is exact in f32.
__device__ __forceinline__ float tf32_round(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

template <bool DISC>
__global__ void __launch_bounds__(NTHR, 1) dtproj_tc_kernel(
    const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
    const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmO0,
    const __grid_constant__ CUtensorMap tmO1, const float* __restrict__ bias, const float* __restrict__ A_log,
    int* __restrict__ status, int H, int R, float dt_min, float dt_max, int ntn, int nitems) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* barA = bars + 0;        // dt_raw block landed
  uint64_t* barW = bars + 1;        // W slab landed
  uint64_t* barB = bars + 2;        // [NBB] B tile landed
  uint64_t* barSplit = bars + 5;    // operands split, channel constants written (NEPI arrivals)
  uint64_t* barMMA = bars + 6;      // [2] the tile's MMAs completed
  uint64_t* barBfree = bars + 8;    // [NBB] epilogue done with that B buffer (NEPI arrivals)
  uint64_t* barTfree = bars + 11;   // [2] epilogue done with that accumulator (NEPI arrivals)
  uint64_t* barDrain = bars + 13;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + OFF_MISC + 4);
  const int per = (nitems + (int)gridDim.x - 1) / (int)gridDim.x;
  const int it0 = (int)blockIdx.x * per, it1 = min(nitems, it0 + per);

  if (tid == 0) {
    mbar_init(barA, 1);
    mbar_init(barW, 1);
    for (int i = 0; i < NBB; ++i) {
      mbar_init(&barB[i], 1);
      mbar_init(&barBfree[i], NEPI);
    }
    mbar_init(barSplit, NEPI);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&barMMA[i], 1);
      mbar_init(&barTfree[i], NEPI);
    }
    mbar_init(barDrain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  auto wait = [&](uint64_t* bar, uint32_t parity, int code) -> bool {
    if (mbar_wait(bar, parity, abort_flag)) return true;
    if (!*abort_flag) {
      *abort_flag = 1;
      atomicExch(status, code);
    }
    return false;
  };
  auto tile_mn = [&](int it, int& m0, int& n0) {
    const int m = it / ntn;
    m0 = m * TM;
    n0 = (it - m * ntn) * TN;
    return m;
  };

  if (warp == NEPI / 32) {
    // ============================================================ loads and MMAs
    if (lane == 0 && it0 < it1) {
      prefetch_tmap(&tmX);
      prefetch_tmap(&tmW);
      if (DISC) prefetch_tmap(&tmB);
      constexpr uint32_t ID = make_idesc_tf32(TM, TN, false, false);
      const int natom = (R + 31) / 32;   // 32-wide K atoms (zero-filled past R)
      int last_m = -1, a_armed = 0, w_armed = 0, b_armed[NBB] = {0, 0, 0};
      bool ok = true;
      auto issue_b = [&](int it) -> bool {   // B tile of tile it -> buffer (it - it0) % NBB
        const int jb = it - it0, bb = jb % NBB;
        if (jb >= NBB && !wait(&barBfree[bb], ((jb - NBB) / NBB) & 1, 9501)) return false;
        int m0, n0;
        tile_mn(it, m0, n0);
        mbar_arrive_expect_tx(&barB[bb], 2 * HALF);
        tma_load_2d(smem + OFF_B + bb * 2 * HALF, &tmB, n0, m0, &barB[bb]);
        tma_load_2d(smem + OFF_B + bb * 2 * HALF + HALF, &tmB, n0 + 32, m0, &barB[bb]);
        ++b_armed[bb];
        return true;
      };
      if (DISC) ok = issue_b(it0);
      for (int it = it0; ok && it < it1; ++it) {
        const int j = it - it0, s = j & 1;
        int m0, n0;
        const int m = tile_mn(it, m0, n0);
        DTP_TRACE(j, 0);
        if (DISC && it + 1 < it1 && !(ok = issue_b(it + 1))) break;   // two tiles ahead of its epilogue
        DTP_TRACE(j, 1);
        // the previous tile's MMAs (and the split before them) are done with W and the dt_raw block
        if (j >= 1 && !(ok = wait(&barMMA[(j - 1) & 1], ((j - 1) >> 1) & 1, 9502))) break;
        DTP_TRACE(j, 2);
        if (m != last_m) {
          mbar_arrive_expect_tx(barA, A_RAW);
          tma_load_2d(smem + OFF_A, &tmX, 0, m0, barA);
          tma_load_2d(smem + OFF_A + A_RAW / 2, &tmX, 32, m0, barA);
          ++a_armed;
          last_m = m;
        }
        mbar_arrive_expect_tx(barW, W_PART);
        tma_load_2d(smem + OFF_WHI, &tmW, n0, 0, barW);
        tma_load_2d(smem + OFF_WHI + W_PART / 2, &tmW, n0 + 32, 0, barW);
        ++w_armed;
        if (!(ok = wait(barSplit, j & 1, 9503))) break;
        if (j >= 2 && !(ok = wait(&barTfree[s], ((j - 2) >> 1) & 1, 9504))) break;
        DTP_TRACE(j, 3);
        tc_fence_after();
        const uint32_t d = tmem + TM_D + (uint32_t)(s * TN);
        const uint64_t dWhi = make_desc_sw128(smem_u32(smem + OFF_WHI), 16);
        const uint64_t dWlo = make_desc_sw128(smem_u32(smem + OFF_WLO), 16);
        // hi.hi + hi.lo + lo.hi; A from TMEM (8 columns per K step), W K-major (32 B per
        // K step, second 32-wide K atom 8 KB further on)
#pragma unroll 1
        for (int p = 0; p < 3; ++p) {
          const uint32_t acol = tmem + (p == 2 ? TM_ALO : TM_AHI);
          const uint64_t w = p == 1 ? dWlo : dWhi;
#pragma unroll 1
          for (int at = 0; at < natom; ++at)
            umma_tf32_tmemA_x4(d, acol + (uint32_t)(32 * at), w + (uint64_t)((at * (W_PART / 2)) >> 4), ID,
                               (p | at) != 0);
        }
        umma_commit(&barMMA[s]);
        DTP_TRACE(j, 4);
      }
      // this thread's MMAs complete before teardown; after a failed wait, the loads it
      // armed complete too (every wait below is bounded)
      umma_commit(barDrain);
      mbar_wait(barDrain, 0, nullptr, 100000000ull);
      if (!ok) {
        if (a_armed) mbar_wait(barA, (a_armed - 1) & 1, nullptr, 100000000ull);
        if (w_armed) mbar_wait(barW, (w_armed - 1) & 1, nullptr, 100000000ull);
        for (int b = 0; b < NBB; ++b)
          if (b_armed[b]) mbar_wait(&barB[b], (b_armed[b] - 1) & 1, nullptr, 100000000ull);
      }
    }
  } else {
    // ============================================================ split + epilogue
    // Warps w, w+4, w+8, w+12 share TMEM lanes 32*(w%4) ..: thread = (tile row r,
    // quarter qt: 16 channels of the epilogue, 16 K columns of the A split).  After
    // the MMAs of tile j complete, the operands of tile j+1 are split first, so its
    // MMAs run while tile j's epilogue computes.
    int last_m = -1, a_seen = 0;
    const int r = tid & (TM - 1), qt = tid / TM;
    const uint32_t tlane = (uint32_t)((warp & 3) * 32) << 16;
    auto split_tile = [&](int it) -> bool {
      const int j = it - it0, s = j & 1;
      int m0, n0;
      const int m = tile_mn(it, m0, n0);
      if (tid == 0) DTP_TRACE(j, 5);
      if (m != last_m) {
        // this thread's 16 K columns of row r: hi and lo into the A columns of TMEM
        if (!wait(barA, a_seen & 1, 9511)) return false;
        ++a_seen;
        last_m = m;
        const uint8_t* row = smem + OFF_A + (qt >> 1) * (A_RAW / 2) + r * 128;
        float hi[16], lo[16];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint32_t q = (uint32_t)((qt & 1) * 4 + c);
          const float4 x = *reinterpret_cast<const float4*>(row + (((q ^ ((uint32_t)r & 7u)) & 7u) << 4));
          const float xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            hi[c * 4 + e] = tf32_round(xs[e]);
            lo[c * 4 + e] = xs[e] - hi[c * 4 + e];
          }
        }
        tmem_st16(tmem + tlane + TM_AHI + (uint32_t)(qt * 16), hi);
        tmem_st16(tmem + tlane + TM_ALO + (uint32_t)(qt * 16), lo);
        tmem_wait_st();
      }
      if (tid == 0) DTP_TRACE(j, 6);
      if (!wait(barW, j & 1, 9512)) return false;
      if (tid == 0) DTP_TRACE(j, 7);
      {
        // W as landed ([k][32 n] 128-byte rows per 32-channel block) -> hi/lo in K-major
        // tiles ([n][32 k] 128-byte rows per 32-wide K atom), the layout the MMA reads
        // (an MN-major tf32 operand read back as zeros here); the slab is read into
        // registers first so the hi tile can be written over it
        constexpr int WE = KM * TN / NEPI;   // elements of the slab per thread
        float wv[WE];
#pragma unroll
        for (int e = 0; e < WE; ++e) {
          const int idx = tid + e * NEPI, k = idx & 63, nn = idx >> 6;
          const uint32_t so = (uint32_t)(nn >> 5) * (W_PART / 2) + (uint32_t)k * 128u +
                              (((((uint32_t)(nn & 31) >> 2) ^ ((uint32_t)k & 7u)) & 7u) << 4) + ((uint32_t)nn & 3u) * 4u;
          wv[e] = *reinterpret_cast<const float*>(smem + OFF_WHI + so);
        }
        named_bar_sync(2, NEPI);
#pragma unroll
        for (int e = 0; e < WE; ++e) {
          const int idx = tid + e * NEPI, k = idx & 63, nn = idx >> 6;
          const uint32_t d = (uint32_t)(k >> 5) * (W_PART / 2) + (uint32_t)nn * 128u +
                             (((((uint32_t)(k & 31) >> 2) ^ ((uint32_t)nn & 7u)) & 7u) << 4) + ((uint32_t)k & 3u) * 4u;
          const float h = tf32_round(wv[e]);
          *reinterpret_cast<float*>(smem + OFF_WHI + d) = h;
          *reinterpret_cast<float*>(smem + OFF_WLO + d) = wv[e] - h;
        }
      }
      float* col = reinterpret_cast<float*>(smem + OFF_COL) + s * 3 * TN;
      if (tid < TN) {
        const int h = n0 + tid;
        col[tid] = h < H ? bias[h] : 0.f;
        if (DISC) {
          const float a = h < H ? -expf(A_log[h]) : -1.f;
          col[TN + tid] = a;
          col[2 * TN + tid] = 1.0f / (a + 1e-12f);
        }
      }
      fence_proxy_async_smem();   // the W tiles are read by the tensor core (async proxy)
      tc_fence_before();          // and so are the A columns written to TMEM
      named_bar_sync(2, NEPI);    // channel constants visible to every epilogue thread
      mbar_arrive(barSplit);
      if (tid == 0) DTP_TRACE(j, 8);
      return true;
    };
    auto epilogue_tile = [&](int it) -> bool {
      const int j = it - it0, s = j & 1, bb = j % NBB;
      int m0, n0;
      tile_mn(it, m0, n0);
      if (DISC && !wait(&barB[bb], (j / NBB) & 1, 9514)) return false;
      if (tid == 0) DTP_TRACE(j, 10);
      const float* col = reinterpret_cast<const float*>(smem + OFF_COL) + s * 3 * TN;
      float acc[16];
      tmem_ld16(tmem + tlane + TM_D + (uint32_t)(s * TN + qt * 16), acc);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&barTfree[s]);   // this thread is done with the accumulator
      // the previous tile's stores have finished reading the staging tiles
      if (tid == 0) bulk_wait_read<0>();
      named_bar_sync(1, NEPI);
      if (tid == 0) DTP_TRACE(j, 11);
      const int hf = qt >> 1;               // 32-channel half (one swizzled [128 x 128 B] tile)
      uint8_t* o0 = smem + OFF_O + hf * 2 * HALF;
      uint8_t* o1 = o0 + HALF;
      const uint8_t* bt = smem + OFF_B + bb * 2 * HALF + hf * HALF;
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {
        const uint32_t q = (uint32_t)((qt & 1) * 4 + q4);   // 16-byte chunk of the 128-byte row
        const uint32_t off = (uint32_t)r * 128u + (((q ^ ((uint32_t)r & 7u)) & 7u) << 4);
        float bv[4] = {0.f, 0.f, 0.f, 0.f};
        if (DISC) {
          const float4 t = *reinterpret_cast<const float4*>(bt + off);
          bv[0] = t.x; bv[1] = t.y; bv[2] = t.z; bv[3] = t.w;
        }
        float y0[4], y1[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int c = qt * 16 + q4 * 4 + e;
          const float v = acc[q4 * 4 + e] + col[c];
          const float dtv = fminf(fmaxf(logf(1.0f + expf(v)), dt_min), dt_max);
          if (DISC) {
            const float x = dtv * col[TN + c];
            const float ex = expf(x);
            y0[e] = ex;
            y1[e] = expm1_guard_f32(x, ex) * col[2 * TN + c] * bv[e];
          } else {
            y0[e] = dtv;
            y1[e] = 0.f;
          }
        }
        *reinterpret_cast<float4*>(o0 + off) = make_float4(y0[0], y0[1], y0[2], y0[3]);
        if (DISC) *reinterpret_cast<float4*>(o1 + off) = make_float4(y1[0], y1[1], y1[2], y1[3]);
      }
      if (DISC) mbar_arrive(&barBfree[bb]);   // done with the B tile
      fence_proxy_async_smem();
      named_bar_sync(1, NEPI);
      if (tid == 0) DTP_TRACE(j, 12);
      if (tid == 0) {
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) {
          uint8_t* p0 = smem + OFF_O + h2 * 2 * HALF;
          tma_store_2d(&tmO0, p0, n0 + 32 * h2, m0);
          if (DISC) tma_store_2d(&tmO1, p0 + HALF, n0 + 32 * h2, m0);
        }
        bulk_commit();
      }
      return true;
    };
    bool ok = it0 >= it1 || split_tile(it0);
    for (int it = it0; ok && it < it1; ++it) {
      const int j = it - it0, s = j & 1;
      if (!(ok = wait(&barMMA[s], (j >> 1) & 1, 9513))) break;
      if (tid == 0) DTP_TRACE(j, 9);
      tc_fence_after();
      if (it + 1 < it1 && !(ok = split_tile(it + 1))) break;
      ok = epilogue_tile(it);
    }
    if (tid == 0) bulk_wait<0>();
  }
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

}  // namespace

#ifdef TSSM_DTPROJ_TRACE
extern "C" int tssm_debug_read_dtp_trace(unsigned long long* out, int n) {
  return cudaMemcpyFromSymbol(out, g_dtp_trace, sizeof(unsigned long long) * (n < 1024 ? n : 1024)) == cudaSuccess ? 0 : 3;
}
#endif

// The tensor-core path: R <= 64, rows of dt_raw, W, B and the outputs 16-byte
// aligned (R % 4 == 0, H % 4 == 0, 16-byte aligned bases), and no dt output in
// the fused form.  Returns TSSM_ERR_UNSUPPORTED when those do not hold, so the
// caller takes the CUDA-core kernel instead.
int launch_dtproj_tc(bool disc, const void* dt_raw, const void* W, const void* bias, const void* A_log, const void* B,
                     void* dt_out, void* Abar, void* Bbar, int64_t rows, int64_t H, int64_t R, double dt_min,
                     double dt_max, cudaStream_t st) {
  if (R > KM || R % 4 || H % 4 || (disc && dt_out) || !aligned16(dt_raw) || !aligned16(W) ||
      (disc ? !(aligned16(B) && aligned16(Abar) && aligned16(Bbar)) : !aligned16(dt_out)) ||
      rows >= (int64_t(1) << 31) || H >= (int64_t(1) << 31))
    return TSSM_ERR_UNSUPPORTED;
  int* status = device_status_ptr();
  if (!status) {
    set_error("dt_project: device status word unavailable");
    return TSSM_ERR_CUDA;
  }
  CUtensorMap mX, mW, mB, mO0, mO1;
  void* o0 = disc ? Abar : dt_out;
  void* o1 = disc ? Bbar : dt_out;
  const void* bsrc = disc ? B : dt_out;
  if (!tmap2d_f32_sw128(&mX, dt_raw, (uint64_t)R, (uint64_t)rows, TM) ||
      !tmap2d_f32_sw128(&mW, W, (uint64_t)H, (uint64_t)R, KM) ||
      !tmap2d_f32_sw128(&mB, bsrc, (uint64_t)H, (uint64_t)rows, TM) ||
      !tmap2d_f32_sw128(&mO0, o0, (uint64_t)H, (uint64_t)rows, TM) ||
      !tmap2d_f32_sw128(&mO1, o1, (uint64_t)H, (uint64_t)rows, TM)) {
    return TSSM_ERR_UNSUPPORTED;   // e.g. a tensor narrower than one box: the CUDA-core kernel takes it
  }
  const int64_t ntm = cdiv(rows, TM), ntn = cdiv(H, TN), nitems = ntm * ntn;
  TSSM_REQUIRE(nitems < (int64_t(1) << 31), "dt_project: size exceeds the grid");
  const int grid = (int)std::min<int64_t>(nitems, num_sms());
  auto kern = disc ? dtproj_tc_kernel<true> : dtproj_tc_kernel<false>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES) != cudaSuccess)
    return check_launch("dt_project: set smem attribute");
  kern<<<grid, NTHR, SMEM_BYTES, st>>>(mX, mW, mB, mO0, mO1, (const float*)bias, (const float*)A_log, status,
                                       (int)H, (int)R, (float)dt_min, (float)dt_max, (int)ntn, (int)nitems);
  return check_launch(disc ? "zoh_discretize_dtproj" : "dt_project_softplus");
}

}  // namespace tssm
