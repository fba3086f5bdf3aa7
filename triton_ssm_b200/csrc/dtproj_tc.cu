// Delta-t projection on tcgen05 tensor cores, alone (dt_project_softplus_kernel,
// discretize_kernel.py:165-213) and fused into the ZOH discretisation with one
// dt per (b, t, h) (discretize_kernel.py:38-54).
//
//   acc = dt_raw W + bias,  dt = clamp(log(1 + exp(acc)), dt_min, dt_max)
//   Abar = exp(dt a), Bbar = expm1*(dt a) / (a + 1e-12) B,  a = -exp(A_log[h])
//
// The contraction dt_raw [rows x R] . W [R x H] (R <= 64) is a dense GEMM,
// computed transposed: a tile is [128 channels x 128 rows] of kind::tf32 MMAs
// with the channel block of W (the A operand, M = channels) held in TMEM for the
// CTA's whole run and the dt_raw rows (the B operand, N = rows, K-major as it
// lies in memory) staged by TMA.  The f32 accumulator then has one channel per
// TMEM lane, so an epilogue thread owns one channel and walks rows: each of its
// warp's loads of B and stores of Abar / Bbar covers 32 consecutive channels of
// one row (128 contiguous bytes), issued straight from registers with no
// staging copy, and the next tile's B values are loaded while this tile's are
// used.  tf32 keeps 11 bits of each operand, so both operands are split exactly
// into hi = tf32(x) and lo = x - hi and the tile is the sum of the three
// products hi.hi + hi.lo + lo.hi (the dropped lo.lo term is below 2^-22 of each
// product: f32-accurate, as the 1e-4 parity bar needs).
//
// exp and log are the hardware approximations, exp(x) = 2^(x log2 e) and
// log(u) = log2(u) ln 2 on ex2 / lg2 (relative error near 2^-22), which is also
// how the reference's tl.exp / tl.log compile.  Full tiles take an epilogue
// without per-row checks whose addresses advance by one row per step.
//
// Persistent CTAs (about one per SM) take a contiguous range of tiles, rows
// fastest within a channel block, so a CTA meets at most two channel blocks:
// both are split into TMEM before the first tile.  Roles:
//   warp 16, one thread: TMA loads of the dt_raw rows (two stages) and the 24
//     MMAs of each tile into one of two TMEM accumulators;
//   warps 0-15, thread = (channel lane, 32-row quarter of the tile): W into TMEM,
//     the in-place hi/lo split of each landed dt_raw stage (the next tile's,
//     before this tile's epilogue, so its MMAs overlap the epilogue), and the
//     epilogue.
// Every mbarrier wait is bounded; a wait that gives up sets the device status
// word and every role leaves its loop; the CTA drains its MMAs and loads
// (bounded) and frees TMEM before it exits.
#include <cudaTypedefs.h>

#include "common.cuh"
#include "tcgen05.cuh"
#include "tmap.cuh"

namespace tssm {
namespace {
using namespace sm100;

constexpr int CM = 128;                      // channels per tile (the MMA's M, one per TMEM lane)
constexpr int RN = 128;                      // rows per tile (the MMA's N)
constexpr int KM = 64;                       // largest dt_rank on this path
constexpr int NEPI = 512;                    // epilogue threads: (channel lane, 32-row quarter)
constexpr int NTHR = NEPI + 32;              // + the load / MMA warp
constexpr int NX = 2;                        // dt_raw stages
constexpr uint32_t X_ATOM = RN * 128;        // 16 KB: 128 rows x 32 f32 of K, 128B swizzle
constexpr uint32_t X_PART = 2 * X_ATOM;      // both K atoms
constexpr uint32_t X_STAGE = 2 * X_PART;     // hi (the landed rows, split in place), then lo
constexpr uint32_t OFF_X = 0;
constexpr uint32_t OFF_BAR = OFF_X + NX * X_STAGE;
constexpr int NBAR = 2 * NX + 5;
constexpr uint32_t OFF_MISC = OFF_BAR + NBAR * 8;
constexpr uint32_t SMEM_BYTES = OFF_MISC + 16 + 1024;   // + slack to align the base to 1024
static_assert(SMEM_BYTES <= 232448, "dt-projection shared-memory layout exceeds the per-CTA limit");
// TMEM columns: two f32 accumulators [128 channels x 128 rows], then two W slots
// (hi: 64 K columns, lo: 64 K columns) for the CTA's first and second channel block
constexpr uint32_t TM_D = 0, TM_W = 2 * RN;
constexpr uint32_t TMEM_COLS = 512;

// Nearest tf32 (the low 13 mantissa bits cleared); x - tf32(x) is exact in f32.
__device__ __forceinline__ float tf32_round(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

constexpr float kLog2e = 1.4426950408889634f, kLn2 = 0.6931471805599453f;

// Per-channel constants of an epilogue thread: bias * log2(e), a, a * log2(e)
// and 1 / (a + 1e-12).
struct ChanConst {
  float bsl, a, al, ra;
};

// dt = clamp(softplus(acc + bias)) with exp(v) = 2^(v log2 e) and
// log(u) = log2(u) ln 2 on the hardware approximations.
__device__ __forceinline__ float softplus_clamped(float acc, const ChanConst& k, float dt_min, float dt_max) {
  const float t = fast_exp2(fmaf(acc, kLog2e, k.bsl));
  return fminf(fmaxf(fast_log2(1.0f + t) * kLn2, dt_min), dt_max);
}

// The fused epilogue over 16 of this thread's rows of one tile (one channel),
// rows I0 .. I0+15 of its 32: stores Abar, Bbar (and dt when dto, on the
// checked path only) row by row, and when NEXT loads the next tile's B values
// into the registers this tile has consumed.  CHECK guards rows past the end
// (nv, nvn valid rows of this tile and the next); without it every access is
// unconditional and each stream's address is bumped by one row.
template <bool CHECK, bool NEXT, int I0>
__device__ __forceinline__ void epi_disc_rows(const float (&acc)[16], float (&bv)[32], const ChanConst& k,
                                              float dt_min, float dt_max, float*& p0, float*& p1, float*& pd,
                                              const float*& pb, int64_t H, int nv, int nvn, bool dto) {
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float dtv = softplus_clamped(acc[i], k, dt_min, dt_max);
    const float x = dtv * k.a;
    const float e = fast_exp2(dtv * k.al);
    const float bb = expm1_guard_f32(x, e) * (k.ra * bv[I0 + i]);
    if (!CHECK || I0 + i < nv) {
      __stcs(p0, e);
      __stcs(p1, bb);
      if (CHECK && dto) __stcs(pd, dtv);
    }
    if (NEXT) bv[I0 + i] = (!CHECK || I0 + i < nvn) ? __ldcs(pb) : 0.f;
    p0 += H;
    p1 += H;
    if (CHECK && dto) pd += H;
    if (NEXT) pb += H;
  }
}

template <bool CHECK, int I0>
__device__ __forceinline__ void epi_dt_rows(const float (&acc)[16], const ChanConst& k, float dt_min, float dt_max,
                                            float*& p0, int64_t H, int nv) {
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float dtv = softplus_clamped(acc[i], k, dt_min, dt_max);
    if (!CHECK || I0 + i < nv) __stcs(p0, dtv);
    p0 += H;
  }
}

template <bool DISC>
__global__ void __launch_bounds__(NTHR, 1) dtproj_tc_kernel(
    const __grid_constant__ CUtensorMap tmX, const float* __restrict__ W, const float* __restrict__ bias,
    const float* __restrict__ A_log, const float* __restrict__ B, float* __restrict__ out0,
    float* __restrict__ out1, float* __restrict__ dt_out, int* __restrict__ status, int rows, int H, int R,
    float dt_min, float dt_max, int nrb, int nitems, int per) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* barX = bars + 0;            // [NX] dt_raw stage landed
  uint64_t* barSplit = bars + NX;       // [NX] stage split (and, first time, W in TMEM) (NEPI arrivals)
  uint64_t* barMMA = bars + 2 * NX;     // [2] the tile's MMAs completed
  uint64_t* barTfree = barMMA + 2;      // [2] epilogue done with that accumulator (NEPI arrivals)
  uint64_t* barDrain = barTfree + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + OFF_MISC + 4);
  const int it0 = (int)blockIdx.x * per, it1 = min(nitems, it0 + per);
  const int ntile = it1 - it0;
  const int cb0 = it0 / nrb;   // the CTA's first channel block (its W slot 0)

  if (tid == 0) {
    for (int i = 0; i < NX; ++i) {
      mbar_init(&barX[i], 1);
      mbar_init(&barSplit[i], NEPI);
    }
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
  const int natom = (R + 31) / 32;   // 32-wide K atoms (zero-filled past R)

  if (warp == NEPI / 32) {
    // ============================================================ loads and MMAs
    if (lane == 0 && ntile > 0) {
      prefetch_tmap(&tmX);
      constexpr uint32_t ID = make_idesc_tf32(CM, RN, false, false);
      int x_armed[NX] = {0, 0};
      bool ok = true;
      auto issue_x = [&](int j) {   // dt_raw rows of tile j -> stage j % NX
        const int st = j % NX, it = it0 + j;
        const int m0 = (it % nrb) * RN;
        uint8_t* dst = smem + OFF_X + st * X_STAGE;
        mbar_arrive_expect_tx(&barX[st], (uint32_t)natom * X_ATOM);
        for (int at = 0; at < natom; ++at) tma_load_2d(dst + at * X_ATOM, &tmX, 32 * at, m0, &barX[st]);
        ++x_armed[st];
      };
      issue_x(0);
      if (ntile > 1) issue_x(1);
      for (int j = 0; ok && j < ntile; ++j) {
        const int s = j & 1, st = j % NX;
        if (!(ok = wait(&barSplit[st], (j / NX) & 1, 9501))) break;
        // the split of tile j followed the completion of tile j-1's MMAs: its stage is free
        if (j >= 1 && j + 1 < ntile) issue_x(j + 1);
        if (j >= 2 && !(ok = wait(&barTfree[s], ((j - 2) >> 1) & 1, 9502))) break;
        tc_fence_after();
        const int slot = (it0 + j) / nrb - cb0;
        const uint32_t d = tmem + TM_D + (uint32_t)(s * RN);
        const uint32_t whi = tmem + TM_W + (uint32_t)(slot * 2 * KM), wlo = whi + KM;
        const uint32_t xs = smem_u32(smem + OFF_X + st * X_STAGE);
        const uint64_t dXhi = make_desc_sw128(xs, 16), dXlo = make_desc_sw128(xs + X_PART, 16);
        // W_hi.x_hi + W_hi.x_lo + W_lo.x_hi; A from TMEM (8 K columns per step), x K-major
        // (32 B per step, the second K atom 16 KB further on)
#pragma unroll 1
        for (int p = 0; p < 3; ++p) {
          const uint32_t a = p == 2 ? wlo : whi;
          const uint64_t x = p == 1 ? dXlo : dXhi;
#pragma unroll 1
          for (int at = 0; at < natom; ++at)
            umma_tf32_tmemA_x4(d, a + (uint32_t)(32 * at), x + (uint64_t)((at * X_ATOM) >> 4), ID,
                               (p | at) != 0);
        }
        umma_commit(&barMMA[s]);
      }
      // this thread's MMAs complete before teardown; after a failed wait, the loads it
      // armed complete too (every wait below is bounded)
      umma_commit(barDrain);
      mbar_wait(barDrain, 0, nullptr, 100000000ull);
      if (!ok)
        for (int st = 0; st < NX; ++st)
          if (x_armed[st]) mbar_wait(&barX[st], (x_armed[st] - 1) & 1, nullptr, 100000000ull);
    }
  } else if (ntile > 0) {
    // ============================================================ W, split, epilogue
    const int wq = warp & 3, qt = warp >> 2;   // TMEM lane quarter (channels), row quarter
    const int co = 32 * wq + lane;             // this thread's channel within a block
    const uint32_t tlane = (uint32_t)(32 * wq) << 16;
    const int nslot = (it1 - 1) / nrb - cb0 + 1;   // 1 or 2 (the host checks)
    // W of the CTA's channel blocks, split, into TMEM: lane = channel, column = k;
    // this thread writes its channel's 16 K columns [16 qt, 16 qt + 16)
    ChanConst kc[2];
#pragma unroll
    for (int sl = 0; sl < 2; ++sl) {
      const int c = (cb0 + sl) * CM + co;
      const bool live = sl < nslot && c < H;
      float hi[16], lo[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const int k = 16 * qt + e;
        const float w = (live && k < R) ? __ldg(W + (int64_t)k * H + c) : 0.f;
        hi[e] = tf32_round(w);
        lo[e] = w - hi[e];
      }
      if (sl < nslot) {
        tmem_st16(tmem + tlane + TM_W + (uint32_t)(sl * 2 * KM + 16 * qt), hi);
        tmem_st16(tmem + tlane + TM_W + (uint32_t)(sl * 2 * KM + KM + 16 * qt), lo);
      }
      kc[sl].bsl = (live ? __ldg(bias + c) : 0.f) * kLog2e;
      kc[sl].a = (DISC && live) ? -expf(__ldg(A_log + c)) : -1.f;
      kc[sl].al = kc[sl].a * kLog2e;
      kc[sl].ra = 1.0f / (kc[sl].a + 1e-12f);
    }
    tmem_wait_st();
    // the landed dt_raw rows of tile j, split in place: hi over the rows, lo beside
    // them (elementwise, so the swizzled layout needs no index arithmetic)
    auto split_tile = [&](int j) -> bool {
      const int st = j % NX;
      if (!wait(&barX[st], (j / NX) & 1, 9511)) return false;
      float4* xh = reinterpret_cast<float4*>(smem + OFF_X + st * X_STAGE);
      float4* xl = reinterpret_cast<float4*>(smem + OFF_X + st * X_STAGE + X_PART);
      const int n4 = natom * (int)(X_ATOM / 16);
      for (int q = tid; q < n4; q += NEPI) {
        const float4 x = xh[q];
        float4 h;
        h.x = tf32_round(x.x); h.y = tf32_round(x.y); h.z = tf32_round(x.z); h.w = tf32_round(x.w);
        xh[q] = h;
        xl[q] = make_float4(x.x - h.x, x.y - h.y, x.z - h.z, x.w - h.w);
      }
      fence_proxy_async_smem();   // the stage is read by the tensor core (async proxy)
      tc_fence_before();          // and, the first time, so are the W columns in TMEM
      mbar_arrive(&barSplit[st]);
      return true;
    };
    // B values of this thread's 32 rows of tile j, one per register
    float bv[32];
    // tile j's first row for this thread, its channel, and how many of its 32 rows exist
    auto tile_rc = [&](int j, int& row0, int& c) -> int {
      const int it = it0 + j;
      row0 = (it % nrb) * RN + 32 * qt;
      c = (it / nrb) * CM + co;
      return c < H ? max(0, min(32, rows - row0)) : 0;
    };
    if (DISC) {
      int row0, c;
      const int nv = tile_rc(0, row0, c);
      const float* bp = B + (int64_t)row0 * H + c;
#pragma unroll
      for (int i = 0; i < 32; ++i) bv[i] = i < nv ? __ldcs(bp + (int64_t)i * H) : 0.f;
    }
    const int64_t H64 = H;
    bool ok = split_tile(0);
    for (int j = 0; ok && j < ntile; ++j) {
      const int s = j & 1;
      ok = wait(&barMMA[s], (j >> 1) & 1, 9512);
      if (ok && j + 1 < ntile) {
        tc_fence_after();
        ok = split_tile(j + 1);
      }
      // the warp leaves together: the TMEM loads below are whole-warp instructions
      if (!(ok = __all_sync(0xffffffffu, ok))) break;
      tc_fence_after();
      int row0, c;
      const int nv = tile_rc(j, row0, c);
      const ChanConst& k = ((it0 + j) / nrb - cb0) ? kc[1] : kc[0];
      const int64_t o = (int64_t)row0 * H + c;
      const bool next = DISC && j + 1 < ntile;
      int row0n = 0, cn = 0;
      const int nvn = next ? tile_rc(j + 1, row0n, cn) : 0;
      float* p0 = out0 + o;
      float* p1 = DISC ? out1 + o : nullptr;
      float* pd = (DISC && dt_out) ? dt_out + o : nullptr;
      const float* pb = B + (int64_t)row0n * H + cn;
      const bool fast = nv == 32 && !pd && (nvn == 32 || !next);
      const bool dto = pd != nullptr;
      // the accumulator's 32 columns in two halves of 16 (register budget)
      const uint32_t dcol = tmem + tlane + TM_D + (uint32_t)(s * RN + 32 * qt);
      float acc[16];
      tmem_ld16(dcol, acc);
      tmem_wait_ld();
      if (DISC) {
        if (fast && next) epi_disc_rows<false, true, 0>(acc, bv, k, dt_min, dt_max, p0, p1, pd, pb, H64, nv, nvn, dto);
        else if (fast) epi_disc_rows<false, false, 0>(acc, bv, k, dt_min, dt_max, p0, p1, pd, pb, H64, nv, nvn, dto);
        else epi_disc_rows<true, true, 0>(acc, bv, k, dt_min, dt_max, p0, p1, pd, pb, H64, nv, nvn, dto);
      } else {
        if (fast) epi_dt_rows<false, 0>(acc, k, dt_min, dt_max, p0, H64, nv);
        else epi_dt_rows<true, 0>(acc, k, dt_min, dt_max, p0, H64, nv);
      }
      tmem_ld16(dcol + 16, acc);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&barTfree[s]);   // this thread is done with the accumulator
      if (DISC) {
        if (fast && next) epi_disc_rows<false, true, 16>(acc, bv, k, dt_min, dt_max, p0, p1, pd, pb, H64, nv, nvn, dto);
        else if (fast) epi_disc_rows<false, false, 16>(acc, bv, k, dt_min, dt_max, p0, p1, pd, pb, H64, nv, nvn, dto);
        else epi_disc_rows<true, true, 16>(acc, bv, k, dt_min, dt_max, p0, p1, pd, pb, H64, nv, nvn, dto);
      } else {
        if (fast) epi_dt_rows<false, 16>(acc, k, dt_min, dt_max, p0, H64, nv);
        else epi_dt_rows<true, 16>(acc, k, dt_min, dt_max, p0, H64, nv);
      }
    }
  }
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

}  // namespace

// The tensor-core path: R <= 64 with R % 4 == 0 and a 16-byte aligned dt_raw
// (its rows are TMA-loaded), fewer than 2^31 rows and channels, and at most two
// channel blocks per CTA (H below about 148 x 128 x the row blocks' count per
// CTA).  Returns TSSM_ERR_UNSUPPORTED when those do not hold, so the caller
// takes the CUDA-core kernel instead.
int launch_dtproj_tc(bool disc, const void* dt_raw, const void* W, const void* bias, const void* A_log, const void* B,
                     void* dt_out, void* Abar, void* Bbar, int64_t rows, int64_t H, int64_t R, double dt_min,
                     double dt_max, cudaStream_t st) {
  if (R > KM || R % 4 || !aligned16(dt_raw) || rows >= (int64_t(1) << 31) - RN || H >= (int64_t(1) << 31) - CM)
    return TSSM_ERR_UNSUPPORTED;
  const int64_t nrb = cdiv(rows, RN), ncb = cdiv(H, CM), nitems = nrb * ncb;
  if (nitems >= (int64_t(1) << 31)) return TSSM_ERR_UNSUPPORTED;
  const int64_t per = cdiv(nitems, std::min<int64_t>(nitems, num_sms()));
  if (per > nrb) return TSSM_ERR_UNSUPPORTED;   // a CTA's range would meet a third channel block
  int* status = device_status_ptr();
  if (!status) {
    set_error("dt_project: device status word unavailable");
    return TSSM_ERR_CUDA;
  }
  CUtensorMap mX;
  if (!tmap2d_f32_sw128(&mX, dt_raw, (uint64_t)R, (uint64_t)rows, RN)) return TSSM_ERR_UNSUPPORTED;
  const int grid = (int)cdiv(nitems, per);
  auto kern = disc ? dtproj_tc_kernel<true> : dtproj_tc_kernel<false>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES) != cudaSuccess)
    return check_launch("dt_project: set smem attribute");
  kern<<<grid, NTHR, SMEM_BYTES, st>>>(mX, (const float*)W, (const float*)bias, (const float*)A_log,
                                       (const float*)B, (float*)(disc ? Abar : dt_out), (float*)Bbar,
                                       (float*)(disc ? dt_out : nullptr), status, (int)rows, (int)H, (int)R,
                                       (float)dt_min, (float)dt_max, (int)nrb, (int)nitems, (int)per);
  return check_launch(disc ? "zoh_discretize_dtproj" : "dt_project_softplus");
}

}  // namespace tssm
