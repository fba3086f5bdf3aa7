// Multi-head chunked SSD scan on tcgen05 tensor cores (configs 2 and 4).
//
// Replaces the multi-head chunked scan of multihead_ssm_kernel.py:19-187 (local
// scan, carry scan, output) for the outer-product state h[b,h,p,n]:
//     h_t = exp(dt_t*A_h) h_{t-1} + beta_t x_t (x) B_t ,  y_t = h_t C_t + D x_t
// with beta_t = dt_t (Euler, multihead_ssm_kernel.py:73) or the ZOH factor of
// discretize_kernel.py:50-54.
//
// One CTA walks one (b, h) stream in chunks of Q = 64 tokens; nothing is
// written to HBM but y (and the optional final state).  Per chunk, with
// s_i = sum_{k<=i} dt_k*A_h (inclusive, within the chunk):
//   MMA1  G    = C B^T                                   [Q x Q]  (K = N)
//   mask  M    = G o exp(s_i - s_j) beta_j [j<=i]  -> bf16 smem
//   MMA2  Y1   = M X                                     [Q x P]  (K = Q)
//   MMA4  S^T  = (diag(exp(s_last - s_j) beta_j) B)^T X  [N x P]  (K = Q)
//   MMA3  Y2   = C H^T   (H = state after the previous chunk, bf16)  (K = N)
//   y_i = Y1_i + exp(s_i) Y2_i + D x_i ;  H <- exp(s_last) H + S   (f32 in registers)
//
// Warp roles (512 threads, one CTA per SM):
//   warp 12     producer: TMA loads of X, B, C (128B swizzle) into a STAGES-deep ring,
//               and, in the same non-blocking event loop, the MMA1 issue;
//   warp 15     decay: streams dt (cp.async) and writes each chunk's decay prefix
//               sums and input coefficients into a DSL-slot ring of its own, so it
//               runs several chunks ahead of the consumers;
//   warp 13     MMA4 and MMA2 issue from one non-blocking event loop (MMA4 waits only
//               for diag(w) B of chunk c and for the state group to have read S of
//               chunk c-2);
//   warp 14     MMA3 issue.  Issuing a tcgen05.mma costs the issuing thread tens of
//               cycles, so the issue work is spread over three threads and each MMA
//               goes out as soon as its inputs are ready;
//   warps 4-7   mask group: G -> M (bf16) and diag(w) B (MMA4's A operand) for chunk c;
//   warps 0-3   state group: H <- exp(s_last) H + S in registers and the bf16 copy
//               of H for the next MMA3 -- the only serial dependence between chunks,
//               kept free of every other job;
//   warps 8-11  output group: y = Y1 + exp(s_i) Y2 + D x into a swizzled tile, one
//               TMA store per chunk.
// G, Y1, Y2 and S are double-buffered in TMEM (8 x 64 = 512 columns), M, diag(w) B,
// the bf16 state tile and the y tile in shared memory.  Every mbarrier wait is
// time-bounded; a wait that gives up sets the device status word and the CTA
// exits cleanly (after its in-flight MMAs, loads and stores complete).
#include <cudaTypedefs.h>

#include "common.cuh"
#include "tcgen05.cuh"
#include "tmap.cuh"

namespace tssm {
#ifdef TSSM_SSD_TRACE
// Debug-only phase timestamps (clock64) of CTA (0,0): [chunk][event].
__device__ unsigned long long g_ssd_trace[64 * 32];
#define SSD_TRACE(chunk, ev)                                                         \
  do {                                                                               \
    if (blockIdx.x == 0 && blockIdx.y == 0 && (chunk) < 64) g_ssd_trace[(chunk) * 32 + (ev)] = clock64(); \
  } while (0)
#else
#define SSD_TRACE(chunk, ev) \
  do {                       \
  } while (0)
#endif
namespace {
using namespace sm100;

constexpr int Q = 64;          // tokens per chunk
constexpr int P = 64;          // head dim
constexpr int TILE = 8192;     // bytes of a [64 x 64] bf16 tile
constexpr int NTHREADS = 512;  // STATE 0-3, MSK 4-7, OUT 8-11, TMA+MMA1 12, MMA4+MMA2 13, MMA3 14, decay 15
constexpr int DT_RING = 4;     // raw dt slots, private to the decay warp
constexpr uint32_t TMEM_COLS = 512;
constexpr float LOG2E = 1.4426950408889634f;
__host__ __device__ constexpr uint32_t col_g(int k) { return 0u + 64u * k; }
__host__ __device__ constexpr uint32_t col_y1(int k) { return 128u + 64u * k; }
__host__ __device__ constexpr uint32_t col_y2(int k) { return 256u + 64u * k; }
__host__ __device__ constexpr uint32_t col_s(int k) { return 384u + 64u * k; }

// Named barriers (0 is __syncthreads).
constexpr uint32_t BAR_STATE = 1, BAR_MSK = 2, BAR_OUT = 3;

template <int NST>
struct Layout {
  static constexpr int NB = NST / 64;                  // 64-wide blocks of B and C along n
  // Who writes diag(w) B (MMA4's A operand).  N=64: the state group, two chunks ahead
  // (the 6-stage ring holds that B tile long before), which keeps the mask group's
  // per-chunk work short.  N=128: the mask group for the chunk it masks, because with
  // 3 stages the B tile two chunks ahead is not loaded yet when the state group runs.
  static constexpr bool BHAT_IN_STATE = NST == 64;
  static constexpr int STAGE_BYTES = TILE * (1 + 2 * NB);
  static constexpr int STAGES = NST == 64 ? 6 : 3;     // X, B, C ring
  static constexpr int DSL = NST == 64 ? 8 : 4;        // decay-data ring
  static constexpr int HS_BYTES = NST * 128;           // state tile: NST rows (n) x 64 p, MN-major
  static constexpr int OFF_BH = STAGES * STAGE_BYTES;  // 2 x diag(w) B (MMA4's A operand)
  static constexpr int OFF_MT = OFF_BH + 2 * NB * TILE; // 2 mask tiles
  static constexpr int OFF_HS = OFF_MT + 2 * TILE;     // 2 bf16 state tiles
  static constexpr int OFF_YS = OFF_HS + 2 * HS_BYTES; // 2 y tiles (TMA store sources)
  static constexpr int OFF_SMALL = OFF_YS + 2 * TILE;  // per decay slot: s, v, w [64] + exp2(s_last)
  static constexpr int SMALL_STRIDE = 224 * 4;        // s [0,72), v [72,144), w [144,208), e_last at 208
  static constexpr int OFF_RAW = OFF_SMALL + DSL * SMALL_STRIDE;  // DT_RING x 64 raw dt
  static constexpr int OFF_DSK = OFF_RAW + DT_RING * 64 * 4;
  static constexpr int OFF_BAR = OFF_DSK + 64 * 4;
  static constexpr int NBAR = 2 * STAGES + 2 * DSL + 20 + 3;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;  // tmem slot, abort flag, issued, consumed
  static constexpr int BYTES = OFF_MISC + 32 + 1024;   // + slack to align the base to 1024
  static_assert(BYTES <= 232448, "SSD shared-memory layout exceeds the per-CTA limit");
};

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ void unpack_bf16x8(uint4 v, float (&f)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&w[k]);
    f[2 * k] = __low2float(b);
    f[2 * k + 1] = __high2float(b);
  }
}

template <int NST, bool ZOH>
__global__ void __launch_bounds__(NTHREADS, 1) ssd_chunk_scan_kernel(
    const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_b,
    const __grid_constant__ CUtensorMap tm_c, const __grid_constant__ CUtensorMap tm_y,
    const float* __restrict__ dt, const float* __restrict__ A_log, const float* __restrict__ Dskip,
    const float* __restrict__ h0, float* __restrict__ h_last, float* __restrict__ decay_log2,
    int* __restrict__ status, int L, int H) {
  using LY = Layout<NST>;
  constexpr int NB = LY::NB;
  constexpr int ST = LY::STAGES;
  constexpr int DSL = LY::DSL;
  extern __shared__ uint8_t smem_raw[];
  // Offset the __shared__ array itself (no integer round trip), so the compiler
  // keeps every access below in the shared address space (LDS/STS, not generic).
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int h = blockIdx.x, b = blockIdx.y;
  const int nchunks = (L + Q - 1) / Q;
  float* dsk = reinterpret_cast<float*>(smem + LY::OFF_DSK);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + LY::OFF_BAR);
  uint64_t* full = bars;               // [ST]  TMA bytes of X, B, C landed
  uint64_t* empty = full + ST;         // [ST]  stage released (output group + MMA4 complete)
  uint64_t* dfull = empty + ST;        // [DSL] decay data written
  uint64_t* dempty = dfull + DSL;      // [DSL] decay slot released (state + output groups)
  uint64_t* gfull = dempty + DSL;      // [2]   MMA1 done
  uint64_t* gfree = gfull + 2;         // [2]   G read by the mask group
  uint64_t* bready = gfull + 4;        // [2]   diag(w) B written (state or mask group, see BHAT_IN_STATE)
  uint64_t* mready = gfull + 6;        // [2]   M written
  uint64_t* sfull = gfull + 8;         // [2]   MMA4 done
  uint64_t* y1full = gfull + 10;       // [2]   MMA2 done
  uint64_t* y2full = gfull + 12;       // [2]   MMA3 done
  uint64_t* sfree = gfull + 14;        // [2]   S read by the state group
  uint64_t* yfree = gfull + 16;        // [2]   Y1, Y2 read by the output group
  uint64_t* hready = gfull + 18;       // [2]   bf16 state tile for MMA3 written
  uint64_t* drain = gfull + 20;        // [3]   final commit of each MMA issuer (1: warp 13, 2: warp 14)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + LY::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + LY::OFF_MISC + 4);
  int* issued = reinterpret_cast<int*>(smem + LY::OFF_MISC + 8);
  int* consumed = reinterpret_cast<int*>(smem + LY::OFF_MISC + 12);

  auto stage_ptr = [&](int s) { return smem + s * LY::STAGE_BYTES; };
  auto small_ptr = [&](int d) { return reinterpret_cast<float*>(smem + LY::OFF_SMALL + d * LY::SMALL_STRIDE); };
  auto mt_ptr = [&](int k) { return smem + LY::OFF_MT + k * TILE; };
  auto bh_ptr = [&](int k) { return smem + LY::OFF_BH + k * NB * TILE; };
  auto hs_ptr = [&](int k) { return smem + LY::OFF_HS + k * LY::HS_BYTES; };
  auto ys_ptr = [&](int k) { return smem + LY::OFF_YS + k * TILE; };

  if (tid == 0) {
    for (int s = 0; s < ST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 2);
    }
    for (int d = 0; d < DSL; ++d) {
      mbar_init(&dfull[d], 1);
      mbar_init(&dempty[d], 2);
    }
    for (int k = 0; k < 23; ++k) mbar_init(&gfull[k], 1);
    *abort_flag = 0;
    *issued = 0;
    *consumed = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  if (tid < 64) dsk[tid] = Dskip[(int64_t)h * P + tid];
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  auto fail = [&](int code) {
    *abort_flag = 1;
    atomicExch(status, code);
  };
  // Waits for this thread's own MMAs before the CTA tears down (bounded).
  auto drain_mmas = [&](uint64_t* bar) {
    umma_commit(bar);
    mbar_wait(bar, 0, nullptr, 100000000ull);
  };

  if (warp == 12) {
    // ================================================================ producer
    // Only TMA loads, so a released stage is refilled as soon as it frees up.
    if (lane == 0) {
      prefetch_tmap(&tm_x);
      prefetch_tmap(&tm_b);
      prefetch_tmap(&tm_c);
      prefetch_tmap(&tm_y);
      int pc = 0;   // next chunk to load
      for (; pc < nchunks; ++pc) {
        const int s = pc % ST;
        if (pc >= ST && !mbar_wait(&empty[s], ((pc / ST) - 1) & 1, abort_flag)) {
          if (!*abort_flag) fail(1001);
          break;
        }
        SSD_TRACE(pc, 0);
        uint8_t* st = stage_ptr(s);
        mbar_arrive_expect_tx(&full[s], LY::STAGE_BYTES);
        tma_load_3d(st, &tm_x, h * P, pc * Q, b, &full[s]);
#pragma unroll
        for (int nb = 0; nb < NB; ++nb) {
          tma_load_3d(st + TILE * (1 + nb), &tm_b, h * NST + nb * 64, pc * Q, b, &full[s]);
          tma_load_3d(st + TILE * (1 + NB + nb), &tm_c, h * NST + nb * 64, pc * Q, b, &full[s]);
        }
      }
      *issued = pc;
    }
  } else if (warp == 15) {
    // ================================================================ decay warp
    // dt streams into a private ring with cp.async, DT_RING-1 chunks ahead; the
    // per-chunk decay data goes to its own DSL-slot ring, so this warp runs up to
    // DSL chunks ahead of the output group.
    const float* dtp = dt + (int64_t)b * L * H + h;
    float* raw = reinterpret_cast<float*>(smem + LY::OFF_RAW);
    const float a = -expf(__ldg(A_log + h));
    const float a2 = a * LOG2E;
    auto issue_dt = [&](int i) {
      if (i < nchunks) {
        float* slot = raw + (i % DT_RING) * 64;
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int t = i * Q + 2 * lane + e;
          if (t < L)
            asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(slot + 2 * lane + e)),
                         "l"(dtp + (int64_t)t * H)
                         : "memory");
          else
            slot[2 * lane + e] = 0.f;
        }
      }
      asm volatile("cp.async.commit_group;" ::: "memory");
    };
    for (int i = 0; i < DT_RING - 1; ++i) issue_dt(i);
    float total_log2 = 0.f;   // log2 of the whole-sequence decay
    for (int c = 0; c < nchunks; ++c) {
      const int ds = c % DSL;
      int bad = 0;   // decided by lane 0, broadcast so the warp stays converged
      if (lane == 0) {
        if (c >= DSL && !mbar_wait(&dempty[ds], ((c / DSL) - 1) & 1, abort_flag)) {
          if (!*abort_flag) fail(1010);
          bad = 1;
        }
        bad |= *abort_flag;
      }
      if (__shfl_sync(0xffffffffu, bad, 0)) break;
      if (lane == 0) SSD_TRACE(c, 19);
      issue_dt(c + DT_RING - 1);
      asm volatile("cp.async.wait_group %0;" ::"n"(DT_RING - 1) : "memory");
      const float* rs = raw + (c % DT_RING) * 64;
      const float d0 = rs[2 * lane], d1 = rs[2 * lane + 1];
      // decay prefix sums (log2 domain) and input coefficients of chunk c
      const float l0 = d0 * a2, l1 = d1 * a2;
      const float pair = l0 + l1;
      float incl = pair;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const float v = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += v;
      }
      const float s0 = incl - pair + l0, s1 = incl;
      const float slast = __shfl_sync(0xffffffffu, incl, 31);
      total_log2 += slast;
      float b0, b1;
      if (ZOH) {
        const float x0 = d0 * a, x1 = d1 * a;
        b0 = zoh_coeff(x0, expf(x0), a);
        b1 = zoh_coeff(x1, expf(x1), a);
      } else {
        b0 = d0;
        b1 = d1;
      }
      // per token: s_j (log2 domain), v_j (below), and the state weight w_j = exp2(s_last - s_j) beta_j;
      // tokens 32..63 sit 4 floats further on, so the two column halves of a warp read different banks
      float* sm = small_ptr(ds);
      const int pad = lane >= 16 ? 4 : 0;
      sm[2 * lane + pad] = s0;
      sm[2 * lane + 1 + pad] = s1;
      // v_j = exp2(s_ref(j) - s_j) * beta_j with ref(j) the last token of j's 4-token
      // sub-block: the mask entry is G_ij * exp2(s_i - s_ref(J)) * v_j
      const float sref = __shfl_sync(0xffffffffu, s1, lane | 1);
      sm[72 + 2 * lane + pad] = exp2f(sref - s0) * b0;
      sm[72 + 2 * lane + 1 + pad] = exp2f(sref - s1) * b1;
      sm[144 + 2 * lane] = exp2f(slast - s0) * b0;
      sm[144 + 2 * lane + 1] = exp2f(slast - s1) * b1;
      if (lane == 0) sm[208] = exp2f(slast);
      __syncwarp();
      if (lane == 0) {
        SSD_TRACE(c, 1);
        mbar_arrive(&dfull[ds]);
      }
    }
    asm volatile("cp.async.wait_all;" ::: "memory");   // no copy may outlive the loop
    if (decay_log2 && lane == 0 && !*abort_flag) decay_log2[(int64_t)b * H + h] = total_log2;
  } else if (warp == 13) {
    // ================================================================ MMA2 + MMA4 issuer
    // Two independent issue streams in one non-blocking event loop, so neither waits
    // behind the other (MMA2, on the way to the output, goes first when both are ready):
    //   MMA2 (Y1 = M X) once M of chunk k2 is written and the output group has read
    //        Y1 of chunk k2-2;
    //   MMA4 (S^T = (diag(w) B)^T X) once diag(w) B of chunk k4 is written and the state
    //        group has read S of chunk k4-2 out of TMEM buffer k4&1.
    // A commit covers every earlier MMA of this thread, so each barrier below is reached
    // no earlier than the MMA it names completes.
    if (lane == 0) {
      constexpr uint32_t ID_MM = make_idesc_bf16(NST, 64, true, true);
      constexpr uint32_t ID_KM = make_idesc_bf16(64, 64, false, true);
      int k4 = 0, k2 = 0;
      uint64_t t_prog = globaltimer_ns();
      while (k4 < nchunks || k2 < nchunks) {
        bool prog = false;
        if (k2 < nchunks) {
          const int s = k2 % ST, kb = k2 & 1;
          if (mbar_test(&mready[kb], (k2 >> 1) & 1) && (k2 < 2 || mbar_test(&yfree[kb], ((k2 - 2) >> 1) & 1)) &&
              mbar_test(&full[s], (k2 / ST) & 1)) {
            tc_fence_after();
            SSD_TRACE(k2, 10);
            const uint64_t dX = make_desc_sw128(smem_u32(stage_ptr(s)), TILE);
            const uint64_t dM = make_desc_sw128(smem_u32(mt_ptr(kb)), 16);
            umma_bf16_x4(tmem + col_y1(kb), dM, dM + 2, dM + 4, dM + 6, dX, dX + 128, dX + 256, dX + 384, ID_KM, 0);
            umma_commit(&y1full[kb]);
            SSD_TRACE(k2, 11);
            ++k2;
            prog = true;
          }
        }
        if (k4 < nchunks) {
          const int s = k4 % ST, kb = k4 & 1;
          if (mbar_test(&bready[kb], (k4 >> 1) & 1) &&
              (k4 < 2 || mbar_test(&sfree[kb], ((k4 - 2) >> 1) & 1)) && mbar_test(&full[s], (k4 / ST) & 1)) {
            tc_fence_after();
            SSD_TRACE(k4, 8);
            const uint64_t dX = make_desc_sw128(smem_u32(stage_ptr(s)), TILE);
            const uint64_t dBh = make_desc_sw128(smem_u32(bh_ptr(kb)), TILE);
            umma_bf16_x4(tmem + col_s(kb), dBh, dBh + 128, dBh + 256, dBh + 384, dX, dX + 128, dX + 256, dX + 384,
                         ID_MM, 0);
            umma_commit(&sfull[kb]);
            umma_commit(&empty[s]);   // MMA4 is the last reader of X apart from the output group
            SSD_TRACE(k4, 9);
            ++k4;
            prog = true;
          }
        }
        if (prog) {
          t_prog = globaltimer_ns();
        } else {
          if (*abort_flag) break;
          if (globaltimer_ns() - t_prog > 2000000000ull) {
            fail(1004);
            break;
          }
        }
      }
      drain_mmas(&drain[1]);
    }
  } else if (warp == 14) {
    // ================================================================ MMA1 + MMA3 issuer
    //   MMA1 (G = C B^T) once the tiles of chunk k1 have landed and the mask group has
    //        read G of chunk k1-2;
    //   MMA3 (Y2 = C H^T) once the state tile of chunk k3-1 is written and the output
    //        group has read Y2 of chunk k3-2.
    if (lane == 0) {
      constexpr uint32_t ID_KK = make_idesc_bf16(64, 64, false, false);
      constexpr uint32_t ID_KM = make_idesc_bf16(64, 64, false, true);
      int k1 = 0, k3 = 0;
      uint64_t t_prog = globaltimer_ns();
      while (k1 < nchunks || k3 < nchunks) {
        bool prog = false;
        if (k1 < nchunks && mbar_test(&full[k1 % ST], (k1 / ST) & 1) &&
            (k1 < 2 || mbar_test(&gfree[k1 & 1], ((k1 - 2) >> 1) & 1))) {
          const int s = k1 % ST, kb = k1 & 1;
          tc_fence_after();
          SSD_TRACE(k1, 2);
          const uint32_t X = smem_u32(stage_ptr(s));
          const uint64_t dB = make_desc_sw128(X + TILE, 16), dC = make_desc_sw128(X + TILE * (1 + NB), 16);
#pragma unroll
          for (int kb4 = 0; kb4 < NST / 64; ++kb4) {   // 64-wide K blocks (tiles) of n
            const uint64_t ko = (uint64_t)(kb4 * TILE) >> 4;
            umma_bf16_x4(tmem + col_g(kb), dC + ko, dC + ko + 2, dC + ko + 4, dC + ko + 6, dB + ko, dB + ko + 2,
                         dB + ko + 4, dB + ko + 6, ID_KK, kb4 > 0);
          }
          umma_commit(&gfull[kb]);
          SSD_TRACE(k1, 3);
          ++k1;
          prog = true;
        }
        if (k3 < nchunks) {
          const int s = k3 % ST, kb = k3 & 1;
          if (mbar_test(&hready[kb], (k3 >> 1) & 1) && (k3 < 2 || mbar_test(&yfree[kb], ((k3 - 2) >> 1) & 1)) &&
              mbar_test(&full[s], (k3 / ST) & 1)) {
            tc_fence_after();
            SSD_TRACE(k3, 12);
            const uint64_t dC = make_desc_sw128(smem_u32(stage_ptr(s)) + TILE * (1 + NB), 16);
            const uint64_t dH = make_desc_sw128(smem_u32(hs_ptr(kb)), TILE);
#pragma unroll
            for (int kb4 = 0; kb4 < NST / 64; ++kb4) {   // 64-wide K blocks of n: C tiles; 16 state rows per step
              const uint64_t ko = (uint64_t)(kb4 * TILE) >> 4;
              const uint64_t ho = 512 * kb4;
              umma_bf16_x4(tmem + col_y2(kb), dC + ko, dC + ko + 2, dC + ko + 4, dC + ko + 6, dH + ho,
                           dH + ho + 128, dH + ho + 256, dH + ho + 384, ID_KM, kb4 > 0);
            }
            umma_commit(&y2full[kb]);
            SSD_TRACE(k3, 13);
            ++k3;
            prog = true;
          }
        }
        if (prog) {
          t_prog = globaltimer_ns();
        } else {
          if (*abort_flag) break;
          if (globaltimer_ns() - t_prog > 2000000000ull) {
            fail(1006);
            break;
          }
        }
      }
      drain_mmas(&drain[2]);
    }
  } else if (warp >= 4 && warp < 8) {
    // ================================================================ mask group
    const int t = tid - 128;
    const int w = warp - 4;
    const int row = w * 16 + (lane & 15);   // token i of the M=64 accumulator rows held by this thread
    const int half = lane >> 4;             // which 32 columns
    const uint32_t lane_base = (uint32_t)(w * 32) << 16;
    for (int c = 0; c < nchunks; ++c) {
      const int kb = c & 1, ds = c % DSL;
      // G of chunk c, its decay data and B tile, mask buffer c&1 free (MMA2 of chunk c-2 done)
      // and, unless BHAT_IN_STATE, diag(w) B buffer c&1 free (MMA4 of chunk c-2 done)
      const bool bad = !mbar_wait_n(abort_flag, &gfull[kb], (c >> 1) & 1, &dfull[ds], (c / DSL) & 1,
                                    c >= 2 ? &y1full[kb] : nullptr, ((c - 2) >> 1) & 1, &full[c % ST],
                                    (c / ST) & 1) ||
                       (!LY::BHAT_IN_STATE && c >= 2 && !mbar_wait(&sfull[kb], ((c - 2) >> 1) & 1, abort_flag));
      if (bad && !*abort_flag) fail(1007);
      if (named_bar_or(BAR_MSK, 128, bad)) break;
      const float* sm = small_ptr(ds);
      if (t == 0) SSD_TRACE(c, 6);
      tc_fence_after();
      // M row `row`, columns [32*half, 32*half+32):
      //     M_ij = G_ij * exp2(s_i - s_ref(J)) * v_j for j <= i (J = 4-token sub-block of j)
      float g[32];
      tmem_ld16x2_32(tmem + lane_base + col_g(kb), g);
      {
        const float si = sm[row + (row >= 32 ? 4 : 0)];
        const float4* vv = reinterpret_cast<const float4*>(sm + 72 + half * 36);
        const int nvalid = row - half * 32;      // columns jj <= nvalid are kept
        float u[8];
#pragma unroll
        for (int J = 0; J < 8; ++J) u[J] = fast_exp2(si - sm[half * 36 + 4 * J + 3]);
        uint8_t* Mt = mt_ptr(kb);
        tmem_wait_ld();
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float4 va = vv[2 * q], vb = vv[2 * q + 1];
          const float v8[8] = {va.x, va.y, va.z, va.w, vb.x, vb.y, vb.z, vb.w};
          float m[8];
#pragma unroll
          for (int e = 0; e < 8; e += 2) {
            const int jj = q * 8 + e;
            const float uu = u[jj >> 2];
            const float2 val = fmul2(fmul2(make_float2(g[jj], g[jj + 1]), make_float2(uu, uu)), make_float2(v8[e], v8[e + 1]));
            m[e] = jj <= nvalid ? val.x : 0.f;
            m[e + 1] = jj + 1 <= nvalid ? val.y : 0.f;
          }
          *reinterpret_cast<uint4*>(Mt + sw128_chunk(row, half * 4 + q)) =
              make_uint4(pack_bf16x2(m[0], m[1]), pack_bf16x2(m[2], m[3]), pack_bf16x2(m[4], m[5]),
                         pack_bf16x2(m[6], m[7]));
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      named_bar_sync(BAR_MSK, 128);
      if (t == 0) {
        SSD_TRACE(c, 7);
        mbar_arrive(&gfree[kb]);
        mbar_arrive(&mready[kb]);
      }
      // then diag(w) B of chunk c (MMA4's A operand), w_j = exp2(s_last - s_j) beta_j
      if (!LY::BHAT_IN_STATE) {
        const float* wv = sm + 144;
#pragma unroll
        for (int nb = 0; nb < NB; ++nb) {
          const uint8_t* Bt = stage_ptr(c % ST) + TILE * (1 + nb);
          uint8_t* Bh = bh_ptr(kb) + TILE * nb;
          uint4 v[4];
#pragma unroll
          for (int it = 0; it < 4; ++it) v[it] = *reinterpret_cast<const uint4*>(Bt + (t + it * 128) * 16);
#pragma unroll
          for (int it = 0; it < 4; ++it) {
            const int idx = t + it * 128;   // 16-byte chunk; row (token) = idx / 8
            const __nv_bfloat162 w2 = __float2bfloat162_rn(wv[idx >> 3]);
            __nv_bfloat162* hv = reinterpret_cast<__nv_bfloat162*>(&v[it]);
            hv[0] = __hmul2(hv[0], w2);
            hv[1] = __hmul2(hv[1], w2);
            hv[2] = __hmul2(hv[2], w2);
            hv[3] = __hmul2(hv[3], w2);
            *reinterpret_cast<uint4*>(Bh + idx * 16) = v[it];
          }
        }
        fence_proxy_async_smem();
        named_bar_sync(BAR_MSK, 128);
        if (t == 0) mbar_arrive(&bready[kb]);
      }
    }
  } else if (warp >= 8) {
    // ================================================================ output group (warps 8-11)
    const int t = tid - 256;
    const int w = warp - 8;
    const int half = lane >> 4;
    const int row = w * 16 + (lane & 15);   // token row of Y1/Y2 (M=64 layout)
    const uint32_t lane_base = (uint32_t)(w * 32) << 16;
    int c = 0;
    for (; c < nchunks; ++c) {
      const int s = c % ST, kb = c & 1, ds = c % DSL;
      if (t == 0 && c >= 2) bulk_wait_read<1>();   // the store of chunk c-2 has left y tile kb
      bool bad = !mbar_wait_n(abort_flag, &y1full[kb], (c >> 1) & 1, &y2full[kb], (c >> 1) & 1, &full[s],
                              (c / ST) & 1, &dfull[ds], (c / DSL) & 1);
      if (bad && !*abort_flag) fail(1009);
      if (named_bar_or(BAR_OUT, 128, bad)) break;
      if (t == 0) SSD_TRACE(c, 16);
      tc_fence_after();
      float y1[32], y2[32];
      tmem_ld16x2_32(tmem + lane_base + col_y1(kb), y1);
      tmem_ld16x2_32(tmem + lane_base + col_y2(kb), y2);
      const float ei = exp2f(small_ptr(ds)[row + (row >= 32 ? 4 : 0)]);
      const uint8_t* X = stage_ptr(s);
      uint8_t* Ys = ys_ptr(kb);
      tmem_wait_ld();
      if (t == 0) SSD_TRACE(c, 17);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int cc = half * 4 + q;
        float xf[8];
        unpack_bf16x8(*reinterpret_cast<const uint4*>(X + sw128_chunk(row, cc)), xf);
        const float4 da = *reinterpret_cast<const float4*>(dsk + cc * 8);
        const float4 db = *reinterpret_cast<const float4*>(dsk + cc * 8 + 4);
        const float d8[8] = {da.x, da.y, da.z, da.w, db.x, db.y, db.z, db.w};
        uint32_t w4[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int jj = q * 8 + 2 * e;
          // (y1 + ei*y2) + d*x, two tokens' columns per packed instruction
          const float2 t2 = ffma2(make_float2(ei, ei), make_float2(y2[jj], y2[jj + 1]), make_float2(y1[jj], y1[jj + 1]));
          const float2 o = ffma2(make_float2(d8[2 * e], d8[2 * e + 1]), make_float2(xf[2 * e], xf[2 * e + 1]), t2);
          w4[e] = pack_bf16x2(o.x, o.y);
        }
        *reinterpret_cast<uint4*>(Ys + sw128_chunk(row, cc)) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
      }
      fence_proxy_async_smem();   // y tile -> visible to the TMA store
      tc_fence_before();
      named_bar_sync(BAR_OUT, 128);
      if (t == 0) {
        tma_store_3d(&tm_y, Ys, h * P, c * Q, b);   // rows past L are clipped by the tensor map
        bulk_commit();
        SSD_TRACE(c, 18);
        mbar_arrive(&yfree[kb]);
        mbar_arrive(&empty[s]);
        mbar_arrive(&dempty[ds]);
      }
    }
    if (t == 0) {
      bulk_wait<0>();   // every y store complete before the CTA exits
      *consumed = c;
    }
  } else {
    // ================================================================ state group (warps 0-3)
    const int half = lane >> 4;
    const int row = warp * 16 + (lane & 15);
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    // State ownership: NST=64 -> S^T row n = row, p in [32*half, +32);  NST=128 -> n = tid, all p.
    constexpr int HP = NST == 64 ? 32 : 64;
    const int n_own = NST == 64 ? row : tid;
    const int p0 = NST == 64 ? 32 * half : 0;
    float hreg[HP];
#pragma unroll
    for (int j = 0; j < HP; ++j) hreg[j] = 0.f;
    if (h0) {
      const float* src = h0 + (((int64_t)b * H + h) * P) * NST + n_own;
#pragma unroll
      for (int j = 0; j < HP; ++j) hreg[j] = src[(int64_t)(p0 + j) * NST];
    }
    // bf16 state tile for MMA3: row n, 64 p contiguous (MN-major B operand), 128B swizzle.
    auto write_hs = [&](uint8_t* Hs) {
#pragma unroll
      for (int q = 0; q < HP / 8; ++q) {
        uint4 o;
        o.x = pack_bf16x2(hreg[8 * q + 0], hreg[8 * q + 1]);
        o.y = pack_bf16x2(hreg[8 * q + 2], hreg[8 * q + 3]);
        o.z = pack_bf16x2(hreg[8 * q + 4], hreg[8 * q + 5]);
        o.w = pack_bf16x2(hreg[8 * q + 6], hreg[8 * q + 7]);
        *reinterpret_cast<uint4*>(Hs + sw128_chunk(n_own, p0 / 8 + q)) = o;
      }
    };
    // diag(w) B of chunk j (MMA4's A operand) into buffer j&1 (BHAT_IN_STATE only; its B
    // tile and decay data have landed, and MMA4 of chunk j-2 is complete)
    auto bhat_rows = [&](int j) {
      const int sj = j % ST, dj = j % DSL;
      const float* wv = small_ptr(dj) + 144;
      const uint8_t* Bt = stage_ptr(sj) + TILE;
      uint8_t* Bh = bh_ptr(j & 1);
      uint4 v[4];
#pragma unroll
      for (int it = 0; it < 4; ++it) v[it] = *reinterpret_cast<const uint4*>(Bt + (tid + it * 128) * 16);
#pragma unroll
      for (int it = 0; it < 4; ++it) {
        const int idx = tid + it * 128;   // 16-byte chunk; row (token) = idx / 8
        const __nv_bfloat162 w2 = __float2bfloat162_rn(wv[idx >> 3]);
        __nv_bfloat162* hv = reinterpret_cast<__nv_bfloat162*>(&v[it]);
        hv[0] = __hmul2(hv[0], w2);
        hv[1] = __hmul2(hv[1], w2);
        hv[2] = __hmul2(hv[2], w2);
        hv[3] = __hmul2(hv[3], w2);
        *reinterpret_cast<uint4*>(Bh + idx * 16) = v[it];
      }
    };
    write_hs(hs_ptr(0));
    bool ok = true;
    if (LY::BHAT_IN_STATE) {   // diag(w) B of the first two chunks
      for (int j = 0; j < 2 && j < nchunks; ++j) {
        const bool bad = !mbar_wait_n(abort_flag, &full[j % ST], (j / ST) & 1, &dfull[j % DSL], (j / DSL) & 1);
        if (bad && !*abort_flag) fail(1017);
        if (named_bar_or(BAR_STATE, 128, bad)) {
          ok = false;
          break;
        }
        bhat_rows(j);
        fence_proxy_async_smem();
        named_bar_sync(BAR_STATE, 128);
        if (tid == 0) mbar_arrive(&bready[j & 1]);
      }
    }
    fence_proxy_async_smem();
    named_bar_sync(BAR_STATE, 128);
    if (tid == 0) mbar_arrive(&hready[0]);
    for (int c = 0; c < nchunks && ok; ++c) {
      const int kb = c & 1, ds = c % DSL;
      const bool nxt = LY::BHAT_IN_STATE && c + 2 < nchunks;   // diag(w) B of chunk c+2 written here
      const int jd = nxt ? c + 2 : c;
      // S of chunk c; decay data up to chunk jd (the decay warp publishes in order); MMA3 of
      // chunk c-1 complete (it read state tile (c+1)&1, which this iteration overwrites);
      // with BHAT_IN_STATE the B tile of chunk c+2
      const bool bad = !mbar_wait_n(abort_flag, &sfull[kb], (c >> 1) & 1, &dfull[jd % DSL], (jd / DSL) & 1,
                                    c >= 1 ? &y2full[(c - 1) & 1] : nullptr, ((c - 1) >> 1) & 1,
                                    nxt ? &full[(c + 2) % ST] : nullptr, ((c + 2) / ST) & 1);
      if (bad && !*abort_flag) fail(1008);
      if (named_bar_or(BAR_STATE, 128, bad)) {
        ok = false;
        break;
      }
      if (tid == 0) SSD_TRACE(c, 14);
      tc_fence_after();
      const float e_last = small_ptr(ds)[208];
      // H <- exp(s_last) H + S ; bf16 copy for MMA3 of chunk c+1
      if (NST == 64) {
        float sv[32];
        tmem_ld16x2_32(tmem + lane_base + col_s(kb), sv);
        tmem_wait_ld();
        const float2 e2 = make_float2(e_last, e_last);
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          const float2 r = ffma2(e2, make_float2(hreg[j], hreg[j + 1]), make_float2(sv[j], sv[j + 1]));
          hreg[j] = r.x;
          hreg[j + 1] = r.y;
        }
      } else {
        float sv[32];
        tmem_ld32(tmem + lane_base + col_s(kb), sv);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; ++j) hreg[j] = e_last * hreg[j] + sv[j];
        tmem_ld32(tmem + lane_base + col_s(kb) + 32, sv);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; ++j) hreg[32 + j] = e_last * hreg[32 + j] + sv[j];
      }
      write_hs(hs_ptr((c + 1) & 1));
      // S of chunk c is read, so MMA4 of chunk c is complete and buffer c&1 may take
      // diag(w) B of chunk c+2
      if (nxt) bhat_rows(c + 2);
      fence_proxy_async_smem();
      tc_fence_before();
      named_bar_sync(BAR_STATE, 128);
      if (tid == 0) {
        SSD_TRACE(c, 15);
        mbar_arrive(&hready[(c + 1) & 1]);
        mbar_arrive(&sfree[kb]);
        mbar_arrive(&dempty[ds]);
        if (nxt) mbar_arrive(&bready[kb]);
      }
    }
    if (ok && h_last && !*abort_flag) {
      float* dst = h_last + (((int64_t)b * H + h) * P) * NST + n_own;
#pragma unroll
      for (int j = 0; j < HP; ++j) dst[(int64_t)(p0 + j) * NST] = hreg[j];
    }
  }
  // ================================================================ teardown
  tc_fence_before();
  __syncthreads();
  if (tid == 0 && *abort_flag) {
    // Drain loads that were issued but never consumed before the CTA exits.
    for (int c = *consumed; c < *issued; ++c) mbar_wait(&full[c % ST], (c / ST) & 1, nullptr, 100000000ull);
  }
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// 3-D bf16 map over [d2][d1][d0] (d0 contiguous) with a {64, 64, 1} box and 128B swizzle.
bool map3d_bf16(CUtensorMap* m, const void* base, uint64_t d0, uint64_t d1, uint64_t d2) {
  auto fn = tmap_encode_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {d0 * 2, d0 * d1 * 2};
  cuuint32_t box[3] = {64, 64, 1};
  cuuint32_t es[3] = {1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int NST, bool ZOH>
int launch_ssd(const CUtensorMap& mx, const CUtensorMap& mb, const CUtensorMap& mc, const CUtensorMap& my,
               const float* dt, const float* A_log, const float* Dskip, const float* h0, float* h_last,
               float* decay_log2, int64_t Bsz, int64_t L, int64_t H, cudaStream_t st) {
  constexpr int bytes = Layout<NST>::BYTES;
  auto kern = ssd_chunk_scan_kernel<NST, ZOH>;
  // The dynamic shared-memory opt-in is per device; it is cheap, so set it on every launch.
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess)
    return check_launch("ssd: set smem attribute");
  int* status = device_status_ptr();
  if (!status) {
    set_error("ssd: device status word unavailable");
    return TSSM_ERR_CUDA;
  }
  dim3 grid((unsigned)H, (unsigned)Bsz);
  kern<<<grid, NTHREADS, bytes, st>>>(mx, mb, mc, my, dt, A_log, Dskip, h0, h_last, decay_log2, status, (int)L,
                                      (int)H);
  return check_launch("ssd_chunk_scan");
}

}  // namespace
}  // namespace tssm

extern "C" int tssm_multihead_ssd(const void* x, const void* dt, const void* A_log, const void* B,
                                  const void* C, const void* Dskip, void* y, const void* h0, void* h_last,
                                  void* decay_log2, int64_t Bsz, int64_t L, int64_t H, int64_t P, int64_t N,
                                  int bdisc, tssm_stream_t stream) {
  using namespace tssm;
  TSSM_REQUIRE(Bsz >= 0 && L >= 0 && H >= 0, "multihead_ssd: negative size");
  if (Bsz * L * H == 0) return TSSM_OK;
  TSSM_REQUIRE(P == 64, "multihead_ssd: head dim P must be 64 (got %lld)", (long long)P);
  TSSM_REQUIRE(N == 64 || N == 128, "multihead_ssd: state size N must be 64 or 128 (got %lld)", (long long)N);
  TSSM_REQUIRE(bdisc == 0 || bdisc == 1, "multihead_ssd: bdisc must be 0 (euler) or 1 (zoh)");
  TSSM_REQUIRE(x && dt && A_log && B && C && Dskip && y, "multihead_ssd: null pointer");
  TSSM_REQUIRE(aligned16(x) && aligned16(B) && aligned16(C) && aligned16(y),
               "multihead_ssd: x, B, C, y must be 16-byte aligned");
  TSSM_REQUIRE(Bsz <= 65535 && H <= 65535 && L < (int64_t(1) << 31) && H * N < (int64_t(1) << 31),
               "multihead_ssd: size out of range");
  CUtensorMap mx, mb, mc, mo;
  if (!map3d_bf16(&mx, x, (uint64_t)(H * P), (uint64_t)L, (uint64_t)Bsz) ||
      !map3d_bf16(&mb, B, (uint64_t)(H * N), (uint64_t)L, (uint64_t)Bsz) ||
      !map3d_bf16(&mc, C, (uint64_t)(H * N), (uint64_t)L, (uint64_t)Bsz) ||
      !map3d_bf16(&mo, y, (uint64_t)(H * P), (uint64_t)L, (uint64_t)Bsz)) {
    set_error("multihead_ssd: cuTensorMapEncodeTiled failed");
    return TSSM_ERR_CUDA;
  }
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const float* dtp = (const float*)dt;
  const float* al = (const float*)A_log;
  const float* dk = (const float*)Dskip;
  const float* hi = (const float*)h0;
  float* ho = (float*)h_last;
  float* dl = (float*)decay_log2;
  if (N == 64)
    return bdisc ? launch_ssd<64, true>(mx, mb, mc, mo, dtp, al, dk, hi, ho, dl, Bsz, L, H, st)
                 : launch_ssd<64, false>(mx, mb, mc, mo, dtp, al, dk, hi, ho, dl, Bsz, L, H, st);
  return bdisc ? launch_ssd<128, true>(mx, mb, mc, mo, dtp, al, dk, hi, ho, dl, Bsz, L, H, st)
               : launch_ssd<128, false>(mx, mb, mc, mo, dtp, al, dk, hi, ho, dl, Bsz, L, H, st);
}

#ifdef TSSM_SSD_TRACE
extern "C" int tssm_debug_read_ssd_trace(unsigned long long* out, int n) {
  return cudaMemcpyFromSymbol(out, tssm::g_ssd_trace, sizeof(unsigned long long) * (n < 2048 ? n : 2048)) ==
                 cudaSuccess ? 0 : 3;
}
#endif
