// Streaming ring-buffer ingest + forward fill + one SSM step (replaces
// streaming_interp_then_ssm_kernel, streaming_inference_kernel.py:74-156).
//
// Per stream b, per event:
//   1. the event (v, m) goes to ring slot nh = (head+1) % KR and tau_new to
//      ring_tau[b, nh] (:105-117);
//   2. for every BLOCK_H-wide feature tile, the nearest older slot whose mask
//      sum over the tile exceeds 0.5 is found (:121-130);
//   3. vhat = the previous slot's values where the event's own tile mask sum is
//      below 0.5 and such a slot exists, else the event's values (:133-143);
//   4. h <- Abar h + Bbar vhat (in place), y = C h + D vhat (:146-156).
// The reference runs one program per (b, H-block), and block 0 rewrites
// ring_head while the others may still be reading it (:115-117), so blocks of
// one stream can pick different slots.  Here one CTA owns a whole stream: every
// thread reads the old head before a barrier, and the new head is stored once,
// after it.  A tile whose new event is observed (mask sum >= 0.5) takes the
// event's values whatever the ring holds, so only the other tiles search.
// Two forms:
//   * 128-feature tiles (the reference's default BLOCK_H) over 16-byte aligned
//     rows: one warp per tile, four features per lane, warp-shuffle mask sums,
//     no barrier after the head read;
//   * any tile width: tile sums in shared memory, a barrier per searched slot,
//     the search ending at the first slot that leaves no tile open.
#include "common.cuh"

namespace tssm {
namespace {

constexpr int RING_THREADS = 256;

// Adds v into the tile sum of feature f; whole-warp aggregation when every lane
// of the warp falls in one tile (tiles are multiples of 32 features and f is
// warp-contiguous).
__device__ __forceinline__ void tile_add(float* sums, int64_t f, int64_t H, int block_h, float v, bool warp_tiles) {
  if (warp_tiles) {
    const int64_t f0 = f - (threadIdx.x & 31);   // first feature of this warp's 32
    if (f0 >= H) return;                          // whole warp past the end (uniform)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if ((threadIdx.x & 31) == 0) atomicAdd(&sums[f0 / block_h], v);
  } else if (f < H) {
    atomicAdd(&sums[f / block_h], v);
  }
}

__global__ void __launch_bounds__(RING_THREADS) ring_ingest_step_kernel(
    float* __restrict__ ring_V, float* __restrict__ ring_M, float* __restrict__ ring_tau,
    int* __restrict__ ring_head, const float* __restrict__ v_new, const float* __restrict__ m_new,
    const float* __restrict__ tau_new, float* __restrict__ h, const float* __restrict__ Abar,
    const float* __restrict__ Bbar, const float* __restrict__ C, const float* __restrict__ D,
    float* __restrict__ y, int64_t H, int KR, int block_h) {
  extern __shared__ float s_dyn[];
  const int64_t ntiles = (H + block_h - 1) / block_h;
  float* s_new = s_dyn;                                        // event mask sum per tile
  float* s_sum = s_dyn + ntiles;                               // slot mask sum per tile
  int* s_prev = reinterpret_cast<int*>(s_dyn + 2 * ntiles);    // resolved slot per tile (-1: none yet)
  const int tid = threadIdx.x;
  const int64_t b = blockIdx.x;
  const bool warp_tiles = (block_h % 32) == 0;
  const int64_t Hpad = warp_tiles ? (H + 31) / 32 * 32 : H;   // whole warps iterate together
  const int head = ring_head[b];
  const int nh = (head + 1) % KR;
  float* rV = ring_V + b * KR * H;
  float* rM = ring_M + b * KR * H;
  for (int64_t t = tid; t < ntiles; t += RING_THREADS) {
    s_new[t] = 0.f;
    s_sum[t] = 0.f;
    s_prev[t] = -1;
  }
  __syncthreads();
  // 1. store the event in slot nh; the event's tile mask sums
  for (int64_t f = tid; f < Hpad; f += RING_THREADS) {
    float m = 0.f;
    if (f < H) {
      const float v = v_new[b * H + f];
      m = m_new[b * H + f];
      rV[(int64_t)nh * H + f] = v;
      rM[(int64_t)nh * H + f] = m;
    }
    tile_add(s_new, f, H, block_h, m, warp_tiles);
  }
  // 2. nearest older slot with a mask sum above 0.5, for the tiles whose event is
  // missing (an observed tile takes the event's values: mark it resolved)
  __syncthreads();
  int open_any = 0;
  for (int64_t t = tid; t < ntiles; t += RING_THREADS) {
    if (s_new[t] >= 0.5f)
      s_prev[t] = KR;   // resolved, value unused
    else
      open_any = 1;
  }
  const bool search = __syncthreads_or(open_any) != 0;
  for (int k = 1; search && k < KR; ++k) {
    const int rk = (nh - k + KR) % KR;
    __syncthreads();   // s_prev / s_sum from the previous round (or the init) are settled
    for (int64_t f = tid; f < Hpad; f += RING_THREADS) {
      const bool open = f < H && s_prev[f / block_h] < 0;
      const float m = open ? rM[(int64_t)rk * H + f] : 0.f;
      tile_add(s_sum, f, H, block_h, m, warp_tiles);
    }
    __syncthreads();
    int unresolved = 0;
    for (int64_t t = tid; t < ntiles; t += RING_THREADS) {
      if (s_prev[t] < 0) {
        if (s_sum[t] > 0.5f)
          s_prev[t] = rk;
        else {
          s_sum[t] = 0.f;
          unresolved = 1;
        }
      }
    }
    if (!__syncthreads_or(unresolved)) break;
  }
  __syncthreads();
  // 3 + 4. forward fill and the step
  for (int64_t f = tid; f < H; f += RING_THREADS) {
    const int64_t t = f / block_h;
    const int pk = s_prev[t];
    const float vh = (pk >= 0 && pk < KR && s_new[t] < 0.5f) ? rV[(int64_t)pk * H + f] : v_new[b * H + f];
    const float hn = Abar[f] * h[b * H + f] + Bbar[f] * vh;
    h[b * H + f] = hn;
    y[b * H + f] = C[b * H + f] * hn + D[f] * vh;
  }
  if (tid == 0) {
    ring_tau[b * KR + nh] = tau_new[b];
    ring_head[b] = nh;   // every thread read the old head before the first barrier
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ void st4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }
__device__ __forceinline__ float sum4(float4 v) { return (v.x + v.y) + (v.z + v.w); }

// 128-feature tiles, H % 4 == 0, 16-byte aligned rows: warp w takes tiles w, w+8, ...
__global__ void __launch_bounds__(RING_THREADS) ring_ingest_step_tile128_kernel(
    float* __restrict__ ring_V, float* __restrict__ ring_M, float* __restrict__ ring_tau,
    int* __restrict__ ring_head, const float* __restrict__ v_new, const float* __restrict__ m_new,
    const float* __restrict__ tau_new, float* __restrict__ h, const float* __restrict__ Abar,
    const float* __restrict__ Bbar, const float* __restrict__ C, const float* __restrict__ D,
    float* __restrict__ y, int64_t H, int KR) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t b = blockIdx.x;
  const int head = ring_head[b];
  const int nh = (head + 1) % KR;
  __syncthreads();   // every thread has read the old head; thread 0 may store the new one
  if (tid == 0) {
    ring_tau[b * KR + nh] = tau_new[b];
    ring_head[b] = nh;
  }
  float* rV = ring_V + b * KR * H;
  float* rM = ring_M + b * KR * H;
  const int64_t ntiles = (H + 127) / 128;
  const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int64_t t = warp; t < ntiles; t += RING_THREADS / 32) {
    const int64_t f = t * 128 + lane * 4;
    const bool act = f < H;   // H % 4 == 0: the four features exist together
    const int64_t o = b * H + f;
    const float4 v = act ? ld4(v_new + o) : z4;
    const float4 m = act ? ld4(m_new + o) : z4;
    const float4 hp = act ? ld4(h + o) : z4;
    const float4 c = act ? ld4(C + o) : z4;
    const float4 ab = act ? ld4(Abar + f) : z4;
    const float4 bb = act ? ld4(Bbar + f) : z4;
    const float4 dd = act ? ld4(D + f) : z4;
    if (act) {
      st4(rV + (int64_t)nh * H + f, v);
      st4(rM + (int64_t)nh * H + f, m);
    }
    float4 vh = v;
    if (warp_sum(sum4(m)) < 0.5f) {   // the event's tile is missing: forward-fill from the nearest observed slot
      for (int k = 1; k < KR; ++k) {
        const int rk = (nh - k + KR) % KR;
        const float4 pm = act ? ld4(rM + (int64_t)rk * H + f) : z4;
        if (warp_sum(sum4(pm)) > 0.5f) {
          if (act) vh = ld4(rV + (int64_t)rk * H + f);
          break;
        }
      }
    }
    if (act) {
      float4 hn, yo;
      hn.x = ab.x * hp.x + bb.x * vh.x;
      hn.y = ab.y * hp.y + bb.y * vh.y;
      hn.z = ab.z * hp.z + bb.z * vh.z;
      hn.w = ab.w * hp.w + bb.w * vh.w;
      yo.x = c.x * hn.x + dd.x * vh.x;
      yo.y = c.y * hn.y + dd.y * vh.y;
      yo.z = c.z * hn.z + dd.z * vh.z;
      yo.w = c.w * hn.w + dd.w * vh.w;
      st4(h + o, hn);
      st4(y + o, yo);
    }
  }
}

}  // namespace
}  // namespace tssm

extern "C" int tssm_ring_ingest_step(void* ring_V, void* ring_M, void* ring_tau, void* ring_head, const void* v_new,
                                     const void* m_new, const void* tau_new, void* h, const void* Abar,
                                     const void* Bbar, const void* C, const void* Dskip, void* y, int64_t Bsz,
                                     int64_t H, int64_t K, int64_t block_h, tssm_stream_t stream) {
  using namespace tssm;
  TSSM_REQUIRE(Bsz >= 0 && H >= 0 && K >= 0, "ring_ingest_step: negative size");
  TSSM_REQUIRE(K + 1 <= 64, "ring_ingest_step: ring of K+1=%lld slots exceeds 64", (long long)(K + 1));
  TSSM_REQUIRE(block_h >= 1, "ring_ingest_step: BLOCK_H must be >= 1");
  if (Bsz * H == 0) return TSSM_OK;
  TSSM_REQUIRE(ring_V && ring_M && ring_tau && ring_head && v_new && m_new && tau_new && h && Abar && Bbar && C &&
                   Dskip && y,
               "ring_ingest_step: null pointer");
  TSSM_REQUIRE(Bsz < (int64_t(1) << 31), "ring_ingest_step: too many streams");
  const int64_t ntiles = cdiv(H, block_h);
  const size_t smem = (size_t)ntiles * 3 * sizeof(float);
  TSSM_REQUIRE(smem <= 200 * 1024, "ring_ingest_step: %lld tiles need too much shared memory", (long long)ntiles);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (block_h == 128 && H % 4 == 0 && aligned16(ring_V) && aligned16(ring_M) && aligned16(v_new) &&
      aligned16(m_new) && aligned16(h) && aligned16(Abar) && aligned16(Bbar) && aligned16(C) && aligned16(Dskip) &&
      aligned16(y)) {
    ring_ingest_step_tile128_kernel<<<(unsigned)Bsz, RING_THREADS, 0, st>>>(
        (float*)ring_V, (float*)ring_M, (float*)ring_tau, (int*)ring_head, (const float*)v_new, (const float*)m_new,
        (const float*)tau_new, (float*)h, (const float*)Abar, (const float*)Bbar, (const float*)C,
        (const float*)Dskip, (float*)y, H, (int)(K + 1));
    return check_launch("ring_ingest_step");
  }
  auto kern = ring_ingest_step_kernel;
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return check_launch("ring_ingest_step: set smem attribute");
  kern<<<(unsigned)Bsz, RING_THREADS, smem, st>>>(
      (float*)ring_V, (float*)ring_M, (float*)ring_tau, (int*)ring_head, (const float*)v_new, (const float*)m_new,
      (const float*)tau_new, (float*)h, (const float*)Abar, (const float*)Bbar, (const float*)C,
      (const float*)Dskip, (float*)y, H, (int)(K + 1), (int)block_h);
  return check_launch("ring_ingest_step");
}
