// Sequence-parallel (L-sharded) multi-head scan: carry combination and
// fix-up of a shard's outputs (config 4).
//
// Rank r scans its slice of the sequence from a zero state (ssd.cu) and
// publishes its final state S_r [B,H,P,N] and the log2 of its whole-slice
// decay, d_r = log2(exp(A_h * sum dt)).  After an all-gather, the state
// entering slice r is the exclusive prefix
//     carry_r = sum_{j<r} (prod_{j<k<r} 2^d_k) S_j,   i.e.  c <- 2^d_j c + S_j for j < r,
// the block-level form of the reference's carry scan (ssm_scan.py:53-65,
// :68-98).  Its effect on the slice's outputs is
//     y[t, p] += exp(A_h * cumdt(t)) * sum_n C[t, n] carry[p, n],
// which decays monotonically; a chunk of 64 tokens whose starting decay is
// exactly 0 in f32 needs no work, nor does any chunk after it.  The first FKC
// chunks of a slice go to FKC CTAs, each of which sums the decay of the tokens
// before its chunk itself and exits when that decay is 0; the last of them
// walks on through the later chunks until the decay reaches 0.
#include "common.cuh"

namespace tssm {
namespace {

constexpr int FQ = 64;    // tokens per fix-up chunk
constexpr int FP = 64;    // head dim
constexpr int FKC = 16;   // CTAs per (slice, sequence, head), one chunk each (the last walks on)

// Slices and sequences: slice j of sequence b has its state at S_all + j*sj +
// b*sb (+ h*P*N) and its log2 decay at d_all + j*dj + b*db (+ h).  The slice
// being fixed is `rank` (or, with pieces > 0, blockIdx.z + 1 of `pieces`
// in-device pieces); its C, dt and y rows are sequence vb = b*vbs + vbo of
// tensors [*, L, ...].
template <int NST>
__global__ void __launch_bounds__(256) ssd_carry_fixup_kernel(
    const float* __restrict__ S_all, const float* __restrict__ d_all, int rank, int pieces, int64_t sj, int64_t sb,
    int64_t dj, int64_t db, const __nv_bfloat16* __restrict__ C, const float* __restrict__ dt,
    const float* __restrict__ A_log, __nv_bfloat16* __restrict__ y, int L, int H) {
  extern __shared__ __align__(16) float fsm[];
  float* carry = fsm;                   // [FP][NST + 1] (padded rows: no bank conflicts)
  float* cs = carry + FP * (NST + 1);   // [FQ][NST + 1]
  float* es = cs + FQ * (NST + 1);      // [FQ] decay factor per token
  __shared__ float s_run;
  __shared__ float s_part[8];
  // chunk-major order: every slice's first chunks are dispatched first (the
  // later chunks' CTAs mostly find a zero decay and exit at once)
  const int h = blockIdx.x % H, kc = blockIdx.x / H, tid = threadIdx.x;
  const int slice = pieces > 0 ? (int)blockIdx.z + 1 : rank;
  const int64_t bo = blockIdx.y;
  const int b = pieces > 0 ? (int)(bo * pieces + slice) : (int)bo;   // sequence of C, dt, y
  const float a2 = -expf(A_log[h]) * 1.4426950408889634f;
  const int warp = tid >> 5, lane = tid & 31;
  // log2 decay from the slice start to this CTA's first chunk (tokens [0, kc FQ))
  const int tstart = kc * FQ;
  if (tstart >= L) return;
  {
    float part = 0.f;
    for (int t = tid; t < tstart; t += 256) part += dt[((int64_t)b * L + t) * H + h] * a2;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
    if (lane == 0) s_part[warp] = part;
    __syncthreads();
    if (tid == 0) {
      float run = 0.f;
#pragma unroll
      for (int w = 0; w < 8; ++w) run += s_part[w];
      s_run = run;
    }
    __syncthreads();
    if (exp2f(s_run) == 0.f) return;   // uniform: this chunk and every later one add exactly 0
  }
  // carry entering this slice
  const int64_t base = bo * sb + (int64_t)h * FP * NST;
  // slices outermost, this thread's FP*NST/256 elements in registers: the loads
  // of one slice are independent, so the chain costs one round trip per slice
  {
    constexpr int EPT = FP * NST / 256;
    float cr[EPT];
#pragma unroll
    for (int k = 0; k < EPT; ++k) cr[k] = 0.f;
    for (int j = 0; j < slice; ++j) {
      const float f = exp2f(d_all[(int64_t)j * dj + bo * db + h]);
      const float* Sj = S_all + j * sj + base;
#pragma unroll
      for (int k = 0; k < EPT; ++k) cr[k] = f * cr[k] + Sj[tid + k * 256];
    }
#pragma unroll
    for (int k = 0; k < EPT; ++k) {
      const int e = tid + k * 256;
      carry[(e / NST) * (NST + 1) + (e % NST)] = cr[k];
    }
  }
  const int tt = tid >> 4, pp = tid & 15;   // 4 tokens x 4 head dims per thread
  __syncthreads();
  for (int t0 = tstart; t0 < L; t0 += FQ) {
    // decay factors of this chunk (warp 0) and the chunk's C rows (all)
    if (warp == 0) {
      float l[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int t = t0 + 2 * lane + e;
        l[e] = t < L ? dt[((int64_t)b * L + t) * H + h] * a2 : 0.f;
      }
      const float pair = l[0] + l[1];
      float incl = pair;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      const float run = s_run;
      es[2 * lane] = exp2f(run + incl - pair + l[0]);
      es[2 * lane + 1] = exp2f(run + incl);
      const float tot = __shfl_sync(0xffffffffu, incl, 31);
      __syncwarp();
      if (lane == 0) s_run = run + tot;
    }
    for (int e = tid; e < FQ * NST / 2; e += 256) {
      const int r = e / (NST / 2), c2 = e - r * (NST / 2);
      const int t = t0 + r;
      float2 v = make_float2(0.f, 0.f);
      if (t < L) v = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(C + (((int64_t)b * L + t) * H + h) * NST)[c2]);
      cs[r * (NST + 1) + 2 * c2] = v.x;
      cs[r * (NST + 1) + 2 * c2 + 1] = v.y;
    }
    __syncthreads();
    if (es[0] == 0.f) break;   // uniform: every later decay is exactly 0 too
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
    for (int n = 0; n < NST; ++n) {
      float cv[4], hv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) cv[i] = cs[(4 * tt + i) * (NST + 1) + n];
#pragma unroll
      for (int j = 0; j < 4; ++j) hv[j] = carry[(4 * pp + j) * (NST + 1) + n];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(cv[i], hv[j], acc[i][j]);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int t = t0 + 4 * tt + i;
      if (t >= L) break;
      const float e = es[4 * tt + i];
      __nv_bfloat16* yr = y + ((int64_t)b * L + t) * H * FP + (int64_t)h * FP + 4 * pp;
#pragma unroll
      for (int j = 0; j < 4; ++j) yr[j] = __float2bfloat16_rn(__bfloat162float(yr[j]) + e * acc[i][j]);
    }
    if (kc != FKC - 1) break;   // one chunk per CTA, except the last CTA of the slice
    __syncthreads();
  }
}

}  // namespace
}  // namespace tssm

namespace tssm {
namespace {
int launch_fixup(const void* S_all, const void* d_all, int rank, int pieces, int64_t sj, int64_t sb, int64_t dj,
                 int64_t db, const void* C, const void* dt, const void* A_log, void* y, dim3 grid, int64_t L,
                 int64_t H, int64_t N, cudaStream_t st) {
  if (N == 64) {
    const size_t smem = sizeof(float) * (64 * 65 + 64 * 65 + 64);
    if (cudaFuncSetAttribute(ssd_carry_fixup_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return check_launch("ssd_carry_fixup: smem");
    ssd_carry_fixup_kernel<64><<<grid, 256, smem, st>>>((const float*)S_all, (const float*)d_all, rank, pieces, sj,
                                                        sb, dj, db, (const __nv_bfloat16*)C, (const float*)dt,
                                                        (const float*)A_log, (__nv_bfloat16*)y, (int)L, (int)H);
  } else {
    const size_t smem = sizeof(float) * (64 * 129 + 64 * 129 + 64);
    if (cudaFuncSetAttribute(ssd_carry_fixup_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return check_launch("ssd_carry_fixup: smem");
    ssd_carry_fixup_kernel<128><<<grid, 256, smem, st>>>((const float*)S_all, (const float*)d_all, rank, pieces, sj,
                                                         sb, dj, db, (const __nv_bfloat16*)C, (const float*)dt,
                                                         (const float*)A_log, (__nv_bfloat16*)y, (int)L, (int)H);
  }
  return check_launch("ssd_carry_fixup");
}
}  // namespace
}  // namespace tssm

extern "C" int tssm_ssd_carry_fixup(const void* S_all, const void* decay_log2_all, int64_t rank, int64_t nranks,
                                    const void* C, const void* dt, const void* A_log, void* y, int64_t Bsz,
                                    int64_t L, int64_t H, int64_t P, int64_t N, tssm_stream_t stream) {
  using namespace tssm;
  TSSM_REQUIRE(rank >= 0 && rank < nranks, "ssd_carry_fixup: rank out of range");
  TSSM_REQUIRE(P == 64 && (N == 64 || N == 128), "ssd_carry_fixup: P must be 64 and N 64 or 128");
  if (rank == 0 || Bsz * L * H == 0) return TSSM_OK;
  TSSM_REQUIRE(S_all && decay_log2_all && C && dt && A_log && y, "ssd_carry_fixup: null pointer");
  TSSM_REQUIRE(Bsz <= 65535 && H <= 65535 && L < (int64_t(1) << 31), "ssd_carry_fixup: size out of range");
  return launch_fixup(S_all, decay_log2_all, (int)rank, 0, Bsz * H * P * N, H * P * N, Bsz * H, H, C, dt, A_log, y,
                      dim3((unsigned)(H * FKC), (unsigned)Bsz), L, H, N, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int tssm_ssd_carry_fixup_pieces(const void* S, const void* decay_log2, int64_t pieces, const void* C,
                                           const void* dt, const void* A_log, void* y, int64_t Bsz, int64_t L,
                                           int64_t H, int64_t P, int64_t N, tssm_stream_t stream) {
  using namespace tssm;
  TSSM_REQUIRE(pieces >= 1 && pieces <= 65535, "ssd_carry_fixup_pieces: pieces in [1, 65535]");
  TSSM_REQUIRE(P == 64 && (N == 64 || N == 128), "ssd_carry_fixup_pieces: P must be 64 and N 64 or 128");
  TSSM_REQUIRE(Bsz >= 0 && L >= 0 && H >= 0 && L % pieces == 0, "ssd_carry_fixup_pieces: L must split into pieces");
  if (pieces == 1 || Bsz * L * H == 0) return TSSM_OK;
  TSSM_REQUIRE(S && decay_log2 && C && dt && A_log && y, "ssd_carry_fixup_pieces: null pointer");
  TSSM_REQUIRE(Bsz <= 65535 && H <= 65535 && L < (int64_t(1) << 31), "ssd_carry_fixup_pieces: size out of range");
  // piece k of sequence b is sequence b*pieces + k of the [Bsz*pieces, L/pieces, ...] views
  return launch_fixup(S, decay_log2, 0, (int)pieces, H * P * N, pieces * H * P * N, H, pieces * H, C, dt, A_log, y,
                      dim3((unsigned)(H * FKC), (unsigned)Bsz, (unsigned)(pieces - 1)), L / pieces, H, N,
                      reinterpret_cast<cudaStream_t>(stream));
}

// ---------------------------------------------------------------------------
// Final state of sequences scanned as in-device pieces: the pieces' states
// chained in order, c <- 2^{d_k} c + S_k, and the summed log2 decay.  One
// thread per four consecutive state elements of one (sequence, head).
namespace tssm {
namespace {
__global__ void __launch_bounds__(256) ssd_pieces_final_state_kernel(
    const float4* __restrict__ S, const float* __restrict__ d, int pieces, float4* __restrict__ state_out,
    float* __restrict__ decay_out, int64_t n4, int64_t hpn4, int pn4, int H) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= n4) return;
  const int64_t b = e / hpn4, rem = e - b * hpn4;
  const int h = (int)(rem / pn4);
  float4 c = make_float4(0.f, 0.f, 0.f, 0.f);
  float dsum = 0.f;
  for (int k = 0; k < pieces; ++k) {
    const int64_t seq = b * pieces + k;
    const float dk = d[seq * H + h];
    const float f = exp2f(dk);
    const float4 s = S[seq * hpn4 + rem];
    c.x = fmaf(f, c.x, s.x);
    c.y = fmaf(f, c.y, s.y);
    c.z = fmaf(f, c.z, s.z);
    c.w = fmaf(f, c.w, s.w);
    dsum += dk;
  }
  if (state_out) state_out[e] = c;
  if (decay_out && rem % pn4 == 0) decay_out[b * H + h] = dsum;
}
}  // namespace
}  // namespace tssm

extern "C" int tssm_ssd_carry_fixup_packed(const void* packed, int64_t rank, int64_t nranks, const void* C,
                                           const void* dt, const void* A_log, void* y, int64_t Bsz, int64_t L,
                                           int64_t H, int64_t P, int64_t N, tssm_stream_t stream) {
  using namespace tssm;
  TSSM_REQUIRE(rank >= 0 && rank < nranks, "ssd_carry_fixup_packed: rank out of range");
  TSSM_REQUIRE(P == 64 && (N == 64 || N == 128), "ssd_carry_fixup_packed: P must be 64 and N 64 or 128");
  TSSM_REQUIRE(Bsz >= 0 && L >= 0 && H >= 0, "ssd_carry_fixup_packed: bad size");
  if (rank == 0 || Bsz * L * H == 0) return TSSM_OK;
  TSSM_REQUIRE(packed && C && dt && A_log && y, "ssd_carry_fixup_packed: null pointer");
  TSSM_REQUIRE(Bsz <= 65535 && H <= 65535 && L < (int64_t(1) << 31), "ssd_carry_fixup_packed: size out of range");
  const int64_t n = Bsz * H * P * N, per_rank = n + Bsz * H;
  const float* base = static_cast<const float*>(packed);
  return launch_fixup(base, base + n, (int)rank, 0, per_rank, H * P * N, per_rank, H, C, dt, A_log, y,
                      dim3((unsigned)(H * FKC), (unsigned)Bsz), L, H, N, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int tssm_ssd_pieces_final_state(const void* S, const void* decay_log2, int64_t pieces, void* state_out,
                                           void* decay_out, int64_t Bsz, int64_t H, int64_t P, int64_t N,
                                           tssm_stream_t stream) {
  using namespace tssm;
  TSSM_REQUIRE(pieces >= 1 && pieces <= 65535, "ssd_pieces_final_state: pieces in [1, 65535]");
  TSSM_REQUIRE(Bsz >= 0 && H >= 0 && P >= 1 && N >= 1 && (P * N) % 4 == 0,
               "ssd_pieces_final_state: bad size (P*N must be a multiple of 4)");
  if (Bsz * H == 0 || (!state_out && !decay_out)) return TSSM_OK;
  TSSM_REQUIRE(S && decay_log2, "ssd_pieces_final_state: null pointer");
  TSSM_REQUIRE(aligned16(S) && (!state_out || aligned16(state_out)), "ssd_pieces_final_state: states must be 16-byte aligned");
  TSSM_REQUIRE(P * N / 4 < (int64_t(1) << 31) && H < (int64_t(1) << 31), "ssd_pieces_final_state: size out of range");
  const int64_t pn4 = P * N / 4, hpn4 = H * pn4, n4 = Bsz * hpn4;
  ssd_pieces_final_state_kernel<<<(unsigned)cdiv(n4, 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const float4*>(S), static_cast<const float*>(decay_log2), (int)pieces,
      static_cast<float4*>(state_out), static_cast<float*>(decay_out), n4, hpn4, (int)pn4, (int)H);
  return check_launch("ssd_pieces_final_state");
}
