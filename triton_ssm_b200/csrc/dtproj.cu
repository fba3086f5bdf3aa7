// Delta-t projection (replaces dt_project_softplus_kernel,
// discretize_kernel.py:165-213) and its fusion into the ZOH discretisation.
//
//   acc[b,t,h] = sum_r dt_raw[b,t,r] W[r,h] + bias[h]          (:193-204)
//   dt         = clamp(log(1 + exp(acc)), dt_min, dt_max)      (:207-210)
// and, fused, with one dt per (b, t, h) (the selective form of
// discretize_kernel.py:38-54):
//   Abar = exp(dt a), Bbar = expm1*(dt a) / (a + 1e-12) B,  a = -exp(A_log[h]).
// The tensor-core kernel (dtproj_tc.cu) takes dt_rank <= 64 with dt_rank % 4 == 0
// and a 16-byte aligned dt_raw; the CUDA-core kernel below takes the rest.  A
// CTA computes a [32 rows x 128 channels] tile: W's 128-column slab and the
// 32 rows of dt_raw sit in shared memory, each thread accumulates 4 rows x 4
// channels over r in the reference's order (one fma per r, two channels per
// packed f32x2 instruction), and the epilogue writes dt, or Abar and Bbar,
// without dt ever reaching HBM.
#include "common.cuh"

namespace tssm {
namespace {

constexpr int DTP_THREADS = 256;
constexpr int DTP_HT = 128;   // channels per CTA
constexpr int DTP_RB = 32;    // (b, t) rows per CTA
constexpr int DTP_RMAX = 256;

// VEC: H % 4 == 0 and 16-byte aligned outputs (and B): float4 stores.
template <bool DISC, bool VEC>
__global__ void __launch_bounds__(DTP_THREADS) dt_project_kernel(
    const float* __restrict__ dt_raw, const float* __restrict__ W, const float* __restrict__ bias,
    const float* __restrict__ A_log, const float* __restrict__ B, float* __restrict__ dt_out,
    float* __restrict__ Abar, float* __restrict__ Bbar, int64_t rows, int64_t H, int R, float dt_min, float dt_max) {
  extern __shared__ __align__(16) float s_dyn[];
  const int R4 = (R + 3) & ~3;            // r padded to a multiple of 4 (zeros)
  const int XS = R4 + 4;                  // row stride of Xs (16-byte aligned)
  float* Ws = s_dyn;                      // [R4][DTP_HT]
  float* Xs = s_dyn + R4 * DTP_HT;        // [DTP_RB][XS]
  const int tid = threadIdx.x, lane = tid & 31, grp = tid >> 5;
  const int64_t r0 = (int64_t)blockIdx.x * DTP_RB;
  const int64_t h0 = (int64_t)blockIdx.y * DTP_HT;
  for (int i = tid; i < R4 * DTP_HT; i += DTP_THREADS) {
    const int r = i / DTP_HT, c = i % DTP_HT;
    Ws[i] = (r < R && h0 + c < H) ? W[(int64_t)r * H + h0 + c] : 0.f;
  }
  for (int i = tid; i < DTP_RB * R4; i += DTP_THREADS) {
    const int row = i / R4, r = i % R4;
    Xs[row * XS + r] = (r < R && r0 + row < rows) ? dt_raw[(r0 + row) * R + r] : 0.f;
  }
  __syncthreads();
  const int hc = lane * 4;
  // acc[i][0] holds channels (hc, hc+1), acc[i][1] (hc+2, hc+3) of row grp+8i; one
  // packed fma per pair and r, in r order (the padding adds exact zeros)
  float2 acc[4][2];
#pragma unroll
  for (int i = 0; i < 4; ++i) acc[i][0] = acc[i][1] = make_float2(0.f, 0.f);
  for (int r = 0; r < R4; r += 4) {
    float4 x[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) x[i] = *reinterpret_cast<const float4*>(Xs + (grp + 8 * i) * XS + r);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float4 w = *reinterpret_cast<const float4*>(Ws + (r + q) * DTP_HT + hc);
      const float2 w01 = make_float2(w.x, w.y), w23 = make_float2(w.z, w.w);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float xv = q == 0 ? x[i].x : q == 1 ? x[i].y : q == 2 ? x[i].z : x[i].w;
        const float2 x2 = make_float2(xv, xv);
        acc[i][0] = ffma2(x2, w01, acc[i][0]);
        acc[i][1] = ffma2(x2, w23, acc[i][1]);
      }
    }
  }
  // per channel: bias, a = -exp(A_log) and 1 / (a + 1e-12) (the reference divides by
  // a + 1e-12 for every element; one reciprocal per channel differs by at most an ulp)
  float bs[4], a[4], ra[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int64_t hh = h0 + hc + k;
    bs[k] = hh < H ? bias[hh] : 0.f;
    a[k] = (DISC && hh < H) ? -expf(A_log[hh]) : -1.f;
    ra[k] = 1.0f / (a[k] + 1e-12f);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t row = r0 + grp + 8 * i;
    if (row >= rows) continue;
    const int64_t base = row * H + h0 + hc;
    float dtv[4], ab[4], bb[4], bin[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float v = (k == 0 ? acc[i][0].x : k == 1 ? acc[i][0].y : k == 2 ? acc[i][1].x : acc[i][1].y) + bs[k];
      dtv[k] = fminf(fmaxf(logf(1.0f + expf(v)), dt_min), dt_max);
    }
    if (DISC) {
      if (VEC && h0 + hc < H) {
        const float4 q = *reinterpret_cast<const float4*>(B + base);
        bin[0] = q.x; bin[1] = q.y; bin[2] = q.z; bin[3] = q.w;
      } else {
#pragma unroll
        for (int k = 0; k < 4; ++k) bin[k] = h0 + hc + k < H ? B[base + k] : 0.f;
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float x = dtv[k] * a[k];
        const float e = expf(x);
        ab[k] = e;
        bb[k] = expm1_guard_f32(x, e) * ra[k] * bin[k];
      }
    }
    if (VEC) {
      if (h0 + hc < H) {
        if (dt_out) *reinterpret_cast<float4*>(dt_out + base) = make_float4(dtv[0], dtv[1], dtv[2], dtv[3]);
        if (DISC) {
          *reinterpret_cast<float4*>(Abar + base) = make_float4(ab[0], ab[1], ab[2], ab[3]);
          *reinterpret_cast<float4*>(Bbar + base) = make_float4(bb[0], bb[1], bb[2], bb[3]);
        }
      }
    } else {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if (h0 + hc + k >= H) continue;
        if (dt_out) dt_out[base + k] = dtv[k];
        if (DISC) {
          Abar[base + k] = ab[k];
          Bbar[base + k] = bb[k];
        }
      }
    }
  }
}

}  // namespace

// dtproj_tc.cu: the same arithmetic with the contraction on tcgen05 tensor cores
// (TSSM_ERR_UNSUPPORTED when its size and alignment conditions do not hold).
int launch_dtproj_tc(bool disc, const void* dt_raw, const void* W, const void* bias, const void* A_log, const void* B,
                     void* dt_out, void* Abar, void* Bbar, int64_t rows, int64_t H, int64_t R, double dt_min,
                     double dt_max, cudaStream_t st);

namespace {

template <bool DISC>
int launch_dtproj(const void* dt_raw, const void* W, const void* bias, const void* A_log, const void* B, void* dt_out,
                  void* Abar, void* Bbar, int64_t rows, int64_t H, int64_t R, double dt_min, double dt_max,
                  cudaStream_t st) {
  const int tc = launch_dtproj_tc(DISC, dt_raw, W, bias, A_log, B, dt_out, Abar, Bbar, rows, H, R, dt_min, dt_max, st);
  if (tc != TSSM_ERR_UNSUPPORTED) return tc;
  const size_t R4 = (size_t)((R + 3) & ~3);
  const size_t smem = (R4 * DTP_HT + (size_t)DTP_RB * (R4 + 4)) * sizeof(float);
  const bool vec = H % 4 == 0 && (!dt_out || aligned16(dt_out)) &&
                   (!DISC || (aligned16(Abar) && aligned16(Bbar) && aligned16(B)));
  auto kern = vec ? dt_project_kernel<DISC, true> : dt_project_kernel<DISC, false>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return check_launch("dt_project: set smem attribute");
  dim3 grid((unsigned)cdiv(rows, DTP_RB), (unsigned)cdiv(H, DTP_HT));
  kern<<<grid, DTP_THREADS, smem, st>>>((const float*)dt_raw, (const float*)W, (const float*)bias,
                                        (const float*)A_log, (const float*)B, (float*)dt_out, (float*)Abar,
                                        (float*)Bbar, rows, H, (int)R, (float)dt_min, (float)dt_max);
  return check_launch(DISC ? "zoh_discretize_dtproj" : "dt_project_softplus");
}

int check_dtproj_sizes(const char* who, int64_t Bsz, int64_t T, int64_t H, int64_t R, double dt_min, double dt_max) {
  TSSM_REQUIRE(Bsz >= 0 && T >= 0 && H >= 0 && R >= 1, "%s: bad size", who);
  TSSM_REQUIRE(R <= DTP_RMAX, "%s: dt_rank %lld exceeds %d", who, (long long)R, DTP_RMAX);
  TSSM_REQUIRE(dt_min <= dt_max, "%s: dt_min > dt_max", who);
  TSSM_REQUIRE(cdiv(Bsz * T, DTP_RB) < (int64_t(1) << 31) && cdiv(H, DTP_HT) <= 65535, "%s: size exceeds the grid",
               who);
  return TSSM_OK;
}

}  // namespace
}  // namespace tssm

extern "C" int tssm_dt_project_softplus(const void* dt_raw, const void* W, const void* bias, void* dt_out,
                                        int64_t Bsz, int64_t T, int64_t H, int64_t R, double dt_min, double dt_max,
                                        tssm_stream_t stream) {
  using namespace tssm;
  if (int rc = check_dtproj_sizes("dt_project_softplus", Bsz, T, H, R, dt_min, dt_max)) return rc;
  if (Bsz * T * H == 0) return TSSM_OK;
  TSSM_REQUIRE(dt_raw && W && bias && dt_out, "dt_project_softplus: null pointer");
  return launch_dtproj<false>(dt_raw, W, bias, nullptr, nullptr, dt_out, nullptr, nullptr, Bsz * T, H, R, dt_min,
                              dt_max, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int tssm_zoh_discretize_dtproj(const void* A_log, const void* B, const void* dt_raw, const void* W,
                                          const void* bias, void* Abar, void* Bbar, void* dt_out, int64_t Bsz,
                                          int64_t T, int64_t H, int64_t R, double dt_min, double dt_max,
                                          tssm_stream_t stream) {
  using namespace tssm;
  if (int rc = check_dtproj_sizes("zoh_discretize_dtproj", Bsz, T, H, R, dt_min, dt_max)) return rc;
  if (Bsz * T * H == 0) return TSSM_OK;
  TSSM_REQUIRE(A_log && B && dt_raw && W && bias && Abar && Bbar, "zoh_discretize_dtproj: null pointer");
  return launch_dtproj<true>(dt_raw, W, bias, A_log, B, dt_out, Abar, Bbar, Bsz * T, H, R, dt_min, dt_max,
                             reinterpret_cast<cudaStream_t>(stream));
}
