// Mean-pooled logit head (replaces mean_pool_logit_kernel,
// streaming_inference_kernel.py:159-194):
//     out[b] = sum_{t,h} W[h] x[b,t,h] / (T*H + 1e-9) + bias
// A CTA reduces 32 rows (t) of one batch row over all H (16-byte loads when
// the rows allow), scales its partial by 1/(T*H + 1e-9) and adds it to out[b]
// with one float atomic; the CTA holding t = 0 also adds the bias.  The order
// of the atomics varies, so the last bits of out may vary between runs.
#include "common.cuh"

namespace tssm {
namespace {

constexpr int POOL_THREADS = 256;
constexpr int POOL_ROWS = 32;

template <typename T, bool VEC>
__global__ void __launch_bounds__(POOL_THREADS) mean_pool_logit_kernel(
    const T* __restrict__ x, const float* __restrict__ W, const float* __restrict__ bias, float* __restrict__ out,
    int64_t Tn, int64_t H, float inv_d) {
  __shared__ float s_part[POOL_THREADS / 32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t b = blockIdx.y;
  const int64_t t0 = (int64_t)blockIdx.x * POOL_ROWS;
  const int64_t t1 = t0 + POOL_ROWS < Tn ? t0 + POOL_ROWS : Tn;
  float acc = 0.f;
  if (VEC) {   // T = float, H % 4 == 0, 16-byte aligned rows
    for (int64_t h = (int64_t)tid * 4; h < H; h += POOL_THREADS * 4) {
      const float4 w = *reinterpret_cast<const float4*>(W + h);
      for (int64_t t = t0; t < t1; ++t) {
        const float4 v = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(x) + (b * Tn + t) * H + h);
        acc += w.x * v.x + w.y * v.y + w.z * v.z + w.w * v.w;
      }
    }
  } else {
    for (int64_t h = tid; h < H; h += POOL_THREADS) {
      const float w = W[h];
      for (int64_t t = t0; t < t1; ++t) acc += w * ldf(x + (b * Tn + t) * H + h);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) s_part[warp] = acc;
  __syncthreads();
  if (tid == 0) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < POOL_THREADS / 32; ++w) s += s_part[w];
    atomicAdd(out + b, s * inv_d + (blockIdx.x == 0 ? bias[0] : 0.f));
  }
}

}  // namespace
}  // namespace tssm

extern "C" int tssm_mean_pool_logit(const void* x, const void* W, const void* bias, void* out, int64_t Bsz, int64_t T,
                                    int64_t H, int dtype, tssm_stream_t stream) {
  using namespace tssm;
  TSSM_REQUIRE(Bsz >= 0 && T >= 0 && H >= 0, "mean_pool_logit: negative size");
  if (Bsz == 0) return TSSM_OK;
  TSSM_REQUIRE(out && bias, "mean_pool_logit: null pointer");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(out, 0, (size_t)Bsz * sizeof(float), st) != cudaSuccess)
    return check_launch("mean_pool_logit: clear out");
  TSSM_REQUIRE(Bsz <= 65535, "mean_pool_logit: batch %lld exceeds 65535", (long long)Bsz);
  const int64_t chunks = T > 0 ? cdiv(T, POOL_ROWS) : 1;   // T = 0 still adds the bias
  TSSM_REQUIRE(chunks < (int64_t(1) << 31), "mean_pool_logit: T too large");
  TSSM_REQUIRE(T * H == 0 || (x && W), "mean_pool_logit: null pointer");
  const float inv_d = (float)(1.0 / ((double)T * (double)H + 1e-9));
  dim3 grid((unsigned)chunks, (unsigned)Bsz);
  const int64_t Te = H == 0 ? 0 : T;   // no features: only the bias
  if (dtype == TSSM_F32) {
    const bool vec = H % 4 == 0 && aligned16(x) && aligned16(W);
    if (vec)
      mean_pool_logit_kernel<float, true><<<grid, POOL_THREADS, 0, st>>>((const float*)x, (const float*)W,
                                                                         (const float*)bias, (float*)out, Te, H, inv_d);
    else
      mean_pool_logit_kernel<float, false><<<grid, POOL_THREADS, 0, st>>>(
          (const float*)x, (const float*)W, (const float*)bias, (float*)out, Te, H, inv_d);
  } else if (dtype == TSSM_BF16) {
    mean_pool_logit_kernel<__nv_bfloat16, false><<<grid, POOL_THREADS, 0, st>>>(
        (const __nv_bfloat16*)x, (const float*)W, (const float*)bias, (float*)out, Te, H, inv_d);
  } else {
    set_error("mean_pool_logit: dtype must be f32 or bf16 (got %d)", dtype);
    return TSSM_ERR_INVALID;
  }
  return check_launch("mean_pool_logit");
}
