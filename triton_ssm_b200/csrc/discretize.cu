// ZOH discretisation (replaces discretize_kernel.py:15-57 and :60-94).
//
// Pure HBM stream: per element one read of B and two writes (Abar, Bbar);
// A_log[H] and dt[Bsz,T] are tiny and stay in L1/L2.  The vector path moves
// four consecutive h per thread (128-bit f32 / 64-bit bf16 accesses).
#include "common.cuh"

namespace tssm {
namespace {

template <typename T> struct vec4;
template <> struct vec4<float> {
  using type = float4;
  __device__ __forceinline__ static void unpack(type v, float (&f)[4]) { f[0] = v.x; f[1] = v.y; f[2] = v.z; f[3] = v.w; }
  __device__ __forceinline__ static type pack(const float (&f)[4]) { return make_float4(f[0], f[1], f[2], f[3]); }
};
template <> struct vec4<__nv_bfloat16> {
  using type = uint2;
  __device__ __forceinline__ static void unpack(type v, float (&f)[4]) {
    __nv_bfloat162 a = *reinterpret_cast<__nv_bfloat162*>(&v.x);
    __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162*>(&v.y);
    f[0] = __low2float(a); f[1] = __high2float(a); f[2] = __low2float(b); f[3] = __high2float(b);
  }
  __device__ __forceinline__ static type pack(const float (&f)[4]) {
    __nv_bfloat162 a = __floats2bfloat162_rn(f[0], f[1]);
    __nv_bfloat162 b = __floats2bfloat162_rn(f[2], f[3]);
    type v;
    v.x = *reinterpret_cast<uint32_t*>(&a);
    v.y = *reinterpret_cast<uint32_t*>(&b);
    return v;
  }
};

template <typename T>
__device__ __forceinline__ void zoh_one(float a, float dtv, float bc, float& abar, float& bbar) {
  const float x = dtv * a;
  const float e = expf(x);
  abar = e;
  const float em1 = std::is_same<T, float>::value ? expm1_guard_f32(x, e) : expm1_guard_bf16(x, e);
  bbar = em1 / (a + 1e-12f) * bc;
}

template <typename T, bool VEC>
__global__ void __launch_bounds__(256) zoh_discretize_kernel(
    const float* __restrict__ A_log, const T* __restrict__ B, const float* __restrict__ dt,
    T* __restrict__ Abar, T* __restrict__ Bbar, int64_t Bsz, int64_t Tn, int64_t H,
    int64_t sBb, int64_t sBt, int64_t sdb, int64_t sdt, int64_t sab, int64_t sat,
    int64_t sbb, int64_t sbt) {
  const int64_t hv = VEC ? (H >> 2) : H;
  const int64_t items = Bsz * Tn * hv;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < items; i += stride) {
    const int64_t row = i / hv;
    const int64_t hi = i - row * hv;
    const int64_t b = row / Tn;
    const int64_t t = row - b * Tn;
    const float dtv = __ldg(dt + b * sdb + t * sdt);
    if constexpr (VEC) {
      const int64_t h0 = hi << 2;
      const float4 al = __ldg(reinterpret_cast<const float4*>(A_log + h0));
      const float alv[4] = {al.x, al.y, al.z, al.w};
      float bc[4], ab[4], bb[4];
      vec4<T>::unpack(*reinterpret_cast<const typename vec4<T>::type*>(B + b * sBb + t * sBt + h0), bc);
#pragma unroll
      for (int k = 0; k < 4; ++k) zoh_one<T>(-expf(alv[k]), dtv, bc[k], ab[k], bb[k]);
      *reinterpret_cast<typename vec4<T>::type*>(Abar + b * sab + t * sat + h0) = vec4<T>::pack(ab);
      *reinterpret_cast<typename vec4<T>::type*>(Bbar + b * sbb + t * sbt + h0) = vec4<T>::pack(bb);
    } else {
      const float a = -expf(__ldg(A_log + hi));
      float ab, bb;
      zoh_one<T>(a, dtv, ldf(B + b * sBb + t * sBt + hi), ab, bb);
      stf(Abar + b * sab + t * sat + hi, ab);
      stf(Bbar + b * sbb + t * sbt + hi, bb);
    }
  }
}

template <typename T>
int launch(const float* A_log, const T* B, const float* dt, T* Abar, T* Bbar, int64_t Bsz,
           int64_t Tn, int64_t H, int64_t sBb, int64_t sBt, int64_t sdb, int64_t sdt, int64_t sab,
           int64_t sat, int64_t sbb, int64_t sbt, cudaStream_t st) {
  const int vbytes = 4 * sizeof(T);
  auto al = [&](const void* p) { return (reinterpret_cast<uintptr_t>(p) % vbytes) == 0; };
  const bool vec = (H % 4 == 0) && sBb % 4 == 0 && sBt % 4 == 0 && sab % 4 == 0 && sat % 4 == 0 &&
                   sbb % 4 == 0 && sbt % 4 == 0 && al(B) && al(Abar) && al(Bbar) && aligned16(A_log);
  const int64_t items = Bsz * Tn * (vec ? H / 4 : H);
  if (items == 0) return TSSM_OK;
  const int threads = 256;
  const int64_t blocks = std::min<int64_t>(cdiv(items, threads), (int64_t)kNumSMs * 16);
  if (vec)
    zoh_discretize_kernel<T, true><<<(unsigned)blocks, threads, 0, st>>>(
        A_log, B, dt, Abar, Bbar, Bsz, Tn, H, sBb, sBt, sdb, sdt, sab, sat, sbb, sbt);
  else
    zoh_discretize_kernel<T, false><<<(unsigned)blocks, threads, 0, st>>>(
        A_log, B, dt, Abar, Bbar, Bsz, Tn, H, sBb, sBt, sdb, sdt, sab, sat, sbb, sbt);
  return check_launch("zoh_discretize");
}

}  // namespace
}  // namespace tssm

extern "C" int tssm_zoh_discretize(const void* A_log, const void* B, const void* dt, void* Abar,
                                   void* Bbar, int64_t Bsz, int64_t T, int64_t H,
                                   int64_t stride_Bb, int64_t stride_Bt, int64_t stride_db,
                                   int64_t stride_dt, int64_t stride_ab, int64_t stride_at,
                                   int64_t stride_bb, int64_t stride_bt, int io_dtype,
                                   tssm_stream_t stream) {
  using namespace tssm;
  TSSM_REQUIRE(Bsz >= 0 && T >= 0 && H >= 0, "zoh_discretize: negative size");
  if (Bsz * T * H == 0) return TSSM_OK;
  TSSM_REQUIRE(A_log && B && dt && Abar && Bbar, "zoh_discretize: null pointer");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (io_dtype == TSSM_F32)
    return launch<float>((const float*)A_log, (const float*)B, (const float*)dt, (float*)Abar,
                         (float*)Bbar, Bsz, T, H, stride_Bb, stride_Bt, stride_db, stride_dt,
                         stride_ab, stride_at, stride_bb, stride_bt, st);
  if (io_dtype == TSSM_BF16)
    return launch<__nv_bfloat16>((const float*)A_log, (const __nv_bfloat16*)B, (const float*)dt,
                                 (__nv_bfloat16*)Abar, (__nv_bfloat16*)Bbar, Bsz, T, H, stride_Bb,
                                 stride_Bt, stride_db, stride_dt, stride_ab, stride_at, stride_bb,
                                 stride_bt, st);
  set_error("zoh_discretize: io_dtype must be f32 or bf16 (got %d)", io_dtype);
  return TSSM_ERR_INVALID;
}
