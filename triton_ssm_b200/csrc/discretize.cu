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

// ra = 1 / (a + 1e-12), once per channel: (exp(x)-1)/(a+1e-12) is taken as a product
// with it (within an ulp of the quotient) instead of a division per element.
template <typename T>
__device__ __forceinline__ void zoh_one(float a, float ra, float dtv, float bc, float& abar, float& bbar) {
  const float x = dtv * a;
  const float e = expf(x);
  abar = e;
  const float em1 = std::is_same<T, float>::value ? expm1_guard_f32(x, e) : expm1_guard_bf16(x, e);
  bbar = em1 * ra * bc;
}

constexpr int ZR = 4;   // rows whose loads one thread has in flight

// ZR rows (nr of them valid) starting at row r0, channels h0 .. h0+W-1 with
// their a = -exp(A_log) and ra = 1/(a + 1e-12).
template <typename T, bool VEC>
__device__ __forceinline__ void zoh_rows(const float (&a)[VEC ? 4 : 1], const float (&ra)[VEC ? 4 : 1],
                                         const T* __restrict__ B, const float* __restrict__ dt,
                                         T* __restrict__ Abar, T* __restrict__ Bbar, int64_t Tn, int64_t h0,
                                         int64_t r0, int nr, int64_t sBb, int64_t sBt, int64_t sdb, int64_t sdt,
                                         int64_t sab, int64_t sat, int64_t sbb, int64_t sbt) {
  const int64_t b0 = r0 / Tn, t0 = r0 - b0 * Tn;
  // every row's loads go out first (ZR of them in flight per thread), then the math and stores
  int64_t bs[ZR], ts[ZR];
  {
    int64_t b = b0, t = t0;
#pragma unroll
    for (int r = 0; r < ZR; ++r) {
      bs[r] = b;
      ts[r] = t;
      if (++t == Tn) { t = 0; ++b; }
    }
  }
  if constexpr (VEC) {
    typename vec4<T>::type bv[ZR];
    float dtv[ZR];
#pragma unroll
    for (int r = 0; r < ZR; ++r) {
      if (r < nr) {
        bv[r] = *reinterpret_cast<const typename vec4<T>::type*>(B + bs[r] * sBb + ts[r] * sBt + h0);
        dtv[r] = __ldg(dt + bs[r] * sdb + ts[r] * sdt);
      }
    }
#pragma unroll
    for (int r = 0; r < ZR; ++r) {
      if (r < nr) {
        float bc[4], ab[4], bb[4];
        vec4<T>::unpack(bv[r], bc);
#pragma unroll
        for (int k = 0; k < 4; ++k) zoh_one<T>(a[k], ra[k], dtv[r], bc[k], ab[k], bb[k]);
        *reinterpret_cast<typename vec4<T>::type*>(Abar + bs[r] * sab + ts[r] * sat + h0) = vec4<T>::pack(ab);
        *reinterpret_cast<typename vec4<T>::type*>(Bbar + bs[r] * sbb + ts[r] * sbt + h0) = vec4<T>::pack(bb);
      }
    }
  } else {
    float bv[ZR], dtv[ZR];
#pragma unroll
    for (int r = 0; r < ZR; ++r) {
      if (r < nr) {
        bv[r] = ldf(B + bs[r] * sBb + ts[r] * sBt + h0);
        dtv[r] = __ldg(dt + bs[r] * sdb + ts[r] * sdt);
      }
    }
#pragma unroll
    for (int r = 0; r < ZR; ++r) {
      if (r < nr) {
        float ab, bb;
        zoh_one<T>(a[0], ra[0], dtv[r], bv[r], ab, bb);
        stf(Abar + bs[r] * sab + ts[r] * sat + h0, ab);
        stf(Bbar + bs[r] * sbb + ts[r] * sbt + h0, bb);
      }
    }
  }
}

// CTA = (a contiguous range of (b, t) rows, 256*W channels): each thread owns
// W channels (W = 4: one 128-bit / 64-bit vector) and walks the range ZR rows
// at a time, so the per-channel a = -exp(A_log) is computed once per thread and
// (b, t) is stepped rather than divided out.  The rows are split evenly over a
// grid of a whole number of CTAs per SM (every SM moves the same bytes: a short
// stream has no tail of half-empty waves), with enough CTAs that every SM keeps
// full occupancy's worth of loads in flight.

template <typename T, bool VEC>
__global__ void __launch_bounds__(256) zoh_discretize_kernel(
    const float* __restrict__ A_log, const T* __restrict__ B, const float* __restrict__ dt,
    T* __restrict__ Abar, T* __restrict__ Bbar, int64_t Bsz, int64_t Tn, int64_t H,
    int64_t sBb, int64_t sBt, int64_t sdb, int64_t sdt, int64_t sab, int64_t sat,
    int64_t sbb, int64_t sbt) {
  constexpr int W = VEC ? 4 : 1;
  const int64_t h0 = ((int64_t)blockIdx.y * blockDim.x + threadIdx.x) * W;
  const int64_t rows = Bsz * Tn;
  const int64_t ra0 = rows * blockIdx.x / gridDim.x, ra1 = rows * (blockIdx.x + 1) / gridDim.x;
  if (h0 >= H || ra0 >= ra1) return;
  float a[W], ra[W];
  if constexpr (VEC) {
    const float4 al = __ldg(reinterpret_cast<const float4*>(A_log + h0));
    a[0] = -expf(al.x); a[1] = -expf(al.y); a[2] = -expf(al.z); a[3] = -expf(al.w);
  } else {
    a[0] = -expf(__ldg(A_log + h0));
  }
#pragma unroll
  for (int k = 0; k < W; ++k) ra[k] = 1.0f / (a[k] + 1e-12f);
  for (int64_t r0 = ra0; r0 < ra1; r0 += ZR)
    zoh_rows<T, VEC>(a, ra, B, dt, Abar, Bbar, Tn, h0, r0, (int)min((int64_t)ZR, ra1 - r0), sBb, sBt, sdb, sdt, sab,
                     sat, sbb, sbt);
}

template <typename T>
int launch(const float* A_log, const T* B, const float* dt, T* Abar, T* Bbar, int64_t Bsz,
           int64_t Tn, int64_t H, int64_t sBb, int64_t sBt, int64_t sdb, int64_t sdt, int64_t sab,
           int64_t sat, int64_t sbb, int64_t sbt, cudaStream_t st) {
  const int vbytes = 4 * sizeof(T);
  auto al = [&](const void* p) { return (reinterpret_cast<uintptr_t>(p) % vbytes) == 0; };
  const bool vec = (H % 4 == 0) && sBb % 4 == 0 && sBt % 4 == 0 && sab % 4 == 0 && sat % 4 == 0 &&
                   sbb % 4 == 0 && sbt % 4 == 0 && al(B) && al(Abar) && al(Bbar) && aligned16(A_log);
  if (Bsz * Tn * H == 0) return TSSM_OK;
  const int64_t gcol = cdiv(vec ? H / 4 : H, 256);
  // up to sixteen 256-thread CTAs per SM per column block (two waves at full
  // occupancy), rows split evenly over them: measured 0.89 of the copy bandwidth
  // at B16 T1024 H1024 against 0.79 with two CTAs per SM and eight rows per step
  const int64_t grow = std::min<int64_t>(cdiv(Bsz * Tn, ZR), std::max<int64_t>(1, 16 * num_sms() / gcol));
  TSSM_REQUIRE(gcol <= 65535, "zoh_discretize: size exceeds the grid");
  const dim3 grid((unsigned)grow, (unsigned)gcol);
  if (vec)
    zoh_discretize_kernel<T, true><<<grid, 256, 0, st>>>(A_log, B, dt, Abar, Bbar, Bsz, Tn, H, sBb, sBt, sdb, sdt,
                                                        sab, sat, sbb, sbt);
  else
    zoh_discretize_kernel<T, false><<<grid, 256, 0, st>>>(A_log, B, dt, Abar, Bbar, Bsz, Tn, H, sBb, sBt, sdb, sdt,
                                                         sab, sat, sbb, sbt);
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
