// Per-token activation quantisation (d3trt/model/quant.py:92-100) and, on a
// weight matrix, per-output-channel weight quantisation (quant.py:77-89).
//
// One warp owns one row. Pass 1 reads the row with 16-byte loads and reduces
// max|x| with warp shuffles; pass 2 re-reads the row (an L1/L2 hit: the row was
// just streamed) and writes the 8-bit codes. HBM traffic is the algorithmic
// minimum: read x once (2 B/elem for bf16), write q (1 B/elem) and the scale.
//
// Bit-exactness with the reference formulas:
//   amax  = max(max_k |x|, 1e-12f)                (fp32, order independent)
//   scale = amax / 448 (fp8) or amax / 127 (int8)   (IEEE fp32 division)
//   fp8 : q = e4m3fn(clamp(x / scale, -448, 448))   cvt.rn.satfinite = RNE
//   int8: q = int8(clamp(rint(x / scale), -127, 127))  rint = half-to-even
// x / scale uses __fdiv_rn (IEEE), never a reciprocal multiply.
#include "common.cuh"

namespace {

constexpr int kWarpsPerCta = 8;

template <typename T>
struct Vec;  // 16-byte vector of T converted to fp32
template <>
struct Vec<float> {
  static constexpr int N = 4;
  __device__ static void load(const float* p, float (&v)[8]) {
    float4 a = __ldg(reinterpret_cast<const float4*>(p));
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  }
};
template <>
struct Vec<__nv_bfloat16> {
  static constexpr int N = 8;
  __device__ static void load(const __nv_bfloat16* p, float (&v)[8]) {
    uint4 a = __ldg(reinterpret_cast<const uint4*>(p));
    const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[2 * i] = __uint_as_float(w[i] << 16);
      v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    }
  }
};
template <>
struct Vec<__half> {
  static constexpr int N = 8;
  __device__ static void load(const __half* p, float (&v)[8]) {
    uint4 a = __ldg(reinterpret_cast<const uint4*>(p));
    const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
      float2 f = __half22float2(h);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  }
};

__device__ __forceinline__ float to_f32(float x) { return x; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ float to_f32(__half x) { return __half2float(x); }

// Two fp32 -> two e4m3fn bytes, round-to-nearest-even, saturating to +-448.
__device__ __forceinline__ uint32_t e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

template <int MODE>
__device__ __forceinline__ uint32_t quant1(float x, float scale) {
  if (MODE == D3B_MODE_FP8) {
    float v = fminf(fmaxf(__fdiv_rn(x, scale), -448.f), 448.f);
    return e4m3x2(v, 0.f) & 0xFFu;
  } else {
    int i = __float2int_rn(__fdiv_rn(x, scale));
    i = min(max(i, -127), 127);
    return static_cast<uint32_t>(i) & 0xFFu;
  }
}

template <typename T, int MODE>
__global__ void __launch_bounds__(kWarpsPerCta * 32) act_quant_kernel(const T* __restrict__ x, int64_t ldx,
                                                                       uint8_t* __restrict__ q,
                                                                       float* __restrict__ scale_out, int64_t M,
                                                                       int64_t K, int vec_ok) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kWarpsPerCta + (threadIdx.x >> 5);
  if (row >= M) return;
  const T* xr = x + row * ldx;
  uint8_t* qr = q + row * K;
  constexpr int VN = Vec<T>::N;

  // ---- pass 1: max |x| ----
  float amax = 0.f;
  int64_t k_vec_end = 0;
  if (vec_ok) {
    k_vec_end = (K / (VN * 32)) * (VN * 32);
#pragma unroll 4
    for (int64_t k = (int64_t)lane * VN; k < k_vec_end; k += 32 * VN) {
      float v[8];
      Vec<T>::load(xr + k, v);
#pragma unroll
      for (int i = 0; i < VN; ++i) amax = fmaxf(amax, fabsf(v[i]));
    }
  }
  for (int64_t k = k_vec_end + lane; k < K; k += 32) amax = fmaxf(amax, fabsf(to_f32(xr[k])));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  amax = fmaxf(amax, 1e-12f);
  const float scale = __fdiv_rn(amax, MODE == D3B_MODE_FP8 ? 448.f : 127.f);
  if (lane == 0) scale_out[row] = scale;

  // ---- pass 2: codes ----
  if (vec_ok) {
#pragma unroll 4
    for (int64_t k = (int64_t)lane * VN; k < k_vec_end; k += 32 * VN) {
      float v[8];
      Vec<T>::load(xr + k, v);
      if (VN == 8) {
        uint32_t w0 = 0, w1 = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) w0 |= quant1<MODE>(v[i], scale) << (8 * i);
#pragma unroll
        for (int i = 0; i < 4; ++i) w1 |= quant1<MODE>(v[4 + i], scale) << (8 * i);
        *reinterpret_cast<uint2*>(qr + k) = make_uint2(w0, w1);
      } else {
        uint32_t w0 = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) w0 |= quant1<MODE>(v[i], scale) << (8 * i);
        *reinterpret_cast<uint32_t*>(qr + k) = w0;
      }
    }
  }
  for (int64_t k = k_vec_end + lane; k < K; k += 32) qr[k] = static_cast<uint8_t>(quant1<MODE>(to_f32(xr[k]), scale));
}

template <typename T>
int launch_typed(const void* x, int64_t ldx, void* q, float* scale, int64_t M, int64_t K, int mode,
                 cudaStream_t stream) {
  const int elem = sizeof(T);
  // 16-byte vector loads need an aligned base and row pitch; 4/8-byte stores
  // need K to keep every row start aligned.
  const int vec_ok = (reinterpret_cast<uintptr_t>(x) % 16 == 0) && ((ldx * elem) % 16 == 0) &&
                     (reinterpret_cast<uintptr_t>(q) % 16 == 0) && (K % 8 == 0);
  const int64_t blocks = (M + kWarpsPerCta - 1) / kWarpsPerCta;
  if (blocks > 0x7FFFFFFF) return D3B_EINVAL;
  dim3 grid((unsigned)blocks), block(kWarpsPerCta * 32);
  if (mode == D3B_MODE_FP8)
    act_quant_kernel<T, D3B_MODE_FP8><<<grid, block, 0, stream>>>(static_cast<const T*>(x), ldx,
                                                                   static_cast<uint8_t*>(q), scale, M, K, vec_ok);
  else
    act_quant_kernel<T, D3B_MODE_INT8><<<grid, block, 0, stream>>>(static_cast<const T*>(x), ldx,
                                                                    static_cast<uint8_t*>(q), scale, M, K, vec_ok);
  return d3b_host::check_launch();
}

}  // namespace

extern "C" int d3b_act_quant(const void* x, int x_dtype, int64_t ldx, void* q, float* scale, int64_t M, int64_t K,
                             int mode, d3b_stream_t stream) {
  if (M < 0 || K <= 0 || ldx < K) return D3B_EINVAL;
  if (mode != D3B_MODE_FP8 && mode != D3B_MODE_INT8) return D3B_EINVAL;
  if (M == 0) return D3B_OK;
  if (!x || !q || !scale) return D3B_EINVAL;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (x_dtype) {
    case D3B_F32: return launch_typed<float>(x, ldx, q, scale, M, K, mode, s);
    case D3B_F16: return launch_typed<__half>(x, ldx, q, scale, M, K, mode, s);
    case D3B_BF16: return launch_typed<__nv_bfloat16>(x, ldx, q, scale, M, K, mode, s);
    default: return D3B_EUNSUPPORTED;
  }
}
