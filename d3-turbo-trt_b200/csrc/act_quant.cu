// Per-token activation quantisation (d3trt/model/quant.py:92-100) and, on a
// weight matrix, per-output-channel weight quantisation (quant.py:77-89).
//
// One warp owns one row. Rows up to 32 lanes x 8 x kMaxVec elements are read
// once into registers with 16-byte loads (all in flight together), reduced to
// max|x| with warp shuffles and quantised from registers: HBM traffic is the
// algorithmic minimum (read x once, write q and the scale). Longer rows use a
// two-pass variant whose second read hits L2.
//
// Bit-exactness with the reference formulas:
//   amax  = max(max_k |x|, 1e-12f)                (fp32, order independent)
//   scale = amax / 448 (fp8) or amax / 127 (int8)   (IEEE fp32 division)
//   fp8 : q = e4m3fn(clamp(x / scale, -448, 448))   cvt.rn.satfinite = RNE
//   int8: q = int8(clamp(rint(x / scale), -127, 127))  rint = half-to-even
// x / scale must be the IEEE quotient RN(x / scale). Per element the kernel
// first forms v = RN(x * RN(1 / scale)), which is within 1.5 ulp of x / scale.
// The code only depends on which side of a rounding boundary of the target
// format (an e4m3 midpoint, or k + 1/2 for int8) the quotient lies; when v is
// 4 ulp or more away from every boundary, v and RN(x / scale) give the same
// code. Otherwise the element is recomputed with __fdiv_rn (IEEE). So the
// codes equal those of the reference's IEEE division in every case.
#include "common.cuh"

namespace {

constexpr int kWarpsPerCta = 8;

template <typename T>
struct Vec;  // 16-byte vector of T converted to fp32
template <>
struct Vec<float> {
  static constexpr int N = 4;
  __device__ static void unpack(uint4 a, float (&v)[8]) {
    v[0] = __uint_as_float(a.x); v[1] = __uint_as_float(a.y); v[2] = __uint_as_float(a.z);
    v[3] = __uint_as_float(a.w);
  }
  __device__ static void load(const float* p, float (&v)[8]) { unpack(__ldg(reinterpret_cast<const uint4*>(p)), v); }
};
template <>
struct Vec<__nv_bfloat16> {
  static constexpr int N = 8;
  __device__ static void load(const __nv_bfloat16* p, float (&v)[8]) { unpack(__ldg(reinterpret_cast<const uint4*>(p)), v); }
  __device__ static void unpack(uint4 a, float (&v)[8]) {
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
  __device__ static void load(const __half* p, float (&v)[8]) { unpack(__ldg(reinterpret_cast<const uint4*>(p)), v); }
  __device__ static void unpack(uint4 a, float (&v)[8]) {
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

// True when v may lie within 4 fp32 ulp of a rounding boundary of the target
// format (then RN(x/s) must be computed exactly). |v| <= 448 (fp8) or 127.
template <int MODE>
__device__ __forceinline__ bool near_boundary(float v) {
  const float a = fabsf(v);
  if (MODE == D3B_MODE_FP8) {
    if (a >= 0.015625f) {  // e4m3 normal range: 3 mantissa bits, tie at dropped bits == 0x80000
      const int dropped = static_cast<int>(__float_as_uint(a) & 0xFFFFFu);
      return abs(dropped - 0x80000) <= 4;
    }
    const float t = a * 512.f;  // subnormal quantum 2^-9 (exact scaling)
    return fabsf(t - floorf(t) - 0.5f) <= 1.0f / 32768.f;
  }
  return fabsf(a - floorf(a) - 0.5f) <= 1.0f / 32768.f;  // 4 ulp at |v| < 128
}

template <int MODE>
__device__ __forceinline__ float quotient(float x, float scale, float rcp) {
  float v = __fmul_rn(x, rcp);
  const float lim = MODE == D3B_MODE_FP8 ? 448.f : 127.f;
  if (near_boundary<MODE>(fminf(fmaxf(v, -lim), lim))) v = __fdiv_rn(x, scale);
  return v;
}

// Two elements -> two codes in the low 16 bits (element 0 in bits 0..7).
template <int MODE>
__device__ __forceinline__ uint32_t quant2(float x0, float x1, float scale, float rcp) {
  const float v0 = quotient<MODE>(x0, scale, rcp), v1 = quotient<MODE>(x1, scale, rcp);
  if (MODE == D3B_MODE_FP8) {
    return e4m3x2(fminf(fmaxf(v0, -448.f), 448.f), fminf(fmaxf(v1, -448.f), 448.f));
  } else {
    const int i0 = min(max(__float2int_rn(v0), -127), 127);
    const int i1 = min(max(__float2int_rn(v1), -127), 127);
    return (static_cast<uint32_t>(i0) & 0xFFu) | ((static_cast<uint32_t>(i1) & 0xFFu) << 8);
  }
}

template <int MODE>
__device__ __forceinline__ uint32_t quant1(float x, float scale, float rcp) {
  return quant2<MODE>(x, 0.f, scale, rcp) & 0xFFu;
}

__device__ __forceinline__ float row_scale(float amax, int mode) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  amax = fmaxf(amax, 1e-12f);
  return __fdiv_rn(amax, mode == D3B_MODE_FP8 ? 448.f : 127.f);
}

// Single pass: the row lives in registers (nvec 16-byte vectors per lane).
constexpr int kMaxVec = 24;
constexpr int kCachedWarps = 4;

template <typename T, int MODE>
__global__ void __launch_bounds__(kCachedWarps * 32) act_quant_cached_kernel(const T* __restrict__ x, int64_t ldx,
                                                                              uint8_t* __restrict__ q,
                                                                              float* __restrict__ scale_out,
                                                                              int64_t M, int64_t K) {
  constexpr int VN = Vec<T>::N;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kCachedWarps + (threadIdx.x >> 5);
  if (row >= M) return;
  const T* xr = x + row * ldx;
  uint8_t* qr = q + row * K;
  const int nvec = static_cast<int>(K / (VN * 32));  // full vectors per lane (K % (VN*32) == 0 here)
  uint4 raw[kMaxVec];
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i)
    if (i < nvec) raw[i] = __ldg(reinterpret_cast<const uint4*>(xr + (int64_t)(i * 32 + lane) * VN));
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    if (i < nvec) {
      float v[8];
      Vec<T>::unpack(raw[i], v);
#pragma unroll
      for (int e = 0; e < VN; ++e) amax = fmaxf(amax, fabsf(v[e]));
    }
  }
  const float scale = row_scale(amax, MODE);
  const float rcp = __frcp_rn(scale);
  if (lane == 0) scale_out[row] = scale;
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    if (i < nvec) {
      float v[8];
      Vec<T>::unpack(raw[i], v);
      uint8_t* dst = qr + (int64_t)(i * 32 + lane) * VN;
      if (VN == 8) {
        const uint32_t w0 = quant2<MODE>(v[0], v[1], scale, rcp) | (quant2<MODE>(v[2], v[3], scale, rcp) << 16);
        const uint32_t w1 = quant2<MODE>(v[4], v[5], scale, rcp) | (quant2<MODE>(v[6], v[7], scale, rcp) << 16);
        *reinterpret_cast<uint2*>(dst) = make_uint2(w0, w1);
      } else {
        *reinterpret_cast<uint32_t*>(dst) =
            quant2<MODE>(v[0], v[1], scale, rcp) | (quant2<MODE>(v[2], v[3], scale, rcp) << 16);
      }
    }
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
  const float scale = row_scale(amax, MODE);
  const float rcp = __frcp_rn(scale);
  if (lane == 0) scale_out[row] = scale;

  // ---- pass 2: codes ----
  if (vec_ok) {
#pragma unroll 4
    for (int64_t k = (int64_t)lane * VN; k < k_vec_end; k += 32 * VN) {
      float v[8];
      Vec<T>::load(xr + k, v);
      if (VN == 8) {
        const uint32_t w0 = quant2<MODE>(v[0], v[1], scale, rcp) | (quant2<MODE>(v[2], v[3], scale, rcp) << 16);
        const uint32_t w1 = quant2<MODE>(v[4], v[5], scale, rcp) | (quant2<MODE>(v[6], v[7], scale, rcp) << 16);
        *reinterpret_cast<uint2*>(qr + k) = make_uint2(w0, w1);
      } else {
        const uint32_t w0 = quant2<MODE>(v[0], v[1], scale, rcp) | (quant2<MODE>(v[2], v[3], scale, rcp) << 16);
        *reinterpret_cast<uint32_t*>(qr + k) = w0;
      }
    }
  }
  for (int64_t k = k_vec_end + lane; k < K; k += 32)
    qr[k] = static_cast<uint8_t>(quant1<MODE>(to_f32(xr[k]), scale, rcp));
}

template <typename T>
int launch_typed(const void* x, int64_t ldx, void* q, float* scale, int64_t M, int64_t K, int mode,
                 cudaStream_t stream) {
  const int elem = sizeof(T);
  // 16-byte vector loads need an aligned base and row pitch; 4/8-byte stores
  // need K to keep every row start aligned.
  const int vec_ok = (reinterpret_cast<uintptr_t>(x) % 16 == 0) && ((ldx * elem) % 16 == 0) &&
                     (reinterpret_cast<uintptr_t>(q) % 16 == 0) && (K % 8 == 0);
  constexpr int VN = Vec<T>::N;
  if (vec_ok && K % (VN * 32) == 0 && K / (VN * 32) <= kMaxVec) {
    const int64_t blocks = (M + kCachedWarps - 1) / kCachedWarps;
    if (blocks > 0x7FFFFFFF) return D3B_EINVAL;
    if (mode == D3B_MODE_FP8)
      act_quant_cached_kernel<T, D3B_MODE_FP8><<<(unsigned)blocks, kCachedWarps * 32, 0, stream>>>(
          static_cast<const T*>(x), ldx, static_cast<uint8_t*>(q), scale, M, K);
    else
      act_quant_cached_kernel<T, D3B_MODE_INT8><<<(unsigned)blocks, kCachedWarps * 32, 0, stream>>>(
          static_cast<const T*>(x), ldx, static_cast<uint8_t*>(q), scale, M, K);
    return d3b_host::check_launch();
  }
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
