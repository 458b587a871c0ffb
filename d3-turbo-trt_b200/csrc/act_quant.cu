// Per-token activation quantisation (d3trt/model/quant.py:92-100) and, on a
// weight matrix, per-output-channel weight quantisation (quant.py:77-89).
//
// bf16 rows of 1025 to 18432 elements (every width of the model: hidden 5120,
// attention 6144, MLP 17408) run one CTA of 128 or 256 threads per row: each
// thread reads at most nine 16-byte vectors of the row into registers (all in
// flight together), max|x| is reduced through the warps and shared memory, and
// the codes are written from the same registers. With under 64 registers per
// thread many rows are in flight per SM, so one row's loads overlap other
// rows' arithmetic (a warp per row held only ~9 warps per SM and left loads
// and arithmetic in separate phases: 1.5-1.9x slower). Narrower bf16 rows run
// one warp per row from registers; f16/f32 input takes two passes: pass 1
// reads the row with 16-byte loads (batches of 8 per lane in flight) and
// reduces max|x| with warp shuffles; pass 2 re-reads the row, which the first
// pass has just brought into L2, and writes the 8-bit codes with 8-byte stores.
// HBM traffic is the algorithmic minimum every way: read x once, write q and
// the scale.
//
// Bit-exactness with the reference formulas:
//   amax  = max(max_k |x|, 1e-12f)                (fp32, order independent)
//   scale = amax / 448 (fp8) or amax / 127 (int8)   (IEEE fp32 division)
//   fp8 : q = e4m3fn(clamp(x / scale, -448, 448))   cvt.rn.satfinite = RNE
//   int8: q = int8(clamp(rint(x / scale), -127, 127))  rint = half-to-even
// x / scale must be the IEEE quotient RN(x / scale). Per element the kernel
// forms v = RN(x * RN(1 / scale)) and converts v shrunk and grown by 2^-21
// relative; when both give the same code, so does RN(x / scale) (rounding is
// monotone and the bracket covers the error of v). Otherwise (about one pair
// in 10^5 on N(0,1) data) the pair is recomputed with __fdiv_rn (IEEE). So the
// codes equal those of the reference's IEEE division in every case.
#include <type_traits>

#include "common.cuh"
#include "quant_codes.cuh"

namespace {

using namespace d3b_quant;

constexpr int kWarpsPerCta = 8;

template <typename T>
struct Vec;  // 16-byte vector of T as fp32
template <>
struct Vec<float> {
  static constexpr int N = 4;
  __device__ static void unpack(uint4 a, float (&v)[8]) {
    v[0] = __uint_as_float(a.x); v[1] = __uint_as_float(a.y); v[2] = __uint_as_float(a.z);
    v[3] = __uint_as_float(a.w);
  }
};
template <>
struct Vec<__nv_bfloat16> {
  static constexpr int N = 8;
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
  __device__ static void unpack(uint4 a, float (&v)[8]) {
    const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  }
};

__device__ __forceinline__ float to_f32(float x) { return x; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ float to_f32(__half x) { return __half2float(x); }

// 8 (bf16/f16) or 4 (f32) codes from one 16-byte vector -> one 8- or 4-byte store.
template <typename T, int MODE>
__device__ __forceinline__ void quant_vec(uint4 raw, float scale, float rcp, uint8_t* dst) {
  float v[8];
  Vec<T>::unpack(raw, v);
  if (Vec<T>::N == 8) {
    const uint32_t w0 = quant2<MODE>(v[0], v[1], scale, rcp) | (quant2<MODE>(v[2], v[3], scale, rcp) << 16);
    const uint32_t w1 = quant2<MODE>(v[4], v[5], scale, rcp) | (quant2<MODE>(v[6], v[7], scale, rcp) << 16);
    *reinterpret_cast<uint2*>(dst) = make_uint2(w0, w1);
  } else {
    *reinterpret_cast<uint32_t*>(dst) =
        quant2<MODE>(v[0], v[1], scale, rcp) | (quant2<MODE>(v[2], v[3], scale, rcp) << 16);
  }
}

// ---------------------------------------------------------------------------
// two-pass warp-per-row kernel; VEC: 16-byte aligned rows with K % 8 == 0
// ---------------------------------------------------------------------------
template <typename T, int MODE, bool VEC>
__global__ void __launch_bounds__(kWarpsPerCta * 32) act_quant_kernel(const T* __restrict__ x, int64_t ldx,
                                                                       uint8_t* __restrict__ q,
                                                                       float* __restrict__ scale_out, int64_t M,
                                                                       int64_t K) {
  constexpr int VN = Vec<T>::N;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kWarpsPerCta + (threadIdx.x >> 5);
  if (row >= M) return;
  const T* xr = x + row * ldx;
  uint8_t* qr = q + row * K;
  float amax = 0.f;
  if (VEC) {
    // batches of kBatch 16-byte loads per lane, all issued before any use
    constexpr int kBatch = 8;
    constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
    const uint4* src = reinterpret_cast<const uint4*>(xr);
    const int nvec = static_cast<int>(K / VN);
    uint32_t m0 = 0, m1 = 0;  // bf16: packed max |x|
    for (int k0 = lane; k0 < nvec; k0 += 32 * kBatch) {
      uint4 raw[kBatch];
#pragma unroll
      for (int u = 0; u < kBatch; ++u)
        raw[u] = k0 + 32 * u < nvec ? __ldg(src + k0 + 32 * u) : make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        if constexpr (kBf16) {
          m0 = umax2(m0, raw[u].x & 0x7FFF7FFFu);
          m1 = umax2(m1, raw[u].y & 0x7FFF7FFFu);
          m0 = umax2(m0, raw[u].z & 0x7FFF7FFFu);
          m1 = umax2(m1, raw[u].w & 0x7FFF7FFFu);
        } else {
          float v[8];
          Vec<T>::unpack(raw[u], v);
#pragma unroll
          for (int e = 0; e < VN; ++e) amax = fmaxf(amax, fabsf(v[e]));
        }
      }
    }
    if constexpr (kBf16) {
      const uint32_t m = umax2(m0, m1);
      amax = __uint_as_float(max(m & 0xFFFFu, m >> 16) << 16);
    }
    const float scale = row_scale(amax, MODE);
    const float rcp = __frcp_rn(scale);
    if (lane == 0) scale_out[row] = scale;
    for (int k0 = lane; k0 < nvec; k0 += 32 * kBatch) {
      uint4 raw[kBatch];
#pragma unroll
      for (int u = 0; u < kBatch; ++u)
        if (k0 + 32 * u < nvec) raw[u] = __ldg(src + k0 + 32 * u);
#pragma unroll
      for (int u = 0; u < kBatch; ++u)
        if (k0 + 32 * u < nvec) {
          if constexpr (kBf16)
            *reinterpret_cast<uint2*>(qr + (int64_t)(k0 + 32 * u) * VN) = quant8_bf16<MODE>(raw[u], scale, rcp);
          else
            quant_vec<T, MODE>(raw[u], scale, rcp, qr + (int64_t)(k0 + 32 * u) * VN);
        }
    }
  } else {
    for (int64_t k = lane; k < K; k += 32) amax = fmaxf(amax, fabsf(to_f32(xr[k])));
    const float scale = row_scale(amax, MODE);
    const float rcp = __frcp_rn(scale);
    if (lane == 0) scale_out[row] = scale;
    for (int64_t k = lane; k < K; k += 32)
      qr[k] = static_cast<uint8_t>(quant2<MODE>(to_f32(xr[k]), 0.f, scale, rcp) & 0xFFu);
  }
}

// ---------------------------------------------------------------------------
// bf16 rows with K <= 32 * 8 * NV: one pass, the row held in registers. Each
// lane issues all of its NV 16-byte loads at once (one memory round trip per
// row), reduces max|x|, and writes the codes from the same registers.
// ---------------------------------------------------------------------------
constexpr int kRegWarps = 4;  // warps (rows) per CTA

template <int MODE, int NV>
__global__ void __launch_bounds__(kRegWarps * 32) act_quant_reg_kernel(const __nv_bfloat16* __restrict__ x,
                                                                        int64_t ldx, uint8_t* __restrict__ q,
                                                                        float* __restrict__ scale_out, int64_t M,
                                                                        int64_t K) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kRegWarps + (threadIdx.x >> 5);
  if (row >= M) return;
  const uint4* src = reinterpret_cast<const uint4*>(x + row * ldx);
  uint8_t* qr = q + row * K;
  const int nvec = static_cast<int>(K / 8);
  uint4 raw[NV];
#pragma unroll
  for (int u = 0; u < NV; ++u)
    raw[u] = lane + 32 * u < nvec ? __ldg(src + lane + 32 * u) : make_uint4(0, 0, 0, 0);
  uint32_t m0 = 0, m1 = 0;
#pragma unroll
  for (int u = 0; u < NV; ++u) {
    m0 = umax2(m0, raw[u].x & 0x7FFF7FFFu);
    m1 = umax2(m1, raw[u].y & 0x7FFF7FFFu);
    m0 = umax2(m0, raw[u].z & 0x7FFF7FFFu);
    m1 = umax2(m1, raw[u].w & 0x7FFF7FFFu);
  }
  const uint32_t m = umax2(m0, m1);
  const float scale = row_scale(__uint_as_float(max(m & 0xFFFFu, m >> 16) << 16), MODE);
  const float rcp = __frcp_rn(scale);
  if (lane == 0) scale_out[row] = scale;
#pragma unroll
  for (int u = 0; u < NV; ++u)
    if (lane + 32 * u < nvec)
      *reinterpret_cast<uint2*>(qr + (int64_t)(lane + 32 * u) * 8) = quant8_bf16<MODE>(raw[u], scale, rcp);
}

// ---------------------------------------------------------------------------
// bf16 rows, one CTA of NT threads per row, NV 16-byte vectors per thread
// (K <= NT * 8 * NV): few registers per thread, so many rows are in flight per
// SM and one row's loads overlap other rows' arithmetic. max|x| is reduced
// within each warp (packed u16 max, shuffles) and across the CTA's warps
// through shared memory; every thread then forms the same scale.
// ---------------------------------------------------------------------------
template <int MODE, int NT, int NV>
__global__ void __launch_bounds__(NT) act_quant_cta_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                                           uint8_t* __restrict__ q, float* __restrict__ scale_out,
                                                           int64_t K) {
  constexpr int NW = NT / 32;
  __shared__ uint32_t wmax[NW];
  const int tid = threadIdx.x, lane = tid & 31;
  const int64_t row = blockIdx.x;
  const uint4* src = reinterpret_cast<const uint4*>(x + row * ldx);
  uint8_t* qr = q + row * K;
  const int nvec = static_cast<int>(K / 8);
  uint4 raw[NV];
#pragma unroll
  for (int u = 0; u < NV; ++u)
    raw[u] = tid + NT * u < nvec ? __ldg(src + tid + NT * u) : make_uint4(0, 0, 0, 0);
  uint32_t m0 = 0, m1 = 0;
#pragma unroll
  for (int u = 0; u < NV; ++u) {
    m0 = umax2(m0, raw[u].x & 0x7FFF7FFFu);
    m1 = umax2(m1, raw[u].y & 0x7FFF7FFFu);
    m0 = umax2(m0, raw[u].z & 0x7FFF7FFFu);
    m1 = umax2(m1, raw[u].w & 0x7FFF7FFFu);
  }
  uint32_t m = umax2(m0, m1);
  m = max(m & 0xFFFFu, m >> 16);  // the largest |x| bit pattern (non-negative bf16 order as integers)
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) wmax[tid >> 5] = m;
  __syncthreads();
  m = wmax[0];
#pragma unroll
  for (int w = 1; w < NW; ++w) m = max(m, wmax[w]);
  const float amax = fmaxf(__uint_as_float(m << 16), 1e-12f);
  const float scale = __fdiv_rn(amax, MODE == D3B_MODE_FP8 ? 448.f : 127.f);
  const float rcp = __frcp_rn(scale);
  if (tid == 0) scale_out[row] = scale;
#pragma unroll
  for (int u = 0; u < NV; ++u)
    if (tid + NT * u < nvec)
      *reinterpret_cast<uint2*>(qr + (int64_t)(tid + NT * u) * 8) = quant8_bf16<MODE>(raw[u], scale, rcp);
}

template <int NT, int NV>
void launch_cta(const __nv_bfloat16* x, int64_t ldx, uint8_t* q, float* scale, int64_t M, int64_t K, int mode,
                cudaStream_t stream) {
  if (mode == D3B_MODE_FP8) act_quant_cta_kernel<D3B_MODE_FP8, NT, NV><<<(unsigned)M, NT, 0, stream>>>(x, ldx, q, scale, K);
  else act_quant_cta_kernel<D3B_MODE_INT8, NT, NV><<<(unsigned)M, NT, 0, stream>>>(x, ldx, q, scale, K);
}

template <int NV>
void launch_reg(const __nv_bfloat16* x, int64_t ldx, uint8_t* q, float* scale, int64_t M, int64_t K, int mode,
                cudaStream_t stream) {
  const dim3 grid((unsigned)((M + kRegWarps - 1) / kRegWarps)), block(kRegWarps * 32);
  if (mode == D3B_MODE_FP8) act_quant_reg_kernel<D3B_MODE_FP8, NV><<<grid, block, 0, stream>>>(x, ldx, q, scale, M, K);
  else act_quant_reg_kernel<D3B_MODE_INT8, NV><<<grid, block, 0, stream>>>(x, ldx, q, scale, M, K);
}

template <typename T>
int launch_typed(const void* x, int64_t ldx, void* q, float* scale, int64_t M, int64_t K, int mode,
                 cudaStream_t stream) {
  const int64_t elem = sizeof(T);
  const bool vec = (reinterpret_cast<uintptr_t>(x) % 16 == 0) && ((ldx * elem) % 16 == 0) &&
                   (reinterpret_cast<uintptr_t>(q) % 16 == 0) && (K % 8 == 0);
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    if (vec && K > 1024 && K <= 256 * 8 * 9 && M <= 0x7FFFFFFF) {
      const auto* xb = static_cast<const __nv_bfloat16*>(x);
      auto* qb = static_cast<uint8_t*>(q);
      const int64_t nv = K / 8;
      if (nv <= 128 * 4) launch_cta<128, 4>(xb, ldx, qb, scale, M, K, mode, stream);
      else if (nv <= 128 * 6) launch_cta<128, 6>(xb, ldx, qb, scale, M, K, mode, stream);
      else if (nv <= 128 * 8) launch_cta<128, 8>(xb, ldx, qb, scale, M, K, mode, stream);
      else launch_cta<256, 9>(xb, ldx, qb, scale, M, K, mode, stream);
      return d3b_host::check_launch();
    }
    if (vec && K <= 32 * 8 * 24 && (M + kRegWarps - 1) / kRegWarps <= 0x7FFFFFFF) {
      const auto* xb = static_cast<const __nv_bfloat16*>(x);
      auto* qb = static_cast<uint8_t*>(q);
      if (K <= 32 * 8 * 16) launch_reg<16>(xb, ldx, qb, scale, M, K, mode, stream);
      else if (K <= 32 * 8 * 20) launch_reg<20>(xb, ldx, qb, scale, M, K, mode, stream);
      else launch_reg<24>(xb, ldx, qb, scale, M, K, mode, stream);
      return d3b_host::check_launch();
    }
  }
  const int64_t blocks = (M + kWarpsPerCta - 1) / kWarpsPerCta;
  if (blocks > 0x7FFFFFFF) return D3B_EINVAL;
  const dim3 grid((unsigned)blocks), block(kWarpsPerCta * 32);
  const T* xt = static_cast<const T*>(x);
  uint8_t* qt = static_cast<uint8_t*>(q);
  if (mode == D3B_MODE_FP8) {
    if (vec) act_quant_kernel<T, D3B_MODE_FP8, true><<<grid, block, 0, stream>>>(xt, ldx, qt, scale, M, K);
    else act_quant_kernel<T, D3B_MODE_FP8, false><<<grid, block, 0, stream>>>(xt, ldx, qt, scale, M, K);
  } else {
    if (vec) act_quant_kernel<T, D3B_MODE_INT8, true><<<grid, block, 0, stream>>>(xt, ldx, qt, scale, M, K);
    else act_quant_kernel<T, D3B_MODE_INT8, false><<<grid, block, 0, stream>>>(xt, ldx, qt, scale, M, K);
  }
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
