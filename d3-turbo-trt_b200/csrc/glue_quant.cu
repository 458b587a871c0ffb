// Two producers of W8A8 linear inputs in the d3 layers, fused with the per-row
// activation quantisation of their consumer (d3trt/model/quant.py:92-100), so the
// bf16 rows never go through HBM:
//
// * SiLU(gate) * up -> down_proj (the MLP, transformers Qwen3_5MLP.forward as the
//   reference's stacks run it; trtllm_stack.py:118-120 with gate_up fused):
//     act = bf16(bf16(silu(gate)) * up),  silu(g) = g / (1 + exp(-g)) in fp32
//     (q, scale) = quantize_rows(act)
//   gate_up rows [M, 2I] (gate first, then up), as the fused gate/up GEMM writes
//   them. One CTA (256 threads) per row keeps the row in registers for rows of up
//   to 24576 elements; the row's max|act| goes through shared memory.
// * gated RMSNorm of the GDN output -> out_proj (Qwen3_5RMSNormGated, called at
//   d3trt/model/core.py:400-401):
//     per head of Dv values: xn = x * rsqrt(mean(x^2) + eps) in fp32,
//     y = bf16(w * bf16(xn)),  out = bf16(y * silu(z)) in fp32
//     (q, scale) = quantize_rows(out) over the token's HV * Dv values
//   One warp per token row (up to 6144 values in registers); a head's Dv values
//   sit in Dv/8 consecutive lanes, so its sum of squares is a sub-warp shuffle
//   reduction in a fixed order.
#include "common.cuh"
#include "quant_codes.cuh"

namespace {

using namespace d3b_quant;

__device__ __forceinline__ float lo_bf(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float hi_bf(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
__device__ __forceinline__ uint32_t pack_bf(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}
__device__ __forceinline__ float round_bf(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
__device__ __forceinline__ float silu(float x) { return x / (1.0f + expf(-x)); }

// ---------------------------------------------------------------------------
constexpr int kMlpThreads = 256;

template <int MODE, int NV>
__global__ void __launch_bounds__(kMlpThreads) silu_mul_quant_kernel(const uint16_t* __restrict__ gu, int64_t ld,
                                                                     int64_t I, uint16_t* __restrict__ act_out,
                                                                     uint8_t* __restrict__ q,
                                                                     float* __restrict__ scale_out) {
  __shared__ float part[kMlpThreads / 32];
  const int64_t row = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nvec = (int)(I / 8);
  const uint16_t* g = gu + row * ld;
  const uint16_t* u = g + I;
  uint4 a[NV];
  uint32_t m0 = 0, m1 = 0;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int v = tid + kMlpThreads * k;
    if (v < nvec) {
      const uint4 gv = __ldg(reinterpret_cast<const uint4*>(g) + v);
      const uint4 uv = __ldg(reinterpret_cast<const uint4*>(u) + v);
      const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w}, uw[4] = {uv.x, uv.y, uv.z, uv.w};
      uint32_t r[4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
        r[i] = pack_bf(__fmul_rn(round_bf(silu(lo_bf(gw[i]))), lo_bf(uw[i])),
                       __fmul_rn(round_bf(silu(hi_bf(gw[i]))), hi_bf(uw[i])));
      a[k] = make_uint4(r[0], r[1], r[2], r[3]);
      m0 = umax2(m0, a[k].x & 0x7FFF7FFFu);
      m1 = umax2(m1, a[k].y & 0x7FFF7FFFu);
      m0 = umax2(m0, a[k].z & 0x7FFF7FFFu);
      m1 = umax2(m1, a[k].w & 0x7FFF7FFFu);
    } else {
      a[k] = make_uint4(0, 0, 0, 0);
    }
  }
  const uint32_t m = umax2(m0, m1);
  float amax = __uint_as_float(max(m & 0xFFFFu, m >> 16) << 16);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if (lane == 0) part[warp] = amax;
  __syncthreads();
  amax = part[0];
#pragma unroll
  for (int w = 1; w < kMlpThreads / 32; ++w) amax = fmaxf(amax, part[w]);
  if (act_out != nullptr) {
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int v = tid + kMlpThreads * k;
      if (v < nvec) reinterpret_cast<uint4*>(act_out + row * I)[v] = a[k];
    }
  }
  if constexpr (MODE != D3B_MODE_NONE) {
    const float scale = __fdiv_rn(fmaxf(amax, 1e-12f), MODE == D3B_MODE_FP8 ? 448.f : 127.f);
    const float rcp = __frcp_rn(scale);
    if (tid == 0) scale_out[row] = scale;
    uint8_t* qr = q + row * I;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int v = tid + kMlpThreads * k;
      if (v < nvec) *reinterpret_cast<uint2*>(qr + (int64_t)v * 8) = quant8_bf16<MODE>(a[k], scale, rcp);
    }
  }
}

// ---------------------------------------------------------------------------
constexpr int kNormWarps = 4;

template <int MODE, int NV, int LPH>  // LPH: lanes per head = Dv / 8
__global__ void __launch_bounds__(kNormWarps * 32) gated_rmsnorm_quant_kernel(
    const uint16_t* __restrict__ x, int64_t ldx, const uint16_t* __restrict__ z, int64_t ldz,
    const uint16_t* __restrict__ w, float eps, int64_t M, int64_t K, uint16_t* __restrict__ out,
    uint8_t* __restrict__ q, float* __restrict__ scale_out) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kNormWarps + (threadIdx.x >> 5);
  if (row >= M) return;
  const int nvec = (int)(K / 8);
  const float inv_d = 1.0f / (float)(LPH * 8);
  // this lane's 8 weights: element (lane % LPH) * 8 .. +8 of every head
  float wv[8];
  {
    const uint4 ww = __ldg(reinterpret_cast<const uint4*>(w) + (lane % LPH));
    const uint32_t wa[4] = {ww.x, ww.y, ww.z, ww.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      wv[2 * i] = lo_bf(wa[i]);
      wv[2 * i + 1] = hi_bf(wa[i]);
    }
  }
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * ldx);
  const uint4* zr = reinterpret_cast<const uint4*>(z + row * ldz);
  uint4 a[NV];
  uint32_t m0 = 0, m1 = 0;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int v = lane + 32 * k;
    const bool in = v < nvec;  // uniform per head: heads never straddle the row's end (K % Dv == 0)
    const uint4 xv = in ? __ldg(xr + v) : make_uint4(0, 0, 0, 0);
    const uint4 zv = in ? __ldg(zr + v) : make_uint4(0, 0, 0, 0);
    const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w}, zw[4] = {zv.x, zv.y, zv.z, zv.w};
    float xf[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      xf[2 * i] = lo_bf(xw[i]);
      xf[2 * i + 1] = hi_bf(xw[i]);
    }
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) ss = fmaf(xf[i], xf[i], ss);
#pragma unroll
    for (int o = LPH / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float rstd = rsqrtf(ss * inv_d + eps);
    uint32_t r[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float y0 = round_bf(__fmul_rn(wv[2 * i], round_bf(__fmul_rn(xf[2 * i], rstd))));
      const float y1 = round_bf(__fmul_rn(wv[2 * i + 1], round_bf(__fmul_rn(xf[2 * i + 1], rstd))));
      r[i] = pack_bf(__fmul_rn(y0, silu(lo_bf(zw[i]))), __fmul_rn(y1, silu(hi_bf(zw[i]))));
    }
    a[k] = in ? make_uint4(r[0], r[1], r[2], r[3]) : make_uint4(0, 0, 0, 0);
    m0 = umax2(m0, a[k].x & 0x7FFF7FFFu);
    m1 = umax2(m1, a[k].y & 0x7FFF7FFFu);
    m0 = umax2(m0, a[k].z & 0x7FFF7FFFu);
    m1 = umax2(m1, a[k].w & 0x7FFF7FFFu);
  }
  if (out != nullptr) {
#pragma unroll
    for (int k = 0; k < NV; ++k)
      if (lane + 32 * k < nvec) reinterpret_cast<uint4*>(out + row * K)[lane + 32 * k] = a[k];
  }
  if constexpr (MODE != D3B_MODE_NONE) {
    const uint32_t m = umax2(m0, m1);
    const float scale = row_scale(__uint_as_float(max(m & 0xFFFFu, m >> 16) << 16), MODE);
    const float rcp = __frcp_rn(scale);
    if (lane == 0) scale_out[row] = scale;
    uint8_t* qr = q + row * K;
#pragma unroll
    for (int k = 0; k < NV; ++k)
      if (lane + 32 * k < nvec) *reinterpret_cast<uint2*>(qr + (int64_t)(lane + 32 * k) * 8) = quant8_bf16<MODE>(a[k], scale, rcp);
  }
}

// The same, one CTA of NT threads per token row for rows of 2048 to 6144 values (the
// model's 48 x 128 = 6144): each thread holds NV <= 3 vectors, so many rows are in
// flight per SM (the warp-per-row form above holds 24 vectors per lane and ~12 warps
// per SM). Vector v = t + NT * k of the row sits in thread t, so a head's LPH vectors
// are still LPH consecutive lanes of one warp (NT is a multiple of 32) and its sum of
// squares is the same sub-warp shuffle reduction; the row's max|out| goes through
// shared memory.
template <int MODE, int NT, int NV, int LPH>
__global__ void __launch_bounds__(NT) gated_rmsnorm_quant_cta_kernel(
    const uint16_t* __restrict__ x, int64_t ldx, const uint16_t* __restrict__ z, int64_t ldz,
    const uint16_t* __restrict__ w, float eps, int64_t K, uint16_t* __restrict__ out, uint8_t* __restrict__ q,
    float* __restrict__ scale_out) {
  __shared__ uint32_t wmax[NT / 32];
  const int tid = threadIdx.x, lane = tid & 31;
  const int64_t row = blockIdx.x;
  const int nvec = (int)(K / 8);
  const float inv_d = 1.0f / (float)(LPH * 8);
  float wv[8];
  {
    const uint4 ww = __ldg(reinterpret_cast<const uint4*>(w) + (tid % LPH));
    const uint32_t wa[4] = {ww.x, ww.y, ww.z, ww.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      wv[2 * i] = lo_bf(wa[i]);
      wv[2 * i + 1] = hi_bf(wa[i]);
    }
  }
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * ldx);
  const uint4* zr = reinterpret_cast<const uint4*>(z + row * ldz);
  uint4 xs[NV], zs[NV];
#pragma unroll
  for (int k = 0; k < NV; ++k) {  // every load in flight before any arithmetic
    const int v = tid + NT * k;
    const bool in = v < nvec;
    xs[k] = in ? __ldg(xr + v) : make_uint4(0, 0, 0, 0);
    zs[k] = in ? __ldg(zr + v) : make_uint4(0, 0, 0, 0);
  }
  uint4 a[NV];
  uint32_t m0 = 0, m1 = 0;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const bool in = tid + NT * k < nvec;  // uniform per head: heads never straddle the row's end
    const uint32_t xw[4] = {xs[k].x, xs[k].y, xs[k].z, xs[k].w}, zw[4] = {zs[k].x, zs[k].y, zs[k].z, zs[k].w};
    float xf[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      xf[2 * i] = lo_bf(xw[i]);
      xf[2 * i + 1] = hi_bf(xw[i]);
    }
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) ss = fmaf(xf[i], xf[i], ss);
#pragma unroll
    for (int o = LPH / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float rstd = rsqrtf(ss * inv_d + eps);
    uint32_t r[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float y0 = round_bf(__fmul_rn(wv[2 * i], round_bf(__fmul_rn(xf[2 * i], rstd))));
      const float y1 = round_bf(__fmul_rn(wv[2 * i + 1], round_bf(__fmul_rn(xf[2 * i + 1], rstd))));
      r[i] = pack_bf(__fmul_rn(y0, silu(lo_bf(zw[i]))), __fmul_rn(y1, silu(hi_bf(zw[i]))));
    }
    a[k] = in ? make_uint4(r[0], r[1], r[2], r[3]) : make_uint4(0, 0, 0, 0);
    m0 = umax2(m0, a[k].x & 0x7FFF7FFFu);
    m1 = umax2(m1, a[k].y & 0x7FFF7FFFu);
    m0 = umax2(m0, a[k].z & 0x7FFF7FFFu);
    m1 = umax2(m1, a[k].w & 0x7FFF7FFFu);
  }
  if (out != nullptr) {
#pragma unroll
    for (int k = 0; k < NV; ++k)
      if (tid + NT * k < nvec) reinterpret_cast<uint4*>(out + row * K)[tid + NT * k] = a[k];
  }
  if constexpr (MODE != D3B_MODE_NONE) {
    uint32_t m = umax2(m0, m1);
    m = max(m & 0xFFFFu, m >> 16);  // the largest |out| bit pattern (non-negative bf16 order as integers)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) wmax[tid >> 5] = m;
    __syncthreads();
    m = wmax[0];
#pragma unroll
    for (int i = 1; i < NT / 32; ++i) m = max(m, wmax[i]);
    const float scale = __fdiv_rn(fmaxf(__uint_as_float(m << 16), 1e-12f), MODE == D3B_MODE_FP8 ? 448.f : 127.f);
    const float rcp = __frcp_rn(scale);
    if (tid == 0) scale_out[row] = scale;
    uint8_t* qr = q + row * K;
#pragma unroll
    for (int k = 0; k < NV; ++k)
      if (tid + NT * k < nvec) *reinterpret_cast<uint2*>(qr + (int64_t)(tid + NT * k) * 8) = quant8_bf16<MODE>(a[k], scale, rcp);
  }
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

template <int MODE, int NV>
void mlp_launch(const uint16_t* gu, int64_t ld, int64_t M, int64_t I, uint16_t* act, uint8_t* q, float* sc,
                cudaStream_t s) {
  silu_mul_quant_kernel<MODE, NV><<<(unsigned)M, kMlpThreads, 0, s>>>(gu, ld, I, act, q, sc);
}

template <int NV>
void mlp_mode(int mode, const uint16_t* gu, int64_t ld, int64_t M, int64_t I, uint16_t* act, uint8_t* q, float* sc,
              cudaStream_t s) {
  if (mode == D3B_MODE_FP8) mlp_launch<D3B_MODE_FP8, NV>(gu, ld, M, I, act, q, sc, s);
  else if (mode == D3B_MODE_INT8) mlp_launch<D3B_MODE_INT8, NV>(gu, ld, M, I, act, q, sc, s);
  else mlp_launch<D3B_MODE_NONE, NV>(gu, ld, M, I, act, q, sc, s);
}

template <int NV, int LPH>
void norm_mode(int mode, const uint16_t* x, int64_t ldx, const uint16_t* z, int64_t ldz, const uint16_t* w, float eps,
               int64_t M, int64_t K, uint16_t* out, uint8_t* q, float* sc, cudaStream_t s) {
  const unsigned grid = (unsigned)((M + kNormWarps - 1) / kNormWarps);
  if (mode == D3B_MODE_FP8)
    gated_rmsnorm_quant_kernel<D3B_MODE_FP8, NV, LPH><<<grid, kNormWarps * 32, 0, s>>>(x, ldx, z, ldz, w, eps, M, K, out, q, sc);
  else if (mode == D3B_MODE_INT8)
    gated_rmsnorm_quant_kernel<D3B_MODE_INT8, NV, LPH><<<grid, kNormWarps * 32, 0, s>>>(x, ldx, z, ldz, w, eps, M, K, out, q, sc);
  else
    gated_rmsnorm_quant_kernel<D3B_MODE_NONE, NV, LPH><<<grid, kNormWarps * 32, 0, s>>>(x, ldx, z, ldz, w, eps, M, K, out, q, sc);
}

template <int NV, int LPH>
void norm_cta_mode(int mode, const uint16_t* x, int64_t ldx, const uint16_t* z, int64_t ldz, const uint16_t* w,
                   float eps, int64_t M, int64_t K, uint16_t* out, uint8_t* q, float* sc, cudaStream_t s) {
  constexpr int NT = 256;
  if (mode == D3B_MODE_FP8)
    gated_rmsnorm_quant_cta_kernel<D3B_MODE_FP8, NT, NV, LPH><<<(unsigned)M, NT, 0, s>>>(x, ldx, z, ldz, w, eps, K, out, q, sc);
  else if (mode == D3B_MODE_INT8)
    gated_rmsnorm_quant_cta_kernel<D3B_MODE_INT8, NT, NV, LPH><<<(unsigned)M, NT, 0, s>>>(x, ldx, z, ldz, w, eps, K, out, q, sc);
  else
    gated_rmsnorm_quant_cta_kernel<D3B_MODE_NONE, NT, NV, LPH><<<(unsigned)M, NT, 0, s>>>(x, ldx, z, ldz, w, eps, K, out, q, sc);
}

template <int LPH>
int norm_nv(int mode, const uint16_t* x, int64_t ldx, const uint16_t* z, int64_t ldz, const uint16_t* w, float eps,
            int64_t M, int64_t K, uint16_t* out, uint8_t* q, float* sc, cudaStream_t s) {
  const int64_t nvec = K / 8;
  if (nvec >= 256 && nvec <= 256 * 3 && M <= 0x7FFFFFFF) {  // one CTA per row (rows of 2048 to 6144 values)
    if (nvec <= 256 * 2) norm_cta_mode<2, LPH>(mode, x, ldx, z, ldz, w, eps, M, K, out, q, sc, s);
    else norm_cta_mode<3, LPH>(mode, x, ldx, z, ldz, w, eps, M, K, out, q, sc, s);
    return d3b_host::check_launch();
  }
  const int nv = (int)((K / 8 + 31) / 32);
  if (nv <= 8) norm_mode<8, LPH>(mode, x, ldx, z, ldz, w, eps, M, K, out, q, sc, s);
  else if (nv <= 16) norm_mode<16, LPH>(mode, x, ldx, z, ldz, w, eps, M, K, out, q, sc, s);
  else norm_mode<24, LPH>(mode, x, ldx, z, ldz, w, eps, M, K, out, q, sc, s);
  return d3b_host::check_launch();
}

}  // namespace

// ---------------------------------------------------------------------------
// Gated DeltaNet gates (d3trt/model/core.py:341-342 through the model's module):
//   beta = bf16(1 / (1 + exp(-b)))                      (torch's sigmoid on bf16)
//   g    = neg_exp_a[h] * softplus(float(a) + dt_bias[h]),
//          softplus(x) = x > 20 ? x : log1p(exp(x))      (torch's softplus, fp32)
// with neg_exp_a = -exp(float(A_log)) and dt_bias as fp32 per value head, formed once by the
// caller. One thread per (token row, value head); a and b are row slices of the fused input
// projection (row strides lda, ldb).
constexpr int kGateThreads = 256;

__global__ void __launch_bounds__(kGateThreads) gdn_gates_kernel(const uint16_t* __restrict__ a, int64_t lda,
                                                                 const uint16_t* __restrict__ b, int64_t ldb,
                                                                 const float* __restrict__ neg_exp_a,
                                                                 const float* __restrict__ dt_bias, float* __restrict__ g,
                                                                 uint16_t* __restrict__ beta, int64_t n, int HV) {
  const int64_t i = (int64_t)blockIdx.x * kGateThreads + threadIdx.x;
  if (i >= n) return;
  const int64_t m = i / HV;
  const int h = (int)(i - m * HV);
  const float x = __fadd_rn(__uint_as_float((uint32_t)a[m * lda + h] << 16), dt_bias[h]);
  const float sp = x > 20.0f ? x : log1pf(expf(x));
  g[i] = __fmul_rn(neg_exp_a[h], sp);
  const float bv = __uint_as_float((uint32_t)b[m * ldb + h] << 16);
  const __nv_bfloat16 r = __float2bfloat16_rn(1.0f / (1.0f + expf(-bv)));
  beta[i] = *reinterpret_cast<const uint16_t*>(&r);
}

extern "C" int d3b_silu_mul_quant(const void* gate_up, int64_t ld, void* act_out, void* q, float* scale, int64_t M,
                                  int64_t I, int mode, d3b_stream_t stream) {
  if (M < 0 || I <= 0 || ld < 2 * I) return D3B_EINVAL;
  if (mode != D3B_MODE_FP8 && mode != D3B_MODE_INT8 && mode != D3B_MODE_NONE) return D3B_EINVAL;
  if (M == 0) return D3B_OK;
  if (!gate_up || (mode == D3B_MODE_NONE && !act_out) || (mode != D3B_MODE_NONE && (!q || !scale)))
    return D3B_EINVAL;
  if (I % 8 || I > (int64_t)kMlpThreads * 8 * 12) return D3B_EUNSUPPORTED;
  if (M > 0x7FFFFFFF) return D3B_EINVAL;
  if (!al16(gate_up) || ld % 8 || (act_out && !al16(act_out)) || (q && !al16(q))) return D3B_EALIGN;
  const auto* gu = static_cast<const uint16_t*>(gate_up);
  auto* act = static_cast<uint16_t*>(act_out);
  auto* qq = static_cast<uint8_t*>(q);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int nv = (int)((I / 8 + kMlpThreads - 1) / kMlpThreads);
  if (nv <= 1) mlp_mode<1>(mode, gu, ld, M, I, act, qq, scale, s);
  else if (nv <= 2) mlp_mode<2>(mode, gu, ld, M, I, act, qq, scale, s);
  else if (nv <= 4) mlp_mode<4>(mode, gu, ld, M, I, act, qq, scale, s);
  else if (nv <= 8) mlp_mode<8>(mode, gu, ld, M, I, act, qq, scale, s);
  else mlp_mode<12>(mode, gu, ld, M, I, act, qq, scale, s);
  return d3b_host::check_launch();
}

extern "C" int d3b_gated_rmsnorm_quant(const void* x, int64_t ldx, const void* z, int64_t ldz, const void* weight,
                                       float eps, int head_dim, void* out, void* q, float* scale, int64_t M, int64_t K,
                                       int mode, d3b_stream_t stream) {
  if (M < 0 || K <= 0 || ldx < K || ldz < K) return D3B_EINVAL;
  if (mode != D3B_MODE_FP8 && mode != D3B_MODE_INT8 && mode != D3B_MODE_NONE) return D3B_EINVAL;
  if (M == 0) return D3B_OK;
  if (!x || !z || !weight || (mode == D3B_MODE_NONE && !out) || (mode != D3B_MODE_NONE && (!q || !scale)))
    return D3B_EINVAL;
  if ((head_dim != 64 && head_dim != 128 && head_dim != 256) || K % head_dim || K > 32 * 8 * 24)
    return D3B_EUNSUPPORTED;
  if ((M + kNormWarps - 1) / kNormWarps > 0x7FFFFFFF) return D3B_EINVAL;
  if (!al16(x) || !al16(z) || !al16(weight) || ldx % 8 || ldz % 8 || (out && !al16(out)) || (q && !al16(q)))
    return D3B_EALIGN;
  const auto* xs = static_cast<const uint16_t*>(x);
  const auto* zs = static_cast<const uint16_t*>(z);
  const auto* ws = static_cast<const uint16_t*>(weight);
  auto* os = static_cast<uint16_t*>(out);
  auto* qq = static_cast<uint8_t*>(q);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (head_dim) {
    case 64: return norm_nv<8>(mode, xs, ldx, zs, ldz, ws, eps, M, K, os, qq, scale, s);
    case 128: return norm_nv<16>(mode, xs, ldx, zs, ldz, ws, eps, M, K, os, qq, scale, s);
    default: return norm_nv<32>(mode, xs, ldx, zs, ldz, ws, eps, M, K, os, qq, scale, s);
  }
}

extern "C" int d3b_gdn_gates(const void* a, int64_t lda, const void* b, int64_t ldb, const float* neg_exp_a,
                             const float* dt_bias, float* g, void* beta, int64_t M, int HV, d3b_stream_t stream) {
  if (M < 0 || HV <= 0 || lda < HV || ldb < HV) return D3B_EINVAL;
  if (M == 0) return D3B_OK;
  if (!a || !b || !neg_exp_a || !dt_bias || !g || !beta) return D3B_EINVAL;
  const int64_t n = M * HV;
  const int64_t blocks = (n + kGateThreads - 1) / kGateThreads;
  if (blocks > 0x7FFFFFFF) return D3B_EINVAL;
  gdn_gates_kernel<<<(unsigned)blocks, kGateThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t*>(a), lda, static_cast<const uint16_t*>(b), ldb, neg_exp_a, dt_bias, g,
      static_cast<uint16_t*>(beta), n, HV);
  return d3b_host::check_launch();
}
