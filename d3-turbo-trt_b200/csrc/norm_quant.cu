// Producers of the W8A8 linears' inputs, fused with the per-row activation
// quantisation (d3trt/model/quant.py:92-100), so the normalised or gated rows
// never go through HBM in bf16:
//
// * add + zero-centred RMSNorm + quant (reference/d3_kernels.py:97-170, the
//   bf16-exact restatement of Qwen3_5RMSNorm; inputs of q/k/v_proj and of the
//   MLP's gate/up projection):
//     hidden = bf16(residual + delta)                 (or residual when no delta)
//     rstd   = rsqrt(mean(hidden^2) + eps)            mean over an fp64 sum,
//                                                      rsqrt correctly rounded
//     normed = bf16((hidden * rstd) * (1 + w))        fp32, no contraction
//     (q, scale) = quantize_rows(normed)
// * sigmoid gate + quant (reference/d3_kernels.py:467-525, core.py:297; input
//   of o_proj):
//     gated  = bf16(attn * bf16(1 / (1 + exp(-gate))))  fp32 arithmetic
//     (q, scale) = quantize_rows(gated)
//
// Rows of 1025 to 6144 elements (every width of the model) run one CTA of 128
// threads per row, narrower ones one warp per row; either way the row stays in
// registers between the reduction and the quantisation, so HBM sees the inputs
// once and the codes (plus, when asked for, hidden / normed / gated in bf16)
// once.
#include <type_traits>

#include "common.cuh"
#include "quant_codes.cuh"

namespace {

using namespace d3b_quant;

constexpr int kWarps = 4;        // rows per CTA
constexpr int kModeNone = D3B_MODE_NONE;  // no quantisation: bf16 rows only

__device__ __forceinline__ float lo_bf16(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float hi_bf16(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
__device__ __forceinline__ uint32_t bf16x2_rn(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

// max |x| of a register row of packed bf16 words, and the row's scale / codes
template <int MODE, int NV>
__device__ __forceinline__ void quantise_row(const uint4 (&x)[NV], int lane, int nvec, uint8_t* qr, float* scale_out,
                                             int64_t row) {
  uint32_t m0 = 0, m1 = 0;
#pragma unroll
  for (int u = 0; u < NV; ++u) {
    m0 = umax2(m0, x[u].x & 0x7FFF7FFFu);
    m1 = umax2(m1, x[u].y & 0x7FFF7FFFu);
    m0 = umax2(m0, x[u].z & 0x7FFF7FFFu);
    m1 = umax2(m1, x[u].w & 0x7FFF7FFFu);
  }
  const uint32_t m = umax2(m0, m1);
  const float scale = row_scale(__uint_as_float(max(m & 0xFFFFu, m >> 16) << 16), MODE);
  const float rcp = __frcp_rn(scale);
  if (lane == 0) scale_out[row] = scale;
#pragma unroll
  for (int u = 0; u < NV; ++u)
    if (lane + 32 * u < nvec)
      *reinterpret_cast<uint2*>(qr + (int64_t)(lane + 32 * u) * 8) = quant8_bf16<MODE>(x[u], scale, rcp);
}

// ---------------------------------------------------------------------------
// add + RMSNorm (+ quant)
// ---------------------------------------------------------------------------
template <int MODE, int NV, bool HAS_DELTA>
__global__ void __launch_bounds__(kWarps * 32) add_rmsnorm_quant_kernel(
    const __nv_bfloat16* __restrict__ residual, int64_t ld_res, const __nv_bfloat16* __restrict__ delta,
    int64_t ld_delta, const float* __restrict__ w1, float eps, const int32_t* __restrict__ rowmask,
    __nv_bfloat16* __restrict__ hidden_out, int64_t ld_hidden, __nv_bfloat16* __restrict__ normed_out,
    int64_t ld_normed, uint8_t* __restrict__ q, float* __restrict__ scale_out, int64_t M, int64_t K) {
  // 1 + w for the whole row in shared memory, read by every row of the CTA
  __shared__ __align__(16) float w_s[32 * 8 * NV];
  for (int i = threadIdx.x; i < K / 4; i += kWarps * 32)
    reinterpret_cast<float4*>(w_s)[i] = __ldg(reinterpret_cast<const float4*>(w1) + i);
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (row >= M) return;
  const int nvec = static_cast<int>(K / 8);
  const uint4* rsrc = reinterpret_cast<const uint4*>(residual + row * ld_res);
  uint4 x[NV];
#pragma unroll
  for (int u = 0; u < NV; ++u) x[u] = lane + 32 * u < nvec ? __ldg(rsrc + lane + 32 * u) : make_uint4(0, 0, 0, 0);
  if constexpr (HAS_DELTA) {
    // delta four vectors at a time, so only one chunk is live beside the row
    const uint4* dsrc = reinterpret_cast<const uint4*>(delta + row * ld_delta);
#pragma unroll
    for (int u0 = 0; u0 < NV; u0 += 4) {
      uint4 dv[4];
#pragma unroll
      for (int c = 0; c < 4; ++c)
        dv[c] = u0 + c < NV && lane + 32 * (u0 + c) < nvec ? __ldg(dsrc + lane + 32 * (u0 + c)) : make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        if (u0 + c >= NV) break;
        uint32_t* a = reinterpret_cast<uint32_t*>(&x[u0 + c]);
        const uint32_t* b = reinterpret_cast<const uint32_t*>(&dv[c]);
#pragma unroll
        for (int i = 0; i < 4; ++i)
          a[i] = bf16x2_rn(__fadd_rn(lo_bf16(a[i]), lo_bf16(b[i])), __fadd_rn(hi_bf16(a[i]), hi_bf16(b[i])));
      }
    }
    uint4* hdst = reinterpret_cast<uint4*>(hidden_out + row * ld_hidden);
#pragma unroll
    for (int u = 0; u < NV; ++u)
      if (lane + 32 * u < nvec) hdst[lane + 32 * u] = x[u];
  }
  // sum of squares in fp64 (each bf16 square is exact there), rounded once to fp32 after the division
  double ss = 0.0;
#pragma unroll
  for (int u = 0; u < NV; ++u) {
    const uint32_t* a = reinterpret_cast<const uint32_t*>(&x[u]);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      // unpacked here by an opaque instruction: otherwise the compiler keeps all
      // 8 * NV fp32 values live until the normalisation below and spills
      uint32_t lw, hw;
      asm volatile("shl.b32 %0, %2, 16;\n\tand.b32 %1, %2, 0xFFFF0000;" : "=r"(lw), "=r"(hw) : "r"(a[i]));
      const double l = __uint_as_float(lw), h = __uint_as_float(hw);
      ss = fma(l, l, ss);
      ss = fma(h, h, ss);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float var = __double2float_rn(ss / static_cast<double>(K));
  const float rstd = __double2float_rn(1.0 / sqrt(static_cast<double>(__fadd_rn(var, eps))));
  const bool keep = rowmask == nullptr || rowmask[row] != 0;
  // normed = bf16((hidden * rstd) * (1 + w)), written over the row in registers
#pragma unroll
  for (int u = 0; u < NV; ++u) {
    const int e = (lane + 32 * u) * 8;
    if (lane + 32 * u < nvec) {
      const float4 wa = *reinterpret_cast<const float4*>(w_s + e);
      const float4 wb = *reinterpret_cast<const float4*>(w_s + e + 4);
      const float w[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
      uint32_t* a = reinterpret_cast<uint32_t*>(&x[u]);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float n0 = __fmul_rn(__fmul_rn(lo_bf16(a[i]), rstd), w[2 * i]);
        const float n1 = __fmul_rn(__fmul_rn(hi_bf16(a[i]), rstd), w[2 * i + 1]);
        a[i] = bf16x2_rn(n0, n1) & (keep ? 0xFFFFFFFFu : 0x80008000u);  // masked: y * 0, sign kept
      }
    }
  }
  if (normed_out != nullptr) {
    uint4* ndst = reinterpret_cast<uint4*>(normed_out + row * ld_normed);
#pragma unroll
    for (int u = 0; u < NV; ++u)
      if (lane + 32 * u < nvec) ndst[lane + 32 * u] = x[u];
  }
  if constexpr (MODE != kModeNone) quantise_row<MODE, NV>(x, lane, nvec, q + row * K, scale_out, row);
}

// ---------------------------------------------------------------------------
// sigmoid gate (+ quant)
// ---------------------------------------------------------------------------
template <int MODE, int NV>
__global__ void __launch_bounds__(kWarps * 32) sigmoid_gate_quant_kernel(
    const __nv_bfloat16* __restrict__ attn, int64_t sab, int64_t sat, int64_t sah,
    const __nv_bfloat16* __restrict__ gate, int64_t sgb, int64_t sgt, int64_t sgh, int T, int D, int64_t rows,
    int64_t K, __nv_bfloat16* __restrict__ gated_out, uint8_t* __restrict__ q, float* __restrict__ scale_out) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int64_t b = row / T, t = row % T;
  const int nvec = static_cast<int>(K / 8);
  const __nv_bfloat16* arow = attn + b * sab + t * sat;
  const __nv_bfloat16* grow = gate + b * sgb + t * sgt;
  uint4 x[NV];
#pragma unroll
  for (int u = 0; u < NV; ++u) {
    const int e = (lane + 32 * u) * 8;
    x[u] = lane + 32 * u < nvec ? __ldg(reinterpret_cast<const uint4*>(arow + (e / D) * sah + e % D))
                                : make_uint4(0, 0, 0, 0);
  }
  // the gate four vectors at a time, so only one chunk is live beside the row
#pragma unroll
  for (int u0 = 0; u0 < NV; u0 += 4) {
    uint4 g[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int e = (lane + 32 * (u0 + c)) * 8;
      g[c] = u0 + c < NV && lane + 32 * (u0 + c) < nvec
                 ? __ldg(reinterpret_cast<const uint4*>(grow + (e / D) * sgh + e % D))
                 : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      if (u0 + c >= NV) break;
      uint32_t* a = reinterpret_cast<uint32_t*>(&x[u0 + c]);
      const uint32_t* gw = reinterpret_cast<const uint32_t*>(&g[c]);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        // sigmoid in fp32 (expf, IEEE division), rounded to bf16, then the bf16 product
        const float s0 = __bfloat162float(__float2bfloat16_rn(1.0f / (1.0f + expf(-lo_bf16(gw[i])))));
        const float s1 = __bfloat162float(__float2bfloat16_rn(1.0f / (1.0f + expf(-hi_bf16(gw[i])))));
        a[i] = bf16x2_rn(__fmul_rn(lo_bf16(a[i]), s0), __fmul_rn(hi_bf16(a[i]), s1));
      }
    }
  }
  if (gated_out != nullptr) {
    uint4* dst = reinterpret_cast<uint4*>(gated_out + row * K);
#pragma unroll
    for (int u = 0; u < NV; ++u)
      if (lane + 32 * u < nvec) dst[lane + 32 * u] = x[u];
  }
  if constexpr (MODE != kModeNone) quantise_row<MODE, NV>(x, lane, nvec, q + row * K, scale_out, row);
}

// ---------------------------------------------------------------------------
// The same two producers with one CTA of NT threads per row (rows of 1025 to
// NT * 8 * NV elements): each thread holds NV 16-byte vectors of the row
// (vector tid + NT * u), so registers stay low and many rows are in flight per
// SM (one row's loads overlap other rows' arithmetic; a warp per row kept the
// phases apart). The row reductions (fp64 sum of squares, max |x|) finish
// through shared memory in a fixed order; 1 + w is read per thread from L2.
// ---------------------------------------------------------------------------
template <int NT>
struct CtaRed {
  double ss[NT / 32];
  uint32_t mx[NT / 32];
};

// the row's scale and codes from the CTA's register rows (every thread forms the same scale)
template <int MODE, int NT, int NV>
__device__ __forceinline__ void quantise_row_cta(const uint4 (&x)[NV], int tid, int nvec, uint8_t* qr,
                                                 float* scale_out, int64_t row, CtaRed<NT>& red) {
  uint32_t m0 = 0, m1 = 0;
#pragma unroll
  for (int u = 0; u < NV; ++u) {
    m0 = umax2(m0, x[u].x & 0x7FFF7FFFu);
    m1 = umax2(m1, x[u].y & 0x7FFF7FFFu);
    m0 = umax2(m0, x[u].z & 0x7FFF7FFFu);
    m1 = umax2(m1, x[u].w & 0x7FFF7FFFu);
  }
  uint32_t m = umax2(m0, m1);
  m = max(m & 0xFFFFu, m >> 16);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((tid & 31) == 0) red.mx[tid >> 5] = m;
  __syncthreads();
  m = red.mx[0];
#pragma unroll
  for (int w = 1; w < NT / 32; ++w) m = max(m, red.mx[w]);
  const float amax = fmaxf(__uint_as_float(m << 16), 1e-12f);
  const float scale = __fdiv_rn(amax, MODE == D3B_MODE_FP8 ? 448.f : 127.f);
  const float rcp = __frcp_rn(scale);
  if (tid == 0) scale_out[row] = scale;
#pragma unroll
  for (int u = 0; u < NV; ++u)
    if (tid + NT * u < nvec)
      *reinterpret_cast<uint2*>(qr + (int64_t)(tid + NT * u) * 8) = quant8_bf16<MODE>(x[u], scale, rcp);
}

template <int MODE, int NT, int NV, bool HAS_DELTA>
__global__ void __launch_bounds__(NT) add_rmsnorm_quant_cta_kernel(
    const __nv_bfloat16* __restrict__ residual, int64_t ld_res, const __nv_bfloat16* __restrict__ delta,
    int64_t ld_delta, const float* __restrict__ w1, float eps, const int32_t* __restrict__ rowmask,
    __nv_bfloat16* __restrict__ hidden_out, int64_t ld_hidden, __nv_bfloat16* __restrict__ normed_out,
    int64_t ld_normed, uint8_t* __restrict__ q, float* __restrict__ scale_out, int64_t K) {
  __shared__ CtaRed<NT> red;
  const int tid = threadIdx.x;
  const int64_t row = blockIdx.x;
  const int nvec = static_cast<int>(K / 8);
  const uint4* rsrc = reinterpret_cast<const uint4*>(residual + row * ld_res);
  uint4 x[NV];
#pragma unroll
  for (int u = 0; u < NV; ++u) x[u] = tid + NT * u < nvec ? __ldg(rsrc + tid + NT * u) : make_uint4(0, 0, 0, 0);
  if constexpr (HAS_DELTA) {
    const uint4* dsrc = reinterpret_cast<const uint4*>(delta + row * ld_delta);
    uint4 dv[NV];
#pragma unroll
    for (int u = 0; u < NV; ++u) dv[u] = tid + NT * u < nvec ? __ldg(dsrc + tid + NT * u) : make_uint4(0, 0, 0, 0);
    uint4* hdst = reinterpret_cast<uint4*>(hidden_out + row * ld_hidden);
#pragma unroll
    for (int u = 0; u < NV; ++u) {
      uint32_t* a = reinterpret_cast<uint32_t*>(&x[u]);
      const uint32_t* b = reinterpret_cast<const uint32_t*>(&dv[u]);
#pragma unroll
      for (int i = 0; i < 4; ++i)
        a[i] = bf16x2_rn(__fadd_rn(lo_bf16(a[i]), lo_bf16(b[i])), __fadd_rn(hi_bf16(a[i]), hi_bf16(b[i])));
      if (tid + NT * u < nvec) hdst[tid + NT * u] = x[u];
    }
  }
  // sum of squares in fp64 (each bf16 square is exact there), rounded once to fp32 after the division
  double ss = 0.0;
#pragma unroll
  for (int u = 0; u < NV; ++u) {
    const uint32_t* a = reinterpret_cast<const uint32_t*>(&x[u]);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const double l = lo_bf16(a[i]), h = hi_bf16(a[i]);
      ss = fma(l, l, ss);
      ss = fma(h, h, ss);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((tid & 31) == 0) red.ss[tid >> 5] = ss;
  __syncthreads();
  ss = red.ss[0];
#pragma unroll
  for (int w = 1; w < NT / 32; ++w) ss += red.ss[w];
  const float var = __double2float_rn(ss / static_cast<double>(K));
  const float rstd = __double2float_rn(1.0 / sqrt(static_cast<double>(__fadd_rn(var, eps))));
  const bool keep = rowmask == nullptr || rowmask[row] != 0;
  // normed = bf16((hidden * rstd) * (1 + w)), written over the row in registers
#pragma unroll
  for (int u = 0; u < NV; ++u) {
    if (tid + NT * u < nvec) {
      const float4* wp = reinterpret_cast<const float4*>(w1 + (int64_t)(tid + NT * u) * 8);
      const float4 wa = __ldg(wp), wb = __ldg(wp + 1);
      const float w[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
      uint32_t* a = reinterpret_cast<uint32_t*>(&x[u]);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float n0 = __fmul_rn(__fmul_rn(lo_bf16(a[i]), rstd), w[2 * i]);
        const float n1 = __fmul_rn(__fmul_rn(hi_bf16(a[i]), rstd), w[2 * i + 1]);
        a[i] = bf16x2_rn(n0, n1) & (keep ? 0xFFFFFFFFu : 0x80008000u);  // masked: y * 0, sign kept
      }
    }
  }
  if (normed_out != nullptr) {
    uint4* ndst = reinterpret_cast<uint4*>(normed_out + row * ld_normed);
#pragma unroll
    for (int u = 0; u < NV; ++u)
      if (tid + NT * u < nvec) ndst[tid + NT * u] = x[u];
  }
  if constexpr (MODE != kModeNone) quantise_row_cta<MODE, NT, NV>(x, tid, nvec, q + row * K, scale_out, row, red);
}

template <int MODE, int NT, int NV>
__global__ void __launch_bounds__(NT) sigmoid_gate_quant_cta_kernel(
    const __nv_bfloat16* __restrict__ attn, int64_t sab, int64_t sat, int64_t sah,
    const __nv_bfloat16* __restrict__ gate, int64_t sgb, int64_t sgt, int64_t sgh, int T, int D, int64_t K,
    __nv_bfloat16* __restrict__ gated_out, uint8_t* __restrict__ q, float* __restrict__ scale_out) {
  __shared__ CtaRed<NT> red;
  const int tid = threadIdx.x;
  const int64_t row = blockIdx.x;
  const int64_t b = row / T, t = row % T;
  const int nvec = static_cast<int>(K / 8);
  const __nv_bfloat16* arow = attn + b * sab + t * sat;
  const __nv_bfloat16* grow = gate + b * sgb + t * sgt;
  uint4 x[NV], g[NV];
#pragma unroll
  for (int u = 0; u < NV; ++u) {
    const int e = (tid + NT * u) * 8;
    const bool in = tid + NT * u < nvec;
    x[u] = in ? __ldg(reinterpret_cast<const uint4*>(arow + (e / D) * sah + e % D)) : make_uint4(0, 0, 0, 0);
    g[u] = in ? __ldg(reinterpret_cast<const uint4*>(grow + (e / D) * sgh + e % D)) : make_uint4(0, 0, 0, 0);
  }
#pragma unroll
  for (int u = 0; u < NV; ++u) {
    uint32_t* a = reinterpret_cast<uint32_t*>(&x[u]);
    const uint32_t* gw = reinterpret_cast<const uint32_t*>(&g[u]);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      // sigmoid in fp32 (expf, IEEE division), rounded to bf16, then the bf16 product
      const float s0 = __bfloat162float(__float2bfloat16_rn(1.0f / (1.0f + expf(-lo_bf16(gw[i])))));
      const float s1 = __bfloat162float(__float2bfloat16_rn(1.0f / (1.0f + expf(-hi_bf16(gw[i])))));
      a[i] = bf16x2_rn(__fmul_rn(lo_bf16(a[i]), s0), __fmul_rn(hi_bf16(a[i]), s1));
    }
  }
  if (gated_out != nullptr) {
    uint4* dst = reinterpret_cast<uint4*>(gated_out + row * K);
#pragma unroll
    for (int u = 0; u < NV; ++u)
      if (tid + NT * u < nvec) dst[tid + NT * u] = x[u];
  }
  if constexpr (MODE != kModeNone) quantise_row_cta<MODE, NT, NV>(x, tid, nvec, q + row * K, scale_out, row, red);
}

constexpr int kCtaThreads = 128;  // rows of 1025 .. 6144 elements: at most six vectors per thread

template <int NV>
void launch_norm_cta(int mode, bool has_delta, const void* residual, int64_t ld_res, const void* delta,
                     int64_t ld_delta, const float* w1, float eps, const int32_t* rowmask, void* hidden_out,
                     int64_t ld_hidden, void* normed_out, int64_t ld_normed, void* q, float* scale, int64_t M,
                     int64_t K, cudaStream_t s) {
  constexpr int NT = kCtaThreads;
  auto* r = static_cast<const __nv_bfloat16*>(residual);
  auto* d = static_cast<const __nv_bfloat16*>(delta);
  auto* h = static_cast<__nv_bfloat16*>(hidden_out);
  auto* n = static_cast<__nv_bfloat16*>(normed_out);
  auto* qq = static_cast<uint8_t*>(q);
  auto go = [&](auto kernel) {
    kernel<<<(unsigned)M, NT, 0, s>>>(r, ld_res, d, ld_delta, w1, eps, rowmask, h, ld_hidden, n, ld_normed, qq, scale,
                                      K);
  };
  if (mode == D3B_MODE_FP8) {
    if (has_delta) go(add_rmsnorm_quant_cta_kernel<D3B_MODE_FP8, NT, NV, true>);
    else go(add_rmsnorm_quant_cta_kernel<D3B_MODE_FP8, NT, NV, false>);
  } else if (mode == D3B_MODE_INT8) {
    if (has_delta) go(add_rmsnorm_quant_cta_kernel<D3B_MODE_INT8, NT, NV, true>);
    else go(add_rmsnorm_quant_cta_kernel<D3B_MODE_INT8, NT, NV, false>);
  } else {
    if (has_delta) go(add_rmsnorm_quant_cta_kernel<kModeNone, NT, NV, true>);
    else go(add_rmsnorm_quant_cta_kernel<kModeNone, NT, NV, false>);
  }
}

template <int NV>
void launch_gate_cta(int mode, const __nv_bfloat16* attn, const int64_t* sa, const __nv_bfloat16* gate,
                     const int64_t* sg, int T, int D, int64_t rows, int64_t K, void* gated_out, void* q, float* scale,
                     cudaStream_t s) {
  constexpr int NT = kCtaThreads;
  auto* go = static_cast<__nv_bfloat16*>(gated_out);
  auto* qq = static_cast<uint8_t*>(q);
  auto run = [&](auto kernel) {
    kernel<<<(unsigned)rows, NT, 0, s>>>(attn, sa[0], sa[1], sa[2], gate, sg[0], sg[1], sg[2], T, D, K, go, qq, scale);
  };
  if (mode == D3B_MODE_FP8) run(sigmoid_gate_quant_cta_kernel<D3B_MODE_FP8, NT, NV>);
  else if (mode == D3B_MODE_INT8) run(sigmoid_gate_quant_cta_kernel<D3B_MODE_INT8, NT, NV>);
  else run(sigmoid_gate_quant_cta_kernel<kModeNone, NT, NV>);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

template <int MODE, int NV>
void launch_norm(bool has_delta, const void* residual, int64_t ld_res, const void* delta, int64_t ld_delta,
                 const float* w1, float eps, const int32_t* rowmask, void* hidden_out, int64_t ld_hidden,
                 void* normed_out, int64_t ld_normed, void* q, float* scale, int64_t M, int64_t K, cudaStream_t s) {
  const dim3 grid((unsigned)((M + kWarps - 1) / kWarps)), block(kWarps * 32);
  auto* r = static_cast<const __nv_bfloat16*>(residual);
  auto* d = static_cast<const __nv_bfloat16*>(delta);
  auto* h = static_cast<__nv_bfloat16*>(hidden_out);
  auto* n = static_cast<__nv_bfloat16*>(normed_out);
  auto* qq = static_cast<uint8_t*>(q);
  if (has_delta)
    add_rmsnorm_quant_kernel<MODE, NV, true><<<grid, block, 0, s>>>(r, ld_res, d, ld_delta, w1, eps, rowmask, h,
                                                                   ld_hidden, n, ld_normed, qq, scale, M, K);
  else
    add_rmsnorm_quant_kernel<MODE, NV, false><<<grid, block, 0, s>>>(r, ld_res, d, ld_delta, w1, eps, rowmask, h,
                                                                    ld_hidden, n, ld_normed, qq, scale, M, K);
}

template <int NV>
void launch_norm_mode(int mode, bool has_delta, const void* residual, int64_t ld_res, const void* delta,
                      int64_t ld_delta, const float* w1, float eps, const int32_t* rowmask, void* hidden_out,
                      int64_t ld_hidden, void* normed_out, int64_t ld_normed, void* q, float* scale, int64_t M,
                      int64_t K, cudaStream_t s) {
  if (mode == D3B_MODE_FP8)
    launch_norm<D3B_MODE_FP8, NV>(has_delta, residual, ld_res, delta, ld_delta, w1, eps, rowmask, hidden_out,
                                  ld_hidden, normed_out, ld_normed, q, scale, M, K, s);
  else if (mode == D3B_MODE_INT8)
    launch_norm<D3B_MODE_INT8, NV>(has_delta, residual, ld_res, delta, ld_delta, w1, eps, rowmask, hidden_out,
                                   ld_hidden, normed_out, ld_normed, q, scale, M, K, s);
  else
    launch_norm<kModeNone, NV>(has_delta, residual, ld_res, delta, ld_delta, w1, eps, rowmask, hidden_out,
                               ld_hidden, normed_out, ld_normed, q, scale, M, K, s);
}

template <int NV>
void launch_gate_mode(int mode, const __nv_bfloat16* attn, const int64_t* sa, const __nv_bfloat16* gate,
                      const int64_t* sg, int T, int D, int64_t rows, int64_t K, void* gated_out, void* q,
                      float* scale, cudaStream_t s) {
  const dim3 grid((unsigned)((rows + kWarps - 1) / kWarps)), block(kWarps * 32);
  auto* go = static_cast<__nv_bfloat16*>(gated_out);
  auto* qq = static_cast<uint8_t*>(q);
  if (mode == D3B_MODE_FP8)
    sigmoid_gate_quant_kernel<D3B_MODE_FP8, NV><<<grid, block, 0, s>>>(attn, sa[0], sa[1], sa[2], gate, sg[0], sg[1],
                                                                         sg[2], T, D, rows, K, go, qq, scale);
  else if (mode == D3B_MODE_INT8)
    sigmoid_gate_quant_kernel<D3B_MODE_INT8, NV><<<grid, block, 0, s>>>(attn, sa[0], sa[1], sa[2], gate, sg[0],
                                                                          sg[1], sg[2], T, D, rows, K, go, qq, scale);
  else
    sigmoid_gate_quant_kernel<kModeNone, NV><<<grid, block, 0, s>>>(attn, sa[0], sa[1], sa[2], gate, sg[0], sg[1],
                                                                      sg[2], T, D, rows, K, go, qq, scale);
}

}  // namespace

extern "C" int d3b_add_rmsnorm_quant(const void* residual, int64_t ld_res, const void* delta, int64_t ld_delta,
                                     const float* weight_plus_one, float eps, const int32_t* rowmask,
                                     void* hidden_out, int64_t ld_hidden, void* normed_out, int64_t ld_normed,
                                     void* q, float* scale, int64_t M, int64_t K, int mode, d3b_stream_t stream) {
  if (M < 0 || K <= 0 || ld_res < K) return D3B_EINVAL;
  if (mode != D3B_MODE_FP8 && mode != D3B_MODE_INT8 && mode != kModeNone) return D3B_EINVAL;
  if (M == 0) return D3B_OK;
  if (!residual || !weight_plus_one) return D3B_EINVAL;
  if (delta && (!hidden_out || ld_delta < K || ld_hidden < K)) return D3B_EINVAL;
  if (normed_out && ld_normed < K) return D3B_EINVAL;
  if (mode != kModeNone && (!q || !scale)) return D3B_EINVAL;
  if (mode == kModeNone && !normed_out) return D3B_EINVAL;
  if (K % 8 || K > 32 * 8 * 24) return D3B_EUNSUPPORTED;  // rows of up to 6144 held in registers
  if (!aligned16(residual) || !aligned16(weight_plus_one) || (ld_res % 8) || (q && !aligned16(q)) ||
      (delta && (!aligned16(delta) || !aligned16(hidden_out) || (ld_delta % 8) || (ld_hidden % 8))) ||
      (normed_out && (!aligned16(normed_out) || (ld_normed % 8))))
    return D3B_EALIGN;
  if ((M + kWarps - 1) / kWarps > 0x7FFFFFFF) return D3B_EINVAL;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const bool has_delta = delta != nullptr;
  if (K > 1024 && M <= 0x7FFFFFFF) {  // a CTA per row
    const int64_t nv = K / 8;
    if (nv <= kCtaThreads * 4)
      launch_norm_cta<4>(mode, has_delta, residual, ld_res, delta, ld_delta, weight_plus_one, eps, rowmask,
                         hidden_out, ld_hidden, normed_out, ld_normed, q, scale, M, K, s);
    else
      launch_norm_cta<6>(mode, has_delta, residual, ld_res, delta, ld_delta, weight_plus_one, eps, rowmask,
                         hidden_out, ld_hidden, normed_out, ld_normed, q, scale, M, K, s);
    return d3b_host::check_launch();
  }
  if (K <= 32 * 8 * 16)
    launch_norm_mode<16>(mode, has_delta, residual, ld_res, delta, ld_delta, weight_plus_one, eps, rowmask,
                         hidden_out, ld_hidden, normed_out, ld_normed, q, scale, M, K, s);
  else if (K <= 32 * 8 * 20)
    launch_norm_mode<20>(mode, has_delta, residual, ld_res, delta, ld_delta, weight_plus_one, eps, rowmask,
                         hidden_out, ld_hidden, normed_out, ld_normed, q, scale, M, K, s);
  else
    launch_norm_mode<24>(mode, has_delta, residual, ld_res, delta, ld_delta, weight_plus_one, eps, rowmask,
                         hidden_out, ld_hidden, normed_out, ld_normed, q, scale, M, K, s);
  return d3b_host::check_launch();
}

extern "C" int d3b_sigmoid_gate_quant(const void* attn, const int64_t* attn_strides, const void* gate,
                                      const int64_t* gate_strides, void* gated_out, void* q, float* scale, int B,
                                      int T, int H, int D, int mode, d3b_stream_t stream) {
  if (B < 0 || T < 0 || H <= 0 || D <= 0) return D3B_EINVAL;
  if (mode != D3B_MODE_FP8 && mode != D3B_MODE_INT8 && mode != kModeNone) return D3B_EINVAL;
  const int64_t rows = (int64_t)B * T, K = (int64_t)H * D;
  if (rows == 0) return D3B_OK;
  if (!attn || !gate || !attn_strides || !gate_strides) return D3B_EINVAL;
  if (mode != kModeNone && (!q || !scale)) return D3B_EINVAL;
  if (mode == kModeNone && !gated_out) return D3B_EINVAL;
  if (D % 8 || K > 32 * 8 * 24) return D3B_EUNSUPPORTED;
  for (int i = 0; i < 3; ++i)
    if (attn_strides[i] % 8 || gate_strides[i] % 8) return D3B_EALIGN;
  if (!aligned16(attn) || !aligned16(gate) || (q && !aligned16(q)) || (gated_out && !aligned16(gated_out)))
    return D3B_EALIGN;
  if ((rows + kWarps - 1) / kWarps > 0x7FFFFFFF) return D3B_EINVAL;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  auto* a = static_cast<const __nv_bfloat16*>(attn);
  auto* g = static_cast<const __nv_bfloat16*>(gate);
  if (K > 1024 && rows <= 0x7FFFFFFF) {  // a CTA per row
    if (K / 8 <= kCtaThreads * 4)
      launch_gate_cta<4>(mode, a, attn_strides, g, gate_strides, T, D, rows, K, gated_out, q, scale, s);
    else
      launch_gate_cta<6>(mode, a, attn_strides, g, gate_strides, T, D, rows, K, gated_out, q, scale, s);
    return d3b_host::check_launch();
  }
  if (K <= 32 * 8 * 16) launch_gate_mode<16>(mode, a, attn_strides, g, gate_strides, T, D, rows, K, gated_out, q, scale, s);
  else if (K <= 32 * 8 * 20)
    launch_gate_mode<20>(mode, a, attn_strides, g, gate_strides, T, D, rows, K, gated_out, q, scale, s);
  else launch_gate_mode<24>(mode, a, attn_strides, g, gate_strides, T, D, rows, K, gated_out, q, scale, s);
  return d3b_host::check_launch();
}
