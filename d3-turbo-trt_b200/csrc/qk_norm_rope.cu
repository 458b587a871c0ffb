// Per-head RMSNorm of the attention layers' queries and keys followed by their
// partial rotary embedding, in one pass (d3trt/model/core.py:233-237: q_norm and
// k_norm are transformers' Qwen3_5RMSNorm, then apply_rotary_pos_emb over the
// first rd = head_dim * partial_rotary_factor dimensions):
//
//   xf = float(x);  r = rsqrt(sum(xf^2) / D + eps)
//   y  = bf16(float(xf * r) * (1 + float(w)))                 (Qwen3_5RMSNorm, fp32)
//   for i < rd:  rot_i = -y[i + rd/2] (i < rd/2), y[i - rd/2] (rd/2 <= i < rd)
//                out_i = bf16(bf16(y_i * cos_i) + bf16(rot_i * sin_i))   (bf16 tensor ops)
//   for i >= rd: out_i = y_i
//
// x is read where the projection left it ([rows, T, heads, D] with any row,
// token and head strides, D contiguous: the query half of q_proj's output is a
// strided slice) and out is written token-major [rows, T, heads, D] (contiguous),
// which the attention kernels read through a [rows, heads, T, D] view. One head
// of D = 128 values is 16 lanes x 8 values (one 16-byte load and store each); its
// sum of squares is a 16-lane shuffle reduction, and a lane's rotary partner
// (rd/2 elements away) is lane ^ (rd/16).
#include "common.cuh"

namespace {

constexpr int kThreads = 256;  // up to 16 heads per CTA

__device__ __forceinline__ float lo_bf(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float hi_bf(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
__device__ __forceinline__ float round_bf(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
__device__ __forceinline__ uint32_t pack_bf(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

template <int RD>  // rotary dimensions, a multiple of 16 up to 128
__global__ void __launch_bounds__(kThreads) qk_norm_rope_kernel(
    const uint16_t* __restrict__ x, int64_t sx_r, int64_t sx_t, int64_t sx_h, const uint16_t* __restrict__ w,
    const uint16_t* __restrict__ cosv, const uint16_t* __restrict__ sinv, int64_t sc_r, int64_t sc_t,
    uint16_t* __restrict__ out, int T, int heads, float eps) {
  // grid: x = (row, token), y = group of blockDim.x / 16 heads; no per-thread division
  const int lane = threadIdx.x & 31, sub = lane & 15;  // sub: the lane's 8 values within its head
  const int64_t rt = blockIdx.x;
  const int t = (int)(rt % T);
  const int64_t r = rt / T;
  const int hh = (int)blockIdx.y * (int)(blockDim.x >> 4) + (int)(threadIdx.x >> 4);
  const bool live = hh < heads;
  const int h = live ? hh : 0;
  const int64_t it = rt * heads + h;  // output head index (token-major)
  const uint4 xv = live ? __ldg(reinterpret_cast<const uint4*>(x + r * sx_r + (int64_t)t * sx_t + (int64_t)h * sx_h) + sub)
                        : make_uint4(0, 0, 0, 0);
  const uint4 wv = __ldg(reinterpret_cast<const uint4*>(w) + sub);
  const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w}, ww[4] = {wv.x, wv.y, wv.z, wv.w};
  float xf[8], w1[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    xf[2 * i] = lo_bf(xw[i]);
    xf[2 * i + 1] = hi_bf(xw[i]);
    w1[2 * i] = __fadd_rn(1.0f, lo_bf(ww[i]));
    w1[2 * i + 1] = __fadd_rn(1.0f, hi_bf(ww[i]));
  }
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) ss = fmaf(xf[i], xf[i], ss);
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float rs = rsqrtf(__fadd_rn(ss * (1.0f / 128.0f), eps));
  float y[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) y[i] = round_bf(__fmul_rn(__fmul_rn(xf[i], rs), w1[i]));
  // the rotary partner's normalised values (rd/2 elements = rd/16 lanes away)
  const uint32_t yp[4] = {pack_bf(y[0], y[1]), pack_bf(y[2], y[3]), pack_bf(y[4], y[5]), pack_bf(y[6], y[7])};
  uint32_t pp[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) pp[i] = __shfl_xor_sync(0xffffffffu, yp[i], RD / 16);
  uint32_t o[4];
  if (sub < RD / 8) {
    const int64_t coff = r * sc_r + (int64_t)t * sc_t;
    const uint4 cv = __ldg(reinterpret_cast<const uint4*>(cosv + coff) + sub);
    const uint4 sv = __ldg(reinterpret_cast<const uint4*>(sinv + coff) + sub);
    const uint32_t cw[4] = {cv.x, cv.y, cv.z, cv.w}, sw[4] = {sv.x, sv.y, sv.z, sv.w};
    const bool first = sub < RD / 16;  // the lane holds elements of the first rotary half
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float p0 = first ? -lo_bf(pp[i]) : lo_bf(pp[i]), p1 = first ? -hi_bf(pp[i]) : hi_bf(pp[i]);
      const float a0 = round_bf(__fmul_rn(y[2 * i], lo_bf(cw[i]))), a1 = round_bf(__fmul_rn(y[2 * i + 1], hi_bf(cw[i])));
      const float b0 = round_bf(__fmul_rn(p0, lo_bf(sw[i]))), b1 = round_bf(__fmul_rn(p1, hi_bf(sw[i])));
      o[i] = pack_bf(__fadd_rn(a0, b0), __fadd_rn(a1, b1));
    }
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) o[i] = yp[i];
  }
  if (live) reinterpret_cast<uint4*>(out + it * 128)[sub] = make_uint4(o[0], o[1], o[2], o[3]);
}

}  // namespace

extern "C" int d3b_qk_norm_rope(const void* x, const int64_t* x_strides, const void* weight, const void* cos,
                                const void* sin, const int64_t* cs_strides, void* out, int rows, int T, int heads,
                                int head_dim, int rotary_dim, float eps, d3b_stream_t stream) {
  if (rows < 0 || T < 0 || heads <= 0) return D3B_EINVAL;
  if (head_dim != 128) return D3B_EUNSUPPORTED;
  if (rotary_dim != 16 && rotary_dim != 32 && rotary_dim != 64 && rotary_dim != 128) return D3B_EUNSUPPORTED;
  if ((int64_t)rows * T == 0) return D3B_OK;
  if (!x || !x_strides || !weight || !cos || !sin || !cs_strides || !out) return D3B_EINVAL;
  const void* ptrs[5] = {x, weight, cos, sin, out};
  for (const void* p : ptrs)
    if (reinterpret_cast<uintptr_t>(p) % 16) return D3B_EALIGN;
  for (int i = 0; i < 3; ++i)
    if (x_strides[i] % 8 || x_strides[i] < 0) return D3B_EALIGN;
  if (cs_strides[0] % 8 || cs_strides[1] % 8 || cs_strides[0] < 0 || cs_strides[1] < 0) return D3B_EALIGN;
  const int64_t tokens = (int64_t)rows * T;
  if (tokens > 0x7FFFFFFF) return D3B_EINVAL;
  // heads per CTA, 16 lanes each, rounded up to whole warps (the shuffles take every lane;
  // a lane past the last head computes head 0 again and stores nothing)
  int per_cta = heads < kThreads / 16 ? heads : kThreads / 16;
  per_cta += per_cta & 1;
  const int groups = (heads + per_cta - 1) / per_cta;
  if (groups > 65535) return D3B_EINVAL;
  const auto* xs = static_cast<const uint16_t*>(x);
  const auto* ws = static_cast<const uint16_t*>(weight);
  const auto* cs = static_cast<const uint16_t*>(cos);
  const auto* sn = static_cast<const uint16_t*>(sin);
  auto* os = static_cast<uint16_t*>(out);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const dim3 grid((unsigned)tokens, (unsigned)groups), block((unsigned)(16 * per_cta));
  switch (rotary_dim) {
    case 16: qk_norm_rope_kernel<16><<<grid, block, 0, s>>>(xs, x_strides[0], x_strides[1], x_strides[2], ws, cs, sn,
                                                            cs_strides[0], cs_strides[1], os, T, heads, eps); break;
    case 32: qk_norm_rope_kernel<32><<<grid, block, 0, s>>>(xs, x_strides[0], x_strides[1], x_strides[2], ws, cs, sn,
                                                            cs_strides[0], cs_strides[1], os, T, heads, eps); break;
    case 64: qk_norm_rope_kernel<64><<<grid, block, 0, s>>>(xs, x_strides[0], x_strides[1], x_strides[2], ws, cs, sn,
                                                            cs_strides[0], cs_strides[1], os, T, heads, eps); break;
    default: qk_norm_rope_kernel<128><<<grid, block, 0, s>>>(xs, x_strides[0], x_strides[1], x_strides[2], ws, cs, sn,
                                                             cs_strides[0], cs_strides[1], os, T, heads, eps); break;
  }
  return d3b_host::check_launch();
}
