// Causal depthwise convolution with SiLU over token-major rows: the GDN layers'
// short convolution (d3trt/model/core.py:311-330 via ops.causal_conv1d,
// d3trt/model/ops.py:266-285: F.conv1d(groups=C, padding=W-1) cut to L, then SiLU).
//
//   out[r, t, c] = silu(bf16( sum_{j<W} w[c, j] * in(r, t - (W-1) + j, c) ))
//   in(r, u, c)  = x[r, u, c] for u >= 0,
//                  tail(r, c, (W-1) + u) for -(W-1) <= u < 0 (question pass: the
//                  snapshot's last W-1 inputs of the state), 0 without a tail
//
// x is the in_proj output as the GEMM leaves it ([rows, T, C], channels
// contiguous), so no transpose or concatenation is made: one thread owns 8
// adjacent channels (one 16-byte load per token, a warp reads 512 contiguous
// bytes) and slides over a run of tokens keeping the last W-1 inputs in
// registers, so every input is read once (plus a W-1 token halo per run); the
// loads run two tokens ahead of the arithmetic.
// Sums in fp32 in kernel order j = 0..W-1, rounded to bf16, SiLU in fp32
// (x / (1 + exp(-x))) rounded to bf16 -- the two roundings of the reference's
// conv1d + silu on bf16 tensors.
#include "common.cuh"

namespace {

constexpr int kConvThreads = 128;
constexpr int kConvRun = 32;  // tokens per thread

__device__ __forceinline__ float bf(uint16_t v) { return __uint_as_float((uint32_t)v << 16); }

template <int W>
__global__ void __launch_bounds__(kConvThreads) causal_conv_silu_kernel(
    const uint16_t* __restrict__ x, int64_t sx_r, int64_t sx_t, const uint16_t* __restrict__ tail, int64_t st_r,
    int64_t st_c, int64_t st_k, const uint16_t* __restrict__ w, uint16_t* __restrict__ out, int T, int C) {
  const int c0 = (blockIdx.x * kConvThreads + threadIdx.x) * 8;
  if (c0 >= C) return;
  const int r = blockIdx.y;
  const int t0 = blockIdx.z * kConvRun;
  const int t1 = min(t0 + kConvRun, T);
  float wv[8][W];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < W; ++j) wv[i][j] = bf(w[(int64_t)(c0 + i) * W + j]);
  float hist[W - 1][8];  // inputs at t0 - (W-1) .. t0 - 1
#pragma unroll
  for (int k = 0; k < W - 1; ++k) {
    const int u = t0 - (W - 1) + k;
    if (u >= 0) {
      const uint4 a = *reinterpret_cast<const uint4*>(x + r * sx_r + (int64_t)u * sx_t + c0);
      const uint32_t ww[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        hist[k][2 * i] = __uint_as_float(ww[i] << 16);
        hist[k][2 * i + 1] = __uint_as_float(ww[i] & 0xFFFF0000u);
      }
    } else if (tail) {
      const uint16_t* tp = tail + r * st_r + (int64_t)((W - 1) + u) * st_k;
#pragma unroll
      for (int i = 0; i < 8; ++i) hist[k][i] = bf(tp[(int64_t)(c0 + i) * st_c]);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) hist[k][i] = 0.f;
    }
  }
  const uint16_t* xr = x + r * sx_r + c0;
  uint16_t* orow = out + ((int64_t)r * T) * C + c0;
  // the next two tokens' inputs are loaded ahead, so their memory latency overlaps this
  // token's arithmetic instead of stalling every step of the run
  auto load_tok = [&](int t) {
    return t < t1 ? *reinterpret_cast<const uint4*>(xr + (int64_t)t * sx_t) : make_uint4(0, 0, 0, 0);
  };
  uint4 ahead0 = load_tok(t0), ahead1 = load_tok(t0 + 1);
  for (int t = t0; t < t1; ++t) {
    const uint4 a = ahead0;
    ahead0 = ahead1;
    ahead1 = load_tok(t + 2);
    const uint32_t ww[4] = {a.x, a.y, a.z, a.w};
    float cur[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      cur[2 * i] = __uint_as_float(ww[i] << 16);
      cur[2 * i + 1] = __uint_as_float(ww[i] & 0xFFFF0000u);
    }
    uint32_t packed[4];
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
      float y[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        float acc = 0.f;
#pragma unroll
        for (int j = 0; j < W - 1; ++j) acc = fmaf(wv[i + e][j], hist[j][i + e], acc);
        acc = fmaf(wv[i + e][W - 1], cur[i + e], acc);
        const float s = __bfloat162float(__float2bfloat16_rn(acc));
        y[e] = s / (1.0f + expf(-s));
      }
      const __nv_bfloat162 p = __floats2bfloat162_rn(y[0], y[1]);
      packed[i / 2] = *reinterpret_cast<const uint32_t*>(&p);
    }
    *reinterpret_cast<uint4*>(orow + (int64_t)t * C) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
#pragma unroll
    for (int k = 0; k < W - 2; ++k)
#pragma unroll
      for (int i = 0; i < 8; ++i) hist[k][i] = hist[k + 1][i];
#pragma unroll
    for (int i = 0; i < 8; ++i) hist[W - 2][i] = cur[i];
  }
}

template <int W>
int launch(const uint16_t* x, int64_t sx_r, int64_t sx_t, const uint16_t* tail, int64_t st_r, int64_t st_c,
           int64_t st_k, const uint16_t* w, uint16_t* out, int rows, int T, int C, cudaStream_t s) {
  const dim3 grid((unsigned)((C / 8 + kConvThreads - 1) / kConvThreads), (unsigned)rows,
                  (unsigned)((T + kConvRun - 1) / kConvRun));
  causal_conv_silu_kernel<W><<<grid, kConvThreads, 0, s>>>(x, sx_r, sx_t, tail, st_r, st_c, st_k, w, out, T, C);
  return d3b_host::check_launch();
}

}  // namespace

extern "C" int d3b_causal_conv1d_silu(const void* x, const int64_t* x_strides, const void* tail,
                                      const int64_t* tail_strides, const void* weight, void* out, int rows, int T,
                                      int C, int W, d3b_stream_t stream) {
  if (rows < 0 || T < 0 || C <= 0 || W < 2 || W > 8) return W > 8 ? D3B_EUNSUPPORTED : D3B_EINVAL;
  if (rows == 0 || T == 0) return D3B_OK;
  if (!x || !x_strides || !weight || !out || (tail && !tail_strides)) return D3B_EINVAL;
  if (rows > 65535 || (T + kConvRun - 1) / kConvRun > 65535) return D3B_EINVAL;
  if (C % 8 || x_strides[0] % 8 || x_strides[1] % 8 || x_strides[1] < C || reinterpret_cast<uintptr_t>(x) % 16 ||
      reinterpret_cast<uintptr_t>(out) % 16)
    return D3B_EALIGN;
  const auto* xs = static_cast<const uint16_t*>(x);
  const auto* ts = static_cast<const uint16_t*>(tail);
  const int64_t st_r = tail ? tail_strides[0] : 0, st_c = tail ? tail_strides[1] : 0, st_k = tail ? tail_strides[2] : 0;
  const auto* ws = static_cast<const uint16_t*>(weight);
  auto* os = static_cast<uint16_t*>(out);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (W) {
    case 2: return launch<2>(xs, x_strides[0], x_strides[1], ts, st_r, st_c, st_k, ws, os, rows, T, C, s);
    case 3: return launch<3>(xs, x_strides[0], x_strides[1], ts, st_r, st_c, st_k, ws, os, rows, T, C, s);
    case 4: return launch<4>(xs, x_strides[0], x_strides[1], ts, st_r, st_c, st_k, ws, os, rows, T, C, s);
    case 5: return launch<5>(xs, x_strides[0], x_strides[1], ts, st_r, st_c, st_k, ws, os, rows, T, C, s);
    case 6: return launch<6>(xs, x_strides[0], x_strides[1], ts, st_r, st_c, st_k, ws, os, rows, T, C, s);
    case 7: return launch<7>(xs, x_strides[0], x_strides[1], ts, st_r, st_c, st_k, ws, os, rows, T, C, s);
    case 8: return launch<8>(xs, x_strides[0], x_strides[1], ts, st_r, st_c, st_k, ws, os, rows, T, C, s);
  }
  return D3B_EUNSUPPORTED;
}
