// Gated delta rule (the GDN layers' scan), token-recurrent form, fp32 state.
//
// Per (row b, value head hv), over tokens t, with q, k L2-normalised and q
// scaled (FLA fused_recurrent_gated_delta_rule, the reference's `recurrent`
// path, d3trt/model/ops.py:327-360, d3trt/model/core.py:360-372):
//   S <- exp(g_t) S;  v' = beta_t (v_t - S^T k_t);  S <- S + k_t v'^T;  o_t = S^T q_t
// S is [K, V] fp32. q/k heads map to value heads as hv / (HV / H), so callers
// pass the un-repeated q/k (the reference repeats them, core.py:345-347). The
// initial state may be shared across rows (row stride 0), so the question pass
// needs no per-row copy of the snapshot's state (core.py:331).
//
// One CTA per (row, value head, 32-column block of V); warp w holds rows
// [32w, 32w + 32) of the state slice in registers, lane = column. The state is
// kept as c * H with a running scalar c, so the decay is one multiply per token
// and each state element costs three FMAs per token (k.S, the rank-1 update,
// q.S). Three CTA barriers per token; the next token's inputs are loaded into
// registers while the current one is computed.
#include "common.cuh"

namespace {

struct GdrParams {
  const void* q;
  const void* k;
  const void* v;
  const float* g;
  const void* beta;
  const float* h0;
  void* o;
  float* ht;
  long long qs[3], ks[3], vs[3], gs[3], bs[3], h0s[3], os[3];  // element strides [b, t, head]; h0: [b, hv, k-row]
  int B, T, H, HV, V;
  float scale;
  int l2norm;
};

template <typename T>
__device__ __forceinline__ float to_f32(T x);
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <>
__device__ __forceinline__ float to_f32<__half>(__half x) { return __half2float(x); }
template <>
__device__ __forceinline__ float to_f32<float>(float x) { return x; }

template <typename T>
__device__ __forceinline__ T from_f32(float x);
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <>
__device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int s = 16; s > 0; s >>= 1) x += __shfl_xor_sync(0xffffffffu, x, s);
  return x;
}

template <int K, typename In, typename BetaT>
__global__ void __launch_bounds__(K) gdr_recurrent_kernel(const __grid_constant__ GdrParams p) {
  constexpr int W = K / 32;
  const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31;
  const int n_vb = p.V >> 5;
  const long long blk = blockIdx.x;
  const int vb = (int)(blk % n_vb);
  const long long bh = blk / n_vb;
  const int b = (int)(bh / p.HV), hv = (int)(bh % p.HV), h = hv / (p.HV / p.H);
  const int j = vb * 32 + lane;

  __shared__ float q_s[K], k_s[K];
  __shared__ float part[2][W];
  __shared__ float red[W][32], red2[W][32];

  float hs[32];
  if (p.h0) {
    const float* src = p.h0 + b * p.h0s[0] + hv * p.h0s[1] + j;
#pragma unroll
    for (int r = 0; r < 32; ++r) hs[r] = src[(long long)(w * 32 + r) * p.h0s[2]];
  } else {
#pragma unroll
    for (int r = 0; r < 32; ++r) hs[r] = 0.f;
  }
  float c = 1.f;  // the state is c * hs

  const In* qp = static_cast<const In*>(p.q) + b * p.qs[0] + h * p.qs[2] + tid;
  const In* kp = static_cast<const In*>(p.k) + b * p.ks[0] + h * p.ks[2] + tid;
  const In* vp = static_cast<const In*>(p.v) + b * p.vs[0] + hv * p.vs[2] + j;
  const float* gp = p.g + b * p.gs[0] + hv * p.gs[2];
  const BetaT* bp = static_cast<const BetaT*>(p.beta) + b * p.bs[0] + hv * p.bs[2];
  In* op = static_cast<In*>(p.o) + b * p.os[0] + hv * p.os[2] + j;

  float qv = 0.f, kv = 0.f, vv = 0.f, gv = 0.f, bv = 0.f;
  if (p.T > 0) {
    qv = to_f32(qp[0]);
    kv = to_f32(kp[0]);
    vv = to_f32(vp[0]);
    gv = gp[0];
    bv = to_f32(bp[0]);
  }
  for (int t = 0; t < p.T; ++t) {
    q_s[tid] = qv;
    k_s[tid] = kv;
    const float sq = warp_sum(qv * qv), sk = warp_sum(kv * kv);
    if (lane == 0) {
      part[0][w] = sq;
      part[1][w] = sk;
    }
    const float v_t = vv, g_t = gv, beta_t = bv;
    __syncthreads();  // B1: raw q, k and their partial norms are visible
    if (t + 1 < p.T) {  // next token's inputs, in flight during this token's math
      qv = to_f32(qp[(long long)(t + 1) * p.qs[1]]);
      kv = to_f32(kp[(long long)(t + 1) * p.ks[1]]);
      vv = to_f32(vp[(long long)(t + 1) * p.vs[1]]);
      gv = gp[(long long)(t + 1) * p.gs[1]];
      bv = to_f32(bp[(long long)(t + 1) * p.bs[1]]);
    }
    float nq = 0.f, nk = 0.f;
#pragma unroll
    for (int i = 0; i < W; ++i) {
      nq += part[0][i];
      nk += part[1][i];
    }
    const float ik = p.l2norm ? 1.f / sqrtf(nk + 1e-6f) : 1.f;
    const float iq = (p.l2norm ? 1.f / sqrtf(nq + 1e-6f) : 1.f) * p.scale;
    c *= expf(g_t);
    if (c < 1e-20f || c > 1e20f) {  // uniform: every thread holds the same c
#pragma unroll
      for (int r = 0; r < 32; ++r) hs[r] *= c;
      c = 1.f;
    }
    float acc = 0.f;
#pragma unroll
    for (int r = 0; r < 32; ++r) acc = fmaf(k_s[w * 32 + r], hs[r], acc);
    red[w][lane] = acc;
    __syncthreads();  // B2: partial k.S per warp
    float kh = 0.f;
#pragma unroll
    for (int i = 0; i < W; ++i) kh += red[i][lane];
    const float vnew = beta_t * (v_t - kh * c * ik);
    const float upd = vnew * ik / c;
    float oacc = 0.f;
#pragma unroll
    for (int r = 0; r < 32; ++r) {
      hs[r] = fmaf(k_s[w * 32 + r], upd, hs[r]);
      oacc = fmaf(q_s[w * 32 + r], hs[r], oacc);
    }
    red2[w][lane] = oacc;
    __syncthreads();  // B3: partial q.S per warp; q_s / k_s / red free again
    if (w == 0) {
      float o = 0.f;
#pragma unroll
      for (int i = 0; i < W; ++i) o += red2[i][lane];
      op[(long long)t * p.os[1]] = from_f32<In>(o * c * iq);
    }
  }
  if (p.ht) {
    float* dst = p.ht + ((long long)bh * K + w * 32) * p.V + j;
#pragma unroll
    for (int r = 0; r < 32; ++r) dst[(long long)r * p.V] = hs[r] * c;
  }
}

template <int K, typename In>
int launch_k(const GdrParams& p, int beta_dtype, long long blocks, cudaStream_t s) {
  switch (beta_dtype) {
    case D3B_F32: gdr_recurrent_kernel<K, In, float><<<(unsigned)blocks, K, 0, s>>>(p); break;
    case D3B_BF16: gdr_recurrent_kernel<K, In, __nv_bfloat16><<<(unsigned)blocks, K, 0, s>>>(p); break;
    case D3B_F16: gdr_recurrent_kernel<K, In, __half><<<(unsigned)blocks, K, 0, s>>>(p); break;
    default: return D3B_EUNSUPPORTED;
  }
  return d3b_host::check_launch();
}

bool aligned(const void* ptr, int bytes) { return reinterpret_cast<uintptr_t>(ptr) % bytes == 0; }

}  // namespace

extern "C" int d3b_gated_delta_rule(const void* q, const int64_t* q_strides, const void* k, const int64_t* k_strides,
                                    const void* v, const int64_t* v_strides, const float* g,
                                    const int64_t* g_strides, const void* beta, int beta_dtype,
                                    const int64_t* beta_strides, const float* h0, const int64_t* h0_strides,
                                    void* o, const int64_t* o_strides, float* ht, int B, int T, int H, int HV,
                                    int K, int V, int dtype, float scale, int l2norm, d3b_stream_t stream) {
  if (B < 0 || T < 0 || H <= 0 || HV <= 0 || HV % H != 0 || V <= 0 || V % 32 != 0) return D3B_EINVAL;
  if (!q_strides || !k_strides || !v_strides || !g_strides || !beta_strides || !o_strides) return D3B_EINVAL;
  if (h0 && !h0_strides) return D3B_EINVAL;
  if (K != 64 && K != 128) return D3B_EUNSUPPORTED;
  if (dtype != D3B_BF16 && dtype != D3B_F16) return D3B_EUNSUPPORTED;
  if (beta_dtype != D3B_F32 && beta_dtype != D3B_BF16 && beta_dtype != D3B_F16) return D3B_EUNSUPPORTED;
  const long long blocks = (long long)B * HV * (V / 32);
  if (blocks == 0) return D3B_OK;
  if (blocks >= (1ll << 31)) return D3B_EINVAL;
  if (T > 0 && (!q || !k || !v || !g || !beta || !o)) return D3B_EINVAL;
  if (!aligned(q, 2) || !aligned(k, 2) || !aligned(v, 2) || !aligned(o, 2) || !aligned(g, 4) ||
      (h0 && !aligned(h0, 4)) || (ht && !aligned(ht, 4)))
    return D3B_EALIGN;
  GdrParams p;
  p.q = q;
  p.k = k;
  p.v = v;
  p.g = g;
  p.beta = beta;
  p.h0 = h0;
  p.o = o;
  p.ht = ht;
  for (int i = 0; i < 3; ++i) {
    p.qs[i] = q_strides[i];
    p.ks[i] = k_strides[i];
    p.vs[i] = v_strides[i];
    p.gs[i] = g_strides[i];
    p.bs[i] = beta_strides[i];
    p.os[i] = o_strides[i];
    p.h0s[i] = h0 ? h0_strides[i] : 0;
  }
  p.B = B;
  p.T = T;
  p.H = H;
  p.HV = HV;
  p.V = V;
  p.scale = scale;
  p.l2norm = l2norm ? 1 : 0;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (K == 128)
    return dtype == D3B_BF16 ? launch_k<128, __nv_bfloat16>(p, beta_dtype, blocks, s)
                             : launch_k<128, __half>(p, beta_dtype, blocks, s);
  return dtype == D3B_BF16 ? launch_k<64, __nv_bfloat16>(p, beta_dtype, blocks, s)
                           : launch_k<64, __half>(p, beta_dtype, blocks, s);
}
