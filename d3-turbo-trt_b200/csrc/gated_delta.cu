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
// One warp per (row, value head, 32-column block of V); lane j owns column j of the
// state, all K rows of it in registers, so both reductions over K (k.S and q.S)
// are thread-local: no shuffles, no barriers. The token's normalised q and k are
// staged once per warp in shared memory (double-buffered, read as broadcasts);
// the next token's q/k travel to shared memory by cp.async while the current one
// is computed. The
// state is kept as c * H with a running scalar c, so the decay costs one
// multiply per token, and the output uses o = S'^T q + (k.q) v' (S' the decayed
// state before the update), so each state element costs three FMAs per token.
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
__global__ void __launch_bounds__(32) gdr_recurrent_kernel(const __grid_constant__ GdrParams p) {
  constexpr int E = K / 32;  // q/k elements each lane loads per token
  static_assert(E == 2 || E == 4, "K is 64 or 128");
  const int lane = threadIdx.x;
  const int n_vb = p.V >> 5;
  const long long blk = blockIdx.x;
  const int vb = (int)(blk % n_vb);
  const long long bh = blk / n_vb;
  const int b = (int)(bh / p.HV), hv = (int)(bh % p.HV), h = hv / (p.HV / p.H);
  const int j = vb * 32 + lane;

  __shared__ __align__(16) float qk_s[2][2][K];  // [buffer][q, k][K], normalised

  float S[K];
  if (p.h0) {
    const float* src = p.h0 + b * p.h0s[0] + hv * p.h0s[1] + j;
#pragma unroll
    for (int r = 0; r < K; ++r) S[r] = src[(long long)r * p.h0s[2]];
  } else {
#pragma unroll
    for (int r = 0; r < K; ++r) S[r] = 0.f;
  }
  float c = 1.f;  // the state is c * S

  const In* qp = static_cast<const In*>(p.q) + b * p.qs[0] + h * p.qs[2] + lane * E;
  const In* kp = static_cast<const In*>(p.k) + b * p.ks[0] + h * p.ks[2] + lane * E;
  const In* vp = static_cast<const In*>(p.v) + b * p.vs[0] + hv * p.vs[2] + j;
  const float* gp = p.g + b * p.gs[0] + hv * p.gs[2];
  const BetaT* bp = static_cast<const BetaT*>(p.beta) + b * p.bs[0] + hv * p.bs[2];
  In* op = static_cast<In*>(p.o) + b * p.os[0] + hv * p.os[2] + j;

  // q/k of the next token arrive in shared memory by cp.async, so nothing is held
  // in registers while they are in flight; each lane copies, and later reads back,
  // its own E elements.
  __shared__ __align__(16) In raw_s[2][2][K];  // [buffer][q, k][K] as loaded
  auto prefetch = [&](int t, int buf) {
    const uint32_t dq = d3b::smem_u32(&raw_s[buf][0][lane * E]);
    const uint32_t dk = d3b::smem_u32(&raw_s[buf][1][lane * E]);
    const In* sq = qp + (long long)t * p.qs[1];
    const In* sk = kp + (long long)t * p.ks[1];
    asm volatile("cp.async.ca.shared.global [%0], [%1], %2;" ::"r"(dq), "l"(sq), "n"(E * 2) : "memory");
    asm volatile("cp.async.ca.shared.global [%0], [%1], %2;" ::"r"(dk), "l"(sk), "n"(E * 2) : "memory");
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  // wait for this lane's copies of one token, normalise, publish to qk_s[buf]; returns k.q
  auto stage = [&](int buf) -> float {
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    float qr[E], kr[E];
#pragma unroll
    for (int e = 0; e < E; ++e) {
      qr[e] = to_f32(raw_s[buf][0][lane * E + e]);
      kr[e] = to_f32(raw_s[buf][1][lane * E + e]);
    }
    float sq = 0.f, sk = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      sq = fmaf(qr[e], qr[e], sq);
      sk = fmaf(kr[e], kr[e], sk);
    }
    sq = warp_sum(sq);
    sk = warp_sum(sk);
    const float ik = p.l2norm ? 1.f / sqrtf(sk + 1e-6f) : 1.f;
    const float iq = (p.l2norm ? 1.f / sqrtf(sq + 1e-6f) : 1.f) * p.scale;
    float kq = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const float qn = qr[e] * iq, kn = kr[e] * ik;
      qk_s[buf][0][lane * E + e] = qn;
      qk_s[buf][1][lane * E + e] = kn;
      kq = fmaf(kn, qn, kq);
    }
    return warp_sum(kq);
  };

  float kq = 0.f, v_t = 0.f, g_t = 0.f, beta_t = 0.f, vv = 0.f, gv = 0.f, bv = 0.f;
  if (p.T > 0) {
    prefetch(0, 0);
    kq = stage(0);
    v_t = to_f32(vp[0]);
    g_t = gp[0];
    beta_t = to_f32(bp[0]);
    if (p.T > 1) prefetch(1, 1);
  }
  __syncwarp();
  for (int t = 0; t < p.T; ++t) {
    const int buf = t & 1;
    if (t + 1 < p.T) {  // the next token's scalars, in flight during this token's math
      vv = to_f32(vp[(long long)(t + 1) * p.vs[1]]);
      gv = gp[(long long)(t + 1) * p.gs[1]];
      bv = to_f32(bp[(long long)(t + 1) * p.bs[1]]);
    }
    c *= expf(g_t);
    if (c < 1e-20f || c > 1e20f) {  // warp-uniform: every lane holds the same c
#pragma unroll
      for (int r = 0; r < K; ++r) S[r] *= c;
      c = 1.f;
    }
    const float4* q4 = reinterpret_cast<const float4*>(qk_s[buf][0]);
    const float4* k4 = reinterpret_cast<const float4*>(qk_s[buf][1]);
    float ak[4] = {0.f, 0.f, 0.f, 0.f}, aq[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int r4 = 0; r4 < K / 4; ++r4) {
      if (r4 % 4 == 0) __syncwarp();  // bounds how far the compiler hoists the shared loads
      const float4 kk = k4[r4], qq = q4[r4];
      ak[0] = fmaf(kk.x, S[4 * r4 + 0], ak[0]);
      ak[1] = fmaf(kk.y, S[4 * r4 + 1], ak[1]);
      ak[2] = fmaf(kk.z, S[4 * r4 + 2], ak[2]);
      ak[3] = fmaf(kk.w, S[4 * r4 + 3], ak[3]);
      aq[0] = fmaf(qq.x, S[4 * r4 + 0], aq[0]);
      aq[1] = fmaf(qq.y, S[4 * r4 + 1], aq[1]);
      aq[2] = fmaf(qq.z, S[4 * r4 + 2], aq[2]);
      aq[3] = fmaf(qq.w, S[4 * r4 + 3], aq[3]);
    }
    const float kh = ((ak[0] + ak[1]) + (ak[2] + ak[3])) * c;
    const float qh = ((aq[0] + aq[1]) + (aq[2] + aq[3])) * c;
    const float vnew = beta_t * (v_t - kh);
    op[(long long)t * p.os[1]] = from_f32<In>(fmaf(kq, vnew, qh));
    const float upd = vnew / c;
#pragma unroll
    for (int r4 = 0; r4 < K / 4; ++r4) {
      if (r4 % 4 == 0) __syncwarp();
      const float4 kk = k4[r4];
      S[4 * r4 + 0] = fmaf(kk.x, upd, S[4 * r4 + 0]);
      S[4 * r4 + 1] = fmaf(kk.y, upd, S[4 * r4 + 1]);
      S[4 * r4 + 2] = fmaf(kk.z, upd, S[4 * r4 + 2]);
      S[4 * r4 + 3] = fmaf(kk.w, upd, S[4 * r4 + 3]);
    }
    if (t + 1 < p.T) {
      kq = stage(buf ^ 1);  // token t+1, copied while token t was computed
      if (t + 2 < p.T) prefetch(t + 2, buf);  // this lane read token t's raw copy one token ago
      v_t = vv;
      g_t = gv;
      beta_t = bv;
      __syncwarp();
    }
  }
  if (p.ht) {
    float* dst = p.ht + (long long)bh * K * p.V + j;
#pragma unroll
    for (int r = 0; r < K; ++r) dst[(long long)r * p.V] = S[r] * c;
  }
}

template <int K, typename In>
int launch_k(const GdrParams& p, int beta_dtype, long long blocks, cudaStream_t s) {
  switch (beta_dtype) {
    case D3B_F32: gdr_recurrent_kernel<K, In, float><<<(unsigned)blocks, 32, 0, s>>>(p); break;
    case D3B_BF16: gdr_recurrent_kernel<K, In, __nv_bfloat16><<<(unsigned)blocks, 32, 0, s>>>(p); break;
    case D3B_F16: gdr_recurrent_kernel<K, In, __half><<<(unsigned)blocks, 32, 0, s>>>(p); break;
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
  // q/k rows are copied E = K/32 elements per lane (cp.async of 2E bytes)
  const int E = K / 32;
  if (!aligned(q, 2 * E) || !aligned(k, 2 * E) || !aligned(v, 2) || !aligned(o, 2) || !aligned(g, 4) ||
      (h0 && !aligned(h0, 4)) || (ht && !aligned(ht, 4)))
    return D3B_EALIGN;
  for (int i = 0; i < 3; ++i)
    if (q_strides[i] % E != 0 || k_strides[i] % E != 0) return D3B_EALIGN;
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
