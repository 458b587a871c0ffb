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
// One warp per (row, value head, 16 state columns); each lane holds an (K/16) x 8
// tile of the state in registers: half-warp lanes split the rows, the two halves
// split the columns. The column sums over K (k.S and q.S) finish with a
// reduce-scatter across the 16 row lanes (8 shuffles: every lane ends with one
// column's total; the tile's columns are kept in a lane-dependent XOR order so no
// level needs a select) and v' goes back with the inverse all-gather (7 shuffles), so
// each lane reads only its K/16 rows of q and k per token: shared-memory traffic
// stays far below the shuffle and FMA work. No barriers. The token's normalised
// q and k are staged once per warp in shared memory (double-buffered);
// q, k and v travel to shared memory by cp.async three tokens ahead of the one
// being computed, g and beta 32 tokens at a time (one value per lane, shuffled). The
// state is kept as c * H with a running scalar c, so the decay costs one
// multiply per token, and the output uses o = S'^T q + (k.q) v' (S' the decayed
// state before the update), so each state element costs three FMAs per token,
// issued as packed fp32x2 FMAs (two rows per instruction).
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

// (d0, d1) += (a0, a1) * (b0, b1): one packed fp32x2 FMA, each lane an IEEE fma
__device__ __forceinline__ void fma2(float& d0, float& d1, float a0, float a1, float b0, float b1) {
  asm("{.reg .b64 x, y, z; mov.b64 x, {%2, %3}; mov.b64 y, {%4, %5}; mov.b64 z, {%0, %1};"
      " fma.rn.f32x2 z, x, y, z; mov.b64 {%0, %1}, z;}"
      : "+f"(d0), "+f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}

template <int K, typename In, typename BetaT>
__global__ void __launch_bounds__(32) gdr_recurrent_kernel(const __grid_constant__ GdrParams p) {
  constexpr int E = K / 32;   // q/k elements each lane copies per token
  constexpr int RL = K / 16;  // state rows per lane
  constexpr unsigned FULL = 0xffffffffu;
  static_assert(RL == 4 || RL == 8, "K is 64 or 128");
  const int lane = threadIdx.x;
  const int hl = lane & 15, cb = lane >> 4;  // row block, column half
  const int jj = (hl >> 1) & 7;  // the column this lane owns after a reduce-scatter
  const int n_vb = p.V >> 4;                  // 16 columns per warp
  const long long blk = blockIdx.x;
  const int vb = (int)(blk % n_vb);
  const long long bh = blk / n_vb;
  const int b = (int)(bh / p.HV), hv = (int)(bh % p.HV), h = hv / (p.HV / p.H);
  const int col0 = vb * 16 + cb * 8;  // first of this lane's 8 state columns
  const int row0 = hl * RL;

  __shared__ __align__(16) float qk_s[2][2][K];  // [buffer][q, k][K], normalised

  // S[i][p] holds state row row0 + i, column col0 + (p ^ jj): with the columns in this
  // lane-dependent order the reduce-scatter keeps and sends fixed positions (no selects)
  float S[RL][8];
  if (p.h0) {
    const float* src = p.h0 + b * p.h0s[0] + hv * p.h0s[1] + (long long)row0 * p.h0s[2] + col0;
#pragma unroll
    for (int i = 0; i < RL; ++i)
#pragma unroll
      for (int c8 = 0; c8 < 8; ++c8) S[i][c8] = src[(long long)i * p.h0s[2] + (c8 ^ jj)];
  } else {
#pragma unroll
    for (int i = 0; i < RL; ++i)
#pragma unroll
      for (int c8 = 0; c8 < 8; ++c8) S[i][c8] = 0.f;
  }
  float c = 1.f;  // the state is c * S

  const In* qp = static_cast<const In*>(p.q) + b * p.qs[0] + h * p.qs[2] + lane * E;
  const In* kp = static_cast<const In*>(p.k) + b * p.ks[0] + h * p.ks[2] + lane * E;
  const float* gp = p.g + b * p.gs[0] + hv * p.gs[2];
  const BetaT* bp = static_cast<const BetaT*>(p.beta) + b * p.bs[0] + hv * p.bs[2];
  In* op = static_cast<In*>(p.o) + b * p.os[0] + hv * p.os[2] + col0 + jj;

  // q, k and v of the next D - 1 tokens travel to shared memory by cp.async, so
  // nothing is held in registers while they are in flight; each lane copies its
  // own E elements of q and k, lanes 0-7 two values of v each. Every prefetch
  // commits one group, empty past the last token, so "token t's copies are done"
  // is always "at most D - 2 newer groups pending".
  constexpr int D = 4;
  __shared__ __align__(16) In raw_s[D][2][K];  // [slot][q, k][K] as loaded
  __shared__ __align__(16) In raw_v[D][16];    // [slot][this warp's 16 columns]
  const In* vrow = static_cast<const In*>(p.v) + b * p.vs[0] + hv * p.vs[2] + vb * 16 + 2 * lane;
  auto prefetch = [&](int t) {
    if (t < p.T) {
      const int slot = t % D;
      const uint32_t dq = d3b::smem_u32(&raw_s[slot][0][lane * E]);
      const uint32_t dk = d3b::smem_u32(&raw_s[slot][1][lane * E]);
      const In* sq = qp + (long long)t * p.qs[1];
      const In* sk = kp + (long long)t * p.ks[1];
      asm volatile("cp.async.ca.shared.global [%0], [%1], %2;" ::"r"(dq), "l"(sq), "n"(E * 2) : "memory");
      asm volatile("cp.async.ca.shared.global [%0], [%1], %2;" ::"r"(dk), "l"(sk), "n"(E * 2) : "memory");
      if (lane < 8) {
        const uint32_t dv = d3b::smem_u32(&raw_v[slot][2 * lane]);
        asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dv), "l"(vrow + (long long)t * p.vs[1])
                     : "memory");
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  // wait for token t's copies, normalise q and k, publish them to qk_s[t & 1]; returns k.q
  auto stage = [&](int t) -> float {
    asm volatile("cp.async.wait_group %0;" ::"n"(D - 2) : "memory");
    const int slot = t % D, buf = t & 1;
    float qr[E], kr[E];
#pragma unroll
    for (int e = 0; e < E; ++e) {
      qr[e] = to_f32(raw_s[slot][0][lane * E + e]);
      kr[e] = to_f32(raw_s[slot][1][lane * E + e]);
    }
    float sq = 0.f, sk = 0.f, sqk = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      sq = fmaf(qr[e], qr[e], sq);
      sk = fmaf(kr[e], kr[e], sk);
      sqk = fmaf(qr[e], kr[e], sqk);
    }
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) {  // three independent butterflies
      sq += __shfl_xor_sync(FULL, sq, m);
      sk += __shfl_xor_sync(FULL, sk, m);
      sqk += __shfl_xor_sync(FULL, sqk, m);
    }
    const float ik = p.l2norm ? rsqrtf(sk + 1e-6f) : 1.f;
    const float iq = (p.l2norm ? rsqrtf(sq + 1e-6f) : 1.f) * p.scale;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      qk_s[buf][0][lane * E + e] = qr[e] * iq;
      qk_s[buf][1][lane * E + e] = kr[e] * ik;
    }
    return sqk * iq * ik;
  };
  // Sum 8 per-column partials (positions p, columns p ^ jj) over the 16 lanes of a
  // half-warp; the partner at lane distance 8 (4, 2) holds my kept columns at
  // positions p ^ 4 (p ^ 2, p ^ 1), so each level sends the upper positions and
  // adds into the lower ones. The lane ends with the total of column jj (lanes hl
  // and hl ^ 1 hold the same one).
  auto reduce_scatter = [&](const float (&a)[8]) -> float {
    float b4[4], b2[2];
#pragma unroll
    for (int i = 0; i < 4; ++i) b4[i] = a[i] + __shfl_xor_sync(FULL, a[4 + i], 8);
#pragma unroll
    for (int i = 0; i < 2; ++i) b2[i] = b4[i] + __shfl_xor_sync(FULL, b4[2 + i], 4);
    const float d = b2[0] + __shfl_xor_sync(FULL, b2[1], 2);
    return d + __shfl_xor_sync(FULL, d, 1);
  };
  // The inverse: every lane gets the values of its 8 columns, in its own order.
  auto all_gather = [&](float u, float (&g8)[8]) {
    g8[0] = u;
    g8[1] = __shfl_xor_sync(FULL, g8[0], 2);
    g8[2] = __shfl_xor_sync(FULL, g8[0], 4);
    g8[3] = __shfl_xor_sync(FULL, g8[1], 4);
#pragma unroll
    for (int i = 0; i < 4; ++i) g8[4 + i] = __shfl_xor_sync(FULL, g8[i], 8);
  };
  // g and beta of 32 tokens at a time: lane l holds token 32 * group + l, one group ahead
  float g_cur = 0.f, b_cur = 0.f, g_nxt = 0.f, b_nxt = 0.f;
  auto load_scalars = [&](int t0, float& gg, float& bb) {
    const int t = t0 + lane;
    if (t < p.T) {
      gg = gp[(long long)t * p.gs[1]];
      bb = to_f32(bp[(long long)t * p.bs[1]]);
    }
  };

#pragma unroll
  for (int i = 0; i < D - 1; ++i) prefetch(i);
  load_scalars(0, g_cur, b_cur);
  load_scalars(32, g_nxt, b_nxt);
  float kq = 0.f;
  if (p.T > 0) kq = stage(0);
  __syncwarp();
  prefetch(D - 1);
  __syncwarp();
  for (int t = 0; t < p.T; ++t) {
    const int buf = t & 1;
    if (t > 0 && (t & 31) == 0) {
      g_cur = g_nxt;
      b_cur = b_nxt;
      load_scalars(t + 32, g_nxt, b_nxt);
    }
    const float g_t = __shfl_sync(FULL, g_cur, t & 31);
    const float beta_t = __shfl_sync(FULL, b_cur, t & 31);
    const float v_t = to_f32(raw_v[t % D][cb * 8 + jj]);
    c *= __expf(g_t);
    if (c < 1e-20f || c > 1e20f) {  // warp-uniform: every lane holds the same c
#pragma unroll
      for (int i = 0; i < RL; ++i)
#pragma unroll
        for (int c8 = 0; c8 < 8; ++c8) S[i][c8] *= c;
      c = 1.f;
    }
    float kr[RL], qr[RL];
#pragma unroll
    for (int i4 = 0; i4 < RL / 4; ++i4) {
      const float4 kk = reinterpret_cast<const float4*>(qk_s[buf][1] + row0)[i4];
      const float4 qq = reinterpret_cast<const float4*>(qk_s[buf][0] + row0)[i4];
      kr[4 * i4 + 0] = kk.x; kr[4 * i4 + 1] = kk.y; kr[4 * i4 + 2] = kk.z; kr[4 * i4 + 3] = kk.w;
      qr[4 * i4 + 0] = qq.x; qr[4 * i4 + 1] = qq.y; qr[4 * i4 + 2] = qq.z; qr[4 * i4 + 3] = qq.w;
    }
    float ak[8], aq[8];
#pragma unroll
    for (int c8 = 0; c8 < 8; ++c8) ak[c8] = aq[c8] = 0.f;
#pragma unroll
    for (int i = 0; i < RL; ++i)
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        fma2(ak[2 * m], ak[2 * m + 1], kr[i], kr[i], S[i][2 * m], S[i][2 * m + 1]);
        fma2(aq[2 * m], aq[2 * m + 1], qr[i], qr[i], S[i][2 * m], S[i][2 * m + 1]);
      }
    const float kh = reduce_scatter(ak) * c;
    const float qh = reduce_scatter(aq) * c;
    const float vnew = beta_t * (v_t - kh);
    if ((hl & 1) == 0) op[(long long)t * p.os[1]] = from_f32<In>(fmaf(kq, vnew, qh));
    float upd[8];
    all_gather(vnew * __frcp_rn(c), upd);
#pragma unroll
    for (int i = 0; i < RL; ++i)
#pragma unroll
      for (int m = 0; m < 4; ++m) fma2(S[i][2 * m], S[i][2 * m + 1], kr[i], kr[i], upd[2 * m], upd[2 * m + 1]);
    if (t + 1 < p.T) {
      kq = stage(t + 1);  // copied while earlier tokens were computed
      __syncwarp();       // every lane has read token t's v: its slot may be refilled
      prefetch(t + D);
      __syncwarp();       // token t+1's normalised q, k visible to all lanes
    }
  }
  if (p.ht) {
    float* dst = p.ht + ((long long)bh * K + row0) * p.V + col0;
#pragma unroll
    for (int i = 0; i < RL; ++i)
#pragma unroll
      for (int c8 = 0; c8 < 8; ++c8) dst[(long long)i * p.V + (c8 ^ jj)] = S[i][c8] * c;
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
  const long long blocks = (long long)B * HV * (V / 16);  // one warp per 16 state columns
  if (blocks == 0) return D3B_OK;
  if (blocks >= (1ll << 31)) return D3B_EINVAL;
  if (T > 0 && (!q || !k || !v || !g || !beta || !o)) return D3B_EINVAL;
  // q/k rows are copied E = K/32 elements per lane (cp.async of 2E bytes)
  const int E = K / 32;
  if (!aligned(q, 2 * E) || !aligned(k, 2 * E) || !aligned(v, 2) || !aligned(o, 2) || !aligned(g, 4) ||
      (h0 && !aligned(h0, 4)) || (ht && !aligned(ht, 4)))
    return D3B_EALIGN;
  for (int i = 0; i < 3; ++i)
    if (q_strides[i] % E != 0 || k_strides[i] % E != 0 || v_strides[i] % 2 != 0) return D3B_EALIGN;
  if (!aligned(v, 4)) return D3B_EALIGN;  // v is copied two values (4 bytes) per lane
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
