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
#include <algorithm>

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

// ---------------------------------------------------------------------------
// Chunked form for blocks of at most 64 tokens (the question pass), K = V = 128,
// one initial state shared by all rows, no final state. With gamma the running
// sum of g inside the block (WY form of the same recurrence):
//   A  = strictly-lower( beta_i (k_i . k_j) e^(gamma_i - gamma_j) )
//   R  = beta_i (v_i - e^gamma_i S0^T k_i)        (rows i)
//   V' = (I + A)^-1 R                             (forward substitution)
//   O  = e^gamma_i S0^T q_i + lower-incl( (q_i . k_j) e^(gamma_i - gamma_j) ) V'
// One work item = two blocks (M = 128 rows) and one value head; a persistent CTA of
// 256 threads per SM loops over work items (TMEM and barriers set up once). The four
// products K K^T, K S0, Q K^T, Q S0 run on tcgen05 into TMEM (bf16 operands,
// fp32 accumulate: 512 columns), the epilogue (two threads per row) forms A, R and
// the decayed P = lower(Q K^T) as bf16, the solve runs with one thread per (state
// column, block) in fp32 registers (column-oriented, A stored transposed), then
// P V' runs on tcgen05 into the freed columns 0..127. q, k, v rows and the state's
// bf16 image arrive by bulk copies during the first phase.
// ---------------------------------------------------------------------------
// Waits (bounded, ignoring the abort flag) for a phase of a barrier that bulk
// copies complete, so a CTA that gave up does not exit with copies into its
// shared memory in flight.
__device__ __forceinline__ void settle(uint64_t* bar, uint32_t parity) {
  const uint32_t addr = d3b::smem_u32(bar);
  const uint64_t t0 = d3b::globaltimer_ns();
  while (!d3b::mbar_try_wait(addr, parity))
    if (d3b::globaltimer_ns() - t0 > D3B_WAIT_LIMIT_NS) break;
}

namespace gdc {

constexpr int KD = 128;             // K = V = 128
constexpr int M = 128;              // two blocks of up to 64 tokens
constexpr int THREADS = 256;          // row phases: two threads per row (64 columns each)
constexpr int CHUNK = M * 128;      // one [128 rows x 64 bf16] 128B-swizzled chunk
constexpr int TILE = 2 * CHUNK;     // a [128 x 128] bf16 operand tile
constexpr int OFF_KN = 0, OFF_QN = TILE, OFF_S0 = 2 * TILE, OFF_P = 3 * TILE, OFF_V = 4 * TILE;
constexpr int R_STRIDE = 132;       // fp32 row stride of R (conflict-free row writes)
constexpr int A_STRIDE = 68;        // fp32 row stride of A
constexpr int OFF_R = 0;            // aliases the K/Q/S0 tiles once their products are done
constexpr int OFF_A = 5 * TILE;
constexpr int SMEM_BYTES = OFF_A + M * A_STRIDE * 4 + 1024;
constexpr int V_STAGE = 272;        // staged v row stride (bytes): 128 rows fit the A region
constexpr int O_STAGE = 272;        // staged output row stride (bytes)
constexpr uint32_t TMEM_COLS = 512;
constexpr int COL_KK = 0, COL_KS = 128, COL_QK = 256, COL_QS = 384, COL_PV = 0;

enum : int { kSiteChunkMma1 = 3001, kSiteChunkMma2 = 3002, kSiteChunkDrain = 3003, kSiteChunkLoad = 3004 };

// Byte offset of element (r, c) of a [128 x 128] bf16 tile held as two [128 x 64]
// chunks in the 128B-swizzle layout (16-byte granule index XOR row % 8); for a
// K-major operand r is the M/N row and c the K index, for an MN-major one r is the
// K index and c the N column.
__device__ __forceinline__ uint32_t sw_off(int r, int c) {
  return (uint32_t)((c >> 6) * CHUNK + r * 128 + ((((c & 63) >> 3) ^ (r & 7)) << 4) + (c & 7) * 2);
}

struct Bars {
  uint64_t load, mma1, mma2, drain;
  uint32_t tmem_slot;
  int abort_flag;
  float gam[M];   // running sum of g within each block
  float beta[M];
};

template <typename In>
__device__ __forceinline__ uint32_t pack2(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

template <typename In>
__device__ __forceinline__ void unpack8(const uint4& u, float* f) {
  const In* h = reinterpret_cast<const In*>(&u);
#pragma unroll
  for (int e = 0; e < 8; ++e) f[e] = to_f32(h[e]);
}

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   d3b::smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(d3b::smem_u32(bar))
               : "memory");
}

// The initial state of each value head as the bf16 MN-major operand tile the chunk
// kernel copies into shared memory with one bulk copy (the shared image of S0).
__global__ void __launch_bounds__(THREADS) s0_tiles_kernel(const float* h0, long long s_hv, long long s_row,
                                                           uint8_t* tiles) {
  const int hv = blockIdx.x, row = threadIdx.x & (M - 1), c0 = (threadIdx.x >> 7) * 64;
  const float* src = h0 + hv * s_hv + row * s_row + c0;
  uint8_t* tile = tiles + (size_t)hv * TILE;
#pragma unroll
  for (int x = 0; x < 8; ++x) {
    const float4 a = reinterpret_cast<const float4*>(src)[2 * x];
    const float4 z = reinterpret_cast<const float4*>(src)[2 * x + 1];
    *reinterpret_cast<uint4*>(tile + sw_off(row, c0 + x * 8)) =
        make_uint4(pack2<__nv_bfloat16>(a.x, a.y), pack2<__nv_bfloat16>(a.z, a.w), pack2<__nv_bfloat16>(z.x, z.y),
                   pack2<__nv_bfloat16>(z.z, z.w));
  }
}

template <typename In, typename BetaT>
__global__ void __launch_bounds__(THREADS, 1) gdr_chunk_kernel(const __grid_constant__ GdrParams p,
                                                             const uint8_t* s0_tiles, int* err) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ Bars bars;
  __shared__ float part[2][2][M];  // [q, k][column half][row] partial sums of squares
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5;
  const int row = tid & (M - 1), half = tid >> 7;  // row phases: one row, 64 of its 128 columns
  const int blk = row >> 6, tl = row & 63;  // the row's token tl of block blk
  volatile int* abort_flag = &bars.abort_flag;
  const int c0 = half * 64;
  const int npairs = (p.B + 1) / 2, n_items = npairs * p.HV;

  if (tid == 0) {
    d3b::mbar_init(&bars.load, THREADS);
    d3b::mbar_init(&bars.mma1, 1);
    d3b::mbar_init(&bars.mma2, 1);
    d3b::mbar_init(&bars.drain, 1);
    bars.abort_flag = 0;
    d3b::fence_barrier_init();
  }
  // persistent: TMEM and the barriers are set up once; each iteration is one work item
  // (two blocks x one value head) and flips the barriers' phase
  if (warp == 0) d3b::tmem_alloc(&bars.tmem_slot, TMEM_COLS);
  d3b::tc_fence_before();
  __syncthreads();
  d3b::tc_fence_after();
  const uint32_t tmem = bars.tmem_slot;
  const uint32_t s_base = d3b::smem_u32(smem);
  bool alive = true;
#pragma unroll 1
  for (int item = blockIdx.x, it = 0; item < n_items && alive; item += gridDim.x, ++it) {
  const uint32_t ph = (uint32_t)it & 1u;
  const int hv = item / npairs, h = hv / (p.HV / p.H);
  const int b = (item % npairs) * 2 + blk;
  const bool valid = b < p.B && tl < p.T;
  // ---- phase 1: q, k, v rows and the head's S0 tile arrive by bulk copies on one
  // mbarrier (one arrival per thread, each with the bytes it copies); g -> gamma, beta
  // raw rows: q and k at 256 B per row (read back with a row-rotated granule order, so
  // the 8 rows a quarter-warp reads hit 8 different bank groups), v at 272 B per row
  uint8_t* stage_q = smem + OFF_P;  // free until the P tile is written
  uint8_t* stage_k = smem + OFF_V;  // free until V' is written
  uint8_t* stage_v = smem + OFF_A;  // free until A is written (after R is formed)
  if (!s0_tiles) {  // no initial state: a zero S0 tile
#pragma unroll
    for (int x = 0; x < TILE / 16 / THREADS; ++x)
      reinterpret_cast<uint4*>(smem + OFF_S0)[x * THREADS + tid] = make_uint4(0, 0, 0, 0);
  }
  if (half == 0 && !valid) {  // padding rows: zeros, so every product and R stay finite there
#pragma unroll
    for (int x = 0; x < 16; ++x) {
      reinterpret_cast<uint4*>(stage_q + row * 256)[x] = make_uint4(0, 0, 0, 0);
      reinterpret_cast<uint4*>(stage_k + row * 256)[x] = make_uint4(0, 0, 0, 0);
      reinterpret_cast<uint4*>(stage_v + row * V_STAGE)[x] = make_uint4(0, 0, 0, 0);
    }
  }
  __syncthreads();  // barrier init visible; the previous item's shared-memory users are done
  d3b::fence_proxy_async_smem();  // generic writes of the previous item before this item's bulk copies
  if (half == 0 && valid) {
    d3b::mbar_arrive_expect_tx(&bars.load, 3 * 256);
    bulk_load(stage_q + row * 256, static_cast<const In*>(p.q) + b * p.qs[0] + (long long)tl * p.qs[1] + h * p.qs[2],
              256, &bars.load);
    bulk_load(stage_k + row * 256, static_cast<const In*>(p.k) + b * p.ks[0] + (long long)tl * p.ks[1] + h * p.ks[2],
              256, &bars.load);
    bulk_load(stage_v + row * V_STAGE,
              static_cast<const In*>(p.v) + b * p.vs[0] + (long long)tl * p.vs[1] + hv * p.vs[2], 256, &bars.load);
  } else if (tid == THREADS - 1 && s0_tiles) {
    d3b::mbar_arrive_expect_tx(&bars.load, TILE);
    bulk_load(smem + OFF_S0, s0_tiles + (size_t)hv * TILE, TILE / 2, &bars.load);
    bulk_load(smem + OFF_S0 + TILE / 2, s0_tiles + (size_t)hv * TILE + TILE / 2, TILE / 2, &bars.load);
  } else {
    d3b::mbar_arrive(&bars.load);
  }
  if (half == 0) {
    bars.gam[row] = valid ? p.g[b * p.gs[0] + (long long)tl * p.gs[1] + hv * p.gs[2]] : 0.f;
    bars.beta[row] = valid ? to_f32(static_cast<const BetaT*>(p.beta)[b * p.bs[0] + (long long)tl * p.bs[1] +
                                                                       hv * p.bs[2]])
                           : 0.f;
  }
  bool ok = d3b::warp_wait(&bars.load, ph, abort_flag, err, kSiteChunkLoad);
  uint4 rq[8], rk[8];  // rq[x] holds columns c0 + gx(x) * 8 .. + 7
  auto gx = [&](int x) { return (x + row) & 7; };
#pragma unroll
  for (int x = 0; x < 8; ++x) {
    rq[x] = reinterpret_cast<const uint4*>(stage_q + row * 256 + half * 128)[gx(x)];
    rk[x] = reinterpret_cast<const uint4*>(stage_k + row * 256 + half * 128)[gx(x)];
  }
  {
    float sq = 0.f, sk = 0.f;
#pragma unroll
    for (int x = 0; x < 8; ++x) {
      float fq[8], fk[8];
      unpack8<In>(rq[x], fq);
      unpack8<In>(rk[x], fk);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        sq = fmaf(fq[e], fq[e], sq);
        sk = fmaf(fk[e], fk[e], sk);
      }
    }
    part[0][half][row] = sq;
    part[1][half][row] = sk;
  }
  __syncthreads();
  float gam = 0.f;
  for (int s = blk * 64; s <= row; ++s) gam += bars.gam[s];
  {
    const float sq = part[0][0][row] + part[0][1][row], sk = part[1][0][row] + part[1][1][row];
    const float iq = (p.l2norm ? 1.f / sqrtf(sq + 1e-6f) : 1.f) * p.scale;
    const float ik = p.l2norm ? 1.f / sqrtf(sk + 1e-6f) : 1.f;
#pragma unroll
    for (int x = 0; x < 8; ++x) {
      float fq[8], fk[8];
      unpack8<In>(rq[x], fq);
      unpack8<In>(rk[x], fk);
      *reinterpret_cast<uint4*>(smem + OFF_QN + sw_off(row, c0 + gx(x) * 8)) =
          make_uint4(pack2<__nv_bfloat16>(fq[0] * iq, fq[1] * iq), pack2<__nv_bfloat16>(fq[2] * iq, fq[3] * iq),
                     pack2<__nv_bfloat16>(fq[4] * iq, fq[5] * iq), pack2<__nv_bfloat16>(fq[6] * iq, fq[7] * iq));
      *reinterpret_cast<uint4*>(smem + OFF_KN + sw_off(row, c0 + gx(x) * 8)) =
          make_uint4(pack2<__nv_bfloat16>(fk[0] * ik, fk[1] * ik), pack2<__nv_bfloat16>(fk[2] * ik, fk[3] * ik),
                     pack2<__nv_bfloat16>(fk[4] * ik, fk[5] * ik), pack2<__nv_bfloat16>(fk[6] * ik, fk[7] * ik));
    }
  }
  __syncthreads();  // every thread has read the raw g values
  if (half == 0) bars.gam[row] = gam;
  d3b::fence_proxy_async_smem();
  d3b::tc_fence_before();
  __syncthreads();
  d3b::tc_fence_after();

  // ---- phase 2: K K^T, K S0, Q K^T, Q S0 -------------------------------------
  if (tid == 0 && ok) {
    constexpr uint32_t id_kk = d3b::make_idesc(1, 1, 1, 0, 0, M, KD);  // both K-major
    constexpr uint32_t id_ks = d3b::make_idesc(1, 1, 1, 0, 1, M, KD);  // B (S0) MN-major
#pragma unroll
    for (int k = 0; k < KD / 16; ++k) {
      const uint32_t koff = (uint32_t)((k >> 2) * CHUNK + (k & 3) * 32);
      const uint64_t a_k = d3b::make_smem_desc(s_base + OFF_KN + koff, 16, 1024, d3b::kLayoutSW128);
      const uint64_t a_q = d3b::make_smem_desc(s_base + OFF_QN + koff, 16, 1024, d3b::kLayoutSW128);
      const uint64_t b_s = d3b::make_smem_desc(s_base + OFF_S0 + k * 16 * 128, CHUNK, 1024, d3b::kLayoutSW128);
      d3b::mma_f16_ss(tmem + COL_KK, a_k, a_k, id_kk, k > 0);
      d3b::mma_f16_ss(tmem + COL_KS, a_k, b_s, id_ks, k > 0);
      d3b::mma_f16_ss(tmem + COL_QK, a_q, a_k, id_kk, k > 0);
      d3b::mma_f16_ss(tmem + COL_QS, a_q, b_s, id_ks, k > 0);
    }
    d3b::mma_commit(&bars.mma1);
  }
  if (ok) ok = d3b::warp_wait(&bars.mma1, ph, abort_flag, err, kSiteChunkMma1);
  d3b::tc_fence_after();

  // ---- phase 3 (row, column half): A, P, R -------------------------------------
  float* Rm = reinterpret_cast<float*>(smem + OFF_R);
  float* Am = reinterpret_cast<float*>(smem + OFF_A);
  const uint32_t lane_addr = tmem + ((uint32_t)((warp & 3) * 32) << 16);
  if (ok) {
    const float beta_i = bars.beta[row];
    const float eg = __expf(gam);
    uint32_t r[32];
#pragma unroll 1
    for (int q2 = 0; q2 < 2; ++q2) {
      const int j0 = c0 + q2 * 32;
      d3b::tmem_ld32(lane_addr + COL_KS + j0, r);
      d3b::tmem_wait_ld();
#pragma unroll
      for (int x = 0; x < 32; x += 8) {
        float fv[8];
        unpack8<In>(*reinterpret_cast<const uint4*>(stage_v + row * V_STAGE + (j0 + x) * 2), fv);
        float4 r0, r1;
        r0.x = beta_i * (fv[0] - eg * __uint_as_float(r[x + 0]));
        r0.y = beta_i * (fv[1] - eg * __uint_as_float(r[x + 1]));
        r0.z = beta_i * (fv[2] - eg * __uint_as_float(r[x + 2]));
        r0.w = beta_i * (fv[3] - eg * __uint_as_float(r[x + 3]));
        r1.x = beta_i * (fv[4] - eg * __uint_as_float(r[x + 4]));
        r1.y = beta_i * (fv[5] - eg * __uint_as_float(r[x + 5]));
        r1.z = beta_i * (fv[6] - eg * __uint_as_float(r[x + 6]));
        r1.w = beta_i * (fv[7] - eg * __uint_as_float(r[x + 7]));
        *reinterpret_cast<float4*>(Rm + row * R_STRIDE + j0 + x) = r0;
        *reinterpret_cast<float4*>(Rm + row * R_STRIDE + j0 + x + 4) = r1;
      }
    }
  }
  __syncthreads();  // R is formed: the staged v rows (A region) are consumed
  if (ok) {
    const float beta_i = bars.beta[row];
    uint32_t r[32];
    {  // A: 32 of the own block's 64 columns of K K^T
      const int jl0 = half * 32;
      d3b::tmem_ld32(lane_addr + COL_KK + blk * 64 + jl0, r);
      d3b::tmem_wait_ld();
      // stored transposed, Am[(blk * 64 + j) * A_STRIDE + i] = A[i][j]: the solve reads columns
#pragma unroll
      for (int x = 0; x < 32; ++x) {
        const int jl = jl0 + x;
        Am[(blk * 64 + jl) * A_STRIDE + tl] =
            jl < tl ? beta_i * __uint_as_float(r[x]) * __expf(gam - bars.gam[blk * 64 + jl]) : 0.f;
      }
    }
    // P: the decayed lower triangle (diagonal included) of Q K^T, zero off the own block.
    // A warp's 32 rows lie in one block, so a column half off that block is all zeros
    // (warp-uniform: no TMEM read there).
    if (half != blk) {
#pragma unroll
      for (int x = 0; x < 64; x += 8)
        *reinterpret_cast<uint4*>(smem + OFF_P + sw_off(row, c0 + x)) = make_uint4(0, 0, 0, 0);
    }
#pragma unroll 1
    for (int q2 = 0; q2 < 2 && half == blk; ++q2) {
      const int j0 = c0 + q2 * 32;
      d3b::tmem_ld32(lane_addr + COL_QK + j0, r);
      d3b::tmem_wait_ld();
#pragma unroll
      for (int x = 0; x < 32; x += 8) {
        float f[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int j = j0 + x + e;
          f[e] = (j & 63) <= tl ? __uint_as_float(r[x + e]) * __expf(gam - bars.gam[j]) : 0.f;
        }
        *reinterpret_cast<uint4*>(smem + OFF_P + sw_off(row, j0 + x)) =
            make_uint4(pack2<__nv_bfloat16>(f[0], f[1]), pack2<__nv_bfloat16>(f[2], f[3]),
                       pack2<__nv_bfloat16>(f[4], f[5]), pack2<__nv_bfloat16>(f[6], f[7]));
      }
    }
  }
  d3b::tc_fence_before();
  __syncthreads();  // R, A, P complete; the staged k rows are consumed (V' overwrites them)

  // ---- phase 4 (thread = state column c of block bk): V' = (I + A)^-1 R --------
  if (ok) {
    const int c = tid & (M - 1), bk = tid >> 7;
    // column-oriented forward substitution: once x[j] is final it updates every later
    // row at once, so the dependent chain is one FMA per row and the rest overlaps
    float x[64];
#pragma unroll
    for (int i = 0; i < 64; ++i) x[i] = Rm[(bk * 64 + i) * R_STRIDE + c];
#pragma unroll
    for (int j = 0; j < 63; ++j) {
      const float xj = x[j];
      const float* col = Am + (bk * 64 + j) * A_STRIDE;  // A[i][j], i = 0..63
#pragma unroll
      for (int i = j + 1; i < ((j + 4) & ~3) && i < 64; ++i) x[i] = fmaf(-col[i], xj, x[i]);
#pragma unroll
      for (int i = (j + 4) & ~3; i < 64; i += 4) {
        const float4 a4 = *reinterpret_cast<const float4*>(col + i);
        x[i] = fmaf(-a4.x, xj, x[i]);
        x[i + 1] = fmaf(-a4.y, xj, x[i + 1]);
        x[i + 2] = fmaf(-a4.z, xj, x[i + 2]);
        x[i + 3] = fmaf(-a4.w, xj, x[i + 3]);
      }
    }
#pragma unroll
    for (int i = 0; i < 64; ++i)
      *reinterpret_cast<__nv_bfloat16*>(smem + OFF_V + sw_off(bk * 64 + i, c)) = __float2bfloat16_rn(x[i]);
  }
  d3b::fence_proxy_async_smem();
  d3b::tc_fence_before();
  __syncthreads();
  d3b::tc_fence_after();

  // ---- phase 5: P V' into columns 0..127 --------------------------------------
  if (tid == 0 && ok) {
    constexpr uint32_t id_pv = d3b::make_idesc(1, 1, 1, 0, 1, M, KD);
#pragma unroll
    for (int k = 0; k < M / 16; ++k) {
      const uint32_t koff = (uint32_t)((k >> 2) * CHUNK + (k & 3) * 32);
      const uint64_t a_p = d3b::make_smem_desc(s_base + OFF_P + koff, 16, 1024, d3b::kLayoutSW128);
      const uint64_t b_v = d3b::make_smem_desc(s_base + OFF_V + k * 16 * 128, CHUNK, 1024, d3b::kLayoutSW128);
      d3b::mma_f16_ss(tmem + COL_PV, a_p, b_v, id_pv, k > 0);
    }
    d3b::mma_commit(&bars.mma2);
  }
  if (ok) ok = d3b::warp_wait(&bars.mma2, ph, abort_flag, err, kSiteChunkMma2);
  d3b::tc_fence_after();

  // ---- phase 6 (row, column half): O = e^gamma (Q S0) + P V' ------------------
  // Rows are gathered in shared memory (the dead K/Q/R space, 272 B per row so a warp's
  // rows hit different banks) and leave with one 256-byte bulk copy each.
  uint8_t* ostage = smem + OFF_KN;
  if (ok) {  // warp-uniform: every lane loads (tcgen05.ld is warp-collective)
    const float eg = __expf(gam);
    uint32_t rs[32], rp[32];
#pragma unroll 1
    for (int q2 = 0; q2 < 2; ++q2) {
      const int j0 = c0 + q2 * 32;
      d3b::tmem_ld32(lane_addr + COL_QS + j0, rs);
      d3b::tmem_ld32(lane_addr + COL_PV + j0, rp);
      d3b::tmem_wait_ld();
#pragma unroll
      for (int x = 0; x < 32; x += 8) {
        float f[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) f[e] = fmaf(eg, __uint_as_float(rs[x + e]), __uint_as_float(rp[x + e]));
        *reinterpret_cast<uint4*>(ostage + row * O_STAGE + (j0 + x) * 2) =
            make_uint4(pack2<In>(f[0], f[1]), pack2<In>(f[2], f[3]), pack2<In>(f[4], f[5]), pack2<In>(f[6], f[7]));
      }
    }
  }
  d3b::fence_proxy_async_smem();
  __syncthreads();
  if (ok && half == 0 && valid) {
    In* orow = static_cast<In*>(p.o) + b * p.os[0] + (long long)tl * p.os[1] + hv * p.os[2];
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], 256;" ::"l"(orow),
                 "r"(d3b::smem_u32(ostage + row * O_STAGE))
                 : "memory");
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");  // the staging rows may be reused
  }

  // every thread's TMEM reads and shared-memory uses of this item are done before the
  // next item's copies and products; a failed wait anywhere ends the loop for the CTA
  d3b::tc_fence_before();
  alive = __syncthreads_and(ok) != 0;
  d3b::tc_fence_after();
  if (!alive) settle(&bars.load, ph);  // no load copy of this item is left in flight
  }

  // ---- teardown: every issued MMA and output copy has completed ---------------
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
  if (tid == 0) {
    d3b::mma_commit(&bars.drain);
    const uint32_t addr = d3b::smem_u32(&bars.drain);
    const uint64_t t0 = d3b::globaltimer_ns();
    while (!d3b::mbar_try_wait(addr, 0)) {
      if (d3b::globaltimer_ns() - t0 > D3B_WAIT_LIMIT_NS) {
        d3b::record_device_error(err, kSiteChunkDrain);
        break;
      }
    }
  }
  d3b::tc_fence_before();
  __syncthreads();
  d3b::tc_fence_after();
  if (warp == 0) d3b::tmem_dealloc(tmem, TMEM_COLS);
}

}  // namespace gdc

template <typename In>
int launch_chunk(const GdrParams& p, int beta_dtype, uint8_t* s0_tiles, cudaStream_t s) {
  static int attr_set[64][3] = {{0}};
  const int dev = d3b_host::current_device();
  int* err = d3b_host::device_error_word();
  if (!err) return D3B_ECUDA;
  if (p.h0) {  // the shared initial state -> one bf16 operand tile per value head
    gdc::s0_tiles_kernel<<<p.HV, gdc::THREADS, 0, s>>>(p.h0, p.h0s[1], p.h0s[2], s0_tiles);
    if (const int st = d3b_host::check_launch()) return st;
  }
  const uint8_t* tiles = p.h0 ? s0_tiles : nullptr;
  const int n_items = ((p.B + 1) / 2) * p.HV;
  const dim3 grid((unsigned)std::min(n_items, d3b_host::num_sms(dev)));  // persistent, one CTA per SM
  auto go = [&](auto kernel, int which) -> int {
    if (dev >= 0 && dev < 64 && !attr_set[dev][which]) {
      if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, gdc::SMEM_BYTES) != cudaSuccess)
        return D3B_ECUDA;
      attr_set[dev][which] = 1;
    }
    kernel<<<grid, gdc::THREADS, gdc::SMEM_BYTES, s>>>(p, tiles, err);
    return d3b_host::check_launch();
  };
  switch (beta_dtype) {
    case D3B_F32: return go(gdc::gdr_chunk_kernel<In, float>, 0);
    case D3B_BF16: return go(gdc::gdr_chunk_kernel<In, __nv_bfloat16>, 1);
    case D3B_F16: return go(gdc::gdr_chunk_kernel<In, __half>, 2);
    default: return D3B_EUNSUPPORTED;
  }
}

// ---------------------------------------------------------------------------
// Chunked form for long sequences (the state pass: one row of thousands of
// tokens with a final state; FLA's chunk_gated_delta_rule, the reference's
// path for it, d3trt/model/ops.py:287-324). Chunks of 64 tokens; gamma is the
// running sum of g inside a chunk, gL its last value. WY form per chunk, with
// the state S_c entering the chunk:
//   A   = strictly-lower( beta_i (k_i . k_j) e^(gamma_i - gamma_j) ),  T = (I + A)^-1
//   W   = T diag(beta e^gamma) K,   U = T diag(beta) V                  (state-free)
//   V'  = U - W S_c
//   S_{c+1} = e^gL S_c + K^T diag(e^(gL - gamma)) V'
//   O   = e^gamma (Q S_c) + lower-incl( (q_i . k_j) e^(gamma_i - gamma_j) ) V'
// Two kernels. gdr_state_prep_kernel (parallel over row x chunk pair x value
// head, persistent) forms everything that does not depend on the state: the
// products K K^T and Q K^T, A, T (forward substitution, one thread per row of
// T), W and U (tcgen05, T as a block-diagonal A operand), and writes each
// chunk's operand tiles to a workspace in the exact shared-memory layouts the
// second kernel's MMAs read. gdr_state_scan_kernel (one CTA per row x value
// head x 64 state columns) carries the state through the chunks in fp32
// registers (one thread per state row); per chunk three tcgen05 products:
//   [W; Q] S_c (M = 128: rows 0-63 W, 64-127 Q)   K^T (e^(gL-gamma) V')   P V'
// with the chunk's tiles double-buffered by bulk copies. Numerics follow FLA's
// chunked kernels: bf16 operands (T, W, U, V', the state image), fp32
// accumulation, fp32 state.
// ---------------------------------------------------------------------------
namespace gds {

using gdc::CHUNK;
using gdc::KD;
using gdc::M;
using gdc::TILE;
using gdc::sw_off;

// ---- workspace: one record per (row, value head, chunk) ----
constexpr int WS_WQ = 0;       // [128 x 128] K-major SW128: rows 0-63 W, rows 64-127 q (normalised, scaled)
constexpr int WS_KH = 32768;   // k (normalised) as the MN-major [M = 128 state rows x K = 64 tokens] operand
constexpr int WS_P = 49152;    // P, [64 x 64] K-major SW128 (rows 64-127 of the scan's [128 x 64] operand)
constexpr int WS_U = 57344;    // U, two [64 tokens x 64 columns] halves, rows of 8 granules at g ^ (token % 8)
constexpr int WS_G = 73728;    // gamma, 64 floats
constexpr int WS_CHUNK = 74752;

// ---- prep kernel ----
constexpr int P_THREADS = 256;
constexpr int P_OFF_KN = 0, P_OFF_QN = TILE, P_OFF_KB = 2 * TILE, P_OFF_VB = 3 * TILE, P_OFF_T = 4 * TILE;
constexpr int P_OFF_P = 5 * TILE, P_OFF_A = 5 * TILE + 16384;
constexpr int P_A_STRIDE = 68;  // fp32 row stride of A (row-major)
constexpr int P_SMEM_BYTES = P_OFF_A + M * P_A_STRIDE * 4 + 1024;
constexpr uint32_t P_TMEM_COLS = 512;
constexpr int P_COL_KK = 0, P_COL_QK = 128, P_COL_W = 256, P_COL_U = 384;

enum : int { kSitePrepLoad = 3101, kSitePrepMma1 = 3102, kSitePrepMma2 = 3103, kSitePrepDrain = 3104,
             kSiteScanFull = 3111, kSiteScanH = 3112, kSiteScanX = 3113, kSiteScanV = 3114, kSiteScanHV = 3115,
             kSiteScanEmpty = 3116, kSiteScanDrain = 3117 };

struct PBars {
  uint64_t load, mma1, mma2, drain;
  uint32_t tmem_slot;
  int abort_flag;
  alignas(16) float gam[M];  // gamma per row (bulk-copied out per chunk: 16-byte aligned)
  float beta[M];
};

__device__ __forceinline__ uint4 pack8_bf16(const float* f) {
  return make_uint4(gdc::pack2<__nv_bfloat16>(f[0], f[1]), gdc::pack2<__nv_bfloat16>(f[2], f[3]),
                    gdc::pack2<__nv_bfloat16>(f[4], f[5]), gdc::pack2<__nv_bfloat16>(f[6], f[7]));
}

__device__ __forceinline__ void bulk_store(void* dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(d3b::smem_u32(src)),
               "r"(bytes)
               : "memory");
}


template <typename In, typename BetaT>
__global__ void __launch_bounds__(P_THREADS, 1)
    gdr_state_prep_kernel(const __grid_constant__ GdrParams p, uint8_t* ws, int NC, int* err) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ PBars bars;
  __shared__ float part[2][2][M];  // [q, k][column half][row] partial sums of squares
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5;
  const int row = tid & (M - 1), half = tid >> 7;  // row phases: one row, 64 of its 128 columns
  const int blk = row >> 6, tl = row & 63;        // the row's token tl of chunk blk of the pair
  volatile int* abort_flag = &bars.abort_flag;
  const int c0 = half * 64;
  const int npairs = (NC + 1) / 2, n_items = p.B * npairs * p.HV;

  if (tid == 0) {
    d3b::mbar_init(&bars.load, P_THREADS);
    d3b::mbar_init(&bars.mma1, 1);
    d3b::mbar_init(&bars.mma2, 1);
    d3b::mbar_init(&bars.drain, 1);
    bars.abort_flag = 0;
    d3b::fence_barrier_init();
  }
  if (warp == 0) d3b::tmem_alloc(&bars.tmem_slot, P_TMEM_COLS);
  d3b::tc_fence_before();
  __syncthreads();
  d3b::tc_fence_after();
  const uint32_t tmem = bars.tmem_slot;
  const uint32_t s_base = d3b::smem_u32(smem);
  const uint32_t lane_addr = tmem + ((uint32_t)((warp & 3) * 32) << 16);
  auto gx = [&](int x) { return (x + row) & 7; };  // row-rotated granule order (conflict-free row reads)
  bool alive = true;
  int it = 0;
#pragma unroll 1
  for (int item = blockIdx.x; item < n_items && alive; item += gridDim.x, ++it) {
    const uint32_t ph = (uint32_t)it & 1u;
    // value heads fastest: the items of one q/k head follow each other (q/k rows reused from L2)
    const int hv = item % p.HV, pair = (item / p.HV) % npairs, b = item / (p.HV * npairs);
    const int h = hv / (p.HV / p.H);
    const int chunk = pair * 2 + blk, tok = chunk * 64 + tl;
    const bool valid = tok < p.T;
    // ---- phase 1: raw q, k, v rows (256 B each) by bulk copies into the regions their
    // normalised tiles later take (every thread reads its row into registers first)
    uint8_t* stage_q = smem + P_OFF_QN;
    uint8_t* stage_k = smem + P_OFF_KN;
    uint8_t* stage_v = smem + P_OFF_VB;
    if (half == 0 && !valid) {  // padding rows: zeros (beta = g = 0: they add nothing)
#pragma unroll
      for (int x = 0; x < 16; ++x) {
        reinterpret_cast<uint4*>(stage_q + row * 256)[x] = make_uint4(0, 0, 0, 0);
        reinterpret_cast<uint4*>(stage_k + row * 256)[x] = make_uint4(0, 0, 0, 0);
        reinterpret_cast<uint4*>(stage_v + row * 256)[x] = make_uint4(0, 0, 0, 0);
      }
    }
    __syncthreads();  // the previous item's shared-memory users (and its copies out) are done
    d3b::fence_proxy_async_smem();
    if (half == 0 && valid) {
      d3b::mbar_arrive_expect_tx(&bars.load, 3 * 256);
      gdc::bulk_load(stage_q + row * 256,
                     static_cast<const In*>(p.q) + b * p.qs[0] + (long long)tok * p.qs[1] + h * p.qs[2], 256,
                     &bars.load);
      gdc::bulk_load(stage_k + row * 256,
                     static_cast<const In*>(p.k) + b * p.ks[0] + (long long)tok * p.ks[1] + h * p.ks[2], 256,
                     &bars.load);
      gdc::bulk_load(stage_v + row * 256,
                     static_cast<const In*>(p.v) + b * p.vs[0] + (long long)tok * p.vs[1] + hv * p.vs[2], 256,
                     &bars.load);
    } else {
      d3b::mbar_arrive(&bars.load);
    }
    if (half == 0) {
      bars.gam[row] = valid ? p.g[b * p.gs[0] + (long long)tok * p.gs[1] + hv * p.gs[2]] : 0.f;
      bars.beta[row] = valid ? to_f32(static_cast<const BetaT*>(p.beta)[b * p.bs[0] + (long long)tok * p.bs[1] +
                                                                       hv * p.bs[2]])
                             : 0.f;
    }
    bool ok = d3b::warp_wait(&bars.load, ph, abort_flag, err, kSitePrepLoad);
    uint4 rq[8], rk[8], rv[8];  // rq[x] holds columns c0 + gx(x) * 8 .. + 7
#pragma unroll
    for (int x = 0; x < 8; ++x) {
      rq[x] = reinterpret_cast<const uint4*>(stage_q + row * 256 + half * 128)[gx(x)];
      rk[x] = reinterpret_cast<const uint4*>(stage_k + row * 256 + half * 128)[gx(x)];
      rv[x] = reinterpret_cast<const uint4*>(stage_v + row * 256 + half * 128)[gx(x)];
    }
    {
      float sq = 0.f, sk = 0.f;
#pragma unroll
      for (int x = 0; x < 8; ++x) {
        float fq[8], fk[8];
        gdc::unpack8<In>(rq[x], fq);
        gdc::unpack8<In>(rk[x], fk);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          sq = fmaf(fq[e], fq[e], sq);
          sk = fmaf(fk[e], fk[e], sk);
        }
      }
      part[0][half][row] = sq;
      part[1][half][row] = sk;
    }
    __syncthreads();  // raw rows are in registers; partial sums and raw g visible
    float gam = 0.f;
    for (int s = blk * 64; s <= row; ++s) gam += bars.gam[s];
    const float sq = part[0][0][row] + part[0][1][row], sk = part[1][0][row] + part[1][1][row];
    const float iq = (p.l2norm ? 1.f / sqrtf(sq + 1e-6f) : 1.f) * p.scale;
    const float ik = p.l2norm ? 1.f / sqrtf(sk + 1e-6f) : 1.f;
    __syncthreads();  // every thread has read the raw g values
    if (half == 0) bars.gam[row] = gam;
    {
      const float bt = bars.beta[row], bte = bt * __expf(gam);
#pragma unroll
      for (int x = 0; x < 8; ++x) {
        float fq[8], fk[8], fv[8], kb[8], vb[8];
        gdc::unpack8<In>(rq[x], fq);
        gdc::unpack8<In>(rk[x], fk);
        gdc::unpack8<In>(rv[x], fv);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          fq[e] *= iq;
          fk[e] = __bfloat162float(__float2bfloat16_rn(fk[e] * ik));  // the bf16 k every product uses
          kb[e] = fk[e] * bte;
          vb[e] = fv[e] * bt;
        }
        const uint32_t off = sw_off(row, c0 + gx(x) * 8);
        *reinterpret_cast<uint4*>(smem + P_OFF_QN + off) = pack8_bf16(fq);
        *reinterpret_cast<uint4*>(smem + P_OFF_KN + off) = pack8_bf16(fk);
        *reinterpret_cast<uint4*>(smem + P_OFF_KB + off) = pack8_bf16(kb);
        *reinterpret_cast<uint4*>(smem + P_OFF_VB + off) = pack8_bf16(vb);
      }
    }
    d3b::fence_proxy_async_smem();
    d3b::tc_fence_before();
    __syncthreads();
    d3b::tc_fence_after();

    // ---- phase 2: K K^T, Q K^T ------------------------------------------------
    if (tid == 0 && ok) {
      constexpr uint32_t id_kk = d3b::make_idesc(1, 1, 1, 0, 0, M, KD);
#pragma unroll
      for (int k = 0; k < KD / 16; ++k) {
        const uint32_t koff = (uint32_t)((k >> 2) * CHUNK + (k & 3) * 32);
        const uint64_t a_k = d3b::make_smem_desc(s_base + P_OFF_KN + koff, 16, 1024, d3b::kLayoutSW128);
        const uint64_t a_q = d3b::make_smem_desc(s_base + P_OFF_QN + koff, 16, 1024, d3b::kLayoutSW128);
        d3b::mma_f16_ss(tmem + P_COL_KK, a_k, a_k, id_kk, k > 0);
        d3b::mma_f16_ss(tmem + P_COL_QK, a_q, a_k, id_kk, k > 0);
      }
      d3b::mma_commit(&bars.mma1);
    }
    if (ok) ok = d3b::warp_wait(&bars.mma1, ph, abort_flag, err, kSitePrepMma1);
    d3b::tc_fence_after();

    // ---- phase 3 (row, column half of the own chunk): A (row-major fp32) and P (bf16) --
    float* Am = reinterpret_cast<float*>(smem + P_OFF_A);
    if (ok) {
      const float beta_i = bars.beta[row];
      const int jl0 = half * 32;
      uint32_t r[32];
      d3b::tmem_ld32(lane_addr + P_COL_KK + blk * 64 + jl0, r);
      d3b::tmem_wait_ld();
#pragma unroll
      for (int x = 0; x < 32; x += 4) {
        float4 a4;
        float* af = reinterpret_cast<float*>(&a4);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int jl = jl0 + x + e;
          af[e] = jl < tl ? beta_i * __uint_as_float(r[x + e]) * __expf(gam - bars.gam[blk * 64 + jl]) : 0.f;
        }
        *reinterpret_cast<float4*>(Am + row * P_A_STRIDE + jl0 + x) = a4;
      }
      d3b::tmem_ld32(lane_addr + P_COL_QK + blk * 64 + jl0, r);
      d3b::tmem_wait_ld();
#pragma unroll
      for (int x = 0; x < 32; x += 8) {
        float f[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int jl = jl0 + x + e;
          f[e] = jl <= tl ? __uint_as_float(r[x + e]) * __expf(gam - bars.gam[blk * 64 + jl]) : 0.f;
        }
        const int g8 = (jl0 + x) >> 3;
        *reinterpret_cast<uint4*>(smem + P_OFF_P + row * 128 + ((g8 ^ (row & 7)) << 4)) = pack8_bf16(f);
      }
    }
    __syncthreads();  // A and P complete

    // ---- phase 4: T = (I + A)^-1, one thread per row of T (threads 0-127) ----------
    // Row i of T solves x (I + A) = e_i from the right: going down from m = 63, x_m
    // is final once every later row has been subtracted, then x_j -= x_m A[m][j]
    // for j < m. Every thread runs the same unrolled steps (rows m > i give x_m = 0),
    // so all lanes read the same A row at the same time (a broadcast).
    if (ok && tid < M) {
      float x[64];
#pragma unroll
      for (int m = 0; m < 64; ++m) x[m] = m == tl ? 1.f : 0.f;
      const float* Ab = Am + blk * 64 * P_A_STRIDE;
#pragma unroll
      for (int m = 63; m >= 1; --m) {
        const float xm = x[m];
        const float* arow = Ab + m * P_A_STRIDE;
#pragma unroll
        for (int j = 0; j < (m & ~3); j += 4) {
          const float4 a4 = *reinterpret_cast<const float4*>(arow + j);
          x[j] = fmaf(-a4.x, xm, x[j]);
          x[j + 1] = fmaf(-a4.y, xm, x[j + 1]);
          x[j + 2] = fmaf(-a4.z, xm, x[j + 2]);
          x[j + 3] = fmaf(-a4.w, xm, x[j + 3]);
        }
#pragma unroll
        for (int j = m & ~3; j < m; ++j) x[j] = fmaf(-arow[j], xm, x[j]);
      }
#pragma unroll
      for (int x8 = 0; x8 < 8; ++x8)
        *reinterpret_cast<uint4*>(smem + P_OFF_T + sw_off(row, blk * 64 + x8 * 8)) = pack8_bf16(x + x8 * 8);
    } else if (ok) {
      // T is block-diagonal: zeros in the other chunk's 64 columns of row tid - 128
      const int r2 = tid - M, ob = 1 - (r2 >> 6);
#pragma unroll
      for (int x8 = 0; x8 < 8; ++x8)
        *reinterpret_cast<uint4*>(smem + P_OFF_T + sw_off(r2, ob * 64 + x8 * 8)) = make_uint4(0, 0, 0, 0);
    }
    d3b::fence_proxy_async_smem();
    d3b::tc_fence_before();
    __syncthreads();
    d3b::tc_fence_after();

    // ---- phase 5: W = T (beta e^gamma K), U = T (beta V) -------------------------
    if (tid == 0 && ok) {
      constexpr uint32_t id_w = d3b::make_idesc(1, 1, 1, 0, 1, M, KD);  // B MN-major
#pragma unroll
      for (int k = 0; k < M / 16; ++k) {
        const uint32_t koff = (uint32_t)((k >> 2) * CHUNK + (k & 3) * 32);
        const uint64_t a_t = d3b::make_smem_desc(s_base + P_OFF_T + koff, 16, 1024, d3b::kLayoutSW128);
        const uint64_t b_k = d3b::make_smem_desc(s_base + P_OFF_KB + k * 16 * 128, CHUNK, 1024, d3b::kLayoutSW128);
        const uint64_t b_v = d3b::make_smem_desc(s_base + P_OFF_VB + k * 16 * 128, CHUNK, 1024, d3b::kLayoutSW128);
        d3b::mma_f16_ss(tmem + P_COL_W, a_t, b_k, id_w, k > 0);
        d3b::mma_f16_ss(tmem + P_COL_U, a_t, b_v, id_w, k > 0);
      }
      d3b::mma_commit(&bars.mma2);
    }
    if (ok) ok = d3b::warp_wait(&bars.mma2, ph, abort_flag, err, kSitePrepMma2);
    d3b::tc_fence_after();

    // ---- phase 6 (row, column half): W as bf16 into the dead KB tile (K-major), U as
    // bf16 rows into the dead VB tile ([chunk][column half][token][64]) -----------
    if (ok) {
      uint32_t r[64];
      d3b::tmem_ld32(lane_addr + P_COL_W + c0, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
      d3b::tmem_ld32(lane_addr + P_COL_W + c0 + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
      d3b::tmem_wait_ld();
#pragma unroll
      for (int x = 0; x < 8; ++x) {
        float f[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) f[e] = __uint_as_float(r[x * 8 + e]);
        *reinterpret_cast<uint4*>(smem + P_OFF_KB + sw_off(row, c0 + x * 8)) = pack8_bf16(f);
      }
      d3b::tmem_ld32(lane_addr + P_COL_U + c0, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
      d3b::tmem_ld32(lane_addr + P_COL_U + c0 + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
      d3b::tmem_wait_ld();
      uint8_t* urow = smem + P_OFF_VB + ((blk * 2 + half) * 64 + tl) * 128;
#pragma unroll
      for (int x = 0; x < 8; ++x) {  // granule x of the row at x ^ (token % 8): conflict-free on both sides
        float f[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) f[e] = __uint_as_float(r[x * 8 + e]);
        *reinterpret_cast<uint4*>(urow + ((x ^ (tl & 7)) << 4)) = pack8_bf16(f);
      }
    }
    d3b::fence_proxy_async_smem();
    __syncthreads();
    // ---- copies out: ten per chunk, one per thread --------------------------------
    if (ok && tid < 20) {
      const int cb = tid / 10, which = tid % 10;
      const int chunk_c = pair * 2 + cb;
      if (chunk_c < NC) {
        uint8_t* dst = ws + (((size_t)b * p.HV + hv) * NC + chunk_c) * WS_CHUNK;
        const uint8_t* src = nullptr;
        uint32_t bytes = 8192;
        switch (which) {
          case 0: dst += WS_WQ; src = smem + P_OFF_KB + cb * 8192; break;                     // W, columns 0-63
          case 1: dst += WS_WQ + 8192; src = smem + P_OFF_QN + cb * 8192; break;              // q, columns 0-63
          case 2: dst += WS_WQ + 16384; src = smem + P_OFF_KB + CHUNK + cb * 8192; break;     // W, columns 64-127
          case 3: dst += WS_WQ + 24576; src = smem + P_OFF_QN + CHUNK + cb * 8192; break;     // q, columns 64-127
          case 4: dst += WS_KH; src = smem + P_OFF_KN + cb * 8192; break;                     // k, state rows 0-63
          case 5: dst += WS_KH + 8192; src = smem + P_OFF_KN + CHUNK + cb * 8192; break;      // k, state rows 64-127
          case 6: dst += WS_P; src = smem + P_OFF_P + cb * 8192; break;
          case 7: dst += WS_U; src = smem + P_OFF_VB + (cb * 2) * 8192; break;
          case 8: dst += WS_U + 8192; src = smem + P_OFF_VB + (cb * 2 + 1) * 8192; break;
          default: dst += WS_G; src = reinterpret_cast<const uint8_t*>(&bars.gam[cb * 64]); bytes = 256; break;
        }
        bulk_store(dst, src, bytes);
        asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");  // the staging may be reused
      }
    }
    d3b::tc_fence_before();
    alive = __syncthreads_and(ok) != 0;
    d3b::tc_fence_after();
    if (!alive) settle(&bars.load, ph);  // no load copy of this item is left in flight
  }

  // ---- teardown: every copy out and every MMA has completed -------------------
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
  if (tid == 0) {
    d3b::mma_commit(&bars.drain);
    const uint32_t addr = d3b::smem_u32(&bars.drain);
    const uint64_t t0 = d3b::globaltimer_ns();
    while (!d3b::mbar_try_wait(addr, 0)) {
      if (d3b::globaltimer_ns() - t0 > D3B_WAIT_LIMIT_NS) {
        d3b::record_device_error(err, kSitePrepDrain);
        break;
      }
    }
  }
  d3b::tc_fence_before();
  __syncthreads();
  d3b::tc_fence_after();
  if (warp == 0) d3b::tmem_dealloc(tmem, P_TMEM_COLS);
}

// ---- scan kernel ----
constexpr int R_THREADS = 192;  // warps 0-3: state rows (TMEM lanes 0-127); warp 4: copies; warp 5: MMAs
constexpr int R_VC = 64;        // state columns per CTA
constexpr int ST_WQ = 0, ST_KH = 32768, ST_PZ = 49152, ST_U = 65536, ST_G = 73728, R_STAGE = 74752;
constexpr int R_OFF_HB = 2 * R_STAGE, R_OFF_VB = R_OFF_HB + 16384, R_OFF_VD = R_OFF_VB + 8192;
constexpr int R_SMEM_BYTES = R_OFF_VD + 8192 + 1024;
constexpr uint32_t R_STAGE_TX = 32768 + 16384 + 8192 + 8192 + 256;
constexpr uint32_t R_TMEM_COLS = 256;
constexpr int R_COL_X = 0, R_COL_D = 64, R_COL_O = 128;

struct RBars {
  uint64_t full[2], empty[2];
  uint64_t h_ready;   // the state image of this chunk is in shared memory (128 row threads)
  uint64_t x_ready;   // [W; Q] S_c is in TMEM
  uint64_t v_ready;   // V' and its decayed copy are in shared memory (64 token threads)
  uint64_t hv_ready;  // K^T V'' and P V' are in TMEM; the state image and V' tiles are free
  uint64_t drain;
  uint32_t tmem_slot;
  int abort_flag;
};

template <typename In>
__global__ void __launch_bounds__(R_THREADS, 1)
    gdr_state_scan_kernel(const __grid_constant__ GdrParams p, const uint8_t* ws, int NC, int* err) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ RBars bars;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int half = (int)(blockIdx.x & 1), bh = (int)(blockIdx.x >> 1);
  const int hv = bh % p.HV, b = bh / p.HV;
  const int c0 = half * R_VC;
  const uint8_t* wsh = ws + ((size_t)b * p.HV + hv) * (size_t)NC * WS_CHUNK;
  volatile int* abort_flag = &bars.abort_flag;
  if (tid == 0) {
    for (int s = 0; s < 2; ++s) {
      d3b::mbar_init(&bars.full[s], 1);
      d3b::mbar_init(&bars.empty[s], 1);
    }
    d3b::mbar_init(&bars.h_ready, 128);
    d3b::mbar_init(&bars.x_ready, 1);
    d3b::mbar_init(&bars.v_ready, 64);
    d3b::mbar_init(&bars.hv_ready, 1);
    d3b::mbar_init(&bars.drain, 1);
    bars.abort_flag = 0;
    d3b::fence_barrier_init();
  }
  // rows 0-63 of each stage's P operand stay zero (rows 64-127 are P)
  for (int i = tid; i < 2 * 512; i += R_THREADS)
    reinterpret_cast<uint4*>(smem + (i >> 9) * R_STAGE + ST_PZ)[i & 511] = make_uint4(0, 0, 0, 0);
  d3b::fence_proxy_async_smem();
  if (warp == 5) d3b::tmem_alloc(&bars.tmem_slot, R_TMEM_COLS);
  d3b::tc_fence_before();
  __syncthreads();
  d3b::tc_fence_after();
  const uint32_t tmem = bars.tmem_slot;
  const uint32_t s_base = d3b::smem_u32(smem);

  if (warp == 4) {
    // ================= copies: chunk c's tiles into stage c % 2 =================
    if (lane == 0) {
      int c = 0;
      for (; c < NC; ++c) {
        const int s = c & 1;
        if (!d3b::mbar_wait(&bars.empty[s], ((uint32_t)(c >> 1) & 1) ^ 1, abort_flag, err, kSiteScanEmpty)) break;
        uint8_t* st = smem + s * R_STAGE;
        const uint8_t* src = wsh + (size_t)c * WS_CHUNK;
        d3b::mbar_arrive_expect_tx(&bars.full[s], R_STAGE_TX);
        gdc::bulk_load(st + ST_WQ, src + WS_WQ, 32768, &bars.full[s]);
        gdc::bulk_load(st + ST_KH, src + WS_KH, 16384, &bars.full[s]);
        gdc::bulk_load(st + ST_PZ + 8192, src + WS_P, 8192, &bars.full[s]);
        gdc::bulk_load(st + ST_U, src + WS_U + half * 8192, 8192, &bars.full[s]);
        gdc::bulk_load(st + ST_G, src + WS_G, 256, &bars.full[s]);
      }
      // the last two stages' copies have landed before the CTA can leave (after an abort too)
      for (int cc = c - 2 < 0 ? 0 : c - 2; cc < c; ++cc) settle(&bars.full[cc & 1], (uint32_t)(cc >> 1) & 1);
    }
  } else if (warp == 5) {
    // ================= MMA issuer =================
    if (lane == 0) {
      constexpr uint32_t id_x = d3b::make_idesc(1, 1, 1, 0, 1, M, R_VC);  // [W; Q] K-major, S image MN-major
      constexpr uint32_t id_d = d3b::make_idesc(1, 1, 1, 1, 1, M, R_VC);  // K^T: A MN-major
      constexpr uint32_t id_o = d3b::make_idesc(1, 1, 1, 0, 1, M, R_VC);  // [0; P] K-major
      for (int c = 0; c < NC; ++c) {
        const int s = c & 1;
        const uint32_t pc = (uint32_t)c & 1;
        const uint32_t st = s_base + s * R_STAGE;
        if (!d3b::mbar_wait(&bars.full[s], (uint32_t)(c >> 1) & 1, abort_flag, err, kSiteScanFull)) break;
        if (!d3b::mbar_wait(&bars.h_ready, pc, abort_flag, err, kSiteScanH)) break;
        d3b::tc_fence_after();
#pragma unroll
        for (int k = 0; k < KD / 16; ++k) {
          const uint64_t a = d3b::make_smem_desc(st + ST_WQ + (k >> 2) * CHUNK + (k & 3) * 32, 16, 1024,
                                                 d3b::kLayoutSW128);
          const uint64_t bd = d3b::make_smem_desc(s_base + R_OFF_HB + k * 2048, 16384, 1024, d3b::kLayoutSW128);
          d3b::mma_f16_ss(tmem + R_COL_X, a, bd, id_x, k > 0);
        }
        d3b::mma_commit(&bars.x_ready);
        if (!d3b::mbar_wait(&bars.v_ready, pc, abort_flag, err, kSiteScanV)) break;
        d3b::tc_fence_after();
#pragma unroll
        for (int k = 0; k < 64 / 16; ++k) {
          const uint64_t a_k = d3b::make_smem_desc(st + ST_KH + k * 2048, 8192, 1024, d3b::kLayoutSW128);
          const uint64_t b_vd = d3b::make_smem_desc(s_base + R_OFF_VD + k * 2048, 8192, 1024, d3b::kLayoutSW128);
          d3b::mma_f16_ss(tmem + R_COL_D, a_k, b_vd, id_d, k > 0);
        }
#pragma unroll
        for (int k = 0; k < 64 / 16; ++k) {
          const uint64_t a_p = d3b::make_smem_desc(st + ST_PZ + k * 32, 16, 1024, d3b::kLayoutSW128);
          const uint64_t b_vb = d3b::make_smem_desc(s_base + R_OFF_VB + k * 2048, 8192, 1024, d3b::kLayoutSW128);
          d3b::mma_f16_ss(tmem + R_COL_O, a_p, b_vb, id_o, k > 0);
        }
        d3b::mma_commit(&bars.hv_ready);
        d3b::mma_commit(&bars.empty[s]);
      }
      d3b::mma_commit(&bars.drain);
      const uint32_t addr = d3b::smem_u32(&bars.drain);
      const uint64_t t0 = d3b::globaltimer_ns();
      while (!d3b::mbar_try_wait(addr, 0)) {
        if (d3b::globaltimer_ns() - t0 > D3B_WAIT_LIMIT_NS) {
          d3b::record_device_error(err, kSiteScanDrain);
          break;
        }
      }
    }
  } else {
    // ================= state rows (thread i = state row i = TMEM lane i) =================
    const int i = tid;
    const uint32_t lane_addr = tmem + ((uint32_t)(warp * 32) << 16);
    float hs[R_VC];
    if (p.h0) {
      const float* src = p.h0 + b * p.h0s[0] + hv * p.h0s[1] + (long long)i * p.h0s[2] + c0;
#pragma unroll
      for (int j = 0; j < R_VC; ++j) hs[j] = src[j];
    } else {
#pragma unroll
      for (int j = 0; j < R_VC; ++j) hs[j] = 0.f;
    }
    const int t = i & 63;  // warps 0-1: token t's V' row; warps 2-3: token t's output row
    bool ok = true;
    for (int c = 0; c < NC; ++c) {
      const int s = c & 1;
      const uint32_t pc = (uint32_t)c & 1;
      const uint8_t* st = smem + s * R_STAGE;
      if (!(ok = d3b::warp_wait(&bars.full[s], (uint32_t)(c >> 1) & 1, abort_flag, err, kSiteScanFull))) break;
      // the chunk's gammas, read before h_ready (after it the stage may be refilled)
      const float gl = reinterpret_cast<const float*>(st + ST_G)[63];
      const float gt = reinterpret_cast<const float*>(st + ST_G)[t];
      // the state image S_c (bf16, MN-major [K = state rows x N = 64 columns])
#pragma unroll
      for (int x8 = 0; x8 < 8; ++x8)
        *reinterpret_cast<uint4*>(smem + R_OFF_HB + i * 128 + ((x8 ^ (i & 7)) << 4)) = pack8_bf16(hs + x8 * 8);
      d3b::fence_proxy_async_smem();
      d3b::tc_fence_before();
      d3b::mbar_arrive(&bars.h_ready);
      if (!(ok = d3b::warp_wait(&bars.x_ready, pc, abort_flag, err, kSiteScanX))) break;
      d3b::tc_fence_after();
      if (warp < 2) {
        // V' = U - W S_c for token t; V'' = e^(gL - gamma_t) V' for the state update
        uint32_t xr[64];
        d3b::tmem_ld32(lane_addr + R_COL_X, *reinterpret_cast<uint32_t(*)[32]>(&xr[0]));
        d3b::tmem_ld32(lane_addr + R_COL_X + 32, *reinterpret_cast<uint32_t(*)[32]>(&xr[32]));
        d3b::tmem_wait_ld();
        const float dk = __expf(gl - gt);
#pragma unroll
        for (int x8 = 0; x8 < 8; ++x8) {
          const uint32_t off = t * 128 + ((x8 ^ (t & 7)) << 4);  // U rows arrive in the same swizzle
          float fu[8], vn[8], vd[8];
          gdc::unpack8<__nv_bfloat16>(*reinterpret_cast<const uint4*>(st + ST_U + off), fu);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            vn[e] = fu[e] - __uint_as_float(xr[x8 * 8 + e]);
            vd[e] = vn[e] * dk;
          }
          *reinterpret_cast<uint4*>(smem + R_OFF_VB + off) = pack8_bf16(vn);
          *reinterpret_cast<uint4*>(smem + R_OFF_VD + off) = pack8_bf16(vd);
        }
        d3b::fence_proxy_async_smem();
        d3b::tc_fence_before();
        d3b::mbar_arrive(&bars.v_ready);
      }
      if (!(ok = d3b::warp_wait(&bars.hv_ready, pc, abort_flag, err, kSiteScanHV))) break;
      d3b::tc_fence_after();
      const float eg = __expf(gl);
#pragma unroll
      for (int q2 = 0; q2 < 2; ++q2) {
        uint32_t d[32];
        d3b::tmem_ld32(lane_addr + R_COL_D + q2 * 32, d);
        d3b::tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; ++j) hs[q2 * 32 + j] = fmaf(eg, hs[q2 * 32 + j], __uint_as_float(d[j]));
      }
      if (warp >= 2) {
        // O = e^gamma_t (Q S_c) + (P V') for token t
        const int tok = c * 64 + t;
        const float eq = __expf(gt);
        In* orow = static_cast<In*>(p.o) + b * p.os[0] + (long long)tok * p.os[1] + hv * p.os[2] + c0;
#pragma unroll
        for (int q2 = 0; q2 < 2; ++q2) {
          uint32_t xq[32], xo[32];
          d3b::tmem_ld32(lane_addr + R_COL_X + q2 * 32, xq);
          d3b::tmem_ld32(lane_addr + R_COL_O + q2 * 32, xo);
          d3b::tmem_wait_ld();
          if (tok < p.T) {
#pragma unroll
            for (int x = 0; x < 32; x += 8) {
              float f[8];
#pragma unroll
              for (int e = 0; e < 8; ++e) f[e] = fmaf(eq, __uint_as_float(xq[x + e]), __uint_as_float(xo[x + e]));
              *reinterpret_cast<uint4*>(orow + q2 * 32 + x) =
                  make_uint4(gdc::pack2<In>(f[0], f[1]), gdc::pack2<In>(f[2], f[3]), gdc::pack2<In>(f[4], f[5]),
                             gdc::pack2<In>(f[6], f[7]));
            }
          }
        }
      }
      d3b::tc_fence_before();
    }
    if (ok && p.ht) {
      float* dst = p.ht + (((long long)b * p.HV + hv) * KD + i) * KD + c0;
#pragma unroll
      for (int j = 0; j < R_VC; j += 4) *reinterpret_cast<float4*>(dst + j) = make_float4(hs[j], hs[j + 1], hs[j + 2], hs[j + 3]);
    }
  }

  d3b::tc_fence_before();
  __syncthreads();
  d3b::tc_fence_after();
  if (warp == 5) d3b::tmem_dealloc(tmem, R_TMEM_COLS);
}

}  // namespace gds

size_t state_workspace_bytes(long long B, long long T, long long HV) {
  const long long NC = (T + 63) / 64;
  return (size_t)(B * HV * NC) * gds::WS_CHUNK;
}

template <typename In>
int launch_state(const GdrParams& p, int beta_dtype, uint8_t* ws, cudaStream_t s) {
  static int attr_set[64][4] = {{0}};
  const int dev = d3b_host::current_device();
  int* err = d3b_host::device_error_word();
  if (!err) return D3B_ECUDA;
  const int NC = (p.T + 63) / 64;
  const long long n_items = (long long)p.B * ((NC + 1) / 2) * p.HV;
  const dim3 grid_p((unsigned)std::min<long long>(n_items, d3b_host::num_sms(dev)));  // persistent
  auto set_smem = [&](auto kernel, int which, int bytes) -> bool {
    if (dev >= 0 && dev < 64 && !attr_set[dev][which]) {
      if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess)
        return false;
      attr_set[dev][which] = 1;
    }
    return true;
  };
  auto prep = [&](auto kernel, int which) -> int {
    if (!set_smem(kernel, which, gds::P_SMEM_BYTES)) return D3B_ECUDA;
    kernel<<<grid_p, gds::P_THREADS, gds::P_SMEM_BYTES, s>>>(p, ws, NC, err);
    return d3b_host::check_launch();
  };
  int st;
  switch (beta_dtype) {
    case D3B_F32: st = prep(gds::gdr_state_prep_kernel<In, float>, 0); break;
    case D3B_BF16: st = prep(gds::gdr_state_prep_kernel<In, __nv_bfloat16>, 1); break;
    case D3B_F16: st = prep(gds::gdr_state_prep_kernel<In, __half>, 2); break;
    default: return D3B_EUNSUPPORTED;
  }
  if (st) return st;
  if (!set_smem(gds::gdr_state_scan_kernel<In>, 3, gds::R_SMEM_BYTES)) return D3B_ECUDA;
  gds::gdr_state_scan_kernel<In><<<(unsigned)(2LL * p.B * p.HV), gds::R_THREADS, gds::R_SMEM_BYTES, s>>>(p, ws, NC, err);
  return d3b_host::check_launch();
}

bool aligned(const void* ptr, int bytes) { return reinterpret_cast<uintptr_t>(ptr) % bytes == 0; }

}  // namespace

extern "C" size_t d3b_gated_delta_workspace_size(int HV, int K, int V) {
  return (HV > 0 && K == 128 && V == 128) ? (size_t)HV * gdc::TILE : 0;
}

extern "C" size_t d3b_gated_delta_state_workspace_size(int B, int T, int HV, int K, int V) {
  return (B > 0 && T > 0 && HV > 0 && K == 128 && V == 128) ? state_workspace_bytes(B, T, HV) : 0;
}

extern "C" int d3b_gated_delta_rule(const void* q, const int64_t* q_strides, const void* k, const int64_t* k_strides,
                                    const void* v, const int64_t* v_strides, const float* g,
                                    const int64_t* g_strides, const void* beta, int beta_dtype,
                                    const int64_t* beta_strides, const float* h0, const int64_t* h0_strides,
                                    void* o, const int64_t* o_strides, float* ht, int B, int T, int H, int HV,
                                    int K, int V, int dtype, float scale, int l2norm, int algo, void* workspace,
                                    size_t workspace_bytes, d3b_stream_t stream) {
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
  if (algo < 0 || algo > 3) return D3B_EINVAL;
  // the chunked form: blocks of <= 64 tokens, K = V = 128, one state for all rows, no final state,
  // 16-byte rows (q, k, v, o: strides in multiples of 8 elements; h0: of 4)
  bool rows16 = aligned(q, 16) && aligned(k, 16) && aligned(v, 16) && aligned(o, 16) && (!h0 || aligned(h0, 16));
  for (int i = 0; i < 3; ++i)
    rows16 = rows16 && q_strides[i] % 8 == 0 && k_strides[i] % 8 == 0 && v_strides[i] % 8 == 0 &&
             o_strides[i] % 8 == 0;
  if (h0) rows16 = rows16 && h0_strides[1] % 4 == 0 && h0_strides[2] % 4 == 0;
  const bool ws_ok = !h0 || (workspace && workspace_bytes >= d3b_gated_delta_workspace_size(HV, K, V) &&
                             aligned(workspace, 16));
  const bool chunk_ok =
      K == 128 && V == 128 && T <= 64 && !ht && (!h0 || h0_strides[0] == 0 || B == 1) && rows16 && ws_ok;
  if (algo == 2 && !chunk_ok) return D3B_EUNSUPPORTED;
  if (algo == 2 || (algo == 0 && chunk_ok && T > 0))
    return dtype == D3B_BF16 ? launch_chunk<__nv_bfloat16>(p, beta_dtype, static_cast<uint8_t*>(workspace), s)
                             : launch_chunk<__half>(p, beta_dtype, static_cast<uint8_t*>(workspace), s);
  // the chunked form with the inter-chunk recurrence: any length, K = V = 128, any initial
  // states, final state, 16-byte rows, a workspace of d3b_gated_delta_state_workspace_size()
  const bool state_ok = K == 128 && V == 128 && T > 0 && rows16 && (!ht || aligned(ht, 16)) && workspace &&
                        aligned(workspace, 256) &&
                        workspace_bytes >= state_workspace_bytes(B, T, HV) && (long long)B * HV * 2 < (1ll << 31);
  if (algo == 3 && !state_ok) return D3B_EUNSUPPORTED;
  if (algo == 3 || (algo == 0 && state_ok))
    return dtype == D3B_BF16 ? launch_state<__nv_bfloat16>(p, beta_dtype, static_cast<uint8_t*>(workspace), s)
                             : launch_state<__half>(p, beta_dtype, static_cast<uint8_t*>(workspace), s);
  if (K == 128)
    return dtype == D3B_BF16 ? launch_k<128, __nv_bfloat16>(p, beta_dtype, blocks, s)
                             : launch_k<128, __half>(p, beta_dtype, blocks, s);
  return dtype == D3B_BF16 ? launch_k<64, __nv_bfloat16>(p, beta_dtype, blocks, s)
                           : launch_k<64, __half>(p, beta_dtype, blocks, s);
}
