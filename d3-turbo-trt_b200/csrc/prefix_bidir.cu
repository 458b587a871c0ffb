// Prefix-bidirectional GQA attention on the 5th-generation tensor cores.
//
// Replaces d3trt/kernels/prefix_bidir.py:187-260 (wrapper) and the Triton
// kernel _prefix_bidir_fwd at :47-131. For question block b, query head h and
// token i < lengths[b], the output row is
//     softmax_j(scale * q[b,h,i] . k_j) . v_j
// over j in {state keys 0..S-1} U {the block's own keys 0..lengths[b]-1}, with
// kv head h / (H/Hkv) (prefix_bidir.py:85). Rows i >= lengths[b] are zero
// (prefix_bidir.py:171-176). With S == 0 the same kernel is the dense
// bidirectional state pass (ops.py:107-124, :174-193).
//
// Work unit (one CTA): (block b, kv head g, tile of T tokens). The GQA group is
// folded into the MMA M dimension: the 128 rows of the Q tile are
// (token t, head-in-group h) -> row t*G + h, so one K/V stream serves all G
// query heads. The 4-D TMA box {D-chunk, G, T, 1} lands the tile directly in
// that order; no pack/unpack gathers and no token-major copies are needed
// (any 16-byte-multiple strides are read as they are).
//
// Key schedule (block sparse, from the lengths table): ceil(S/BN) state tiles
// then ceil(len_b/BN) own-block tiles; only the last state tile and the own
// tiles carry a key mask. Nothing outside [state | own block] is touched.
//
// Two kernels share this work unit, the key schedule and the softmax:
//   D <= 128  prefix_bidir_2c_kernel: one Q tile per CTA, two CTAs per SM
//             (the tensor core alternates between the two CTAs' chains).
//   D == 256  prefix_bidir_kernel: one Q tile per CTA, one CTA per SM, S
//             double-buffered in TMEM (O alone takes 256 columns).
// Both use one thread per Q row for the softmax: tcgen05.ld of the S row,
// online softmax in the log2 domain, P as bf16/f16 written back to TMEM for
// the TS-form PV MMA (V read MN-major from shared memory), O rescaled in TMEM
// only when the running max grows by more than 2^8 (otherwise the stale max
// is kept), final O / l in the epilogue.
//
// D == 256 kernel roles (6 warps):
//   warp 0      TMA producer: Q once, then K/V tiles into a ring of slots in
//               the order the MMA issuer consumes them (K0, K1, V0, K2, V1, ..)
//   warp 1      TMEM owner + tcgen05.mma issuer (one thread)
//                 S[j%2] = Q K_j^T              (SS form, both K-major, fp32)
//                 O     += P[j%2] V_j            (TS form: P from TMEM, V MN-major)
//   warps 2..5  softmax + epilogue
// TMEM (512 columns): O [0,D) | S0 | S1 (BN each) | P0 | P1 (BN/2 each).
#include "common.cuh"

namespace {

constexpr int BM = 128;
constexpr int NUM_THREADS = 192;
constexpr float kRescaleThreshold = 8.0f;  // log2 units: rescale O when max grows by > 2^8

enum {
  kSiteQ = 2001,
  kSiteSlotEmpty = 2002,
  kSiteSlotFull = 2003,
  kSiteSFree = 2004,
  kSitePFull = 2005,
  kSiteSFull = 2006,
  kSitePFree = 2007,
  kSiteFinal = 2008,
  kSiteDrain = 2009
};

template <int D, int BN>
struct Cfg {
  static constexpr int CH = D >= 64 ? 64 : D;  // elements per swizzle row
  static constexpr int ROWB = CH * 2;          // bytes per smem row (128 or 64)
  static constexpr int NCH = D / CH;           // swizzle chunks along D
  static constexpr uint32_t LAYOUT = ROWB == 128 ? d3b::kLayoutSW128 : d3b::kLayoutSW64;
  static constexpr int SBO = 8 * ROWB;               // 8-row core-matrix group stride
  static constexpr int Q_BYTES = BM * D * 2;         // Q tile
  static constexpr int SLOT_BYTES = BN * D * 2;      // one K or V tile
  static constexpr int Q_CHUNK = BM * ROWB;          // one D chunk of Q
  static constexpr int SLOT_CHUNK = BN * ROWB;       // one D chunk of a K/V tile
  static constexpr int NSLOT_RAW = (200 * 1024 - Q_BYTES) / SLOT_BYTES;
  static constexpr int NSLOT = NSLOT_RAW > 8 ? 8 : NSLOT_RAW;
  static constexpr int SMEM_BYTES = Q_BYTES + NSLOT * SLOT_BYTES + 1024;
  static constexpr int COL_O = 0;
  static constexpr int COL_S = D;            // + b*BN
  static constexpr int COL_P = D + 2 * BN;   // + b*BN/2
  static constexpr uint32_t TMEM_COLS = 512;
  static_assert(D + 3 * BN <= 512, "TMEM budget");
  static_assert(NSLOT >= 2, "smem budget");
};

struct __align__(8) Bars {
  uint64_t q_full;
  uint64_t slot_full[8];
  uint64_t slot_empty[8];
  uint64_t s_full[2];
  uint64_t s_free[2];
  uint64_t p_full[2];
  uint64_t p_free[2];
  uint64_t drain;
  uint32_t tmem_slot;
  int abort_flag;
};

struct Params {
  const int32_t* lengths;
  void* out;
  int64_t out_sb, out_sh, out_sl;  // element strides
  int H, Hkv, G, T, S, L;
  float scale_log2;
  int* err;
};

// Item i of the K/V stream -> (is_v, kv tile j) for n tiles:
// K0, K1, V0, K2, V1, ..., K_{n-1}, V_{n-2}, V_{n-1}.
__device__ __forceinline__ void stream_item(int i, int n, int& is_v, int& j) {
  if (i == 0) { is_v = 0; j = 0; }
  else if (i == 2 * n - 1) { is_v = 1; j = n - 1; }
  else if (i & 1) { is_v = 0; j = (i + 1) >> 1; }
  else { is_v = 1; j = (i >> 1) - 1; }
}

template <int FP16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  return FP16 ? d3b::pack_f16x2(lo, hi) : d3b::pack_bf16x2(lo, hi);
}

__device__ __forceinline__ float max3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// Max of N values: three-input max, 8 independent accumulators (short
// dependency chains; N/2 + 4 instructions).
template <int N>
__device__ __forceinline__ float max_n(const float* v) {
  float a[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) a[k] = v[k];
#pragma unroll
  for (int c = 8; c < N; c += 16)
#pragma unroll
    for (int k = 0; k < 8; ++k) a[k] = max3(a[k], v[c + k], v[c + 8 + k]);
  return max3(max3(a[0], a[1], a[2]), max3(a[3], a[4], a[5]), fmaxf(a[6], a[7]));
}

// (d0, d1) = (a0, a1) * (b, b) + (c, c) as one packed fp32x2 FMA.
__device__ __forceinline__ void fma2_bc(float& d0, float& d1, float a0, float a1, float b, float c) {
  asm("{.reg .b64 x, y, z; mov.b64 x, {%2, %3}; mov.b64 y, {%4, %4}; mov.b64 z, {%5, %5};"
      " fma.rn.f32x2 x, x, y, z; mov.b64 {%0, %1}, x;}"
      : "=f"(d0), "=f"(d1) : "f"(a0), "f"(a1), "f"(b), "f"(c));
}
// (d0, d1) = (a0, a1) * (b0, b1) + (c, c)
__device__ __forceinline__ void fma2_c(float& d0, float& d1, float a0, float a1, float b0, float b1, float c) {
  asm("{.reg .b64 x, y, z; mov.b64 x, {%2, %3}; mov.b64 y, {%4, %5}; mov.b64 z, {%6, %6};"
      " fma.rn.f32x2 x, x, y, z; mov.b64 {%0, %1}, x;}"
      : "=f"(d0), "=f"(d1) : "f"(a0), "f"(a1), "f"(b0), "f"(b1), "f"(c));
}
// (a0, a1) += (b0, b1)
__device__ __forceinline__ void add2(float& a0, float& a1, float b0, float b1) {
  asm("{.reg .b64 x, y; mov.b64 x, {%0, %1}; mov.b64 y, {%2, %3}; add.rn.f32x2 x, x, y; mov.b64 {%0, %1}, x;}"
      : "+f"(a0), "+f"(a1) : "f"(b0), "f"(b1));
}

// 2^x for a pair on the FMA pipe (x <= 8): Cody-Waite range reduction
// x = r + f with r = round(x) (the 1.5 * 2^23 shifter puts r in the low
// mantissa bits of t), f in [-1/2, 1/2], 2^f from a degree-3 polynomial
// (least-squares fit of 2^f on Chebyshev nodes of [-1/2, 1/2], max relative
// error 7.8e-5, well below the bf16 rounding of P), and 2^r added to the
// exponent field. Inputs below -126 are clamped: 2^-126 stands for 0.
__device__ __forceinline__ void exp2_poly2(float x0, float x1, float& p0, float& p1) {
  constexpr float kShift = 12582912.f;  // 1.5 * 2^23
  x0 = fmaxf(x0, -126.f);
  x1 = fmaxf(x1, -126.f);
  float t0, t1, r0, r1, f0, f1;
  fma2_bc(t0, t1, x0, x1, 1.f, kShift);      // t = x + shift (round to nearest integer)
  fma2_bc(r0, r1, t0, t1, 1.f, -kShift);     // r = round(x)
  fma2_c(f0, f1, r0, r1, -1.f, -1.f, 0.f);   // -r
  add2(f0, f1, x0, x1);                      // f = x - r
  float q0, q1;
  fma2_bc(q0, q1, f0, f1, 0.05508868396282196f, 0.24260404706001282f);
  fma2_c(q0, q1, q0, q1, f0, f1, 0.6932762265205383f);
  fma2_c(q0, q1, q0, q1, f0, f1, 0.9999289512634277f);
  p0 = __int_as_float(__float_as_int(q0) + (__float_as_int(t0) << 23));
  p1 = __int_as_float(__float_as_int(q1) + (__float_as_int(t1) << 23));
}

// P = 2^(s * sl2 - m) for one row of N scores: packed pairs into pk (bf16 or
// f16), returns the row sum of the fp32 values. One pair in four goes through
// the FMA-pipe exponential, the rest through MUFU ex2, so neither unit alone
// bounds the softmax.
template <int N, int FP16>
__device__ __forceinline__ float exp_row(const float* s, float sl2, float m, uint32_t* pk) {
  float part[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int c = 0; c < N; c += 2) {
    float x0, x1, p0, p1;
    fma2_bc(x0, x1, s[c], s[c + 1], sl2, -m);
    if (((c >> 1) & 3) == 3) {
      exp2_poly2(x0, x1, p0, p1);
    } else {
      p0 = d3b::ex2_approx(x0);
      p1 = d3b::ex2_approx(x1);
    }
    const int k = ((c >> 1) & 3) * 2;
    add2(part[k], part[k + 1], p0, p1);
    pk[c / 2] = pack2<FP16>(p0, p1);
  }
  return ((part[0] + part[1]) + (part[2] + part[3])) + ((part[4] + part[5]) + (part[6] + part[7]));
}

template <int D, int BN, int FP16>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    prefix_bidir_kernel(const __grid_constant__ CUtensorMap mapQ, const __grid_constant__ CUtensorMap mapKs,
                        const __grid_constant__ CUtensorMap mapVs, const __grid_constant__ CUtensorMap mapKq,
                        const __grid_constant__ CUtensorMap mapVq, const Params p) {
  using C = Cfg<D, BN>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ Bars bars;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
  const int G = p.G, T = p.T;
  const int len_b = p.lengths[b];
  const int rows_used = G * T;
  const int tok0 = tile * T;

  // ---- rows of this tile that need no attention: zero-fill and leave ----
  if (tok0 >= len_b) {
    if (warp >= 2) {
      const int r = (warp & 3) * 32 + lane;
      const int tok = tok0 + r / G, h = r % G;
      if (r < rows_used && tok < p.L) {
        uint4* dst = reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.out) + (int64_t)b * p.out_sb +
                                              (int64_t)(g * G + h) * p.out_sh + (int64_t)tok * p.out_sl);
#pragma unroll
        for (int i = 0; i < D / 8; ++i) dst[i] = make_uint4(0, 0, 0, 0);
      }
    }
    return;
  }

  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sKV = smem + C::Q_BYTES;
  volatile int* abort_flag = &bars.abort_flag;
  const int n_s = (p.S + BN - 1) / BN;
  const int n_o = (len_b + BN - 1) / BN;
  const int n = n_s + n_o;

  if (threadIdx.x == 0) {
    d3b::mbar_init(&bars.q_full, 1);
    for (int s = 0; s < C::NSLOT; ++s) {
      d3b::mbar_init(&bars.slot_full[s], 1);
      d3b::mbar_init(&bars.slot_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      d3b::mbar_init(&bars.s_full[i], 1);
      d3b::mbar_init(&bars.s_free[i], 128);
      d3b::mbar_init(&bars.p_full[i], 128);
      d3b::mbar_init(&bars.p_free[i], 1);
    }
    d3b::mbar_init(&bars.drain, 1);
    bars.abort_flag = 0;
    d3b::fence_barrier_init();
  }
  // Rows the TMA box does not cover (G does not divide 128) are zeroed so the
  // MMA never reads uninitialised shared memory.
  if (rows_used < BM) {
    for (int i = threadIdx.x; i < C::NCH * (BM - rows_used) * C::ROWB / 16; i += NUM_THREADS) {
      const int per_chunk = (BM - rows_used) * C::ROWB / 16;
      const int c = i / per_chunk, o = i % per_chunk;
      reinterpret_cast<uint4*>(sQ + c * C::Q_CHUNK + rows_used * C::ROWB)[o] = make_uint4(0, 0, 0, 0);
    }
    d3b::fence_proxy_async_smem();
  }
  if (warp == 1) d3b::tmem_alloc(&bars.tmem_slot, C::TMEM_COLS);
  d3b::tc_fence_before();
  __syncthreads();
  d3b::tc_fence_after();
  const uint32_t tmem_base = bars.tmem_slot;

  if (warp == 0) {
    // ================= TMA producer =================
    if (lane == 0) {
      d3b::tma_prefetch_desc(&mapQ);
      d3b::tma_prefetch_desc(&mapKq);
      d3b::tma_prefetch_desc(&mapVq);
      if (n_s) {
        d3b::tma_prefetch_desc(&mapKs);
        d3b::tma_prefetch_desc(&mapVs);
      }
      d3b::mbar_arrive_expect_tx(&bars.q_full, C::NCH * rows_used * C::ROWB);
#pragma unroll
      for (int c = 0; c < C::NCH; ++c)
        d3b::tma_load_4d(sQ + c * C::Q_CHUNK, &mapQ, &bars.q_full, c * C::CH, g * G, tok0, b);
      int stage = 0;
      uint32_t phase = 0;
      for (int i = 0; i < 2 * n; ++i) {
        int is_v, j;
        stream_item(i, n, is_v, j);
        if (!d3b::mbar_wait(&bars.slot_empty[stage], phase ^ 1, abort_flag, p.err, kSiteSlotEmpty)) break;
        d3b::mbar_arrive_expect_tx(&bars.slot_full[stage], C::SLOT_BYTES);
        uint8_t* dst = sKV + stage * C::SLOT_BYTES;
        if (j < n_s) {
          const CUtensorMap* m = is_v ? &mapVs : &mapKs;
#pragma unroll
          for (int c = 0; c < C::NCH; ++c)
            d3b::tma_load_3d(dst + c * C::SLOT_CHUNK, m, &bars.slot_full[stage], c * C::CH, j * BN, g);
        } else {
          const CUtensorMap* m = is_v ? &mapVq : &mapKq;
#pragma unroll
          for (int c = 0; c < C::NCH; ++c)
            d3b::tma_load_4d(dst + c * C::SLOT_CHUNK, m, &bars.slot_full[stage], c * C::CH, (j - n_s) * BN, g, b);
        }
        if (++stage == C::NSLOT) { stage = 0; phase ^= 1; }
      }
    }
  } else if (warp == 1) {
    // ================= MMA issuer =================
    if (lane == 0) {
      constexpr uint32_t fmt = FP16 ? 0u : 1u;
      constexpr uint32_t idesc_qk = d3b::make_idesc(1, fmt, fmt, 0, 0, BM, BN);
      constexpr uint32_t idesc_pv = d3b::make_idesc(1, fmt, fmt, 0, 1, BM, D);
      const uint32_t q_addr = d3b::smem_u32(sQ), kv_addr = d3b::smem_u32(sKV);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = d3b::mbar_wait(&bars.q_full, 0, abort_flag, p.err, kSiteQ);

      auto issue_qk = [&](int sb) -> bool {  // S[sb] = Q K^T from the next slot
        if (!d3b::mbar_wait(&bars.slot_full[stage], phase, abort_flag, p.err, kSiteSlotFull)) return false;
        d3b::tc_fence_after();
        const uint32_t k_addr = kv_addr + stage * C::SLOT_BYTES;
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const int c = (k * 16) / C::CH, off = ((k * 16) % C::CH) * 2;
          const uint64_t ad = d3b::make_smem_desc(q_addr + c * C::Q_CHUNK + off, 16, C::SBO, C::LAYOUT);
          const uint64_t bd = d3b::make_smem_desc(k_addr + c * C::SLOT_CHUNK + off, 16, C::SBO, C::LAYOUT);
          d3b::mma_f16_ss(tmem_base + C::COL_S + sb * BN, ad, bd, idesc_qk, k > 0 ? 1u : 0u);
        }
        d3b::mma_commit(&bars.s_full[sb]);
        d3b::mma_commit(&bars.slot_empty[stage]);
        if (++stage == C::NSLOT) { stage = 0; phase ^= 1; }
        return true;
      };

      if (ok) ok = issue_qk(0);
      for (int j = 0; j < n && ok; ++j) {
        if (j + 1 < n) {
          const int b1 = (j + 1) & 1;
          const uint32_t u1 = (uint32_t)((j + 1) >> 1);
          if (!d3b::mbar_wait(&bars.s_free[b1], (u1 & 1) ^ 1, abort_flag, p.err, kSiteSFree)) break;
          d3b::tc_fence_after();
          if (!issue_qk(b1)) break;
        }
        const int pb = j & 1;
        const uint32_t u = (uint32_t)(j >> 1);
        if (!d3b::mbar_wait(&bars.p_full[pb], u & 1, abort_flag, p.err, kSitePFull)) break;
        d3b::tc_fence_after();
        if (!d3b::mbar_wait(&bars.slot_full[stage], phase, abort_flag, p.err, kSiteSlotFull)) break;
        d3b::tc_fence_after();
        const uint32_t v_addr = kv_addr + stage * C::SLOT_BYTES;
#pragma unroll
        for (int k = 0; k < BN / 16; ++k) {
          // 16 keys: rows [16k, 16k+16) of the V tile; D spans NCH chunks at LBO.
          const uint64_t bd = d3b::make_smem_desc(v_addr + k * 16 * C::ROWB, C::SLOT_CHUNK, C::SBO, C::LAYOUT);
          d3b::mma_f16_ts(tmem_base + C::COL_O, tmem_base + C::COL_P + pb * (BN / 2) + k * 8, bd, idesc_pv,
                          (j > 0 || k > 0) ? 1u : 0u);
        }
        d3b::mma_commit(&bars.p_free[pb]);
        d3b::mma_commit(&bars.slot_empty[stage]);
        if (++stage == C::NSLOT) { stage = 0; phase ^= 1; }
      }
      d3b::mma_commit(&bars.drain);
      const uint32_t addr = d3b::smem_u32(&bars.drain);
      const uint64_t t0 = d3b::globaltimer_ns();
      while (!d3b::mbar_try_wait(addr, 0)) {
        if (d3b::globaltimer_ns() - t0 > D3B_WAIT_LIMIT_NS) {
          d3b::record_device_error(p.err, kSiteDrain);
          break;
        }
      }
    }
  } else {
    // ================= softmax + epilogue (warps 2..5) =================
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_addr = tmem_base + ((uint32_t)(quarter * 32) << 16);
    const float sl2 = p.scale_log2;
    float m_ref = -INFINITY, l_sum = 0.f;
    bool ok = true;
    for (int j = 0; j < n; ++j) {
      const int sb = j & 1;
      const uint32_t u = (uint32_t)(j >> 1);
      if (!d3b::warp_wait(&bars.s_full[sb], u & 1, abort_flag, p.err, kSiteSFull)) { ok = false; break; }
      d3b::tc_fence_after();
      float s[BN];
#pragma unroll
      for (int c = 0; c < BN / 32; ++c)
        d3b::tmem_ld32(lane_addr + C::COL_S + sb * BN + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&s[c * 32]));
      d3b::tmem_wait_ld();
      d3b::tc_fence_before();
      d3b::mbar_arrive(&bars.s_free[sb]);

      const int valid = j < n_s ? p.S - j * BN : len_b - (j - n_s) * BN;
      if (valid < BN) {
#pragma unroll
        for (int c = 0; c < BN; ++c)
          if (c >= valid) s[c] = -INFINITY;
      }
      const float m_tile = max_n<BN>(s) * sl2;
      // Lazy rescale, decided per warp: tcgen05.ld/st are warp-collective, so
      // if any row of the warp needs a new reference max, every row of the
      // warp moves to its exact running max (alpha = 1 where it is unchanged).
      const bool rescale = __any_sync(0xffffffffu, m_tile > m_ref + kRescaleThreshold);
      const float m_new = rescale ? fmaxf(m_ref, m_tile) : m_ref;
      const float alpha = rescale ? d3b::ex2_approx(m_ref - m_new) : 1.f;
      uint32_t pk[BN / 2];
      const float rowsum = exp_row<BN, FP16>(s, sl2, m_new, pk);
      // P[sb] is free once PV_{j-2} (its previous reader) has completed.
      if (!d3b::warp_wait(&bars.p_free[sb], (u & 1) ^ 1, abort_flag, p.err, kSitePFree)) { ok = false; break; }
      d3b::tc_fence_after();
#pragma unroll
      for (int c = 0; c < BN / 64; ++c)
        d3b::tmem_st32(lane_addr + C::COL_P + sb * (BN / 2) + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&pk[c * 32]));
      if (BN % 64) d3b::tmem_st16(lane_addr + C::COL_P + sb * (BN / 2) + (BN / 64) * 32,
                                   *reinterpret_cast<uint32_t(*)[16]>(&pk[(BN / 64) * 32]));
      if (rescale && j > 0) {
        // O must hold every PV up to j-1: wait for PV_{j-1}'s commit.
        const int pb1 = (j - 1) & 1;
        const uint32_t u1 = (uint32_t)((j - 1) >> 1);
        if (!d3b::warp_wait(&bars.p_free[pb1], u1 & 1, abort_flag, p.err, kSitePFree)) { ok = false; break; }
        d3b::tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32];
          d3b::tmem_ld32(lane_addr + C::COL_O + c * 32, o);
          d3b::tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          d3b::tmem_st32(lane_addr + C::COL_O + c * 32, o);
        }
      }
      l_sum = l_sum * alpha + rowsum;
      m_ref = m_new;
      d3b::tmem_wait_st();
      d3b::tc_fence_before();
      d3b::mbar_arrive(&bars.p_full[sb]);
    }
    if (ok) {
      const int jl = n - 1;
      ok = d3b::warp_wait(&bars.p_free[jl & 1], (uint32_t)(jl >> 1) & 1, abort_flag, p.err, kSiteFinal);
    }
    if (ok) {
      d3b::tc_fence_after();
      const int tok = tok0 + r / G, h = r % G;
      const bool in_tensor = r < rows_used && tok < p.L;
      const bool real = tok < len_b;
      const float inv_l = 1.f / l_sum;
      uint16_t* dst_row = static_cast<uint16_t*>(p.out) + (int64_t)b * p.out_sb + (int64_t)(g * G + h) * p.out_sh +
                          (int64_t)tok * p.out_sl;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        d3b::tmem_ld32(lane_addr + C::COL_O + c * 32, o);
        d3b::tmem_wait_ld();
        if (in_tensor) {
          uint32_t w[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            w[i] = real ? pack2<FP16>(__uint_as_float(o[2 * i]) * inv_l, __uint_as_float(o[2 * i + 1]) * inv_l) : 0u;
          uint4* dst = reinterpret_cast<uint4*>(dst_row + c * 32);
#pragma unroll
          for (int i = 0; i < 4; ++i) dst[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
        }
      }
    }
  }

  d3b::tc_fence_before();
  __syncthreads();
  d3b::tc_fence_after();
  if (warp == 1) d3b::tmem_dealloc(tmem_base, C::TMEM_COLS);
}

// ===========================================================================
// One Q tile per CTA, two CTAs per SM (D <= 128).
//
// 256 TMEM columns per CTA: O (D) | S (128 keys); P (bf16/f16) goes into the
// upper half of S once S has been read. Two co-resident CTAs share the SM's
// tensor core, so while one CTA's softmax runs, the other's QK^T / PV execute;
// each CTA's chain QK(j) -> softmax(j) -> PV(j) -> QK(j+1) needs no
// cross-CTA ordering. Shared memory stays under half an SM (Q + two 32 KB K/V
// slots at D = 128).
// Warps 0-3 softmax + epilogue, warp 4 TMA producer, warp 5 TMEM + MMA. At
// 128 registers per thread a softmax thread holds 64 scores at a time: it
// reduces keys 0-63, then 64-127, turns the second half into P, reloads the
// first half and turns it into P. P is published in those two halves
// (separate barriers), so the first four PV MMAs run while the softmax still
// exponentiates keys 0-63. (An 8-warp variant that lends the softmax 200
// registers through setmaxnreg, to keep all 128 scores in registers,
// measured slower.)
// QK(j+1) overwrites S, whose upper half still holds P(j) for PV(j). Both are
// issued by the same thread in that order, and tcgen05.mma operations of one
// issuing thread execute in issue order on the SM's tensor core, so QK(j+1)
// cannot write S before PV(j) has read P(j). This is an observed property of
// the hardware, not one of the PTX ISA's guaranteed "pipelined" pairs (those
// cover MMAs on the same accumulator). Building with -DD3B_STRICT_MMA_ORDER=1
// instead waits for PV(j)'s commit before issuing QK(j+1) (slower: the tensor
// pipe drains once per key tile); the parity tests pass in both builds.
// Either way, s_full(j+1) is a tcgen05.commit after PV(j), so O is complete
// when the softmax sees S(j+1) and may rescale O without further
// synchronisation.
// ===========================================================================
#ifndef D3B_STRICT_MMA_ORDER
#define D3B_STRICT_MMA_ORDER 0
#endif
constexpr int C2_THREADS = 192;

template <int D>
struct Cfg2C {
  static constexpr int BN = 128;
  static constexpr int CH = D >= 64 ? 64 : D;
  static constexpr int ROWB = CH * 2;
  static constexpr int NCH = D / CH;
  static constexpr uint32_t LAYOUT = ROWB == 128 ? d3b::kLayoutSW128 : d3b::kLayoutSW64;
  static constexpr int SBO = 8 * ROWB;
  static constexpr int Q_BYTES = BM * D * 2;
  static constexpr int SLOT_BYTES = BN * D * 2;
  static constexpr int Q_CHUNK = BM * ROWB;
  static constexpr int SLOT_CHUNK = BN * ROWB;
  static constexpr int NSLOT_RAW = (110 * 1024 - Q_BYTES - 1024) / SLOT_BYTES;
  static constexpr int NSLOT = NSLOT_RAW > 8 ? 8 : NSLOT_RAW;
  static constexpr int SMEM_BYTES = Q_BYTES + NSLOT * SLOT_BYTES + 1024;
  static constexpr int COL_O = 0;
  static constexpr int COL_S = D;
  static constexpr uint32_t TMEM_COLS = 256;
  static_assert(D + BN <= 256, "TMEM budget");
  static_assert(NSLOT >= 2, "smem budget");
  static_assert(SMEM_BYTES <= 113 * 1024, "two CTAs per SM");
};

struct __align__(8) Bars2C {
  uint64_t q_full;
  uint64_t slot_full[8];
  uint64_t slot_empty[8];
  uint64_t s_full;
  uint64_t p_full[2];  // halves of P: [0] keys 0-63, [1] keys 64-127
  uint64_t o_final;
  uint64_t pv_done;  // only with D3B_STRICT_MMA_ORDER
  uint64_t drain;
  uint32_t tmem_slot;
  int abort_flag;
};

enum {
  kSite2CQ = 5001, kSite2CSlotEmpty, kSite2CSlotFull, kSite2CPFull, kSite2CSFull, kSite2CFinal, kSite2CDrain,
  kSite2CPvDone
};

// Zero the output rows of a Q tile that holds no real token (rows past the
// tensor's L are skipped).
template <int D>
__device__ __forceinline__ void zero_tile_rows(const Params& p, int b, int g, int tok0, int quarter, int lane) {
  const int r = quarter * 32 + lane;
  const int tok = tok0 + r / p.G, h = r % p.G;
  if (r < p.G * p.T && tok < p.L) {
    uint4* dst = reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.out) + (int64_t)b * p.out_sb +
                                          (int64_t)(g * p.G + h) * p.out_sh + (int64_t)tok * p.out_sl);
#pragma unroll
    for (int i = 0; i < D / 8; ++i) dst[i] = make_uint4(0, 0, 0, 0);
  }
}

// 64 columns of this thread's TMEM row into registers, keys >= valid masked.
__device__ __forceinline__ void load64(uint32_t addr, int key0, int valid, float (&s)[64]) {
  d3b::tmem_ld32(addr, *reinterpret_cast<uint32_t(*)[32]>(&s[0]));
  d3b::tmem_ld32(addr + 32, *reinterpret_cast<uint32_t(*)[32]>(&s[32]));
  d3b::tmem_wait_ld();
  if (valid - key0 < 64) {
#pragma unroll
    for (int c = 0; c < 64; ++c)
      if (key0 + c >= valid) s[c] = -INFINITY;
  }
}

template <int D, int FP16>
__global__ void __launch_bounds__(C2_THREADS, 2)
    prefix_bidir_2c_kernel(const __grid_constant__ CUtensorMap mapQ, const __grid_constant__ CUtensorMap mapKs,
                           const __grid_constant__ CUtensorMap mapVs, const __grid_constant__ CUtensorMap mapKq,
                           const __grid_constant__ CUtensorMap mapVq, const Params p) {
  using C = Cfg2C<D>;
  constexpr int BN = C::BN;
  extern __shared__ uint8_t smem_raw[];
  __shared__ Bars2C bars;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
  const int G = p.G, T = p.T;
  const int rows_used = G * T;
  const int len_b = p.lengths[b];
  const int tok0 = tile * T;
  if (tok0 >= len_b) {  // no real token in this tile: zero-fill and leave
    if (warp < 4) zero_tile_rows<D>(p, b, g, tok0, warp, lane);
    return;
  }
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sKV = smem + C::Q_BYTES;
  volatile int* abort_flag = &bars.abort_flag;
  const int n_s = (p.S + BN - 1) / BN;
  const int n = n_s + (len_b + BN - 1) / BN;

  if (threadIdx.x == 0) {
    d3b::mbar_init(&bars.q_full, 1);
    for (int i = 0; i < C::NSLOT; ++i) {
      d3b::mbar_init(&bars.slot_full[i], 1);
      d3b::mbar_init(&bars.slot_empty[i], 1);
    }
    d3b::mbar_init(&bars.s_full, 1);
    d3b::mbar_init(&bars.p_full[0], 128);
    d3b::mbar_init(&bars.p_full[1], 128);
    d3b::mbar_init(&bars.o_final, 1);
    d3b::mbar_init(&bars.pv_done, 1);
    d3b::mbar_init(&bars.drain, 1);
    bars.abort_flag = 0;
    d3b::fence_barrier_init();
  }
  if (rows_used < BM) {
    const int per_chunk = (BM - rows_used) * C::ROWB / 16;
    for (int i = threadIdx.x; i < C::NCH * per_chunk; i += C2_THREADS) {
      const int c = i / per_chunk, o = i % per_chunk;
      reinterpret_cast<uint4*>(sQ + c * C::Q_CHUNK + rows_used * C::ROWB)[o] = make_uint4(0, 0, 0, 0);
    }
    d3b::fence_proxy_async_smem();
  }
  if (warp == 5) d3b::tmem_alloc(&bars.tmem_slot, C::TMEM_COLS);
  d3b::tc_fence_before();
  __syncthreads();
  d3b::tc_fence_after();
  const uint32_t tmem_base = bars.tmem_slot;

  if (warp == 4) {
    // ================= TMA producer: Q, then K_0, V_0, K_1, V_1, ... =================
    if (lane == 0) {
      d3b::tma_prefetch_desc(&mapQ);
      d3b::tma_prefetch_desc(&mapKq);
      d3b::tma_prefetch_desc(&mapVq);
      if (n_s) {
        d3b::tma_prefetch_desc(&mapKs);
        d3b::tma_prefetch_desc(&mapVs);
      }
      d3b::mbar_arrive_expect_tx(&bars.q_full, C::NCH * rows_used * C::ROWB);
#pragma unroll
      for (int c = 0; c < C::NCH; ++c)
        d3b::tma_load_4d(sQ + c * C::Q_CHUNK, &mapQ, &bars.q_full, c * C::CH, g * G, tok0, b);
      int stage = 0;
      uint32_t phase = 0;
      for (int i = 0; i < 2 * n; ++i) {
        const int is_v = i & 1, j = i >> 1;
        if (!d3b::mbar_wait(&bars.slot_empty[stage], phase ^ 1, abort_flag, p.err, kSite2CSlotEmpty)) break;
        d3b::mbar_arrive_expect_tx(&bars.slot_full[stage], C::SLOT_BYTES);
        uint8_t* dst = sKV + stage * C::SLOT_BYTES;
        if (j < n_s) {
          const CUtensorMap* m = is_v ? &mapVs : &mapKs;
#pragma unroll
          for (int c = 0; c < C::NCH; ++c)
            d3b::tma_load_3d(dst + c * C::SLOT_CHUNK, m, &bars.slot_full[stage], c * C::CH, j * BN, g);
        } else {
          const CUtensorMap* m = is_v ? &mapVq : &mapKq;
#pragma unroll
          for (int c = 0; c < C::NCH; ++c)
            d3b::tma_load_4d(dst + c * C::SLOT_CHUNK, m, &bars.slot_full[stage], c * C::CH, (j - n_s) * BN, g,
                             b);
        }
        if (++stage == C::NSLOT) { stage = 0; phase ^= 1; }
      }
    }
  } else if (warp == 5) {
    // ================= MMA issuer =================
    if (lane == 0) {
      constexpr uint32_t fmt = FP16 ? 0u : 1u;
      constexpr uint32_t idesc_qk = d3b::make_idesc(1, fmt, fmt, 0, 0, BM, BN);
      constexpr uint32_t idesc_pv = d3b::make_idesc(1, fmt, fmt, 0, 1, BM, D);
      const uint64_t dq0 = d3b::make_smem_desc(d3b::smem_u32(sQ), 16, C::SBO, C::LAYOUT);
      const uint64_t dk0 = d3b::make_smem_desc(d3b::smem_u32(sKV), 16, C::SBO, C::LAYOUT);
      const uint64_t dv0 = d3b::make_smem_desc(d3b::smem_u32(sKV), C::SLOT_CHUNK, C::SBO, C::LAYOUT);
      auto slot_of = [&](int item) { return item % C::NSLOT; };
      auto wait_item = [&](int item) -> bool {
        return d3b::mbar_wait(&bars.slot_full[slot_of(item)], (uint32_t)(item / C::NSLOT) & 1, abort_flag, p.err,
                              kSite2CSlotFull);
      };
      auto qk = [&](int item) {
        const uint64_t dk = dk0 + (uint64_t)((slot_of(item) * C::SLOT_BYTES) >> 4);
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const int c = (k * 16) / C::CH, off = ((k * 16) % C::CH) * 2;
          d3b::mma_f16_ss(tmem_base + C::COL_S, dq0 + (uint64_t)((c * C::Q_CHUNK + off) >> 4),
                          dk + (uint64_t)((c * C::SLOT_CHUNK + off) >> 4), idesc_qk, k > 0 ? 1u : 0u);
        }
        d3b::mma_commit(&bars.s_full);
      };
      // O (+)= P V, the half with keys 64-127 first (the softmax publishes it first)
      auto pv = [&](int item, bool accumulate, uint32_t use) -> bool {
        const uint64_t dv = dv0 + (uint64_t)((slot_of(item) * C::SLOT_BYTES) >> 4);
        const uint32_t a_tmem = tmem_base + C::COL_S + BN / 2;
        bool first = true;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int h = 1 - hh;
          if (!d3b::mbar_wait(&bars.p_full[h], use & 1, abort_flag, p.err, kSite2CPFull)) return false;
          d3b::tc_fence_after();
#pragma unroll
          for (int k = h * BN / 32; k < (h + 1) * BN / 32; ++k) {
            d3b::mma_f16_ts(tmem_base + C::COL_O, a_tmem + k * 8, dv + (uint64_t)((k * 16 * C::ROWB) >> 4),
                            idesc_pv, (accumulate || !first) ? 1u : 0u);
            first = false;
          }
        }
        return true;
      };
      bool ok = d3b::mbar_wait(&bars.q_full, 0, abort_flag, p.err, kSite2CQ);
      if (ok && (ok = wait_item(0))) {
        d3b::tc_fence_after();
        qk(0);
        d3b::mma_commit(&bars.slot_empty[slot_of(0)]);
      }
      for (int j = 0; j < n && ok; ++j) {
        const int it_v = 2 * j + 1;
        if (!(ok = wait_item(it_v))) break;
        if (!(ok = pv(it_v, j > 0, (uint32_t)j))) break;
        d3b::mma_commit(&bars.slot_empty[slot_of(it_v)]);
        if (j + 1 < n) {  // QK(j+1): in issue order after PV(j), which read P from S
          const int it_k = 2 * (j + 1);
          if (D3B_STRICT_MMA_ORDER) {
            d3b::mma_commit(&bars.pv_done);
            if (!(ok = d3b::mbar_wait(&bars.pv_done, (uint32_t)(j & 1), abort_flag, p.err, kSite2CPvDone))) break;
          }
          if (!(ok = wait_item(it_k))) break;
          d3b::tc_fence_after();
          qk(it_k);
          d3b::mma_commit(&bars.slot_empty[slot_of(it_k)]);
        }
      }
      if (ok) d3b::mma_commit(&bars.o_final);
      d3b::mma_commit(&bars.drain);
      const uint32_t addr = d3b::smem_u32(&bars.drain);
      const uint64_t t0 = d3b::globaltimer_ns();
      while (!d3b::mbar_try_wait(addr, 0)) {
        if (d3b::globaltimer_ns() - t0 > D3B_WAIT_LIMIT_NS) {
          d3b::record_device_error(p.err, kSite2CDrain);
          break;
        }
      }
    }
  } else {
    // ================= softmax + epilogue (warps 0-3) =================
    const int quarter = warp;
    const int r = quarter * 32 + lane;
    const uint32_t lane_addr = tmem_base + ((uint32_t)(quarter * 32) << 16);
    const uint32_t col_s = C::COL_S, col_p = C::COL_S + BN / 2, col_o = C::COL_O;
    const float sl2 = p.scale_log2;
    float m_ref = -INFINITY, l_sum = 0.f;
    bool ok = true;
    for (int j = 0; j < n; ++j) {
      if (!d3b::warp_wait(&bars.s_full, (uint32_t)(j & 1), abort_flag, p.err, kSite2CSFull)) { ok = false; break; }
      d3b::tc_fence_after();
      const int valid = j < n_s ? p.S - j * BN : len_b - (j - n_s) * BN;
      float s[64];
      load64(lane_addr + col_s, 0, valid, s);
      const float m_lo = max_n<64>(s);
      load64(lane_addr + col_s + 64, 64, valid, s);  // keys 64-127 stay in registers
      const float m_tile = fmaxf(m_lo, max_n<64>(s)) * sl2;
      const bool rescale = __any_sync(0xffffffffu, m_tile > m_ref + kRescaleThreshold);
      const float m_new = rescale ? fmaxf(m_ref, m_tile) : m_ref;
      const float alpha = rescale ? d3b::ex2_approx(m_ref - m_new) : 1.f;
      if (rescale && j > 0) {
        // s_full(j) is a commit issued after PV(j-1): O is complete here
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32];
          d3b::tmem_ld32(lane_addr + col_o + c * 32, o);
          d3b::tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          d3b::tmem_st32(lane_addr + col_o + c * 32, o);
        }
      }
      // P into the upper half of S (whose values are all in registers), keys
      // 64-127 first: the MMA thread consumes that half first.
      uint32_t pk[32];
      // keys 64-127 -> P columns 32-63 (S columns 96-127, held in registers)
      float rowsum = exp_row<64, FP16>(s, sl2, m_new, pk);
      d3b::tmem_st32(lane_addr + col_p + 32, pk);
      d3b::tmem_wait_st();
      d3b::tc_fence_before();
      d3b::mbar_arrive(&bars.p_full[1]);
      // keys 0-63 (reloaded) -> P columns 0-31 (S columns 64-95, consumed above)
      load64(lane_addr + col_s, 0, valid, s);
      rowsum += exp_row<64, FP16>(s, sl2, m_new, pk);
      d3b::tmem_st32(lane_addr + col_p, pk);
      d3b::tmem_wait_st();
      d3b::tc_fence_before();
      d3b::mbar_arrive(&bars.p_full[0]);
      l_sum = l_sum * alpha + rowsum;
      m_ref = m_new;
    }
    if (ok) ok = d3b::warp_wait(&bars.o_final, 0, abort_flag, p.err, kSite2CFinal);
    if (ok) {
      d3b::tc_fence_after();
      const int tok = tok0 + r / G, h = r % G;
      const bool in_tensor = r < rows_used && tok < p.L;
      const bool real = tok < len_b;
      const float inv_l = 1.f / l_sum;
      uint16_t* dst_row = static_cast<uint16_t*>(p.out) + (int64_t)b * p.out_sb + (int64_t)(g * G + h) * p.out_sh +
                          (int64_t)tok * p.out_sl;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        d3b::tmem_ld32(lane_addr + col_o + c * 32, o);
        d3b::tmem_wait_ld();
        if (in_tensor) {
          uint32_t w[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            w[i] = real ? pack2<FP16>(__uint_as_float(o[2 * i]) * inv_l, __uint_as_float(o[2 * i + 1]) * inv_l) : 0u;
          uint4* dst = reinterpret_cast<uint4*>(dst_row + c * 32);
#pragma unroll
          for (int i = 0; i < 4; ++i) dst[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
        }
      }
    }
  }

  d3b::tc_fence_before();
  __syncthreads();
  d3b::tc_fence_after();
  if (warp == 5) d3b::tmem_dealloc(tmem_base, C::TMEM_COLS);
}

template <int D, int FP16>
int launch_2c(const CUtensorMap* maps, const Params& prm, dim3 grid, cudaStream_t stream) {
  using C = Cfg2C<D>;
  static int attr_set[64] = {0};
  const int dev = d3b_host::current_device();
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    if (cudaFuncSetAttribute(prefix_bidir_2c_kernel<D, FP16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             C::SMEM_BYTES) != cudaSuccess)
      return D3B_ECUDA;
    attr_set[dev] = 1;
  }
  prefix_bidir_2c_kernel<D, FP16><<<grid, C2_THREADS, C::SMEM_BYTES, stream>>>(maps[0], maps[1], maps[2], maps[3],
                                                                             maps[4], prm);
  return d3b_host::check_launch();
}

template <int D, int BN, int FP16>
int launch(const CUtensorMap* maps, const Params& prm, dim3 grid, cudaStream_t stream) {
  using C = Cfg<D, BN>;
  static int attr_set[64] = {0};
  const int dev = d3b_host::current_device();
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    if (cudaFuncSetAttribute(prefix_bidir_kernel<D, BN, FP16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             C::SMEM_BYTES) != cudaSuccess)
      return D3B_ECUDA;
    attr_set[dev] = 1;
  }
  prefix_bidir_kernel<D, BN, FP16><<<grid, NUM_THREADS, C::SMEM_BYTES, stream>>>(maps[0], maps[1], maps[2], maps[3],
                                                                                 maps[4], prm);
  return d3b_host::check_launch();
}

template <int FP16>
int dispatch(int D, const CUtensorMap* maps, const Params& prm, dim3 grid, cudaStream_t s) {
  // D = 256 (O needs 256 TMEM columns): one tile per CTA, one CTA per SM.
  if (D == 256) return launch<256, 64, FP16>(maps, prm, grid, s);
  // D <= 128: one tile per CTA, two CTAs per SM.
  switch (D) {
    case 32: return launch_2c<32, FP16>(maps, prm, grid, s);
    case 64: return launch_2c<64, FP16>(maps, prm, grid, s);
    case 128: return launch_2c<128, FP16>(maps, prm, grid, s);
  }
  return D3B_EUNSUPPORTED;
}

}  // namespace

extern "C" int d3b_prefix_bidir(const void* q, const int64_t* q_strides, const void* k_state, const void* v_state,
                                const int64_t* kv_strides, const void* k_q, const void* v_q,
                                const int64_t* kq_strides, const int32_t* lengths, int B, int H, int Hkv, int S, int L,
                                int D, int dtype, float scale, void* out, const int64_t* out_strides,
                                d3b_stream_t stream) {
  if (B < 0 || H <= 0 || Hkv <= 0 || S < 0 || L < 0) return D3B_EINVAL;
  if (H % Hkv) return D3B_EINVAL;
  if (dtype != D3B_BF16 && dtype != D3B_F16) return D3B_EUNSUPPORTED;
  if (D != 32 && D != 64 && D != 128 && D != 256) return D3B_EUNSUPPORTED;
  const int G = H / Hkv;
  if (G > BM) return D3B_EUNSUPPORTED;
  if (!(scale > 0.f)) return D3B_EINVAL;
  if (B == 0 || L == 0) return D3B_OK;
  if (!q || !q_strides || !k_q || !v_q || !kq_strides || !lengths || !out || !out_strides) return D3B_EINVAL;
  if (S > 0 && (!k_state || !v_state || !kv_strides)) return D3B_EINVAL;
  if (B > 65535 || Hkv > 65535) return D3B_EINVAL;
  // every pointer 16-byte aligned and every stride a multiple of 8 elements
  const void* ptrs[6] = {q, k_q, v_q, out, S > 0 ? k_state : q, S > 0 ? v_state : q};
  for (const void* ptr : ptrs)
    if (reinterpret_cast<uintptr_t>(ptr) % 16) return D3B_EALIGN;
  for (int i = 0; i < 3; ++i)
    if (q_strides[i] % 8 || kq_strides[i] % 8 || out_strides[i] % 8 || q_strides[i] <= 0 || kq_strides[i] <= 0 ||
        out_strides[i] <= 0)
      return D3B_EALIGN;
  if (S > 0 && (kv_strides[0] % 8 || kv_strides[1] % 8 || kv_strides[0] <= 0 || kv_strides[1] <= 0))
    return D3B_EALIGN;

  const int CH = D >= 64 ? 64 : D;
  const CUtensorMapSwizzle sw = D >= 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  const CUtensorMapDataType dt = dtype == D3B_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const int BN = D == 256 ? 64 : 128;
  const int T = BM / G;

  CUtensorMap maps[5];
  int rc;
  {  // Q: [B, H, L, D] -> dims {D, H, L, B}, box {CH, G, T, 1}
    const uint64_t dims[4] = {(uint64_t)D, (uint64_t)H, (uint64_t)L, (uint64_t)B};
    const uint64_t st[3] = {(uint64_t)q_strides[1] * 2, (uint64_t)q_strides[2] * 2, (uint64_t)q_strides[0] * 2};
    const uint32_t box[4] = {(uint32_t)CH, (uint32_t)G, (uint32_t)T, 1};
    if ((rc = d3b_host::encode_tiled(&maps[0], dt, 4, q, dims, st, box, sw))) return rc;
  }
  {  // own-block K/V: [B, Hkv, L, D] -> dims {D, L, Hkv, B}, box {CH, BN, 1, 1}
    const uint64_t dims[4] = {(uint64_t)D, (uint64_t)L, (uint64_t)Hkv, (uint64_t)B};
    const uint64_t st[3] = {(uint64_t)kq_strides[2] * 2, (uint64_t)kq_strides[1] * 2, (uint64_t)kq_strides[0] * 2};
    const uint32_t box[4] = {(uint32_t)CH, (uint32_t)BN, 1, 1};
    if ((rc = d3b_host::encode_tiled(&maps[3], dt, 4, k_q, dims, st, box, sw))) return rc;
    if ((rc = d3b_host::encode_tiled(&maps[4], dt, 4, v_q, dims, st, box, sw))) return rc;
  }
  if (S > 0) {  // state K/V: [Hkv, S, D] -> dims {D, S, Hkv}, box {CH, BN, 1}
    const uint64_t dims[3] = {(uint64_t)D, (uint64_t)S, (uint64_t)Hkv};
    const uint64_t st[2] = {(uint64_t)kv_strides[1] * 2, (uint64_t)kv_strides[0] * 2};
    const uint32_t box[3] = {(uint32_t)CH, (uint32_t)BN, 1};
    if ((rc = d3b_host::encode_tiled(&maps[1], dt, 3, k_state, dims, st, box, sw))) return rc;
    if ((rc = d3b_host::encode_tiled(&maps[2], dt, 3, v_state, dims, st, box, sw))) return rc;
  } else {  // never read when S == 0
    maps[1] = maps[3];
    maps[2] = maps[4];
  }

  Params prm;
  prm.lengths = lengths;
  prm.out = out;
  prm.out_sb = out_strides[0];
  prm.out_sh = out_strides[1];
  prm.out_sl = out_strides[2];
  prm.H = H;
  prm.Hkv = Hkv;
  prm.G = G;
  prm.T = T;
  prm.S = S;
  prm.L = L;
  prm.scale_log2 = (float)((double)scale * 1.4426950408889634);
  prm.err = d3b_host::device_error_word();
  if (!prm.err) return D3B_ECUDA;

  const int tiles = (L + T - 1) / T;
  if (tiles > 0x7FFFFFFF) return D3B_EINVAL;
  dim3 grid(tiles, Hkv, B);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  return dtype == D3B_F16 ? dispatch<1>(D, maps, prm, grid, s) : dispatch<0>(D, maps, prm, grid, s);
}
