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
// Two kernels share this work unit, the key schedule and the softmax; both run
// one CTA per SM with S and P double-buffered in TMEM:
//   prefix_bidir_dual_kernel (every D): QK^T and PV issued by two threads,
//             two softmax warpgroups on alternating key tiles; 128-key tiles,
//             64-key tiles for D = 256 (O alone takes 256 TMEM columns).
//   prefix_bidir_kernel (D = 256 with D3B_ATTN_D256=single): one
//             MMA-issuing thread, one softmax warpgroup, 64-key tiles.
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

#include <algorithm>
#include <cstdlib>
#include <map>
#include <mutex>
#include <queue>
#include <string>
#include <tuple>
#include <vector>

namespace {

constexpr int BM = 128;
constexpr int NUM_THREADS = 192;
constexpr float kRescaleThreshold = 8.0f;  // log2 units: rescale O when max grows by > 2^8
#ifndef D3B_POLY8
#define D3B_POLY8 1  // FMA-pipe exponentials per eight pairs in the D <= 128 softmax
#endif

enum {
  kSiteQ = 2001,
  kSiteSlotEmpty = 2002,
  kSiteSlotFull = 2003,
  kSiteSFree = 2004,
  kSitePFull = 2005,
  kSiteSFull = 2006,
  kSitePFree = 2007,
  kSiteFinal = 2008,
  kSiteDrain = 2009,
  kSiteBadLength = 2010
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
  int last_arrival;  // split launch: this CTA's piece completed its unit
};

struct Params {
  const int32_t* lengths;
  void* out;
  int64_t out_sb, out_sh, out_sl;  // element strides
  // A Q tile holds G query heads (of one KV head's group) x T tokens. When the
  // group is split (hsplit > 1) into hsplit head groups of G heads each, Hkv
  // counts the head groups and K/V head = group / hsplit.
  int H, Hkv, G, T, S, L, hsplit;
  float scale_log2;
  int* err;
  // Launch plan of the D <= 128 kernel (1-D grid). Unit u = (b * Hkv + g) *
  // tiles + tile has n_full key-tile iterations (state tiles, then
  // ceil(L / BN) own tiles). CTA u < whole_units runs unit u whole. The last
  // split_units units run as `pieces` CTAs each: CTA whole_units + k *
  // split_units + r is piece k of unit whole_units + r, iterations
  // [0, piece0) for k = 0, then consecutive runs of piece_rest.
  int tiles, n_full, whole_units, split_units, pieces, piece0, piece_rest;
  float* part;  // split pieces' partial results, one slot per piece CTA
  int* count;   // per split unit: iterations accounted for (zero between launches)
};

// Real tokens of question block b. The table lives in device memory, so the
// host cannot check it: a value outside [0, L] is clamped (every access stays
// inside the caller's [B, *, L, D] tensors) and reported through the device
// error word (site kSiteBadLength), which voids the launch's results.
__device__ __forceinline__ int block_length(const Params& p, int b) {
  const int n = p.lengths[b];
  if (n < 0 || n > p.L) {
    d3b::record_device_error(p.err, kSiteBadLength);
    return n < 0 ? 0 : p.L;
  }
  return n;
}

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

// Max of N values (N a multiple of 8): three-input max, 8 independent
// accumulators (short dependency chains; about N/2 + 4 instructions).
template <int N>
__device__ __forceinline__ float max_n(const float* v) {
  static_assert(N >= 8 && N % 8 == 0, "max_n takes multiples of 8");
  float a[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) a[k] = v[k];
#pragma unroll
  for (int c = 8; c + 16 <= N; c += 16)
#pragma unroll
    for (int k = 0; k < 8; ++k) a[k] = max3(a[k], v[c + k], v[c + 8 + k]);
  if constexpr ((N - 8) % 16 == 8) {  // the last 8 values
#pragma unroll
    for (int k = 0; k < 8; ++k) a[k] = fmaxf(a[k], v[N - 8 + k]);
  }
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
// f16), returns the row sum of the fp32 values. POLY8 pairs in every eight go
// through the FMA-pipe exponential, the rest through MUFU ex2, so neither unit
// alone bounds the softmax.
template <int N, int FP16, int POLY8 = 2>
__device__ __forceinline__ float exp_row(const float* s, float sl2, float m, uint32_t* pk) {
  float part[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int c = 0; c < N; c += 2) {
    float x0, x1, p0, p1;
    fma2_bc(x0, x1, s[c], s[c + 1], sl2, -m);
    if (((c >> 1) & 7) >= 8 - POLY8) {
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

// Partial result of one piece of a split unit (fp32): O as [D/4][128 rows]
// float4 (a warp's 32 rows form one coalesced 512-byte run), then the row's
// reference max (log2 units, scale applied) m[128] and row sum l[128].
template <int D>
struct PartSlot {
  static constexpr int FLOATS = BM * D + 2 * BM;
};

// This CTA's unit and iteration range [a, e) in a launch with split units
// (1-D grid); slot >= 0 for a piece of a split unit.
__device__ __forceinline__ void cta_work(const Params& p, int& u, int& a, int& e, int& slot) {
  const int bid = blockIdx.x;
  if (bid < p.whole_units) {
    u = bid;
    a = 0;
    e = p.n_full;
    slot = -1;
    return;
  }
  const int q = bid - p.whole_units, k = q / p.split_units, r = q % p.split_units;
  u = p.whole_units + r;
  slot = q;
  a = k == 0 ? 0 : p.piece0 + (k - 1) * p.piece_rest;
  e = k == 0 ? p.piece0 : min(p.n_full, a + p.piece_rest);
}

// Adds this piece's iterations to its unit's count; true for the piece that
// completes the unit (which then merges every piece and resets the count).
__device__ __forceinline__ bool count_piece(const Params& p, int r, int add) {
  __threadfence();  // the CTA's partial rows (ordered before by a CTA barrier) before the count
  const int before = atomicAdd(&p.count[r], add);
  const bool last = before + add == p.n_full;
  if (last) {
    p.count[r] = 0;  // ready for the next launch
    __threadfence();
  }
  return last;
}

// Merge the pieces of split unit r for one row half (wg: columns [wg*D/2,
// (wg+1)*D/2)) and store it: O = sum_k 2^(m_k - m) O_k, l = sum_k 2^(m_k - m) l_k
// over the pieces with l_k > 0, output O / l (zero for padding rows).
template <int D, int FP16>
__device__ void merge_unit(const Params& p, int r, int b, int g, int tok0, int len_b, int wg, int row) {
  constexpr int OH = D / 2;
  const int tok = tok0 + row / p.G, h = row % p.G;
  if (!(row < p.G * p.T && tok < p.L)) return;
  const bool real = tok < len_b;
  float mx = -INFINITY;
  for (int k = 0; k < p.pieces; ++k) {
    const float* ps = p.part + (int64_t)(k * p.split_units + r) * PartSlot<D>::FLOATS;
    if (__ldcg(ps + BM * D + BM + row) > 0.f) mx = fmaxf(mx, __ldcg(ps + BM * D + row));
  }
  float acc[OH];
#pragma unroll
  for (int c = 0; c < OH; ++c) acc[c] = 0.f;
  float lt = 0.f;
  for (int k = 0; k < p.pieces; ++k) {
    const float* ps = p.part + (int64_t)(k * p.split_units + r) * PartSlot<D>::FLOATS;
    const float ls = __ldcg(ps + BM * D + BM + row);
    if (!(ls > 0.f)) continue;
    const float w = d3b::ex2_approx(__ldcg(ps + BM * D + row) - mx);
    lt += ls * w;
    const float4* os = reinterpret_cast<const float4*>(ps);
#pragma unroll
    for (int c = 0; c < OH; c += 4) {
      const float4 v = __ldcg(os + (wg * OH + c) / 4 * BM + row);
      acc[c] += v.x * w;
      acc[c + 1] += v.y * w;
      acc[c + 2] += v.z * w;
      acc[c + 3] += v.w * w;
    }
  }
  const float inv_l = 1.f / lt;
  uint4* dst = reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.out) + (int64_t)b * p.out_sb +
                                        (int64_t)(g * p.G + h) * p.out_sh + (int64_t)tok * p.out_sl + wg * OH);
#pragma unroll
  for (int c = 0; c < OH; c += 8) {
    uint4 v;
    v.x = real ? pack2<FP16>(acc[c] * inv_l, acc[c + 1] * inv_l) : 0u;
    v.y = real ? pack2<FP16>(acc[c + 2] * inv_l, acc[c + 3] * inv_l) : 0u;
    v.z = real ? pack2<FP16>(acc[c + 4] * inv_l, acc[c + 5] * inv_l) : 0u;
    v.w = real ? pack2<FP16>(acc[c + 6] * inv_l, acc[c + 7] * inv_l) : 0u;
    dst[c / 8] = v;
  }
}

// SPLIT: a launch with split units (1-D grid, the unit or piece of cta_work;
// a piece writes its partial to its slot and the piece that completes the
// unit merges them). Without it the grid is (tile, head group, block), one
// CTA per unit.
template <int D, int BN, int FP16, bool SPLIT>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    prefix_bidir_kernel(const __grid_constant__ CUtensorMap mapQ, const __grid_constant__ CUtensorMap mapKs,
                        const __grid_constant__ CUtensorMap mapVs, const __grid_constant__ CUtensorMap mapKq,
                        const __grid_constant__ CUtensorMap mapVq, const Params p) {
  using C = Cfg<D, BN>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ Bars bars;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int tile, g, b, unit = 0, a = 0, e = 0x7FFFFFFF, slot = -1;  // key tiles [a, e) of the unit
  if constexpr (SPLIT) {
    cta_work(p, unit, a, e, slot);
    tile = unit % p.tiles;
    g = (unit / p.tiles) % p.Hkv;
    b = unit / (p.tiles * p.Hkv);
  } else {
    tile = blockIdx.x;
    g = blockIdx.y;
    b = blockIdx.z;
  }
  const int kvh = g / p.hsplit;  // g: head group
  const int G = p.G, T = p.T;
  const int len_b = block_length(p, b);
  const int rows_used = G * T;
  const int tok0 = tile * T;

  // ---- rows of this tile that need no attention: zero-fill (once per unit) and leave ----
  if (tok0 >= len_b) {
    if (warp >= 2 && a == 0) {
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
  const int n = max(0, min(e, n_s + n_o) - a);  // this CTA's key tiles: a, a + 1, ..
  if constexpr (SPLIT) {
    if (n == 0) {
      // A piece of a split unit with no real key tile: an empty partial (l = 0),
      // counted in like any other piece.
      if (threadIdx.x < BM) {
        float* ps = p.part + (int64_t)slot * PartSlot<D>::FLOATS;
        ps[BM * D + threadIdx.x] = -INFINITY;
        ps[BM * D + BM + threadIdx.x] = 0.f;
      }
      __syncthreads();
      if (threadIdx.x == 0) bars.last_arrival = count_piece(p, unit - p.whole_units, e - a);
      __syncthreads();
      if (bars.last_arrival) {
        __threadfence();
        for (int i = threadIdx.x; i < 2 * BM; i += NUM_THREADS)
          merge_unit<D, FP16>(p, unit - p.whole_units, b, g, tok0, len_b, i / BM, i % BM);
      }
      return;
    }
  }

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
        const int kt = a + j;  // key tile of the unit
        if (kt < n_s) {
          const CUtensorMap* m = is_v ? &mapVs : &mapKs;
#pragma unroll
          for (int c = 0; c < C::NCH; ++c)
            d3b::tma_load_3d(dst + c * C::SLOT_CHUNK, m, &bars.slot_full[stage], c * C::CH, kt * BN, kvh);
        } else {
          const CUtensorMap* m = is_v ? &mapVq : &mapKq;
#pragma unroll
          for (int c = 0; c < C::NCH; ++c)
            d3b::tma_load_4d(dst + c * C::SLOT_CHUNK, m, &bars.slot_full[stage], c * C::CH, (kt - n_s) * BN, kvh, b);
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

      const int kt = a + j;  // key tile of the unit
      const int valid = kt < n_s ? p.S - kt * BN : len_b - (kt - n_s) * BN;
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
      // a piece of a split unit writes its raw O, m and l to its slot instead
      float* ps = nullptr;
      if constexpr (SPLIT) {
        if (slot >= 0) ps = p.part + (int64_t)slot * PartSlot<D>::FLOATS;
      }
      if (ps) {
        ps[BM * D + r] = m_ref;
        ps[BM * D + BM + r] = l_sum;
      }
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        d3b::tmem_ld32(lane_addr + C::COL_O + c * 32, o);
        d3b::tmem_wait_ld();
        if (ps) {
          uint4* os = reinterpret_cast<uint4*>(ps);
#pragma unroll
          for (int k = 0; k < 8; ++k)
            os[(c * 32 + 4 * k) / 4 * BM + r] = make_uint4(o[4 * k], o[4 * k + 1], o[4 * k + 2], o[4 * k + 3]);
        } else if (in_tensor) {
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
    if constexpr (SPLIT) {
      if (slot >= 0) {
        // Piece of a split unit: count it in; the piece that completes the unit
        // merges every piece's partial (both column halves of its row). Every
        // softmax thread reaches this point exactly once (failed waits only skip
        // work above), so the named barrier over the 128 softmax threads cannot
        // be left waiting.
        __threadfence();
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (threadIdx.x == 64)
          bars.last_arrival = *abort_flag ? 0 : (int)count_piece(p, unit - p.whole_units, e - a);
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (bars.last_arrival) {
          __threadfence();
          merge_unit<D, FP16>(p, unit - p.whole_units, b, g, tok0, len_b, 0, r);
          merge_unit<D, FP16>(p, unit - p.whole_units, b, g, tok0, len_b, 1, r);
        }
      }
    }
  }

  d3b::tc_fence_before();
  __syncthreads();
  d3b::tc_fence_after();
  if (warp == 1) d3b::tmem_dealloc(tmem_base, C::TMEM_COLS);
}

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

// ===========================================================================
// One Q tile per CTA, one CTA per SM, two MMA-issuing threads (D <= 128).
//
// A tcgen05.mma stream from one issuing thread runs an M128·N128·K16 bf16
// instruction in ~84 cycles (76% of the tensor rate); two threads issuing
// independent MMAs on the same SM share the tensor core at up to its full
// rate (measured on this B200: 128 cycles per instruction each when both
// streams use the same operand form, ~167 each for an SS stream next to a TS
// stream). So QK^T and PV get one issuing thread each:
//   warp 9  (lane 0)  S[j%2] = Q K_j^T   (SS: Q and K from shared memory)
//   warp 10 (lane 0)  O += P[j%2] V_j     (TS: P from TMEM, V from shared memory)
// TMEM (512 columns): O [0,D) | S0 [128,256) | S1 [256,384) | P0 [384,448) |
// P1 [448,512). With S and P double-buffered, QK(j+1) runs while the softmax
// works on S(j), and PV(j) while it works on S(j+1).
// Softmax: 8 warps in two groups of four, one thread per row in each group.
// Group 0 takes the even key tiles (S0, P0), group 1 the odd ones (S1, P1),
// so the two groups work half a tile apart and one group's waits overlap the
// other's arithmetic. The per-row reference max is handed from tile to tile
// through shared memory (see the softmax section).
// Warp 8 streams Q and then K_0, K_1, ... into the K ring (read by the QK
// thread), warp 11 streams V_0, V_1, ... into the V ring (read by the PV
// thread): each ring has one producer and one consumer that take its tiles in
// order (an mbarrier parity wait may not run more than one phase ahead), and
// K tiles never wait behind a full V ring.
// Bounds measured on this B200 for this design, per 128-key tile: tensor
// 16 x 64 cycles at the full rate; MUFU 128 x 128 exponentials / 16 per cycle
// = 1024 cycles (one pair in eight goes to the FMA pipe instead); shared
// memory 160 KB (Q, K, V operand reads + K/V TMA writes) at ~128 B/cycle.
// ===========================================================================
constexpr int DU_THREADS = 384;  // 8 softmax warps, K producer, QK issuer, PV issuer, V producer

template <int D>
struct CfgDual {
  static constexpr int BN = D == 256 ? 64 : 128;  // keys per tile (D = 256: O takes 256 TMEM columns)
  static constexpr int CH = D >= 64 ? 64 : D;
  static constexpr int ROWB = CH * 2;
  static constexpr int NCH = D / CH;
  static constexpr uint32_t LAYOUT = ROWB == 128 ? d3b::kLayoutSW128 : d3b::kLayoutSW64;
  static constexpr int SBO = 8 * ROWB;
  static constexpr int Q_BYTES = BM * D * 2;
  static constexpr int SLOT_BYTES = BN * D * 2;
  static constexpr int Q_CHUNK = BM * ROWB;
  static constexpr int SLOT_CHUNK = BN * ROWB;
  // 227 KB of shared memory per CTA, minus the static barriers/exchange arrays
  static constexpr int NSLOT_RAW = (227 * 1024 - 4096 - 1024 - Q_BYTES) / SLOT_BYTES;
  static constexpr int NK_RAW = (NSLOT_RAW + 1) / 2;
  static constexpr int NK = NK_RAW > 8 ? 8 : NK_RAW;                  // K ring slots
  static constexpr int NV = NSLOT_RAW - NK > 8 ? 8 : NSLOT_RAW - NK;  // V ring slots
  static constexpr int SMEM_BYTES = Q_BYTES + (NK + NV) * SLOT_BYTES + 1024;
  static constexpr int COL_O = 0;
  static constexpr int COL_S = D == 256 ? 256 : 128;  // + b * BN
  static constexpr int COL_P = COL_S + 2 * BN;        // + b * BN / 2 (384 either way)
  static constexpr int OH = D / 2;                    // O columns per softmax half
  static constexpr uint32_t TMEM_COLS = 512;
  static_assert(D <= COL_S && COL_P + BN <= (int)TMEM_COLS, "TMEM budget");
  static_assert(NK >= 2 && NV >= 2, "smem budget");
};

struct __align__(8) BarsDual {
  uint64_t q_full;
  uint64_t q_empty;  // the unit's QK^T MMAs have completed: Q may be reloaded
  uint64_t k_full[8], k_empty[8];  // K ring
  uint64_t v_full[8], v_empty[8];  // V ring
  uint64_t s_full[2];   // QK(j) committed into S[j%2]
  uint64_t s_free[2];   // softmax group j%2 has read S[j%2]
  uint64_t p_full[2];   // softmax group j%2 has written P[j%2]
  uint64_t p_free[2];   // PV(j) committed: P[j%2] is free and O holds PV(0..j)
  uint64_t mdone[2];    // reference max of tile j published (by group j%2)
  uint64_t xsum[4];     // per-group sums exchanged for the epilogue (per warp pair)
  uint64_t o_final;     // the unit's last PV committed: O is complete
  uint64_t o_free;      // the epilogue has read O: the next unit's first PV may overwrite it
  uint64_t drain_qk, drain_pv;
  uint32_t tmem_slot;
  int abort_flag;
  int last_arrival;  // split unit: this CTA's piece completed the unit
};

enum {
  kSiteDuQ = 6001, kSiteDuSlotK, kSiteDuSlotV, kSiteDuSlotEmpty, kSiteDuSFree, kSiteDuSFull, kSiteDuPFull,
  kSiteDuPFree, kSiteDuXMax, kSiteDuFinal, kSiteDuDrain
};

// Columns [c0, c0 + W) of this thread's TMEM row, scaled by f, written back (W = 16 or 32 multiple).
template <int W>
__device__ __forceinline__ void scale_cols(uint32_t addr, float f) {
  if constexpr (W % 32 == 0) {
#pragma unroll 1
    for (int c = 0; c < W / 32; ++c) {
      uint32_t o[32];
      d3b::tmem_ld32(addr + c * 32, o);
      d3b::tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * f);
      d3b::tmem_st32(addr + c * 32, o);
    }
  } else {
    static_assert(W == 16, "half-row width");
    uint32_t o[16];
    d3b::tmem_ld16(addr, o);
    d3b::tmem_wait_ld();
#pragma unroll
    for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * f);
    d3b::tmem_st16(addr, o);
  }
}

// One work item of the D <= 128 kernel: a unit (block b, kv head g, Q tile at
// token tok0) and its key-tile range [a, a + n); n == 0 when the tile holds no
// real token (its rows are zero-filled) or, in a split launch, when the piece
// has no real key tile.
struct Work {
  int unit, b, g, kvh, tok0, len_b, a, n;  // g: head group, kvh: its K/V head
};

// Item i of this CTA. Without SPLIT the launch is persistent: CTA c takes units
// c, c + gridDim.x, ... (all of a launch's units have the same number of key
// tiles up to the blocks' lengths, so a static round robin balances them).
// With SPLIT each CTA has one item, the unit or piece of cta_work.
template <bool SPLIT, int BN>
__device__ __forceinline__ bool work_item(const Params& p, int i, int n_s, Work& w) {
  int e;
  if constexpr (SPLIT) {
    if (i > 0) return false;
    int slot;
    cta_work(p, w.unit, w.a, e, slot);
  } else {
    w.unit = (int)blockIdx.x + i * (int)gridDim.x;
    if (w.unit >= p.whole_units) return false;
    w.a = 0;
    e = p.n_full;
  }
  const int tile = w.unit % p.tiles;
  w.g = (w.unit / p.tiles) % p.Hkv;
  w.kvh = w.g / p.hsplit;
  w.b = w.unit / (p.tiles * p.Hkv);
  w.len_b = block_length(p, w.b);
  w.tok0 = tile * p.T;
  w.n = w.tok0 >= w.len_b ? 0 : max(0, min(e, n_s + (w.len_b + BN - 1) / BN) - w.a);
  return true;
}

// SPLIT: the launch has split units (1-D grid, one unit or piece per CTA,
// partial merge). Without it the kernel is persistent: min(units, SMs) CTAs,
// each looping over its units with TMEM, the barriers and the rings set up
// once. Every ring, S/P buffer and barrier phase counts on across units (tile
// jg of the CTA's sequence, non-empty unit ie), so the next unit's Q and first
// K/V tiles load, and its first QK^T runs, while the softmax warps finish the
// previous unit's epilogue. Q is single-buffered: its load waits for the last
// QK^T of the previous unit (q_empty); O is reused: the first PV of a unit
// waits until the epilogue has read the previous unit's O (o_free).
template <int D, int FP16, bool SPLIT>
__global__ void __launch_bounds__(DU_THREADS, 1)
    prefix_bidir_dual_kernel(const __grid_constant__ CUtensorMap mapQ, const __grid_constant__ CUtensorMap mapKs,
                             const __grid_constant__ CUtensorMap mapVs, const __grid_constant__ CUtensorMap mapKq,
                             const __grid_constant__ CUtensorMap mapVq, const Params p) {
  using C = CfgDual<D>;
  constexpr int BN = C::BN;
  extern __shared__ uint8_t smem_raw[];
  __shared__ BarsDual bars;
  __shared__ float mref_s[2][BM];   // reference max of the last tile of each group, per row
  __shared__ float lsum_s[2][BM];   // epilogue exchange: running sums and their references
  __shared__ float mlast_s[2][BM];
  __shared__ int work_s[4];  // split launch: unit, end of range, slot, start of range (reloaded where used)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.G, T = p.T;
  const int rows_used = G * T;
  const int n_s = (p.S + BN - 1) / BN;
  if constexpr (SPLIT) {
    int unit, a, e, slot;
    cta_work(p, unit, a, e, slot);
    const int tile = unit % p.tiles, g = (unit / p.tiles) % p.Hkv, b = unit / (p.tiles * p.Hkv);
    const int len_b = block_length(p, b);
    const int tok0 = tile * T;
    if (tok0 >= len_b) {  // no real token in this tile: zero-fill (once per unit) and leave
      if (warp < 4 && a == 0) zero_tile_rows<D>(p, b, g, tok0, warp, lane);
      return;
    }
    const int n = max(0, min(e, n_s + (len_b + BN - 1) / BN) - a);
    if (n == 0) {
      // A piece of a split unit with no real key tile: an empty partial (l = 0),
      // counted in like any other piece.
      if (threadIdx.x < BM) {
        float* ps = p.part + (int64_t)slot * PartSlot<D>::FLOATS;
        ps[BM * D + threadIdx.x] = -INFINITY;
        ps[BM * D + BM + threadIdx.x] = 0.f;
      }
      __syncthreads();
      if (threadIdx.x == 0) bars.last_arrival = count_piece(p, unit - p.whole_units, e - a);
      __syncthreads();
      if (bars.last_arrival && threadIdx.x < 2 * BM) {
        __threadfence();
        merge_unit<D, FP16>(p, unit - p.whole_units, b, g, tok0, len_b, threadIdx.x / BM, threadIdx.x % BM);
      }
      return;
    }
    if (threadIdx.x == 0) {
      work_s[0] = unit;
      work_s[1] = e;
      work_s[2] = slot;
      work_s[3] = a;
    }
  }
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = smem + C::Q_BYTES;
  uint8_t* sV = sK + C::NK * C::SLOT_BYTES;
  volatile int* abort_flag = &bars.abort_flag;

  if (threadIdx.x == 0) {
    d3b::mbar_init(&bars.q_full, 1);
    d3b::mbar_init(&bars.q_empty, 1);
    for (int i = 0; i < 8; ++i) {
      d3b::mbar_init(&bars.k_full[i], 1);
      d3b::mbar_init(&bars.k_empty[i], 1);
      d3b::mbar_init(&bars.v_full[i], 1);
      d3b::mbar_init(&bars.v_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      d3b::mbar_init(&bars.s_full[i], 1);
      d3b::mbar_init(&bars.s_free[i], 128);
      d3b::mbar_init(&bars.p_full[i], 128);
      d3b::mbar_init(&bars.p_free[i], 1);
      d3b::mbar_init(&bars.mdone[i], 128);
    }
    for (int q = 0; q < 4; ++q) d3b::mbar_init(&bars.xsum[q], 64);
    d3b::mbar_init(&bars.o_final, 1);
    d3b::mbar_init(&bars.o_free, 256);
    d3b::mbar_init(&bars.drain_qk, 1);
    d3b::mbar_init(&bars.drain_pv, 1);
    bars.abort_flag = 0;
    d3b::fence_barrier_init();
  }
  if (rows_used < BM) {  // rows no Q box covers stay zero for every unit
    const int per_chunk = (BM - rows_used) * C::ROWB / 16;
    for (int i = threadIdx.x; i < C::NCH * per_chunk; i += DU_THREADS) {
      const int c = i / per_chunk, o = i % per_chunk;
      reinterpret_cast<uint4*>(sQ + c * C::Q_CHUNK + rows_used * C::ROWB)[o] = make_uint4(0, 0, 0, 0);
    }
    d3b::fence_proxy_async_smem();
  }
  if (warp == 9) d3b::tmem_alloc(&bars.tmem_slot, C::TMEM_COLS);
  d3b::tc_fence_before();
  __syncthreads();
  d3b::tc_fence_after();
  const uint32_t tmem_base = bars.tmem_slot;
  constexpr uint32_t fmt = FP16 ? 0u : 1u;

  if (warp >= 8) {
    // Registers: launched at 168 per thread (384 threads); the producer / MMA
    // warpgroup gives back to 48 and the softmax warpgroups rise to 224
    // (128 * 48 + 256 * 224 = 63488 <= 384 * 168), so a softmax thread keeps
    // a whole 128-key row of S in registers.
    asm volatile("setmaxnreg.dec.sync.aligned.u32 48;" ::: "memory");
   if (warp == 8 || warp == 11) {
    // ================= TMA producers: warp 8 Q and K tiles, warp 11 V tiles =================
    // (one producer per ring, so K tiles never wait behind a full V ring)
    if (lane == 0) {
      const bool is_v = warp == 11;
      if (is_v) {
        if (n_s) d3b::tma_prefetch_desc(&mapVs);
        d3b::tma_prefetch_desc(&mapVq);
      } else {
        d3b::tma_prefetch_desc(&mapQ);
        d3b::tma_prefetch_desc(&mapKq);
        if (n_s) d3b::tma_prefetch_desc(&mapKs);
      }
      const int nslot = is_v ? C::NV : C::NK;
      uint64_t* fulls = is_v ? bars.v_full : bars.k_full;
      uint64_t* empties = is_v ? bars.v_empty : bars.k_empty;
      uint8_t* ring = is_v ? sV : sK;
      const CUtensorMap* m_state = is_v ? &mapVs : &mapKs;
      const CUtensorMap* m_own = is_v ? &mapVq : &mapKq;
      int slot = 0, ie = 0;
      uint32_t ph = 0;
      bool ok = true;
      Work w;
      for (int i = 0; ok && work_item<SPLIT, BN>(p, i, n_s, w); ++i) {
        if (w.n == 0) continue;
        if (!is_v) {
          // Q of this unit: the previous unit's QK^T MMAs have all completed
          if (ie > 0 && !(ok = d3b::mbar_wait(&bars.q_empty, (uint32_t)(ie - 1) & 1, abort_flag, p.err, kSiteDuQ)))
            break;
          d3b::mbar_arrive_expect_tx(&bars.q_full, C::NCH * rows_used * C::ROWB);
#pragma unroll
          for (int c = 0; c < C::NCH; ++c)
            d3b::tma_load_4d(sQ + c * C::Q_CHUNK, &mapQ, &bars.q_full, c * C::CH, w.g * G, w.tok0, w.b);
        }
        for (int j = 0; j < w.n; ++j) {
          if (!(ok = d3b::mbar_wait(&empties[slot], ph ^ 1, abort_flag, p.err, kSiteDuSlotEmpty))) break;
          uint64_t* full = &fulls[slot];
          uint8_t* dst = ring + slot * C::SLOT_BYTES;
          d3b::mbar_arrive_expect_tx(full, C::SLOT_BYTES);
          const int kt = w.a + j;  // key tile of the unit
          if (kt < n_s) {
#pragma unroll
            for (int c = 0; c < C::NCH; ++c)
              d3b::tma_load_3d(dst + c * C::SLOT_CHUNK, m_state, full, c * C::CH, kt * BN, w.kvh);
          } else {
#pragma unroll
            for (int c = 0; c < C::NCH; ++c)
              d3b::tma_load_4d(dst + c * C::SLOT_CHUNK, m_own, full, c * C::CH, (kt - n_s) * BN, w.kvh, w.b);
          }
          if (++slot == nslot) { slot = 0; ph ^= 1; }
        }
        ++ie;
      }
    }
  } else if (warp == 9) {
    // ================= QK^T issuer =================
    if (lane == 0) {
      constexpr uint32_t idesc_qk = d3b::make_idesc(1, fmt, fmt, 0, 0, BM, BN);
      const uint64_t dq0 = d3b::make_smem_desc(d3b::smem_u32(sQ), 16, C::SBO, C::LAYOUT);
      const uint64_t dk0 = d3b::make_smem_desc(d3b::smem_u32(sK), 16, C::SBO, C::LAYOUT);
      bool ok = true;
      int jg = 0, ie = 0;
      Work w;
      for (int i = 0; ok && work_item<SPLIT, BN>(p, i, n_s, w); ++i) {
        if (w.n == 0) continue;
        if (!(ok = d3b::mbar_wait(&bars.q_full, (uint32_t)ie & 1, abort_flag, p.err, kSiteDuQ))) break;
        for (int j = 0; j < w.n; ++j, ++jg) {
          const int sb = jg & 1;
          const uint32_t u = (uint32_t)(jg >> 1);
          // S[sb] was last read by the softmax of tile jg-2
          if (!(ok = d3b::mbar_wait(&bars.s_free[sb], (u & 1) ^ 1, abort_flag, p.err, kSiteDuSFree))) break;
          const int slot = jg % C::NK;
          if (!(ok = d3b::mbar_wait(&bars.k_full[slot], (uint32_t)(jg / C::NK) & 1, abort_flag, p.err,
                                    kSiteDuSlotK)))
            break;
          d3b::tc_fence_after();
          const uint64_t dk = dk0 + (uint64_t)((slot * C::SLOT_BYTES) >> 4);
#pragma unroll
          for (int k = 0; k < D / 16; ++k) {
            const int c = (k * 16) / C::CH, off = ((k * 16) % C::CH) * 2;
            d3b::mma_f16_ss(tmem_base + C::COL_S + sb * BN, dq0 + (uint64_t)((c * C::Q_CHUNK + off) >> 4),
                            dk + (uint64_t)((c * C::SLOT_CHUNK + off) >> 4), idesc_qk, k > 0 ? 1u : 0u);
          }
          d3b::mma_commit(&bars.s_full[sb]);
          d3b::mma_commit(&bars.k_empty[slot]);
        }
        if (!ok) break;
        d3b::mma_commit(&bars.q_empty);  // the unit's QK^T MMAs have read Q
        ++ie;
      }
      d3b::mma_commit(&bars.drain_qk);
      const uint32_t addr = d3b::smem_u32(&bars.drain_qk);
      const uint64_t t0 = d3b::globaltimer_ns();
      while (!d3b::mbar_try_wait(addr, 0)) {
        if (d3b::globaltimer_ns() - t0 > D3B_WAIT_LIMIT_NS) {
          d3b::record_device_error(p.err, kSiteDuDrain);
          break;
        }
      }
    }
  } else if (warp == 10) {
    // ================= PV issuer =================
    if (lane == 0) {
      constexpr uint32_t idesc_pv = d3b::make_idesc(1, fmt, fmt, 0, 1, BM, D);
      const uint64_t dv0 = d3b::make_smem_desc(d3b::smem_u32(sV), C::SLOT_CHUNK, C::SBO, C::LAYOUT);
      bool ok = true;
      int jg = 0, ie = 0;
      Work w;
      for (int i = 0; ok && work_item<SPLIT, BN>(p, i, n_s, w); ++i) {
        if (w.n == 0) continue;
        for (int j = 0; j < w.n; ++j, ++jg) {
          const int sb = jg & 1;
          const uint32_t u = (uint32_t)(jg >> 1);
          if (!(ok = d3b::mbar_wait(&bars.p_full[sb], u & 1, abort_flag, p.err, kSiteDuPFull))) break;
          // O of the previous unit has been read by the epilogue before this unit's first PV overwrites it
          if (j == 0 && ie > 0 &&
              !(ok = d3b::mbar_wait(&bars.o_free, (uint32_t)(ie - 1) & 1, abort_flag, p.err, kSiteDuFinal)))
            break;
          const int slot = jg % C::NV;
          if (!(ok = d3b::mbar_wait(&bars.v_full[slot], (uint32_t)(jg / C::NV) & 1, abort_flag, p.err,
                                    kSiteDuSlotV)))
            break;
          d3b::tc_fence_after();
          const uint64_t dv = dv0 + (uint64_t)((slot * C::SLOT_BYTES) >> 4);
#pragma unroll
          for (int k = 0; k < BN / 16; ++k)
            d3b::mma_f16_ts(tmem_base + C::COL_O, tmem_base + C::COL_P + sb * (BN / 2) + k * 8,
                            dv + (uint64_t)((k * 16 * C::ROWB) >> 4), idesc_pv, (j > 0 || k > 0) ? 1u : 0u);
          d3b::mma_commit(&bars.p_free[sb]);
          d3b::mma_commit(&bars.v_empty[slot]);
        }
        if (!ok) break;
        d3b::mma_commit(&bars.o_final);  // O holds the unit's PV(0..n-1)
        ++ie;
      }
      d3b::mma_commit(&bars.drain_pv);
      const uint32_t addr = d3b::smem_u32(&bars.drain_pv);
      const uint64_t t0 = d3b::globaltimer_ns();
      while (!d3b::mbar_try_wait(addr, 0)) {
        if (d3b::globaltimer_ns() - t0 > D3B_WAIT_LIMIT_NS) {
          d3b::record_device_error(p.err, kSiteDuDrain);
          break;
        }
      }
    }
   }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 224;" ::: "memory");
    // ================= softmax + epilogue (warps 0-7) =================
    // Group wg (warps 4wg .. 4wg+3, one thread per row) takes the key tiles of
    // odd or even position jg in the CTA's tile sequence, with S[wg] and P[wg].
    // Within a unit both groups scale P by the same per-row reference max,
    // decided tile by tile in order: tile jg reads the reference of tile jg-1
    // (from the other group, through shared memory), raises it only if its own
    // max exceeds it by more than 2^8, and publishes its own; the first tile of
    // a unit ignores the value it reads (the wait keeps the groups in step).
    // Each group keeps its own running sum l (with the reference of its last
    // tile); the two are combined in the epilogue.
    const int wg = warp >> 2, quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_addr = tmem_base + ((uint32_t)(quarter * 32) << 16);
    const uint32_t col_s = C::COL_S + wg * BN, col_p = C::COL_P + wg * (BN / 2);
    const float sl2 = p.scale_log2;
    bool ok = true;
    int jg = 0, ie = 0;
    Work w;
    for (int i = 0; ok && work_item<SPLIT, BN>(p, i, n_s, w); ++i) {
      if (w.n == 0) {
        if (wg == 0) zero_tile_rows<D>(p, w.b, w.g, w.tok0, quarter, lane);
        continue;
      }
      float m_last = -INFINITY, l_sum = 0.f;
      for (int j = (wg ^ jg) & 1; j < w.n; j += 2) {
        const int t = jg + j;
        const uint32_t u = (uint32_t)(t >> 1);
        if (!d3b::warp_wait(&bars.s_full[wg], u & 1, abort_flag, p.err, kSiteDuSFull)) { ok = false; break; }
        d3b::tc_fence_after();
        float s[BN];
#pragma unroll
        for (int c = 0; c < BN / 32; ++c)
          d3b::tmem_ld32(lane_addr + col_s + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&s[c * 32]));
        d3b::tmem_wait_ld();
        d3b::tc_fence_before();
        d3b::mbar_arrive(&bars.s_free[wg]);
        const int kt = w.a + j;  // key tile of the unit
        const int valid = kt < n_s ? p.S - kt * BN : w.len_b - (kt - n_s) * BN;
        if (valid < BN) {
#pragma unroll
          for (int c = 0; c < BN; ++c)
            if (c >= valid) s[c] = -INFINITY;
        }
        const float m_tile = max_n<BN>(s) * sl2;
        float m_prev = -INFINITY;
        if (t > 0) {
          if (!d3b::warp_wait(&bars.mdone[(t - 1) & 1], (uint32_t)((t - 1) >> 1) & 1, abort_flag, p.err,
                              kSiteDuXMax)) {
            ok = false;
            break;
          }
          if (j > 0) m_prev = mref_s[(t - 1) & 1][r];
        }
        // Lazy rescale, decided per warp: tcgen05.ld/st are warp-collective.
        const bool rescale = __any_sync(0xffffffffu, m_tile > m_prev + kRescaleThreshold);
        const float m_new = rescale ? fmaxf(m_prev, m_tile) : m_prev;
        mref_s[wg][r] = m_new;
        d3b::mbar_arrive(&bars.mdone[wg]);
        if (rescale && j > 0) {
          // O holds PV(0..j-1) scaled to m_prev: wait for PV(j-1), then rescale
          if (!d3b::warp_wait(&bars.p_free[(t - 1) & 1], (uint32_t)((t - 1) >> 1) & 1, abort_flag, p.err,
                              kSiteDuPFree)) {
            ok = false;
            break;
          }
          d3b::tc_fence_after();
          scale_cols<D>(lane_addr + C::COL_O, d3b::ex2_approx(m_prev - m_new));
        }
        // P[wg] is free once PV(t-2) has completed
        if (!d3b::warp_wait(&bars.p_free[wg], (u & 1) ^ 1, abort_flag, p.err, kSiteDuPFree)) { ok = false; break; }
        d3b::tc_fence_after();
        float rowsum = 0.f;
#pragma unroll
        for (int qq = 0; qq < BN / 32; ++qq) {
          uint32_t pk[16];
          rowsum += exp_row<32, FP16, D3B_POLY8>(s + qq * 32, sl2, m_new, pk);
          d3b::tmem_st16(lane_addr + col_p + qq * 16, pk);
        }
        d3b::tmem_wait_st();
        d3b::tc_fence_before();
        d3b::mbar_arrive(&bars.p_full[wg]);
        l_sum = (m_last == m_new ? l_sum : l_sum * d3b::ex2_approx(m_last - m_new)) + rowsum;
        m_last = m_new;
      }
      if (ok) ok = d3b::warp_wait(&bars.o_final, (uint32_t)ie & 1, abort_flag, p.err, kSiteDuFinal);
      if (ok) {
        lsum_s[wg][r] = l_sum;
        mlast_s[wg][r] = m_last;
        d3b::mbar_arrive(&bars.xsum[quarter]);
        ok = d3b::warp_wait(&bars.xsum[quarter], (uint32_t)ie & 1, abort_flag, p.err, kSiteDuXMax);
      }
      if (!ok) break;
      d3b::tc_fence_after();
      // O is scaled to the last tile's reference, the larger of the two groups' last references
      const float m0 = mlast_s[0][r], m1 = mlast_s[1][r];
      const float m_fin = fmaxf(m0, m1);
      const float l = lsum_s[0][r] * d3b::ex2_approx(m0 - m_fin) + lsum_s[1][r] * d3b::ex2_approx(m1 - m_fin);
      const int tok = w.tok0 + r / G, h = r % G;
      const bool in_tensor = r < rows_used && tok < p.L;
      const bool real = tok < w.len_b;
      const float inv_l = 1.f / l;
      // each group normalises and stores half of the D columns (a piece of a
      // split unit writes its raw half of O, with m and l, to its slot instead)
      uint16_t* dst_row = static_cast<uint16_t*>(p.out) + (int64_t)w.b * p.out_sb +
                          (int64_t)(w.g * G + h) * p.out_sh + (int64_t)tok * p.out_sl + wg * C::OH;
      float* ps = nullptr;
      if constexpr (SPLIT) {
        const int slot_e = reinterpret_cast<volatile int*>(work_s)[2];
        if (slot_e >= 0) ps = p.part + (int64_t)slot_e * PartSlot<D>::FLOATS;
      }
      if (ps && wg == 0) {
        ps[BM * D + r] = m_fin;
        ps[BM * D + BM + r] = l;
      }
      if constexpr (C::OH % 32 == 0) {
        uint32_t o[C::OH];
#pragma unroll
        for (int c = 0; c < C::OH / 32; ++c)
          d3b::tmem_ld32(lane_addr + C::COL_O + wg * C::OH + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&o[c * 32]));
        d3b::tmem_wait_ld();
        // O is in registers: the next unit's first PV may overwrite it
        d3b::tc_fence_before();
        d3b::mbar_arrive(&bars.o_free);
        if (ps) {
          uint4* os = reinterpret_cast<uint4*>(ps);
#pragma unroll
          for (int k = 0; k < C::OH / 4; ++k)
            os[(wg * C::OH + 4 * k) / 4 * BM + r] = make_uint4(o[4 * k], o[4 * k + 1], o[4 * k + 2], o[4 * k + 3]);
        } else if (in_tensor) {
          uint4* dst = reinterpret_cast<uint4*>(dst_row);
#pragma unroll
          for (int i8 = 0; i8 < C::OH / 8; ++i8) {
            uint32_t v[4];
#pragma unroll
            for (int k = 0; k < 4; ++k)
              v[k] = real ? pack2<FP16>(__uint_as_float(o[8 * i8 + 2 * k]) * inv_l,
                                        __uint_as_float(o[8 * i8 + 2 * k + 1]) * inv_l)
                          : 0u;
            dst[i8] = make_uint4(v[0], v[1], v[2], v[3]);
          }
        }
      } else {
        uint32_t o[16];
        d3b::tmem_ld16(lane_addr + C::COL_O + wg * C::OH, o);
        d3b::tmem_wait_ld();
        d3b::tc_fence_before();
        d3b::mbar_arrive(&bars.o_free);
        if (ps) {
          uint4* os = reinterpret_cast<uint4*>(ps);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            os[(wg * C::OH + 4 * k) / 4 * BM + r] = make_uint4(o[4 * k], o[4 * k + 1], o[4 * k + 2], o[4 * k + 3]);
        } else if (in_tensor) {
          uint32_t v[8];
#pragma unroll
          for (int k = 0; k < 8; ++k)
            v[k] = real ? pack2<FP16>(__uint_as_float(o[2 * k]) * inv_l, __uint_as_float(o[2 * k + 1]) * inv_l) : 0u;
          uint4* dst = reinterpret_cast<uint4*>(dst_row);
          dst[0] = make_uint4(v[0], v[1], v[2], v[3]);
          dst[1] = make_uint4(v[4], v[5], v[6], v[7]);
        }
      }
      jg += w.n;
      ++ie;
    }
    if constexpr (SPLIT) {
      const volatile int* wv = work_s;
      if (wv[2] >= 0) {
        const int unit_e = wv[0], end_e = wv[1];
        const int b = unit_e / (p.tiles * p.Hkv), g = (unit_e / p.tiles) % p.Hkv, tok0 = (unit_e % p.tiles) * T;
        // Piece of a split unit: count it in; the piece that completes the unit
        // merges every piece's partial. Every softmax thread reaches this point
        // exactly once (failed waits only skip work above), so the named barrier
        // over the 256 softmax threads cannot be left waiting.
        __threadfence();
        asm volatile("bar.sync 1, 256;" ::: "memory");
        if (threadIdx.x == 0)
          bars.last_arrival = *abort_flag ? 0 : (int)count_piece(p, unit_e - p.whole_units, end_e - wv[3]);
        asm volatile("bar.sync 1, 256;" ::: "memory");
        if (bars.last_arrival) {
          __threadfence();
          merge_unit<D, FP16>(p, unit_e - p.whole_units, b, g, tok0, block_length(p, b), wg, r);
        }
      }
    }
  }

  d3b::tc_fence_before();
  __syncthreads();
  d3b::tc_fence_after();
  if (warp == 9) d3b::tmem_dealloc(tmem_base, C::TMEM_COLS);
}

template <int D, int FP16, bool SPLIT>
int launch_dual_as(const CUtensorMap* maps, const Params& prm, dim3 grid, cudaStream_t stream) {
  using C = CfgDual<D>;
  static int attr_set[64] = {0};
  const int dev = d3b_host::current_device();
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    if (cudaFuncSetAttribute(prefix_bidir_dual_kernel<D, FP16, SPLIT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             C::SMEM_BYTES) != cudaSuccess)
      return D3B_ECUDA;
    attr_set[dev] = 1;
  }
  prefix_bidir_dual_kernel<D, FP16, SPLIT><<<grid, DU_THREADS, C::SMEM_BYTES, stream>>>(maps[0], maps[1], maps[2],
                                                                                       maps[3], maps[4], prm);
  return d3b_host::check_launch();
}

template <int D, int FP16>
int launch_dual(const CUtensorMap* maps, const Params& prm, dim3 grid, cudaStream_t stream) {
  return prm.split_units ? launch_dual_as<D, FP16, true>(maps, prm, grid, stream)
                         : launch_dual_as<D, FP16, false>(maps, prm, grid, stream);
}

// ===========================================================================
// CTA-pair form of the D = 128 kernel (cluster of 2, tcgen05 cta_group::2).
//
// Bounds of the one-CTA kernel above, per 128-key tile: tensor 1024 cycles,
// MUFU ~900, shared memory 160 KB at ~128 B/cycle (~1250 cycles) - the SS
// QK^T at N = 128 alone reads its operands at the full shared-memory rate. A
// pair of CTAs on two SMs takes two Q tiles of the same (block, kv head) as one
// M = 256 operand: S = Q K^T is one M256·N128 MMA whose B operand (the key
// tile) is split between the CTAs (CTA r holds keys 64r .. 64r+63, both
// 64-column halves of D), and O += P V one M256·N128 MMA whose B operand (the
// value tile) is split by columns (CTA r holds all 128 keys, columns
// 64r .. 64r+63). Each SM then writes 32 KB of K/V per tile instead of 64 and
// reads 96 KB of operands instead of 128: ~96 KB per tile, under the tensor
// bound.
//   rank 0, warp 9  (lane 0)  S[j%2] = Q K_j^T for both CTAs
//   rank 0, warp 10 (lane 0)  O += P[j%2] V_j for both CTAs
//   both ranks, warp 8: this CTA's Q tile and key halves; warp 11: value halves;
//     the loads complete on rank 0's full barriers, which rank 0 arms with the
//     pair's bytes
//   both ranks, warps 0-7: softmax and epilogue of this CTA's 128 rows, as in
//     the one-CTA kernel; the barriers the issuers wait on (s_free, p_full,
//     o_free) live in rank 0 and count both CTAs' threads, the ones the CTA's
//     own threads wait on (s_full, p_free, o_final, q_empty, k/v_empty) get the
//     issuer's commits in both CTAs (tcgen05.commit multicast).
// Units: pair unit = (block b, kv head g, Q tiles 2t and 2t+1); rank r takes
// tile 2t + r. Both ranks run the same number of key tiles (the lower tile's
// count: it always holds the block's first tokens), so a tile with no real
// token computes rows that its epilogue writes as zeros. Launch: persistent,
// one cluster per two SMs, clusters walking the pair units; used when every
// (block, kv head) has an even number of Q tiles.
// ===========================================================================
struct CfgPair {
  static constexpr int D = 128, BN = 128, CH = 64, ROWB = 128, NCH = 2;
  static constexpr uint32_t LAYOUT = d3b::kLayoutSW128;
  static constexpr int SBO = 8 * ROWB;
  static constexpr int Q_BYTES = BM * D * 2;      // this CTA's 128 rows
  static constexpr int Q_CHUNK = BM * ROWB;
  static constexpr int K_ROWS = BN / 2;           // this CTA's keys of a key tile
  static constexpr int K_CHUNK = K_ROWS * ROWB;   // 8 KB
  static constexpr int SLOT_BYTES = NCH * K_CHUNK;  // 16 KB: a key half, or a value half (128 keys x 64 columns)
  static constexpr int NSLOT = (227 * 1024 - 4096 - 1024 - Q_BYTES) / SLOT_BYTES;
  static constexpr int NK = NSLOT / 2 + NSLOT % 2 > 8 ? 8 : NSLOT / 2 + NSLOT % 2;
  static constexpr int NV = NSLOT - NK > 8 ? 8 : NSLOT - NK;
  static constexpr int SMEM_BYTES = Q_BYTES + (NK + NV) * SLOT_BYTES + 1024;
  static constexpr int COL_O = 0, COL_S = 128, COL_P = 384, OH = D / 2;
  static constexpr uint32_t TMEM_COLS = 512;
  static_assert(NK >= 2 && NV >= 2, "smem budget");
};

// Pair unit i of this cluster (persistent: clusters walk the pair units).
__device__ __forceinline__ bool pair_item(const Params& p, int i, int n_s, uint32_t rank, Work& w) {
  const int half_tiles = p.tiles >> 1;
  const int pu = (int)(blockIdx.x >> 1) + i * (int)(gridDim.x >> 1);
  if (pu >= p.whole_units) return false;  // whole_units counts pair units in this launch
  const int tp = pu % half_tiles;
  w.g = (pu / half_tiles) % p.Hkv;
  w.kvh = w.g / p.hsplit;
  w.b = pu / (half_tiles * p.Hkv);
  w.unit = pu;
  w.len_b = block_length(p, w.b);
  w.tok0 = (2 * tp + (int)rank) * p.T;
  w.a = 0;
  const int tok_lo = 2 * tp * p.T;
  w.n = tok_lo >= w.len_b ? 0 : min(p.n_full, n_s + (w.len_b + 127) / 128);
  return true;
}

template <int FP16>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(DU_THREADS, 1)
    prefix_bidir_pair_kernel(const __grid_constant__ CUtensorMap mapQ, const __grid_constant__ CUtensorMap mapKs,
                             const __grid_constant__ CUtensorMap mapVs, const __grid_constant__ CUtensorMap mapKq,
                             const __grid_constant__ CUtensorMap mapVq, const Params p) {
  using C = CfgPair;
  constexpr int D = C::D, BN = C::BN;
  extern __shared__ uint8_t smem_raw[];
  __shared__ BarsDual bars;
  __shared__ float mref_s[2][BM];
  __shared__ float lsum_s[2][BM];
  __shared__ float mlast_s[2][BM];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = d3b::cluster_ctarank();
  const int G = p.G;
  const int rows_used = G * p.T;
  const int n_s = (p.S + BN - 1) / BN;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = smem + C::Q_BYTES;
  uint8_t* sV = sK + C::NK * C::SLOT_BYTES;
  volatile int* abort_flag = &bars.abort_flag;

  if (threadIdx.x == 0) {
    d3b::mbar_init(&bars.q_full, 1);
    d3b::mbar_init(&bars.q_empty, 1);
    for (int i = 0; i < 8; ++i) {
      d3b::mbar_init(&bars.k_full[i], 1);
      d3b::mbar_init(&bars.k_empty[i], 1);
      d3b::mbar_init(&bars.v_full[i], 1);
      d3b::mbar_init(&bars.v_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      d3b::mbar_init(&bars.s_full[i], 1);
      d3b::mbar_init(&bars.s_free[i], 2 * 128);  // rank 0's: both CTAs' group i
      d3b::mbar_init(&bars.p_full[i], 2 * 128);  // rank 0's: both CTAs' group i
      d3b::mbar_init(&bars.p_free[i], 1);
      d3b::mbar_init(&bars.mdone[i], 128);
    }
    for (int q = 0; q < 4; ++q) d3b::mbar_init(&bars.xsum[q], 64);
    d3b::mbar_init(&bars.o_final, 1);
    d3b::mbar_init(&bars.o_free, 2 * 256);  // rank 0's: both CTAs' epilogues
    d3b::mbar_init(&bars.drain_qk, 1);
    d3b::mbar_init(&bars.drain_pv, 1);
    bars.abort_flag = 0;
    d3b::fence_barrier_init();
  }
  if (rows_used < BM) {  // rows no Q box covers stay zero for every unit
    const int per_chunk = (BM - rows_used) * C::ROWB / 16;
    for (int i = threadIdx.x; i < C::NCH * per_chunk; i += DU_THREADS) {
      const int c = i / per_chunk, o = i % per_chunk;
      reinterpret_cast<uint4*>(sQ + c * C::Q_CHUNK + rows_used * C::ROWB)[o] = make_uint4(0, 0, 0, 0);
    }
    d3b::fence_proxy_async_smem();
  }
  if (warp == 9) d3b::tmem_alloc_pair(&bars.tmem_slot, C::TMEM_COLS);
  d3b::tc_fence_before();
  d3b::cluster_sync();  // both CTAs' barriers initialised before any remote arrive, load or commit
  d3b::tc_fence_after();
  const uint32_t tmem_base = bars.tmem_slot;
  constexpr uint32_t fmt = FP16 ? 0u : 1u;

  if (warp >= 8) {
    // Register split as in the one-CTA kernel: 128 * 48 + 256 * 224 <= 384 * 168.
    asm volatile("setmaxnreg.dec.sync.aligned.u32 48;" ::: "memory");
   if (warp == 8 || warp == 11) {
    // ======== TMA producers (both ranks): warp 8 Q and key halves, warp 11 value halves ========
    if (lane == 0) {
      const bool is_v = warp == 11;
      if (is_v) {
        if (n_s) d3b::tma_prefetch_desc(&mapVs);
        d3b::tma_prefetch_desc(&mapVq);
      } else {
        d3b::tma_prefetch_desc(&mapQ);
        d3b::tma_prefetch_desc(&mapKq);
        if (n_s) d3b::tma_prefetch_desc(&mapKs);
      }
      const int nslot = is_v ? C::NV : C::NK;
      uint64_t* fulls = is_v ? bars.v_full : bars.k_full;
      uint64_t* empties = is_v ? bars.v_empty : bars.k_empty;
      uint8_t* ring = is_v ? sV : sK;
      int slot = 0, ie = 0;
      uint32_t ph = 0;
      bool ok = true;
      Work w;
      for (int i = 0; ok && pair_item(p, i, n_s, rank, w); ++i) {
        if (w.n == 0) continue;
        if (!is_v) {
          // this CTA's Q tile: the previous unit's QK^T MMAs have all completed
          if (ie > 0 && !(ok = d3b::mbar_wait(&bars.q_empty, (uint32_t)(ie - 1) & 1, abort_flag, p.err, kSiteDuQ)))
            break;
          if (rank == 0) d3b::mbar_arrive_expect_tx(&bars.q_full, 2 * C::NCH * rows_used * C::ROWB);
          const uint32_t leader_q = d3b::cluster_addr(&bars.q_full, 0);
#pragma unroll
          for (int c = 0; c < C::NCH; ++c)
            d3b::tma_load_4d_pair(sQ + c * C::Q_CHUNK, &mapQ, leader_q, c * C::CH, w.g * G, w.tok0, w.b);
        }
        for (int j = 0; j < w.n; ++j) {
          if (!(ok = d3b::mbar_wait(&empties[slot], ph ^ 1, abort_flag, p.err, kSiteDuSlotEmpty))) break;
          // rank 0 arms the slot with both CTAs' bytes; rank 1's copies may land first
          if (rank == 0) d3b::mbar_arrive_expect_tx(&fulls[slot], 2 * C::SLOT_BYTES);
          const uint32_t leader_full = d3b::cluster_addr(&fulls[slot], 0);
          uint8_t* dst = ring + slot * C::SLOT_BYTES;
          const int kt = w.a + j;  // key tile of the unit
          if (is_v) {  // all 128 keys, this CTA's 64 columns
            if (kt < n_s)
              d3b::tma_load_3d_pair(dst, &mapVs, leader_full, (int)rank * C::CH, kt * BN, w.kvh);
            else
              d3b::tma_load_4d_pair(dst, &mapVq, leader_full, (int)rank * C::CH, (kt - n_s) * BN, w.kvh, w.b);
          } else {  // this CTA's 64 keys, both column halves
#pragma unroll
            for (int c = 0; c < C::NCH; ++c) {
              if (kt < n_s)
                d3b::tma_load_3d_pair(dst + c * C::K_CHUNK, &mapKs, leader_full, c * C::CH,
                                      kt * BN + (int)rank * C::K_ROWS, w.kvh);
              else
                d3b::tma_load_4d_pair(dst + c * C::K_CHUNK, &mapKq, leader_full, c * C::CH,
                                      (kt - n_s) * BN + (int)rank * C::K_ROWS, w.kvh, w.b);
            }
          }
          if (++slot == nslot) { slot = 0; ph ^= 1; }
        }
        ++ie;
      }
    }
  } else if (warp == 9) {
    // ================= QK^T issuer (rank 0) =================
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc_qk = d3b::make_idesc(1, fmt, fmt, 0, 0, 2 * BM, BN);
      const uint64_t dq0 = d3b::make_smem_desc(d3b::smem_u32(sQ), 16, C::SBO, C::LAYOUT);
      const uint64_t dk0 = d3b::make_smem_desc(d3b::smem_u32(sK), 16, C::SBO, C::LAYOUT);
      bool ok = true;
      int jg = 0, ie = 0;
      Work w;
      for (int i = 0; ok && pair_item(p, i, n_s, rank, w); ++i) {
        if (w.n == 0) continue;
        if (!(ok = d3b::mbar_wait(&bars.q_full, (uint32_t)ie & 1, abort_flag, p.err, kSiteDuQ))) break;
        for (int j = 0; j < w.n; ++j, ++jg) {
          const int sb = jg & 1;
          const uint32_t u = (uint32_t)(jg >> 1);
          // S[sb] was last read by both CTAs' softmax of tile jg-2
          if (!(ok = d3b::mbar_wait(&bars.s_free[sb], (u & 1) ^ 1, abort_flag, p.err, kSiteDuSFree))) break;
          const int slot = jg % C::NK;
          if (!(ok = d3b::mbar_wait(&bars.k_full[slot], (uint32_t)(jg / C::NK) & 1, abort_flag, p.err,
                                    kSiteDuSlotK)))
            break;
          d3b::tc_fence_after();
          const uint64_t dk = dk0 + (uint64_t)((slot * C::SLOT_BYTES) >> 4);
#pragma unroll
          for (int k = 0; k < D / 16; ++k) {
            const int c = (k * 16) / C::CH, off = ((k * 16) % C::CH) * 2;
            d3b::mma_f16_ss_pair(tmem_base + C::COL_S + sb * BN, dq0 + (uint64_t)((c * C::Q_CHUNK + off) >> 4),
                                 dk + (uint64_t)((c * C::K_CHUNK + off) >> 4), idesc_qk, k > 0 ? 1u : 0u);
          }
          d3b::mma_commit_pair(&bars.s_full[sb], 0x3);
          d3b::mma_commit_pair(&bars.k_empty[slot], 0x3);
        }
        if (!ok) break;
        d3b::mma_commit_pair(&bars.q_empty, 0x3);  // the unit's QK^T MMAs have read both Q tiles
        ++ie;
      }
      d3b::mma_commit_pair(&bars.drain_qk, 0x1);
      const uint32_t addr = d3b::smem_u32(&bars.drain_qk);
      const uint64_t t0 = d3b::globaltimer_ns();
      while (!d3b::mbar_try_wait(addr, 0)) {
        if (d3b::globaltimer_ns() - t0 > D3B_WAIT_LIMIT_NS) {
          d3b::record_device_error(p.err, kSiteDuDrain);
          break;
        }
      }
    }
  } else if (warp == 10) {
    // ================= PV issuer (rank 0) =================
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc_pv = d3b::make_idesc(1, fmt, fmt, 0, 1, 2 * BM, D);
      const uint64_t dv0 = d3b::make_smem_desc(d3b::smem_u32(sV), C::SLOT_BYTES, C::SBO, C::LAYOUT);
      bool ok = true;
      int jg = 0, ie = 0;
      Work w;
      for (int i = 0; ok && pair_item(p, i, n_s, rank, w); ++i) {
        if (w.n == 0) continue;
        for (int j = 0; j < w.n; ++j, ++jg) {
          const int sb = jg & 1;
          const uint32_t u = (uint32_t)(jg >> 1);
          if (!(ok = d3b::mbar_wait(&bars.p_full[sb], u & 1, abort_flag, p.err, kSiteDuPFull))) break;
          // both CTAs' epilogues have read the previous unit's O
          if (j == 0 && ie > 0 &&
              !(ok = d3b::mbar_wait(&bars.o_free, (uint32_t)(ie - 1) & 1, abort_flag, p.err, kSiteDuFinal)))
            break;
          const int slot = jg % C::NV;
          if (!(ok = d3b::mbar_wait(&bars.v_full[slot], (uint32_t)(jg / C::NV) & 1, abort_flag, p.err,
                                    kSiteDuSlotV)))
            break;
          d3b::tc_fence_after();
          const uint64_t dv = dv0 + (uint64_t)((slot * C::SLOT_BYTES) >> 4);
#pragma unroll
          for (int k = 0; k < BN / 16; ++k)
            d3b::mma_f16_ts_pair(tmem_base + C::COL_O, tmem_base + C::COL_P + sb * (BN / 2) + k * 8,
                                 dv + (uint64_t)((k * 16 * C::ROWB) >> 4), idesc_pv, (j > 0 || k > 0) ? 1u : 0u);
          d3b::mma_commit_pair(&bars.p_free[sb], 0x3);
          d3b::mma_commit_pair(&bars.v_empty[slot], 0x3);
        }
        if (!ok) break;
        d3b::mma_commit_pair(&bars.o_final, 0x3);  // both CTAs' O hold the unit's PV(0..n-1)
        ++ie;
      }
      d3b::mma_commit_pair(&bars.drain_pv, 0x1);
      const uint32_t addr = d3b::smem_u32(&bars.drain_pv);
      const uint64_t t0 = d3b::globaltimer_ns();
      while (!d3b::mbar_try_wait(addr, 0)) {
        if (d3b::globaltimer_ns() - t0 > D3B_WAIT_LIMIT_NS) {
          d3b::record_device_error(p.err, kSiteDuDrain);
          break;
        }
      }
    }
  }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 224;" ::: "memory");
    // ================= softmax + epilogue (warps 0-7 of both ranks) =================
    // As in the one-CTA kernel, on this CTA's 128 rows; the arrivals the issuers
    // wait for go to rank 0's barriers.
    const int wg = warp >> 2, quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_addr = tmem_base + ((uint32_t)(quarter * 32) << 16);
    const uint32_t col_s = C::COL_S + wg * BN, col_p = C::COL_P + wg * (BN / 2);
    const uint32_t s_free_r = d3b::cluster_addr(&bars.s_free[wg], 0);
    const uint32_t p_full_r = d3b::cluster_addr(&bars.p_full[wg], 0);
    const uint32_t o_free_r = d3b::cluster_addr(&bars.o_free, 0);
    const float sl2 = p.scale_log2;
    bool ok = true;
    int jg = 0, ie = 0;
    Work w;
    for (int i = 0; ok && pair_item(p, i, n_s, rank, w); ++i) {
      if (w.n == 0) {
        if (wg == 0) zero_tile_rows<D>(p, w.b, w.g, w.tok0, quarter, lane);
        continue;
      }
      float m_last = -INFINITY, l_sum = 0.f;
      for (int j = (wg ^ jg) & 1; j < w.n; j += 2) {
        const int t = jg + j;
        const uint32_t u = (uint32_t)(t >> 1);
        if (!d3b::warp_wait(&bars.s_full[wg], u & 1, abort_flag, p.err, kSiteDuSFull)) { ok = false; break; }
        d3b::tc_fence_after();
        float s[BN];
#pragma unroll
        for (int c = 0; c < BN / 32; ++c)
          d3b::tmem_ld32(lane_addr + col_s + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&s[c * 32]));
        d3b::tmem_wait_ld();
        d3b::tc_fence_before();
        d3b::mbar_arrive_cluster(s_free_r);
        const int kt = w.a + j;
        const int valid = kt < n_s ? p.S - kt * BN : w.len_b - (kt - n_s) * BN;
        if (valid < BN) {
#pragma unroll
          for (int c = 0; c < BN; ++c)
            if (c >= valid) s[c] = -INFINITY;
        }
        const float m_tile = max_n<BN>(s) * sl2;
        float m_prev = -INFINITY;
        if (t > 0) {
          if (!d3b::warp_wait(&bars.mdone[(t - 1) & 1], (uint32_t)((t - 1) >> 1) & 1, abort_flag, p.err,
                              kSiteDuXMax)) {
            ok = false;
            break;
          }
          if (j > 0) m_prev = mref_s[(t - 1) & 1][r];
        }
        const bool rescale = __any_sync(0xffffffffu, m_tile > m_prev + kRescaleThreshold);
        const float m_new = rescale ? fmaxf(m_prev, m_tile) : m_prev;
        mref_s[wg][r] = m_new;
        d3b::mbar_arrive(&bars.mdone[wg]);
        if (rescale && j > 0) {
          if (!d3b::warp_wait(&bars.p_free[(t - 1) & 1], (uint32_t)((t - 1) >> 1) & 1, abort_flag, p.err,
                              kSiteDuPFree)) {
            ok = false;
            break;
          }
          d3b::tc_fence_after();
          scale_cols<D>(lane_addr + C::COL_O, d3b::ex2_approx(m_prev - m_new));
        }
        if (!d3b::warp_wait(&bars.p_free[wg], (u & 1) ^ 1, abort_flag, p.err, kSiteDuPFree)) { ok = false; break; }
        d3b::tc_fence_after();
        float rowsum = 0.f;
#pragma unroll
        for (int qq = 0; qq < BN / 32; ++qq) {
          uint32_t pk[16];
          rowsum += exp_row<32, FP16, D3B_POLY8>(s + qq * 32, sl2, m_new, pk);
          d3b::tmem_st16(lane_addr + col_p + qq * 16, pk);
        }
        d3b::tmem_wait_st();
        d3b::tc_fence_before();
        d3b::mbar_arrive_cluster(p_full_r);
        l_sum = (m_last == m_new ? l_sum : l_sum * d3b::ex2_approx(m_last - m_new)) + rowsum;
        m_last = m_new;
      }
      if (ok) ok = d3b::warp_wait(&bars.o_final, (uint32_t)ie & 1, abort_flag, p.err, kSiteDuFinal);
      if (ok) {
        lsum_s[wg][r] = l_sum;
        mlast_s[wg][r] = m_last;
        d3b::mbar_arrive(&bars.xsum[quarter]);
        ok = d3b::warp_wait(&bars.xsum[quarter], (uint32_t)ie & 1, abort_flag, p.err, kSiteDuXMax);
      }
      if (!ok) break;
      d3b::tc_fence_after();
      const float m0 = mlast_s[0][r], m1 = mlast_s[1][r];
      const float m_fin = fmaxf(m0, m1);
      const float l = lsum_s[0][r] * d3b::ex2_approx(m0 - m_fin) + lsum_s[1][r] * d3b::ex2_approx(m1 - m_fin);
      const int tok = w.tok0 + r / G, h = r % G;
      const bool in_tensor = r < rows_used && tok < p.L;
      const bool real = tok < w.len_b;
      const float inv_l = 1.f / l;
      uint16_t* dst_row = static_cast<uint16_t*>(p.out) + (int64_t)w.b * p.out_sb +
                          (int64_t)(w.g * G + h) * p.out_sh + (int64_t)tok * p.out_sl + wg * C::OH;
      uint32_t o[C::OH];
#pragma unroll
      for (int c = 0; c < C::OH / 32; ++c)
        d3b::tmem_ld32(lane_addr + C::COL_O + wg * C::OH + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&o[c * 32]));
      d3b::tmem_wait_ld();
      // O is in registers: the next unit's first PV may overwrite it
      d3b::tc_fence_before();
      d3b::mbar_arrive_cluster(o_free_r);
      if (in_tensor) {
        uint4* dst = reinterpret_cast<uint4*>(dst_row);
#pragma unroll
        for (int i8 = 0; i8 < C::OH / 8; ++i8) {
          uint32_t v[4];
#pragma unroll
          for (int k = 0; k < 4; ++k)
            v[k] = real ? pack2<FP16>(__uint_as_float(o[8 * i8 + 2 * k]) * inv_l,
                                      __uint_as_float(o[8 * i8 + 2 * k + 1]) * inv_l)
                        : 0u;
          dst[i8] = make_uint4(v[0], v[1], v[2], v[3]);
        }
      }
      jg += w.n;
      ++ie;
    }
  }

  __syncwarp();  // lanes that skipped a role loop rejoin before the aligned cluster barrier
  d3b::tc_fence_before();
  d3b::cluster_sync();  // rank 0's MMAs (which write both TMEMs) are drained before either CTA frees TMEM
  d3b::tc_fence_after();
  if (warp == 9) d3b::tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
}

template <int FP16>
int launch_pair(const CUtensorMap* maps, const Params& prm, int pair_units, cudaStream_t stream) {
  using C = CfgPair;
  static int attr_set[64] = {0};
  const int dev = d3b_host::current_device();
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    if (cudaFuncSetAttribute(prefix_bidir_pair_kernel<FP16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             C::SMEM_BYTES) != cudaSuccess)
      return D3B_ECUDA;
    attr_set[dev] = 1;
  }
  // Pairs that fit at once (an SM left alone in its GPC takes none), queried once per device.
  static int max_pairs_of[64] = {0};
  int max_pairs = (dev >= 0 && dev < 64) ? max_pairs_of[dev] : 0;
  if (max_pairs <= 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * 256);
    cfg.blockDim = dim3(DU_THREADS);
    cfg.dynamicSmemBytes = C::SMEM_BYTES;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, prefix_bidir_pair_kernel<FP16>, &cfg) != cudaSuccess ||
        clusters <= 0) {
      cudaGetLastError();
      clusters = d3b_host::num_sms(dev) / 2;
    }
    max_pairs = clusters;
    if (dev >= 0 && dev < 64) max_pairs_of[dev] = clusters;
  }
  const int pairs = std::max(1, std::min(pair_units, max_pairs));
  prefix_bidir_pair_kernel<FP16><<<dim3(2 * pairs), DU_THREADS, C::SMEM_BYTES, stream>>>(maps[0], maps[5], maps[2],
                                                                                         maps[6], maps[4], prm);
  return d3b_host::check_launch();
}

template <int D, int BN, int FP16, bool SPLIT>
int launch_as(const CUtensorMap* maps, const Params& prm, dim3 grid, cudaStream_t stream) {
  using C = Cfg<D, BN>;
  static int attr_set[64] = {0};
  const int dev = d3b_host::current_device();
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    if (cudaFuncSetAttribute(prefix_bidir_kernel<D, BN, FP16, SPLIT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             C::SMEM_BYTES) != cudaSuccess)
      return D3B_ECUDA;
    attr_set[dev] = 1;
  }
  prefix_bidir_kernel<D, BN, FP16, SPLIT><<<grid, NUM_THREADS, C::SMEM_BYTES, stream>>>(maps[0], maps[1], maps[2],
                                                                                        maps[3], maps[4], prm);
  return d3b_host::check_launch();
}

// grid: (tiles, head groups, blocks) one CTA per unit; grid_split: the 1-D
// grid of a launch with split units
template <int D, int BN, int FP16>
int launch(const CUtensorMap* maps, const Params& prm, dim3 grid, dim3 grid_split, cudaStream_t stream) {
  return prm.split_units ? launch_as<D, BN, FP16, true>(maps, prm, grid_split, stream)
                         : launch_as<D, BN, FP16, false>(maps, prm, grid, stream);
}

// D = 256 runs on the two-issuer kernel (64-key tiles); D3B_ATTN_D256=single in
// the environment selects the one-issuer kernel instead (read once per process).
bool d256_single_issuer() {
  static const bool on = [] {
    const char* v = std::getenv("D3B_ATTN_D256");
    return v && std::string(v) == "single";
  }();
  return on;
}

template <int FP16>
int dispatch(int D, const CUtensorMap* maps, const Params& prm, dim3 grid, dim3 grid_dual, cudaStream_t s) {
  // one unit (or piece of a unit) per CTA, one CTA per SM
  if (D == 256 && d256_single_issuer()) return launch<256, 64, FP16>(maps, prm, grid, grid_dual, s);
  switch (D) {
    case 256: return launch_dual<256, FP16>(maps, prm, grid_dual, s);
    case 32: return launch_dual<32, FP16>(maps, prm, grid_dual, s);
    case 64: return launch_dual<64, FP16>(maps, prm, grid_dual, s);
    case 128: return launch_dual<128, FP16>(maps, prm, grid_dual, s);
  }
  return D3B_EUNSUPPORTED;
}

// ---------------------------------------------------------------------------
// Launch plan of the D <= 128 kernel. Units take equal time (n key tiles) and
// one CTA runs per SM, dispatched in block order. With U units on P SMs the
// first U - U % P units fill whole waves; the last R = U % P units would leave
// P - R SMs idle for a whole unit, so they may be cut into pieces instead: a
// first piece of piece0 iterations, then runs of piece_rest. The plan is the
// one with the shortest makespan of greedy (list) dispatch of the pieces in
// block order, with a fixed per-CTA cost (start-up, pipeline fill, epilogue,
// merge) of kCtaCost iterations; it is kept only if it saves >= 3 %.
// kCtaCost comes from B200 timings of one CTA per unit at D = 128: 33-tile
// units (config 3a) take 37.9 us per wave, 129-tile units (configs 3b, 5)
// 121.2 us, i.e. 0.87 us per key tile plus ~9 us per CTA. Cutting is limited
// to the regime where it measured faster: units of >= kMinSplitTiles key
// tiles (states of 8k tokens and more) and at most kMaxFullWaves full waves
// before the tail. A 32-block shard of config 5 (one rank of eight): 0.43 ms
// against 0.47 ms uncut; config 3a's 33-tile units cut (26 + 7): 88 us
// against 76 us uncut, so short units stay whole.
// ---------------------------------------------------------------------------
constexpr double kCtaCost = 12.0;
constexpr int kMinSplitTiles = 64;
constexpr int kMaxFullWaves = 7;

struct TailPlan {
  int split_units = 0, pieces = 0, piece0 = 0, piece_rest = 0;
  double makespan = 0.0;
};

double tail_makespan(int R, int n, int P, int piece0, int rest) {
  // pieces are dispatched piece 0 of every split unit first, then piece 1, ...
  std::priority_queue<double, std::vector<double>, std::greater<double>> sm;
  for (int i = 0; i < P; ++i) sm.push(0.0);
  double mk = 0.0;
  for (int a = 0, k = 0; a < n; ++k) {
    const int len = std::min(n - a, k == 0 ? piece0 : rest);
    for (int r = 0; r < R; ++r) {
      double t = sm.top();
      sm.pop();
      t += len + kCtaCost;
      mk = std::max(mk, t);
      sm.push(t);
    }
    a += len;
  }
  return mk;
}

TailPlan plan_tail(int units, int n, int P) {
  TailPlan best;
  const int R = P > 0 ? units % P : 0;
  best.makespan = n + kCtaCost;
  // 256: the fixed count region of the workspace
  if (R == 0 || n < kMinSplitTiles || units / P > kMaxFullWaves || R > 256) return best;
  TailPlan cand;
  auto consider = [&](int piece0, int rest) {
    const double mk = tail_makespan(R, n, P, piece0, rest);
    if (mk < cand.makespan || cand.pieces == 0) {
      cand.makespan = mk;
      cand.split_units = R;
      cand.piece0 = piece0;
      cand.piece_rest = rest;
      cand.pieces = 1 + (n - piece0 + rest - 1) / rest;
    }
  };
  for (int t = (n + 1) / 2; t < n; ++t) consider(t, n - t);  // a big and a small piece
  for (int k = 3; k <= 8 && k <= n; ++k) {                    // k near-equal pieces
    const int len = (n + k - 1) / k;
    consider(len, len);
  }
  if (cand.pieces > 1 && cand.makespan <= 0.97 * best.makespan) return cand;
  return best;
}

// Cached per (units, n, SMs): the plan is host arithmetic, but a call should not redo it.
TailPlan cached_plan(int units, int n, int P) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, int>, TailPlan> cache;
  std::lock_guard<std::mutex> lock(mu);
  const auto key = std::make_tuple(units, n, P);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  if (cache.size() > 4096) cache.clear();
  const TailPlan t = plan_tail(units, n, P);
  cache.emplace(key, t);
  return t;
}

// The CTA-pair kernel serves D = 128 with an even number of Q tiles per
// (block, kv head) in long launches: at least kPairMinWaves units per SM and no
// cut tail. B200 timings against the one-CTA kernel: 64 blocks of 64 tokens
// over a 16384-token state (6.9 units per SM) 0.825 vs 0.855 ms; config 3a
// (1.7 units per SM) 77 vs 76 us, so short launches stay on one CTA per unit.
// D3B_ATTN_PAIR=0 in the environment turns it off (read once per process).
constexpr int64_t kPairMinWaves = 4;
bool pair_kernel_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("D3B_ATTN_PAIR");
    return !(v && v[0] == '0');
  }();
  return on;
}

// Workspace layout: the per-unit counts first, in a region of fixed size for
// every shape (split_units < SMs <= kMaxCounts), so partial slots written for
// one shape never land where another shape's counts must read zero; then one
// partial slot per piece.
constexpr int kMaxCounts = 256;
constexpr size_t kCountBytes = kMaxCounts * sizeof(int);

// Q tile shape for G query heads per KV head and L tokens per block: Gs of
// the G heads by T = BM / Gs tokens, Gs a divisor of G, the one with the fewest
// tiles per (block, KV head) (G / Gs head groups x ceil(L / T) token tiles),
// ties to the largest Gs. Token-aligned tiles of the whole group leave rows
// empty when G does not divide BM: G = 6, L = 64 takes 4 tiles of 21 tokens
// (384 of 512 rows used), 3 head groups of 2 heads x 64 tokens fill 3 tiles.
// Every K/V tile is read once per tile, so fewer tiles also means fewer reads.
struct TileShape {
  int Gs, T, hsplit;
  int64_t tiles;  // token tiles per head group
};
TileShape tile_shape(int G, int L) {
  TileShape best{G, BM / G, 1, (L + BM / G - 1) / (BM / G)};
  for (int gs = G - 1; gs >= 1; --gs) {
    if (G % gs) continue;
    const int t = BM / gs;
    const int64_t tiles = (L + t - 1) / t;
    if ((int64_t)(G / gs) * tiles < (int64_t)best.hsplit * best.tiles) best = {gs, t, G / gs, tiles};
  }
  return best;
}

size_t plan_bytes(const TailPlan& t, int D, size_t* count_bytes) {
  if (count_bytes) *count_bytes = kCountBytes;
  if (!t.split_units) return 0;
  return kCountBytes + (size_t)t.split_units * t.pieces * (size_t)(BM * D + 2 * BM) * sizeof(float);
}

}  // namespace

static int prefix_bidir_impl(const void* q, const int64_t* q_strides, const void* k_state, const void* v_state,
                             const int64_t* kv_strides, const void* k_q, const void* v_q, const int64_t* kq_strides,
                             const int32_t* lengths, int B, int H, int Hkv, int S, int L, int D, int dtype,
                             float scale, void* out, const int64_t* out_strides, void* workspace,
                             size_t workspace_bytes, d3b_stream_t stream) {
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
  const TileShape shape = tile_shape(G, L);
  const int T = shape.T;
  if ((int64_t)Hkv * shape.hsplit > 65535) return D3B_EINVAL;

  // 0 Q, 1/2 state K/V, 3/4 own K/V; the pair kernel's key halves: 5 state K, 6 own K (64-key boxes)
  CUtensorMap maps[7];
  int rc;
  {  // Q: [B, H, L, D] -> dims {D, H, L, B}, box {CH, Gs, T, 1}
    const uint64_t dims[4] = {(uint64_t)D, (uint64_t)H, (uint64_t)L, (uint64_t)B};
    const uint64_t st[3] = {(uint64_t)q_strides[1] * 2, (uint64_t)q_strides[2] * 2, (uint64_t)q_strides[0] * 2};
    const uint32_t box[4] = {(uint32_t)CH, (uint32_t)shape.Gs, (uint32_t)T, 1};
    if ((rc = d3b_host::encode_tiled(&maps[0], dt, 4, q, dims, st, box, sw))) return rc;
  }
  {  // own-block K/V: [B, Hkv, L, D] -> dims {D, L, Hkv, B}, box {CH, BN, 1, 1}
    const uint64_t dims[4] = {(uint64_t)D, (uint64_t)L, (uint64_t)Hkv, (uint64_t)B};
    const uint64_t st[3] = {(uint64_t)kq_strides[2] * 2, (uint64_t)kq_strides[1] * 2, (uint64_t)kq_strides[0] * 2};
    const uint32_t box[4] = {(uint32_t)CH, (uint32_t)BN, 1, 1};
    if ((rc = d3b_host::encode_tiled(&maps[3], dt, 4, k_q, dims, st, box, sw))) return rc;
    if ((rc = d3b_host::encode_tiled(&maps[4], dt, 4, v_q, dims, st, box, sw))) return rc;
    if (D == 128) {
      const uint32_t half[4] = {(uint32_t)CH, (uint32_t)BN / 2, 1, 1};
      if ((rc = d3b_host::encode_tiled(&maps[6], dt, 4, k_q, dims, st, half, sw))) return rc;
    }
  }
  if (S > 0) {  // state K/V: [Hkv, S, D] -> dims {D, S, Hkv}, box {CH, BN, 1}
    const uint64_t dims[3] = {(uint64_t)D, (uint64_t)S, (uint64_t)Hkv};
    const uint64_t st[2] = {(uint64_t)kv_strides[1] * 2, (uint64_t)kv_strides[0] * 2};
    const uint32_t box[3] = {(uint32_t)CH, (uint32_t)BN, 1};
    if ((rc = d3b_host::encode_tiled(&maps[1], dt, 3, k_state, dims, st, box, sw))) return rc;
    if ((rc = d3b_host::encode_tiled(&maps[2], dt, 3, v_state, dims, st, box, sw))) return rc;
    if (D == 128) {
      const uint32_t half[3] = {(uint32_t)CH, (uint32_t)BN / 2, 1};
      if ((rc = d3b_host::encode_tiled(&maps[5], dt, 3, k_state, dims, st, half, sw))) return rc;
    }
  } else {  // never read when S == 0
    maps[1] = maps[3];
    maps[2] = maps[4];
    maps[5] = maps[6];
  }

  Params prm;
  prm.lengths = lengths;
  prm.out = out;
  prm.out_sb = out_strides[0];
  prm.out_sh = out_strides[1];
  prm.out_sl = out_strides[2];
  prm.H = H;
  prm.Hkv = Hkv * shape.hsplit;  // head groups
  prm.G = shape.Gs;
  prm.T = T;
  prm.hsplit = shape.hsplit;
  prm.S = S;
  prm.L = L;
  prm.scale_log2 = (float)((double)scale * 1.4426950408889634);
  prm.err = d3b_host::device_error_word();
  if (!prm.err) return D3B_ECUDA;

  const int64_t tiles = shape.tiles;
  const int64_t units = tiles * prm.Hkv * B;
  const int64_t n_full = (int64_t)(S + BN - 1) / BN + (L + BN - 1) / BN;
  if (units > 0x7FFFFFFF || n_full > 0x7FFFFFFF) return D3B_EINVAL;
  prm.tiles = (int)tiles;
  prm.n_full = (int)n_full;
  prm.whole_units = (int)units;
  prm.split_units = prm.pieces = prm.piece0 = prm.piece_rest = 0;
  prm.part = nullptr;
  prm.count = nullptr;
  int64_t ctas = units;
  if (workspace) {
    const TailPlan t = cached_plan((int)units, (int)n_full, d3b_host::num_sms(d3b_host::current_device()));
    if (t.split_units) {
      size_t count_bytes = 0;
      if (workspace_bytes < plan_bytes(t, D, &count_bytes)) return D3B_ENOSPACE;
      if (reinterpret_cast<uintptr_t>(workspace) % 256) return D3B_EALIGN;
      prm.whole_units = (int)units - t.split_units;
      prm.split_units = t.split_units;
      prm.pieces = t.pieces;
      prm.piece0 = t.piece0;
      prm.piece_rest = t.piece_rest;
      prm.count = static_cast<int*>(workspace);
      prm.part = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + count_bytes);
      ctas = prm.whole_units + (int64_t)t.split_units * t.pieces;
    }
  }
  if (ctas > 0x7FFFFFFF) return D3B_EINVAL;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int64_t sms = d3b_host::num_sms(d3b_host::current_device());
  // (whole GQA groups only: the pair kernel with split head groups has not been measured)
  if (D == 128 && tiles % 2 == 0 && shape.hsplit == 1 && !prm.split_units && units >= kPairMinWaves * sms &&
      pair_kernel_enabled()) {
    // CTA pairs: both Q tiles of a pair unit share every key and value tile
    prm.whole_units = (int)(units / 2);
    prm.part = nullptr;
    prm.count = nullptr;
    return dtype == D3B_F16 ? launch_pair<1>(maps, prm, prm.whole_units, s)
                            : launch_pair<0>(maps, prm, prm.whole_units, s);
  }
  const dim3 grid((unsigned)tiles, (unsigned)prm.Hkv, B);
  // D <= 128: one CTA per unit or piece in a split launch, else a persistent
  // grid of at most one CTA per SM looping over the units
  const dim3 grid_dual = prm.split_units ? dim3((unsigned)ctas)
                                         : dim3((unsigned)std::max<int64_t>(1, std::min<int64_t>(units, sms)));
  return dtype == D3B_F16 ? dispatch<1>(D, maps, prm, grid, grid_dual, s)
                          : dispatch<0>(D, maps, prm, grid, grid_dual, s);
}

extern "C" size_t d3b_prefix_bidir_workspace_size(int B, int H, int Hkv, int S, int L, int D) {
  if (B <= 0 || H <= 0 || Hkv <= 0 || S < 0 || L <= 0 || H % Hkv || H / Hkv > BM) return 0;
  if (D != 32 && D != 64 && D != 128 && D != 256) return 0;
  const int BN = D == 256 ? 64 : 128;
  const TileShape shape = tile_shape(H / Hkv, L);
  const int64_t units = shape.tiles * shape.hsplit * Hkv * B;
  const int64_t n_full = (int64_t)(S + BN - 1) / BN + (L + BN - 1) / BN;
  if (units > 0x7FFFFFFF || n_full > 0x7FFFFFFF) return 0;
  const TailPlan t = cached_plan((int)units, (int)n_full, d3b_host::num_sms(d3b_host::current_device()));
  return t.split_units ? plan_bytes(t, D, nullptr) : 0;
}

extern "C" int d3b_prefix_bidir(const void* q, const int64_t* q_strides, const void* k_state, const void* v_state,
                                const int64_t* kv_strides, const void* k_q, const void* v_q,
                                const int64_t* kq_strides, const int32_t* lengths, int B, int H, int Hkv, int S, int L,
                                int D, int dtype, float scale, void* out, const int64_t* out_strides,
                                d3b_stream_t stream) {
  return prefix_bidir_impl(q, q_strides, k_state, v_state, kv_strides, k_q, v_q, kq_strides, lengths, B, H, Hkv, S, L,
                           D, dtype, scale, out, out_strides, nullptr, 0, stream);
}

extern "C" int d3b_prefix_bidir_ws(const void* q, const int64_t* q_strides, const void* k_state, const void* v_state,
                                   const int64_t* kv_strides, const void* k_q, const void* v_q,
                                   const int64_t* kq_strides, const int32_t* lengths, int B, int H, int Hkv, int S,
                                   int L, int D, int dtype, float scale, void* out, const int64_t* out_strides,
                                   void* workspace, size_t workspace_bytes, d3b_stream_t stream) {
  return prefix_bidir_impl(q, q_strides, k_state, v_state, kv_strides, k_q, v_q, kq_strides, lengths, B, H, Hkv, S, L,
                           D, dtype, scale, out, out_strides, workspace, workspace_bytes, stream);
}
