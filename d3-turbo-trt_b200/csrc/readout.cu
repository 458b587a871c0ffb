// 255-way fp32 readout softmax at the selected positions
// (d3trt/model/trtllm_stack.py:451-468, = hf_stack.py:67-84):
//   logits = f32(hidden) @ R^T ; logits[b, j >= counts[b]] = -inf ;
//   probs  = softmax(logits / T)
//
// One launch. The grid is (row groups of 8) x (option groups of 32). A CTA
// stages K-chunks of its 8 hidden rows in shared memory (as fp32); each warp
// computes 4 options x 8 rows of dot products with fp32 FMAs (the reference
// computes in fp32, so no tensor-core rounding is introduced), streaming R
// with 16-byte loads, 16 of them in flight per lane; the hidden chunk is staged
// with 16-byte loads that are all issued before the first store. Logits go to the
// workspace. The last CTA of a row group to finish (an atomic ticket per row
// group) runs the masked softmax with one warp per row and resets the ticket,
// so the workspace is ready for the next call.
//
// Workspace layout: [tickets: kMaxGroups x u32 at offset 0][logits: B x n_opt f32].
// The ticket region never moves, so one zero-filled workspace serves calls of
// any shape (B <= 8 * kMaxGroups).
#include <algorithm>
#include <mutex>

#include "common.cuh"

namespace {

constexpr int kRows = 8;        // hidden rows per CTA (= warps per CTA)
constexpr int kOpts = 32;       // options per CTA
constexpr int kOptsPerWarp = kOpts / kRows;
constexpr int kChunk = 1024;    // K elements staged per step (8 rows x 4 KB)
constexpr int kUnroll = 4;      // float4 steps per lane kept in flight, per option
constexpr int kMaxOpts = 1024;  // softmax keeps n_opt/32 logits per lane
constexpr int kMaxGroups = 4096;
constexpr size_t kTicketBytes = kMaxGroups * sizeof(unsigned int);

// 16 bytes of hidden as fp32 (8 bf16/f16 or 4 f32 values)
__device__ __forceinline__ int unpack16(uint4 a, const float*, float (&v)[8]) {
  v[0] = __uint_as_float(a.x); v[1] = __uint_as_float(a.y); v[2] = __uint_as_float(a.z); v[3] = __uint_as_float(a.w);
  return 4;
}
__device__ __forceinline__ int unpack16(uint4 a, const __nv_bfloat16*, float (&v)[8]) {
  const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = __uint_as_float(w[i] << 16);
    v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
  return 8;
}
__device__ __forceinline__ int unpack16(uint4 a, const __half*, float (&v)[8]) {
  const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
  return 8;
}

__device__ __forceinline__ float load_h(const float* p) { return __ldg(p); }
__device__ __forceinline__ float load_h(const __nv_bfloat16* p) { return __bfloat162float(*p); }
__device__ __forceinline__ float load_h(const __half* p) { return __half2float(*p); }

// Masked softmax of NR rows of logits (one warp, rows row0 .. row0+NR-1,
// handled together so their loads and reductions overlap):
// logits[j >= counts[row]] = -inf, probs = softmax(logits / temperature); a row
// with count <= 0 is all NaN, as the reference's softmax of an all -inf row.
// PER = values per lane (n_opt <= 32 * PER).
template <int PER, int NR>
__device__ __forceinline__ void rows_softmax(int row0, int B, int n_opt, const int32_t* __restrict__ counts,
                                             float temperature, const float* logits, float* __restrict__ probs,
                                             int lane) {
  float v[NR][PER];
  float mx[NR], sum[NR];
  int cnt[NR];
#pragma unroll
  for (int q = 0; q < NR; ++q) {
    const int row = row0 + q;
    cnt[q] = row < B ? counts[row] : 0;
    mx[q] = -INFINITY;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int j = lane + 32 * i;
      float x = -INFINITY;
      if (row < B && j < n_opt && j < cnt[q]) x = __ldcg(logits + (int64_t)row * n_opt + j) / temperature;
      v[q][i] = x;
      mx[q] = fmaxf(mx[q], x);
    }
  }
#pragma unroll
  for (int s = 16; s > 0; s >>= 1)
#pragma unroll
    for (int q = 0; q < NR; ++q) mx[q] = fmaxf(mx[q], __shfl_xor_sync(0xffffffffu, mx[q], s));
#pragma unroll
  for (int q = 0; q < NR; ++q) {
    sum[q] = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const float e = (v[q][i] == -INFINITY) ? 0.f : expf(v[q][i] - mx[q]);
      v[q][i] = e;
      sum[q] += e;
    }
  }
#pragma unroll
  for (int s = 16; s > 0; s >>= 1)
#pragma unroll
    for (int q = 0; q < NR; ++q) sum[q] += __shfl_xor_sync(0xffffffffu, sum[q], s);
#pragma unroll
  for (int q = 0; q < NR; ++q) {
    const int row = row0 + q;
    if (row >= B) continue;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int j = lane + 32 * i;
      if (j < n_opt) probs[(int64_t)row * n_opt + j] = (cnt[q] > 0) ? v[q][i] / sum[q] : __int_as_float(0x7fc00000);
    }
  }
}

// One warp, one row.
__device__ __forceinline__ void softmax_row(int row, int B, int n_opt, const int32_t* __restrict__ counts,
                                            float temperature, const float* logits, float* __restrict__ probs,
                                            int lane) {
  if (n_opt <= 32 * 8) rows_softmax<8, 1>(row, B, n_opt, counts, temperature, logits, probs, lane);
  else if (n_opt <= 32 * 16) rows_softmax<16, 1>(row, B, n_opt, counts, temperature, logits, probs, lane);
  else rows_softmax<32, 1>(row, B, n_opt, counts, temperature, logits, probs, lane);
}

template <typename T, bool VEC>
__global__ void __launch_bounds__(kRows * 32) readout_kernel(const T* __restrict__ hidden,
                                                              const float* __restrict__ R,
                                                              const int32_t* __restrict__ counts, float temperature,
                                                              float* __restrict__ probs, int B, int K, int n_opt,
                                                              float* __restrict__ logits_ws,
                                                              unsigned int* __restrict__ tickets) {
  __shared__ __align__(16) float hs[kRows][kChunk];
  __shared__ int s_last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r0 = blockIdx.x * kRows;
  const int o0 = blockIdx.y * kOpts + warp * kOptsPerWarp;

  float acc[kOptsPerWarp][kRows];
#pragma unroll
  for (int o = 0; o < kOptsPerWarp; ++o)
#pragma unroll
    for (int r = 0; r < kRows; ++r) acc[o][r] = 0.f;
  const float* rrow[kOptsPerWarp];
#pragma unroll
  for (int o = 0; o < kOptsPerWarp; ++o) rrow[o] = R + (int64_t)min(o0 + o, n_opt - 1) * K;

  for (int kc = 0; kc < K; kc += kChunk) {
    const int kn = min(kChunk, K - kc);
    __syncthreads();
    if (VEC) {
      // 16-byte loads, all issued before any store: kRows * kChunk / (per * 256) per thread
      constexpr int per = 16 / sizeof(T);
      constexpr int kLoads = kRows * kChunk / per / (kRows * 32);
      uint4 raw[kLoads];
#pragma unroll
      for (int i = 0; i < kLoads; ++i) {
        const int e = (threadIdx.x + i * kRows * 32) * per;  // element index in the [kRows][kChunk] tile
        const int r = e / kChunk, k = e % kChunk;
        const int row = r0 + r;
        raw[i] = (row < B && k < kn) ? __ldg(reinterpret_cast<const uint4*>(hidden + (int64_t)row * K + kc + k))
                                     : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int i = 0; i < kLoads; ++i) {
        const int e = (threadIdx.x + i * kRows * 32) * per;
        const int r = e / kChunk, k = e % kChunk;
        float v[8];
        unpack16(raw[i], static_cast<const T*>(nullptr), v);
        *reinterpret_cast<float4*>(&hs[r][k]) = make_float4(v[0], v[1], v[2], v[3]);
        if (per == 8) *reinterpret_cast<float4*>(&hs[r][k + 4]) = make_float4(v[4], v[5], v[6], v[7]);
      }
    } else {
      for (int i = threadIdx.x; i < kRows * kChunk; i += blockDim.x) {
        const int r = i / kChunk, k = i % kChunk;
        const int row = r0 + r;
        hs[r][k] = (row < B && k < kn) ? load_h(hidden + (int64_t)row * K + kc + k) : 0.f;
      }
    }
    __syncthreads();
    if (VEC) {
      // kn is a multiple of 4; lanes cover 128 consecutive k per step
      for (int k0 = lane * 4; k0 < kn; k0 += 128 * kUnroll) {
        float4 w[kUnroll][kOptsPerWarp];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u)
#pragma unroll
          for (int o = 0; o < kOptsPerWarp; ++o) {
            const int k = k0 + u * 128;
            w[u][o] = k < kn ? __ldg(reinterpret_cast<const float4*>(rrow[o] + kc + k)) : make_float4(0, 0, 0, 0);
          }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          const int k = k0 + u * 128;
          if (k >= kn) break;
#pragma unroll
          for (int r = 0; r < kRows; ++r) {
            const float4 h = *reinterpret_cast<const float4*>(&hs[r][k]);
#pragma unroll
            for (int o = 0; o < kOptsPerWarp; ++o) {
              acc[o][r] = fmaf(h.x, w[u][o].x, acc[o][r]);
              acc[o][r] = fmaf(h.y, w[u][o].y, acc[o][r]);
              acc[o][r] = fmaf(h.z, w[u][o].z, acc[o][r]);
              acc[o][r] = fmaf(h.w, w[u][o].w, acc[o][r]);
            }
          }
        }
      }
    } else {
      for (int k = lane; k < kn; k += 32) {
#pragma unroll
        for (int o = 0; o < kOptsPerWarp; ++o) {
          const float w = __ldg(rrow[o] + kc + k);
#pragma unroll
          for (int r = 0; r < kRows; ++r) acc[o][r] = fmaf(hs[r][k], w, acc[o][r]);
        }
      }
    }
  }
#pragma unroll
  for (int o = 0; o < kOptsPerWarp; ++o)
#pragma unroll
    for (int r = 0; r < kRows; ++r) {
      float v = acc[o][r];
#pragma unroll
      for (int s = 16; s > 0; s >>= 1) v += __shfl_xor_sync(0xffffffffu, v, s);
      acc[o][r] = v;
    }
  if (lane == 0) {
#pragma unroll
    for (int o = 0; o < kOptsPerWarp; ++o)
#pragma unroll
      for (int r = 0; r < kRows; ++r) {
        const int row = r0 + r, opt = o0 + o;
        if (row < B && opt < n_opt) logits_ws[(int64_t)row * n_opt + opt] = acc[o][r];
      }
  }

  // ---- last CTA of this row group runs the softmax ----
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned int ticket = atomicAdd(&tickets[blockIdx.x], 1u);
    s_last = (ticket == gridDim.y - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();

  softmax_row(r0 + warp, B, n_opt, counts, temperature, logits_ws, probs, lane);
  if (threadIdx.x == 0) tickets[blockIdx.x] = 0u;
}

// ---------------------------------------------------------------------------
// Tiled split-K readout (the d3b_readout path for 16-byte aligned rows):
// grid (row tiles of 64, option tiles of 64, K splits). A CTA stages its rows
// of hidden and its options of R for 64 k at a time in shared memory (as
// fp32, k-major, double-buffered) and each thread accumulates a 4 x 4 block of
// dot products with fp32 FMAs, so every element of R read from L2 serves 64
// rows. Each CTA writes its partial sums; the last CTA of a (row tile, option
// tile) to finish (atomic ticket) adds the K splits in split order (so the
// result does not depend on CTA timing) into the logits, and the last option
// tile of a row tile runs the masked softmax of its 64 rows. Tickets are reset
// by whoever used them last, so the workspace is ready for the next call.
// ---------------------------------------------------------------------------
constexpr int kTR = 64;          // rows per tile
constexpr int kTO = 64;          // options per tile
constexpr int kKC = 64;          // k per shared-memory stage
constexpr int kTiledSmem = 2 * kKC * (kTR + 4) * 4 + 2 * kKC * (kTO + 4) * 4;  // 69632 bytes
constexpr int kMaxSplit = 32;    // K splits at most
constexpr int kTiledTicketWords = 16384;  // ticket1: row tiles x option tiles (<= 512 x 16), ticket2: row tiles
constexpr size_t kTiledTicketBytes = kTiledTicketWords * sizeof(unsigned int);

template <typename T>
__device__ __forceinline__ void load_hidden8(const T* p, bool ok, float (&v)[8]) {
  if constexpr (sizeof(T) == 4) {
    const float4 a = ok ? __ldg(reinterpret_cast<const float4*>(p)) : make_float4(0.f, 0.f, 0.f, 0.f);
    const float4 b = ok ? __ldg(reinterpret_cast<const float4*>(p) + 1) : make_float4(0.f, 0.f, 0.f, 0.f);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
    const uint4 a = ok ? __ldg(reinterpret_cast<const uint4*>(p)) : make_uint4(0, 0, 0, 0);
    unpack16(a, static_cast<const T*>(nullptr), v);
  }
}

template <typename T>
__global__ void __launch_bounds__(256) readout_tiled_kernel(const T* __restrict__ hidden, const float* __restrict__ R,
                                                            int B, int K, int n_opt,
                                                            int kper, int b_pad, int o_pad,
                                                            float* __restrict__ partials) {
  // [2 buffers][kKC][64 + 4] for hidden, then the same for R (dynamic: 69.6 KB)
  extern __shared__ __align__(16) float smem_f[];
  auto hs = [&](int buf, int k) -> float* { return smem_f + (buf * kKC + k) * (kTR + 4); };
  auto rs = [&](int buf, int k) -> float* { return smem_f + 2 * kKC * (kTR + 4) + (buf * kKC + k) * (kTO + 4); };
  const int t = threadIdx.x;
  const int tr = blockIdx.x, to = blockIdx.y, kz = blockIdx.z;
  const int r0 = tr * kTR, o0 = to * kTO;
  const int kb = kz * kper, ke = min(K, kb + kper);
  // loader roles: hidden row r0 + t/4 at k offsets (t%4)*8 and 32 + (t%4)*8;
  // R options o0 + t/8 and o0 + 32 + t/8 at k offsets (t%8)*4 and 32 + (t%8)*4
  const int hr = t >> 2, hk = (t & 3) * 8;
  const int ro = t >> 3, rk = (t & 7) * 4;
  const bool h_row_ok = r0 + hr < B;
  const bool r_ok0 = o0 + ro < n_opt, r_ok1 = o0 + 32 + ro < n_opt;
  const T* hp = hidden + (int64_t)min(r0 + hr, B - 1) * K;
  const float* rp0 = R + (int64_t)min(o0 + ro, n_opt - 1) * K;
  const float* rp1 = R + (int64_t)min(o0 + 32 + ro, n_opt - 1) * K;
  float hv[2][8];
  float4 rv[2][2];
  auto fetch = [&](int k0) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int kh = k0 + 32 * h;
      const bool hk_ok = kh + hk < ke, rk_ok = kh + rk < ke;  // K, kper and k0 are multiples of 8
      load_hidden8<T>(hp + kh + hk, h_row_ok && hk_ok, hv[h]);
      rv[h][0] = (r_ok0 && rk_ok) ? __ldg(reinterpret_cast<const float4*>(rp0 + kh + rk)) : make_float4(0.f, 0.f, 0.f, 0.f);
      rv[h][1] = (r_ok1 && rk_ok) ? __ldg(reinterpret_cast<const float4*>(rp1 + kh + rk)) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  auto stash = [&](int buf) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
#pragma unroll
      for (int i = 0; i < 8; ++i) hs(buf, 32 * h + hk + i)[hr] = hv[h][i];
      const float a[4] = {rv[h][0].x, rv[h][0].y, rv[h][0].z, rv[h][0].w};
      const float c[4] = {rv[h][1].x, rv[h][1].y, rv[h][1].z, rv[h][1].w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        rs(buf, 32 * h + rk + i)[ro] = a[i];
        rs(buf, 32 * h + rk + i)[32 + ro] = c[i];
      }
    }
  };
  const int ty = t >> 4, tx = t & 15;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  fetch(kb);
  stash(0);
  __syncthreads();
  int buf = 0;
  for (int k0 = kb; k0 < ke; k0 += kKC) {
    const bool more = k0 + kKC < ke;
    if (more) fetch(k0 + kKC);
#pragma unroll 8
    for (int kk = 0; kk < kKC; ++kk) {
      const float4 a = *reinterpret_cast<const float4*>(hs(buf, kk) + ty * 4);
      const float4 b = *reinterpret_cast<const float4*>(rs(buf, kk) + tx * 4);
      const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    if (more) stash(buf ^ 1);
    __syncthreads();
    buf ^= 1;
  }
  // partial sums of this K split: partials[kz][row][opt], padded to b_pad x o_pad
#pragma unroll
  for (int i = 0; i < 4; ++i)
    *reinterpret_cast<float4*>(partials + ((int64_t)kz * b_pad + r0 + ty * 4 + i) * o_pad + o0 + tx * 4) =
        make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);

}

// Second kernel of the tiled readout: one CTA per row adds the K-split partial
// logits in split order, then runs the masked softmax of the row.
__global__ void __launch_bounds__(256) readout_reduce_softmax_kernel(const float* __restrict__ partials,
                                                                     const int32_t* __restrict__ counts,
                                                                     float temperature, float* __restrict__ probs,
                                                                     int n_opt, int ksplit, int b_pad, int o_pad) {
  __shared__ float red[8];
  __shared__ float bcast;
  const int row = blockIdx.x, t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int cnt = counts[row];
  constexpr int kPer = kMaxOpts / 256;
  float v[kPer];
  float mx = -INFINITY;
  const int64_t zstride = (int64_t)b_pad * o_pad;
  const float* base = partials + (int64_t)row * o_pad;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int j = t + 256 * i;
    float x = -INFINITY;
    if (j < n_opt) {
      float acc = 0.f;
      int z = 0;
      for (; z + 4 <= ksplit; z += 4) {  // four loads in flight, added in split order
        const float p0 = base[z * zstride + j], p1 = base[(z + 1) * zstride + j];
        const float p2 = base[(z + 2) * zstride + j], p3 = base[(z + 3) * zstride + j];
        acc += p0; acc += p1; acc += p2; acc += p3;
      }
      for (; z < ksplit; ++z) acc += base[z * zstride + j];
      if (j < cnt) x = acc / temperature;
    }
    v[i] = x;
    mx = fmaxf(mx, x);
  }
#pragma unroll
  for (int s = 16; s > 0; s >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, s));
  if (lane == 0) red[warp] = mx;
  __syncthreads();
  if (t == 0) {
    float m = red[0];
    for (int w = 1; w < 8; ++w) m = fmaxf(m, red[w]);
    bcast = m;
  }
  __syncthreads();
  mx = bcast;
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const float e = (v[i] == -INFINITY) ? 0.f : expf(v[i] - mx);
    v[i] = e;
    sum += e;
  }
#pragma unroll
  for (int s = 16; s > 0; s >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, s);
  __syncthreads();
  if (lane == 0) red[warp] = sum;
  __syncthreads();
  if (t == 0) {
    float m = 0.f;
    for (int w = 0; w < 8; ++w) m += red[w];  // fixed order
    bcast = m;
  }
  __syncthreads();
  sum = bcast;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int j = t + 256 * i;
    // a row with count <= 0 is all -inf in the reference; softmax gives NaN
    if (j < n_opt) probs[(int64_t)row * n_opt + j] = (cnt > 0) ? v[i] / sum : __int_as_float(0x7fc00000);
  }
}

struct TiledShape {
  int kper, ksplit, b_pad, o_pad;
};

inline TiledShape tiled_shape(int B, int K, int n_opt) {
  TiledShape sh;
  sh.b_pad = (B + kTR - 1) / kTR * kTR;
  sh.o_pad = (n_opt + kTO - 1) / kTO * kTO;
  const int tiles = (sh.b_pad / kTR) * (sh.o_pad / kTO);
  const int sms = std::max(1, d3b_host::num_sms(d3b_host::current_device()));
  int want = (3 * sms + tiles - 1) / tiles;                 // about three CTAs per SM
  want = std::max(1, std::min(want, std::min(kMaxSplit, K / 128)));  // at least 128 k per split
  sh.kper = ((K + want - 1) / want + kKC - 1) / kKC * kKC;
  sh.ksplit = (K + sh.kper - 1) / sh.kper;
  return sh;
}

template <typename T>
void launch_tiled(const void* hidden, const float* readout, const int32_t* counts, float temperature, float* probs,
                  int B, int K, int n_opt, float* partials, cudaStream_t s) {
  const TiledShape sh = tiled_shape(B, K, n_opt);
  const dim3 grid(sh.b_pad / kTR, sh.o_pad / kTO, sh.ksplit), block(256);
  static int attr_set[64] = {0};
  const int dev = d3b_host::current_device();
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    cudaFuncSetAttribute(readout_tiled_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTiledSmem);
    attr_set[dev] = 1;
  }
  readout_tiled_kernel<T><<<grid, block, kTiledSmem, s>>>(static_cast<const T*>(hidden), readout, B, K, n_opt, sh.kper,
                                                          sh.b_pad, sh.o_pad, partials);
  readout_reduce_softmax_kernel<<<B, 256, 0, s>>>(partials, counts, temperature, probs, n_opt, sh.ksplit, sh.b_pad,
                                                  sh.o_pad);
}

template <typename T>
void launch_typed(const void* hidden, const float* readout, const int32_t* counts, float temperature, float* probs,
                  int B, int K, int n_opt, float* logits, unsigned int* tickets, cudaStream_t s) {
  dim3 grid((B + kRows - 1) / kRows, (n_opt + kOpts - 1) / kOpts), block(kRows * 32);
  // vector path: 16-byte aligned rows of hidden and readout (K * sizeof(T) and K * 4 multiples of 16)
  const bool vec = (K % 8 == 0) && (reinterpret_cast<uintptr_t>(readout) % 16 == 0) &&
                   (reinterpret_cast<uintptr_t>(hidden) % 16 == 0);
  if (vec)
    readout_kernel<T, true><<<grid, block, 0, s>>>(static_cast<const T*>(hidden), readout, counts, temperature,
                                                   probs, B, K, n_opt, logits, tickets);
  else
    readout_kernel<T, false><<<grid, block, 0, s>>>(static_cast<const T*>(hidden), readout, counts, temperature,
                                                    probs, B, K, n_opt, logits, tickets);
}

}  // namespace

// Workspace of d3b_readout:
//   [tickets: kTiledTicketBytes][logits: B x n_opt f32][partials: kMaxSplit x b_pad x o_pad f32]
// (the fallback kernel for unaligned rows uses the first kTicketBytes of the
// ticket region and the logits).
extern "C" size_t d3b_readout_workspace_size(int B, int n_opt) {
  if (B <= 0 || n_opt <= 0) return 0;
  const size_t b_pad = (size_t)(B + kTR - 1) / kTR * kTR, o_pad = (size_t)(n_opt + kTO - 1) / kTO * kTO;
  return kTiledTicketBytes + (((size_t)B * n_opt * sizeof(float) + 255) & ~(size_t)255) +
         (size_t)kMaxSplit * b_pad * o_pad * sizeof(float);
}

extern "C" int d3b_readout(const void* hidden, int h_dtype, const float* readout, const int32_t* counts,
                           float temperature, float* probs, int B, int K, int n_opt, void* workspace,
                           size_t workspace_bytes, d3b_stream_t stream) {
  if (B < 0 || K <= 0 || n_opt <= 0 || n_opt > kMaxOpts) return D3B_EINVAL;
  if (B > kRows * kMaxGroups) return D3B_EINVAL;
  if (!(temperature > 0.f)) return D3B_EINVAL;
  if (B == 0) return D3B_OK;
  if (!hidden || !readout || !counts || !probs || !workspace) return D3B_EINVAL;
  if (workspace_bytes < d3b_readout_workspace_size(B, n_opt)) return D3B_ENOSPACE;
  if (reinterpret_cast<uintptr_t>(workspace) % 16) return D3B_EALIGN;
  unsigned int* tickets = static_cast<unsigned int*>(workspace);
  float* logits = reinterpret_cast<float*>(static_cast<char*>(workspace) + kTiledTicketBytes);
  float* partials = reinterpret_cast<float*>(static_cast<char*>(workspace) + kTiledTicketBytes +
                                             (((size_t)B * n_opt * sizeof(float) + 255) & ~(size_t)255));
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int esize = h_dtype == D3B_F32 ? 4 : 2;
  const bool tiled = (K % 8 == 0) && (reinterpret_cast<uintptr_t>(readout) % 16 == 0) &&
                     (reinterpret_cast<uintptr_t>(hidden) % 16 == 0) && ((int64_t)K * esize % 16 == 0);
  switch (h_dtype) {
    case D3B_F32:
      if (tiled) launch_tiled<float>(hidden, readout, counts, temperature, probs, B, K, n_opt, partials, s);
      else launch_typed<float>(hidden, readout, counts, temperature, probs, B, K, n_opt, logits, tickets, s);
      break;
    case D3B_F16:
      if (tiled) launch_tiled<__half>(hidden, readout, counts, temperature, probs, B, K, n_opt, partials, s);
      else launch_typed<__half>(hidden, readout, counts, temperature, probs, B, K, n_opt, logits, tickets, s);
      break;
    case D3B_BF16:
      if (tiled)
        launch_tiled<__nv_bfloat16>(hidden, readout, counts, temperature, probs, B, K, n_opt, partials, s);
      else launch_typed<__nv_bfloat16>(hidden, readout, counts, temperature, probs, B, K, n_opt, logits, tickets, s);
      break;
    default: return D3B_EUNSUPPORTED;
  }
  return d3b_host::check_launch();
}

namespace {

// ===========================================================================
// Tensor-core readout for bf16 hidden rows (the model's final-norm output).
//
// The fp32 readout matrix is split once into three bf16 planes,
// R = r0 + r1 + r2 with r0 = bf16(R), r1 = bf16(R - r0), r2 = bf16(R - r0 - r1)
// (each difference is exact in fp32, and the three planes carry all 24 bits of
// R). Every product of a bf16 hidden value with a plane value is exact in fp32,
// so hidden . R = sum_p hidden . r_p is an fp32 dot product that differs from
// the reference's SGEMM only in summation order. The products run on tcgen05
// (kind::f16, bf16 x bf16, fp32 accumulate in TMEM): one CTA per (128-row tile,
// 256-option tile, K split) streams its hidden rows and the three planes' rows
// by TMA in 64-wide K chunks (two stages), accumulates all three planes into one
// 128 x 256 fp32 accumulator, and writes it as one split's partial logits; the
// reduce/softmax kernel above then adds the splits in order and applies the mask,
// the temperature and the softmax.
// ===========================================================================
constexpr int kTcRows = 128, kTcOpts = 256, kTcK = 64;   // tile and K chunk
constexpr int kTcChunkA = kTcRows * kTcK * 2;            // 16 KB
constexpr int kTcChunkB = kTcOpts * kTcK * 2;            // 32 KB per plane
constexpr int kTcStage = kTcChunkA + 3 * kTcChunkB;      // 112 KB
constexpr int kTcSmem = 2 * kTcStage + 1024;
constexpr int kTcChunksPerCta = 4;  // 2-5 chunks per CTA time alike at 255 x 5120 x 255 (23.5 us); 4 halves the partials of 2
constexpr int kTcMaxSplit = 128;

enum : int { kSiteTcFull = 4101, kSiteTcEmpty = 4102, kSiteTcDone = 4103 };

struct TcBars {
  uint64_t full[2], empty[2], done;
  uint32_t tmem_slot;
  int abort_flag;
};

__global__ void __launch_bounds__(128, 1)
    readout_tc_kernel(const __grid_constant__ CUtensorMap mapH, const __grid_constant__ CUtensorMap mapP, int K,
                      int o_pad, int b_pad, int kper, float* __restrict__ partials, int* err) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ TcBars bars;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5;
  const int r0 = blockIdx.x * kTcRows, o0 = blockIdx.y * kTcOpts, kz = blockIdx.z;
  const int kb = kz * kper, ke = min(K, kb + kper);
  const int nch = (ke - kb + kTcK - 1) / kTcK;
  volatile int* abort_flag = &bars.abort_flag;
  if (tid == 0) {
    for (int s = 0; s < 2; ++s) {
      d3b::mbar_init(&bars.full[s], 1);
      d3b::mbar_init(&bars.empty[s], 1);
    }
    d3b::mbar_init(&bars.done, 1);
    bars.abort_flag = 0;
    d3b::fence_barrier_init();
  }
  if (warp == 0) d3b::tmem_alloc(&bars.tmem_slot, 256);
  d3b::tc_fence_before();
  __syncthreads();
  d3b::tc_fence_after();
  const uint32_t tmem = bars.tmem_slot;
  bool ok = true;
  if (tid == 0) {
    // one thread loads and issues: chunk c in stage c % 2; planes p at option rows p * o_pad + o0
    d3b::tma_prefetch_desc(&mapH);
    d3b::tma_prefetch_desc(&mapP);
    auto load = [&](int c) {
      uint8_t* st = smem + (c & 1) * kTcStage;
      const int k0 = kb + c * kTcK;
      d3b::mbar_arrive_expect_tx(&bars.full[c & 1], kTcStage);
      d3b::tma_load_2d(st, &mapH, &bars.full[c & 1], k0, r0);
#pragma unroll
      for (int p = 0; p < 3; ++p)
        d3b::tma_load_2d(st + kTcChunkA + p * kTcChunkB, &mapP, &bars.full[c & 1], k0, p * o_pad + o0);
    };
    constexpr uint32_t idesc = d3b::make_idesc(1, 1, 1, 0, 0, kTcRows, kTcOpts);
    const uint32_t s_base = d3b::smem_u32(smem);
    for (int c = 0; c < nch && c < 2; ++c) load(c);
    for (int c = 0; c < nch; ++c) {
      const int s = c & 1;
      if (!(ok = d3b::mbar_wait(&bars.full[s], (uint32_t)(c >> 1) & 1, abort_flag, err, kSiteTcFull))) break;
      d3b::tc_fence_after();
      const uint32_t st = s_base + s * kTcStage;
#pragma unroll
      for (int p = 0; p < 3; ++p)
#pragma unroll
        for (int k = 0; k < kTcK / 16; ++k) {
          const uint64_t a = d3b::make_smem_desc(st + k * 32, 16, 1024, d3b::kLayoutSW128);
          const uint64_t b = d3b::make_smem_desc(st + kTcChunkA + p * kTcChunkB + k * 32, 16, 1024, d3b::kLayoutSW128);
          d3b::mma_f16_ss(tmem, a, b, idesc, (c > 0 || p > 0 || k > 0) ? 1u : 0u);
        }
      d3b::mma_commit(&bars.empty[s]);
      if (c + 2 < nch) {
        if (!(ok = d3b::mbar_wait(&bars.empty[s], (uint32_t)(c >> 1) & 1, abort_flag, err, kSiteTcEmpty))) break;
        load(c + 2);
      }
    }
    d3b::mma_commit(&bars.done);
  }
  __syncwarp();
  // epilogue: thread = row r0 + tid (TMEM lane), 256 partial logits of this split
  ok = d3b::warp_wait(&bars.done, 0, abort_flag, err, kSiteTcDone);
  d3b::tc_fence_after();
  if (ok) {
    const uint32_t lane_addr = tmem + ((uint32_t)(warp * 32) << 16);
    float* dst = partials + ((int64_t)kz * b_pad + r0 + tid) * o_pad + o0;
#pragma unroll 1
    for (int c = 0; c < kTcOpts / 32; ++c) {
      uint32_t v[32];
      d3b::tmem_ld32(lane_addr + c * 32, v);
      d3b::tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 32; i += 4)
        *reinterpret_cast<float4*>(dst + c * 32 + i) =
            make_float4(__uint_as_float(v[i]), __uint_as_float(v[i + 1]), __uint_as_float(v[i + 2]),
                        __uint_as_float(v[i + 3]));
    }
  }
  d3b::tc_fence_before();
  __syncthreads();
  d3b::tc_fence_after();
  if (warp == 0) d3b::tmem_dealloc(tmem, 256);
}

// R fp32 [n_opt, K] -> three bf16 planes [3][o_pad][K] (rows >= n_opt zero)
__global__ void __launch_bounds__(256) readout_split_kernel(const float* __restrict__ R, int n_opt, int K, int o_pad,
                                                            __nv_bfloat16* __restrict__ planes) {
  const int64_t n = (int64_t)o_pad * K;
  for (int64_t i = (int64_t)blockIdx.x * 256 + threadIdx.x; i < n; i += (int64_t)gridDim.x * 256) {
    const int64_t o = i / K;
    const float x = o < n_opt ? R[i] : 0.f;
    const __nv_bfloat16 a = __float2bfloat16_rn(x);
    const float r1 = x - __bfloat162float(a);  // exact
    const __nv_bfloat16 b = __float2bfloat16_rn(r1);
    const __nv_bfloat16 c = __float2bfloat16_rn(r1 - __bfloat162float(b));  // exact difference
    planes[i] = a;
    planes[n + i] = b;
    planes[2 * n + i] = c;
  }
}

struct TcShape {
  int b_pad, o_pad, kper, ksplit;
};

inline TcShape tc_shape(int B, int K, int n_opt) {
  TcShape sh;
  sh.b_pad = (B + kTcRows - 1) / kTcRows * kTcRows;
  sh.o_pad = (n_opt + kTcOpts - 1) / kTcOpts * kTcOpts;
  const int chunks = (K + kTcK - 1) / kTcK;
  sh.ksplit = std::min(kTcMaxSplit, std::max(1, (chunks + kTcChunksPerCta - 1) / kTcChunksPerCta));
  sh.kper = (chunks + sh.ksplit - 1) / sh.ksplit * kTcK;
  sh.ksplit = (K + sh.kper - 1) / sh.kper;
  return sh;
}

}  // namespace

extern "C" size_t d3b_readout_planes_size(int n_opt, int K) {
  if (n_opt <= 0 || K <= 0) return 0;
  return (size_t)3 * ((n_opt + kTcOpts - 1) / kTcOpts * kTcOpts) * K * 2;
}

extern "C" int d3b_readout_split(const float* readout, int n_opt, int K, void* planes, d3b_stream_t stream) {
  if (n_opt <= 0 || K <= 0 || !readout || !planes) return D3B_EINVAL;
  const int o_pad = (n_opt + kTcOpts - 1) / kTcOpts * kTcOpts;
  const int64_t n = (int64_t)o_pad * K;
  const int blocks = (int)std::min<int64_t>((n + 255) / 256, 4096);
  readout_split_kernel<<<blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      readout, n_opt, K, o_pad, static_cast<__nv_bfloat16*>(planes));
  return d3b_host::check_launch();
}

extern "C" size_t d3b_readout_planes_workspace_size(int B, int K, int n_opt) {
  if (B <= 0 || K <= 0 || n_opt <= 0) return 0;
  const TcShape sh = tc_shape(B, K, n_opt);
  return (size_t)sh.ksplit * sh.b_pad * sh.o_pad * sizeof(float);
}

extern "C" int d3b_readout_planes(const void* hidden, const void* planes, const int32_t* counts, float temperature,
                                  float* probs, int B, int K, int n_opt, void* workspace, size_t workspace_bytes,
                                  d3b_stream_t stream) {
  if (B < 0 || K <= 0 || n_opt <= 0 || n_opt > kMaxOpts) return D3B_EINVAL;
  if (!(temperature > 0.f)) return D3B_EINVAL;
  if (B == 0) return D3B_OK;
  if (!hidden || !planes || !counts || !probs || !workspace) return D3B_EINVAL;
  if (K % 8) return D3B_EUNSUPPORTED;  // rows of 16-byte multiples (TMA)
  if (reinterpret_cast<uintptr_t>(hidden) % 16 || reinterpret_cast<uintptr_t>(planes) % 16 ||
      reinterpret_cast<uintptr_t>(workspace) % 16)
    return D3B_EALIGN;
  if (workspace_bytes < d3b_readout_planes_workspace_size(B, K, n_opt)) return D3B_ENOSPACE;
  const TcShape sh = tc_shape(B, K, n_opt);
  int* err = d3b_host::device_error_word();
  if (!err) return D3B_ECUDA;
  CUtensorMap maps[2];
  int rc;
  {  // hidden [B, K] bf16: dims {K, B}, box {64, 128}; rows past B read as zero
    const uint64_t dims[2] = {(uint64_t)K, (uint64_t)B};
    const uint64_t st[1] = {(uint64_t)K * 2};
    const uint32_t box[2] = {(uint32_t)kTcK, (uint32_t)kTcRows};
    if ((rc = d3b_host::encode_tiled(&maps[0], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, hidden, dims, st, box,
                                     CU_TENSOR_MAP_SWIZZLE_128B)))
      return rc;
  }
  {  // planes [3 * o_pad, K] bf16: box {64, 256}
    const uint64_t dims[2] = {(uint64_t)K, (uint64_t)3 * sh.o_pad};
    const uint64_t st[1] = {(uint64_t)K * 2};
    const uint32_t box[2] = {(uint32_t)kTcK, (uint32_t)kTcOpts};
    if ((rc = d3b_host::encode_tiled(&maps[1], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, planes, dims, st, box,
                                     CU_TENSOR_MAP_SWIZZLE_128B)))
      return rc;
  }
  static int attr_set[64] = {0};
  const int dev = d3b_host::current_device();
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    if (cudaFuncSetAttribute(readout_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem) != cudaSuccess)
      return D3B_ECUDA;
    attr_set[dev] = 1;
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  float* partials = static_cast<float*>(workspace);
  const dim3 grid(sh.b_pad / kTcRows, sh.o_pad / kTcOpts, sh.ksplit);
  readout_tc_kernel<<<grid, 128, kTcSmem, s>>>(maps[0], maps[1], K, sh.o_pad, sh.b_pad, sh.kper, partials, err);
  if (const int st = d3b_host::check_launch()) return st;
  readout_reduce_softmax_kernel<<<B, 256, 0, s>>>(partials, counts, temperature, probs, n_opt, sh.ksplit, sh.b_pad,
                                                  sh.o_pad);
  return d3b_host::check_launch();
}

namespace {
}  // namespace

// ===========================================================================
// Readout without any allocation.
//
// Some callers cannot allocate device memory at call time: code that runs
// while a CUDA graph is being captured, host runtimes that hand the library
// only input and output buffers, or processes whose allocator is owned by
// someone else. For them this entry point keeps the readout's scratch (the
// ticket counters and the logits) in one fixed array that lives in the
// library itself. Every GPU that loads the library holds these bytes until
// the process exits.
//
// Limits: B * n_opt * 4 bytes of logits plus the ticket region must fit in
// kNoAllocScratchBytes (1 MiB), i.e. up to 258048 logits (B = 255 questions
// at 255 options needs 65025); larger requests return D3B_ENOSPACE before any
// work is enqueued.
//
// All calls on a device share the array and it keeps the last call's
// contents. Each call clears the ticket counters it uses on its own stream
// before the kernel runs; the logits need no clearing (every logit is written
// before it is read). Two calls whose work overlaps on the GPU (different
// streams, no ordering between them) race on the array and give wrong results.
//
// Set-up: the first call on a device looks up the array's device address
// (cudaGetSymbolAddress) with that device current and caches it. Make that
// first call before any stream capture begins.
// ===========================================================================
namespace {

constexpr size_t kNoAllocScratchBytes = 1u << 20;
static __device__ __align__(256) unsigned char g_readout_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mu;
void* g_noalloc_addr[64] = {nullptr};

// Device address of g_readout_scratch on the current device (the symbol's
// name in host code is only a stand-in, never a device address).
int noalloc_scratch(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return D3B_ECUDA;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_addr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_readout_scratch) != cudaSuccess || !p) return D3B_ECUDA;
    g_noalloc_addr[dev] = p;
  }
  *out = g_noalloc_addr[dev];
  return D3B_OK;
}

}  // namespace

extern "C" int d3b_readout_noalloc(const void* hidden, int h_dtype, const float* readout, const int32_t* counts,
                                   float temperature, float* probs, int B, int K, int n_opt, d3b_stream_t stream) {
  if (B < 0 || K <= 0 || n_opt <= 0 || n_opt > kMaxOpts) return D3B_EINVAL;
  if (B > kRows * kMaxGroups) return D3B_EINVAL;
  if (!(temperature > 0.f)) return D3B_EINVAL;
  if (B == 0) return D3B_OK;
  if (!hidden || !readout || !counts || !probs) return D3B_EINVAL;
  if (h_dtype != D3B_F32 && h_dtype != D3B_F16 && h_dtype != D3B_BF16) return D3B_EUNSUPPORTED;
  if (kTicketBytes + (((size_t)B * n_opt * sizeof(float) + 255) & ~(size_t)255) > kNoAllocScratchBytes)
    return D3B_ENOSPACE;
  void* scratch = nullptr;
  const int rc = noalloc_scratch(&scratch);
  if (rc != D3B_OK) return rc;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // the ticket counters must start at zero: clear the ones this launch uses
  const size_t groups = (size_t)(B + kRows - 1) / kRows;
  if (cudaMemsetAsync(scratch, 0, groups * sizeof(unsigned int), s) != cudaSuccess) return D3B_ECUDA;
  unsigned int* tickets = static_cast<unsigned int*>(scratch);
  float* logits = reinterpret_cast<float*>(static_cast<char*>(scratch) + kTicketBytes);
  switch (h_dtype) {
    case D3B_F32: launch_typed<float>(hidden, readout, counts, temperature, probs, B, K, n_opt, logits, tickets, s); break;
    case D3B_F16: launch_typed<__half>(hidden, readout, counts, temperature, probs, B, K, n_opt, logits, tickets, s); break;
    default:
      launch_typed<__nv_bfloat16>(hidden, readout, counts, temperature, probs, B, K, n_opt, logits, tickets, s);
      break;
  }
  return d3b_host::check_launch();
}
