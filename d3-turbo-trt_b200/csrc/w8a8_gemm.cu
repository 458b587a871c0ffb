// W8A8 scaled GEMM on the 5th-generation tensor cores (tcgen05), sm_100a.
//
//   y[m, n] = (sum_k qa[m, k] * qw[n, k]) * sa[m] * sw[n]
//
// Replaces torch._scaled_mm rowwise (d3trt/model/quant.py:164-179, e4m3 x e4m3
// with fp32 accumulate, bf16 out) and torch._int_mm + the ATen dequant chain
// (quant.py:190-197, int8 x int8 with int32 accumulate).
//
// Structure (one persistent CTA per SM, 6 warps):
//   warp 0      TMA producer: A tile 128x128 B and B tile 256x128 B per stage,
//               128-byte swizzle, 4-stage ring (48 KB per stage)
//   warp 1      TMEM owner + MMA issuer (one thread): 4 x tcgen05.mma
//               (M=128, N=256, K=32) per stage, kind::f8f6f4 (e4m3) or
//               kind::i8 (s8, s32 accumulate), then tcgen05.commit to release
//               the stage; one commit per tile to hand the accumulator over
//   warps 2..5  epilogue: tcgen05.ld 32 lanes x 32 columns, multiply by
//               sa[m] then sw[n] in fp32 ((acc * sa) * sw, the reference
//               order), round to bf16/f16 or store f32 / raw int32
// The accumulator is double-buffered in TMEM (2 x 256 columns of 512), so the
// epilogue of tile t overlaps the main loop of tile t+1.
#include "common.cuh"

namespace {

constexpr int BM = 128, BN = 256, BK = 128;  // BK in bytes = elements (8-bit)
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK;               // 16 KB
constexpr int B_BYTES = BN * BK;               // 32 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;  // 48 KB
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024;
constexpr int NUM_THREADS = 192;
constexpr uint32_t TMEM_COLS = 512;

// Wait-site codes (device error word): 1000 + role.
enum { kSiteProducer = 1001, kSiteMma = 1002, kSiteMmaAcc = 1003, kSiteEpi = 1004, kSiteDrain = 1005 };

struct __align__(8) Barriers {
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t drain;
  uint32_t tmem_slot;
  int abort_flag;
};

__device__ __forceinline__ void store_chunk(void* out, int64_t ldo, int out_kind, int row, int M, int n_base, int N,
                                            const uint32_t (&acc)[32], float sa_row, const float* __restrict__ sw,
                                            bool is_int) {
  if (row >= M) return;
  if (out_kind == D3B_I32 || out_kind == D3B_F32) {
    uint32_t* dst = reinterpret_cast<uint32_t*>(out) + (int64_t)row * ldo + n_base;
#pragma unroll
    for (int g = 0; g < 8; ++g) {
      const int n = n_base + g * 4;
      if (n + 4 > N) break;
      uint4 v;
      if (out_kind == D3B_I32) {
        v = make_uint4(acc[4 * g], acc[4 * g + 1], acc[4 * g + 2], acc[4 * g + 3]);
      } else {
        const float4 w = __ldg(reinterpret_cast<const float4*>(sw + n));
        float f[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float a = is_int ? (float)(int)acc[4 * g + j] : __uint_as_float(acc[4 * g + j]);
          f[j] = a * sa_row;
        }
        v = make_uint4(__float_as_uint(f[0] * w.x), __float_as_uint(f[1] * w.y), __float_as_uint(f[2] * w.z),
                       __float_as_uint(f[3] * w.w));
      }
      *reinterpret_cast<uint4*>(dst + g * 4) = v;
    }
    return;
  }
  // 16-bit outputs: 8 elements (16 bytes) per store
  uint16_t* dst = reinterpret_cast<uint16_t*>(out) + (int64_t)row * ldo + n_base;
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const int n = n_base + g * 8;
    if (n + 8 > N) break;
    const float4 w0 = __ldg(reinterpret_cast<const float4*>(sw + n));
    const float4 w1 = __ldg(reinterpret_cast<const float4*>(sw + n + 4));
    const float ws[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
    float f[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t raw = acc[8 * g + j];
      const float a = is_int ? (float)(int)raw : __uint_as_float(raw);
      f[j] = (a * sa_row) * ws[j];
    }
    uint4 v;
    if (out_kind == D3B_BF16) {
      v = make_uint4(d3b::pack_bf16x2(f[0], f[1]), d3b::pack_bf16x2(f[2], f[3]), d3b::pack_bf16x2(f[4], f[5]),
                     d3b::pack_bf16x2(f[6], f[7]));
    } else {
      v = make_uint4(d3b::pack_f16x2(f[0], f[1]), d3b::pack_f16x2(f[2], f[3]), d3b::pack_f16x2(f[4], f[5]),
                     d3b::pack_f16x2(f[6], f[7]));
    }
    *reinterpret_cast<uint4*>(dst + g * 8) = v;
  }
}

template <int MODE>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    w8a8_gemm_kernel(const __grid_constant__ CUtensorMap mapA, const __grid_constant__ CUtensorMap mapB,
                     const float* __restrict__ sa, const float* __restrict__ sw, void* __restrict__ out, int64_t ldo,
                     int M, int N, int K, int out_kind, int* err) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ Barriers bars;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_m = (M + BM - 1) / BM, num_n = (N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int num_kb = (K + BK - 1) / BK;
  volatile int* abort_flag = &bars.abort_flag;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      d3b::mbar_init(&bars.full[s], 1);
      d3b::mbar_init(&bars.empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      d3b::mbar_init(&bars.tfull[a], 1);
      d3b::mbar_init(&bars.tempty[a], 128);
    }
    d3b::mbar_init(&bars.drain, 1);
    bars.abort_flag = 0;
    d3b::fence_barrier_init();
    d3b::tma_prefetch_desc(&mapA);
    d3b::tma_prefetch_desc(&mapB);
  }
  if (warp == 1) d3b::tmem_alloc(&bars.tmem_slot, TMEM_COLS);
  d3b::tc_fence_before();
  __syncthreads();
  d3b::tc_fence_after();
  const uint32_t tmem_base = bars.tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int t = blockIdx.x; t < num_tiles && !*abort_flag; t += gridDim.x) {
        const int m0 = (t % num_m) * BM, n0 = (t / num_m) * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!d3b::mbar_wait(&bars.empty[stage], phase ^ 1, abort_flag, err, kSiteProducer)) break;
          d3b::mbar_arrive_expect_tx(&bars.full[stage], STAGE_BYTES);
          d3b::tma_load_2d(sA + stage * A_BYTES, &mapA, &bars.full[stage], kb * BK, m0);
          d3b::tma_load_2d(sB + stage * B_BYTES, &mapB, &bars.full[stage], kb * BK, n0);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = MODE == D3B_MODE_FP8 ? d3b::make_idesc(1, 0, 0, 0, 0, BM, BN)   // f32 <- e4m3
                                                       : d3b::make_idesc(2, 1, 1, 0, 0, BM, BN);  // s32 <- s8
      const uint32_t a_base = d3b::smem_u32(sA), b_base = d3b::smem_u32(sB);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      for (int t = blockIdx.x; t < num_tiles && !*abort_flag; t += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!d3b::mbar_wait(&bars.tempty[acc], acc_phase ^ 1, abort_flag, err, kSiteMmaAcc)) break;
        d3b::tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!d3b::mbar_wait(&bars.full[stage], phase, abort_flag, err, kSiteMma)) break;
          d3b::tc_fence_after();
#pragma unroll
          for (int k = 0; k < BK / 32; ++k) {
            const uint64_t ad = d3b::make_smem_desc(a_base + stage * A_BYTES + k * 32, 16, 1024, d3b::kLayoutSW128);
            const uint64_t bd = d3b::make_smem_desc(b_base + stage * B_BYTES + k * 32, 16, 1024, d3b::kLayoutSW128);
            const uint32_t accum = (kb > 0 || k > 0) ? 1u : 0u;
            if (MODE == D3B_MODE_FP8)
              d3b::mma_f8f6f4_ss(d_tmem, ad, bd, idesc, accum);
            else
              d3b::mma_i8_ss(d_tmem, ad, bd, idesc, accum);
          }
          d3b::mma_commit(&bars.empty[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        d3b::mma_commit(&bars.tfull[acc]);
      }
      // Drain: arrive once every MMA issued above has completed, so TMEM is
      // never released under a running MMA (also on the abort path).
      d3b::mma_commit(&bars.drain);
      const uint32_t addr = d3b::smem_u32(&bars.drain);
      const uint64_t t0 = d3b::globaltimer_ns();
      while (!d3b::mbar_try_wait(addr, 0)) {
        if (d3b::globaltimer_ns() - t0 > D3B_WAIT_LIMIT_NS) {
          d3b::record_device_error(err, kSiteDrain);
          break;
        }
      }
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    const int row_in_tile = quarter * 32 + lane;
    const bool is_int = MODE == D3B_MODE_INT8;
    int local = 0;
    for (int t = blockIdx.x; t < num_tiles && !*abort_flag; t += gridDim.x, ++local) {
      const int m0 = (t % num_m) * BM, n0 = (t / num_m) * BN;
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!d3b::warp_wait(&bars.tfull[acc], acc_phase, abort_flag, err, kSiteEpi)) break;
      d3b::tc_fence_after();
      const int row = m0 + row_in_tile;
      const float sa_row = (out_kind != D3B_I32 && row < M) ? __ldg(sa + row) : 0.f;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        d3b::tmem_ld32(tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN + c * 32, r);
        d3b::tmem_wait_ld();
        if (c == BN / 32 - 1) {
          // every TMEM read of this accumulator is done: hand it back
          d3b::tc_fence_before();
          d3b::mbar_arrive(&bars.tempty[acc]);
        }
        store_chunk(out, ldo, out_kind, row, M, n0 + c * 32, N, r, sa_row, sw, is_int);
      }
    }
  }

  d3b::tc_fence_before();
  __syncthreads();
  d3b::tc_fence_after();
  if (warp == 1) d3b::tmem_dealloc(tmem_base, TMEM_COLS);
}

// ===========================================================================
// CTA-pair form (cluster of 2, tcgen05 cta_group::2) for M >= 512: the pair owns
// a 256 x 256 output tile. Each CTA TMA-loads its own 128 rows of A and its own
// 128 rows of B per stage (no multicast), both completing on rank 0's "full"
// barrier, which rank 0 alone arms with the pair's bytes; rank 0's MMA thread issues M=256 N=256 K=32 instructions that read A
// and B from both CTAs' shared memory and accumulate 128 rows x 256 columns into
// each CTA's TMEM. Compared with one CTA per SM (M=128, N=256), each SM writes
// and feeds the tensor core 32 KB of operands per 4 instructions instead of
// 48 KB, so shared-memory bandwidth no longer caps the MMA rate, and 6 stages
// fit. Commits go to both CTAs' barriers (tcgen05.commit multicast); each CTA's
// epilogue hands the accumulator back to rank 0 with a remote arrive.
// ===========================================================================
constexpr int P_BM = 128, P_BN = 256, P_STAGES = 6;
constexpr int P_A_BYTES = P_BM * BK;                     // 16 KB: this CTA's 128 rows of A
constexpr int P_B_BYTES = (P_BN / 2) * BK;               // 16 KB: this CTA's 128 rows of B
constexpr int P_STAGE_BYTES = P_A_BYTES + P_B_BYTES;
constexpr int P_SMEM_BYTES = P_STAGES * P_STAGE_BYTES + 1024;

enum { kSitePairProducer = 1101, kSitePairMma, kSitePairMmaAcc, kSitePairEpi, kSitePairDrain };

struct __align__(8) PairBarriers {
  uint64_t full[P_STAGES];   // rank 0: both CTAs' loads of the stage (rank 0 arms it with all bytes)
  uint64_t empty[P_STAGES];  // each CTA: the pair's MMAs of the stage are done
  uint64_t tfull[2];         // each CTA: accumulator ready
  uint64_t tempty[2];        // rank 0: both CTAs' epilogues done with the accumulator (256 arrivals)
  uint64_t drain;
  uint32_t tmem_slot;
  int abort_flag;
};

template <int MODE>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NUM_THREADS, 1)
    w8a8_gemm_pair_kernel(const __grid_constant__ CUtensorMap mapA, const __grid_constant__ CUtensorMap mapB,
                          const float* __restrict__ sa, const float* __restrict__ sw, void* __restrict__ out,
                          int64_t ldo, int M, int N, int K, int out_kind, int* err) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ PairBarriers bars;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + P_STAGES * P_A_BYTES;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = d3b::cluster_ctarank();
  const int pair = blockIdx.x >> 1, pairs = gridDim.x >> 1;
  const int num_m = (M + 2 * P_BM - 1) / (2 * P_BM), num_n = (N + P_BN - 1) / P_BN;
  const int num_tiles = num_m * num_n;
  const int num_kb = (K + BK - 1) / BK;
  volatile int* abort_flag = &bars.abort_flag;

  if (threadIdx.x == 0) {
    for (int s = 0; s < P_STAGES; ++s) {
      d3b::mbar_init(&bars.full[s], 1);
      d3b::mbar_init(&bars.empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      d3b::mbar_init(&bars.tfull[a], 1);
      d3b::mbar_init(&bars.tempty[a], 256);
    }
    d3b::mbar_init(&bars.drain, 1);
    bars.abort_flag = 0;
    d3b::fence_barrier_init();
    d3b::tma_prefetch_desc(&mapA);
    d3b::tma_prefetch_desc(&mapB);
  }
  if (warp == 1) d3b::tmem_alloc_pair(&bars.tmem_slot, TMEM_COLS);
  d3b::tc_fence_before();
  d3b::cluster_sync();  // both CTAs' barriers initialised before any remote arrive or commit
  d3b::tc_fence_after();
  const uint32_t tmem_base = bars.tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer (each CTA: its halves of A and B) ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int t = pair; t < num_tiles && !*abort_flag; t += pairs) {
        const int m0 = (t % num_m) * 2 * P_BM + (int)rank * P_BM, n0 = (t / num_m) * P_BN + (int)rank * (P_BN / 2);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!d3b::mbar_wait(&bars.empty[stage], phase ^ 1, abort_flag, err, kSitePairProducer)) break;
          // rank 0 arms the stage with both CTAs' bytes; rank 1's loads only complete
          // bytes on it (they may land before the arming: the phase still waits for
          // rank 0's arrival)
          if (rank == 0) d3b::mbar_arrive_expect_tx(&bars.full[stage], 2 * P_STAGE_BYTES);
          const uint32_t leader_full = d3b::cluster_addr(&bars.full[stage], 0);
          d3b::tma_load_2d_pair(sA + stage * P_A_BYTES, &mapA, leader_full, kb * BK, m0);
          d3b::tma_load_2d_pair(sB + stage * P_B_BYTES, &mapB, leader_full, kb * BK, n0);
          if (++stage == P_STAGES) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (rank 0 only) ----------------
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = MODE == D3B_MODE_FP8 ? d3b::make_idesc(1, 0, 0, 0, 0, 2 * P_BM, P_BN)
                                                       : d3b::make_idesc(2, 1, 1, 0, 0, 2 * P_BM, P_BN);
      const uint32_t a_base = d3b::smem_u32(sA), b_base = d3b::smem_u32(sB);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      for (int t = pair; t < num_tiles && !*abort_flag; t += pairs, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!d3b::mbar_wait(&bars.tempty[acc], acc_phase ^ 1, abort_flag, err, kSitePairMmaAcc)) break;
        d3b::tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * P_BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!d3b::mbar_wait(&bars.full[stage], phase, abort_flag, err, kSitePairMma)) break;
          d3b::tc_fence_after();
#pragma unroll
          for (int k = 0; k < BK / 32; ++k) {
            const uint64_t ad = d3b::make_smem_desc(a_base + stage * P_A_BYTES + k * 32, 16, 1024, d3b::kLayoutSW128);
            const uint64_t bd = d3b::make_smem_desc(b_base + stage * P_B_BYTES + k * 32, 16, 1024, d3b::kLayoutSW128);
            const uint32_t accum = (kb > 0 || k > 0) ? 1u : 0u;
            if (MODE == D3B_MODE_FP8)
              d3b::mma_f8f6f4_pair(d_tmem, ad, bd, idesc, accum);
            else
              d3b::mma_i8_pair(d_tmem, ad, bd, idesc, accum);
          }
          d3b::mma_commit_pair(&bars.empty[stage], 0x3);
          if (++stage == P_STAGES) { stage = 0; phase ^= 1; }
        }
        d3b::mma_commit_pair(&bars.tfull[acc], 0x3);
      }
      d3b::mma_commit_pair(&bars.drain, 0x1);
      const uint32_t addr = d3b::smem_u32(&bars.drain);
      const uint64_t t0 = d3b::globaltimer_ns();
      while (!d3b::mbar_try_wait(addr, 0)) {
        if (d3b::globaltimer_ns() - t0 > D3B_WAIT_LIMIT_NS) {
          d3b::record_device_error(err, kSitePairDrain);
          break;
        }
      }
    }
  } else {
    // ---------------- epilogue (warps 2..5 of each CTA: its 128 rows) ----------------
    const int quarter = warp & 3;
    const int row_in_tile = quarter * 32 + lane;
    const bool is_int = MODE == D3B_MODE_INT8;
    int local = 0;
    for (int t = pair; t < num_tiles && !*abort_flag; t += pairs, ++local) {
      const int m0 = (t % num_m) * 2 * P_BM + (int)rank * P_BM, n0 = (t / num_m) * P_BN;
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!d3b::warp_wait(&bars.tfull[acc], acc_phase, abort_flag, err, kSitePairEpi)) break;
      d3b::tc_fence_after();
      const int row = m0 + row_in_tile;
      const float sa_row = (out_kind != D3B_I32 && row < M) ? __ldg(sa + row) : 0.f;
#pragma unroll 1
      for (int c = 0; c < P_BN / 32; ++c) {
        uint32_t r[32];
        d3b::tmem_ld32(tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * P_BN + c * 32, r);
        d3b::tmem_wait_ld();
        if (c == P_BN / 32 - 1) {
          d3b::tc_fence_before();
          d3b::mbar_arrive_cluster(d3b::cluster_addr(&bars.tempty[acc], 0));  // to rank 0
        }
        store_chunk(out, ldo, out_kind, row, M, n0 + c * 32, N, r, sa_row, sw, is_int);
      }
    }
  }

  __syncwarp();  // lanes that skipped a role loop rejoin before the aligned cluster barrier
  d3b::tc_fence_before();
  d3b::cluster_sync();  // rank 0's MMAs (which write both TMEMs) are drained before either CTA frees TMEM
  d3b::tc_fence_after();
  if (warp == 1) d3b::tmem_dealloc_pair(tmem_base, TMEM_COLS);
}

template <int MODE>
int launch_pair(const CUtensorMap& mA, const CUtensorMap& mB, const float* sa, const float* sw, void* y, int64_t ldy,
                int M, int N, int K, int out_kind, cudaStream_t stream) {
  static int attr_set[64] = {0};
  const int dev = d3b_host::current_device();
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    if (cudaFuncSetAttribute(w8a8_gemm_pair_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             P_SMEM_BYTES) != cudaSuccess)
      return D3B_ECUDA;
    attr_set[dev] = 1;
  }
  int* err = d3b_host::device_error_word();
  if (!err) return D3B_ECUDA;
  const int tiles = ((M + 2 * P_BM - 1) / (2 * P_BM)) * ((N + P_BN - 1) / P_BN);
  // Pairs that fit at once (SM pairs of a GPC with one free SM stay idle), queried once per device.
  static int max_pairs_of[64] = {0};
  int max_pairs = (dev >= 0 && dev < 64) ? max_pairs_of[dev] : 0;
  if (max_pairs <= 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * 256);
    cfg.blockDim = dim3(NUM_THREADS);
    cfg.dynamicSmemBytes = P_SMEM_BYTES;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, w8a8_gemm_pair_kernel<MODE>, &cfg) != cudaSuccess || clusters <= 0) {
      cudaGetLastError();
      clusters = d3b_host::num_sms(dev) / 2;
    }
    max_pairs = clusters;
    if (dev >= 0 && dev < 64) max_pairs_of[dev] = clusters;
  }
  const int pairs = tiles < max_pairs ? tiles : max_pairs;
  w8a8_gemm_pair_kernel<MODE><<<2 * pairs, NUM_THREADS, P_SMEM_BYTES, stream>>>(mA, mB, sa, sw, y, ldy, M, N, K,
                                                                               out_kind, err);
  return d3b_host::check_launch();
}

template <int MODE>
int launch(const CUtensorMap& mA, const CUtensorMap& mB, const float* sa, const float* sw, void* y, int64_t ldy,
           int M, int N, int K, int out_kind, cudaStream_t stream) {
  static int attr_set[64] = {0};
  const int dev = d3b_host::current_device();
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    if (cudaFuncSetAttribute(w8a8_gemm_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) !=
        cudaSuccess)
      return D3B_ECUDA;
    attr_set[dev] = 1;
  }
  int* err = d3b_host::device_error_word();
  if (!err) return D3B_ECUDA;
  const int tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  const int grid = tiles < d3b_host::num_sms(dev) ? tiles : d3b_host::num_sms(dev);
  w8a8_gemm_kernel<MODE><<<grid, NUM_THREADS, SMEM_BYTES, stream>>>(mA, mB, sa, sw, y, ldy, M, N, K, out_kind, err);
  return d3b_host::check_launch();
}

}  // namespace

extern "C" int d3b_w8a8_gemm(const void* qa, const void* qw, const float* sa, const float* sw, void* y, int64_t ldy,
                             int64_t M, int64_t N, int64_t K, int mode, int out_kind, d3b_stream_t stream) {
  if (M < 0 || N <= 0 || K <= 0 || M > 0x7FFFFFFF || N > 0x7FFFFFFF || K > 0x7FFFFFFF) return D3B_EINVAL;
  if (K % 16 != 0 || N % 16 != 0) return D3B_EINVAL;
  if (mode != D3B_MODE_FP8 && mode != D3B_MODE_INT8) return D3B_EINVAL;
  if (out_kind != D3B_BF16 && out_kind != D3B_F16 && out_kind != D3B_F32 && out_kind != D3B_I32)
    return D3B_EUNSUPPORTED;
  if (out_kind == D3B_I32 && mode != D3B_MODE_INT8) return D3B_EUNSUPPORTED;
  if (ldy < N) return D3B_EINVAL;
  if (M == 0) return D3B_OK;
  if (!qa || !qw || !y) return D3B_EINVAL;
  if (out_kind != D3B_I32 && (!sa || !sw)) return D3B_EINVAL;
  const int esize = (out_kind == D3B_BF16 || out_kind == D3B_F16) ? 2 : 4;
  if (reinterpret_cast<uintptr_t>(y) % 16 || (ldy * esize) % 16) return D3B_EALIGN;
  if (sw && reinterpret_cast<uintptr_t>(sw) % 16) return D3B_EALIGN;

  CUtensorMap mA, mB;
  const uint64_t dA[2] = {(uint64_t)K, (uint64_t)M}, dB[2] = {(uint64_t)K, (uint64_t)N};
  const uint64_t st[1] = {(uint64_t)K};
  const bool pair = M >= 512;  // CTA pairs: 256 x 256 tiles, each CTA loads 128 rows of B
  const uint32_t boxA[2] = {BK, BM}, boxB[2] = {BK, pair ? (uint32_t)(P_BN / 2) : (uint32_t)BN};
  int rc = d3b_host::encode_tiled(&mA, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, qa, dA, st, boxA,
                                  CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = d3b_host::encode_tiled(&mB, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, qw, dB, st, boxB, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (pair) {
    if (mode == D3B_MODE_FP8)
      return launch_pair<D3B_MODE_FP8>(mA, mB, sa, sw, y, ldy, (int)M, (int)N, (int)K, out_kind, s);
    return launch_pair<D3B_MODE_INT8>(mA, mB, sa, sw, y, ldy, (int)M, (int)N, (int)K, out_kind, s);
  }
  if (mode == D3B_MODE_FP8) return launch<D3B_MODE_FP8>(mA, mB, sa, sw, y, ldy, (int)M, (int)N, (int)K, out_kind, s);
  return launch<D3B_MODE_INT8>(mA, mB, sa, sw, y, ldy, (int)M, (int)N, (int)K, out_kind, s);
}
