// 255-way fp32 readout softmax at the selected positions
// (d3trt/model/trtllm_stack.py:451-468, = hf_stack.py:67-84):
//   logits = f32(hidden) @ R^T ; logits[b, j >= counts[b]] = -inf ;
//   probs  = softmax(logits / T)
//
// One launch. The grid is (row groups of 8) x (option groups of 32). A CTA
// stages K-chunks of its 8 hidden rows in shared memory (as fp32), each warp
// computes 4 options x 8 rows of dot products with fp32 FMAs (the reference
// computes in fp32, so no tensor-core rounding is introduced), and writes its
// logits to the workspace. The last CTA of a row group to finish (an atomic
// ticket per row group) runs the masked softmax with one warp per row and
// resets the ticket to zero, so the workspace is ready for the next call.
#include "common.cuh"

namespace {

constexpr int kRows = 8;        // hidden rows per CTA (= warps per CTA)
constexpr int kOpts = 32;       // options per CTA
constexpr int kOptsPerWarp = kOpts / kRows;
constexpr int kChunk = 512;     // K elements staged per step
constexpr int kMaxOpts = 1024;  // softmax keeps n_opt/32 logits per lane

__device__ __forceinline__ float load_h(const float* p) { return __ldg(p); }
__device__ __forceinline__ float load_h(const __nv_bfloat16* p) { return __bfloat162float(*p); }
__device__ __forceinline__ float load_h(const __half* p) { return __half2float(*p); }

template <typename T>
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

  for (int kc = 0; kc < K; kc += kChunk) {
    const int kn = min(kChunk, K - kc);
    __syncthreads();
    for (int i = threadIdx.x; i < kRows * kChunk; i += blockDim.x) {
      const int r = i / kChunk, k = i % kChunk;
      const int row = r0 + r;
      hs[r][k] = (row < B && k < kn) ? load_h(hidden + (int64_t)row * K + kc + k) : 0.f;
    }
    __syncthreads();
    for (int k = lane; k < kn; k += 32) {
      float h[kRows];
#pragma unroll
      for (int r = 0; r < kRows; ++r) h[r] = hs[r][k];
#pragma unroll
      for (int o = 0; o < kOptsPerWarp; ++o) {
        const int opt = o0 + o;
        const float w = opt < n_opt ? __ldg(R + (int64_t)opt * K + kc + k) : 0.f;
#pragma unroll
        for (int r = 0; r < kRows; ++r) acc[o][r] = fmaf(h[r], w, acc[o][r]);
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

  const int row = r0 + warp;
  if (row < B) {
    constexpr int kPer = kMaxOpts / 32;
    const int cnt = counts[row];
    float v[kPer];
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int j = lane + 32 * i;
      float x = -INFINITY;
      if (j < n_opt && j < cnt) x = __ldcg(logits_ws + (int64_t)row * n_opt + j) / temperature;
      v[i] = x;
      mx = fmaxf(mx, x);
    }
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, s));
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const float e = (v[i] == -INFINITY) ? 0.f : expf(v[i] - mx);
      v[i] = e;
      sum += e;
    }
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, s);
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int j = lane + 32 * i;
      // A row with count <= 0 is all -inf in the reference; softmax gives NaN.
      if (j < n_opt) probs[(int64_t)row * n_opt + j] = (cnt > 0) ? v[i] / sum : __int_as_float(0x7fc00000);
    }
  }
  if (threadIdx.x == 0) tickets[blockIdx.x] = 0u;
}

size_t ws_layout(int B, int n_opt, size_t* tickets_off) {
  const size_t logits = ((size_t)B * n_opt * sizeof(float) + 255) & ~(size_t)255;
  const size_t groups = (size_t)(B + kRows - 1) / kRows;
  *tickets_off = logits;
  return logits + ((groups * sizeof(unsigned int) + 255) & ~(size_t)255);
}

}  // namespace

extern "C" size_t d3b_readout_workspace_size(int B, int n_opt) {
  if (B <= 0 || n_opt <= 0) return 0;
  size_t off;
  return ws_layout(B, n_opt, &off);
}

extern "C" int d3b_readout(const void* hidden, int h_dtype, const float* readout, const int32_t* counts,
                           float temperature, float* probs, int B, int K, int n_opt, void* workspace,
                           size_t workspace_bytes, d3b_stream_t stream) {
  if (B < 0 || K <= 0 || n_opt <= 0 || n_opt > kMaxOpts) return D3B_EINVAL;
  if (!(temperature > 0.f)) return D3B_EINVAL;
  if (B == 0) return D3B_OK;
  if (!hidden || !readout || !counts || !probs || !workspace) return D3B_EINVAL;
  size_t tickets_off;
  const size_t need = ws_layout(B, n_opt, &tickets_off);
  if (workspace_bytes < need) return D3B_ENOSPACE;
  float* logits = static_cast<float*>(workspace);
  unsigned int* tickets = reinterpret_cast<unsigned int*>(static_cast<char*>(workspace) + tickets_off);
  dim3 grid((B + kRows - 1) / kRows, (n_opt + kOpts - 1) / kOpts), block(kRows * 32);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (h_dtype) {
    case D3B_F32:
      readout_kernel<float><<<grid, block, 0, s>>>(static_cast<const float*>(hidden), readout, counts, temperature,
                                                   probs, B, K, n_opt, logits, tickets);
      break;
    case D3B_F16:
      readout_kernel<__half><<<grid, block, 0, s>>>(static_cast<const __half*>(hidden), readout, counts,
                                                    temperature, probs, B, K, n_opt, logits, tickets);
      break;
    case D3B_BF16:
      readout_kernel<__nv_bfloat16><<<grid, block, 0, s>>>(static_cast<const __nv_bfloat16*>(hidden), readout,
                                                           counts, temperature, probs, B, K, n_opt, logits, tickets);
      break;
    default: return D3B_EUNSUPPORTED;
  }
  return d3b_host::check_launch();
}
