// Library-wide C ABI pieces: status strings, the device error word, TMA
// descriptor encoding through the driver entry point, and the wait-limit
// self-test kernel.
#include <mutex>

#include "common.cuh"

// One error word per device; kernels receive its device address as an argument.
__device__ int g_d3b_device_error = 0;

namespace d3b_host {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult qres;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &qres) == cudaSuccess &&
        qres == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

int encode_tiled(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base, const uint64_t* dims,
                 const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = get_encode_fn();
  if (!fn) return D3B_ECUDA;
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0) return D3B_EALIGN;
  cuuint64_t d[5];
  cuuint64_t s[4];
  cuuint32_t b[5];
  cuuint32_t e[5];
  for (int i = 0; i < rank; ++i) {
    if (dims[i] == 0 || dims[i] > (1ull << 32)) return D3B_EINVAL;
    if (box[i] == 0 || box[i] > 256) return D3B_EINVAL;
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
  }
  for (int i = 0; i < rank - 1; ++i) {
    if (strides_bytes[i] % 16 != 0 || strides_bytes[i] >= (1ull << 40)) return D3B_EALIGN;
    s[i] = strides_bytes[i];
  }
  CUresult r = fn(map, dtype, (cuuint32_t)rank, const_cast<void*>(base), d, s, b, e, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? D3B_OK : D3B_EINVAL;
}

int current_device() {
  int dev = 0;
  cudaGetDevice(&dev);
  return dev;
}

int num_sms(int device) {
  static int cache[64] = {0};
  if (device >= 0 && device < 64 && cache[device]) return cache[device];
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || n <= 0) n = 148;
  if (device >= 0 && device < 64) cache[device] = n;
  return n;
}

int* device_error_word() {
  static int* cache[64] = {nullptr};
  static std::mutex mu;
  const int dev = current_device();
  std::lock_guard<std::mutex> lock(mu);
  if (dev >= 0 && dev < 64 && cache[dev]) return cache[dev];
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_d3b_device_error) != cudaSuccess) return nullptr;
  if (dev >= 0 && dev < 64) cache[dev] = static_cast<int*>(p);
  return static_cast<int*>(p);
}

int check_launch() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? D3B_OK : D3B_ECUDA;
}

}  // namespace d3b_host

// ---------------------------------------------------------------------------
// wait-limit self-test: one warp waits on an mbarrier that never completes
// ---------------------------------------------------------------------------
__global__ void d3b_selftest_wait_kernel(uint64_t limit_ns, int* err) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    d3b::mbar_init(&bar, 1);
    d3b::fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t addr = d3b::smem_u32(&bar);
    const uint64_t t0 = d3b::globaltimer_ns();
    // Phase 0 never completes: nothing arrives on the barrier.
    while (!d3b::mbar_try_wait(addr, 0)) {
      if (d3b::globaltimer_ns() - t0 > limit_ns) {
        d3b::record_device_error(err, 9001);
        break;
      }
    }
  }
  __syncthreads();
}

extern "C" {

int d3b_version(void) { return 100; }

const char* d3b_error_string(int status) {
  switch (status) {
    case D3B_OK: return "ok";
    case D3B_EINVAL: return "invalid argument (shape, size or value)";
    case D3B_EALIGN: return "pointer or stride is not aligned as the kernel requires (16 bytes)";
    case D3B_EUNSUPPORTED: return "unsupported dtype, head_dim or group size";
    case D3B_ECUDA: return "a CUDA runtime/driver call failed";
    case D3B_ETIMEOUT: return "a device-side wait ran past its wall-clock limit";
    case D3B_ENOSPACE: return "workspace or fixed scratch too small for this request";
    default: return "unknown status";
  }
}

int d3b_device_error(d3b_stream_t stream, int reset) {
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (cudaStreamSynchronize(s) != cudaSuccess) return D3B_ECUDA;
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_d3b_device_error, sizeof(int)) != cudaSuccess) return D3B_ECUDA;
  if (reset && v) {
    int zero = 0;
    if (cudaMemcpyToSymbol(g_d3b_device_error, &zero, sizeof(int)) != cudaSuccess) return D3B_ECUDA;
  }
  return v;
}

int d3b_selftest_wait_timeout(int limit_ms, d3b_stream_t stream) {
  if (limit_ms <= 0 || limit_ms > 5000) return D3B_EINVAL;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int* err = d3b_host::device_error_word();
  if (!err) return D3B_ECUDA;
  d3b_selftest_wait_kernel<<<1, 32, 0, s>>>((uint64_t)limit_ms * 1000000ull, err);
  return d3b_host::check_launch();
}

}  // extern "C"
