// State snapshots: the multi-segment copy that packs one state pass's per-layer
// tensors into a single device block, and the host-side arena that places those
// blocks inside one caller-owned HBM buffer.
//
// The reference caches a snapshot as a list of tensors that may be views into
// much larger buffers (d3trt/model/core.py:321, `tail = mixed[:, :, -window:]`
// keeps the whole in_proj_qkv output alive). Packing copies exactly the bytes
// each tensor covers, so a cached state holds what its byte count says.
//
// Copy kernel: HBM-bound. A persistent grid walks 32 KiB tiles of all segments
// of one launch; each thread moves 4 accesses of the segment's widest aligned
// width (16 B in the common case) with all loads issued before the stores.
// The segment table is the kernel parameter (__grid_constant__), so a launch
// needs no device-side table and no host->device copy.
#include <algorithm>
#include <iterator>
#include <map>
#include <mutex>
#include <new>

#include "common.cuh"

namespace {

constexpr int kMaxSegs = 128;
constexpr int kTileShift = 15;  // 32 KiB of one segment per tile
constexpr int kThreads = 256;
constexpr int kUnroll = 8;  // contiguous runs: 16-byte accesses in flight per thread (128 KiB per SM)
constexpr int kUnrollStrided = 4;
constexpr uint64_t kMaxVecs = 1ull << 31;  // accesses per (split) segment

struct Seg {
  const unsigned char* src;
  unsigned char* dst;
  long long s_outer, s_row, d_outer, d_row;  // byte strides
  unsigned outer, rows, row_vecs, vshift;    // shape in accesses of (1 << vshift) bytes each
};

struct SegTable {
  Seg seg[kMaxSegs];
  unsigned prefix[kMaxSegs + 1];  // tiles before segment i; prefix[n] = tiles of the launch
  int n;
};

static_assert(sizeof(SegTable) < 32000, "segment table must fit the kernel parameter space");

template <typename V>
__device__ __forceinline__ void copy_flat(const Seg& s, unsigned vbeg, unsigned vend) {
  const V* src = reinterpret_cast<const V*>(s.src);
  V* dst = reinterpret_cast<V*>(s.dst);
#pragma unroll 1
  for (unsigned base = vbeg + threadIdx.x; base < vend; base += kUnroll * kThreads) {
    V v[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const unsigned i = base + u * kThreads;
      if (i < vend) v[u] = __ldcs(src + i);
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const unsigned i = base + u * kThreads;
      if (i < vend) dst[i] = v[u];
    }
  }
}

// Several rows per tile: each access index is split into (outer, row, column).
template <typename V>
__device__ __forceinline__ void copy_strided(const Seg& s, unsigned vbeg, unsigned vend) {
  constexpr int U = kUnrollStrided;
#pragma unroll 1
  for (unsigned base = vbeg + threadIdx.x; base < vend; base += U * kThreads) {
    V v[U];
    unsigned char* dst[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const unsigned i = base + u * kThreads;
      if (i < vend) {
        const unsigned q = i / s.row_vecs;
        const unsigned o = q / s.rows;
        const long long r = q - o * s.rows;
        const long long col = (long long)(i - q * s.row_vecs) * (long long)sizeof(V);
        v[u] = __ldcs(reinterpret_cast<const V*>(s.src + (long long)o * s.s_outer + r * s.s_row + col));
        dst[u] = s.dst + (long long)o * s.d_outer + r * s.d_row + col;
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (base + u * kThreads < vend) *reinterpret_cast<V*>(dst[u]) = v[u];
  }
}

// One instantiation per access width and per shape (one contiguous run, or rows)
// keeps each path's registers to itself.
template <typename V, bool kFlat>
__global__ void __launch_bounds__(kThreads, 4) copy_segments_kernel(const __grid_constant__ SegTable t) {
  const unsigned total = t.prefix[t.n];
#pragma unroll 1
  for (unsigned tile = blockIdx.x; tile < total; tile += gridDim.x) {
    int lo = 0, hi = t.n;  // largest lo with prefix[lo] <= tile
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (t.prefix[mid] <= tile) lo = mid; else hi = mid;
    }
    const Seg s = t.seg[lo];  // uniform per tile: one copy in registers
    constexpr unsigned per_tile = (1u << kTileShift) / sizeof(V);
    const unsigned nvec = s.outer * s.rows * s.row_vecs;
    const unsigned vbeg = (tile - t.prefix[lo]) * per_tile;
    const unsigned vend = min(vbeg + per_tile, nvec);
    if constexpr (kFlat)
      copy_flat<V>(s, vbeg, vend);
    else
      copy_strided<V>(s, vbeg, vend);
  }
}

// Widest access (log2 bytes, at most 16 B) dividing every address, row size and used stride.
int vec_shift(const d3b_copy_segment& g) {
  uint64_t bits = (uint64_t)(uintptr_t)g.src | (uint64_t)(uintptr_t)g.dst | (uint64_t)g.row_bytes;
  if (g.rows > 1) bits |= (uint64_t)g.src_row_stride | (uint64_t)g.dst_row_stride;
  if (g.outer > 1) bits |= (uint64_t)g.src_outer_stride | (uint64_t)g.dst_outer_stride;
  int sh = 4;
  while (sh > 0 && (bits & ((1ull << sh) - 1))) --sh;
  return sh;
}

struct Launcher {
  SegTable table[5][2];  // [log2(access bytes)][one contiguous run]
  cudaStream_t stream;
  int status = D3B_OK;

  explicit Launcher(cudaStream_t s) : stream(s) {
    for (auto& per_width : table)
      for (SegTable& t : per_width) {
        t.n = 0;
        t.prefix[0] = 0;
      }
  }

  template <typename V>
  void launch(const SegTable& t, bool flat, int grid) {
    if (flat)
      copy_segments_kernel<V, true><<<grid, kThreads, 0, stream>>>(t);
    else
      copy_segments_kernel<V, false><<<grid, kThreads, 0, stream>>>(t);
  }

  void flush(int sh, int flat) {
    SegTable& t = table[sh][flat];
    if (status != D3B_OK || t.n == 0) return;
    const unsigned tiles = t.prefix[t.n];
    const int grid = (int)std::min<unsigned>(tiles, (unsigned)d3b_host::num_sms(d3b_host::current_device()) * 4u);
    switch (sh) {
      case 4: launch<uint4>(t, flat, grid); break;
      case 3: launch<uint2>(t, flat, grid); break;
      case 2: launch<unsigned int>(t, flat, grid); break;
      case 1: launch<unsigned short>(t, flat, grid); break;
      default: launch<unsigned char>(t, flat, grid); break;
    }
    status = d3b_host::check_launch();
    t.n = 0;
  }

  void flush_all() {
    for (int sh = 4; sh >= 0; --sh)
      for (int flat = 1; flat >= 0; --flat) flush(sh, flat);
  }

  // Append one piece of at most kMaxVecs accesses.
  void add(const unsigned char* src, unsigned char* dst, long long s_outer, long long s_row, long long d_outer,
           long long d_row, uint64_t outer, uint64_t rows, uint64_t row_vecs, int sh) {
    const int flat = (outer == 1 && rows == 1) ? 1 : 0;
    SegTable& t = table[sh][flat];
    if (t.n == kMaxSegs) flush(sh, flat);
    if (status != D3B_OK) return;
    Seg& s = t.seg[t.n];
    s.src = src;
    s.dst = dst;
    s.s_outer = s_outer;
    s.s_row = s_row;
    s.d_outer = d_outer;
    s.d_row = d_row;
    s.outer = (unsigned)outer;
    s.rows = (unsigned)rows;
    s.row_vecs = (unsigned)row_vecs;
    s.vshift = (unsigned)sh;
    const uint64_t tiles = (outer * rows * row_vecs + (1ull << (kTileShift - sh)) - 1) >> (kTileShift - sh);
    t.prefix[t.n + 1] = t.prefix[t.n] + (unsigned)tiles;
    ++t.n;
    // keep the launch's tile count well inside 32 bits
    if (t.prefix[t.n] > (1u << 30)) flush(sh, flat);
  }

  // Split a validated segment into pieces of at most kMaxVecs accesses.
  int segment(const d3b_copy_segment& g) {
    const int sh = vec_shift(g);
    const uint64_t row_vecs = (uint64_t)g.row_bytes >> sh;
    const uint64_t outer = (uint64_t)g.outer, rows = (uint64_t)g.rows;
    const unsigned char* src = static_cast<const unsigned char*>(g.src);
    unsigned char* dst = static_cast<unsigned char*>(g.dst);
    if (outer == 1 && rows == 1) {  // one contiguous run
      for (uint64_t v = 0; v < row_vecs; v += kMaxVecs) {
        const uint64_t n = std::min<uint64_t>(kMaxVecs, row_vecs - v);
        add(src + (v << sh), dst + (v << sh), 0, 0, 0, 0, 1, 1, n, sh);
      }
      return status;
    }
    if (row_vecs >= kMaxVecs) return D3B_EINVAL;  // rows of 32 GiB and more are not split
    if (rows * row_vecs >= kMaxVecs) {            // split every outer index into row chunks
      const uint64_t per = kMaxVecs / row_vecs;
      for (uint64_t o = 0; o < outer; ++o)
        for (uint64_t r = 0; r < rows; r += per)
          add(src + (long long)o * g.src_outer_stride + (long long)r * g.src_row_stride,
              dst + (long long)o * g.dst_outer_stride + (long long)r * g.dst_row_stride, 0, g.src_row_stride, 0,
              g.dst_row_stride, 1, std::min(per, rows - r), row_vecs, sh);
      return status;
    }
    const uint64_t per = kMaxVecs / (rows * row_vecs);
    for (uint64_t o = 0; o < outer; o += per)
      add(src + (long long)o * g.src_outer_stride, dst + (long long)o * g.dst_outer_stride, g.src_outer_stride,
          g.src_row_stride, g.dst_outer_stride, g.dst_row_stride, std::min(per, outer - o), rows, row_vecs, sh);
    return status;
  }
};

struct Arena {
  std::mutex mu;
  uint64_t capacity = 0, align = 256, live_bytes = 0;
  std::map<uint64_t, uint64_t> holes;  // offset -> size of each free range
  std::map<uint64_t, uint64_t> live;   // offset -> size of each live block
};

}  // namespace

extern "C" {

int d3b_copy_segments(const d3b_copy_segment* segments, int n, d3b_stream_t stream) {
  if (n < 0 || (n > 0 && !segments)) return D3B_EINVAL;
  for (int i = 0; i < n; ++i) {
    const d3b_copy_segment& g = segments[i];
    if (g.outer < 0 || g.rows < 0 || g.row_bytes < 0) return D3B_EINVAL;
    if (g.outer == 0 || g.rows == 0 || g.row_bytes == 0) continue;
    if (!g.src || !g.dst) return D3B_EINVAL;
    if (g.outer >= (1ll << 31) || g.rows >= (1ll << 31)) return D3B_EINVAL;
  }
  Launcher* l = new (std::nothrow) Launcher(reinterpret_cast<cudaStream_t>(stream));
  if (!l) return D3B_ENOSPACE;
  int st = D3B_OK;
  for (int i = 0; i < n && st == D3B_OK; ++i) {
    const d3b_copy_segment& g = segments[i];
    if (g.outer == 0 || g.rows == 0 || g.row_bytes == 0) continue;
    st = l->segment(g);
  }
  if (st == D3B_OK) {
    l->flush_all();
    st = l->status;
  }
  delete l;
  return st;
}

int d3b_arena_create(uint64_t capacity, uint64_t alignment, void** arena) {
  if (!arena || alignment < 16 || alignment > (1ull << 30) || (alignment & (alignment - 1))) return D3B_EINVAL;
  Arena* a = new (std::nothrow) Arena();
  if (!a) return D3B_ENOSPACE;
  a->capacity = capacity;
  a->align = alignment;
  if (capacity >= alignment) a->holes[0] = capacity & ~(alignment - 1);
  *arena = a;
  return D3B_OK;
}

int d3b_arena_alloc(void* arena, uint64_t bytes, uint64_t* offset) {
  Arena* a = static_cast<Arena*>(arena);
  if (!a || !offset || bytes == 0 || bytes > (1ull << 62)) return D3B_EINVAL;
  const uint64_t need = (bytes + a->align - 1) & ~(a->align - 1);
  std::lock_guard<std::mutex> lock(a->mu);
  auto best = a->holes.end();
  for (auto it = a->holes.begin(); it != a->holes.end(); ++it)
    if (it->second >= need && (best == a->holes.end() || it->second < best->second)) best = it;
  if (best == a->holes.end()) return D3B_ENOSPACE;
  const uint64_t off = best->first, size = best->second;
  a->holes.erase(best);
  if (size > need) a->holes[off + need] = size - need;
  a->live[off] = need;
  a->live_bytes += need;
  *offset = off;
  return D3B_OK;
}

int d3b_arena_free(void* arena, uint64_t offset) {
  Arena* a = static_cast<Arena*>(arena);
  if (!a) return D3B_EINVAL;
  std::lock_guard<std::mutex> lock(a->mu);
  auto it = a->live.find(offset);
  if (it == a->live.end()) return D3B_EINVAL;
  uint64_t off = it->first, size = it->second;
  a->live.erase(it);
  a->live_bytes -= size;
  auto next = a->holes.lower_bound(off);
  if (next != a->holes.end() && next->first == off + size) {
    size += next->second;
    next = a->holes.erase(next);
  }
  if (next != a->holes.begin()) {
    auto prev = std::prev(next);
    if (prev->first + prev->second == off) {
      prev->second += size;
      return D3B_OK;
    }
  }
  a->holes[off] = size;
  return D3B_OK;
}

int d3b_arena_stats(void* arena, uint64_t* stats) {
  Arena* a = static_cast<Arena*>(arena);
  if (!a || !stats) return D3B_EINVAL;
  std::lock_guard<std::mutex> lock(a->mu);
  uint64_t free_bytes = 0, largest = 0;
  for (const auto& h : a->holes) {
    free_bytes += h.second;
    largest = std::max(largest, h.second);
  }
  stats[0] = a->live_bytes;
  stats[1] = free_bytes;
  stats[2] = largest;
  stats[3] = a->live.size();
  return D3B_OK;
}

void d3b_arena_destroy(void* arena) { delete static_cast<Arena*>(arena); }

}  // extern "C"
