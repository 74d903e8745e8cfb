// tkv_blockops.cu -- page and ring-row moves of the paged KIVI cache
// (tkv_copy_pages, tkv_swap_pages, tkv_copy_ring_rows, tkv_swap_ring_rows).
//
// The reference moves fp16 blocks with one element (copy_blocks_kernel) or
// one byte (swap_blocks_kernel) per thread, third_party/vllm_kernels/
// cache_kernels.cu:107-168.  Here every move is one kernel over "segments":
// a page (all kv heads of one page id are contiguous in the pool,
// n_kv_heads * page_bytes bytes) or a ring row (n_kv_heads * ring_cap * D * 4
// bytes), both multiples of 16 bytes.  Work units are (pair, 16 KB chunk);
// each thread keeps four 16-byte loads in flight before storing, which is
// what a copy over PCIe (pinned host images, reached through their mapped
// device address) needs to cover its latency.  HBM-bound on the device, PCIe
// bound to and from the host.
#include <string.h>

#include <algorithm>

#include "tkv_common.cuh"

namespace {

constexpr int kThreads = 256;
constexpr int kVecPerThread = 4;
constexpr int kChunkVecs = kThreads * kVecPerThread;  // 16 KB per work unit

__global__ void __launch_bounds__(kThreads) move_segments_kernel(
    const uint4* __restrict__ src, int64_t src_count, uint4* __restrict__ dst, int64_t dst_count,
    const int32_t* __restrict__ mapping, int n, int64_t seg_vecs, int64_t chunks, int err_bit,
    int* err) {
  const int64_t units = (int64_t)n * chunks;
  for (int64_t u = blockIdx.x; u < units; u += gridDim.x) {
    const int i = (int)(u / chunks);
    const int64_t c = u - (int64_t)i * chunks;
    const int32_t s = mapping[2 * i], d = mapping[2 * i + 1];
    if (s < 0 || s >= src_count || d < 0 || d >= dst_count) {
      if (c == 0 && threadIdx.x == 0) tkv::set_err(err, err_bit);
      continue;
    }
    const uint4* sp = src + (int64_t)s * seg_vecs;
    uint4* dp = dst + (int64_t)d * seg_vecs;
    const int64_t v0 = c * kChunkVecs + threadIdx.x;
    uint4 r[kVecPerThread];
#pragma unroll
    for (int k = 0; k < kVecPerThread; ++k) {
      const int64_t v = v0 + k * kThreads;
      if (v < seg_vecs) r[k] = sp[v];
    }
#pragma unroll
    for (int k = 0; k < kVecPerThread; ++k) {
      const int64_t v = v0 + k * kThreads;
      if (v < seg_vecs) dp[v] = r[k];
    }
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

bool cache_ok(const tkv_cache_t* c) {
  if (!c || !c->pool || !c->ring || c->num_pages <= 0 || c->max_seqs <= 0) return false;
  tkv_format_t chk;
  const tkv_format_t& f = c->fmt;
  if (tkv_format_init(&chk, f.head_dim, f.group_size, f.residual, f.bits, f.n_kv_heads) != TKV_OK)
    return false;
  return memcmp(&chk, &f, sizeof(chk)) == 0 && aligned16(c->pool) && aligned16(c->ring);
}

int64_t page_seg_bytes(const tkv_format_t& f) { return (int64_t)f.n_kv_heads * f.page_bytes; }
int64_t row_seg_bytes(const tkv_format_t& f) { return tkv_ring_bytes(&f, 1); }

// The device address of a caller's image buffer: device or managed memory as
// is, page-locked host memory through its mapped address; pageable host
// memory (which a kernel cannot reach) is rejected.
int device_view(void* p, void** out) {
  cudaPointerAttributes at;
  if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
    (void)cudaGetLastError();
    return TKV_INVALID_ARGUMENT;
  }
  switch (at.type) {
    case cudaMemoryTypeDevice:
    case cudaMemoryTypeManaged: *out = p; return TKV_OK;
    case cudaMemoryTypeHost:
      if (!at.devicePointer) return TKV_INVALID_ARGUMENT;
      *out = at.devicePointer;
      return TKV_OK;
    default: return TKV_INVALID_ARGUMENT;
  }
}

int launch_moves(const void* src, int64_t src_count, void* dst, int64_t dst_count,
                 const int32_t* mapping, int n, int64_t seg_bytes, int err_bit, int* err,
                 cudaStream_t stream) {
  // the mapping may also sit in page-locked host memory; pageable memory is rejected
  void* map = nullptr;
  if (int st = device_view(const_cast<int32_t*>(mapping), &map)) return st;
  const int64_t seg_vecs = seg_bytes / 16;
  const int64_t chunks = (seg_vecs + kChunkVecs - 1) / kChunkVecs;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return TKV_BACKEND_ERROR;
  const int64_t units = (int64_t)n * chunks;
  const int grid = (int)std::min<int64_t>(units, (int64_t)sms * 8);
  move_segments_kernel<<<grid, kThreads, 0, stream>>>(
      static_cast<const uint4*>(src), src_count, static_cast<uint4*>(dst), dst_count,
      static_cast<const int32_t*>(map), n, seg_vecs, chunks, err_bit, err);
  return cudaGetLastError() == cudaSuccess ? TKV_OK : TKV_BACKEND_ERROR;
}

int check_common(const tkv_cache_t* cache, const int32_t* mapping, int n) {
  if (!cache_ok(cache) || n < 0) return TKV_INVALID_ARGUMENT;
  if (n > 0 && !mapping) return TKV_INVALID_ARGUMENT;
  return TKV_OK;
}

int swap(void* base, int64_t base_count, void* images, int64_t capacity, const int32_t* mapping,
         int n, int direction, int64_t seg, int bit, int* err, cudaStream_t stream) {
  if (!images || capacity <= 0 || (direction != 0 && direction != 1)) return TKV_INVALID_ARGUMENT;
  if (n == 0) return TKV_OK;
  void* img = nullptr;
  if (int st = device_view(images, &img)) return st;
  if (!aligned16(img)) return TKV_INVALID_ARGUMENT;
  if (direction == 0)
    return launch_moves(base, base_count, img, capacity, mapping, n, seg, bit, err, stream);
  return launch_moves(img, capacity, base, base_count, mapping, n, seg, bit, err, stream);
}

}  // namespace

extern "C" {

int tkv_copy_pages(const tkv_cache_t* cache, const int32_t* mapping, int n, int* err_flag,
                   void* stream) {
  if (int st = check_common(cache, mapping, n)) return st;
  if (n == 0) return TKV_OK;
  return launch_moves(cache->pool, cache->num_pages, cache->pool, cache->num_pages, mapping, n,
                      page_seg_bytes(cache->fmt), TKV_ERR_BAD_PAGE, err_flag,
                      static_cast<cudaStream_t>(stream));
}

int tkv_swap_pages(const tkv_cache_t* cache, void* images, int64_t capacity,
                   const int32_t* mapping, int n, int direction, int* err_flag, void* stream) {
  if (int st = check_common(cache, mapping, n)) return st;
  return swap(cache->pool, cache->num_pages, images, capacity, mapping, n, direction,
              page_seg_bytes(cache->fmt), TKV_ERR_BAD_PAGE, err_flag,
              static_cast<cudaStream_t>(stream));
}

int tkv_copy_ring_rows(const tkv_cache_t* cache, const int32_t* mapping, int n, int* err_flag,
                       void* stream) {
  if (int st = check_common(cache, mapping, n)) return st;
  if (n == 0) return TKV_OK;
  return launch_moves(cache->ring, cache->max_seqs, cache->ring, cache->max_seqs, mapping, n,
                      row_seg_bytes(cache->fmt), TKV_ERR_BAD_SLOT, err_flag,
                      static_cast<cudaStream_t>(stream));
}

int tkv_swap_ring_rows(const tkv_cache_t* cache, void* images, int64_t capacity,
                       const int32_t* mapping, int n, int direction, int* err_flag,
                       void* stream) {
  if (int st = check_common(cache, mapping, n)) return st;
  return swap(cache->ring, cache->max_seqs, images, capacity, mapping, n, direction,
              row_seg_bytes(cache->fmt), TKV_ERR_BAD_SLOT, err_flag,
              static_cast<cudaStream_t>(stream));
}

}  // extern "C"
