// tkv_noalloc.cu -- decode attention for callers that cannot allocate device
// memory.
//
// tkv_paged_decode needs a caller-provided workspace (the split-KV partials
// and the persistent kernel's work counters).  Some callers have no way to
// provide one: a kernel plugin handed only the engine's tensors, a host whose
// allocator owns all device memory and forbids side allocations, or a decode
// loop that must not call cudaMalloc (it can synchronise the device) in the
// per-token path.  tkv_paged_decode_noalloc runs the same kernel with the
// workspace taken from a fixed static device array instead.
//
// The array below lives in every GPU that loads this library, for the life of
// the process.  Host code never dereferences its name: on the host the symbol
// is only a stand-in, so its device address is fetched with
// cudaGetSymbolAddress once per device, with that device current, on the
// first call made on it.
#include <mutex>

#include "tkv_common.cuh"

namespace {

constexpr size_t kScratchBytes = TKV_NOALLOC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_decode_scratch[kScratchBytes];

std::mutex g_setup_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Per-device set-up: device address of the scratch array, zeroed once (its
// work and completion counters must start at zero; the decode kernel leaves
// them zero after every call).
int scratch_for_current_device(void** ptr, cudaStream_t stream) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return TKV_BACKEND_ERROR;
  std::lock_guard<std::mutex> lock(g_setup_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_decode_scratch) != cudaSuccess || p == nullptr)
      return TKV_BACKEND_ERROR;
    if (cudaMemsetAsync(p, 0, kScratchBytes, stream) != cudaSuccess) return TKV_BACKEND_ERROR;
    g_scratch_ptr[dev] = p;
  }
  *ptr = g_scratch_ptr[dev];
  return TKV_OK;
}

}  // namespace

extern "C" {

int tkv_paged_decode_noalloc(const tkv_cache_t* cache, const void* q, int q_dtype, void* out,
                             int out_dtype, const int32_t* block_tables, int max_blocks_per_seq,
                             const int32_t* seq_lens, const int32_t* seq_slots, int num_seqs,
                             int num_q_heads, float scale, int max_context_len, int* err_flag,
                             void* stream) {
  if (!cache || num_seqs <= 0 || num_q_heads <= 0 || max_context_len < 0)
    return TKV_INVALID_ARGUMENT;
  const size_t need =
      tkv_decode_workspace_bytes(num_seqs, num_q_heads, cache->fmt.head_dim, max_context_len);
  if (need == 0) return TKV_INVALID_ARGUMENT;
  if (need > kScratchBytes) return TKV_OUT_OF_MEMORY;  // larger than the static scratch
  void* scratch = nullptr;
  const int st = scratch_for_current_device(&scratch, static_cast<cudaStream_t>(stream));
  if (st != TKV_OK) return st;
  return tkv_paged_decode(cache, q, q_dtype, out, out_dtype, block_tables, max_blocks_per_seq,
                          seq_lens, seq_slots, num_seqs, num_q_heads, scale, max_context_len,
                          scratch, kScratchBytes, err_flag, stream);
}

}  // extern "C"
