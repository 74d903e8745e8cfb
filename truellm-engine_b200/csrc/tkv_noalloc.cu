// tkv_noalloc.cu -- decode attention for callers that cannot allocate device
// memory.
//
// tkv_paged_decode needs a caller-provided workspace (the split-KV partials
// and their completion counters).  Some callers have no way to
// provide one: a kernel plugin handed only the engine's tensors, a host whose
// allocator owns all device memory and forbids side allocations, or a decode
// loop that must not call cudaMalloc (it can synchronise the device) in the
// per-token path.  tkv_paged_decode_noalloc runs the same kernel with the
// workspace taken from a fixed static device array instead.
//
// The array below lives in every GPU that loads this library, for the life of
// the process.  Host code never dereferences its name: on the host the symbol
// is only a stand-in, so every call looks up its device address with
// cudaGetSymbolAddress, for the device that is current (a cheap host-side
// lookup, correct also after cudaDeviceReset gives the device a new context).
#include "tkv_common.cuh"

namespace {

constexpr size_t kScratchBytes = TKV_NOALLOC_SCRATCH_BYTES;

static __device__ __align__(256) unsigned char g_decode_scratch[kScratchBytes];

// Bytes at the start of the decode workspace that must be zero when a call
// begins: the per-(sequence, kv head) completion counters (256 bytes of
// reserved space, then num_seqs * num_q_heads counters rounded up to 256).
size_t counter_bytes(int num_seqs, int num_q_heads) {
  return 256 + ((size_t)num_seqs * (size_t)num_q_heads * 4 + 255) / 256 * 256;
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
  if (cudaGetSymbolAddress(&scratch, g_decode_scratch) != cudaSuccess || scratch == nullptr)
    return TKV_BACKEND_ERROR;
  // Every call shares the array: clear its counters (stream-ordered) so the
  // call does not depend on what an earlier call left there.
  if (cudaMemsetAsync(scratch, 0, counter_bytes(num_seqs, num_q_heads),
                      static_cast<cudaStream_t>(stream)) != cudaSuccess)
    return TKV_BACKEND_ERROR;
  return tkv_paged_decode(cache, q, q_dtype, out, out_dtype, block_tables, max_blocks_per_seq,
                          seq_lens, seq_slots, num_seqs, num_q_heads, scale, max_context_len,
                          scratch, kScratchBytes, err_flag, stream);
}

}  // extern "C"
