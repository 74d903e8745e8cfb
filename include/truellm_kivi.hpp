// truellm_kivi.hpp -- C++ drop-in adapter over the truellm_kivi C ABI.
//
// Header-only; link libtruellm_kivi.so.  It keeps the reference's C++ entry
// points for the KIVI path with the reference's error behaviour, so an engine
// built against truellm's own headers can switch by changing one include and
// one namespace:
//
//   * kivi_params_supported / kivi_compressed_bytes / kivi_compress /
//     kivi_decompress  (kivi_cache.cuh:32-84): unsupported parameters or
//     n_vecs <= 0 are a silent no-op, as in kivi_cache.cu:219-220.  A status
//     the reference has no equivalent for (odd group_size, CUDA launch
//     failure) throws std::runtime_error instead of computing garbage.
//   * KvCompressionPass  (kv_compression_pass.h:38-58): same constructor,
//     init / run / enabled.  The KIVI half maps the config exactly as
//     kv_compression_pass.cpp:29-67 does (n_outliers = residual_length,
//     group = bits == 4 ? 16 : 8) and is disabled, not thrown, when those
//     parameters are unsupported.  run() rounds K and V through the reference
//     format in place with one launch each and no scratch, so the
//     reference's 16-token prefill limit does not apply.  The VQ half of the
//     reference pass is not part of this library: enabled() reports KIVI only.
//     CUDA failures throw std::runtime_error (kv_compression_pass.cpp:16-24).
//   * KiviPageAllocator -- CudaAllocator's page bookkeeping for the KIVI
//     cache (bool / -1 returns as in cuda_allocator.cpp), plus copy_pages /
//     swap_pages / copy_ring_rows / swap_ring_rows (copy_blocks / swap_blocks).
//   * PagedKiviCache -- the new paged KIVI cache (a view over caller-owned
//     buffers, like the reference's TrueBuffer): append (the reshape_and_cache
//     slot) and decode (the paged_attention_v1/v2 slot), throwing
//     std::invalid_argument / std::runtime_error on a non-OK status.
#pragma once

#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>

#include <cuda_fp16.h>
#include <cuda_runtime_api.h>

#include "truellm_kivi.h"

namespace truellm {
namespace kivi_b200 {

inline void throw_on(int status, const char* what) {
  if (status == TKV_OK) return;
  const std::string msg = std::string(what) + ": " + tkv_status_string(status);
  if (status == TKV_INVALID_ARGUMENT) throw std::invalid_argument(msg);
  throw std::runtime_error(msg);
}

// ---------------------------------------------------------------- reference format
inline bool kivi_params_supported(int head_dim, int n_outliers, int group_size) {
  return tkv_kivi_params_supported(head_dim, n_outliers, group_size) != 0;
}

inline size_t kivi_compressed_bytes(int head_dim, int n_outliers, int group_size) {
  return tkv_kivi_compressed_bytes(head_dim, n_outliers, group_size);
}

inline void kivi_compress(const __half* d_kv_in, uint8_t* d_out, int n_vecs, int head_dim,
                          int n_outliers, int group_size, cudaStream_t stream) {
  if (n_vecs <= 0 || !kivi_params_supported(head_dim, n_outliers, group_size)) return;
  throw_on(tkv_kivi_compress(d_kv_in, d_out, n_vecs, head_dim, n_outliers, group_size, stream),
           "kivi_compress");
}

inline void kivi_decompress(const uint8_t* d_in, __half* d_kv_out, int n_vecs, int head_dim,
                            int n_outliers, int group_size, cudaStream_t stream) {
  if (n_vecs <= 0 || !kivi_params_supported(head_dim, n_outliers, group_size)) return;
  throw_on(tkv_kivi_decompress(d_in, d_kv_out, n_vecs, head_dim, n_outliers, group_size,
                               stream),
           "kivi_decompress");
}

// ---------------------------------------------------------------- compression pass
class KvCompressionPass {
 public:
  // Config: truellm::CompressionConfig (config_schema.h:144-159) or any type
  // with kv_kivi.{enabled, bits, residual_length}.
  template <class Config>
  KvCompressionPass(const Config& cfg, int n_layers, int n_kv_heads, int head_dim,
                    int block_size)
      : kivi_enabled_(cfg.kv_kivi.enabled),
        n_layers_(n_layers),
        n_kv_heads_(n_kv_heads),
        head_dim_(head_dim),
        block_size_(block_size),
        n_outliers_(cfg.kv_kivi.residual_length),
        group_size_(cfg.kv_kivi.bits == 4 ? 16 : 8) {
    if (kivi_enabled_ && !kivi_params_supported(head_dim_, n_outliers_, group_size_))
      kivi_enabled_ = false;
  }

  // No scratch to allocate: kept for call-site compatibility.
  template <class Allocator>
  void init(Allocator* /*allocator*/, cudaStream_t /*stream*/) {}

  void run(int /*layer_idx*/, int seq_len, void* k_ptr, void* v_ptr, cudaStream_t stream) {
    if (!kivi_enabled_ || seq_len <= 0) return;
    const int n_vecs = seq_len * n_kv_heads_;
    throw_on(tkv_kivi_roundtrip_inplace(k_ptr, n_vecs, head_dim_, n_outliers_, group_size_,
                                        stream),
             "KvCompressionPass::run (K)");
    throw_on(tkv_kivi_roundtrip_inplace(v_ptr, n_vecs, head_dim_, n_outliers_, group_size_,
                                        stream),
             "KvCompressionPass::run (V)");
  }

  bool enabled() const { return kivi_enabled_; }
  int n_outliers() const { return n_outliers_; }
  int group_size() const { return group_size_; }

 private:
  bool kivi_enabled_;
  int n_layers_, n_kv_heads_, head_dim_, block_size_;
  int n_outliers_, group_size_;
};

// ---------------------------------------------------------------- paged cache
class PagedKiviCache {
 public:
  // pool: num_pages * n_kv_heads * page_bytes() bytes; ring: ring_bytes()
  // bytes, zeroed before first use; both 16-byte aligned, owned by the caller.
  PagedKiviCache(void* pool, void* ring, int num_pages, int max_seqs, int head_dim,
                 int group_size, int residual, int bits, int n_kv_heads) {
    throw_on(tkv_format_init(&c_.fmt, head_dim, group_size, residual, bits, n_kv_heads),
             "PagedKiviCache format");
    c_.pool = pool;
    c_.ring = ring;
    c_.num_pages = num_pages;
    c_.max_seqs = max_seqs;
  }

  static tkv_format_t format(int head_dim, int group_size, int residual, int bits,
                             int n_kv_heads) {
    tkv_format_t f{};
    throw_on(tkv_format_init(&f, head_dim, group_size, residual, bits, n_kv_heads), "format");
    return f;
  }
  int64_t page_bytes() const { return c_.fmt.page_bytes; }
  int64_t pool_bytes() const { return c_.fmt.page_bytes * c_.fmt.n_kv_heads * c_.num_pages; }
  int64_t ring_bytes() const { return tkv_ring_bytes(&c_.fmt, c_.max_seqs); }
  const tkv_cache_t& c_struct() const { return c_; }

  // The reshape_and_cache slot (cache_kernels.cu:47-94): quantize-on-append.
  void append(const void* k_new, const void* v_new, int in_dtype, const int32_t* cu_new,
              const int32_t* seq_lens_old, const int32_t* block_tables, int max_blocks_per_seq,
              const int32_t* seq_slots, int num_seqs, int total_new_tokens, int max_new_tokens,
              int* err_flag, cudaStream_t stream) const {
    throw_on(tkv_paged_append(&c_, k_new, v_new, in_dtype, cu_new, seq_lens_old, block_tables,
                              max_blocks_per_seq, seq_slots, num_seqs, total_new_tokens,
                              max_new_tokens, err_flag, stream),
             "PagedKiviCache::append");
  }

  static size_t decode_workspace_bytes(int num_seqs, int num_q_heads, int head_dim,
                                       int max_context_len) {
    return tkv_decode_workspace_bytes(num_seqs, num_q_heads, head_dim, max_context_len);
  }

  // Chunked prefill (the reference's token-by-token prefill, cuda_engine.cpp:842-860):
  // each sequence's last cu_q[s+1]-cu_q[s] tokens attend causally to the cache.
  void prefill(const void* q, int q_dtype, void* out, int out_dtype, const int32_t* cu_q,
               const int32_t* block_tables, int max_blocks_per_seq, const int32_t* seq_lens,
               const int32_t* seq_slots, int num_seqs, int num_q_heads, int total_q_tokens,
               int max_q_tokens, float scale, int* err_flag, cudaStream_t stream) const {
    throw_on(tkv_paged_prefill(&c_, q, q_dtype, out, out_dtype, cu_q, block_tables,
                               max_blocks_per_seq, seq_lens, seq_slots, num_seqs, num_q_heads,
                               total_q_tokens, max_q_tokens, scale, err_flag, stream),
             "PagedKiviCache::prefill");
  }

  // The paged_attention_v1/v2 slot (cuda_engine.cpp:1137-1159).
  void decode(const void* q, int q_dtype, void* out, int out_dtype, const int32_t* block_tables,
              int max_blocks_per_seq, const int32_t* seq_lens, const int32_t* seq_slots,
              int num_seqs, int num_q_heads, float scale, int max_context_len, void* workspace,
              size_t workspace_bytes, int* err_flag, cudaStream_t stream) const {
    throw_on(tkv_paged_decode(&c_, q, q_dtype, out, out_dtype, block_tables, max_blocks_per_seq,
                              seq_lens, seq_slots, num_seqs, num_q_heads, scale, max_context_len,
                              workspace, workspace_bytes, err_flag, stream),
             "PagedKiviCache::decode");
  }

  // The same two slots with the engine's tensor views, for an engine that
  // keeps its call sites shaped like cuda_engine.cpp:48-62, where
  // paged_attention_v1/v2 and reshape_and_cache take truellm::TrueBuffer
  // (include/truellm/types.h:69-77).  Buf is any view with TrueBuffer's
  // fields (data, dtype, ndim, shape[4]); dtype holds truellm::DataType,
  // whose F32 / F16 / BF16 / I32 values equal TKV_F32 / TKV_F16 / TKV_BF16 /
  // TKV_I32.  Shapes are read from the views:
  //   decode: out, q [num_seqs, num_q_heads, head_dim]; block_tables
  //           [num_seqs, max_blocks_per_seq] int32; seq_lens [num_seqs] int32.
  //   append: key, value [total_new_tokens, n_kv_heads, head_dim]; cu_new
  //           [num_seqs + 1] int32; seq_lens_old [num_seqs] int32;
  //           block_tables [num_seqs, max_blocks_per_seq] int32.
  // A view of the wrong element type or rank throws, as a wrong argument to
  // the pointer forms does.
  template <class Buf>
  void decode(Buf& out, const Buf& q, const Buf& block_tables, const Buf& seq_lens, float scale,
              int max_context_len, void* workspace, size_t workspace_bytes, int* err_flag,
              cudaStream_t stream, const int32_t* seq_slots = nullptr) const {
    check_view(q, 3, -1, "decode: q");
    check_view(out, 3, -1, "decode: out");
    check_view(block_tables, 2, TKV_I32, "decode: block_tables");
    check_view(seq_lens, 1, TKV_I32, "decode: seq_lens");
    decode(q.data, static_cast<int>(q.dtype), out.data, static_cast<int>(out.dtype),
           static_cast<const int32_t*>(block_tables.data), static_cast<int>(block_tables.shape[1]),
           static_cast<const int32_t*>(seq_lens.data), seq_slots,
           static_cast<int>(q.shape[0]), static_cast<int>(q.shape[1]), scale, max_context_len,
           workspace, workspace_bytes, err_flag, stream);
  }
  template <class Buf>
  void append(const Buf& key, const Buf& value, const Buf& cu_new, const Buf& seq_lens_old,
              const Buf& block_tables, int max_new_tokens, int* err_flag, cudaStream_t stream,
              const int32_t* seq_slots = nullptr) const {
    check_view(key, 3, -1, "append: key");
    check_view(value, 3, static_cast<int>(key.dtype), "append: value");
    check_view(cu_new, 1, TKV_I32, "append: cu_new");
    check_view(seq_lens_old, 1, TKV_I32, "append: seq_lens_old");
    check_view(block_tables, 2, TKV_I32, "append: block_tables");
    append(key.data, value.data, static_cast<int>(key.dtype),
           static_cast<const int32_t*>(cu_new.data),
           static_cast<const int32_t*>(seq_lens_old.data),
           static_cast<const int32_t*>(block_tables.data), static_cast<int>(block_tables.shape[1]),
           seq_slots, static_cast<int>(seq_lens_old.shape[0]), static_cast<int>(key.shape[0]),
           max_new_tokens, err_flag, stream);
  }

 private:
  template <class Buf>
  static void check_view(const Buf& b, int ndim, int dtype, const char* what) {
    if (b.data == nullptr || b.ndim != ndim ||
        (dtype >= 0 && static_cast<int>(b.dtype) != dtype))
      throw_on(TKV_INVALID_ARGUMENT, what);
  }
  tkv_cache_t c_{};
};

// ---------------------------------------------------------------- page allocator
// CudaAllocator's bookkeeping (cuda_allocator.h:38-160) for the KIVI cache,
// with the reference's bool / -1 returns.  Host only; the device half of
// copy / evict / reload is copy_ring_rows / swap_pages / swap_ring_rows below.
class KiviPageAllocator {
 public:
  KiviPageAllocator(const tkv_format_t& fmt, int num_pages, int max_seqs, int max_blocks_per_seq)
      : max_blocks_(max_blocks_per_seq), num_pages_(num_pages) {
    throw_on(tkv_allocator_create(&fmt, num_pages, max_seqs, max_blocks_per_seq, &a_),
             "KiviPageAllocator");
  }
  ~KiviPageAllocator() { tkv_allocator_destroy(a_); }
  KiviPageAllocator(const KiviPageAllocator&) = delete;
  KiviPageAllocator& operator=(const KiviPageAllocator&) = delete;

  bool allocate_sequence(uint64_t seq_id, int num_prompt_tokens, int32_t* ring_row = nullptr) {
    return tkv_allocator_add_sequence(a_, seq_id, num_prompt_tokens, ring_row) == TKV_OK;
  }
  // Pages added so the table covers new_len tokens, or -1.
  int extend_sequence(uint64_t seq_id, int new_len) {
    int added = 0;
    return tkv_allocator_extend(a_, seq_id, new_len, &added) == TKV_OK ? added : -1;
  }
  void free_sequence(uint64_t seq_id) { tkv_allocator_free_sequence(a_, seq_id); }
  // Shares src's pages; the caller copies ring row *src_row to *dst_row.
  bool copy_sequence(uint64_t src_id, uint64_t dst_id, int32_t* src_row = nullptr,
                     int32_t* dst_row = nullptr) {
    return tkv_allocator_fork(a_, src_id, dst_id, src_row, dst_row) == TKV_OK;
  }
  // block_tables [n][max_blocks_per_seq()] (-1 padded), seq_lens [n], ring_rows [n].
  void block_tables(const uint64_t* seq_ids, int n, int32_t* block_tables, int32_t* seq_lens,
                    int32_t* ring_rows) const {
    throw_on(tkv_allocator_tables(a_, seq_ids, n, block_tables, seq_lens, ring_rows),
             "KiviPageAllocator::block_tables");
  }
  // pages: capacity max_blocks_per_seq(); released on return.
  bool evict_sequence(uint64_t seq_id, int32_t* pages, int* n_pages, int32_t* ring_row) {
    return tkv_allocator_evict(a_, seq_id, pages, n_pages, ring_row) == TKV_OK;
  }
  bool reload_sequence(uint64_t seq_id, int32_t* pages, int* n_pages, int32_t* ring_row) {
    return tkv_allocator_reload(a_, seq_id, pages, n_pages, ring_row) == TKV_OK;
  }
  tkv_allocator_stats_t stats() const {
    tkv_allocator_stats_t s{};
    throw_on(tkv_allocator_stats(a_, &s), "KiviPageAllocator::stats");
    return s;
  }
  int num_free_blocks() const { return stats().pages_free; }
  int num_total_blocks() const { return num_pages_; }
  int block_size() const { return TKV_PAGE_SIZE; }
  int max_blocks_per_seq() const { return max_blocks_; }

 private:
  tkv_allocator_t* a_ = nullptr;
  int max_blocks_, num_pages_;
};

// copy_blocks / swap_blocks (cache_kernels.cu:234-283) for KIVI pages and ring rows.
inline void copy_pages(const tkv_cache_t& c, const int32_t* mapping, int n, int* err,
                       cudaStream_t stream) {
  throw_on(tkv_copy_pages(&c, mapping, n, err, stream), "copy_pages");
}
inline void swap_pages(const tkv_cache_t& c, void* images, int64_t capacity,
                       const int32_t* mapping, int n, int direction, int* err,
                       cudaStream_t stream) {
  throw_on(tkv_swap_pages(&c, images, capacity, mapping, n, direction, err, stream),
           "swap_pages");
}
inline void copy_ring_rows(const tkv_cache_t& c, const int32_t* mapping, int n, int* err,
                           cudaStream_t stream) {
  throw_on(tkv_copy_ring_rows(&c, mapping, n, err, stream), "copy_ring_rows");
}
inline void swap_ring_rows(const tkv_cache_t& c, void* images, int64_t capacity,
                           const int32_t* mapping, int n, int direction, int* err,
                           cudaStream_t stream) {
  throw_on(tkv_swap_ring_rows(&c, images, capacity, mapping, n, direction, err, stream),
           "swap_ring_rows");
}

}  // namespace kivi_b200
}  // namespace truellm
