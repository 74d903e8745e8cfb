// tkv_api.cu -- the extern "C" boundary declared in include/truellm_kivi.h:
// argument validation, format math, kernel launches and kernel manifests.
// Nothing here allocates device memory or synchronises the host.
#include <limits.h>
#include <math.h>
#include <string.h>

#include "tkv_common.cuh"

using namespace tkv;

namespace {

cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

bool fmt_ok(const tkv_format_t* f) {
  if (!f) return false;
  tkv_format_t chk;
  if (tkv_format_init(&chk, f->head_dim, f->group_size, f->residual, f->bits, f->n_kv_heads) !=
      TKV_OK)
    return false;
  return memcmp(&chk, f, sizeof(chk)) == 0;
}

bool cache_ok(const tkv_cache_t* c) {
  return c && c->pool && c->ring && c->num_pages > 0 && c->max_seqs > 0 && fmt_ok(&c->fmt);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int ref_check(int head_dim, int n_outliers, int group_size) {
  if (!tkv_kivi_params_supported(head_dim, n_outliers, group_size)) return TKV_INVALID_ARGUMENT;
  // Odd group sizes make the reference's records overrun their stride
  // (kivi_cache.cuh:41 reserves group_size/2 + 4 bytes, a full odd group
  // writes one more), so neighbouring vectors overlap: not supported here.
  if (group_size % 2 != 0) return TKV_INVALID_ARGUMENT;
  return TKV_OK;
}

int manifest_init(void*) { return 0; }
void manifest_shutdown(void*) {}

truellm_kernel_manifest_t g_attention_manifest = {
    TRUELLM_KERNEL_ABI_VERSION,
    "kivi_paged_attention_sm100a",
    "1.0.0",
    TRUELLM_KERNEL_ATTENTION,
    10,
    0,
    manifest_init,
    manifest_shutdown,
    nullptr,
};

truellm_kernel_manifest_t g_cache_manifest = {
    TRUELLM_KERNEL_ABI_VERSION,
    "kivi_paged_append_sm100a",
    "1.0.0",
    TRUELLM_KERNEL_CACHE,
    10,
    0,
    manifest_init,
    manifest_shutdown,
    nullptr,
};

}  // namespace

extern "C" {

int tkv_abi_version(void) { return TKV_ABI_VERSION; }

const char* tkv_status_string(int status) {
  switch (status) {
    case TKV_OK: return "ok";
    case TKV_INVALID_ARGUMENT: return "invalid argument";
    case TKV_NOT_IMPLEMENTED: return "not implemented";
    case TKV_OUT_OF_MEMORY: return "out of memory";
    case TKV_BACKEND_ERROR: return "CUDA error";
    default: return "unknown status";
  }
}

int tkv_format_init(tkv_format_t* f, int head_dim, int group_size, int residual, int bits,
                    int n_kv_heads) {
  if (!f) return TKV_INVALID_ARGUMENT;
  if (head_dim != 64 && head_dim != 128) return TKV_NOT_IMPLEMENTED;
  if (group_size != 16 && group_size != 32 && group_size != 64 && group_size != 128)
    return TKV_NOT_IMPLEMENTED;
  if (bits != 4 && bits != 2) return TKV_NOT_IMPLEMENTED;
  if (residual < 0 || residual > (1 << 20) || n_kv_heads <= 0) return TKV_INVALID_ARGUMENT;
  memset(f, 0, sizeof(*f));
  f->head_dim = head_dim;
  f->group_size = group_size;
  f->residual = residual;
  f->bits = bits;
  f->n_kv_heads = n_kv_heads;
  f->ring_cap = (residual + group_size + TKV_PAGE_SIZE - 1) / TKV_PAGE_SIZE * TKV_PAGE_SIZE;
  f->n_vgroups = (head_dim + group_size - 1) / group_size;
  const int codes = TKV_PAGE_SIZE * head_dim * bits / 8;
  f->k_codes_off = 0;
  f->v_codes_off = codes;
  f->v_meta_off = 2 * codes;
  f->k_meta_off = f->v_meta_off + TKV_PAGE_SIZE * f->n_vgroups * 4;
  f->k_meta_slice = head_dim * 4 * TKV_PAGE_SIZE / group_size;
  const int64_t pb = f->k_meta_off + f->k_meta_slice;
  f->page_bytes = (pb + 15) / 16 * 16;
  return TKV_OK;
}

int64_t tkv_ring_bytes(const tkv_format_t* f, int max_seqs) {
  if (!fmt_ok(f) || max_seqs < 0) return -1;
  return (int64_t)max_seqs * f->n_kv_heads * f->ring_cap * f->head_dim * 2 * 2;
}

int tkv_quantized_len(const tkv_format_t* f, int len) {
  if (!f || f->group_size <= 0) return 0;
  int x = len - f->residual;
  return x > 0 ? f->group_size * (x / f->group_size) : 0;
}

// ---------------------------------------------------------------------------
// reference format
// ---------------------------------------------------------------------------
size_t tkv_kivi_compressed_bytes(int head_dim, int n_outliers, int group_size) {
  if (group_size <= 0) return 0;
  int n_res = head_dim - n_outliers;
  int n_groups = (n_res + group_size - 1) / group_size;
  return (size_t)n_outliers * 3 + (size_t)n_groups * (size_t)(group_size / 2 + 4);
}

int tkv_kivi_params_supported(int head_dim, int n_outliers, int group_size) {
  return head_dim > 0 && head_dim <= 128 && n_outliers >= 0 && n_outliers <= 64 &&
         group_size > 0 && n_outliers <= head_dim;
}

int tkv_kivi_compress(const void* d_in, void* d_out, int n_vecs, int head_dim, int n_outliers,
                      int group_size, void* stream) {
  if (n_vecs < 0 || (!d_in && n_vecs) || (!d_out && n_vecs)) return TKV_INVALID_ARGUMENT;
  int st = ref_check(head_dim, n_outliers, group_size);
  if (st != TKV_OK) return st;
  if (n_vecs == 0) return TKV_OK;
  return launch_ref_kivi(0, d_in, d_out, n_vecs, head_dim, n_outliers, group_size,
                         as_stream(stream));
}

int tkv_kivi_decompress(const void* d_in, void* d_out, int n_vecs, int head_dim, int n_outliers,
                        int group_size, void* stream) {
  if (n_vecs < 0 || (!d_in && n_vecs) || (!d_out && n_vecs)) return TKV_INVALID_ARGUMENT;
  int st = ref_check(head_dim, n_outliers, group_size);
  if (st != TKV_OK) return st;
  if (n_vecs == 0) return TKV_OK;
  return launch_ref_kivi(1, d_in, d_out, n_vecs, head_dim, n_outliers, group_size,
                         as_stream(stream));
}

int tkv_kivi_roundtrip_inplace(void* d_kv, int n_vecs, int head_dim, int n_outliers,
                               int group_size, void* stream) {
  if (n_vecs < 0 || (!d_kv && n_vecs)) return TKV_INVALID_ARGUMENT;
  int st = ref_check(head_dim, n_outliers, group_size);
  if (st != TKV_OK) return st;
  if (n_vecs == 0) return TKV_OK;
  return launch_ref_kivi(2, d_kv, d_kv, n_vecs, head_dim, n_outliers, group_size,
                         as_stream(stream));
}

// ---------------------------------------------------------------------------
// paged append
// ---------------------------------------------------------------------------
int tkv_paged_append(const tkv_cache_t* cache, const void* k_new, const void* v_new, int in_dtype,
                     const int32_t* cu_new, const int32_t* seq_lens_old,
                     const int32_t* block_tables, int max_blocks_per_seq,
                     const int32_t* seq_slots, int num_seqs, int total_new_tokens,
                     int max_new_tokens, int* err_flag, void* stream) {
  if (!cache_ok(cache)) return TKV_INVALID_ARGUMENT;
  if (in_dtype != TKV_F16 && in_dtype != TKV_BF16) return TKV_NOT_IMPLEMENTED;
  if (num_seqs < 0 || num_seqs > 65535 || max_new_tokens < 0 || total_new_tokens < 0 ||
      max_blocks_per_seq <= 0)
    return TKV_INVALID_ARGUMENT;
  if (num_seqs == 0 || max_new_tokens == 0) return TKV_OK;
  if (!k_new || !v_new || !cu_new || !seq_lens_old || !block_tables) return TKV_INVALID_ARGUMENT;
  if (!aligned16(k_new) || !aligned16(v_new) || !aligned16(cache->pool) ||
      !aligned16(cache->ring))
    return TKV_INVALID_ARGUMENT;
  const tkv_format_t& f = cache->fmt;
  AppendArgs a;
  a.pool = static_cast<uint8_t*>(cache->pool);
  a.ring = static_cast<uint16_t*>(cache->ring);
  a.num_pages = cache->num_pages;
  a.max_seqs = cache->max_seqs;
  a.n_kv_heads = f.n_kv_heads;
  a.head_dim = f.head_dim;
  a.group = f.group_size;
  a.residual = f.residual;
  a.bits = f.bits;
  a.ring_cap = f.ring_cap;
  a.n_vgroups = f.n_vgroups;
  a.k_codes_off = f.k_codes_off;
  a.v_codes_off = f.v_codes_off;
  a.v_meta_off = f.v_meta_off;
  a.k_meta_off = f.k_meta_off;
  a.k_meta_slice = f.k_meta_slice;
  a.page_bytes = f.page_bytes;
  a.k_new = k_new;
  a.v_new = v_new;
  a.in_bf16 = in_dtype == TKV_BF16;
  a.cu_new = cu_new;
  a.lens_old = seq_lens_old;
  a.block_tables = block_tables;
  a.max_blocks = max_blocks_per_seq;
  a.seq_slots = seq_slots;
  a.total_new = total_new_tokens;
  a.max_new = max_new_tokens;
  a.err = err_flag;
  return launch_append(a, num_seqs, as_stream(stream));
}

// ---------------------------------------------------------------------------
// paged decode
// ---------------------------------------------------------------------------
int tkv_decode_num_splits(int max_context_len) {
  if (max_context_len < 0) return 0;
  return (max_context_len + TKV_SPLIT_TOKENS - 1) / TKV_SPLIT_TOKENS + 1;
}

size_t tkv_decode_workspace_bytes(int num_seqs, int num_q_heads, int head_dim,
                                  int max_context_len) {
  if (num_seqs <= 0 || num_q_heads <= 0 || head_dim <= 0 || max_context_len < 0) return 0;
  return stream_workspace_bytes(num_seqs, num_q_heads, head_dim);
}

int tkv_decode_launches(int num_seqs, int num_q_heads, int num_kv_heads, int max_context_len) {
  if (num_seqs <= 0 || num_q_heads <= 0 || num_kv_heads <= 0 || num_q_heads % num_kv_heads != 0 ||
      max_context_len < 0)
    return 0;
  return stream_decode_launches(num_seqs, num_kv_heads);
}

size_t tkv_decode_range_workspace_bytes(int num_seqs, int num_q_heads, int head_dim,
                                        int split_lo, int split_hi) {
  if (num_seqs <= 0 || num_q_heads <= 0 || head_dim <= 0 || split_lo < 0 ||
      split_hi < split_lo)
    return 0;
  return stream_workspace_bytes(num_seqs, num_q_heads, head_dim);
}

// Arguments of the stream decode shared by tkv_paged_decode and
// tkv_paged_decode_range; TKV_OK when they are valid.
static int stream_args(StreamArgs& a, const tkv_cache_t* cache, const void* q, int q_dtype,
                       const int32_t* block_tables, int max_blocks_per_seq,
                       const int32_t* seq_lens, const int32_t* seq_slots, int num_seqs,
                       int num_q_heads, float scale, int* err_flag) {
  if (!cache_ok(cache)) return TKV_INVALID_ARGUMENT;
  const tkv_format_t& f = cache->fmt;
  if (q_dtype != TKV_F16 && q_dtype != TKV_BF16) return TKV_NOT_IMPLEMENTED;
  if (num_seqs <= 0 || num_seqs > 65535 || num_q_heads <= 0) return TKV_INVALID_ARGUMENT;
  if (num_q_heads % f.n_kv_heads != 0) return TKV_INVALID_ARGUMENT;
  const int grp = num_q_heads / f.n_kv_heads;
  if (grp > 8) return TKV_NOT_IMPLEMENTED;  // one mma n-tile of 8 q heads per kv head
  if (!q || !block_tables || !seq_lens || max_blocks_per_seq <= 0) return TKV_INVALID_ARGUMENT;
  if (!(scale > 0.f) || !isfinite(scale)) return TKV_INVALID_ARGUMENT;
  // q rows, pool pages and ring chunks are moved by 16-byte bulk copies
  if (!aligned16(q) || !aligned16(cache->pool) || !aligned16(cache->ring))
    return TKV_INVALID_ARGUMENT;
  memset(&a, 0, sizeof(a));
  a.pool = static_cast<const uint8_t*>(cache->pool);
  a.ring = static_cast<const uint16_t*>(cache->ring);
  a.num_pages = cache->num_pages;
  a.max_seqs = cache->max_seqs;
  a.n_kv_heads = f.n_kv_heads;
  a.residual = f.residual;
  a.ring_cap = f.ring_cap;
  a.q = q;
  a.q_bf16 = q_dtype == TKV_BF16;
  a.block_tables = block_tables;
  a.max_blocks = max_blocks_per_seq;
  a.seq_lens = seq_lens;
  a.seq_slots = seq_slots;
  a.num_seqs = num_seqs;
  a.num_q_heads = num_q_heads;
  a.grp = grp;
  a.max_len = INT_MAX;
  a.alpha = scale * 1.4426950408889634f;
  a.pg_lo = 0;
  a.pg_hi = INT_MAX;
  a.include_residual = 1;
  a.err = err_flag;
  return TKV_OK;
}

static int decode_partials_impl(const tkv_cache_t* cache, const void* q, int q_dtype,
                                const int32_t* block_tables, int max_blocks_per_seq,
                                const int32_t* seq_lens, const int32_t* seq_slots, int num_seqs,
                                int num_q_heads, float scale, int split_lo, int split_hi,
                                int include_residual, float* part_ml, float* part_o,
                                void* work, unsigned int* bh_count, void* out, int out_dtype,
                                int* err_flag, cudaStream_t stream,
                                int split_pages = kSplitPages) {
  if (!cache_ok(cache)) return TKV_INVALID_ARGUMENT;
  const tkv_format_t& f = cache->fmt;
  if (q_dtype != TKV_F16 && q_dtype != TKV_BF16) return TKV_NOT_IMPLEMENTED;
  if (num_seqs <= 0 || num_seqs > 65535 || num_q_heads <= 0) return TKV_INVALID_ARGUMENT;
  if (num_q_heads % f.n_kv_heads != 0) return TKV_INVALID_ARGUMENT;
  const int grp = num_q_heads / f.n_kv_heads;
  if (grp > 8) return TKV_NOT_IMPLEMENTED;  // one mma n-tile of 8 q heads per kv head
  if (!q || !block_tables || !seq_lens || !part_ml || !part_o || !work ||
      max_blocks_per_seq <= 0)
    return TKV_INVALID_ARGUMENT;
  if (split_lo < 0 || split_hi < split_lo || !(scale > 0.f) || !isfinite(scale))
    return TKV_INVALID_ARGUMENT;
  if (!aligned16(cache->pool) || !aligned16(cache->ring)) return TKV_INVALID_ARGUMENT;
  DecodeArgs a;
  memset(&a, 0, sizeof(a));
  a.pool = static_cast<const uint8_t*>(cache->pool);
  a.ring = static_cast<const uint16_t*>(cache->ring);
  a.num_pages = cache->num_pages;
  a.max_seqs = cache->max_seqs;
  a.n_kv_heads = f.n_kv_heads;
  a.group = f.group_size;
  a.residual = f.residual;
  a.ring_cap = f.ring_cap;
  a.k_codes_off = f.k_codes_off;
  a.v_codes_off = f.v_codes_off;
  a.v_meta_off = f.v_meta_off;
  a.k_meta_off = f.k_meta_off;
  a.k_meta_slice = f.k_meta_slice;
  a.page_bytes = f.page_bytes;
  a.q = q;
  a.q_bf16 = q_dtype == TKV_BF16;
  a.block_tables = block_tables;
  a.max_blocks = max_blocks_per_seq;
  a.seq_lens = seq_lens;
  a.seq_slots = seq_slots;
  a.num_seqs = num_seqs;
  a.num_q_heads = num_q_heads;
  a.grp = grp;
  a.alpha = scale * 1.4426950408889634f;
  a.split_lo = split_lo;
  a.split_hi = split_hi;
  a.split_pages = split_pages;
  a.include_residual = include_residual ? 1 : 0;
  a.n_slots = (split_hi - split_lo) + a.include_residual;
  a.part_ml = part_ml;
  a.part_o = part_o;
  a.work = static_cast<unsigned int*>(work);
  a.bh_count = bh_count;
  a.fuse_merge = bh_count != nullptr && out != nullptr && a.include_residual;
  a.out = out;
  a.out_dtype = out_dtype;
  a.err = err_flag;
  if (a.n_slots == 0) return TKV_OK;
  return launch_decode_splits(a, f.head_dim, f.bits, f.n_vgroups, stream);
}

int tkv_paged_decode_partials(const tkv_cache_t* cache, const void* q, int q_dtype,
                              const int32_t* block_tables, int max_blocks_per_seq,
                              const int32_t* seq_lens, const int32_t* seq_slots, int num_seqs,
                              int num_q_heads, float scale, int split_lo, int split_hi,
                              int include_residual, float* part_ml, float* part_o, void* work,
                              int* err_flag, void* stream) {
  return decode_partials_impl(cache, q, q_dtype, block_tables, max_blocks_per_seq, seq_lens,
                              seq_slots, num_seqs, num_q_heads, scale, split_lo, split_hi,
                              include_residual, part_ml, part_o, work, nullptr, nullptr, 0,
                              err_flag, as_stream(stream));
}

int tkv_paged_decode_range(const tkv_cache_t* cache, const void* q, int q_dtype,
                           const int32_t* block_tables, int max_blocks_per_seq,
                           const int32_t* seq_lens, const int32_t* seq_slots, int num_seqs,
                           int num_q_heads, float scale, int split_lo, int split_hi,
                           int include_residual, float* out_ml, float* out_o, void* workspace,
                           size_t workspace_bytes, int* err_flag, void* stream) {
  if (!cache_ok(cache) || !out_ml || !out_o || !workspace || !aligned16(workspace))
    return TKV_INVALID_ARGUMENT;
  if (num_seqs <= 0 || num_q_heads <= 0 || split_lo < 0 || split_hi < split_lo)
    return TKV_INVALID_ARGUMENT;
  if (split_hi == split_lo && !include_residual) return TKV_INVALID_ARGUMENT;  // nothing to do
  const int D = cache->fmt.head_dim;
  if (workspace_bytes < stream_workspace_bytes(num_seqs, num_q_heads, D))
    return TKV_INVALID_ARGUMENT;
  StreamArgs a;
  const int st = stream_args(a, cache, q, q_dtype, block_tables, max_blocks_per_seq, seq_lens,
                             seq_slots, num_seqs, num_q_heads, scale, err_flag);
  if (st != TKV_OK) return st;
  constexpr int kMaxSplit = INT_MAX / kSplitPages;
  a.pg_lo = split_lo < kMaxSplit ? split_lo * kSplitPages : INT_MAX;
  a.pg_hi = split_hi < kMaxSplit ? split_hi * kSplitPages : INT_MAX;
  a.include_residual = include_residual ? 1 : 0;
  a.mode = kStreamPartials;
  a.out = out_o;
  a.out_dtype = TKV_F32;
  return launch_stream_decode(a, D, cache->fmt.bits, cache->fmt.group_size, workspace,
                              workspace_bytes, out_ml, as_stream(stream));
}

// ---------------------------------------------------------------------------
// token split over peer memory
// ---------------------------------------------------------------------------
static_assert(TKV_MAX_PEERS == kMaxPeers, "exchange struct and kernels agree");
static_assert(sizeof(cudaIpcMemHandle_t) == TKV_IPC_HANDLE_BYTES, "IPC handle size");
static_assert(kExStateOff >= 2 * kMaxPeers * 4 && kExStateOff + 12 <= kExHeader, "header layout");

size_t tkv_exchange_buffer_bytes(int world, int num_seqs, int num_q_heads, int head_dim) {
  if (world < 1 || world > kMaxPeers || num_seqs <= 0 || num_q_heads <= 0 || head_dim <= 0)
    return 0;
  return kExHeader + 2ull * static_cast<size_t>(world) * static_cast<size_t>(num_seqs) *
                         static_cast<size_t>(num_q_heads) * (kExRowPad + head_dim) * sizeof(float);
}

// The device view of an exchange; TKV_OK when it is well formed.
static int ex_pub(ExPub& x, const tkv_exchange_t* ex, int num_seqs, int num_q_heads, int D) {
  if (!ex || ex->world < 1 || ex->world > kMaxPeers || ex->rank < 0 || ex->rank >= ex->world)
    return TKV_INVALID_ARGUMENT;
  if (num_seqs <= 0 || num_q_heads <= 0 || static_cast<long long>(num_seqs) * num_q_heads >
                                               static_cast<long long>(INT_MAX))
    return TKV_INVALID_ARGUMENT;
  memset(&x, 0, sizeof(x));
  for (int r = 0; r < ex->world; ++r) {
    if (!ex->buffers[r] || !aligned16(ex->buffers[r])) return TKV_INVALID_ARGUMENT;
    x.set0[r] = reinterpret_cast<float*>(static_cast<uint8_t*>(ex->buffers[r]) + kExHeader);
    x.flags[r] = static_cast<uint32_t*>(ex->buffers[r]);
  }
  x.state = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(ex->buffers[ex->rank]) + kExStateOff);
  x.world = ex->world;
  x.rank = ex->rank;
  x.rows = num_seqs * num_q_heads;
  x.rs = kExRowPad + D;
  x.set_floats = static_cast<long long>(ex->world) * x.rows * x.rs;
  return TKV_OK;
}

int tkv_device_alloc(size_t bytes, void** ptr) {
  if (!ptr || bytes == 0) return TKV_INVALID_ARGUMENT;
  *ptr = nullptr;
  if (cudaMalloc(ptr, bytes) != cudaSuccess) return TKV_OUT_OF_MEMORY;
  if (cudaMemset(*ptr, 0, bytes) != cudaSuccess) {
    cudaFree(*ptr);
    *ptr = nullptr;
    return TKV_BACKEND_ERROR;
  }
  return TKV_OK;
}

int tkv_device_free(void* ptr) {
  if (!ptr) return TKV_OK;
  return cudaFree(ptr) == cudaSuccess ? TKV_OK : TKV_BACKEND_ERROR;
}

int tkv_ipc_get_handle(const void* ptr, void* handle) {
  if (!ptr || !handle) return TKV_INVALID_ARGUMENT;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, const_cast<void*>(ptr)) != cudaSuccess) return TKV_BACKEND_ERROR;
  memcpy(handle, &h, sizeof(h));
  return TKV_OK;
}

int tkv_ipc_open_handle(const void* handle, void** ptr) {
  if (!handle || !ptr) return TKV_INVALID_ARGUMENT;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  *ptr = nullptr;
  return cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess
             ? TKV_OK
             : TKV_BACKEND_ERROR;
}

int tkv_ipc_close_handle(void* ptr) {
  if (!ptr) return TKV_INVALID_ARGUMENT;
  return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? TKV_OK : TKV_BACKEND_ERROR;
}

int tkv_exchange_decode_range(const tkv_cache_t* cache, const void* q, int q_dtype,
                              const int32_t* block_tables, int max_blocks_per_seq,
                              const int32_t* seq_lens, const int32_t* seq_slots, int num_seqs,
                              int num_q_heads, float scale, int split_lo, int split_hi,
                              int include_residual, const tkv_exchange_t* ex, void* workspace,
                              size_t workspace_bytes, int* err_flag, void* stream) {
  if (!cache_ok(cache) || split_lo < 0 || split_hi < split_lo) return TKV_INVALID_ARGUMENT;
  const int D = cache->fmt.head_dim;
  ExPub pub;
  int st = ex_pub(pub, ex, num_seqs, num_q_heads, D);
  if (st != TKV_OK) return st;
  if (split_hi == split_lo && !include_residual)  // nothing here: empty partials
    return launch_ex_publish_empty(pub, D, as_stream(stream));
  if (!workspace || !aligned16(workspace) ||
      workspace_bytes < stream_workspace_bytes(num_seqs, num_q_heads, D))
    return TKV_INVALID_ARGUMENT;
  StreamArgs a;
  st = stream_args(a, cache, q, q_dtype, block_tables, max_blocks_per_seq, seq_lens, seq_slots,
                   num_seqs, num_q_heads, scale, err_flag);
  if (st != TKV_OK) return st;
  constexpr int kMaxSplit = INT_MAX / kSplitPages;
  a.pg_lo = split_lo < kMaxSplit ? split_lo * kSplitPages : INT_MAX;
  a.pg_hi = split_hi < kMaxSplit ? split_hi * kSplitPages : INT_MAX;
  a.include_residual = include_residual ? 1 : 0;
  a.mode = kStreamPartials;
  a.out = nullptr;
  a.out_dtype = TKV_F32;
  return launch_stream_decode(a, D, cache->fmt.bits, cache->fmt.group_size, workspace,
                              workspace_bytes, nullptr, as_stream(stream), &pub);
}

int tkv_exchange_merge(const tkv_exchange_t* ex, int num_seqs, int num_q_heads, int head_dim,
                       void* out, int out_dtype, int* err_flag, void* stream) {
  if (!out || (head_dim != 64 && head_dim != 128)) return TKV_INVALID_ARGUMENT;
  if (out_dtype != TKV_F32 && out_dtype != TKV_F16 && out_dtype != TKV_BF16)
    return TKV_NOT_IMPLEMENTED;
  ExPub pub;
  const int st = ex_pub(pub, ex, num_seqs, num_q_heads, head_dim);
  if (st != TKV_OK) return st;
  return launch_ex_merge(pub, head_dim, out, out_dtype, err_flag, as_stream(stream));
}

int tkv_paged_prefill(const tkv_cache_t* cache, const void* q, int q_dtype, void* out,
                      int out_dtype, const int32_t* cu_q, const int32_t* block_tables,
                      int max_blocks_per_seq, const int32_t* seq_lens, const int32_t* seq_slots,
                      int num_seqs, int num_q_heads, int total_q_tokens, int max_q_tokens,
                      float scale, int* err_flag, void* stream) {
  if (!cache_ok(cache)) return TKV_INVALID_ARGUMENT;
  if (q_dtype != TKV_F16 && q_dtype != TKV_BF16) return TKV_NOT_IMPLEMENTED;
  if (out_dtype != TKV_F32 && out_dtype != TKV_F16 && out_dtype != TKV_BF16)
    return TKV_NOT_IMPLEMENTED;
  const tkv_format_t& f = cache->fmt;
  if (num_seqs < 0 || num_q_heads <= 0 || num_q_heads % f.n_kv_heads != 0 ||
      total_q_tokens < 0 || max_q_tokens < 0 || max_blocks_per_seq <= 0)
    return TKV_INVALID_ARGUMENT;
  if (num_seqs == 0 || max_q_tokens == 0 || total_q_tokens == 0) return TKV_OK;
  if (!q || !out || !cu_q || !block_tables || !seq_lens || !aligned16(out))
    return TKV_INVALID_ARGUMENT;
  PrefillArgs a;
  a.pool = static_cast<const uint8_t*>(cache->pool);
  a.ring = static_cast<const uint16_t*>(cache->ring);
  a.num_pages = cache->num_pages;
  a.max_seqs = cache->max_seqs;
  a.n_kv_heads = f.n_kv_heads;
  a.residual = f.residual;
  a.ring_cap = f.ring_cap;
  a.q = q;
  a.q_bf16 = q_dtype == TKV_BF16;
  a.out = out;
  a.out_dtype = out_dtype;
  a.cu_q = cu_q;
  a.block_tables = block_tables;
  a.max_blocks = max_blocks_per_seq;
  a.seq_lens = seq_lens;
  a.seq_slots = seq_slots;
  a.num_seqs = num_seqs;
  a.num_q_heads = num_q_heads;
  a.grp = num_q_heads / f.n_kv_heads;
  a.total_q = total_q_tokens;
  a.max_q = max_q_tokens;
  a.n_rt = 0;
  a.alpha = scale * 1.4426950408889634f;
  a.err = err_flag;
  return launch_prefill(a, f.head_dim, f.bits, f.group_size, as_stream(stream));
}

int tkv_merge_partials(const float* part_ml, const float* part_o, int n_slots, int num_seqs,
                       int num_q_heads, int head_dim, void* out, int out_dtype, void* stream) {
  if (!part_ml || !part_o || !out || n_slots <= 0 || num_seqs <= 0 || num_seqs > 65535 ||
      num_q_heads <= 0 || head_dim <= 0)
    return TKV_INVALID_ARGUMENT;
  if (out_dtype != TKV_F32 && out_dtype != TKV_F16 && out_dtype != TKV_BF16)
    return TKV_NOT_IMPLEMENTED;
  return launch_merge(part_ml, part_o, n_slots, num_seqs, num_q_heads, head_dim, out, out_dtype,
                      as_stream(stream));
}

int tkv_paged_decode(const tkv_cache_t* cache, const void* q, int q_dtype, void* out,
                     int out_dtype, const int32_t* block_tables, int max_blocks_per_seq,
                     const int32_t* seq_lens, const int32_t* seq_slots, int num_seqs,
                     int num_q_heads, float scale, int max_context_len, void* workspace,
                     size_t workspace_bytes, int* err_flag, void* stream) {
  if (!cache_ok(cache) || max_context_len < 0 || !out || !workspace) return TKV_INVALID_ARGUMENT;
  if (num_seqs <= 0 || num_q_heads <= 0) return TKV_INVALID_ARGUMENT;
  const int D = cache->fmt.head_dim;
  const size_t need = tkv_decode_workspace_bytes(num_seqs, num_q_heads, D, max_context_len);
  if (workspace_bytes < need || !aligned16(workspace)) return TKV_INVALID_ARGUMENT;
  if (out_dtype != TKV_F32 && out_dtype != TKV_F16 && out_dtype != TKV_BF16)
    return TKV_NOT_IMPLEMENTED;
  StreamArgs a;
  const int st = stream_args(a, cache, q, q_dtype, block_tables, max_blocks_per_seq, seq_lens,
                             seq_slots, num_seqs, num_q_heads, scale, err_flag);
  if (st != TKV_OK) return st;
  a.max_len = max_context_len;  // longer sequences: TKV_ERR_BAD_LENGTH, zero output
  a.mode = stream_decode_launches(num_seqs, a.n_kv_heads) == 2 ? kStreamPartials : kStreamFused;
  a.out = out;
  a.out_dtype = out_dtype;
  return launch_stream_decode(a, D, cache->fmt.bits, cache->fmt.group_size, workspace,
                              workspace_bytes, nullptr, as_stream(stream));
}

// ---------------------------------------------------------------------------
// kernel registry
// ---------------------------------------------------------------------------
truellm_kernel_manifest_t* truellm_kernel_init(void) { return &g_attention_manifest; }
truellm_kernel_manifest_t* tkv_cache_kernel_manifest(void) { return &g_cache_manifest; }

}  // extern "C"
