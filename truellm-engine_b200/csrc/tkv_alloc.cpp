// tkv_alloc.cpp -- host page allocator of the paged KIVI cache (the
// tkv_allocator_* entry points of include/truellm_kivi.h).
//
// Bookkeeping only: free lists of page ids and ring rows, page reference
// counts, per-sequence tables and eviction records.  It follows the
// reference's CudaAllocator (src/inference/backends/cuda/cuda_allocator.cpp):
// the free list hands out the lowest id first (:97-99), a page returns to the
// list when its count drops to zero (:120-127), copy_sequence shares pages by
// count (:187-203), and eviction releases the pages and keeps the page count
// for the reload (:318-378).  Unlike the reference, every operation either
// completes or leaves the state unchanged (allocate_sequence rolls back,
// :147-153; reload_sequence does not), a duplicate or evicted id is an error
// rather than a silent overwrite, and each sequence also owns a ring row.
#include <algorithm>
#include <cstring>
#include <mutex>
#include <new>
#include <unordered_map>
#include <vector>

#include "truellm_kivi.h"

struct tkv_allocator {
  tkv_format_t fmt;
  int num_pages = 0, max_seqs = 0, max_blocks = 0;

  struct Seq {
    std::vector<int32_t> pages;  // table order; empty while evicted
    int len = 0;
    int32_t row = -1;            // ring row, -1 while evicted
    bool evicted = false;
    int evicted_pages = 0;
  };

  std::vector<int32_t> free_pages;  // stack: back() is the next page handed out
  std::vector<int32_t> free_rows;
  std::vector<int32_t> refs;        // per page
  std::unordered_map<uint64_t, Seq> seqs;
  int shared = 0;                   // pages with refs > 1
  mutable std::mutex mu;

  int pages_for(int len) const { return tkv_quantized_len(&fmt, len) / TKV_PAGE_SIZE; }

  int32_t take_page() {
    int32_t id = free_pages.back();
    free_pages.pop_back();
    refs[id] = 1;
    return id;
  }

  void release_page(int32_t id) {
    if (refs[id] == 2) --shared;
    if (--refs[id] == 0) free_pages.push_back(id);
  }

  void share_page(int32_t id) {
    if (++refs[id] == 2) ++shared;
  }

  int32_t take_row() {
    int32_t r = free_rows.back();
    free_rows.pop_back();
    return r;
  }
};

namespace {

bool len_ok(const tkv_allocator* a, int len) {
  return len >= 0 && a->pages_for(len) <= a->max_blocks;
}

}  // namespace

extern "C" {

int tkv_allocator_create(const tkv_format_t* fmt, int num_pages, int max_seqs,
                         int max_blocks_per_seq, tkv_allocator_t** out) {
  if (!fmt || !out || num_pages <= 0 || max_seqs <= 0 || max_blocks_per_seq <= 0)
    return TKV_INVALID_ARGUMENT;
  *out = nullptr;
  tkv_format_t chk;
  if (tkv_format_init(&chk, fmt->head_dim, fmt->group_size, fmt->residual, fmt->bits,
                      fmt->n_kv_heads) != TKV_OK ||
      std::memcmp(&chk, fmt, sizeof(chk)) != 0)
    return TKV_INVALID_ARGUMENT;
  auto* a = new (std::nothrow) tkv_allocator;
  if (!a) return TKV_OUT_OF_MEMORY;
  try {
    a->fmt = *fmt;
    a->num_pages = num_pages;
    a->max_seqs = max_seqs;
    a->max_blocks = max_blocks_per_seq;
    a->refs.assign(num_pages, 0);
    a->free_pages.resize(num_pages);
    for (int i = 0; i < num_pages; ++i) a->free_pages[i] = num_pages - 1 - i;
    a->free_rows.resize(max_seqs);
    for (int i = 0; i < max_seqs; ++i) a->free_rows[i] = max_seqs - 1 - i;
  } catch (const std::bad_alloc&) {
    delete a;
    return TKV_OUT_OF_MEMORY;
  }
  *out = a;
  return TKV_OK;
}

void tkv_allocator_destroy(tkv_allocator_t* a) { delete a; }

int tkv_allocator_pages_for(const tkv_allocator_t* a, int len) {
  if (!a || len < 0) return -1;
  return a->pages_for(len);
}

int tkv_allocator_add_sequence(tkv_allocator_t* a, uint64_t seq_id, int num_tokens,
                               int32_t* ring_row) {
  if (!a || !len_ok(a, num_tokens)) return TKV_INVALID_ARGUMENT;
  std::lock_guard<std::mutex> lock(a->mu);
  if (a->seqs.count(seq_id)) return TKV_INVALID_ARGUMENT;
  const int need = a->pages_for(num_tokens);
  if ((int)a->free_pages.size() < need || a->free_rows.empty()) return TKV_OUT_OF_MEMORY;
  // Every step that can throw comes before pages or a row are taken: the
  // entry is created, then its page list reserved (erased again on failure),
  // so an allocation failure leaves the allocator as it was.
  decltype(a->seqs.begin()) it;
  try {
    it = a->seqs.emplace(seq_id, tkv_allocator::Seq{}).first;
  } catch (const std::bad_alloc&) {
    return TKV_OUT_OF_MEMORY;
  }
  try {
    it->second.pages.reserve(need);
  } catch (const std::bad_alloc&) {
    a->seqs.erase(it);
    return TKV_OUT_OF_MEMORY;
  }
  for (int i = 0; i < need; ++i) it->second.pages.push_back(a->take_page());
  it->second.len = num_tokens;
  it->second.row = a->take_row();
  if (ring_row) *ring_row = it->second.row;
  return TKV_OK;
}

int tkv_allocator_extend(tkv_allocator_t* a, uint64_t seq_id, int new_len, int* n_new) {
  if (!a || !len_ok(a, new_len)) return TKV_INVALID_ARGUMENT;
  std::lock_guard<std::mutex> lock(a->mu);
  auto it = a->seqs.find(seq_id);
  if (it == a->seqs.end() || it->second.evicted || new_len < it->second.len)
    return TKV_INVALID_ARGUMENT;
  auto& s = it->second;
  const int need = a->pages_for(new_len) - (int)s.pages.size();
  if (need > (int)a->free_pages.size()) return TKV_OUT_OF_MEMORY;
  try {
    s.pages.reserve(s.pages.size() + std::max(need, 0));
  } catch (const std::bad_alloc&) {
    return TKV_OUT_OF_MEMORY;
  }
  for (int i = 0; i < need; ++i) s.pages.push_back(a->take_page());
  s.len = new_len;
  if (n_new) *n_new = std::max(need, 0);
  return TKV_OK;
}

int tkv_allocator_free_sequence(tkv_allocator_t* a, uint64_t seq_id) {
  if (!a) return TKV_INVALID_ARGUMENT;
  std::lock_guard<std::mutex> lock(a->mu);
  auto it = a->seqs.find(seq_id);
  if (it == a->seqs.end()) return TKV_OK;
  for (int32_t p : it->second.pages) a->release_page(p);
  if (it->second.row >= 0) a->free_rows.push_back(it->second.row);
  a->seqs.erase(it);
  return TKV_OK;
}

int tkv_allocator_fork(tkv_allocator_t* a, uint64_t src_id, uint64_t dst_id, int32_t* src_row,
                       int32_t* dst_row) {
  if (!a || src_id == dst_id) return TKV_INVALID_ARGUMENT;
  std::lock_guard<std::mutex> lock(a->mu);
  auto it = a->seqs.find(src_id);
  if (it == a->seqs.end() || it->second.evicted || a->seqs.count(dst_id))
    return TKV_INVALID_ARGUMENT;
  if (a->free_rows.empty()) return TKV_OUT_OF_MEMORY;
  try {
    tkv_allocator::Seq d;
    d.pages = it->second.pages;
    d.len = it->second.len;
    auto& slot = a->seqs[dst_id];  // may rehash: `it` is not used below
    d.row = a->take_row();
    for (int32_t p : d.pages) a->share_page(p);
    slot = std::move(d);
    if (dst_row) *dst_row = slot.row;
    if (src_row) *src_row = a->seqs.at(src_id).row;
  } catch (const std::bad_alloc&) {
    return TKV_OUT_OF_MEMORY;
  }
  return TKV_OK;
}

int tkv_allocator_tables(const tkv_allocator_t* a, const uint64_t* seq_ids, int n,
                         int32_t* block_tables, int32_t* seq_lens, int32_t* ring_rows) {
  if (!a || n < 0 || (n > 0 && !seq_ids)) return TKV_INVALID_ARGUMENT;
  std::lock_guard<std::mutex> lock(a->mu);
  for (int i = 0; i < n; ++i) {  // validate all before writing any
    auto it = a->seqs.find(seq_ids[i]);
    if (it == a->seqs.end() || it->second.evicted) return TKV_INVALID_ARGUMENT;
  }
  for (int i = 0; i < n; ++i) {
    const auto& s = a->seqs.find(seq_ids[i])->second;
    if (block_tables) {
      int32_t* row = block_tables + (size_t)i * a->max_blocks;
      std::copy(s.pages.begin(), s.pages.end(), row);
      std::fill(row + s.pages.size(), row + a->max_blocks, -1);
    }
    if (seq_lens) seq_lens[i] = s.len;
    if (ring_rows) ring_rows[i] = s.row;
  }
  return TKV_OK;
}

int tkv_allocator_sequence(const tkv_allocator_t* a, uint64_t seq_id, int* len, int* n_pages,
                           int32_t* ring_row, int* evicted) {
  if (!a) return TKV_INVALID_ARGUMENT;
  std::lock_guard<std::mutex> lock(a->mu);
  auto it = a->seqs.find(seq_id);
  if (it == a->seqs.end()) return TKV_INVALID_ARGUMENT;
  const auto& s = it->second;
  if (len) *len = s.len;
  if (n_pages) *n_pages = s.evicted ? s.evicted_pages : (int)s.pages.size();
  if (ring_row) *ring_row = s.row;
  if (evicted) *evicted = s.evicted ? 1 : 0;
  return TKV_OK;
}

int tkv_allocator_stats(const tkv_allocator_t* a, tkv_allocator_stats_t* out) {
  if (!a || !out) return TKV_INVALID_ARGUMENT;
  std::lock_guard<std::mutex> lock(a->mu);
  std::memset(out, 0, sizeof(*out));
  out->pages_total = a->num_pages;
  out->pages_free = (int32_t)a->free_pages.size();
  out->pages_used = a->num_pages - out->pages_free;
  out->pages_shared = a->shared;
  out->rows_total = a->max_seqs;
  out->rows_free = (int32_t)a->free_rows.size();
  out->sequences = (int32_t)a->seqs.size();
  for (const auto& kv : a->seqs) out->evicted += kv.second.evicted ? 1 : 0;
  out->utilization_pct = 100.f * out->pages_used / a->num_pages;
  return TKV_OK;
}

int tkv_allocator_evict(tkv_allocator_t* a, uint64_t seq_id, int32_t* pages, int* n_pages,
                        int32_t* ring_row) {
  if (!a) return TKV_INVALID_ARGUMENT;
  std::lock_guard<std::mutex> lock(a->mu);
  auto it = a->seqs.find(seq_id);
  if (it == a->seqs.end() || it->second.evicted) return TKV_INVALID_ARGUMENT;
  auto& s = it->second;
  if (!s.pages.empty() && !pages) return TKV_INVALID_ARGUMENT;
  std::copy(s.pages.begin(), s.pages.end(), pages);
  if (n_pages) *n_pages = (int)s.pages.size();
  if (ring_row) *ring_row = s.row;
  for (int32_t p : s.pages) a->release_page(p);
  a->free_rows.push_back(s.row);
  s.evicted_pages = (int)s.pages.size();
  s.pages.clear();
  s.pages.shrink_to_fit();
  s.row = -1;
  s.evicted = true;
  return TKV_OK;
}

int tkv_allocator_reload(tkv_allocator_t* a, uint64_t seq_id, int32_t* pages, int* n_pages,
                         int32_t* ring_row) {
  if (!a) return TKV_INVALID_ARGUMENT;
  std::lock_guard<std::mutex> lock(a->mu);
  auto it = a->seqs.find(seq_id);
  if (it == a->seqs.end() || !it->second.evicted) return TKV_INVALID_ARGUMENT;
  auto& s = it->second;
  const int need = s.evicted_pages;
  if (need > 0 && !pages) return TKV_INVALID_ARGUMENT;
  if ((int)a->free_pages.size() < need || a->free_rows.empty()) return TKV_OUT_OF_MEMORY;
  try {
    s.pages.reserve(need);
  } catch (const std::bad_alloc&) {
    return TKV_OUT_OF_MEMORY;
  }
  for (int i = 0; i < need; ++i) s.pages.push_back(a->take_page());
  s.row = a->take_row();
  s.evicted = false;
  s.evicted_pages = 0;
  std::copy(s.pages.begin(), s.pages.end(), pages);
  if (n_pages) *n_pages = need;
  if (ring_row) *ring_row = s.row;
  return TKV_OK;
}

}  // extern "C"
