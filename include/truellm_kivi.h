/*
 * truellm_kivi.h -- C ABI of the B200 (sm_100a) KIVI quantized-KV attention path.
 *
 * Drop-in boundary for truellm-engine's quantized-KV hot path.  Every entry
 * point takes plain pointers, sizes and a cudaStream_t (passed as void*), returns
 * an int status (tkv_status_t, same values as truellm::ErrorCode in the
 * reference's include/truellm/types.h:20-32), never throws and never
 * synchronises the host.  The caller owns every device buffer; workspace
 * sizes come from the *_bytes query functions, so nothing is allocated on the
 * hot path (reference convention: pre-allocated v2 temps,
 * src/inference/backends/cuda/cuda_engine.cpp:273-285).
 *
 * Paths in comments are relative to the truellm-engine source tree.
 *
 * ---------------------------------------------------------------------------
 * Paged KIVI cache format (version TKV_FORMAT_VERSION)
 * ---------------------------------------------------------------------------
 * Parameters: P = 16 tokens per page (the reference's paged_kv_block_size),
 * D = head_dim in {64, 128}, G = group_size in {16, 32, 64, 128},
 * R = residual_length >= 0, b = bits in {4, 2}.
 *
 * A sequence of length L keeps n_q = G * floor(max(L - R, 0) / G) tokens
 * quantised in pages and the n_r = L - n_q most recent tokens (R <= n_r < R+G
 * once L >= R) in fp16 in a per-sequence ring.
 *
 * Keys are quantised per channel over groups of G consecutive tokens, values
 * per token over groups of G consecutive channels, both with the reference
 * quantizer (kivi_cache.cu:92-124: min/max, scale = qmax/range, round half to
 * even, fp16 step = 1/scale, fp16 zero = min), qmax = 15 for b = 4 and 3 for
 * b = 2.  bf16 inputs are first rounded to fp16 (round to nearest even), so the
 * quantised bytes do not depend on how tokens were split into append calls.
 *
 * Page pool (per layer): [num_pages][n_kv_heads][page_bytes], the same
 * block-major, head-minor order as the reference pool
 * (third_party/vllm_kernels/cache_kernels.cu:27-37).  Block table entry
 * block_tables[s][j] is the physical page of tokens [16j, 16j+16) of sequence
 * s (slot = page * 16 + offset, cuda_allocator.cpp:273); unused entries are -1.
 * One (page, head) block holds, at the offsets reported by tkv_format_init():
 *   K codes  [16 tokens][D*b/8 bytes], channel c at bit c*b of the row
 *            (lowest bits = lowest channel; b = 4 is the reference's nibble
 *            order, low nibble = even index, kivi_cache.cu:113).
 *   V codes  16*D*b/8 bytes in "fragment order": the code of (channel c,
 *            token t) sits in 32-bit word w of lane l, where
 *              mb = c/16, g = (c%16)%8, rh = (c%16)/8, th = t/8,
 *              tig = (t%8)/2, e = t%2, l = 4*g + tig, k = 2*rh + th,
 *              b=4: w = mb,    bit = 4*(k + 4*e)
 *              b=2: w = mb/2,  bit = 2*(4*(mb%2) + k + 8*e)
 *            and word w of lane l is stored at byte
 *              ((w / VW) * 32 + l) * 4*VW + (w % VW) * 4,  VW = min(D*b/64, 4)
 *              (D*b/64 words per lane).
 *            (This is the A-operand register layout of mma.m16n8k16 for
 *            V^T tiles, so the decode kernel reads it with 16-byte loads.)
 *   V meta   [16 tokens][ceil(D/G) groups][fp16 step, fp16 zero].
 *   K meta   slice i (i = page index within its key group) of the group's
 *            [D][fp16 step, fp16 zero] array: D*4*16/G bytes.
 * page_bytes is the sum rounded up to 16.  D=128, G=128: 2176 B (b=4),
 * 1152 B (b=2).
 *
 * Residual ring: [max_seqs][n_kv_heads][ring_cap/16 chunks][2][16*D] fp16 with
 * ring_cap = round_up(R + G, 16); token t of a sequence lives in slot
 * t % ring_cap.  Within a chunk, the K block (index 0) stores element
 * (token t, channel c) at half offset ((c/16)*32 + l)*8 + 2*r + e with
 * cc = c%16, l = 4*(t%8) + (cc%8)/2, r = 2*(cc/8) + t/8, e = cc%2, and the V
 * block (index 1) at ((c/16)*32 + l)*8 + 2*r + e with cc = c%16,
 * l = 4*(cc%8) + (t%8)/2, r = 2*(t/8) + cc/8, e = t%2.
 * Ring rows are indexed by seq_slots[s] (or s when seq_slots is NULL).
 */
#ifndef TRUELLM_KIVI_H
#define TRUELLM_KIVI_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define TKV_API __attribute__((visibility("default")))
#else
#define TKV_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define TKV_ABI_VERSION 1
#define TKV_FORMAT_VERSION 1
#define TKV_PAGE_SIZE 16
#ifndef TKV_SPLIT_TOKENS
#define TKV_SPLIT_TOKENS 512 /* decode split (flash-decoding partition) length */
#endif

/* Status codes: the values of truellm::ErrorCode (include/truellm/types.h:20-32). */
typedef enum tkv_status {
  TKV_OK = 0,
  TKV_INVALID_ARGUMENT = 1,
  TKV_NOT_IMPLEMENTED = 3,
  TKV_OUT_OF_MEMORY = 4,
  TKV_BACKEND_ERROR = 5,
} tkv_status_t;

/* Element types: the values of truellm::DataType (include/truellm/types.h:47-53).
 * TKV_I32 only describes index views (block tables, lengths) in the C++
 * adapter's tensor-view overloads; no entry point takes it as a q, K/V or
 * output type. */
typedef enum tkv_dtype { TKV_F32 = 0, TKV_F16 = 1, TKV_BF16 = 2, TKV_I32 = 3 } tkv_dtype_t;

/* Bits set in the device error word (err_flag arguments) by bounds checks. */
#define TKV_ERR_BAD_PAGE 0x1    /* block-table entry outside [0, num_pages)    */
#define TKV_ERR_BAD_SLOT 0x2    /* ring row outside [0, max_seqs)              */
#define TKV_ERR_BAD_LENGTH 0x4  /* length or token count out of range          */
#define TKV_ERR_TIMEOUT 0x8     /* a bounded barrier wait gave up              */

/* Layout of one paged KIVI cache (one layer).  Filled by tkv_format_init. */
typedef struct tkv_format {
  int32_t head_dim, group_size, residual, bits, n_kv_heads;
  int32_t ring_cap;      /* R + G rounded up to 16                       */
  int32_t n_vgroups;     /* ceil(D / G)                                   */
  int32_t k_codes_off, v_codes_off, v_meta_off, k_meta_off, k_meta_slice;
  int64_t page_bytes;    /* bytes of one (page, kv head) block            */
} tkv_format_t;

/* Device buffers of one paged KIVI cache (one layer). */
typedef struct tkv_cache {
  void* pool;         /* [num_pages][n_kv_heads][page_bytes]                */
  void* ring;         /* [max_seqs][n_kv_heads][ring_cap/16][2][16*D] fp16  */
  int32_t num_pages;  /* pages in the pool (bounds for block-table entries) */
  int32_t max_seqs;   /* rows in the ring                                   */
  tkv_format_t fmt;
} tkv_cache_t;

/* ---------------------------------------------------------------- */
/* Library                                                           */
/* ---------------------------------------------------------------- */
TKV_API int tkv_abi_version(void);
TKV_API const char* tkv_status_string(int status);

/* Validates the parameters and fills *fmt.  Replaces the size math of
 * kivi_compressed_bytes (kivi_cache.cuh:32-43) for the paged format. */
TKV_API int tkv_format_init(tkv_format_t* fmt, int head_dim, int group_size, int residual, int bits,
                    int n_kv_heads);
/* Bytes of the ring for max_seqs sequences. */
TKV_API int64_t tkv_ring_bytes(const tkv_format_t* fmt, int max_seqs);
/* Quantised-token count n_q for a sequence of length len. */
TKV_API int tkv_quantized_len(const tkv_format_t* fmt, int len);

/* ---------------------------------------------------------------- */
/* Reference-format KIVI (per-vector outliers + INT4 channel groups)  */
/* ---------------------------------------------------------------- */
/* Same value as kivi_compressed_bytes (kivi_cache.cuh:32-43). */
TKV_API size_t tkv_kivi_compressed_bytes(int head_dim, int n_outliers, int group_size);
/* Same rule as kivi_params_supported (kivi_cache.cu:205-211). */
TKV_API int tkv_kivi_params_supported(int head_dim, int n_outliers, int group_size);
/* Replaces truellm::kivi_compress (kivi_cache.cuh:74-78, kivi_cache.cu:213-225):
 * fp16 [n_vecs, head_dim] -> bytes [n_vecs, kivi_compressed_bytes], byte for
 * byte the reference kernel's output (slack bytes of a partial last group are
 * not written).  Unsupported parameters return TKV_INVALID_ARGUMENT without
 * launching (the reference wrapper silently returns). */
TKV_API int tkv_kivi_compress(const void* d_in_f16, void* d_out, int n_vecs, int head_dim, int n_outliers,
                      int group_size, void* stream);
/* Replaces truellm::kivi_decompress (kivi_cache.cuh:80-84, kivi_cache.cu:227-239). */
TKV_API int tkv_kivi_decompress(const void* d_in, void* d_out_f16, int n_vecs, int head_dim,
                        int n_outliers, int group_size, void* stream);
/* Fused compress + decompress in place, one pass, no scratch: the result the
 * reference's KvCompressionPass::run_kivi produces with two launches per
 * tensor through a scratch buffer (kv_compression_pass.cpp:184-216). */
TKV_API int tkv_kivi_roundtrip_inplace(void* d_kv_f16, int n_vecs, int head_dim, int n_outliers,
                               int group_size, void* stream);

/* ---------------------------------------------------------------- */
/* Paged KIVI: quantize-on-append                                     */
/* ---------------------------------------------------------------- */
/* Replaces reshape_and_cache (cuda_engine.cpp:48-50, cache_kernels.cu:202-232)
 * for the KIVI cache.  Appends, for each sequence s, the tokens
 * k_new/v_new[cu_new[s] : cu_new[s+1]] ([T_total, n_kv_heads, D], fp16 or bf16)
 * after its seq_lens_old[s] existing tokens: every key/value group that becomes
 * complete is quantised into its pages, the rest goes to the fp16 ring.  The
 * block table must already cover the new length.  total_new_tokens is the
 * number of rows in k_new / v_new; max_new_tokens bounds cu_new[s+1]-cu_new[s]
 * (it sizes the grid).  Sequences whose offsets fall outside these bounds are
 * skipped and flagged with TKV_ERR_BAD_LENGTH.  Two kernel launches. */
TKV_API int tkv_paged_append(const tkv_cache_t* cache, const void* k_new, const void* v_new, int in_dtype,
                     const int32_t* cu_new, const int32_t* seq_lens_old,
                     const int32_t* block_tables, int max_blocks_per_seq,
                     const int32_t* seq_slots, int num_seqs, int total_new_tokens,
                     int max_new_tokens, int* err_flag, void* stream);

/* ---------------------------------------------------------------- */
/* Paged KIVI: decode attention                                       */
/* ---------------------------------------------------------------- */
/* Number of split slots per sequence: ceil(max_context_len / TKV_SPLIT_TOKENS) + 1
 * (the last one holds the fp16 residual). */
TKV_API int tkv_decode_num_splits(int max_context_len);
/* Workspace bytes for tkv_paged_decode: per-(sequence, kv head) completion
 * counters and the partials of pairs whose pages are spread over several
 * warps (one slot per pair plus one per resident warp of the GPU).  Zero the
 * whole workspace once when it is allocated; every call leaves the counters
 * zero again.  Calls that share a workspace must not overlap on the GPU.  The
 * size does not depend on max_context_len. */
TKV_API size_t tkv_decode_workspace_bytes(int num_seqs, int num_q_heads, int head_dim,
                                  int max_context_len);
/* Kernel launches tkv_paged_decode makes for these sizes on the current
 * device: 1 (merge fused into the decode launch) or 2 (fewer than one
 * (sequence, kv head) pair per 16 resident warps: pairs spread over many warps
 * each, whose merge runs in a separate slot-parallel launch).  0 for invalid
 * sizes (num_q_heads not a multiple of num_kv_heads included). */
TKV_API int tkv_decode_launches(int num_seqs, int num_q_heads, int num_kv_heads,
                                int max_context_len);
/* Workspace bytes for tkv_paged_decode_range over splits [split_lo, split_hi)
 * (with the finer internal splits the range may use). */
TKV_API size_t tkv_decode_range_workspace_bytes(int num_seqs, int num_q_heads, int head_dim,
                                                int split_lo, int split_hi);

/* Replaces paged_attention_v1/v2 (cuda_engine.cpp:51-62,
 * paged_attention_v1.cu:177-213, paged_attention_v2.cu:176-251) for the KIVI
 * cache: out[s, h, :] = softmax(scale * q[s,h,:] . K^T) V over the
 * seq_lens[s] tokens of sequence s, kv head = h / (num_q_heads / n_kv_heads)
 * (megakernel.cu:270-277).  q, out: [num_seqs, num_q_heads, D]; q is fp16 or
 * bf16, out is fp16, bf16 or f32.  Every resident warp of the GPU takes an
 * equal-cost range of the call's (sequence, kv head) pages and residual
 * chunks; a pair spread over several warps is merged by log-sum-exp
 * (paged_attention_v2.cu:132-170) in the warp that finishes its last part
 * (one launch) or, when pairs are fewer than one per 16 resident warps, in a
 * second slot-parallel launch (tkv_decode_launches).  Sequences longer than
 * max_context_len (or than max_blocks_per_seq pages) set TKV_ERR_BAD_LENGTH
 * in *err_flag and get a zero output row. */
TKV_API int tkv_paged_decode(const tkv_cache_t* cache, const void* q, int q_dtype, void* out,
                     int out_dtype, const int32_t* block_tables, int max_blocks_per_seq,
                     const int32_t* seq_lens, const int32_t* seq_slots, int num_seqs,
                     int num_q_heads, float scale, int max_context_len, void* workspace,
                     size_t workspace_bytes, int* err_flag, void* stream);

/* Size of the static device scratch used by tkv_paged_decode_noalloc. */
#define TKV_NOALLOC_SCRATCH_BYTES (16u << 20)

/* tkv_paged_decode without a workspace argument.  No counterpart in the
 * reference.  For callers that cannot allocate device memory -- a kernel
 * plugin that only receives the engine's tensors, a host whose allocator owns
 * all device memory, or a decode loop that must not call cudaMalloc -- the
 * split-KV partials and work counters live in a static device array of
 * TKV_NOALLOC_SCRATCH_BYTES that every GPU loading this library keeps until
 * the process exits.  Nothing is allocated.  Every call looks up the array's
 * device address on the current device and clears its completion counters
 * with a stream-ordered memset on `stream` before the decode launch.  Calls
 * whose tkv_decode_workspace_bytes() exceeds the scratch return
 * TKV_OUT_OF_MEMORY without launching.  All calls on a device share the
 * array, so calls that overlap on the GPU race; it keeps the last call's
 * partials. */
TKV_API int tkv_paged_decode_noalloc(const tkv_cache_t* cache, const void* q, int q_dtype,
                                     void* out, int out_dtype, const int32_t* block_tables,
                                     int max_blocks_per_seq, const int32_t* seq_lens,
                                     const int32_t* seq_slots, int num_seqs, int num_q_heads,
                                     float scale, int max_context_len, int* err_flag,
                                     void* stream);

/* Split-KV partials only (for sequences split across GPUs): computes the
 * quantised splits [split_lo, split_hi) of every sequence, plus the residual
 * split when include_residual != 0, into
 *   part_ml [n_split_slots][num_seqs][num_q_heads][2] f32  (m in log2 units, l)
 *   part_o  [n_split_slots][num_seqs][num_q_heads][D] f32  (unnormalised)
 * slot index = split - split_lo for quantised splits and split_hi - split_lo
 * for the residual.  Empty slots get m = -inf, l = 0.  work: 8 bytes of
 * device memory, zero before the first call and left zero by every call
 * (the persistent kernel's work counters). */
TKV_API int tkv_paged_decode_partials(const tkv_cache_t* cache, const void* q, int q_dtype,
                              const int32_t* block_tables, int max_blocks_per_seq,
                              const int32_t* seq_lens, const int32_t* seq_slots, int num_seqs,
                              int num_q_heads, float scale, int split_lo, int split_hi,
                              int include_residual, float* part_ml, float* part_o, void* work,
                              int* err_flag, void* stream);

/* One GPU's share of a decode whose quantised splits are spread over GPUs
 * (one long sequence split by tokens): the quantised splits [split_lo,
 * split_hi) of every sequence, plus the residual split when include_residual
 * != 0, reduced on the GPU (a second, slot-parallel kernel) to ONE
 * unnormalised partial per (sequence, q head):
 *   out_ml [num_seqs][num_q_heads][2] f32  (m in log2 units, l)
 *   out_o  [num_seqs][num_q_heads][D] f32
 * i.e. one slot of the tkv_paged_decode_partials layout, so the slots of all
 * GPUs, gathered in any order, go to tkv_merge_partials.  A (sequence, q head)
 * with no token in the range gets m = -inf, l = 0, o = 0.  No counterpart in
 * the reference (paged_attention_v2.cu keeps every partition on one GPU).
 * workspace: tkv_decode_range_workspace_bytes(num_seqs, num_q_heads, D,
 * split_lo, split_hi) bytes, 16-byte aligned, zeroed once as for
 * tkv_paged_decode (every call leaves its counters zero).  Two
 * launches. */
TKV_API int tkv_paged_decode_range(const tkv_cache_t* cache, const void* q, int q_dtype,
                                   const int32_t* block_tables, int max_blocks_per_seq,
                                   const int32_t* seq_lens, const int32_t* seq_slots,
                                   int num_seqs, int num_q_heads, float scale, int split_lo,
                                   int split_hi, int include_residual, float* out_ml,
                                   float* out_o, void* workspace, size_t workspace_bytes,
                                   int* err_flag, void* stream);

/* Chunked-prefill attention over the KIVI cache.  The reference runs its
 * prefill attention token by token (cuda_engine.cpp:842-860); this is one
 * launch for a batch of chunks.  For sequence s, the n_s = cu_q[s+1] - cu_q[s]
 * query rows q[cu_q[s] .. cu_q[s+1]) are its last n_s tokens (already appended
 * with tkv_paged_append), at positions p = seq_lens[s] - n_s + i; each
 * attends causally to tokens [0, p] with the decode's math and kv-head
 * mapping.  q: [total_q_tokens, num_q_heads, D] fp16 or bf16; out: same
 * shape, fp16, bf16 or f32, 16-byte aligned.  max_q_tokens bounds n_s (it
 * sizes the grid).  Sequences with n_s > seq_lens[s] or n_s > max_q_tokens
 * are skipped and flagged TKV_ERR_BAD_LENGTH.  One launch, no workspace. */
TKV_API int tkv_paged_prefill(const tkv_cache_t* cache, const void* q, int q_dtype, void* out,
                              int out_dtype, const int32_t* cu_q, const int32_t* block_tables,
                              int max_blocks_per_seq, const int32_t* seq_lens,
                              const int32_t* seq_slots, int num_seqs, int num_q_heads,
                              int total_q_tokens, int max_q_tokens, float scale, int* err_flag,
                              void* stream);

/* Log-sum-exp merge of n_slots partial sets laid out as above
 * (paged_attention_v2.cu:132-170) into out [num_seqs, num_q_heads, D]. */
TKV_API int tkv_merge_partials(const float* part_ml, const float* part_o, int n_slots, int num_seqs,
                       int num_q_heads, int head_dim, void* out, int out_dtype, void* stream);

/* ---------------------------------------------------------------- */
/* Token-split decode over peer memory (GPUs of one node)             */
/* ---------------------------------------------------------------- */
/* Replaces the all-gather of split-KV partials that a token-split decode
 * needs (the reference's collective plumbing, multi_gpu.cpp:200-230, has no
 * split-KV path): every GPU stores its one-slot partial straight into every
 * peer's exchange buffer over NVLink from the kernel that reduces it, raises
 * a flag there, and merges the slots of all GPUs once their flags are up.
 * No NCCL call and no multicast.
 *
 * Exchange buffer of one GPU (tkv_exchange_buffer_bytes, allocated with
 * tkv_device_alloc so it can be shared, zeroed): a 256-byte header (flags
 * [2][TKV_MAX_PEERS] u32 written by the peers, then this GPU's step and
 * arrival counters) and two parity sets of world x num_seqs x num_q_heads
 * rows of (m, l, pad, pad, o[D]) f32.  Consecutive steps alternate sets, so a
 * GPU may run one step ahead of a peer without overwriting what the peer has
 * not merged yet. */
#define TKV_MAX_PEERS 8
#define TKV_IPC_HANDLE_BYTES 64

typedef struct tkv_exchange {
  int world;                    /* GPUs in the exchange, 1..TKV_MAX_PEERS        */
  int rank;                     /* this GPU's index in [0, world)                 */
  void* buffers[TKV_MAX_PEERS]; /* buffers[r]: GPU r's exchange buffer as mapped
                                   in this process (buffers[rank] = own)          */
} tkv_exchange_t;

TKV_API size_t tkv_exchange_buffer_bytes(int world, int num_seqs, int num_q_heads,
                                         int head_dim);
/* Zeroed device memory that can be shared with other processes
 * (cudaMalloc + cudaMemset), and its release. */
TKV_API int tkv_device_alloc(size_t bytes, void** ptr);
TKV_API int tkv_device_free(void* ptr);
/* CUDA IPC: the TKV_IPC_HANDLE_BYTES handle of an allocation from
 * tkv_device_alloc, opened in another process on the same node (peer access
 * enabled), and closed. */
TKV_API int tkv_ipc_get_handle(const void* ptr, void* handle);
TKV_API int tkv_ipc_open_handle(const void* handle, void** ptr);
TKV_API int tkv_ipc_close_handle(void* ptr);

/* This GPU's share of the token split (the arguments of
 * tkv_paged_decode_range), reduced to one partial per (sequence, q head) and
 * published to every GPU of the exchange.  A GPU whose range is empty
 * (split_hi == split_lo and include_residual == 0) publishes empty partials.
 * Every GPU of the exchange makes the same calls in the same order. */
TKV_API int tkv_exchange_decode_range(const tkv_cache_t* cache, const void* q, int q_dtype,
                                      const int32_t* block_tables, int max_blocks_per_seq,
                                      const int32_t* seq_lens, const int32_t* seq_slots,
                                      int num_seqs, int num_q_heads, float scale, int split_lo,
                                      int split_hi, int include_residual,
                                      const tkv_exchange_t* ex, void* workspace,
                                      size_t workspace_bytes, int* err_flag, void* stream);
/* Waits (bounded: about 2 s, then TKV_ERR_TIMEOUT in *err_flag and a zero
 * output) until every GPU has published this step, merges the world slots by
 * log-sum-exp into out [num_seqs, num_q_heads, head_dim] and advances this
 * GPU's step.  One launch. */
TKV_API int tkv_exchange_merge(const tkv_exchange_t* ex, int num_seqs, int num_q_heads,
                               int head_dim, void* out, int out_dtype, int* err_flag,
                               void* stream);

/* ---------------------------------------------------------------- */
/* Page allocator (host)                                              */
/* ---------------------------------------------------------------- */
/* Replaces the bookkeeping of CudaAllocator
 * (src/inference/backends/cuda/cuda_allocator.{h,cpp}) for the KIVI cache:
 * a free list of page ids (lowest id handed out first,
 * cuda_allocator.cpp:97-99), per-page reference counts for shared pages
 * (copy_sequence, cuda_allocator.cpp:205-217), per-sequence block tables with
 * -1 padding (:231-253), and eviction bookkeeping (:318-380).  One allocator
 * serves every layer: a page id and a ring row name the same slot in each
 * layer's cache, as a block id does across the reference's per-layer pools.
 *
 * Differences the KIVI format brings:
 *   * a sequence of length L holds n_q(L) / 16 pages (whole key groups only);
 *     its n_r most recent tokens live in its ring row, which the allocator
 *     also hands out (one per live sequence, max_seqs rows);
 *   * a page is written once, when its key group is flushed, and never again,
 *     so pages shared by tkv_allocator_fork stay valid for both sequences
 *     without copy-on-write; the fork's ring row must be copied on the device
 *     (tkv_copy_ring_rows) before either sequence appends again;
 *   * the block-table width is a constructor argument (the reference caps it
 *     at 2048 blocks = 32K tokens, cuda_allocator.cpp:76).
 * All functions are thread-safe (one mutex, as cuda_allocator.h:14-16), touch
 * no device memory and never block on the GPU.  Errors: TKV_INVALID_ARGUMENT
 * (unknown / duplicate / evicted sequence, length beyond the table width),
 * TKV_OUT_OF_MEMORY (not enough free pages or ring rows; nothing changes). */
typedef struct tkv_allocator tkv_allocator_t;

typedef struct tkv_allocator_stats {
  int32_t pages_total, pages_used, pages_free, pages_shared; /* shared: refcount > 1 */
  int32_t rows_total, rows_free;
  int32_t sequences, evicted;
  float utilization_pct; /* 100 * pages_used / pages_total (KvCacheStats) */
} tkv_allocator_stats_t;

TKV_API int tkv_allocator_create(const tkv_format_t* fmt, int num_pages, int max_seqs,
                                 int max_blocks_per_seq, tkv_allocator_t** out);
TKV_API void tkv_allocator_destroy(tkv_allocator_t* a);
/* Pages for n_q(len) tokens: the block-table entries a sequence of length len uses. */
TKV_API int tkv_allocator_pages_for(const tkv_allocator_t* a, int len);
/* allocate_sequence (cuda_allocator.cpp:129-158): a ring row plus the pages of
 * a sequence of num_tokens tokens.  *ring_row (may be NULL) gets the row. */
TKV_API int tkv_allocator_add_sequence(tkv_allocator_t* a, uint64_t seq_id, int num_tokens,
                                       int32_t* ring_row);
/* extend_sequence (cuda_allocator.cpp:160-171), by length: makes the table
 * cover new_len tokens (allocating the pages of every key group that the
 * append up to new_len will flush) and records new_len as the length.
 * *n_new (may be NULL) gets the number of pages added. */
TKV_API int tkv_allocator_extend(tkv_allocator_t* a, uint64_t seq_id, int new_len, int* n_new);
/* free_sequence (cuda_allocator.cpp:173-185); unknown ids are a no-op (TKV_OK). */
TKV_API int tkv_allocator_free_sequence(tkv_allocator_t* a, uint64_t seq_id);
/* copy_sequence (cuda_allocator.cpp:187-203): dst shares src's pages
 * (reference counted) and length, and gets a ring row of its own.  The caller
 * copies ring row *src_row to *dst_row in every layer (tkv_copy_ring_rows). */
TKV_API int tkv_allocator_fork(tkv_allocator_t* a, uint64_t src_id, uint64_t dst_id,
                               int32_t* src_row, int32_t* dst_row);
/* Batched get_device_block_table (cuda_allocator.cpp:231-253), filled on the
 * host: block_tables [n][max_blocks_per_seq] (-1 padded), seq_lens [n] and
 * ring rows [n] (either may be NULL) for the sequences seq_ids[0..n). */
TKV_API int tkv_allocator_tables(const tkv_allocator_t* a, const uint64_t* seq_ids, int n,
                                 int32_t* block_tables, int32_t* seq_lens, int32_t* ring_rows);
/* Length, page count, ring row (-1 when evicted) and evicted flag of one sequence. */
TKV_API int tkv_allocator_sequence(const tkv_allocator_t* a, uint64_t seq_id, int* len,
                                   int* n_pages, int32_t* ring_row, int* evicted);
TKV_API int tkv_allocator_stats(const tkv_allocator_t* a, tkv_allocator_stats_t* out);
/* evict_sequence bookkeeping (cuda_allocator.cpp:318-350): writes the
 * sequence's pages (in table order, capacity max_blocks_per_seq) and ring row,
 * then releases them.  The caller moves them to host memory
 * (tkv_swap_pages / tkv_swap_ring_rows) on a stream that orders the copy
 * before any later write to the released pages. */
TKV_API int tkv_allocator_evict(tkv_allocator_t* a, uint64_t seq_id, int32_t* pages,
                                int* n_pages, int32_t* ring_row);
/* reload_sequence bookkeeping (cuda_allocator.cpp:352-378): fresh pages and a
 * ring row for an evicted sequence, written to pages / *ring_row; the caller
 * copies the saved images back.  Out of pages or rows: TKV_OUT_OF_MEMORY and
 * the sequence stays evicted (the reference leaves a partial table). */
TKV_API int tkv_allocator_reload(tkv_allocator_t* a, uint64_t seq_id, int32_t* pages,
                                 int* n_pages, int32_t* ring_row);

/* ---------------------------------------------------------------- */
/* Page and ring-row moves (device)                                   */
/* ---------------------------------------------------------------- */
/* The KIVI format is position independent: a (page, kv head) block holds its
 * codes and meta, a ring row its fp16 tokens, so pages and rows move as bytes.
 * mapping: device int32 [n][2] = {src, dst} index pairs (destinations distinct
 * and not sources of other pairs).  Pairs with an index out of range are
 * skipped and flagged TKV_ERR_BAD_PAGE / TKV_ERR_BAD_SLOT in *err_flag (may be
 * NULL).  One launch each, 16-byte loads and stores. */
/* copy_blocks (cache_kernels.cu:107-127,234-260): pool page -> pool page. */
TKV_API int tkv_copy_pages(const tkv_cache_t* cache, const int32_t* mapping, int n,
                           int* err_flag, void* stream);
/* swap_blocks (cache_kernels.cu:138-168,262-283) for pages: between the pool
 * and `images` [capacity][n_kv_heads][page_bytes] in pinned host memory (or
 * device memory).  direction 0: pool page src -> image dst; 1: image src ->
 * pool page dst.  Host memory that is not page-locked is rejected with
 * TKV_INVALID_ARGUMENT before launching. */
TKV_API int tkv_swap_pages(const tkv_cache_t* cache, void* images, int64_t capacity,
                           const int32_t* mapping, int n, int direction, int* err_flag,
                           void* stream);
/* Ring row -> ring row (the device half of tkv_allocator_fork). */
TKV_API int tkv_copy_ring_rows(const tkv_cache_t* cache, const int32_t* mapping, int n,
                               int* err_flag, void* stream);
/* Ring rows between the ring and `images` [capacity][tkv_ring_bytes(fmt, 1)]
 * bytes, directions as tkv_swap_pages. */
TKV_API int tkv_swap_ring_rows(const tkv_cache_t* cache, void* images, int64_t capacity,
                               const int32_t* mapping, int n, int direction, int* err_flag,
                               void* stream);

/* ---------------------------------------------------------------- */
/* Kernel registry (include/truellm/kernel.h:23-57)                   */
/* ---------------------------------------------------------------- */
#ifndef TRUELLM_KERNEL_ABI_VERSION
#define TRUELLM_KERNEL_ABI_VERSION 1
typedef enum truellm_kernel_category {
  TRUELLM_KERNEL_ATTENTION = 0,
  TRUELLM_KERNEL_ACTIVATION = 1,
  TRUELLM_KERNEL_LAYERNORM = 2,
  TRUELLM_KERNEL_GEMM = 3,
  TRUELLM_KERNEL_CACHE = 4,
  TRUELLM_KERNEL_CUSTOM = 99,
} truellm_kernel_category_t;

typedef struct truellm_kernel_manifest {
  uint32_t abi_version;
  const char* name;
  const char* version;
  truellm_kernel_category_t category;
  uint32_t min_sm_major;
  uint32_t min_sm_minor;
  int (*initialize)(void* engine_ctx);
  void (*shutdown)(void* engine_ctx);
  void* kernel_state;
} truellm_kernel_manifest_t;
#endif

/* The entry point a kernel plugin exports (include/truellm/kernel.h:10-12):
 * the attention manifest of this library. */
TKV_API truellm_kernel_manifest_t* truellm_kernel_init(void);
/* The cache (quantize-on-append) manifest, TRUELLM_KERNEL_CACHE. */
TKV_API truellm_kernel_manifest_t* tkv_cache_kernel_manifest(void);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* TRUELLM_KIVI_H */
