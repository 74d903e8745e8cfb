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

/* Element types: the values of truellm::DataType (include/truellm/types.h:47-53). */
typedef enum tkv_dtype { TKV_F32 = 0, TKV_F16 = 1, TKV_BF16 = 2 } tkv_dtype_t;

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
/* Workspace bytes for tkv_paged_decode: work counters, per-(sequence, kv head)
 * completion counters and the split partials.  Zero the whole workspace once
 * when it is allocated; every call leaves the counters zero again.  Calls that
 * share a workspace must not overlap on the GPU.  Launches with few work items
 * (num_seqs * num_q_heads * splits small: long single sequences, few kv heads)
 * use 128-token splits internally; the size accounts for that. */
TKV_API size_t tkv_decode_workspace_bytes(int num_seqs, int num_q_heads, int head_dim,
                                  int max_context_len);
/* Kernel launches tkv_paged_decode makes for these sizes: 1 (merge fused into
 * the decode launch) or 2 (contexts beyond 64K tokens: a separate
 * slot-parallel merge). */
TKV_API int tkv_decode_launches(int num_seqs, int num_q_heads, int max_context_len);
/* Workspace bytes for tkv_paged_decode_range over splits [split_lo, split_hi)
 * (with the finer internal splits the range may use). */
TKV_API size_t tkv_decode_range_workspace_bytes(int num_seqs, int num_q_heads, int head_dim,
                                                int split_lo, int split_hi);

/* Replaces paged_attention_v1/v2 (cuda_engine.cpp:51-62,
 * paged_attention_v1.cu:177-213, paged_attention_v2.cu:176-251) for the KIVI
 * cache: out[s, h, :] = softmax(scale * q[s,h,:] . K^T) V over the
 * seq_lens[s] tokens of sequence s, kv head = h / (num_q_heads / n_kv_heads)
 * (megakernel.cu:270-277).  q, out: [num_seqs, num_q_heads, D]; q is fp16 or
 * bf16, out is fp16, bf16 or f32.  Split-KV over TKV_SPLIT_TOKENS-token splits
 * plus a log-sum-exp merge (paged_attention_v2.cu:132-170), done by the warp
 * that finishes the last split of each (sequence, kv head): one launch.
 * Contexts beyond 64K tokens merge in a second, slot-parallel launch
 * (tkv_decode_launches). */
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
 * the process exits.  Nothing is allocated.  The first call on a device looks
 * up the array's device address and zeroes the array (stream-ordered on
 * `stream`); make that first call before any stream capture.  Calls whose
 * tkv_decode_workspace_bytes() exceeds the scratch return TKV_OUT_OF_MEMORY
 * without launching.  All calls on a device share the array, so calls that
 * overlap on the GPU race; it keeps the last call's partials. */
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
 * split_lo, split_hi) bytes (a smaller one of at least the 512-token-split
 * size makes the launch keep 512-token splits), 16-byte aligned, zeroed once
 * as for tkv_paged_decode (every call leaves its counters zero).  Two
 * launches. */
TKV_API int tkv_paged_decode_range(const tkv_cache_t* cache, const void* q, int q_dtype,
                                   const int32_t* block_tables, int max_blocks_per_seq,
                                   const int32_t* seq_lens, const int32_t* seq_slots,
                                   int num_seqs, int num_q_heads, float scale, int split_lo,
                                   int split_hi, int include_residual, float* out_ml,
                                   float* out_o, void* workspace, size_t workspace_bytes,
                                   int* err_flag, void* stream);

/* Log-sum-exp merge of n_slots partial sets laid out as above
 * (paged_attention_v2.cu:132-170) into out [num_seqs, num_q_heads, D]. */
TKV_API int tkv_merge_partials(const float* part_ml, const float* part_o, int n_slots, int num_seqs,
                       int num_q_heads, int head_dim, void* out, int out_dtype, void* stream);

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
