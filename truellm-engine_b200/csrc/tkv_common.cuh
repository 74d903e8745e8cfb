// tkv_common.cuh -- shared device helpers for the sm_100a KIVI kernels:
// bulk (TMA 1-D) copies completed on mbarriers with bounded waits, the
// mma.m16n8k16 tensor-core op, code extraction and the reference quantizer's
// arithmetic.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <float.h>
#include <stdint.h>

#include "truellm_kivi.h"  // include/ is on the include path

namespace tkv {

constexpr int kPage = TKV_PAGE_SIZE;
constexpr int kSplitTokens = TKV_SPLIT_TOKENS;
constexpr int kSplitPages = kSplitTokens / kPage;  // 32
// Pages per split for launches whose 512-token items would not give every
// resident warp ~2 items (one long sequence, few kv heads): 128 tokens, a
// multiple of every key group (G <= 128).
constexpr int kFineSplitPages = 8;
static_assert(kSplitPages % kFineSplitPages == 0, "fine splits tile the coarse ones");
// Above this many split slots per sequence (contexts beyond 64K tokens at
// 512-token splits) the merge runs as its own slot-parallel kernel instead of
// in the decode launch's last warp per (sequence, kv head), whose serial merge
// of that many slots would be the launch's tail.
constexpr int kWideMergeSlots = 129;
// A bounded mbarrier wait gives up after this many try_wait polls, each of
// which suspends the thread for at most kSuspendNs while the phase is still
// open (about 2 s in total), then reports TKV_ERR_TIMEOUT instead of
// spinning forever.
constexpr uint32_t kMaxPolls = 2000;
constexpr uint32_t kSuspendNs = 1000000;

__device__ __forceinline__ void set_err(int* err, int bit) {
  if (err) atomicOr(err, bit);
}

// ---------------------------------------------------------------------------
// mbarrier + bulk copy (cp.async.bulk, no multicast)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}

// Returns true when the phase with the given parity has completed.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
      "selp.u32 %0, 1, 0, p;\n"
      "}\n"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendNs)
      : "memory");
  return done != 0;
}

// Bounded wait; on timeout sets TKV_ERR_TIMEOUT and returns false.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
  for (uint32_t i = 0; i < kMaxPolls; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  set_err(err, TKV_ERR_TIMEOUT);
  return false;
}

// Non-blocking check of the phase with the given parity.
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      "selp.u32 %0, 1, 0, p;\n"
      "}\n"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// mbar_wait with a non-blocking first check: a phase that has already
// completed (the common case in a deep enough ring) costs no suspend.
__device__ __forceinline__ bool mbar_wait_fast(uint64_t* bar, uint32_t parity, int* err) {
  return mbar_test(bar, parity) || mbar_wait(bar, parity, err);
}

// 1-D bulk copy global -> shared, completion counted on `bar` (bytes % 16 == 0,
// both addresses 16-byte aligned).
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src_gmem, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
          smem_u32(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Per-thread asynchronous copies global -> shared (cp.async), completed by
// cp_async_wait_all (all of this thread's outstanding copies).
__device__ __forceinline__ void cp_async16(void* dst_smem, const void* src_gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_u32(dst_smem)),
               "l"(src_gmem)
               : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst_smem, const void* src_gmem) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(smem_u32(dst_smem)),
               "l"(src_gmem)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;\n" ::: "memory");
}
// 16-byte cp.async with an L2 cache policy
__device__ __forceinline__ void cp_async16_hint(void* dst_smem, const void* src_gmem,
                                                uint64_t policy) {
  asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;\n" ::"r"(
                   smem_u32(dst_smem)),
               "l"(src_gmem), "l"(policy)
               : "memory");
}
// Arrives on `bar` once every cp.async this thread issued before has landed;
// the arrival is one of the barrier's expected count (.noinc).
__device__ __forceinline__ void cp_async_mbar_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];\n" ::"r"(smem_u32(bar))
               : "memory");
}

// L2 policy for data read once per launch (cache pages): evict it first, so
// lines that are read again soon (split partials) stay in L2.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;\n" : "=l"(pol));
  return pol;
}

// bulk_g2s with an L2 cache policy
__device__ __forceinline__ void bulk_g2s_hint(void* dst_smem, const void* src_gmem,
                                              uint32_t bytes, uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], "
      "[%1], %2, [%3], %4;\n" ::"r"(smem_u32(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// ---------------------------------------------------------------------------
// tensor core: D = A(16x16 f16) * B(16x8 f16) + C (f32), mma.sync m16n8k16
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ float2 unpack_h2(uint32_t u) {
  __half2 h = *reinterpret_cast<__half2*>(&u);
  return __half22float2(h);
}

// (x & mask) | bits as one LOP3.  Keeping both constants in registers lets
// ptxas emit a single LOP3 (SASS LOP3 takes at most one immediate).
__device__ __forceinline__ uint32_t and_or(uint32_t x, uint32_t mask, uint32_t bits) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;\n" : "=r"(r) : "r"(x), "r"(mask), "r"(bits));
  return r;
}

// Codes -> f16 pairs holding 1 + code/16 (exact).  For 4-bit codes the pair is
// the nibbles at bits [s0, s0+4) and [s0+16, s0+20) of w; for 2-bit codes the
// 2-bit fields at the same positions.  SHIFT moves bit s0 to bit 6.
template <int SHIFT>
__device__ __forceinline__ uint32_t ext4(uint32_t w) {
  uint32_t x = SHIFT >= 0 ? (w << SHIFT) : (w >> (-SHIFT));
  return and_or(x, 0x03C003C0u, 0x3C003C00u);
}
template <int SHIFT>
__device__ __forceinline__ uint32_t ext2(uint32_t w) {
  uint32_t x = SHIFT >= 0 ? (w << SHIFT) : (w >> (-SHIFT));
  return and_or(x, 0x00C000C0u, 0x3C003C00u);
}

// Codes -> exact integer-valued f16 pairs.  lop3 ORs the masked code bits
// into the mantissa of 1024.0 (0x6400), giving 1024 + c * 2^k; one HFMA2 by
// (2^-k, -1024 * 2^-k) then yields c exactly.  MASK selects the code pair.
template <uint32_t MASK>
__device__ __forceinline__ uint32_t code_pair(uint32_t w) {
  constexpr uint32_t lo = MASK & 0xffffu;
  constexpr int k = lo == 0x000fu || lo == 0x0003u ? 0 : lo == 0x000cu ? 2 : lo == 0x00f0u || lo == 0x0030u ? 4 : 6;
  constexpr uint32_t mul = k == 0 ? 0x3C003C00u : k == 2 ? 0x34003400u : k == 4 ? 0x2C002C00u : 0x24002400u;
  constexpr uint32_t add = k == 0 ? 0xE400E400u : k == 2 ? 0xDC00DC00u : k == 4 ? 0xD400D400u : 0xCC00CC00u;
  uint32_t x = and_or(w, MASK, 0x64006400u);
  uint32_t r;
  asm("fma.rn.f16x2 %0, %1, %2, %3;\n" : "=r"(r) : "r"(x), "r"(mul), "r"(add));
  return r;
}

// fp16x2 fused multiply-add, round to nearest even: d = a * b + c.
__device__ __forceinline__ uint32_t hfma2(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;\n" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// 2^x with the hardware approximation (ex2.approx, relative error ~2^-22;
// 2^-inf = +0).  Used for softmax weights and LSE merge factors.
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}

// ---------------------------------------------------------------------------
// reference quantizer arithmetic (kivi_cache.cu:92-124), IEEE ops spelled out
// so no contraction or fast-math can change a bit.
// ---------------------------------------------------------------------------
struct QParams {
  float gmin;
  float scale;  // qmax / range, or 0 when degenerate
  uint16_t hstep, hzero;
};

__device__ __forceinline__ QParams quant_params(float gmin, float gmax, int qmax) {
  QParams p;
  float range = __fsub_rn(gmax, gmin);
  bool degenerate = !(range > 1e-6f);
  p.scale = degenerate ? 0.f : __fdiv_rn(static_cast<float>(qmax), range);
  float step = degenerate ? 0.f : __fdiv_rn(1.f, p.scale);
  bool gmin_ok = (gmin == gmin) && (gmin > -FLT_MAX) && (gmin < FLT_MAX);
  p.gmin = gmin;
  __half hs = __float2half_rn(step);
  __half hz = __float2half_rn(gmin_ok ? gmin : 0.f);
  p.hstep = *reinterpret_cast<uint16_t*>(&hs);
  p.hzero = *reinterpret_cast<uint16_t*>(&hz);
  return p;
}

__device__ __forceinline__ int quant_code(float x, const QParams& p, int qmax) {
  int q = __float2int_rn(__fmul_rn(__fsub_rn(x, p.gmin), p.scale));
  q = q < 0 ? 0 : q;
  return q > qmax ? qmax : q;
}

// ---------------------------------------------------------------------------
// kernel argument blocks (filled by tkv_api.cu)
// ---------------------------------------------------------------------------
struct AppendArgs {
  uint8_t* pool;
  uint16_t* ring;
  int num_pages, max_seqs, n_kv_heads, head_dim, group, residual, bits, ring_cap, n_vgroups;
  int k_codes_off, v_codes_off, v_meta_off, k_meta_off, k_meta_slice;
  int64_t page_bytes;
  const void* k_new;
  const void* v_new;
  bool in_bf16;
  const int32_t* cu_new;
  const int32_t* lens_old;
  const int32_t* block_tables;
  int max_blocks;
  const int32_t* seq_slots;
  int total_new;  // rows in k_new / v_new
  int max_new;
  int* err;
};

struct DecodeArgs {
  const uint8_t* pool;
  const uint16_t* ring;
  int num_pages, max_seqs, n_kv_heads, group, residual, ring_cap;
  int k_codes_off, v_codes_off, v_meta_off, k_meta_off, k_meta_slice;
  int64_t page_bytes;
  const void* q;
  bool q_bf16;
  const int32_t* block_tables;
  int max_blocks;
  const int32_t* seq_lens;
  const int32_t* seq_slots;
  int num_seqs, num_q_heads, grp;
  float alpha;  // scale * log2(e)
  int split_lo, split_hi, include_residual, n_slots;  // splits of split_pages pages
  int split_pages;          // kSplitPages, or kFineSplitPages for launches with few items
  int n_items;              // n_slots * num_seqs * n_kv_heads
  unsigned int* work;       // [0] next work item, [1] finished warps; zero between launches
  unsigned int* bh_count;   // [num_seqs * n_kv_heads] finished slots; zero between launches
  int fuse_merge;           // 1: the warp finishing a (sequence, kv head) merges it into out
  void* out;                // [num_seqs, num_q_heads, D] when fuse_merge
  int out_dtype;
  float* part_ml;
  float* part_o;
  int* err;
};

struct PrefillArgs {
  const uint8_t* pool;
  const uint16_t* ring;
  int num_pages, max_seqs, n_kv_heads, residual, ring_cap;
  const void* q;
  bool q_bf16;
  void* out;
  int out_dtype;
  const int32_t* cu_q;
  const int32_t* block_tables;
  int max_blocks;
  const int32_t* seq_lens;
  const int32_t* seq_slots;
  int num_seqs, num_q_heads, grp, total_q;
  int max_q;    // bound on the query tokens of one sequence
  int n_rt;     // query-row tiles per (sequence, kv head), set by the launcher
  float alpha;  // scale * log2(e)
  int* err;
};

// Balanced ("stream") decode: see tkv_stream.cu.
constexpr int kStreamFused = 0;     // the last warp of each pair merges into out
constexpr int kStreamPartials = 1;  // partials + pair_info; stream_merge_kernel merges

struct StreamArgs {
  const uint8_t* pool;
  const uint16_t* ring;
  int num_pages, max_seqs, n_kv_heads, residual, ring_cap;
  const void* q;
  int q_bf16;
  const int32_t* block_tables;
  int max_blocks;
  const int32_t* seq_lens;
  const int32_t* seq_slots;
  int num_seqs, num_q_heads, grp;
  int max_len;           // longer sequences are flagged TKV_ERR_BAD_LENGTH
  float alpha;           // scale * log2(e)
  int pg_lo, pg_hi;      // quantised pages [pg_lo, pg_hi) of every sequence
  int include_residual;  // 1: the fp16 residual tokens too
  int n_warps;           // warps launched (bounded by the workspace's partial slots)
  int warp_smem;         // shared memory bytes of one warp
  int mode;              // kStreamFused or kStreamPartials
  unsigned int* pair_count;  // [num_seqs * n_kv_heads], zero between launches (fused)
  int2* pair_info;           // [num_seqs * n_kv_heads] (first slot, slots) (partials)
  float* part_ml;            // [slots][grp][2]  (m in log2 units, l)
  float* part_o;             // [slots][grp][D]
  void* out;                 // fused: [num_seqs, num_q_heads, D] in out_dtype
  int out_dtype;
  int* err;
};

// Token-split exchange over peer memory (tkv_exchange.cu).  Exchange buffer
// of one GPU: [header 256 B: u32 flags[2][kMaxPeers] (flags[s][r] = step + 1
// once GPU r has published step `step` of parity s), u32 counters at
// kExStateOff: step, publish arrivals, merge arrivals][set 0][set 1]; a set
// holds world x rows rows of kExRowPad + D floats: (m log2, l, -, -, o[D]).
constexpr int kMaxPeers = 8;
constexpr int kExHeader = 256;
constexpr int kExStateOff = 128;
constexpr int kExRowPad = 4;
struct ExPub {
  float* set0[kMaxPeers];      // each GPU's set 0 (its buffer + kExHeader), mapped here
  uint32_t* flags[kMaxPeers];  // each GPU's flags[2][kMaxPeers]
  uint32_t* state;             // this GPU's counters: [0] step, [1] publish and [2] merge arrivals
  int world, rank, rows, rs;   // rows = num_seqs * num_q_heads; rs = kExRowPad + D floats
  long long set_floats;        // world * rows * rs
};

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
  return t;
}

// Stores the reduced row (M, L, O) of row i0 into slot `rank` of every GPU's
// set (step parity) -- called by all threads of a CTA for their channels --
// then counts the CTA; the last CTA of the launch raises this GPU's flag on
// every GPU.  `step` is the exchange step read at kernel start.
__device__ __forceinline__ void ex_store_row(const ExPub& x, uint32_t step, int64_t i0, int c,
                                             float o) {
  const long long off = (step & 1u) * x.set_floats + (static_cast<long long>(x.rank) * x.rows + i0) * x.rs;
  for (int r = 0; r < x.world; ++r) x.set0[r][off + kExRowPad + c] = o;
}
__device__ __forceinline__ void ex_store_ml(const ExPub& x, uint32_t step, int64_t i0, float m,
                                            float l) {
  const long long off = (step & 1u) * x.set_floats + (static_cast<long long>(x.rank) * x.rows + i0) * x.rs;
  for (int r = 0; r < x.world; ++r) {
    x.set0[r][off] = m;
    x.set0[r][off + 1] = l;
  }
}
__device__ __forceinline__ void ex_signal(const ExPub& x, uint32_t step) {
  // the barrier orders the CTA's peer stores before thread 0's system fence
  // (fences are cumulative), which orders them before the CTA's arrival
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const unsigned int n = gridDim.x * gridDim.y;
    if (atomicAdd(&x.state[1], 1u) == n - 1) {
      x.state[1] = 0u;
      __threadfence_system();  // every CTA's stores (ordered by their fences) before the flags
      for (int r = 0; r < x.world; ++r)
        st_release_sys(&x.flags[r][(step & 1u) * kMaxPeers + x.rank], step + 1u);
    }
  }
}

// Workspace of the stream decode for these sizes (the query functions' value).
size_t stream_workspace_bytes(int num_seqs, int num_q_heads, int head_dim);
// Launches the stream decode: fused (one launch) or partials + merge (two
// launches; out_ml != nullptr: the merge writes unnormalised (M, L) and O;
// pub != nullptr: the merge publishes them to the exchange instead).
int launch_stream_decode(StreamArgs a, int head_dim, int bits, int group, void* workspace,
                         size_t workspace_bytes, float* out_ml, cudaStream_t stream,
                         const ExPub* pub = nullptr);
// 1 or 2: the launches tkv_paged_decode makes for these sizes.
int stream_decode_launches(int num_seqs, int num_kv_heads);
// tkv_exchange.cu: empty partials of a GPU without splits; the wait + merge.
int launch_ex_publish_empty(const ExPub& pub, int head_dim, cudaStream_t stream);
int launch_ex_merge(const ExPub& pub, int head_dim, void* out, int out_dtype, int* err,
                    cudaStream_t stream);

int launch_ref_kivi(int mode, const void* in, void* out, int n_vecs, int head_dim, int n_outliers,
                    int group_size, cudaStream_t stream);
int launch_append(const AppendArgs& a, int num_seqs, cudaStream_t stream);
int launch_decode_splits(DecodeArgs a, int head_dim, int bits, int n_vgroups, cudaStream_t stream);
int launch_reduce(const float* part_ml, const float* part_o, int n_slots, int num_seqs,
                  int num_q_heads, int head_dim, float* out_ml, float* out_o, cudaStream_t stream);
int launch_prefill(const PrefillArgs& a, int head_dim, int bits, int group, cudaStream_t stream);
int launch_merge(const float* part_ml, const float* part_o, int n_slots, int num_seqs,
                 int num_q_heads, int head_dim, void* out, int out_dtype, cudaStream_t stream);

}  // namespace tkv
