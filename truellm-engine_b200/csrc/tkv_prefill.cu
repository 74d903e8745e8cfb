// tkv_prefill.cu -- chunked-prefill attention over the paged KIVI cache on sm_100a.
//
// The reference's prefill (src/inference/backends/cuda/cuda_engine.cpp:842-860)
// runs its attention token by token; here a chunk of new tokens, already
// appended to the cache, attends to the whole cached history in one launch.
// Query row (token i of sequence b's n_b-token chunk, q head) sits at position
// p = seq_lens[b] - n_b + i and attends causally to tokens [0, p], read where
// the cache holds them: pages below n_q, the fp16 ring above.  Attention math
// as the megakernel (third_party/custom_kernels/megakernel.cu:267-350):
// score = scale * q.k, kv head = q head / (Hq/Hkv), max-subtracted softmax,
// fp32 accumulation.
//
// The query rows of one (sequence, kv head) are rho = i * grp + j (token i,
// q head j of the kv head's group), so the grp q heads of a kv head share
// every dequantised page.  Keys and values are dequantised exactly, to the
// fp16 values the reference decompress writes, fp16(code * step + zero) for
// keys (per channel) and values (per token), and the contractions run on the
// 5th-generation tensor cores (tcgen05.mma, operands in shared memory, S and
// O accumulators in tensor memory); prefill_umma_kernel below describes the
// pipeline.  Key channels sit in the operand in the order a code word unpacks
// into f16 pairs ((c, c+4) for 4-bit words, (c, c+8) for 2-bit), and Q is
// staged in the same order; ring tiles (the fp16 window) are scattered into
// that order.
#include <atomic>

#include "tkv_frag.cuh"
#include "tkv_umma.cuh"

namespace tkv {

constexpr int kMaxPrefillDevices = 64;

namespace {

__device__ __forceinline__ float load_qv(const PrefillArgs& a, int64_t idx) {
  if (a.q_bf16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(a.q)[idx]);
  return __half2float(reinterpret_cast<const __half*>(a.q)[idx]);
}

// value_frag() registers hold 1024 + c (tokens 2tig, 2tig+1) and 64 + c
// (tokens 2tig+8, 2tig+9) for 4-bit codes, 1 + c/16 for 2-bit codes; one
// HFMA2 with these f16x2 constants recovers the integer codes exactly.
template <int BITS> struct VCode;
template <> struct VCode<4> {
  static constexpr uint32_t kMul = 0x3C003C00u, kAddLo = 0xE400E400u, kAddHi = 0xD400D400u;
};
template <> struct VCode<2> {
  static constexpr uint32_t kMul = 0x4C004C00u, kAddLo = 0xCC00CC00u, kAddHi = 0xCC00CC00u;
};

}  // namespace

namespace {

// Position of key channel c in the shared K tile (inverse of the unpack order).
template <int BITS>
__device__ __forceinline__ constexpr int kpos(int c) {
  return BITS == 4 ? (c & ~7) + 2 * (c & 3) + ((c >> 2) & 1)
                   : (c & ~15) + 2 * (c & 7) + ((c >> 3) & 1);
}
// Key channel at position p of the shared K tile.
template <int BITS>
__device__ __forceinline__ constexpr int kchan_at(int p) {
  return BITS == 4 ? (p & ~7) + ((p & 7) >> 1) + 4 * (p & 1)
                   : (p & ~15) + ((p & 15) >> 1) + 8 * (p & 1);
}

}  // namespace

// ---------------------------------------------------------------------------
// Chunked prefill on the 5th-generation tensor cores (tcgen05): one CTA of
// two warpgroups per 256 query rows of a (sequence, kv head), each warpgroup
// owning 128 rows (the MMA's M) and its own S and O in tensor memory; 64-token
// KV tiles shared by both.  Per tile the CTA's threads dequantise the tile's
// four 16-token pages (or fp16 ring chunks) exactly straight into the K-major
// shared-memory operand layouts of tkv_umma.cuh: K [64 tokens][D channels]
// (channels in the code-unpack order, Q staged in the same order) and V^T
// [D channels][64 tokens].  One thread issues S = Q K^T (D/16 MMAs, N = 64)
// into tensor memory; each thread then owns one query row: it loads the row's
// 64 scores with tcgen05.ld, masks them causally, runs the online softmax
// (exp2 domain, lazy rescale: when a warp's running maxima move, its rows of O
// are rescaled in tensor memory) and writes the row's weights P as f16 pairs
// into tensor memory over the scores it has read (tcgen05.st, 32 columns);
// O += P V (4 MMAs, N = D) then takes its A operand from tensor memory.  Software pipeline: while tile j's softmax runs,
// S of tile j+1 is on the tensor cores (its K already dequantised), and
// O += P V of tile j runs while tile j+1's successor is dequantised; the next
// tile's code words are loaded into registers one tile ahead.  Tensor memory
// per warpgroup (256 columns): S of even and odd tiles in [0, 128) (P_j over
// the first 32 columns of S_j's buffer), O in [128, 128 + D).  S_{j+2} reuses
// S_j's buffer only after O += P_j V_j of both warpgroups is done.
// ---------------------------------------------------------------------------
// Lazy rescale of the tcgen05 prefill: a row's running maximum (log2 units)
// moves only when a tile's maximum exceeds it by more than this, so the O
// rescale in tensor memory (a read and a write of the row's D columns) is
// rare.  The weights written to the f16 P operand are then at most 2^8 = 256,
// well inside the f16 range, and f16 keeps the same relative precision at any
// magnitude.
constexpr float kPrefillLazyLog2 = 8.0f;
constexpr int kUmmaRows = 128;  // query rows per softmax warpgroup (the MMA's M)
constexpr int kUmmaWG = 2;      // softmax warpgroups per CTA
constexpr int kUmmaTN = 64;     // tokens per KV tile
constexpr int kUmmaSoftmax = 128 * kUmmaWG;  // softmax threads: one query row each
constexpr int kUmmaProducers = 256;          // dequantising (producer) threads
constexpr int kUmmaCtaThreads = kUmmaSoftmax + kUmmaProducers + 32;  // + the MMA warp
// named barriers: 1, 2 the softmax warpgroups (0 is __syncthreads)
constexpr int kBarSoftmax = 1;

// Named-barrier AND over `nthreads` threads (whole warps) of barrier `id`.
__device__ __forceinline__ bool bar_and(int id, int nthreads, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 q, %1, 0;\n\t"
      "bar.red.and.pred p, %2, %3, q;\n\tselp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(v)), "r"(id), "r"(nthreads)
      : "memory");
  return r != 0;
}

template <int D>
struct UmmaSmem {
  // K and V triple-buffered: the producers dequantise up to two tiles ahead
  // of the softmax (P lives in tensor memory)
  static constexpr int K_BYTES = kUmmaTN * D * 2, V_BYTES = D * kUmmaTN * 2;
  static constexpr int Q_BYTES = kUmmaRows * D * 2;
  static constexpr int Q_OFF = 0;  // one Q operand per warpgroup
  static constexpr int K_OFF = Q_OFF + kUmmaWG * Q_BYTES;
  static constexpr int V_OFF = K_OFF + 3 * K_BYTES;
  static constexpr int BAR_OFF = V_OFF + 3 * V_BYTES;
  static constexpr int BYTES = BAR_OFF + 256;
  // tensor memory: per warpgroup 256 columns, S of even and odd tiles, then O
  static constexpr uint32_t TWG = 256, TCOLS = 512;
  static_assert(2 * kUmmaTN + D <= TWG, "a warpgroup's S and O fit its columns");
  static_assert(BYTES <= (1 << 18), "descriptor address fields (addr >> 4, 14 bits) never carry");
};

template <int D, int BITS, int G>
__global__ void __launch_bounds__(kUmmaCtaThreads, 1) prefill_umma_kernel(PrefillArgs a) {
  using F = Fmt<D, BITS, G>;
  using SM = UmmaSmem<D>;
  constexpr int NT = kUmmaProducers, TN = kUmmaTN, NSUB = TN / kPage;
  constexpr int WPR = D * BITS / 32;          // key-code words per token row
  constexpr int CPW = 32 / BITS;              // channels per key word
  constexpr int HP = CPW / 2;                 // f16 pairs per key word
  constexpr int KW = kPage * WPR;             // key (and value) code words per page
  constexpr int KPT = (KW + NT - 1) / NT;     // code words per thread
  constexpr int MVEC = CPW / 4;               // 16-byte key-meta vectors per word's channels
  constexpr int VMW = BITS == 4 ? 4 : 8;      // value (step, zero) words per value word
  constexpr int RV = 2 * D;                   // 16-byte vectors per ring K (or V) block
  constexpr int RPT = (RV + NT - 1) / NT;
  constexpr int PSLOT = KPT * (2 + VMW), RSLOT = RPT * 8;
  constexpr int SLOT = PSLOT > RSLOT ? PSLOT : RSLOT;  // registers of one 16-token sub-tile
  // key groups of one tile: sub-tile s uses key meta km[s / PPG] (G < 64) or km[0]
  constexpr int NKM = F::PPG >= NSUB ? 1 : NSUB / F::PPG;
  static_assert(F::PPG % NSUB == 0 || NSUB % F::PPG == 0, "tiles and key groups nest");
  static_assert(NT % WPR == 0, "a thread's key words share their channels");
  static_assert(KPT * NT == KW || KW < NT, "code words per thread");
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* const Qs = smem + SM::Q_OFF;
  uint8_t* const Ks = smem + SM::K_OFF;
  uint8_t* const Vs = smem + SM::V_OFF;
  // Pipeline barriers (tile j uses parity class j % 2 or j % 3, phase j / 2 or j / 3):
  //   sdone[b]     S_j = Q K_j^T of both softmax warpgroups done (commit)
  //   odone[w][b]  warpgroup w's O += P_j V_j done (commit)
  //   vfree[v]     both warpgroups' O += P_j V_j done (2 commits)
  //   pready[w][b] warpgroup w's P_j written to tensor memory (128 arrivals)
  //   tready[v]    K_j and V_j stored (256 producer arrivals)
  //   kfree[v]     S_j done: K buffer j % 3 may be overwritten (commit)
  uint64_t* const bars = reinterpret_cast<uint64_t*>(smem + SM::BAR_OFF);
  uint64_t* const sdone = bars;
  uint64_t* const odone = bars + 2;   // [w * 2 + b]
  uint64_t* const vfree = bars + 6;
  uint64_t* const pready = bars + 9;  // [w * 2 + b]
  uint64_t* const tready = bars + 13;
  uint64_t* const kfree = bars + 16;
  uint32_t* const tslot = reinterpret_cast<uint32_t*>(bars + 19);
  const int ctid = threadIdx.x, warp = ctid >> 5;
  const int wg = ctid >> 7, wt = ctid & 127;  // warpgroup, row in the warpgroup (softmax)
  const bool producer = ctid >= kUmmaSoftmax && ctid < kUmmaSoftmax + kUmmaProducers;
  const bool mma_warp = ctid >= kUmmaSoftmax + kUmmaProducers;

  const int64_t bid = blockIdx.x;
  const int rt = a.n_rt - 1 - (int)(bid % a.n_rt);
  const int bh = (int)(bid / a.n_rt);
  const int b = bh / a.n_kv_heads, h = bh - b * a.n_kv_heads;
  const int L = a.seq_lens[b];
  const int q0 = a.cu_q[b], n = a.cu_q[b + 1] - q0;
  if (L < 0 || L > a.max_blocks * kPage || n < 0 || n > L || n > a.max_q || q0 < 0 ||
      q0 + n > a.total_q) {
    if (rt == 0 && h == 0 && ctid == 0) set_err(a.err, TKV_ERR_BAD_LENGTH);
    return;
  }
  const int rows = n * a.grp, r0 = rt * kUmmaSoftmax;
  if (r0 >= rows) return;
  const int rho = r0 + ctid;
  const bool valid = ctid < kUmmaSoftmax && rho < rows;
  const int qi = valid ? rho / a.grp : 0;
  const int plim = valid ? L - n + qi : -1;  // causal limit of this thread's row
  const int kv_end = L - n + min(rows - 1, r0 + kUmmaSoftmax - 1) / a.grp + 1;
  const int64_t qrow = ((int64_t)(q0 + qi) * a.num_q_heads + h * a.grp + (valid ? rho % a.grp : 0)) * D;
  const int nq = nq_len(L, a.residual, G);
  const int32_t* bt = a.block_tables + (int64_t)b * a.max_blocks;
  const int n_pages = min(nq, (kv_end + kPage - 1) / kPage * kPage) / kPage;
  const int n_chunks = kv_end > nq ? (kv_end - nq + kPage - 1) / kPage : 0;
  const int n16 = n_pages + n_chunks;
  const int n_tiles = (n16 + NSUB - 1) / NSUB;

  const int n_read = min(nq / kPage, (n_pages + F::PPG - 1) / F::PPG * F::PPG);
  bool bad = false;
  for (int p = ctid; p < n_read; p += kUmmaCtaThreads) {
    const int ph = bt[p];
    bad |= ph < 0 || ph >= a.num_pages;
  }
  if (__syncthreads_or(bad)) {
    if (ctid == 0) set_err(a.err, TKV_ERR_BAD_PAGE);
    return;
  }
  int row = 0;
  if (n_chunks > 0) {
    row = a.seq_slots ? a.seq_slots[b] : b;
    if (row < 0 || row >= a.max_seqs) {
      if (ctid == 0) set_err(a.err, TKV_ERR_BAD_SLOT);
      return;
    }
  }

  // ---- tensor memory, barriers, the Q operand (softmax threads: one row each) ----
  if (warp == 0) umma::alloc(tslot, SM::TCOLS);
  if (ctid == 0) {
    for (int i = 0; i < 6; ++i) mbar_init(&bars[i], 1);                 // sdone, odone
    for (int i = 6; i < 9; ++i) mbar_init(&bars[i], 2);                 // vfree
    for (int i = 9; i < 13; ++i) mbar_init(&bars[i], kUmmaRows);        // pready
    for (int i = 13; i < 16; ++i) mbar_init(&bars[i], kUmmaProducers);  // tready
    for (int i = 16; i < 19; ++i) mbar_init(&bars[i], 1);               // kfree
    fence_mbar_init();
  }
  if (ctid < kUmmaSoftmax) {
#pragma unroll
    for (int k8 = 0; k8 < D; k8 += 8) {
      uint32_t w[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int c0 = kchan_at<BITS>(k8 + 2 * e), c1 = kchan_at<BITS>(k8 + 2 * e + 1);
        w[e] = pack_h2(valid ? load_qv(a, qrow + c0) : 0.f, valid ? load_qv(a, qrow + c1) : 0.f);
      }
      *reinterpret_cast<uint4*>(Qs + wg * SM::Q_BYTES + umma::umma_off(wt, k8, D)) =
          make_uint4(w[0], w[1], w[2], w[3]);
    }
    umma::fence_smem_to_async();
  }
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tmem = *tslot;
  constexpr uint32_t idS = umma::idesc_f16(kUmmaRows, TN, false);
  constexpr uint32_t idO = umma::idesc_f16(kUmmaRows, D, false);
  bool ok = true;

  if (producer) {
    // ======================= producer warpgroups =======================
    const int tid = ctid - kUmmaSoftmax;  // 0 .. NT-1
    const uint8_t* pool_h = a.pool + (int64_t)h * F::PB;
    const int64_t page_stride = (int64_t)a.n_kv_heads * F::PB;
    constexpr int CHUNK = 2 * F::RBLK;
    const uint8_t* ring_base =
        reinterpret_cast<const uint8_t*>(a.ring) +
        (((int64_t)row * a.n_kv_heads + h) * (a.ring_cap / kPage)) * CHUNK;
    // Key code words are taken token-fastest: thread tid holds word column
    // tid / 16 (channels kc0.. in tile order) of token tid % 16 of a page, so
    // the 16-byte stores of 8 consecutive lanes fill one 128-byte core matrix
    // of the K operand (no bank conflicts).
    static_assert(KW <= NT, "one key word per thread and page");
    const int kc0 = (tid / kPage) * CPW;
    // this thread's store offsets in the operand tiles (sub-tile, half and
    // neighbour offsets are compile-time): its key word (token tid % 16,
    // channels kc0..), its value word's first (channel, token) pair
    const uint32_t k_off = umma::umma_off(tid % kPage, tid < KW ? kc0 : 0, D);
    const uint32_t v_off = umma::umma_off(16 * (BITS == 4 ? (tid >> 5) : 2 * (tid >> 5)) + ((tid & 31) >> 2),
                                          2 * (tid & 3), TN);
    // ---- registers of the next tile: NSUB sub-tiles of code words or ring vectors ----
    uint32_t reg[NSUB][SLOT];
    uint4 km[NKM][MVEC];
    uint4 kml[MVEC];  // key meta of the group the previous tile ended in
  #pragma unroll
    for (int v = 0; v < MVEC; ++v) kml[v] = make_uint4(0, 0, 0, 0);
    // page ids of the next tile load_tile reads, and of the pages holding this
    // thread's key meta for the key groups starting in it: loaded one call
    // ahead, so the code-word loads never wait on a block-table load
    int pid_n[NSUB], mid_n[NKM][MVEC];
    auto fetch_ids = [&](int jt) {
  #pragma unroll
      for (int s = 0; s < NSUB; ++s) {
        const int j = jt * NSUB + s;
        pid_n[s] = j < n_pages ? bt[j] : 0;
      }
  #pragma unroll
      for (int g = 0; g < NKM; ++g) {
        const int j = jt * NSUB + (F::PPG >= NSUB ? 0 : g * F::PPG);
        // threads without a key word (tid >= KW) have kc0 >= D: they fetch no meta
        const bool starts = tid < KW && j < n_pages && j % F::PPG == 0;
  #pragma unroll
        for (int v = 0; v < MVEC; ++v)
          mid_n[g][v] = starts ? bt[j + (4 * (kc0 + 4 * v)) / F::KMS] : 0;
      }
    };
    fetch_ids(0);
    auto load_tile = [&](int jt) {
      int pid[NSUB], mid[NKM][MVEC];
  #pragma unroll
      for (int s = 0; s < NSUB; ++s) pid[s] = pid_n[s];
  #pragma unroll
      for (int g = 0; g < NKM; ++g)
  #pragma unroll
        for (int v = 0; v < MVEC; ++v) mid[g][v] = mid_n[g][v];
      fetch_ids(jt + 1);
  #pragma unroll
      for (int s = 0; s < NSUB; ++s) {
        const int j = jt * NSUB + s;
        if (j < n_pages) {
          const uint8_t* pg = pool_h + (int64_t)pid[s] * page_stride;
  #pragma unroll
          for (int k = 0; k < KPT; ++k) {
            const int u = tid + k * NT;
            if (u >= KW) continue;
            reg[s][k * (2 + VMW)] =
                __ldg(reinterpret_cast<const uint32_t*>(pg) + (u % kPage) * WPR + u / kPage);
            const int l = u & 31, w = u >> 5;
            reg[s][k * (2 + VMW) + 1] = __ldg(reinterpret_cast<const uint32_t*>(
                pg + F::V_CODES_OFF + ((w / F::VW) * 32 + l) * 4 * F::VW + (w % F::VW) * 4));
            const uint32_t* vmp = reinterpret_cast<const uint32_t*>(pg + F::V_META_OFF);
            const int t0 = 2 * (l & 3);
            if constexpr (F::NVG == 1) {
              // one value group per token: (step, zero) of tokens t0, t0+1 and
              // t0+8, t0+9 as two 8-byte loads (the same for both 2-bit halves)
              const uint2 m0 = __ldg(reinterpret_cast<const uint2*>(vmp + t0));
              const uint2 m1 = __ldg(reinterpret_cast<const uint2*>(vmp + t0 + 8));
  #pragma unroll
              for (int x = 0; x < VMW; x += 4) {
                reg[s][k * (2 + VMW) + 2 + x] = m0.x;
                reg[s][k * (2 + VMW) + 3 + x] = m0.y;
                reg[s][k * (2 + VMW) + 4 + x] = m1.x;
                reg[s][k * (2 + VMW) + 5 + x] = m1.y;
              }
            } else {
  #pragma unroll
              for (int x = 0; x < VMW; ++x) {
                const int mb = BITS == 4 ? w : 2 * w + (x >> 2);
                const int t = t0 + (x & 1) + 8 * ((x >> 1) & 1);
                reg[s][k * (2 + VMW) + 2 + x] = __ldg(vmp + t * F::NVG + (16 * mb) / G);
              }
            }
          }
          const int ki = F::PPG >= NSUB ? 0 : s / (F::PPG >= NSUB ? 1 : F::PPG);
          if (j % F::PPG == 0 && tid < KW) {  // a new key group: this thread's channels
  #pragma unroll
            for (int v = 0; v < MVEC; ++v) {
              const int off = 4 * (kc0 + 4 * v);
              km[ki][v] = __ldg(reinterpret_cast<const uint4*>(
                  pool_h + (int64_t)mid[ki][v] * page_stride + F::BODY + off % F::KMS));
            }
          } else if (s == 0) {  // the group the previous tile ended in
  #pragma unroll
            for (int v = 0; v < MVEC; ++v) km[0][v] = kml[v];
          }
        } else if (j < n16) {
          const int t0 = nq + (j - n_pages) * kPage;
          const uint8_t* ck = ring_base + (int64_t)((t0 % a.ring_cap) / kPage) * CHUNK;
  #pragma unroll
          for (int k = 0; k < RPT; ++k) {
            const int u = tid + k * NT;
            if (u >= RV) continue;
            const uint4 x = __ldg(reinterpret_cast<const uint4*>(ck) + u);
            const uint4 y = __ldg(reinterpret_cast<const uint4*>(ck + F::RBLK) + u);
            reg[s][8 * k + 0] = x.x; reg[s][8 * k + 1] = x.y; reg[s][8 * k + 2] = x.z; reg[s][8 * k + 3] = x.w;
            reg[s][8 * k + 4] = y.x; reg[s][8 * k + 5] = y.y; reg[s][8 * k + 6] = y.z; reg[s][8 * k + 7] = y.w;
          }
        }
      }
  #pragma unroll
      for (int v = 0; v < MVEC; ++v) kml[v] = km[NKM - 1][v];
    };

    // dequantise the registers of tile jt into the K and V^T operand tiles
    auto store_tile = [&](int jt, uint8_t* kd, uint8_t* vd) {
      // the (step, zero) f16 pairs of this thread's key channels, once per key
      // group of the tile (not per 16-token page)
      uint32_t spk[NKM][HP], zpk[NKM][HP];
  #pragma unroll
      for (int ki = 0; ki < NKM; ++ki) {
        uint32_t mw[CPW];
  #pragma unroll
        for (int v = 0; v < MVEC; ++v) {
          mw[4 * v + 0] = km[ki][v].x; mw[4 * v + 1] = km[ki][v].y;
          mw[4 * v + 2] = km[ki][v].z; mw[4 * v + 3] = km[ki][v].w;
        }
  #pragma unroll
        for (int i = 0; i < HP; ++i) {
          spk[ki][i] = __byte_perm(mw[i], mw[i + HP], 0x5410);
          zpk[ki][i] = __byte_perm(mw[i], mw[i + HP], 0x7632);
        }
      }
  #pragma unroll
      for (int s = 0; s < NSUB; ++s) {
        const int j = jt * NSUB + s;
        const int tb = s * kPage;  // the sub-tile's first token in the tile
        if (j < n_pages) {
          const int ki = F::PPG >= NSUB ? 0 : s / (F::PPG >= NSUB ? 1 : F::PPG);
          const uint32_t(&sp)[HP] = spk[ki];
          const uint32_t(&zp)[HP] = zpk[ki];
  #pragma unroll
          for (int k = 0; k < KPT; ++k) {
            const int u = tid + k * NT;
            if (u >= KW) continue;
            const uint32_t x = reg[s][k * (2 + VMW)], x8 = x >> 8;
            uint32_t hv[HP];
  #pragma unroll
            for (int i = 0; i < HP; ++i) {
              uint32_t c;
              if (BITS == 4) {
                c = (i & 1) ? code_pair<0x00F000F0u>(i < 2 ? x : x8)
                            : code_pair<0x000F000Fu>(i < 2 ? x : x8);
              } else {
                const uint32_t y = i < 4 ? x : x8;
                c = (i & 3) == 0 ? code_pair<0x00030003u>(y)
                  : (i & 3) == 1 ? code_pair<0x000C000Cu>(y)
                  : (i & 3) == 2 ? code_pair<0x00300030u>(y)
                                 : code_pair<0x00C000C0u>(y);
              }
              hv[i] = hfma2(c, sp[i], zp[i]);
            }
  #pragma unroll
            for (int q = 0; q < HP / 4; ++q)
              *reinterpret_cast<uint4*>(kd + k_off + s * 32 * D + q * 128) =
                  make_uint4(hv[4 * q], hv[4 * q + 1], hv[4 * q + 2], hv[4 * q + 3]);
            // value word (lane l, word w): channels 16mb + l/4 and 16mb + 8 + l/4
            // (mb = w, or 2w + half for 2-bit codes), tokens 2(l%4), +1, +8, +9;
            // v_off carries the lane's part of those offsets
  #pragma unroll
            for (int half = 0; half < (BITS == 4 ? 1 : 2); ++half) {
              const uint32_t* m4 = &reg[s][k * (2 + VMW) + 2 + 4 * half];
              const uint32_t s01 = __byte_perm(m4[0], m4[1], 0x5410), z01 = __byte_perm(m4[0], m4[1], 0x7632);
              const uint32_t s89 = __byte_perm(m4[2], m4[3], 0x5410), z89 = __byte_perm(m4[2], m4[3], 0x7632);
              uint32_t r[4];
              if (BITS == 4 || half == 0)
                value_frag<BITS, 0>(&reg[s][k * (2 + VMW) + 1], r);
              else
                value_frag<BITS, (BITS == 2 ? 1 : 0)>(&reg[s][k * (2 + VMW) + 1], r);
              const uint32_t v0 = hfma2(hfma2(r[0], VCode<BITS>::kMul, VCode<BITS>::kAddLo), s01, z01);
              const uint32_t v1 = hfma2(hfma2(r[1], VCode<BITS>::kMul, VCode<BITS>::kAddLo), s01, z01);
              const uint32_t v2 = hfma2(hfma2(r[2], VCode<BITS>::kMul, VCode<BITS>::kAddHi), s89, z89);
              const uint32_t v3 = hfma2(hfma2(r[3], VCode<BITS>::kMul, VCode<BITS>::kAddHi), s89, z89);
              // rows 16 mb + gl (+8), tokens tb + tl (+8): v_off plus constants
              uint8_t* const vp = vd + v_off + s * 256 + half * 32 * TN;
              *reinterpret_cast<uint32_t*>(vp) = v0;
              *reinterpret_cast<uint32_t*>(vp + 16 * TN) = v1;
              *reinterpret_cast<uint32_t*>(vp + 128) = v2;
              *reinterpret_cast<uint32_t*>(vp + 16 * TN + 128) = v3;
            }
          }
        } else if (j < n16) {
          const int t0 = nq + (j - n_pages) * kPage;
  #pragma unroll
          for (int k = 0; k < RPT; ++k) {
            const int u = tid + k * NT;
            if (u >= RV) continue;
            const int c16 = u >> 5, l = u & 31;
  #pragma unroll
            for (int r = 0; r < 4; ++r) {
              const uint32_t kx = reg[s][8 * k + r], vx = reg[s][8 * k + 4 + r];
              // K block: word r holds channels cc, cc+1 of token t
              const int t = 8 * (r & 1) + (l >> 2), cc = 8 * (r >> 1) + 2 * (l & 3);
              const int c = 16 * c16 + cc;
              *reinterpret_cast<uint16_t*>(kd + umma::umma_off(tb + t, kpos<BITS>(c), D)) =
                  static_cast<uint16_t>(kx & 0xffffu);
              *reinterpret_cast<uint16_t*>(kd + umma::umma_off(tb + t, kpos<BITS>(c + 1), D)) =
                  static_cast<uint16_t>(kx >> 16);
              // V block: word r holds tokens tv, tv+1 of channel 16c16 + cv;
              // tokens past the end (stale ring slots) become 0
              const int tv = 8 * (r >> 1) + 2 * (l & 3), cv = 8 * (r & 1) + (l >> 2);
              const uint32_t msk = (t0 + tv < L ? 0x0000ffffu : 0u) | (t0 + tv + 1 < L ? 0xffff0000u : 0u);
              *reinterpret_cast<uint32_t*>(vd + umma::umma_off(16 * c16 + cv, tb + tv, TN)) = vx & msk;
            }
          }
        } else {
          // past the last token of the CTA's rows: zero K rows and V^T columns
          for (int i = tid; i < kPage * D / 8; i += NT) {
            const int t = i / (D / 8), c8 = (i % (D / 8)) * 8;
            *reinterpret_cast<uint4*>(kd + umma::umma_off(tb + t, c8, D)) = make_uint4(0, 0, 0, 0);
          }
          for (int i = tid; i < D * 2; i += NT) {
            const int c = i >> 1, t8 = (i & 1) * 8;
            *reinterpret_cast<uint4*>(vd + umma::umma_off(c, tb + t8, TN)) = make_uint4(0, 0, 0, 0);
          }
        }
      }
    };


    if (n_tiles > 0) load_tile(0);
    for (int jt = 0; jt < n_tiles; ++jt) {
      // K buffer jt % 3 once S_{jt-3} has read it; V buffer jt % 3 once both
      // warpgroups' O += P_{jt-3} V_{jt-3} have
      if (jt >= 3 && !mbar_wait(&kfree[jt % 3], ((jt - 3) / 3) & 1, a.err)) break;
      if (jt >= 3 && !mbar_wait(&vfree[jt % 3], ((jt - 3) / 3) & 1, a.err)) break;
      umma::fence_after_sync();
      store_tile(jt, Ks + (jt % 3) * SM::K_BYTES, Vs + (jt % 3) * SM::V_BYTES);
      if (jt + 1 < n_tiles) load_tile(jt + 1);  // in flight while the tensor cores run
      umma::fence_smem_to_async();
      mbar_arrive(&tready[jt % 3]);
    }
  } else if (mma_warp) {
    // ======================= the MMA warp (lane 0 issues) =======================
    // per tile j: S_{j+1} (as soon as K_{j+1} is stored and O += P_{j-1}
    // V_{j-1} of both warpgroups, which reads P_{j-1} from S_{j+1}'s buffer,
    // is done), then O += P_j V_j of each warpgroup as its P_j lands
    if ((ctid & 31) == 0 && n_tiles > 0) {
      bool mok = true;
      int last_s = -1, last_pv = -1;
      // Operand descriptors are built once; the k-slice kk of an operand
      // starts 256 kk bytes further, i.e. 16 kk in the descriptor's address
      // field (shared-memory addresses stay below 2^18, so the field does not
      // carry).
      const uint64_t dq0 = umma::smem_desc(smem_u32(Qs), 128, 16 * D);
      const uint64_t dq1 = umma::smem_desc(smem_u32(Qs + SM::Q_BYTES), 128, 16 * D);
      const uint64_t dk0 = umma::smem_desc(smem_u32(Ks), 128, 16 * D);
      const uint64_t dv0 = umma::smem_desc(smem_u32(Vs), 128, 16 * TN);
      constexpr uint64_t kKStep = SM::K_BYTES >> 4, kVStep = SM::V_BYTES >> 4;
      auto issue_s = [&](int j) {
        umma::fence_after_sync();
        const uint64_t dk = dk0 + (j % 3) * kKStep;
        const uint32_t t0 = tmem + (j & 1) * TN;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          umma::mma_f16(t0, dq0 + 16 * kk, dk + 16 * kk, idS, kk > 0);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          umma::mma_f16(t0 + SM::TWG, dq1 + 16 * kk, dk + 16 * kk, idS, kk > 0);
        umma::commit(&sdone[j & 1]);
        umma::commit(&kfree[j % 3]);
        last_s = j;
      };
      mok = mbar_wait(&tready[0], 0, a.err);
      if (mok) issue_s(0);
      for (int j = 0; mok && j < n_tiles; ++j) {
        if (j + 1 < n_tiles) {
          mok = mbar_wait(&tready[(j + 1) % 3], ((j + 1) / 3) & 1, a.err) &&
                (j < 1 || (mbar_wait(&odone[(j - 1) & 1], ((j - 1) >> 1) & 1, a.err) &&
                           mbar_wait(&odone[2 + ((j - 1) & 1)], ((j - 1) >> 1) & 1, a.err)));
          if (!mok) break;
          issue_s(j + 1);
        }
        const uint64_t dv = dv0 + (j % 3) * kVStep;
#pragma unroll
        for (int w = 0; w < kUmmaWG; ++w) {
          if (!mbar_wait(&pready[2 * w + (j & 1)], (j >> 1) & 1, a.err)) {
            mok = false;
            break;
          }
          umma::fence_after_sync();
          // P_j: 8 columns of f16 pairs per 16 tokens, over S_j's buffer
          const uint32_t tp = tmem + w * SM::TWG + (j & 1) * TN;
#pragma unroll
          for (int kk = 0; kk < TN / 16; ++kk)
            umma::mma_f16_ta(tmem + w * SM::TWG + 2 * TN, tp + 8 * kk, dv + 16 * kk, idO,
                             j > 0 || kk > 0);
          umma::commit(&odone[2 * w + (j & 1)]);
          umma::commit(&vfree[j % 3]);
          last_pv = j;
        }
      }
      // no MMA may still run when tensor memory is released
      if (last_s >= 0) mbar_wait(&sdone[last_s & 1], (last_s >> 1) & 1, nullptr);
      if (last_pv >= 0) {
        mbar_wait(&odone[last_pv & 1], (last_pv >> 1) & 1, nullptr);
        mbar_wait(&odone[2 + (last_pv & 1)], (last_pv >> 1) & 1, nullptr);
      }
    }
  } else {
    // ======================= softmax warpgroups =======================
    const uint32_t tS = tmem + wg * SM::TWG, tO = tS + 2 * TN;  // this warpgroup's columns
    const uint32_t lane_base = static_cast<uint32_t>(32 * (warp & 3)) << 16;
    const float alpha = a.alpha;
    float m_run = -INFINITY, l_run = 0.f;
    // warpgroup wg's O += P_j V_j (and its MMAs before) done
    // (warp-uniform results: the tensor-memory loads after a wait are
    // whole-warp instructions)
    auto wait_o = [&](int j) {
      ok = __all_sync(0xffffffffu, mbar_wait(&odone[2 * wg + (j & 1)], (j >> 1) & 1, a.err)) && ok;
      umma::fence_after_sync();
    };
    for (int jt = 0; jt < n_tiles; ++jt) {
      const int b = jt & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(&sdone[b], (jt >> 1) & 1, a.err)) && ok;
      if (!ok) break;
      umma::fence_after_sync();
      // the row's 64 scores as two 32-column halves of tensor memory: a pass
      // for the maximum, then one for the weights (32 score registers live)
      const uint32_t tSj = tS + b * TN;
      const int tile0 = jt * TN;
      const bool masked = tile0 + TN - 1 > plim;
      static_assert(TN == 64, "the row's scores are read as two 32-column halves");
      auto load_half = [&](int hf, float (&x)[32]) {
        umma::ld32(tSj + lane_base + 32 * hf, x);
        umma::wait_ld();
        if (masked) {
#pragma unroll
          for (int c = 0; c < 32; ++c) x[c] = tile0 + 32 * hf + c <= plim ? x[c] : -INFINITY;
        }
      };
      float mx = -INFINITY;
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        float x[32];
        load_half(hf, x);
#pragma unroll
        for (int c = 0; c < 32; c += 2) mx = fmaxf(mx, fmaxf(x[c], x[c + 1]));
      }
      mx *= alpha;  // alpha > 0 keeps the order
      const bool need = mx > m_run + kPrefillLazyLog2;
      if (__any_sync(0xffffffffu, need)) {
        const float mnew = need ? fmaxf(m_run, mx) : m_run;
        const float f = m_run == -INFINITY ? 0.f : fast_exp2(m_run - mnew);
        l_run *= f;
        m_run = mnew;
        if (jt > 0) {  // this warp's rows of O in tensor memory, once O += P V of tile jt-1 is in
          wait_o(jt - 1);
#pragma unroll
          for (int c0 = 0; c0 < D; c0 += 16) {
            float o[16];
            umma::ld16(tO + lane_base + c0, o);
            umma::wait_ld();
#pragma unroll
            for (int c = 0; c < 16; ++c) o[c] *= f;
            umma::st16(tO + lane_base + c0, o);
          }
          umma::wait_st();
        }
      }
      // P_jt over the scores already read: tokens 32 hf .. 32 hf + 31 as 16
      // columns of f16 pairs at column 16 hf of S_jt's buffer (O += P_{jt-2}
      // V_{jt-2}, the buffer's last reader, finished before S_jt was issued)
      const float nb = m_run == -INFINITY ? 0.f : -m_run;
      float2 sum2 = make_float2(0.f, 0.f);
      const float2 al2 = make_float2(alpha, alpha), nb2 = make_float2(nb, nb);
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        float x[32];
        load_half(hf, x);
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          uint32_t pw[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int c = 16 * q + 2 * e;
            const float2 y = ffma2(make_float2(x[c], x[c + 1]), al2, nb2);
            const float2 pp = make_float2(fast_exp2(y.x), fast_exp2(y.y));
            sum2 = fadd2(sum2, pp);
            pw[e] = pack_h2(pp.x, pp.y);
          }
          umma::st8(tSj + lane_base + 16 * hf + 8 * q, pw);
        }
      }
      l_run += sum2.x + sum2.y;
      umma::wait_st();
      umma::fence_before_sync();
      mbar_arrive(&pready[2 * wg + b]);  // P_jt (and any O rescale) in place
      if (!ok) break;
    }
    if (ok && n_tiles > 0) wait_o(n_tiles - 1);
    if (bar_and(kBarSoftmax + wg, 128, ok) && n_tiles > 0) {
      // ---- normalise and write this thread's row ----
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
#pragma unroll
      for (int c0 = 0; c0 < D; c0 += 32) {
        float o[32];
        umma::ld32(tO + lane_base + c0, o);
        umma::wait_ld();
        if (valid) {
#pragma unroll
          for (int c = 0; c < 32; c += 8) {
            const int64_t oi = qrow + c0 + c;
            if (a.out_dtype == TKV_F32) {
              float4* dst = reinterpret_cast<float4*>(static_cast<float*>(a.out) + oi);
              dst[0] = make_float4(o[c] * inv, o[c + 1] * inv, o[c + 2] * inv, o[c + 3] * inv);
              dst[1] = make_float4(o[c + 4] * inv, o[c + 5] * inv, o[c + 6] * inv, o[c + 7] * inv);
            } else if (a.out_dtype == TKV_BF16) {
              uint32_t w[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const __nv_bfloat162 hh = __floats2bfloat162_rn(o[c + 2 * e] * inv, o[c + 2 * e + 1] * inv);
                w[e] = *reinterpret_cast<const uint32_t*>(&hh);
              }
              *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(a.out) + oi) =
                  make_uint4(w[0], w[1], w[2], w[3]);
            } else {
              uint32_t w[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) w[e] = pack_h2(o[c + 2 * e] * inv, o[c + 2 * e + 1] * inv);
              *reinterpret_cast<uint4*>(static_cast<__half*>(a.out) + oi) = make_uint4(w[0], w[1], w[2], w[3]);
            }
          }
        }
      }
    }
  }
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  if (warp == 0) umma::dealloc(tmem, SM::TCOLS);
}

template <int D, int BITS, int G>
static int launch_prefill_umma_t(PrefillArgs a, cudaStream_t stream) {
  using SM = UmmaSmem<D>;
  const int64_t tiles = ((int64_t)a.max_q * a.grp + kUmmaSoftmax - 1) / kUmmaSoftmax;
  const int64_t blocks = (int64_t)a.num_seqs * a.n_kv_heads * tiles;
  if (blocks <= 0) return TKV_OK;
  if (blocks > 0x7fffffffLL) return TKV_INVALID_ARGUMENT;
  static std::atomic<int> attr_set[kMaxPrefillDevices];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return TKV_BACKEND_ERROR;
  if (dev < 0 || dev >= kMaxPrefillDevices || !attr_set[dev].load(std::memory_order_relaxed)) {
    if (cudaFuncSetAttribute(prefill_umma_kernel<D, BITS, G>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, SM::BYTES) != cudaSuccess)
      return TKV_BACKEND_ERROR;
    if (dev >= 0 && dev < kMaxPrefillDevices) attr_set[dev].store(1, std::memory_order_relaxed);
  }
  a.n_rt = (int)tiles;
  prefill_umma_kernel<D, BITS, G><<<(unsigned)blocks, kUmmaCtaThreads, SM::BYTES, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? TKV_OK : TKV_BACKEND_ERROR;
}

template <int D, int BITS>
static int launch_prefill_g(const PrefillArgs& a, int G, cudaStream_t stream) {
  switch (G) {
    case 16: return launch_prefill_umma_t<D, BITS, 16>(a, stream);
    case 32: return launch_prefill_umma_t<D, BITS, 32>(a, stream);
    case 64: return launch_prefill_umma_t<D, BITS, 64>(a, stream);
    case 128: return launch_prefill_umma_t<D, BITS, 128>(a, stream);
    default: return TKV_NOT_IMPLEMENTED;
  }
}

int launch_prefill(const PrefillArgs& a, int head_dim, int bits, int group, cudaStream_t stream) {
  if (head_dim == 128)
    return bits == 4 ? launch_prefill_g<128, 4>(a, group, stream)
                     : launch_prefill_g<128, 2>(a, group, stream);
  if (head_dim == 64)
    return bits == 4 ? launch_prefill_g<64, 4>(a, group, stream)
                     : launch_prefill_g<64, 2>(a, group, stream);
  return TKV_NOT_IMPLEMENTED;
}

}  // namespace tkv
