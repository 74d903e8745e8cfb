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
// A CTA of 4 warps owns 64 query rows of one (sequence, kv head): rows
// rho = i * grp + j (token i, q head j of the kv head's group), 16 per warp,
// so the grp q heads of a kv head share every dequantised page.  Per 16-token
// tile the CTA's threads dequantise the page's codes -- exactly, to the fp16
// values the reference decompress writes, fp16(code * step + zero) for keys
// (per channel) and values (per token) -- into a K tile [16][D] and a V^T
// tile [D][16] in shared memory (double-buffered, one __syncthreads per tile);
// each warp then runs
//   * S = Q K^T on mma.m16n8k16 (A = its 16 query rows as exact fp16, B from
//     the K tile by ldmatrix), causal mask per row;
//   * online softmax per row in the exp2 domain (lazy rescale, as decode);
//   * O += P V (P from the S accumulators without shuffles, B from the V^T
//     tile by ldmatrix).
// Key channels sit in the tile in the order a code word unpacks into f16
// pairs ((c, c+4) for 4-bit words, (c, c+8) for 2-bit), and Q is loaded in the
// same order; ring tiles (the fp16 window) are scattered into that order.
// The next tile's code words are loaded into registers before the current
// tile's MMAs, so their latency overlaps them.
#include <atomic>

#include "tkv_frag.cuh"
#include "tkv_umma.cuh"

namespace tkv {

constexpr int kMaxPrefillDevices = 64;

namespace {

// S accumulators after the mask for tokens t0 + 8*nt + 2*tig + e against the
// rows' causal limits pa (row g) and pb (row g+8).
__device__ __forceinline__ void causal_mask(float (&s)[2][4], int t0, int tig, int pa, int pb) {
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
    const int t = t0 + 8 * nt + 2 * tig;
    s[nt][0] = t <= pa ? s[nt][0] : -INFINITY;
    s[nt][1] = t + 1 <= pa ? s[nt][1] : -INFINITY;
    s[nt][2] = t <= pb ? s[nt][2] : -INFINITY;
    s[nt][3] = t + 1 <= pb ? s[nt][3] : -INFINITY;
  }
}

template <int D>
struct RowState {
  float m[2];          // running max (log2 units) of rows g, g+8
  float l[2];          // this lane's partial sums of p
  float o[D / 8][4];   // O fragments: n-tile nt covers channels 8nt..8nt+7
};

// Online-softmax step for one 16-token tile; s holds raw scores on entry
// (-inf where masked) and the unnormalised weights on return.
template <int D>
__device__ __forceinline__ void row_softmax(RowState<D>& st, float (&s)[2][4], float alpha) {
  float t[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    float x = fmaxf(fmaxf(s[0][2 * r], s[0][2 * r + 1]), fmaxf(s[1][2 * r], s[1][2 * r + 1]));
    x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, 1));
    x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, 2));
    t[r] = x * alpha;
  }
  const bool need = t[0] > st.m[0] + kLazyLog2 || t[1] > st.m[1] + kLazyLog2;
  if (__any_sync(0xffffffffu, need)) {
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const float mnew = fmaxf(st.m[r], t[r]);
      const float f = st.m[r] == -INFINITY ? 0.f : fast_exp2(st.m[r] - mnew);
      st.l[r] *= f;
#pragma unroll
      for (int nt = 0; nt < D / 8; ++nt) {
        st.o[nt][2 * r] *= f;
        st.o[nt][2 * r + 1] *= f;
      }
      st.m[r] = mnew;
    }
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const float nbase = st.m[r] == -INFINITY ? 0.f : -st.m[r];
    float sum = 0.f;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      s[nt][2 * r] = fast_exp2(fmaf(s[nt][2 * r], alpha, nbase));
      s[nt][2 * r + 1] = fast_exp2(fmaf(s[nt][2 * r + 1], alpha, nbase));
      sum += s[nt][2 * r] + s[nt][2 * r + 1];
    }
    st.l[r] += sum;
  }
}

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

__device__ __forceinline__ void ldsm_x4(const void* p, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_u32(p))
               : "memory");
}

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

template <int D, int BITS, int G, int NW>
__global__ void __launch_bounds__(32 * NW, 2) prefill_cta_kernel(PrefillArgs a) {
  using F = Fmt<D, BITS, G>;
  constexpr int NT = 32 * NW, NKB = D / 16;
  constexpr int WPR = D * BITS / 32;          // key-code words per token row
  constexpr int CPW = 32 / BITS;              // channels per key word
  constexpr int HP = CPW / 2;                 // f16 pairs per key word
  constexpr int KW = kPage * WPR;             // key (and value) code words per page
  constexpr int KPT = (KW + NT - 1) / NT;     // code words per thread
  constexpr int MVEC = CPW / 4;               // 16-byte key-meta vectors per word's channels
  constexpr int VMW = BITS == 4 ? 4 : 8;      // value (step, zero) words per value word
  constexpr int RV = 2 * D;                   // 16-byte vectors per ring K (or V) block
  constexpr int RPT = (RV + NT - 1) / NT;
  constexpr int KS = D + 8, VS = kPage + 8;   // padded row strides (halves)
  static_assert(NT % WPR == 0, "a thread's key words share their channels");
  __shared__ __align__(16) __half Kt[2][kPage][KS];
  __shared__ __align__(16) __half Vt[2][D][VS];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, tig = lane & 3;

  const int64_t bid = blockIdx.x;
  const int rt = a.n_rt - 1 - (int)(bid % a.n_rt);
  const int bh = (int)(bid / a.n_rt);
  const int b = bh / a.n_kv_heads, h = bh - b * a.n_kv_heads;
  const int L = a.seq_lens[b];
  const int q0 = a.cu_q[b], n = a.cu_q[b + 1] - q0;
  // n > max_q: the grid has row tiles for max_q tokens only, so the chunk's
  // later rows would stay unwritten; flag the sequence instead
  if (L < 0 || L > a.max_blocks * kPage || n < 0 || n > L || n > a.max_q || q0 < 0 ||
      q0 + n > a.total_q) {
    if (rt == 0 && h == 0 && tid == 0) set_err(a.err, TKV_ERR_BAD_LENGTH);
    return;
  }
  const int rows = n * a.grp, r0 = rt * 16 * NW;
  if (r0 >= rows) return;
  const int ra = r0 + 16 * warp + g, rb = ra + 8;
  const bool va = ra < rows, vb = rb < rows;
  const int ia = va ? ra / a.grp : n - 1, ib = vb ? rb / a.grp : n - 1;
  const int pa = L - n + ia, pb = L - n + ib;
  const int kv_end = L - n + min(rows - 1, r0 + 16 * NW - 1) / a.grp + 1;
  const int64_t qa = ((int64_t)(q0 + ia) * a.num_q_heads + h * a.grp + (va ? ra % a.grp : 0)) * D;
  const int64_t qb = ((int64_t)(q0 + ib) * a.num_q_heads + h * a.grp + (vb ? rb % a.grp : 0)) * D;
  const int nq = nq_len(L, a.residual, G);
  const int32_t* bt = a.block_tables + (int64_t)b * a.max_blocks;
  const int n_pages = min(nq, (kv_end + kPage - 1) / kPage * kPage) / kPage;
  const int n_chunks = kv_end > nq ? (kv_end - nq + kPage - 1) / kPage : 0;
  const int n_tiles = n_pages + n_chunks;

  // every page read (the tiles' pages and their groups' key meta) in range
  const int n_read = min(nq / kPage, (n_pages + F::PPG - 1) / F::PPG * F::PPG);
  bool bad = false;
  for (int p = tid; p < n_read; p += NT) {
    const int ph = bt[p];
    bad |= ph < 0 || ph >= a.num_pages;
  }
  if (__syncthreads_or(bad)) {
    if (tid == 0) set_err(a.err, TKV_ERR_BAD_PAGE);
    return;
  }
  int row = 0;
  if (n_chunks > 0) {
    row = a.seq_slots ? a.seq_slots[b] : b;
    if (row < 0 || row >= a.max_seqs) {
      if (tid == 0) set_err(a.err, TKV_ERR_BAD_SLOT);
      return;
    }
  }

  // A operand: this warp's rows g, g+8 as exact f16, channels in tile order
  uint32_t aq[NKB][4];
#pragma unroll
  for (int kb = 0; kb < NKB; ++kb)
#pragma unroll
    for (int hi = 0; hi < 2; ++hi) {
      const int c0 = kchan_at<BITS>(16 * kb + 8 * hi + 2 * tig);
      const int c1 = kchan_at<BITS>(16 * kb + 8 * hi + 2 * tig + 1);
      aq[kb][2 * hi + 0] = pack_h2(va ? load_qv(a, qa + c0) : 0.f, va ? load_qv(a, qa + c1) : 0.f);
      aq[kb][2 * hi + 1] = pack_h2(vb ? load_qv(a, qb + c0) : 0.f, vb ? load_qv(a, qb + c1) : 0.f);
    }

  const uint8_t* pool_h = a.pool + (int64_t)h * F::PB;
  const int64_t page_stride = (int64_t)a.n_kv_heads * F::PB;
  constexpr int CHUNK = 2 * F::RBLK;
  const uint8_t* ring_base =
      reinterpret_cast<const uint8_t*>(a.ring) +
      (((int64_t)row * a.n_kv_heads + h) * (a.ring_cap / kPage)) * CHUNK;
  const int kc0 = (tid % WPR) * CPW;  // first channel of this thread's key words

  // ---------------- registers of the next tile ----------------
  uint32_t kw[KPT], vw[KPT], vm[KPT][VMW];
  uint4 km[MVEC];
  uint4 rk[RPT], rv[RPT];
  auto load_tile = [&](int j) {
    if (j < n_pages) {
      const uint8_t* pg = pool_h + (int64_t)bt[j] * page_stride;
#pragma unroll
      for (int k = 0; k < KPT; ++k) {
        const int u = tid + k * NT;
        if (u >= KW) continue;
        kw[k] = __ldg(reinterpret_cast<const uint32_t*>(pg) + u);
        const int l = u & 31, w = u >> 5;
        vw[k] = __ldg(reinterpret_cast<const uint32_t*>(
            pg + F::V_CODES_OFF + ((w / F::VW) * 32 + l) * 4 * F::VW + (w % F::VW) * 4));
        const uint32_t* vmp = reinterpret_cast<const uint32_t*>(pg + F::V_META_OFF);
        const int t0 = 2 * (l & 3);
#pragma unroll
        for (int x = 0; x < VMW; ++x) {
          // 4-bit: tokens t0, t0+1, t0+8, t0+9 of m-block w; 2-bit: the same
          // for m-blocks 2w (x < 4) and 2w+1
          const int mb = BITS == 4 ? w : 2 * w + (x >> 2);
          const int t = t0 + (x & 1) + 8 * ((x >> 1) & 1);
          vm[k][x] = __ldg(vmp + t * F::NVG + (16 * mb) / G);
        }
      }
      if (j % F::PPG == 0 && tid < KW) {  // a new key group: this thread's channels
        const int grp = j / F::PPG;
#pragma unroll
        for (int v = 0; v < MVEC; ++v) {
          const int off = 4 * (kc0 + 4 * v);
          const int ph = bt[grp * F::PPG + off / F::KMS];
          km[v] = __ldg(reinterpret_cast<const uint4*>(pool_h + (int64_t)ph * page_stride +
                                                        F::BODY + off % F::KMS));
        }
      }
    } else {
      const int t0 = nq + (j - n_pages) * kPage;
      const uint8_t* ck = ring_base + (int64_t)((t0 % a.ring_cap) / kPage) * CHUNK;
#pragma unroll
      for (int k = 0; k < RPT; ++k) {
        const int u = tid + k * NT;
        if (u >= RV) continue;
        rk[k] = __ldg(reinterpret_cast<const uint4*>(ck) + u);
        rv[k] = __ldg(reinterpret_cast<const uint4*>(ck + F::RBLK) + u);
      }
    }
  };
  auto store_tile = [&](int j, int buf) {
    if (j < n_pages) {
      uint32_t mw[CPW];
#pragma unroll
      for (int v = 0; v < MVEC; ++v) {
        mw[4 * v + 0] = km[v].x; mw[4 * v + 1] = km[v].y;
        mw[4 * v + 2] = km[v].z; mw[4 * v + 3] = km[v].w;
      }
      uint32_t sp[HP], zp[HP];
#pragma unroll
      for (int i = 0; i < HP; ++i) {
        sp[i] = __byte_perm(mw[i], mw[i + HP], 0x5410);
        zp[i] = __byte_perm(mw[i], mw[i + HP], 0x7632);
      }
#pragma unroll
      for (int k = 0; k < KPT; ++k) {
        const int u = tid + k * NT;
        if (u >= KW) continue;
        const uint32_t x = kw[k], x8 = kw[k] >> 8;
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
        __half* dst = &Kt[buf][u / WPR][kc0];
#pragma unroll
        for (int q = 0; q < HP / 4; ++q)
          reinterpret_cast<uint4*>(dst)[q] = make_uint4(hv[4 * q], hv[4 * q + 1], hv[4 * q + 2],
                                                        hv[4 * q + 3]);
        // value word (lane l, word w): channels 16mb+gl and 16mb+8+gl, tokens
        // tl, tl+1, tl+8, tl+9
        const int l = u & 31, w = u >> 5, gl = l >> 2, tl = 2 * (l & 3);
#pragma unroll
        for (int half = 0; half < (BITS == 4 ? 1 : 2); ++half) {
          const int mb = BITS == 4 ? w : 2 * w + half;
          const uint32_t* m4 = &vm[k][4 * half];
          const uint32_t s01 = __byte_perm(m4[0], m4[1], 0x5410), z01 = __byte_perm(m4[0], m4[1], 0x7632);
          const uint32_t s89 = __byte_perm(m4[2], m4[3], 0x5410), z89 = __byte_perm(m4[2], m4[3], 0x7632);
          uint32_t r[4];
          if (BITS == 4 || half == 0)
            value_frag<BITS, 0>(&vw[k], r);
          else
            value_frag<BITS, (BITS == 2 ? 1 : 0)>(&vw[k], r);
          const uint32_t v0 = hfma2(hfma2(r[0], VCode<BITS>::kMul, VCode<BITS>::kAddLo), s01, z01);
          const uint32_t v1 = hfma2(hfma2(r[1], VCode<BITS>::kMul, VCode<BITS>::kAddLo), s01, z01);
          const uint32_t v2 = hfma2(hfma2(r[2], VCode<BITS>::kMul, VCode<BITS>::kAddHi), s89, z89);
          const uint32_t v3 = hfma2(hfma2(r[3], VCode<BITS>::kMul, VCode<BITS>::kAddHi), s89, z89);
          *reinterpret_cast<uint32_t*>(&Vt[buf][16 * mb + gl][tl]) = v0;
          *reinterpret_cast<uint32_t*>(&Vt[buf][16 * mb + 8 + gl][tl]) = v1;
          *reinterpret_cast<uint32_t*>(&Vt[buf][16 * mb + gl][tl + 8]) = v2;
          *reinterpret_cast<uint32_t*>(&Vt[buf][16 * mb + 8 + gl][tl + 8]) = v3;
        }
      }
    } else {
      const int t0 = nq + (j - n_pages) * kPage;
#pragma unroll
      for (int k = 0; k < RPT; ++k) {
        const int u = tid + k * NT;
        if (u >= RV) continue;
        const int c16 = u >> 5, l = u & 31;
        const uint32_t kx[4] = {rk[k].x, rk[k].y, rk[k].z, rk[k].w};
        const uint32_t vx[4] = {rv[k].x, rv[k].y, rv[k].z, rv[k].w};
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          // K block: word r holds channels cc, cc+1 of token t
          const int t = 8 * (r & 1) + (l >> 2), cc = 8 * (r >> 1) + 2 * (l & 3);
          const int c = 16 * c16 + cc;
          Kt[buf][t][kpos<BITS>(c)] = __ushort_as_half(static_cast<unsigned short>(kx[r] & 0xffffu));
          Kt[buf][t][kpos<BITS>(c + 1)] = __ushort_as_half(static_cast<unsigned short>(kx[r] >> 16));
          // V block: word r holds tokens tv, tv+1 of channel 16c16 + cv; tokens
          // past the end (stale ring slots) become 0
          const int tv = 8 * (r >> 1) + 2 * (l & 3), cv = 8 * (r & 1) + (l >> 2);
          const uint32_t msk = (t0 + tv < L ? 0x0000ffffu : 0u) | (t0 + tv + 1 < L ? 0xffff0000u : 0u);
          *reinterpret_cast<uint32_t*>(&Vt[buf][16 * c16 + cv][tv]) = vx[r] & msk;
        }
      }
    }
  };

  RowState<D> st;
  st.m[0] = st.m[1] = -INFINITY;
  st.l[0] = st.l[1] = 0.f;
#pragma unroll
  for (int nt = 0; nt < D / 8; ++nt) st.o[nt][0] = st.o[nt][1] = st.o[nt][2] = st.o[nt][3] = 0.f;
  const float alpha = a.alpha;
  const int mi = lane >> 3, mr = lane & 7;

  load_tile(0);
  store_tile(0, 0);
  __syncthreads();
  for (int j = 0; j < n_tiles; ++j) {
    const int buf = j & 1;
    if (j + 1 < n_tiles) load_tile(j + 1);  // in flight during this tile's MMAs
    // ---- S = Q K^T over the tile's 16 tokens ----
    float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int kb = 0; kb < NKB; ++kb) {
      uint32_t b0, b1, b2, b3;
      ldsm_x4(&Kt[buf][(mi >> 1) * 8 + mr][16 * kb + (mi & 1) * 8], b0, b1, b2, b3);
      mma16816(s[0], aq[kb][0], aq[kb][1], aq[kb][2], aq[kb][3], b0, b1);
      mma16816(s[1], aq[kb][0], aq[kb][1], aq[kb][2], aq[kb][3], b2, b3);
    }
    const int t0 = j < n_pages ? j * kPage : nq + (j - n_pages) * kPage;
    if (t0 + kPage - 1 > min(pa, pb)) causal_mask(s, t0, tig, pa, pb);
    row_softmax<D>(st, s, alpha);
    // ---- O += P V ----
    const uint32_t a0 = pack_h2(s[0][0], s[0][1]);
    const uint32_t a1 = pack_h2(s[0][2], s[0][3]);
    const uint32_t a2 = pack_h2(s[1][0], s[1][1]);
    const uint32_t a3 = pack_h2(s[1][2], s[1][3]);
#pragma unroll
    for (int mb = 0; mb < D / 16; ++mb) {
      uint32_t b0, b1, b2, b3;
      ldsm_x4(&Vt[buf][16 * mb + (mi >> 1) * 8 + mr][(mi & 1) * 8], b0, b1, b2, b3);
      mma16816(st.o[2 * mb], a0, a1, a2, a3, b0, b1);
      mma16816(st.o[2 * mb + 1], a0, a1, a2, a3, b2, b3);
    }
    if (j + 1 < n_tiles) store_tile(j + 1, buf ^ 1);
    __syncthreads();
  }

  // ---- normalise and write this warp's rows ----
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    st.l[r] += __shfl_xor_sync(0xffffffffu, st.l[r], 1);
    st.l[r] += __shfl_xor_sync(0xffffffffu, st.l[r], 2);
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    if (!(r == 0 ? va : vb)) continue;
    const float inv = 1.f / st.l[r];
    const int64_t ob = r == 0 ? qa : qb;
#pragma unroll
    for (int nt = 0; nt < D / 8; ++nt) {
      const float o0 = st.o[nt][2 * r] * inv, o1 = st.o[nt][2 * r + 1] * inv;
      const int64_t oi = ob + 8 * nt + 2 * tig;
      if (a.out_dtype == TKV_F32) {
        *reinterpret_cast<float2*>(static_cast<float*>(a.out) + oi) = make_float2(o0, o1);
      } else if (a.out_dtype == TKV_BF16) {
        *reinterpret_cast<__nv_bfloat162*>(static_cast<__nv_bfloat16*>(a.out) + oi) =
            __floats2bfloat162_rn(o0, o1);
      } else {
        *reinterpret_cast<__half2*>(static_cast<__half*>(a.out) + oi) = __floats2half2_rn(o0, o1);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// The same attention on the 5th-generation tensor cores (tcgen05): one CTA of
// two warpgroups per 256 query rows of a (sequence, kv head), each warpgroup
// owning 128 rows (the MMA's M) and its own S and O in tensor memory; 64-token
// KV tiles shared by both.  Per tile the CTA's threads dequantise the tile's four 16-token
// pages (or fp16 ring chunks) exactly, as above, straight into the K-major
// shared-memory operand layouts of tkv_umma.cuh: K [64 tokens][D channels]
// (channels in the code-unpack order, Q staged in the same order) and V^T
// [D channels][64 tokens].  One thread issues S = Q K^T (D/16 MMAs, N = 64)
// into tensor memory; each thread then owns one query row: it loads the row's
// 64 scores with tcgen05.ld, masks them causally, runs the online softmax
// (exp2 domain, lazy rescale: when a warp's running maxima move, its rows of O
// are rescaled in tensor memory) and stores the row's weights P as f16 into
// its warpgroup's P tile; one thread of the warpgroup issues O += P V (4 MMAs,
// N = D) into tensor memory.  Software pipeline: while tile j's softmax runs,
// S of tile j+1 is on the tensor cores (its K already dequantised), and
// O += P V of tile j runs while tile j+1's successor is dequantised; the next
// tile's code words are loaded into registers one tile ahead.  Tensor memory
// per warpgroup (256 columns): S of even and odd tiles in [0, 128), O in
// [128, 128 + D).
// ---------------------------------------------------------------------------
constexpr int kUmmaRows = 128;  // query rows per warpgroup (the MMA's M)
constexpr int kUmmaWG = 2;      // warpgroups per CTA
constexpr int kUmmaTN = 64;     // tokens per KV tile
constexpr int kUmmaThreads = 128 * kUmmaWG;

template <int D>
struct UmmaSmem {
  // K double-, V triple- and P double-buffered: tile j+1 is dequantised and
  // its S issued while tile j's softmax runs, and O += P_j V_j runs while
  // tile j+2 is dequantised
  static constexpr int K_BYTES = kUmmaTN * D * 2, V_BYTES = D * kUmmaTN * 2;
  static constexpr int P_BYTES = kUmmaRows * kUmmaTN * 2, Q_BYTES = kUmmaRows * D * 2;
  static constexpr int Q_OFF = 0;  // one Q operand per warpgroup
  static constexpr int K_OFF = Q_OFF + kUmmaWG * Q_BYTES;
  static constexpr int V_OFF = K_OFF + 2 * K_BYTES;
  static constexpr int P_OFF = V_OFF + 3 * V_BYTES;  // [warpgroup][2]
  static constexpr int BAR_OFF = P_OFF + 2 * kUmmaWG * P_BYTES;
  static constexpr int BYTES = BAR_OFF + 64;
  // tensor memory: per warpgroup 256 columns, S of even and odd tiles, then O
  static constexpr uint32_t TWG = 256, TCOLS = 512;
  static_assert(2 * kUmmaTN + D <= TWG, "a warpgroup's S and O fit its columns");
};

template <int D, int BITS, int G>
__global__ void __launch_bounds__(kUmmaThreads, 1) prefill_umma_kernel(PrefillArgs a) {
  using F = Fmt<D, BITS, G>;
  using SM = UmmaSmem<D>;
  constexpr int NT = kUmmaThreads, TN = kUmmaTN, NSUB = TN / kPage;
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
  uint8_t* const Ps = smem + SM::P_OFF;
  // bars[b]: S of tiles j = b (mod 2) done (both warpgroups); bars[2 + 2 w + b]:
  // warpgroup w's O += P_j V_j of those tiles done
  uint64_t* const bars = reinterpret_cast<uint64_t*>(smem + SM::BAR_OFF);
  uint32_t* const tslot = reinterpret_cast<uint32_t*>(bars + 6);
  const int tid = threadIdx.x, warp = tid >> 5;
  const int wg = tid >> 7, wt = tid & 127;  // warpgroup, row in the warpgroup

  const int64_t bid = blockIdx.x;
  const int rt = a.n_rt - 1 - (int)(bid % a.n_rt);
  const int bh = (int)(bid / a.n_rt);
  const int b = bh / a.n_kv_heads, h = bh - b * a.n_kv_heads;
  const int L = a.seq_lens[b];
  const int q0 = a.cu_q[b], n = a.cu_q[b + 1] - q0;
  if (L < 0 || L > a.max_blocks * kPage || n < 0 || n > L || n > a.max_q || q0 < 0 ||
      q0 + n > a.total_q) {
    if (rt == 0 && h == 0 && tid == 0) set_err(a.err, TKV_ERR_BAD_LENGTH);
    return;
  }
  const int rows = n * a.grp, r0 = rt * kUmmaThreads;
  if (r0 >= rows) return;
  const int rho = r0 + tid;
  const bool valid = rho < rows;
  const int qi = valid ? rho / a.grp : 0;
  const int plim = valid ? L - n + qi : -1;  // causal limit of this thread's row
  const int kv_end = L - n + min(rows - 1, r0 + kUmmaThreads - 1) / a.grp + 1;
  const int64_t qrow = ((int64_t)(q0 + qi) * a.num_q_heads + h * a.grp + (valid ? rho % a.grp : 0)) * D;
  const int nq = nq_len(L, a.residual, G);
  const int32_t* bt = a.block_tables + (int64_t)b * a.max_blocks;
  const int n_pages = min(nq, (kv_end + kPage - 1) / kPage * kPage) / kPage;
  const int n_chunks = kv_end > nq ? (kv_end - nq + kPage - 1) / kPage : 0;
  const int n16 = n_pages + n_chunks;
  const int n_tiles = (n16 + NSUB - 1) / NSUB;

  const int n_read = min(nq / kPage, (n_pages + F::PPG - 1) / F::PPG * F::PPG);
  bool bad = false;
  for (int p = tid; p < n_read; p += NT) {
    const int ph = bt[p];
    bad |= ph < 0 || ph >= a.num_pages;
  }
  if (__syncthreads_or(bad)) {
    if (tid == 0) set_err(a.err, TKV_ERR_BAD_PAGE);
    return;
  }
  int row = 0;
  if (n_chunks > 0) {
    row = a.seq_slots ? a.seq_slots[b] : b;
    if (row < 0 || row >= a.max_seqs) {
      if (tid == 0) set_err(a.err, TKV_ERR_BAD_SLOT);
      return;
    }
  }

  // ---- tensor memory, barriers, the Q operand ----
  if (warp == 0) umma::alloc(tslot, SM::TCOLS);
  if (tid == 0) {
    for (int i = 0; i < 6; ++i) mbar_init(&bars[i], 1);
    fence_mbar_init();
  }
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
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tmem = *tslot;
  const uint32_t tS = tmem + wg * SM::TWG, tO = tS + 2 * TN;  // this warpgroup's columns
  const uint32_t lane_base = static_cast<uint32_t>(32 * (warp & 3)) << 16;

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
  // channels kc0..), its value word's first (channel, token) pair, its P row
  const uint32_t k_off = umma::umma_off(tid % kPage, tid < KW ? kc0 : 0, D);
  const uint32_t v_off = umma::umma_off(16 * (BITS == 4 ? (tid >> 5) : 2 * (tid >> 5)) + ((tid & 31) >> 2),
                                        2 * (tid & 3), TN);
  const uint32_t p_off = umma::umma_off(wt, 0, TN);

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
#pragma unroll
    for (int s = 0; s < NSUB; ++s) {
      const int j = jt * NSUB + s;
      const int tb = s * kPage;  // the sub-tile's first token in the tile
      if (j < n_pages) {
        const int ki = F::PPG >= NSUB ? 0 : s / (F::PPG >= NSUB ? 1 : F::PPG);
        uint32_t mw[CPW];
#pragma unroll
        for (int v = 0; v < MVEC; ++v) {
          mw[4 * v + 0] = km[ki][v].x; mw[4 * v + 1] = km[ki][v].y;
          mw[4 * v + 2] = km[ki][v].z; mw[4 * v + 3] = km[ki][v].w;
        }
        uint32_t sp[HP], zp[HP];
#pragma unroll
        for (int i = 0; i < HP; ++i) {
          sp[i] = __byte_perm(mw[i], mw[i + HP], 0x5410);
          zp[i] = __byte_perm(mw[i], mw[i + HP], 0x7632);
        }
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
          // value word (lane l, word w): channels 16mb+gl and 16mb+8+gl, tokens
          // tl, tl+1, tl+8, tl+9
          const int l = u & 31, w = u >> 5, gl = l >> 2, tl = 2 * (l & 3);
#pragma unroll
          for (int half = 0; half < (BITS == 4 ? 1 : 2); ++half) {
            const int mb = BITS == 4 ? w : 2 * w + half;
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

  constexpr uint32_t idS = umma::idesc_f16(kUmmaRows, TN, false);
  constexpr uint32_t idO = umma::idesc_f16(kUmmaRows, D, false);
  const float alpha = a.alpha;
  float m_run = -INFINITY, l_run = 0.f;
  bool ok = true;
  // A parity wait on an mbarrier targets the oldest of its phases not yet
  // known to be complete, at most one phase behind: tile j's S and O MMAs
  // commit to barriers of parity class j & 1, phase j >> 1.
  auto wait_o = [&](int j, int w) {  // warpgroup w's O += P_j V_j (and its MMAs before) done
    ok = mbar_wait(&bars[2 + 2 * w + (j & 1)], (j >> 1) & 1, a.err) && ok;
    umma::fence_after_sync();
  };
  auto issue_s = [&](int j) {  // S_j = Q K_j^T of both warpgroups into their S[j & 1]
    if (tid == 0) {
      umma::fence_after_sync();
      const uint32_t kb = smem_u32(Ks + (j & 1) * SM::K_BYTES);
#pragma unroll
      for (int w = 0; w < kUmmaWG; ++w)
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          umma::mma_f16(tmem + w * SM::TWG + (j & 1) * TN,
                        umma::smem_desc(smem_u32(Qs + w * SM::Q_BYTES) + 256 * kk, 128, 16 * D),
                        umma::smem_desc(kb + 256 * kk, 128, 16 * D), idS, kk > 0);
      umma::commit(&bars[j & 1]);
    }
  };
  if (n_tiles > 0) {
    load_tile(0);
    store_tile(0, Ks, Vs);
    if (n_tiles > 1) load_tile(1);
    umma::fence_smem_to_async();
    umma::fence_before_sync();
    __syncthreads();
    issue_s(0);
  }
  for (int jt = 0; jt < n_tiles; ++jt) {
    const int b = jt & 1;
    if (jt >= 2) {
      // the P buffer b of this warpgroup, and when tile jt+1 is dequantised
      // below, the V^T buffer (jt + 1) % 3 read by both warpgroups.  A wait on
      // the other warpgroup's barrier is made only before the CTA-wide barrier
      // of this iteration, which keeps that warpgroup from completing a second
      // phase of it first (in the last tile there is no such barrier).
      if (jt + 1 < n_tiles) {
        wait_o(jt - 2, 0);
        wait_o(jt - 2, 1);
      } else {
        wait_o(jt - 2, wg);
      }
    }
    if (jt + 1 < n_tiles) {
      store_tile(jt + 1, Ks + ((jt + 1) & 1) * SM::K_BYTES, Vs + ((jt + 1) % 3) * SM::V_BYTES);
      if (jt + 2 < n_tiles) load_tile(jt + 2);  // in flight during this tile's softmax
      umma::fence_smem_to_async();
      umma::fence_before_sync();
      if (!__syncthreads_and(ok)) {
        ok = false;
        break;
      }
      issue_s(jt + 1);
    }
    ok = mbar_wait(&bars[b], (jt >> 1) & 1, a.err) && ok;
    umma::fence_after_sync();
    // the row's scores in two 32-column halves: a pass for the maximum, then
    // one for the weights (tensor memory is read twice, the registers once)
    const uint32_t tSj = tS + b * TN;
    const int tile0 = jt * TN;
    const bool masked = tile0 + TN - 1 > plim;
    static_assert(TN == 64, "the row's scores are read as two 32-column halves");
    auto load_row = [&](float (&x0)[32], float (&x1)[32]) {  // both halves, one wait
      umma::ld32(tSj + lane_base, x0);
      umma::ld32(tSj + lane_base + 32, x1);
      umma::wait_ld();
      if (masked) {
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          x0[c] = tile0 + c <= plim ? x0[c] : -INFINITY;
          x1[c] = tile0 + 32 + c <= plim ? x1[c] : -INFINITY;
        }
      }
    };
    float mx = -INFINITY;
    {
      float x0[32], x1[32];
      load_row(x0, x1);
#pragma unroll
      for (int c = 0; c < 32; ++c) mx = fmaxf(mx, fmaxf(x0[c], x1[c]));
    }
    mx *= alpha;  // alpha > 0 keeps the order
    const bool need = mx > m_run + kLazyLog2;
    if (__any_sync(0xffffffffu, need)) {
      const float mnew = need ? fmaxf(m_run, mx) : m_run;
      const float f = m_run == -INFINITY ? 0.f : fast_exp2(m_run - mnew);
      l_run *= f;
      m_run = mnew;
      if (jt > 0) {  // this warp's rows of O in tensor memory, once O += P V of tile jt-1 is in
        wait_o(jt - 1, wg);
#pragma unroll
        for (int c0 = 0; c0 < D; c0 += 32) {
          float o[32];
          umma::ld32(tO + lane_base + c0, o);
          umma::wait_ld();
#pragma unroll
          for (int c = 0; c < 32; ++c) o[c] *= f;
          umma::st32(tO + lane_base + c0, o);
        }
        umma::wait_st();
      }
    }
    const float nb = m_run == -INFINITY ? 0.f : -m_run;
    uint8_t* const pd = Ps + (2 * wg + b) * SM::P_BYTES;
    float2 sum2 = make_float2(0.f, 0.f);
    const float2 al2 = make_float2(alpha, alpha), nb2 = make_float2(nb, nb);
    float xr[2][32];
    load_row(xr[0], xr[1]);
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const float (&x)[32] = xr[hf];
#pragma unroll
      for (int c8 = 0; c8 < 32; c8 += 8) {
        uint32_t w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 y = ffma2(make_float2(x[c8 + 2 * e], x[c8 + 2 * e + 1]), al2, nb2);
          const float2 pp = make_float2(fast_exp2(y.x), fast_exp2(y.y));
          sum2 = fadd2(sum2, pp);
          w[e] = pack_h2(pp.x, pp.y);
        }
        *reinterpret_cast<uint4*>(pd + p_off + (32 * hf + c8) * 16) =
            make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
    l_run += sum2.x + sum2.y;
    umma::fence_smem_to_async();
    umma::fence_before_sync();
    // this warpgroup's 128 threads only (named barrier 1 + wg)
    asm volatile("bar.sync %0, %1;\n" ::"r"(1 + wg), "r"(128) : "memory");
    if (wt == 0) {  // O += P_jt V_jt of this warpgroup
      umma::fence_after_sync();
      const uint32_t vb = smem_u32(Vs + (jt % 3) * SM::V_BYTES);
#pragma unroll
      for (int kk = 0; kk < TN / 16; ++kk)
        umma::mma_f16(tO, umma::smem_desc(smem_u32(pd) + 256 * kk, 128, 16 * TN),
                      umma::smem_desc(vb + 256 * kk, 128, 16 * TN), idO, jt > 0 || kk > 0);
      umma::commit(&bars[2 + 2 * wg + b]);
    }
  }
  if (ok && n_tiles > 0) wait_o(n_tiles - 1, wg);
  if (__syncthreads_and(ok) && n_tiles > 0) {
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
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  if (warp == 0) umma::dealloc(tmem, SM::TCOLS);
}

template <int D, int BITS, int G>
static int launch_prefill_umma_t(PrefillArgs a, cudaStream_t stream) {
  using SM = UmmaSmem<D>;
  const int64_t tiles = ((int64_t)a.max_q * a.grp + kUmmaThreads - 1) / kUmmaThreads;
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
  prefill_umma_kernel<D, BITS, G><<<(unsigned)blocks, kUmmaThreads, SM::BYTES, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? TKV_OK : TKV_BACKEND_ERROR;
}

constexpr int kPrefillWarps = 4;  // 16 query rows each: 64 rows per CTA

template <int D, int BITS, int G>
static int launch_prefill_t(PrefillArgs a, cudaStream_t stream) {
  constexpr int NW = kPrefillWarps;
  const int64_t tiles = ((int64_t)a.max_q * a.grp + 16 * NW - 1) / (16 * NW);
  const int64_t blocks = (int64_t)a.num_seqs * a.n_kv_heads * tiles;
  if (blocks <= 0) return TKV_OK;
  if (blocks > 0x7fffffffLL) return TKV_INVALID_ARGUMENT;
  a.n_rt = (int)tiles;
  prefill_cta_kernel<D, BITS, G, NW><<<(unsigned)blocks, 32 * NW, 0, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? TKV_OK : TKV_BACKEND_ERROR;
}

#ifdef TKV_PREFILL_MMA_SYNC
#define TKV_PREFILL_LAUNCH launch_prefill_t
#else
#define TKV_PREFILL_LAUNCH launch_prefill_umma_t
#endif
template <int D, int BITS>
static int launch_prefill_g(const PrefillArgs& a, int G, cudaStream_t stream) {
  switch (G) {
    case 16: return TKV_PREFILL_LAUNCH<D, BITS, 16>(a, stream);
    case 32: return TKV_PREFILL_LAUNCH<D, BITS, 32>(a, stream);
    case 64: return TKV_PREFILL_LAUNCH<D, BITS, 64>(a, stream);
    case 128: return TKV_PREFILL_LAUNCH<D, BITS, 128>(a, stream);
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
