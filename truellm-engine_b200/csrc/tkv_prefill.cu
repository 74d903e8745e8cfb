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
// One warp per CTA owns a tile of 16 query rows of one (sequence, kv head):
// rows rho = i * grp + j (token i, q head j of the kv head's group), so the
// grp q heads of one kv head share every dequantised K/V fragment.  Per page
// the warp dequantises keys and values straight into mma.m16n8k16 fragments
// (the decode kernel's key_frag / value_frag, with the MMA roles swapped:
// Q is the A operand, the key and value fragments are B operands), so each
// page's dequantisation serves 16 query rows instead of the decode's grp:
//   * S = Q K^T: A = Q (16 rows x 16 channels, exact fp16, channels in the
//     thread's key-code order), B = the page's key fragments (two 8-token
//     n-tiles); exact fp16 keys as in decode;
//   * online softmax per row in the exp2 domain, causal mask per row;
//   * O += P V with V dequantised to fp16(code * step + zero) -- the value the
//     reference decompress writes -- per token, so values and keys are both
//     the reference's fp16 numbers; P moves from the S accumulator layout to
//     the A layout without shuffles.
// Code words are read with 16-byte loads one page ahead of use (registers),
// the key-group meta one group ahead; no barrier waits, no shared-memory
// staging beyond the warp's key-meta slice.
#include "tkv_frag.cuh"

namespace tkv {

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

template <int D, int NVG>
struct RowState {
  float m[2];          // running max (log2 units) of rows g, g+8
  float l[2];          // this lane's partial sums of p
  float o[D / 8][4];   // O fragments: n-tile nt covers channels 8nt..8nt+7
};

// Online-softmax step for one 16-token tile; s holds raw scores on entry
// (-inf where masked) and the unnormalised weights on return.
template <int D, int NVG>
__device__ __forceinline__ void row_softmax(RowState<D, NVG>& st, float (&s)[2][4], float alpha) {
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

// The key-code words of rows g and g+8 (this thread's channel chunk) and the
// value-code words and per-token value meta of one page, from global memory.
template <int D, int BITS, int NVG>
struct PageWords {
  uint32_t wg[D * BITS / 128], wh[D * BITS / 128];
  uint32_t vw[D * BITS / 64];
  uint32_t vm[4][NVG];  // (step, zero) of tokens 2tig, 2tig+1, 2tig+8, 2tig+9
};

template <int D, int BITS, int G>
__device__ __forceinline__ void load_page(PageWords<D, BITS, Fmt<D, BITS, G>::NVG>& pw,
                                          const uint8_t* pg, int lane) {
  using F = Fmt<D, BITS, G>;
  const int g = lane >> 2, tig = lane & 3;
  constexpr int TB = F::RB / 4;  // key-code bytes per thread per row
  if constexpr (TB == 16) {
    const uint4 x = __ldg(reinterpret_cast<const uint4*>(pg + g * F::RB + tig * 16));
    const uint4 y = __ldg(reinterpret_cast<const uint4*>(pg + (g + 8) * F::RB + tig * 16));
    pw.wg[0] = x.x; pw.wg[1] = x.y; pw.wg[2] = x.z; pw.wg[3] = x.w;
    pw.wh[0] = y.x; pw.wh[1] = y.y; pw.wh[2] = y.z; pw.wh[3] = y.w;
  } else if constexpr (TB == 8) {
    const uint2 x = __ldg(reinterpret_cast<const uint2*>(pg + g * F::RB + tig * 8));
    const uint2 y = __ldg(reinterpret_cast<const uint2*>(pg + (g + 8) * F::RB + tig * 8));
    pw.wg[0] = x.x; pw.wg[1] = x.y;
    pw.wh[0] = y.x; pw.wh[1] = y.y;
  } else {
    pw.wg[0] = __ldg(reinterpret_cast<const uint32_t*>(pg + g * F::RB + tig * 4));
    pw.wh[0] = __ldg(reinterpret_cast<const uint32_t*>(pg + (g + 8) * F::RB + tig * 4));
  }
  const uint8_t* vc = pg + F::V_CODES_OFF;
#pragma unroll
  for (int v = 0; v < F::VWN / F::VW; ++v) {
    if constexpr (F::VW == 4) {
      const uint4 x = __ldg(reinterpret_cast<const uint4*>(vc + (v * 32 + lane) * 16));
      pw.vw[4 * v + 0] = x.x; pw.vw[4 * v + 1] = x.y; pw.vw[4 * v + 2] = x.z; pw.vw[4 * v + 3] = x.w;
    } else {
      const uint2 x = __ldg(reinterpret_cast<const uint2*>(vc + lane * 8));
      pw.vw[0] = x.x; pw.vw[1] = x.y;
    }
  }
  const uint32_t* vm = reinterpret_cast<const uint32_t*>(pg + F::V_META_OFF);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int t = 2 * tig + (k & 1) + 8 * (k >> 1);
#pragma unroll
    for (int vg = 0; vg < F::NVG; ++vg) pw.vm[k][vg] = __ldg(vm + t * F::NVG + vg);
  }
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

#ifndef TKV_PREFILL_MIN_BLOCKS
#define TKV_PREFILL_MIN_BLOCKS 8  // resident warps per SM the register budget targets
#endif

template <int D, int BITS, int G>
__global__ void __launch_bounds__(32, TKV_PREFILL_MIN_BLOCKS) prefill_kernel(PrefillArgs a) {
  using F = Fmt<D, BITS, G>;
  constexpr int NVG = F::NVG, NKB = F::NKB;
  __shared__ __align__(16) uint8_t meta[F::META];  // current key group's [D][step, zero]
  const int lane = threadIdx.x, g = lane >> 2, tig = lane & 3;

  // heavy tiles first: the last row tiles of a chunk see the longest histories
  const int64_t bid = blockIdx.x;
  const int rt = a.n_rt - 1 - (int)(bid % a.n_rt);
  const int bh = (int)(bid / a.n_rt);
  const int b = bh / a.n_kv_heads, h = bh - b * a.n_kv_heads;
  const int L = a.seq_lens[b];
  const int q0 = a.cu_q[b], n = a.cu_q[b + 1] - q0;
  if (L < 0 || L > a.max_blocks * kPage || n < 0 || n > L || q0 < 0 || q0 + n > a.total_q) {
    if (rt == 0 && h == 0 && lane == 0) set_err(a.err, TKV_ERR_BAD_LENGTH);
    return;
  }
  const int rows = n * a.grp, r0 = rt * 16;
  if (r0 >= rows) return;
  // this lane's rows g and g+8 of the tile: token i, q head j; padded rows
  // (beyond the chunk) compute with q = 0 and position L-1, and write nothing
  const int ra = r0 + g, rb = r0 + g + 8;
  const bool va = ra < rows, vb = rb < rows;
  const int ia = va ? ra / a.grp : n - 1, ib = vb ? rb / a.grp : n - 1;
  const int pa = L - n + ia, pb = L - n + ib;
  const int last_row = min(rows - 1, r0 + 15);
  const int kv_end = L - n + last_row / a.grp + 1;  // tokens [0, kv_end) are needed
  const int64_t qa = ((int64_t)(q0 + ia) * a.num_q_heads + h * a.grp + (va ? ra % a.grp : 0)) * D;
  const int64_t qb = ((int64_t)(q0 + ib) * a.num_q_heads + h * a.grp + (vb ? rb % a.grp : 0)) * D;
  const int nq = nq_len(L, a.residual, G);
  const int32_t* bt = a.block_tables + (int64_t)b * a.max_blocks;
  const int n_pages = min(nq, (kv_end + kPage - 1) / kPage * kPage) / kPage;
  const float alpha = a.alpha;

  // every page this tile reads (its pages and the key meta of their whole
  // groups) must be in range
  const int n_read = min(nq / kPage, (n_pages + F::PPG - 1) / F::PPG * F::PPG);
  bool bad = false;
  for (int p = lane; p < n_read; p += 32) {
    const int ph = bt[p];
    bad |= ph < 0 || ph >= a.num_pages;
  }
  if (__any_sync(0xffffffffu, bad)) {
    if (lane == 0) set_err(a.err, TKV_ERR_BAD_PAGE);
    return;
  }
  int row = 0;
  if (kv_end > nq) {
    row = a.seq_slots ? a.seq_slots[b] : b;
    if (row < 0 || row >= a.max_seqs) {
      if (lane == 0) set_err(a.err, TKV_ERR_BAD_SLOT);
      return;
    }
  }

  RowState<D, NVG> st;
  st.m[0] = st.m[1] = -INFINITY;
  st.l[0] = st.l[1] = 0.f;
#pragma unroll
  for (int nt = 0; nt < D / 8; ++nt) st.o[nt][0] = st.o[nt][1] = st.o[nt][2] = st.o[nt][3] = 0.f;

  const uint8_t* pool_h = a.pool + (int64_t)h * F::PB;
  const int64_t page_stride = (int64_t)a.n_kv_heads * F::PB;

  // =================== quantised pages ===================
  if (n_pages > 0) {
    // A operand: q rows g, g+8 as exact f16, channels in the thread's key-code order
    uint32_t aq[NKB][4];
#pragma unroll
    for (int kb = 0; kb < NKB; ++kb)
#pragma unroll
      for (int hi = 0; hi < 2; ++hi) {
        const int c0 = tig * F::CH + kchan<BITS>(kb, hi, 0);
        const int c1 = tig * F::CH + kchan<BITS>(kb, hi, 1);
        aq[kb][2 * hi + 0] = pack_h2(va ? load_qv(a, qa + c0) : 0.f, va ? load_qv(a, qa + c1) : 0.f);
        aq[kb][2 * hi + 1] = pack_h2(vb ? load_qv(a, qb + c0) : 0.f, vb ? load_qv(a, qb + c1) : 0.f);
      }
    // key-group meta: META bytes from the group's PPG pages, one 16-byte
    // vector per lane (lanes beyond META / 16 idle), a group ahead
    constexpr int MV = F::META / 16;
    static_assert(MV <= 32, "key meta of a group fits one vector per lane");
    auto load_meta = [&](int grp) {
      uint4 x = make_uint4(0, 0, 0, 0);
      if (lane < MV) {
        const int slice = lane * 16 / F::KMS, off = lane * 16 % F::KMS;
        const int ph = bt[grp * F::PPG + slice];
        x = __ldg(reinterpret_cast<const uint4*>(pool_h + ph * page_stride + F::BODY + off));
      }
      return x;
    };
    const int ngroups = n_pages / F::PPG + (n_pages % F::PPG ? 1 : 0);
    uint4 mnext = load_meta(0);
    PageWords<D, BITS, NVG> cur, nxt;
    load_page<D, BITS, G>(cur, pool_h + bt[0] * page_stride, lane);
    int pgi = 0;
    for (int grp = 0; grp < ngroups; ++grp) {
      __syncwarp();
      if (lane < MV) reinterpret_cast<uint4*>(meta)[lane] = mnext;
      __syncwarp();
      if (grp + 1 < ngroups) mnext = load_meta(grp + 1);
      uint32_t ks[NKB][2], kz[NKB][2];
      const uint32_t* mwords = reinterpret_cast<const uint32_t*>(meta);
#pragma unroll
      for (int kb = 0; kb < NKB; ++kb)
#pragma unroll
        for (int hi = 0; hi < 2; ++hi) {
          const uint32_t m0 = mwords[tig * F::CH + kchan<BITS>(kb, hi, 0)];
          const uint32_t m1 = mwords[tig * F::CH + kchan<BITS>(kb, hi, 1)];
          ks[kb][hi] = __byte_perm(m0, m1, 0x5410);
          kz[kb][hi] = __byte_perm(m0, m1, 0x7632);
        }
      const int pend = min(n_pages, (grp + 1) * F::PPG);
      for (; pgi < pend; ++pgi) {
        if (pgi + 1 < n_pages) load_page<D, BITS, G>(nxt, pool_h + bt[pgi + 1] * page_stride, lane);
        // ---- S = Q K^T over the page's 16 tokens (two 8-token n-tiles) ----
        float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
        for (int kb = 0; kb < NKB; ++kb) {
          uint32_t r[4];
          switch (kb) {
#define TKV_KF(K)                                                                            \
  case K:                                                                                    \
    key_frag<BITS, (K < NKB ? K : 0)>(cur.wg, cur.wh, ks[K < NKB ? K : 0], kz[K < NKB ? K : 0], \
                                      r);                                                    \
    break;
            TKV_KF(0) TKV_KF(1) TKV_KF(2) TKV_KF(3) TKV_KF(4) TKV_KF(5) TKV_KF(6) TKV_KF(7)
#undef TKV_KF
          }
          mma16816(s[0], aq[kb][0], aq[kb][1], aq[kb][2], aq[kb][3], r[0], r[2]);
          mma16816(s[1], aq[kb][0], aq[kb][1], aq[kb][2], aq[kb][3], r[1], r[3]);
        }
        const int t0 = pgi * kPage;
        if (t0 + kPage - 1 > min(pa, pb)) causal_mask(s, t0, tig, pa, pb);
        row_softmax<D, NVG>(st, s, alpha);
        // ---- O += P V with V = fp16(code * step + zero), the reference
        //      decompress value, per token (step, zero) ----
        const uint32_t a0 = pack_h2(s[0][0], s[0][1]);  // row g,   tokens 2tig, 2tig+1
        const uint32_t a1 = pack_h2(s[0][2], s[0][3]);  // row g+8
        const uint32_t a2 = pack_h2(s[1][0], s[1][1]);  // row g,   tokens 2tig+8, 2tig+9
        const uint32_t a3 = pack_h2(s[1][2], s[1][3]);  // row g+8
#pragma unroll
        for (int vg = 0; vg < NVG; ++vg) {
          const uint32_t s01 = __byte_perm(cur.vm[0][vg], cur.vm[1][vg], 0x5410);
          const uint32_t z01 = __byte_perm(cur.vm[0][vg], cur.vm[1][vg], 0x7632);
          const uint32_t s89 = __byte_perm(cur.vm[2][vg], cur.vm[3][vg], 0x5410);
          const uint32_t z89 = __byte_perm(cur.vm[2][vg], cur.vm[3][vg], 0x7632);
#pragma unroll
          for (int k = 0; k < F::MB_PER_VG; ++k) {
            const int mb = vg * F::MB_PER_VG + k;
            uint32_t r[4];
            switch (mb) {
#define TKV_VF(M)                                      \
  case M:                                              \
    value_frag<BITS, (M < D / 16 ? M : 0)>(cur.vw, r); \
    break;
              TKV_VF(0) TKV_VF(1) TKV_VF(2) TKV_VF(3) TKV_VF(4) TKV_VF(5) TKV_VF(6) TKV_VF(7)
#undef TKV_VF
            }
            // registers 0, 1 hold tokens 2tig, 2tig+1; registers 2, 3 tokens 2tig+8, 2tig+9
            const uint32_t v0 = hfma2(hfma2(r[0], VCode<BITS>::kMul, VCode<BITS>::kAddLo), s01, z01);
            const uint32_t v1 = hfma2(hfma2(r[1], VCode<BITS>::kMul, VCode<BITS>::kAddLo), s01, z01);
            const uint32_t v2 = hfma2(hfma2(r[2], VCode<BITS>::kMul, VCode<BITS>::kAddHi), s89, z89);
            const uint32_t v3 = hfma2(hfma2(r[3], VCode<BITS>::kMul, VCode<BITS>::kAddHi), s89, z89);
            mma16816(st.o[2 * mb], a0, a1, a2, a3, v0, v2);      // channels 16mb .. 16mb+7
            mma16816(st.o[2 * mb + 1], a0, a1, a2, a3, v1, v3);  // channels 16mb+8 .. 16mb+15
          }
        }
        cur = nxt;
      }
    }
  }

  // =================== fp16 ring: tokens [nq, kv_end) ===================
  if (kv_end > nq) {
    constexpr int CHUNK = 2 * F::RBLK;
    const int64_t chunks_per_row = a.ring_cap / kPage;
    const uint8_t* ring_base = reinterpret_cast<const uint8_t*>(a.ring) +
                               (((int64_t)row * a.n_kv_heads + h) * chunks_per_row) * CHUNK;
    // A operand in natural channel order (the ring's fragment layout)
    uint32_t aq[NKB][4];
#pragma unroll
    for (int kb = 0; kb < NKB; ++kb)
#pragma unroll
      for (int hi = 0; hi < 2; ++hi) {
        const int c = 16 * kb + 2 * tig + 8 * hi;
        aq[kb][2 * hi + 0] = pack_h2(va ? load_qv(a, qa + c) : 0.f, va ? load_qv(a, qa + c + 1) : 0.f);
        aq[kb][2 * hi + 1] = pack_h2(vb ? load_qv(a, qb + c) : 0.f, vb ? load_qv(a, qb + c + 1) : 0.f);
      }
    const int n_chunks = (kv_end - nq + kPage - 1) / kPage;
    for (int ci = 0; ci < n_chunks; ++ci) {
      const int t0 = nq + ci * kPage;
      const uint8_t* ck =
          ring_base + (int64_t)((t0 % a.ring_cap) / kPage) * CHUNK;
      const uint8_t* cv = ck + F::RBLK;
      float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
      for (int kb = 0; kb < NKB; ++kb) {
        const uint4 x = __ldg(reinterpret_cast<const uint4*>(ck + (kb * 32 + lane) * 16));
        mma16816(s[0], aq[kb][0], aq[kb][1], aq[kb][2], aq[kb][3], x.x, x.z);
        mma16816(s[1], aq[kb][0], aq[kb][1], aq[kb][2], aq[kb][3], x.y, x.w);
      }
      causal_mask(s, t0, tig, pa, pb);  // also covers stale slots: tokens >= L > p
      row_softmax<D, NVG>(st, s, alpha);
      const uint32_t a0 = pack_h2(s[0][0], s[0][1]);
      const uint32_t a1 = pack_h2(s[0][2], s[0][3]);
      const uint32_t a2 = pack_h2(s[1][0], s[1][1]);
      const uint32_t a3 = pack_h2(s[1][2], s[1][3]);
      // zero the values of tokens past the end (stale ring slots)
      const int tt = t0 + 2 * tig;
      const uint32_t m01 = (tt < L ? 0x0000ffffu : 0u) | (tt + 1 < L ? 0xffff0000u : 0u);
      const uint32_t m23 = (tt + 8 < L ? 0x0000ffffu : 0u) | (tt + 9 < L ? 0xffff0000u : 0u);
#pragma unroll
      for (int mb = 0; mb < D / 16; ++mb) {
        const uint4 x = __ldg(reinterpret_cast<const uint4*>(cv + (mb * 32 + lane) * 16));
        mma16816(st.o[2 * mb], a0, a1, a2, a3, x.x & m01, x.z & m23);
        mma16816(st.o[2 * mb + 1], a0, a1, a2, a3, x.y & m01, x.w & m23);
      }
    }
  }

  // =================== normalise and write ===================
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

template <int D, int BITS, int G>
static int launch_prefill_t(const PrefillArgs& a, int64_t blocks, cudaStream_t stream) {
  prefill_kernel<D, BITS, G><<<(unsigned)blocks, 32, 0, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? TKV_OK : TKV_BACKEND_ERROR;
}

template <int D, int BITS>
static int launch_prefill_g(const PrefillArgs& a, int G, int64_t blocks, cudaStream_t stream) {
  switch (G) {
    case 16: return launch_prefill_t<D, BITS, 16>(a, blocks, stream);
    case 32: return launch_prefill_t<D, BITS, 32>(a, blocks, stream);
    case 64: return launch_prefill_t<D, BITS, 64>(a, blocks, stream);
    case 128: return launch_prefill_t<D, BITS, 128>(a, blocks, stream);
    default: return TKV_NOT_IMPLEMENTED;
  }
}

int launch_prefill(const PrefillArgs& a, int head_dim, int bits, int group, cudaStream_t stream) {
  const int64_t blocks = (int64_t)a.num_seqs * a.n_kv_heads * a.n_rt;
  if (blocks <= 0) return TKV_OK;
  if (blocks > 0x7fffffffLL) return TKV_INVALID_ARGUMENT;
  if (head_dim == 128)
    return bits == 4 ? launch_prefill_g<128, 4>(a, group, blocks, stream)
                     : launch_prefill_g<128, 2>(a, group, blocks, stream);
  if (head_dim == 64)
    return bits == 4 ? launch_prefill_g<64, 4>(a, group, blocks, stream)
                     : launch_prefill_g<64, 2>(a, group, blocks, stream);
  return TKV_NOT_IMPLEMENTED;
}

}  // namespace tkv
