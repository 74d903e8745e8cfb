// tkv_decode.cu -- paged KIVI decode attention on sm_100a.
//
// Replaces paged_attention_v1/v2 (third_party/vllm_kernels/paged_attention_v1.cu,
// paged_attention_v2.cu) for a KIVI-compressed cache, with the attention math
// of the megakernel (third_party/custom_kernels/megakernel.cu:267-350):
// score = scale * q.k, kv_head = q_head / (Hq/Hkv), max-subtracted softmax,
// out = sum p v, fp32 accumulation.
//
// Work decomposition (flash-decoding): grid = (split slot, kv head, sequence).
// A quantised split covers TKV_SPLIT_TOKENS = 512 tokens = 32 pages; each of
// the CTA's 4 warps owns 8 consecutive pages (one 128-token key group at
// G = 128).  The last slot of a sequence covers the fp16 residual ring.  Every
// CTA writes one unnormalised partial (m, l, o[D]) per q head; a second
// kernel merges the partials with the log-sum-exp rule of
// paged_attention_v2.cu:132-170.
//
// Per warp:
//   * lane 0 issues one 1-D TMA bulk copy (cp.async.bulk, no multicast) per
//     (page, head) block into shared memory, completing on an mbarrier;
//   * QK^T runs on the tensor cores as S^T[16 tokens x 8 heads] =
//     K[16 x D] * Q^T[D x 8] with mma.m16n8k16 (f16 in, f32 accumulate).
//     A fragments are built straight from the packed codes in registers: a
//     LOP3 puts a code pair into the mantissa of 1024.0, one HFMA2 recovers
//     the integer codes, a second HFMA2 applies the per-channel (step, zero)
//     -- k = fp16(code * step + zero), the value the reference decompress
//     writes -- and q stays exact in f16, so scores differ from the
//     reference only by fp32 summation order;
//   * online softmax in the exp2 domain with warp shuffles;
//   * PV runs as O^T[D x 8] += V^T[D x 16] * P'^T[16 x 8] where P' = p * step_v
//     (per-token value scale folded into P) and the value zero points are
//     added once per head at the end.  P^T is moved from the S^T accumulator
//     layout into the B-operand layout with 4 shuffles + 2 PRMT.
// Tensor cores are used because at GQA 4 the INT4 cache carries ~7.5 MAC per
// HBM byte, above what the FP32 pipes can issue at HBM speed.
#include "tkv_common.cuh"

namespace tkv {

constexpr int kDecodeWarps = 4;
constexpr int kPagesPerWarp = kSplitPages / kDecodeWarps;  // 8


__device__ __forceinline__ int nq_len(int len, int R, int G) {
  int x = len - R;
  return x > 0 ? G * (x / G) : 0;
}

// Channel (relative to the thread's chunk of D/4 channels) that feeds k-slot
// (2*tig + 8*hi + e) of k-block kb, for the canonical row-major key codes.
template <int BITS>
__device__ __forceinline__ constexpr int kchan(int kb, int hi, int e) {
  return BITS == 4 ? 8 * (kb / 2) + 2 * (kb % 2) + hi + 4 * e
                   : 16 * (kb / 4) + 2 * (kb % 4) + hi + 8 * e;
}

// A-fragment registers (R0..R3 = {a0a1},{a2a3},{a4a5},{a6a7}) of k-block KB:
// fp16 keys dequantised exactly as the reference decompress rounds them,
// k = fp16(code * step + zero), from the thread's key-code words of rows g (wg)
// and g+8 (wh) and the per-channel (step, zero) pairs of this key group.
template <int BITS, int KB>
__device__ __forceinline__ void key_frag(const uint32_t* wg, const uint32_t* wh,
                                         const uint32_t (&ks)[2], const uint32_t (&kz)[2],
                                         uint32_t (&r)[4]) {
  if (BITS == 4) {
    constexpr int j = KB / 2;
    if (KB % 2 == 0) {  // nibbles (0,4) -> hi 0, (1,5) -> hi 1
      r[0] = hfma2(code_pair<0x000F000Fu>(wg[j]), ks[0], kz[0]);
      r[1] = hfma2(code_pair<0x000F000Fu>(wh[j]), ks[0], kz[0]);
      r[2] = hfma2(code_pair<0x00F000F0u>(wg[j]), ks[1], kz[1]);
      r[3] = hfma2(code_pair<0x00F000F0u>(wh[j]), ks[1], kz[1]);
    } else {            // nibbles (2,6) -> hi 0, (3,7) -> hi 1
      const uint32_t g8 = wg[j] >> 8, h8 = wh[j] >> 8;
      r[0] = hfma2(code_pair<0x000F000Fu>(g8), ks[0], kz[0]);
      r[1] = hfma2(code_pair<0x000F000Fu>(h8), ks[0], kz[0]);
      r[2] = hfma2(code_pair<0x00F000F0u>(g8), ks[1], kz[1]);
      r[3] = hfma2(code_pair<0x00F000F0u>(h8), ks[1], kz[1]);
    }
  } else {
    // 2-bit codes i and i+8 pair up; kb = 4j + i/2, hi = i%2
    constexpr int j = KB / 4, u = KB % 4;
    const uint32_t g_ = u < 2 ? wg[j] : (wg[j] >> 8);
    const uint32_t h_ = u < 2 ? wh[j] : (wh[j] >> 8);
    constexpr uint32_t m0 = (u % 2 == 0) ? 0x00030003u : 0x00300030u;  // i = 2u (mod 4)
    constexpr uint32_t m1 = (u % 2 == 0) ? 0x000C000Cu : 0x00C000C0u;  // i = 2u+1 (mod 4)
    r[0] = hfma2(code_pair<m0>(g_), ks[0], kz[0]);
    r[1] = hfma2(code_pair<m0>(h_), ks[0], kz[0]);
    r[2] = hfma2(code_pair<m1>(g_), ks[1], kz[1]);
    r[3] = hfma2(code_pair<m1>(h_), ks[1], kz[1]);
  }
}

// A-fragment registers of m-block MB of V^T from the lane's value-code words.
template <int BITS, int MB>
__device__ __forceinline__ void value_frag(const uint32_t* vw, uint32_t (&r)[4]) {
  if (BITS == 4) {
    const uint32_t w = vw[MB];
    r[0] = ext4<6>(w);   // k=0: rows g,   tokens 2tig, 2tig+1
    r[2] = ext4<2>(w);   // k=1: rows g,   tokens +8
    r[1] = ext4<-2>(w);  // k=2: rows g+8, tokens 2tig, 2tig+1
    r[3] = ext4<-6>(w);  // k=3: rows g+8, tokens +8
  } else {
    const uint32_t w = vw[MB / 2];
    constexpr int base = 4 * (MB % 2);
    r[0] = ext2<6 - 2 * (base + 0)>(w);
    r[2] = ext2<6 - 2 * (base + 1)>(w);
    r[1] = ext2<6 - 2 * (base + 2)>(w);
    r[3] = ext2<6 - 2 * (base + 3)>(w);
  }
}

template <int D, int NVG>
struct WarpState {
  float m[2];          // running max (log2 units) of heads 2tig, 2tig+1
  float l[2];          // partial sum of p over this thread's rows
  float w[NVG][2];     // partial value-zero correction per value group
  float o[D / 16][4];  // O^T accumulator fragments
  __device__ void init() {
    m[0] = m[1] = -INFINITY;
    l[0] = l[1] = 0.f;
#pragma unroll
    for (int v = 0; v < NVG; ++v) w[v][0] = w[v][1] = 0.f;
#pragma unroll
    for (int i = 0; i < D / 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  }
};

// Online-softmax update for one 16-token tile.  s[4]: S^T accumulator
// (rows g, g+8; cols 2tig, 2tig+1), already in log2 units; invalid entries
// must be -inf.  Returns p in s.
template <int D, int NVG>
__device__ __forceinline__ void softmax_tile(WarpState<D, NVG>& st, float (&s)[4]) {
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    float t = fmaxf(s[hh], s[2 + hh]);
    t = fmaxf(t, __shfl_xor_sync(0xffffffffu, t, 4));
    t = fmaxf(t, __shfl_xor_sync(0xffffffffu, t, 8));
    t = fmaxf(t, __shfl_xor_sync(0xffffffffu, t, 16));
    const float mnew = fmaxf(st.m[hh], t);
    // mnew == -inf only when every score so far is masked: keep p = 0 then.
    const float msafe = (mnew == -INFINITY) ? 0.f : mnew;
    const float r = fast_exp2(st.m[hh] - msafe);
    s[hh] = fast_exp2(s[hh] - msafe);
    s[2 + hh] = fast_exp2(s[2 + hh] - msafe);
    if (r != 1.f) {
      st.l[hh] *= r;
#pragma unroll
      for (int v = 0; v < NVG; ++v) st.w[v][hh] *= r;
#pragma unroll
      for (int i = 0; i < D / 16; ++i) {
        st.o[i][hh] *= r;
        st.o[i][2 + hh] *= r;
      }
    }
    st.l[hh] += s[hh] + s[2 + hh];
    st.m[hh] = mnew;
  }
}

// Moves P'^T from the S^T accumulator layout (h2a = row g, h2b = row g+8,
// each (head 2tig, 2tig+1)) into the mma B-operand layout for head g.
__device__ __forceinline__ void p_to_bfrag(uint32_t h2a, uint32_t h2b, int lane, uint32_t& b01,
                                           uint32_t& b23) {
  const int g = lane >> 2, tig = lane & 3;
  const int src0 = (2 * tig) * 4 + (g >> 1), src1 = (2 * tig + 1) * 4 + (g >> 1);
  const uint32_t sel = (g & 1) ? 0x7632u : 0x5410u;
  const uint32_t x0 = __shfl_sync(0xffffffffu, h2a, src0);
  const uint32_t x1 = __shfl_sync(0xffffffffu, h2a, src1);
  const uint32_t x2 = __shfl_sync(0xffffffffu, h2b, src0);
  const uint32_t x3 = __shfl_sync(0xffffffffu, h2b, src1);
  b01 = __byte_perm(x0, x1, sel);
  b23 = __byte_perm(x2, x3, sel);
}

__device__ __forceinline__ float load_q(const DecodeArgs& a, int64_t idx) {
  if (a.q_bf16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(a.q)[idx]);
  return __half2float(reinterpret_cast<const __half*>(a.q)[idx]);
}

// ---------------------------------------------------------------------------
// quantised pages of one warp
// ---------------------------------------------------------------------------
template <int D, int BITS, int NVG>
__device__ void warp_quantized(const DecodeArgs& a, WarpState<D, NVG>& st, uint8_t* wsmem,
                               uint64_t* bars, int b, int h, int page_lo, int n_pages,
                               bool issue) {
  const int lane = threadIdx.x & 31, g = lane >> 2, tig = lane & 3;
  constexpr int NKB = D / 16;
  constexpr int CH = D / 4;          // channels per thread chunk
  constexpr int RB = D * BITS / 8;   // key-code bytes per token row
  constexpr int TW = RB / 16;        // key-code words per thread per row (RB/4/4)
  constexpr int VWN = D * BITS / 64; // value-code words per lane
  constexpr int VW = VWN < 4 ? VWN : 4;
  constexpr int MB_PER_VG = (D / 16) / NVG;
  const int64_t pb = a.page_bytes;
  const int32_t* bt = a.block_tables + (int64_t)b * a.max_blocks;

  // ---- issue all page loads of this warp (lane 0) ----
  if (issue && lane == 0) {
    for (int i = 0; i < n_pages; ++i) {
      const int phys = bt[page_lo + i];
      if (phys < 0 || phys >= a.num_pages) {
        set_err(a.err, TKV_ERR_BAD_PAGE);
        mbar_arrive(&bars[i]);
      } else {
        mbar_arrive_expect_tx(&bars[i], static_cast<uint32_t>(pb));
        bulk_g2s(wsmem + (int64_t)i * pb, a.pool + ((int64_t)phys * a.n_kv_heads + h) * pb,
                 static_cast<uint32_t>(pb), &bars[i]);
      }
    }
  }

  // ---- B operand: q of head g as exact f16, in this thread's key-channel
  //      order (k-slot 2tig+8hi+e <-> channel tig*CH + kchan(kb, hi, e)) ----
  const int hq = h * a.grp + g;
  uint32_t bq[NKB][2];
  {
    const bool ok = g < a.grp;
    const int64_t qb = ((int64_t)b * a.num_q_heads + hq) * D + tig * CH;
#pragma unroll
    for (int kb = 0; kb < NKB; ++kb)
#pragma unroll
      for (int hi = 0; hi < 2; ++hi) {
        const float f0 = ok ? load_q(a, qb + kchan<BITS>(kb, hi, 0)) : 0.f;
        const float f1 = ok ? load_q(a, qb + kchan<BITS>(kb, hi, 1)) : 0.f;
        bq[kb][hi] = pack_h2(f0, f1);
      }
  }
  const bool hv0 = 2 * tig < a.grp, hv1 = 2 * tig + 1 < a.grp;

  const int pages_per_group = a.group / kPage;
  for (int p0 = 0; p0 < n_pages; p0 += pages_per_group) {
    // wait for the whole key group (its meta is spread over its pages)
    for (int i = 0; i < pages_per_group; ++i) mbar_wait(&bars[p0 + i], 0, a.err);

    // ---- per-channel (step, zero) pairs of this key group, as f16x2 ----
    uint32_t ks[NKB][2], kz[NKB][2];
#pragma unroll
    for (int kb = 0; kb < NKB; ++kb)
#pragma unroll
      for (int hi = 0; hi < 2; ++hi) {
        uint32_t mw[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int c = tig * CH + kchan<BITS>(kb, hi, e);
          const int byte = c * 4;
          const int pi = byte / a.k_meta_slice, off = byte % a.k_meta_slice;
          mw[e] = *reinterpret_cast<const uint32_t*>(wsmem + (int64_t)(p0 + pi) * pb +
                                                     a.k_meta_off + off);
        }
        ks[kb][hi] = __byte_perm(mw[0], mw[1], 0x5410);  // (step c0, step c1)
        kz[kb][hi] = __byte_perm(mw[0], mw[1], 0x7632);  // (zero c0, zero c1)
      }

    for (int pi = 0; pi < pages_per_group; ++pi) {
      const uint8_t* pg = wsmem + (int64_t)(p0 + pi) * pb;
      // ---- S^T = K Q^T (exact fp16 products, fp32 accumulation) ----
      uint32_t wg[TW > 0 ? TW : 1], wh[TW > 0 ? TW : 1];
      {
        const uint8_t* kc = pg + a.k_codes_off;
        if (RB / 4 == 16) {  // 16 bytes per thread per row
          const uint4 x = *reinterpret_cast<const uint4*>(kc + g * RB + tig * 16);
          const uint4 y = *reinterpret_cast<const uint4*>(kc + (g + 8) * RB + tig * 16);
          wg[0] = x.x; wg[1] = x.y; wg[2] = x.z; wg[3] = x.w;
          wh[0] = y.x; wh[1] = y.y; wh[2] = y.z; wh[3] = y.w;
        } else if (RB / 4 == 8) {
          const uint2 x = *reinterpret_cast<const uint2*>(kc + g * RB + tig * 8);
          const uint2 y = *reinterpret_cast<const uint2*>(kc + (g + 8) * RB + tig * 8);
          wg[0] = x.x; wg[1] = x.y;
          wh[0] = y.x; wh[1] = y.y;
        } else {
          wg[0] = *reinterpret_cast<const uint32_t*>(kc + g * RB + tig * 4);
          wh[0] = *reinterpret_cast<const uint32_t*>(kc + (g + 8) * RB + tig * 4);
        }
      }
      float s[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int kb = 0; kb < NKB; ++kb) {
        uint32_t r[4];
        switch (kb) {  // template dispatch on the unrolled index
#define TKV_KF(K) \
  case K:         \
    key_frag<BITS, (K < NKB ? K : 0)>(wg, wh, ks[K < NKB ? K : 0], kz[K < NKB ? K : 0], r); \
    break;
          TKV_KF(0) TKV_KF(1) TKV_KF(2) TKV_KF(3) TKV_KF(4) TKV_KF(5) TKV_KF(6) TKV_KF(7)
#undef TKV_KF
        }
        mma16816(s, r[0], r[1], r[2], r[3], bq[kb][0], bq[kb][1]);
      }
      s[0] = hv0 ? s[0] * a.alpha : -INFINITY;
      s[1] = hv1 ? s[1] * a.alpha : -INFINITY;
      s[2] = hv0 ? s[2] * a.alpha : -INFINITY;
      s[3] = hv1 ? s[3] * a.alpha : -INFINITY;
      softmax_tile<D, NVG>(st, s);

      // ---- O^T += V^T P'^T ----
      uint32_t vw[VWN];
      {
        const uint8_t* vc = pg + a.v_codes_off;
#pragma unroll
        for (int v = 0; v < VWN / VW; ++v) {
          if (VW == 4) {
            const uint4 x = *reinterpret_cast<const uint4*>(vc + (v * 32 + lane) * 16);
            vw[4 * v + 0] = x.x; vw[4 * v + 1] = x.y; vw[4 * v + 2] = x.z; vw[4 * v + 3] = x.w;
          } else {
            const uint2 x = *reinterpret_cast<const uint2*>(vc + lane * 8);
            vw[0] = x.x; vw[1] = x.y;
          }
        }
      }
      const uint32_t* vm = reinterpret_cast<const uint32_t*>(pg + a.v_meta_off);
#pragma unroll
      for (int vg = 0; vg < NVG; ++vg) {
        const float2 sza = unpack_h2(vm[g * NVG + vg]);        // token g
        const float2 szb = unpack_h2(vm[(g + 8) * NVG + vg]);  // token g+8
        const uint32_t h2a = pack_h2(s[0] * sza.x, s[1] * sza.x);
        const uint32_t h2b = pack_h2(s[2] * szb.x, s[3] * szb.x);
        const float2 ra = unpack_h2(h2a), rb = unpack_h2(h2b);
        st.w[vg][0] += s[0] * sza.y + s[2] * szb.y - 16.f * (ra.x + rb.x);
        st.w[vg][1] += s[1] * sza.y + s[3] * szb.y - 16.f * (ra.y + rb.y);
        uint32_t b01, b23;
        p_to_bfrag(h2a, h2b, lane, b01, b23);
#pragma unroll
        for (int k = 0; k < MB_PER_VG; ++k) {
          const int mb = vg * MB_PER_VG + k;
          uint32_t r[4];
          switch (mb) {
#define TKV_VF(M) \
  case M:         \
    value_frag<BITS, (M < D / 16 ? M : 0)>(vw, r); \
    break;
            TKV_VF(0) TKV_VF(1) TKV_VF(2) TKV_VF(3) TKV_VF(4) TKV_VF(5) TKV_VF(6) TKV_VF(7)
#undef TKV_VF
          }
          mma16816(st.o[mb], r[0], r[1], r[2], r[3], b01, b23);
        }
      }
    }
  }
  // finalise: O^T = 16 * acc + per-head value-zero correction
#pragma unroll
  for (int vg = 0; vg < NVG; ++vg)
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      float w = st.w[vg][hh];
      w += __shfl_xor_sync(0xffffffffu, w, 4);
      w += __shfl_xor_sync(0xffffffffu, w, 8);
      w += __shfl_xor_sync(0xffffffffu, w, 16);
      st.w[vg][hh] = w;
    }
#pragma unroll
  for (int mb = 0; mb < D / 16; ++mb) {
    const int vg = mb / MB_PER_VG;
#pragma unroll
    for (int i = 0; i < 4; ++i) st.o[mb][i] = fmaf(16.f, st.o[mb][i], st.w[vg][i & 1]);
  }
}

// ---------------------------------------------------------------------------
// fp16 residual ring of one sequence: this warp's 16-token chunks
// ---------------------------------------------------------------------------
template <int D, int NVG>
__device__ void warp_residual(const DecodeArgs& a, WarpState<D, NVG>& st, uint8_t* wsmem,
                              uint64_t* bars, int b, int h, int row, int nq, int len) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, tig = lane & 3;
  constexpr int NKB = D / 16;
  constexpr int CHUNK_BYTES = 2 * kPage * D * 2;  // K block + V block
  const int n_chunks = (len - nq + kPage - 1) / kPage;
  const int64_t chunks_per_row = a.ring_cap / kPage;
  const uint8_t* ring_base =
      reinterpret_cast<const uint8_t*>(a.ring) +
      (((int64_t)row * a.n_kv_heads + h) * chunks_per_row) * CHUNK_BYTES;
  // my chunks: warp, warp + 4, ...
  const int mine = n_chunks > warp ? (n_chunks - warp + kDecodeWarps - 1) / kDecodeWarps : 0;
  auto issue = [&](int k) {
    if (lane == 0) {
      const int ci = warp + k * kDecodeWarps;
      const int tok = nq + ci * kPage;
      const int chunk = (tok % a.ring_cap) / kPage;
      mbar_arrive_expect_tx(&bars[k & 1], CHUNK_BYTES);
      bulk_g2s(wsmem + (k & 1) * CHUNK_BYTES, ring_base + (int64_t)chunk * CHUNK_BYTES,
               CHUNK_BYTES, &bars[k & 1]);
    }
  };
  if (mine > 0) issue(0);
  if (mine > 1) issue(1);

  // Q fragments (identity channel order, exact f16), head g; the softmax scale
  // is applied to the fp32 accumulator
  const int hq = h * a.grp + g;
  const bool hok = g < a.grp;
  uint32_t bq[NKB][2];
  {
    const int64_t qb = ((int64_t)b * a.num_q_heads + hq) * D;
#pragma unroll
    for (int kb = 0; kb < NKB; ++kb)
#pragma unroll
      for (int hi = 0; hi < 2; ++hi) {
        const int c = 16 * kb + 2 * tig + 8 * hi;
        const float f0 = hok ? load_q(a, qb + c) : 0.f;
        const float f1 = hok ? load_q(a, qb + c + 1) : 0.f;
        bq[kb][hi] = pack_h2(f0, f1);
      }
  }
  const bool hv0 = 2 * tig < a.grp, hv1 = 2 * tig + 1 < a.grp;

  for (int k = 0; k < mine; ++k) {
    mbar_wait(&bars[k & 1], (k >> 1) & 1, a.err);
    const uint8_t* ck = wsmem + (k & 1) * CHUNK_BYTES;
    const uint8_t* cv = ck + CHUNK_BYTES / 2;
    const int ci = warp + k * kDecodeWarps;
    const int tb = nq + ci * kPage;  // first token of the chunk
    const bool vg0 = tb + g < len, vg8 = tb + g + 8 < len;
    float s[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int kb = 0; kb < NKB; ++kb) {
      const uint4 x = *reinterpret_cast<const uint4*>(ck + (kb * 32 + lane) * 16);
      mma16816(s, x.x, x.y, x.z, x.w, bq[kb][0], bq[kb][1]);
    }
    s[0] = (hv0 && vg0) ? s[0] * a.alpha : -INFINITY;
    s[1] = (hv1 && vg0) ? s[1] * a.alpha : -INFINITY;
    s[2] = (hv0 && vg8) ? s[2] * a.alpha : -INFINITY;
    s[3] = (hv1 && vg8) ? s[3] * a.alpha : -INFINITY;
    softmax_tile<D, NVG>(st, s);
    const uint32_t h2a = pack_h2(s[0], s[1]);
    const uint32_t h2b = pack_h2(s[2], s[3]);
    uint32_t b01, b23;
    p_to_bfrag(h2a, h2b, lane, b01, b23);
    // zero the V^T columns of tokens past the end (their ring slots may hold
    // stale data, and 0 * inf would poison the sum)
    const int t0 = tb + 2 * tig;
    const uint32_t m01 = (t0 < len ? 0x0000ffffu : 0u) | (t0 + 1 < len ? 0xffff0000u : 0u);
    const uint32_t m23 = (t0 + 8 < len ? 0x0000ffffu : 0u) | (t0 + 9 < len ? 0xffff0000u : 0u);
#pragma unroll
    for (int mb = 0; mb < D / 16; ++mb) {
      const uint4 x = *reinterpret_cast<const uint4*>(cv + (mb * 32 + lane) * 16);
      mma16816(st.o[mb], x.x & m01, x.y & m01, x.z & m23, x.w & m23, b01, b23);
    }
    __syncwarp();
    if (k + 2 < mine) issue(k + 2);
  }
}

// ---------------------------------------------------------------------------
// split kernel
// ---------------------------------------------------------------------------
template <int D, int BITS, int NVG>
__global__ void __launch_bounds__(kDecodeWarps * 32, 3) decode_split_kernel(DecodeArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int slot = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, tig = lane & 3;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);  // 8 per warp
  uint8_t* wsmem = smem + 512 + warp * a.warp_smem;
  uint64_t* wbars = bars + warp * 8;

  const int len = a.seq_lens[b];
  const int64_t ml_base = ((int64_t)slot * a.num_seqs + b) * a.num_q_heads + h * a.grp;
  if (len < 0 || len > a.max_blocks * kPage) {
    if (threadIdx.x == 0) set_err(a.err, TKV_ERR_BAD_LENGTH);
  }
  const bool len_ok = len >= 0 && len <= a.max_blocks * kPage;
  const int nq = len_ok ? nq_len(len, a.residual, a.group) : 0;
  const int n_qsplit = a.split_hi - a.split_lo;
  const bool is_res = a.include_residual && slot == n_qsplit;

  // which work does this CTA have?
  int page_lo = 0, n_pages = 0;
  int row = 0;
  bool work = false;
  if (len_ok && !is_res && slot < n_qsplit) {
    const int sp = a.split_lo + slot;
    page_lo = sp * kSplitPages + warp * kPagesPerWarp;
    const int nqp = nq / kPage;
    n_pages = min(kPagesPerWarp, nqp - page_lo);
    if (n_pages < 0) n_pages = 0;
    work = sp * kSplitPages < nqp;
  } else if (len_ok && is_res && len > nq) {
    row = a.seq_slots ? a.seq_slots[b] : b;
    if (row < 0 || row >= a.max_seqs) {
      if (threadIdx.x == 0) set_err(a.err, TKV_ERR_BAD_SLOT);
    } else {
      work = true;
    }
  }
  if (!work) {  // empty slot: m = -inf, l = 0 for every q head of this kv head
    for (int j = threadIdx.x; j < a.grp; j += blockDim.x) {
      a.part_ml[(ml_base + j) * 2 + 0] = -INFINITY;
      a.part_ml[(ml_base + j) * 2 + 1] = 0.f;
    }
    return;
  }

  if (lane == 0) {
    for (int i = 0; i < 8; ++i) mbar_init(&wbars[i], 1);
    fence_mbar_init();
  }
  __syncwarp();

  WarpState<D, NVG> st;
  st.init();
  if (!is_res) {
    if (n_pages > 0)
      warp_quantized<D, BITS, NVG>(a, st, wsmem, wbars, b, h, page_lo, n_pages, true);
  } else {
    warp_residual<D, NVG>(a, st, wsmem, wbars, b, h, row, nq, len);
  }

  // ---- reduce l over the 8 row groups, then merge the 4 warps ----
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    float l = st.l[hh];
    l += __shfl_xor_sync(0xffffffffu, l, 4);
    l += __shfl_xor_sync(0xffffffffu, l, 8);
    l += __shfl_xor_sync(0xffffffffu, l, 16);
    st.l[hh] = l;
  }
  __syncwarp();
  // per-warp staging (reuses this warp's page buffers): m[8], l[8], o[8][D]
  float* stg = reinterpret_cast<float*>(wsmem);
  if (g == 0) {
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      stg[2 * tig + hh] = st.m[hh];
      stg[8 + 2 * tig + hh] = st.l[hh];
    }
  }
#pragma unroll
  for (int mb = 0; mb < D / 16; ++mb)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int c = 16 * mb + g + ((i >> 1) << 3);
      const int hd = 2 * tig + (i & 1);
      stg[16 + hd * D + c] = st.o[mb][i];
    }
  __syncthreads();
  for (int idx = threadIdx.x; idx < a.grp * D; idx += blockDim.x) {
    const int hd = idx / D, c = idx % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kDecodeWarps; ++w) {
      const float* sw = reinterpret_cast<const float*>(smem + 512 + w * a.warp_smem);
      M = fmaxf(M, sw[hd]);
    }
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kDecodeWarps; ++w) {
        const float* sw = reinterpret_cast<const float*>(smem + 512 + w * a.warp_smem);
        const float mw = sw[hd];
        if (mw == -INFINITY) continue;
        const float f = fast_exp2(mw - M);
        L = fmaf(sw[8 + hd], f, L);
        O = fmaf(sw[16 + hd * D + c], f, O);
      }
    }
    a.part_o[(ml_base + hd) * D + c] = O;
    if (c == 0) {
      a.part_ml[(ml_base + hd) * 2 + 0] = M;
      a.part_ml[(ml_base + hd) * 2 + 1] = L;
    }
  }
}

// ---------------------------------------------------------------------------
// merge kernel: one CTA per (q head, sequence)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(128) merge_kernel(const float* __restrict__ part_ml,
                                                    const float* __restrict__ part_o, int n_slots,
                                                    int num_seqs, int num_q_heads, int D,
                                                    void* __restrict__ out, int out_dtype) {
  const int hq = blockIdx.x, b = blockIdx.y;
  const int64_t stride = (int64_t)num_seqs * num_q_heads;
  const int64_t i0 = (int64_t)b * num_q_heads + hq;
  float M = -INFINITY;
  for (int s = 0; s < n_slots; ++s) M = fmaxf(M, part_ml[(s * stride + i0) * 2]);
  float L = 0.f;
  if (M != -INFINITY)
    for (int s = 0; s < n_slots; ++s) {
      const float m = part_ml[(s * stride + i0) * 2];
      if (m != -INFINITY) L = fmaf(part_ml[(s * stride + i0) * 2 + 1], fast_exp2(m - M), L);
    }
  const float inv = L > 0.f ? 1.f / L : 0.f;
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    float O = 0.f;
    if (M != -INFINITY)
      for (int s = 0; s < n_slots; ++s) {
        const float m = part_ml[(s * stride + i0) * 2];
        if (m != -INFINITY) O = fmaf(part_o[(s * stride + i0) * D + c], fast_exp2(m - M), O);
      }
    const float v = O * inv;
    const int64_t oi = i0 * D + c;
    if (out_dtype == TKV_F32)
      static_cast<float*>(out)[oi] = v;
    else if (out_dtype == TKV_BF16)
      static_cast<__nv_bfloat16*>(out)[oi] = __float2bfloat16_rn(v);
    else
      static_cast<__half*>(out)[oi] = __float2half_rn(v);
  }
}

// ---------------------------------------------------------------------------
// host launchers
// ---------------------------------------------------------------------------
template <int D, int BITS, int NVG>
static int launch_split_t(const DecodeArgs& a, dim3 grid, size_t smem, cudaStream_t stream) {
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(decode_split_kernel<D, BITS, NVG>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             227 * 1024) != cudaSuccess)
      return TKV_BACKEND_ERROR;
    attr = true;
  }
  decode_split_kernel<D, BITS, NVG><<<grid, kDecodeWarps * 32, smem, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? TKV_OK : TKV_BACKEND_ERROR;
}

template <int D, int BITS>
static int launch_split_d(const DecodeArgs& a, int nvg, dim3 grid, size_t smem,
                          cudaStream_t stream) {
  switch (nvg) {
    case 1: return launch_split_t<D, BITS, 1>(a, grid, smem, stream);
    case 2: return launch_split_t<D, BITS, 2>(a, grid, smem, stream);
    case 4: return launch_split_t<D, BITS, 4>(a, grid, smem, stream);
    case 8:
      if constexpr (D / 16 >= 8) return launch_split_t<D, BITS, 8>(a, grid, smem, stream);
      break;
  }
  return TKV_NOT_IMPLEMENTED;
}

int warp_smem_bytes(int head_dim, int64_t page_bytes) {
  const int64_t quant = kPagesPerWarp * page_bytes;
  const int64_t resid = 2 * (2 * kPage * head_dim * 2);
  const int64_t stage = (16 + 8 * head_dim) * 4;
  int64_t m = quant > resid ? quant : resid;
  m = m > stage ? m : stage;
  return static_cast<int>((m + 127) / 128 * 128);
}

int launch_decode_splits(DecodeArgs a, int head_dim, int bits, int n_vgroups, cudaStream_t stream) {
  a.warp_smem = warp_smem_bytes(head_dim, a.page_bytes);
  const size_t smem = 512 + static_cast<size_t>(kDecodeWarps) * a.warp_smem;
  if (smem > 227 * 1024) return TKV_NOT_IMPLEMENTED;
  dim3 grid(a.n_slots, a.n_kv_heads, a.num_seqs);
  if (head_dim == 128)
    return bits == 4 ? launch_split_d<128, 4>(a, n_vgroups, grid, smem, stream)
                     : launch_split_d<128, 2>(a, n_vgroups, grid, smem, stream);
  if (head_dim == 64)
    return bits == 4 ? launch_split_d<64, 4>(a, n_vgroups, grid, smem, stream)
                     : launch_split_d<64, 2>(a, n_vgroups, grid, smem, stream);
  return TKV_NOT_IMPLEMENTED;
}

int launch_merge(const float* part_ml, const float* part_o, int n_slots, int num_seqs,
                 int num_q_heads, int head_dim, void* out, int out_dtype, cudaStream_t stream) {
  dim3 grid(num_q_heads, num_seqs);
  merge_kernel<<<grid, 128, 0, stream>>>(part_ml, part_o, n_slots, num_seqs, num_q_heads,
                                         head_dim, out, out_dtype);
  return cudaGetLastError() == cudaSuccess ? TKV_OK : TKV_BACKEND_ERROR;
}

}  // namespace tkv
