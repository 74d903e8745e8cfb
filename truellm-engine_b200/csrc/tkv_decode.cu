// tkv_decode.cu -- paged KIVI decode attention on sm_100a.
//
// Replaces paged_attention_v1/v2 (third_party/vllm_kernels/paged_attention_v1.cu,
// paged_attention_v2.cu) for a KIVI-compressed cache, with the attention math
// of the megakernel (third_party/custom_kernels/megakernel.cu:267-350):
// score = scale * q.k, kv_head = q_head / (Hq/Hkv), max-subtracted softmax,
// out = sum p v, fp32 accumulation.
//
// Work decomposition (flash-decoding): a work item is (split slot, sequence,
// kv head).  A quantised split covers TKV_SPLIT_TOKENS = 512 tokens = 32
// pages; one more slot per sequence covers the fp16 residual ring.  The split
// kernel is persistent: one warp per CTA, as many CTAs as fit on the GPU, each
// taking items from a global counter until none are left.  Every item leaves
// one unnormalised partial (m, l, o[D]) per q head; a second kernel merges the
// partials with the log-sum-exp rule of paged_attention_v2.cu:132-170.
//
// Per warp:
//   * a 6-stage ring in shared memory, filled by 1-D TMA bulk copies
//     (cp.async.bulk, no multicast) of each page's codes + value meta, one
//     mbarrier per stage; the key-group meta slices are fetched one group
//     ahead into a double buffer;
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
#include <atomic>

#include "tkv_decode_common.cuh"

namespace tkv {

// Writes this warp's partial (m, l, o[D]) for the q heads of kv head h.
template <int D, int NVG>
__device__ __forceinline__ void write_partial(const DecodeArgs& a, WarpState<D, NVG>& st,
                                              int64_t ml_base, float oscale) {
  const int lane = threadIdx.x & 31, g = lane >> 2, tig = lane & 3;
  constexpr int MB_PER_VG = (D / 16) / NVG;
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    float l = st.l[hh];
    l += __shfl_xor_sync(0xffffffffu, l, 4);
    l += __shfl_xor_sync(0xffffffffu, l, 8);
    l += __shfl_xor_sync(0xffffffffu, l, 16);
    st.l[hh] = l;
#pragma unroll
    for (int vg = 0; vg < NVG; ++vg) {
      float w = st.w[vg][hh];
      w += __shfl_xor_sync(0xffffffffu, w, 4);
      w += __shfl_xor_sync(0xffffffffu, w, 8);
      w += __shfl_xor_sync(0xffffffffu, w, 16);
      st.w[vg][hh] = w;
    }
  }
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    const int hd = 2 * tig + hh;
    if (hd >= a.grp) continue;
    float* po = a.part_o + (ml_base + hd) * D;
#pragma unroll
    for (int mb = 0; mb < D / 16; ++mb) {
      const int vg = mb / MB_PER_VG;
      // O^T = oscale * acc + value-zero correction (0 for the fp16 ring)
      const float o0 = fmaf(oscale, st.o[mb][hh], st.w[vg][hh]);
      const float o1 = fmaf(oscale, st.o[mb][2 + hh], st.w[vg][hh]);
      po[16 * mb + g] = o0;
      po[16 * mb + g + 8] = o1;
    }
    if (g == 0) {
      a.part_ml[(ml_base + hd) * 2 + 0] = st.m[hh];
      a.part_ml[(ml_base + hd) * 2 + 1] = st.l[hh];
    }
  }
}

// ---------------------------------------------------------------------------
// persistent split kernel: each resident warp takes work items
// (split slot, sequence, kv head) from a global counter until none are left
// ---------------------------------------------------------------------------
#ifndef TKV_DECODE_MIN_BLOCKS
#define TKV_DECODE_MIN_BLOCKS 12  // resident warps per SM the register budget targets
#endif
#ifndef TKV_QK_CHAINS
#define TKV_QK_CHAINS 1  // independent accumulator chains per page in QK^T
#endif

template <int D, int BITS, int G>
__global__ void __launch_bounds__(32, TKV_DECODE_MIN_BLOCKS) decode_warp_kernel(DecodeArgs a) {
  using F = Fmt<D, BITS, G>;
  constexpr int NVG = F::NVG, NP = F::NP, ST = F::ST, SB = F::SB;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);  // ST ring + 2 meta barriers
  uint8_t* ring = smem + 128;
  uint8_t* meta = ring + ST * SB;  // 2 x key-group meta [D][step, zero]
  const int lane = threadIdx.x, g = lane >> 2, tig = lane & 3;
  const bool hok = g < a.grp;
  const int n_qsplit = a.split_hi - a.split_lo;
  const int per_slot = a.num_seqs * a.n_kv_heads;
  const float alpha = a.alpha;
  const uint64_t pol = l2_evict_first_policy();  // cache pages and ring: read once

  if (lane == 0) {
    for (int i = 0; i < ST + 2; ++i) mbar_init(&bars[i], 1);
    fence_mbar_init();
  }
  __syncwarp();
  // ring and meta-buffer positions carry over from item to item
  int stage = 0;
  uint32_t phase = 0;
  int gcount = 0;  // key groups consumed so far (meta buffer = gcount & 1)
  // After a bounded wait gives up (TKV_ERR_TIMEOUT set) the warp waits no
  // more, finishes its current item without waiting and takes no new one, so
  // a stuck copy costs one timeout per warp, not one per stage.
  bool dead = false;

  // After an item's partial is written: with fuse_merge, the warp that
  // finishes the last of the nv + 1 written items of (sequence b, kv head h)
  // (its nv quantised splits that hold pages, then the residual) merges them
  // into out and resets the pair's counter for the next launch.
  auto item_done = [&](int b, int h, int nv) {
    if (!a.fuse_merge) return;
    __syncwarp();
    __threadfence();  // publish this warp's partial before counting it
    unsigned int old = 0;
    if (lane == 0) old = atomicAdd(&a.bh_count[b * a.n_kv_heads + h], 1u);
    old = __shfl_sync(0xffffffffu, old, 0);
    if (old != static_cast<unsigned int>(nv)) return;
    __threadfence();  // every other warp's partial of this pair is visible now
    if (lane == 0) a.bh_count[b * a.n_kv_heads + h] = 0u;
    const int64_t i0 = (int64_t)b * a.num_q_heads + h * a.grp;
    merge_heads<4>(a.part_ml, a.part_o, a.n_slots, nv, nv + 1,
                   (int64_t)a.num_seqs * a.num_q_heads, i0, a.grp, D, a.out, a.out_dtype, lane,
                   i0);
  };

  for (;;) {
    if (dead) break;
    int item = 0;
    if (lane == 0) item = static_cast<int>(atomicAdd(&a.work[0], 1u));
    item = __shfl_sync(0xffffffffu, item, 0);
    if (item >= a.n_items) break;
    // residual slot first (largest items), then quantised splits in order
    const int sidx = item / per_slot, rem = item - sidx * per_slot;
    const int b = rem / a.n_kv_heads, h = rem - b * a.n_kv_heads;
    const bool is_res = a.include_residual && sidx == 0;
    const int slot = a.include_residual ? (sidx == 0 ? n_qsplit : sidx - 1) : sidx;
    const int64_t ml_base = ((int64_t)slot * a.num_seqs + b) * a.num_q_heads + h * a.grp;
    const int len = a.seq_lens[b];
    const bool len_ok = len >= 0 && len <= a.max_blocks * kPage;
    if (!len_ok && lane == 0 && h == 0) set_err(a.err, TKV_ERR_BAD_LENGTH);
    const int nq = len_ok ? nq_len(len, a.residual, G) : 0;
    const int32_t* bt = a.block_tables + (int64_t)b * a.max_blocks;
    // quantised splits of this sequence that hold pages; the fused merge
    // counts and reads only those and the residual slot
    const int nv =
        max(0, min(n_qsplit, (nq / kPage + a.split_pages - 1) / a.split_pages - a.split_lo));
    const bool real = is_res || slot < nv;

    int n_units = 0, page_lo = 0, row = 0, my_phys = 0;
    if (len_ok && !is_res) {
      page_lo = (a.split_lo + slot) * a.split_pages;
      n_units = min(a.split_pages, nq / kPage - page_lo);  // pages, a multiple of PPG
      if (n_units > 0) {
        my_phys = lane < n_units ? bt[page_lo + lane] : 0;
        if (__any_sync(0xffffffffu, my_phys < 0 || my_phys >= a.num_pages)) {
          if (lane == 0) set_err(a.err, TKV_ERR_BAD_PAGE);
          n_units = 0;
        }
      }
    } else if (len_ok && is_res && len > nq) {
      row = a.seq_slots ? a.seq_slots[b] : b;
      if (row < 0 || row >= a.max_seqs) {
        if (lane == 0) set_err(a.err, TKV_ERR_BAD_SLOT);
      } else {
        n_units = ((len - nq + kPage - 1) / kPage) * 2;  // K block + V block per chunk
      }
    }
    if (n_units <= 0) {
      // the fused merge reads only written slots, the standalone merge every slot
      if (lane < a.grp && (real || !a.fuse_merge)) {
        a.part_ml[(ml_base + lane) * 2 + 0] = -INFINITY;
        a.part_ml[(ml_base + lane) * 2 + 1] = 0.f;
      }
      if (real) item_done(b, h, nv);
      continue;
    }

    WarpState<D, NVG> st;
    st.init();
    const int64_t qrow = ((int64_t)b * a.num_q_heads + h * a.grp + g) * D;

    if (!is_res) {
      // =================== quantised split ===================
      const int n_steps = n_units / NP;
      const uint8_t* pool_h = a.pool + (int64_t)h * F::PB;
      const int64_t page_stride = (int64_t)a.n_kv_heads * F::PB;
      // step j (NP pages) goes to ring stage stg: lane 0 posts the byte count,
      // lanes 0..NP-1 issue one page copy each (one warp instruction)
      auto issue_step = [&](int j, int stg) {
        const int ph = __shfl_sync(0xffffffffu, my_phys, (j * NP + lane) & 31);
        if (lane == 0) mbar_arrive_expect_tx(&bars[stg], NP * F::BODY);
        __syncwarp();
        if (lane < NP)
          bulk_g2s_hint(ring + stg * SB + lane * F::BODY, pool_h + ph * page_stride, F::BODY,
                        &bars[stg], pol);
      };
      // the group's key-meta slices, lanes 0..PPG-1 one slice each
      auto issue_meta = [&](int grp, int buf) {
        const int ph = __shfl_sync(0xffffffffu, my_phys, (grp * F::PPG + lane) & 31);
        uint64_t* bar = &bars[ST + buf];
        if (lane == 0) mbar_arrive_expect_tx(bar, F::META);
        __syncwarp();
        if (lane < F::PPG)
          bulk_g2s_hint(meta + buf * F::META + lane * F::KMS,
                        pool_h + ph * page_stride + F::BODY, F::KMS, bar, pol);
      };
      issue_meta(0, gcount & 1);
      {
        int s2 = stage;
        for (int j = 0; j < min(ST, n_steps); ++j) {
          issue_step(j, s2);
          s2 = s2 + 1 == ST ? 0 : s2 + 1;
        }
      }
      // B operand: q of head g as exact f16 in this thread's key-channel order
      uint32_t bq[F::NKB][2];
#pragma unroll
      for (int kb = 0; kb < F::NKB; ++kb)
#pragma unroll
        for (int hi = 0; hi < 2; ++hi) {
          const int64_t c0 = qrow + tig * F::CH + kchan<BITS>(kb, hi, 0);
          const int64_t c1 = qrow + tig * F::CH + kchan<BITS>(kb, hi, 1);
          bq[kb][hi] = pack_h2(hok ? load_q(a, c0) : 0.f, hok ? load_q(a, c1) : 0.f);
        }

      const int ngroups = n_units / F::PPG;
      int j = 0;  // step index within the item
      for (int grp = 0; grp < ngroups; ++grp, ++gcount) {
        const int buf = gcount & 1;
        if (grp + 1 < ngroups) issue_meta(grp + 1, buf ^ 1);
        if (!dead && !mbar_wait(&bars[ST + buf], (gcount >> 1) & 1, a.err)) dead = true;
        // per-channel (step, zero) pairs of this key group as f16x2
        uint32_t ks[F::NKB][2], kz[F::NKB][2];
        const uint32_t* mwords = reinterpret_cast<const uint32_t*>(meta + buf * F::META);
#pragma unroll
        for (int kb = 0; kb < F::NKB; ++kb)
#pragma unroll
          for (int hi = 0; hi < 2; ++hi) {
            const uint32_t m0 = mwords[tig * F::CH + kchan<BITS>(kb, hi, 0)];
            const uint32_t m1 = mwords[tig * F::CH + kchan<BITS>(kb, hi, 1)];
            ks[kb][hi] = __byte_perm(m0, m1, 0x5410);
            kz[kb][hi] = __byte_perm(m0, m1, 0x7632);
          }
        for (int pi = 0; pi < F::PPG; pi += NP, ++j) {
          if (!dead && !mbar_wait(&bars[stage], phase, a.err)) dead = true;
          const uint8_t* sbase = ring + stage * SB;
          // ---- S^T = K Q^T for NP pages (independent MMA chains).  Columns of
          //      padded heads (>= grp) see q = 0: their weights are computed and
          //      never used. ----
          float sc[NP][4];
#pragma unroll
          for (int p = 0; p < NP; ++p) {
            uint32_t wg[F::TW], wh[F::TW];
            load_key_words<D, BITS>(sbase + p * F::BODY, g, tig, wg, wh);
            sc[p][0] = sc[p][1] = sc[p][2] = sc[p][3] = 0.f;
            float sx[4] = {0.f, 0.f, 0.f, 0.f};  // second chain (odd k-blocks)
#pragma unroll
            for (int kb = 0; kb < F::NKB; ++kb) {
              uint32_t r[4];
              switch (kb) {
#define TKV_KF(K)                                                                              \
  case K:                                                                                      \
    key_frag<BITS, (K < F::NKB ? K : 0)>(wg, wh, ks[K < F::NKB ? K : 0], kz[K < F::NKB ? K : 0], \
                                         r);                                                   \
    break;
                TKV_KF(0) TKV_KF(1) TKV_KF(2) TKV_KF(3) TKV_KF(4) TKV_KF(5) TKV_KF(6) TKV_KF(7)
#undef TKV_KF
              }
              if (TKV_QK_CHAINS == 2 && (kb & 1))
                mma16816(sx, r[0], r[1], r[2], r[3], bq[kb][0], bq[kb][1]);
              else
                mma16816(sc[p], r[0], r[1], r[2], r[3], bq[kb][0], bq[kb][1]);
            }
            if (TKV_QK_CHAINS == 2) {
#pragma unroll
              for (int i = 0; i < 4; ++i) sc[p][i] += sx[i];
            }
          }
          softmax_update<D, NVG, NP>(st, sc, alpha);
          // ---- O^T += V^T P'^T, P' = p * step_v (per token) ----
#pragma unroll
          for (int p = 0; p < NP; ++p) {
            const uint8_t* pg = sbase + p * F::BODY;
            uint32_t vw[F::VWN];
            load_value_words<D, BITS>(pg + F::V_CODES_OFF, lane, vw);
            const uint32_t* vm = reinterpret_cast<const uint32_t*>(pg + F::V_META_OFF);
#pragma unroll
            for (int vg = 0; vg < NVG; ++vg) {
              const float2 sza = unpack_h2(vm[g * NVG + vg]);        // token g:   (step, zero)
              const float2 szb = unpack_h2(vm[(g + 8) * NVG + vg]);  // token g+8
              const uint32_t h2a = pack_h2(sc[p][0] * sza.x, sc[p][1] * sza.x);
              const uint32_t h2b = pack_h2(sc[p][2] * szb.x, sc[p][3] * szb.x);
              const float2 ra = unpack_h2(h2a), rb = unpack_h2(h2b);
              constexpr float blo = VEnc<BITS>::kBetaLo, bhi = VEnc<BITS>::kBetaHi;
              st.w[vg][0] += fmaf(sc[p][0], sza.y, fmaf(sc[p][2], szb.y, -(blo * ra.x + bhi * rb.x)));
              st.w[vg][1] += fmaf(sc[p][1], sza.y, fmaf(sc[p][3], szb.y, -(blo * ra.y + bhi * rb.y)));
              uint32_t b01, b23;
              p_to_bfrag(h2a, h2b, lane, b01, b23);
#pragma unroll
              for (int k = 0; k < F::MB_PER_VG; ++k) {
                const int mb = vg * F::MB_PER_VG + k;
                uint32_t r[4];
                switch (mb) {
#define TKV_VF(M)                                         \
  case M:                                                 \
    value_frag<BITS, (M < D / 16 ? M : 0)>(vw, r);        \
    break;
                  TKV_VF(0) TKV_VF(1) TKV_VF(2) TKV_VF(3) TKV_VF(4) TKV_VF(5) TKV_VF(6) TKV_VF(7)
#undef TKV_VF
                }
                mma16816(st.o[mb], r[0], r[1], r[2], r[3], b01, b23);
              }
            }
          }
          __syncwarp();
          if (j + ST < n_steps) issue_step(j + ST, stage);
          if (++stage == ST) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      write_partial<D, NVG>(a, st, ml_base, VEnc<BITS>::kScale);
      item_done(b, h, nv);
      continue;
    }

    // =================== fp16 residual ring ===================
    // unit 2*ci = K block of 16-token chunk ci, unit 2*ci+1 = its V block
    constexpr int CHUNK = 2 * F::RBLK;
    const int64_t chunks_per_row = a.ring_cap / kPage;
    const uint8_t* ring_base = reinterpret_cast<const uint8_t*>(a.ring) +
                               (((int64_t)row * a.n_kv_heads + h) * chunks_per_row) * CHUNK;
    const int n = n_units;
    auto issue_unit = [&](int u, int stg) {  // one lane per unit
      const int ci = u >> 1;
      const int chunk = ((nq + ci * kPage) % a.ring_cap) / kPage;
      mbar_arrive_expect_tx(&bars[stg], F::RBLK);
      bulk_g2s_hint(ring + stg * SB, ring_base + (int64_t)chunk * CHUNK + (u & 1) * F::RBLK,
                    F::RBLK, &bars[stg], pol);
    };
    // units u0 .. u0+cnt-1 into consecutive stages from istage, one per lane
    int issued = 0;
    int istage = stage;  // stage of the next unit to issue
    auto issue_units = [&](int lim) {
      const int cnt = lim - issued;
      if (lane < cnt) issue_unit(issued + lane, (istage + lane) % ST);
      istage = (istage + cnt) % ST;
      issued = lim;
    };
    issue_units(min(ST, n));
    uint32_t bq[F::NKB][2];
#pragma unroll
    for (int kb = 0; kb < F::NKB; ++kb)
#pragma unroll
      for (int hi = 0; hi < 2; ++hi) {
        const int c = 16 * kb + 2 * tig + 8 * hi;
        bq[kb][hi] = pack_h2(hok ? load_q(a, qrow + c) : 0.f, hok ? load_q(a, qrow + c + 1) : 0.f);
      }
    const bool hv0 = 2 * tig < a.grp, hv1 = 2 * tig + 1 < a.grp;
    const int n_chunks = n >> 1;
    for (int ci = 0; ci < n_chunks; ++ci) {
      const int sk = stage;
      if (!dead && !mbar_wait(&bars[stage], phase, a.err)) dead = true;
      if (++stage == ST) {
        stage = 0;
        phase ^= 1u;
      }
      const int sv = stage;
      if (!dead && !mbar_wait(&bars[stage], phase, a.err)) dead = true;
      if (++stage == ST) {
        stage = 0;
        phase ^= 1u;
      }
      const int tb = nq + ci * kPage;
      const bool vg0 = tb + g < len, vg8 = tb + g + 8 < len;
      float sc[1][4] = {{0.f, 0.f, 0.f, 0.f}};
      float (&s)[4] = sc[0];
      const uint8_t* ck = ring + sk * SB;
#pragma unroll
      for (int kb = 0; kb < F::NKB; ++kb) {
        const uint4 x = *reinterpret_cast<const uint4*>(ck + (kb * 32 + lane) * 16);
        mma16816(s, x.x, x.y, x.z, x.w, bq[kb][0], bq[kb][1]);
      }
      s[0] = (hv0 && vg0) ? s[0] : -INFINITY;
      s[1] = (hv1 && vg0) ? s[1] : -INFINITY;
      s[2] = (hv0 && vg8) ? s[2] : -INFINITY;
      s[3] = (hv1 && vg8) ? s[3] : -INFINITY;
      softmax_update<D, NVG, 1>(st, sc, alpha);
      uint32_t b01, b23;
      p_to_bfrag(pack_h2(s[0], s[1]), pack_h2(s[2], s[3]), lane, b01, b23);
      // zero the V^T columns of tokens past the end (stale ring slots)
      const int t0 = tb + 2 * tig;
      const uint32_t m01 = (t0 < len ? 0x0000ffffu : 0u) | (t0 + 1 < len ? 0xffff0000u : 0u);
      const uint32_t m23 = (t0 + 8 < len ? 0x0000ffffu : 0u) | (t0 + 9 < len ? 0xffff0000u : 0u);
      const uint8_t* cv = ring + sv * SB;
#pragma unroll
      for (int mb = 0; mb < D / 16; ++mb) {
        const uint4 x = *reinterpret_cast<const uint4*>(cv + (mb * 32 + lane) * 16);
        mma16816(st.o[mb], x.x & m01, x.y & m01, x.z & m23, x.w & m23, b01, b23);
      }
      __syncwarp();
      issue_units(min(n, 2 * (ci + 1) + ST));
    }
    write_partial<D, NVG>(a, st, ml_base, 1.f);
    item_done(b, h, nv);
  }

  if (dead) {
    // let the copies still in flight into this warp's ring and meta buffers
    // land before the warp exits (each wait bounded again)
    for (int i = 0; i < ST; ++i) {
      const int s2 = (stage + i) % ST;
      mbar_wait(&bars[s2], s2 >= stage ? phase : phase ^ 1u, nullptr);
    }
    for (int i = 0; i < 2; ++i) mbar_wait(&bars[ST + ((gcount + i) & 1)], ((gcount + i) >> 1) & 1, nullptr);
  }
  // the last warp to finish resets the work counters for the next launch
  if (lane == 0) {
    __threadfence();
    const unsigned int done = atomicAdd(&a.work[1], 1u);
    if (done == gridDim.x - 1) {
      a.work[0] = 0u;
      a.work[1] = 0u;
      __threadfence();
    }
  }
}

// merge kernel: one warp per (q head, sequence); same per-head arithmetic as
// the merge fused into the decode kernel, so both give identical outputs
__global__ void __launch_bounds__(32) merge_kernel(const float* __restrict__ part_ml,
                                                   const float* __restrict__ part_o, int n_slots,
                                                   int num_seqs, int num_q_heads, int D,
                                                   void* __restrict__ out, int out_dtype) {
  const int64_t i0 = (int64_t)blockIdx.y * num_q_heads + blockIdx.x;
  merge_heads<1>(part_ml, part_o, n_slots, n_slots, n_slots, (int64_t)num_seqs * num_q_heads, i0,
                 1, D, out, out_dtype, threadIdx.x, i0);
}

// Merge of many partial slots, one CTA of kReduceWarps warps per (q head,
// sequence): warp w combines a contiguous block of slots (merge_heads with
// RED), then the warps' partials are combined in shared memory with the same
// log-sum-exp rule.  out_ml != nullptr: the combined unnormalised partial
// (M, L) to out_ml and O to out (f32); otherwise O / L to out in out_dtype.
constexpr int kReduceWarps = 8;

__global__ void __launch_bounds__(32 * kReduceWarps) wide_merge_kernel(
    const float* __restrict__ part_ml, const float* __restrict__ part_o, int n_slots,
    int num_seqs, int num_q_heads, int D, void* __restrict__ out, int out_dtype,
    float* __restrict__ out_ml) {
  __shared__ float s_ml[kReduceWarps][2];
  __shared__ float s_o[kReduceWarps][128];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t stride = (int64_t)num_seqs * num_q_heads;
  const int64_t i0 = (int64_t)blockIdx.y * num_q_heads + blockIdx.x;
  const int per = (n_slots + kReduceWarps - 1) / kReduceWarps;
  const int s0 = min(n_slots, warp * per), cnt = min(n_slots, s0 + per) - s0;
  if (cnt > 0) {
    // slots s0 .. s0+cnt-1 as a block of their own: shift the base pointers
    merge_heads<1, true>(part_ml + s0 * stride * 2, part_o + s0 * stride * D, cnt, cnt, cnt,
                         stride, i0, 1, D, &s_o[warp][0], TKV_F32, lane, 0, &s_ml[warp][0]);
  } else if (lane == 0) {
    s_ml[warp][0] = -INFINITY;
    s_ml[warp][1] = 0.f;
  }
  __syncthreads();
  float M = -INFINITY;
  for (int w = 0; w < kReduceWarps; ++w) M = fmaxf(M, s_ml[w][0]);
  float L = 0.f;
  for (int w = 0; w < kReduceWarps; ++w) {
    const float m = s_ml[w][0];
    if (m != -INFINITY) L = fmaf(s_ml[w][1], fast_exp2(m - M), L);
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    float acc = 0.f;
    for (int w = 0; w < kReduceWarps; ++w) {
      const float m = s_ml[w][0];
      if (m != -INFINITY) acc = fmaf(s_o[w][c], fast_exp2(m - M), acc);
    }
    const int64_t oi = i0 * D + c;
    if (out_ml) {
      static_cast<float*>(out)[oi] = acc;
    } else {
      const float v = acc * inv;
      if (out_dtype == TKV_F32)
        static_cast<float*>(out)[oi] = v;
      else if (out_dtype == TKV_BF16)
        static_cast<__nv_bfloat16*>(out)[oi] = __float2bfloat16_rn(v);
      else
        static_cast<__half*>(out)[oi] = __float2half_rn(v);
    }
  }
  if (out_ml && threadIdx.x == 0) {
    out_ml[i0 * 2 + 0] = M;
    out_ml[i0 * 2 + 1] = L;
  }
}

// ---------------------------------------------------------------------------
// host launchers
// ---------------------------------------------------------------------------
template <int D, int BITS, int G>
static int launch_warp_t(const DecodeArgs& a, cudaStream_t stream) {
  constexpr int smem = decode_smem_bytes<D, BITS, G>();
  // CTAs that fit on each device at once (computed per device, thread-safe)
  static std::atomic<int> cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return TKV_BACKEND_ERROR;
  int resident = dev >= 0 && dev < 64 ? cache[dev].load(std::memory_order_relaxed) : 0;
  if (resident <= 0) {
    int sms = 0, per_sm = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaFuncSetAttribute(decode_warp_kernel<D, BITS, G>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_warp_kernel<D, BITS, G>, 32,
                                                      smem) != cudaSuccess ||
        per_sm <= 0)
      return TKV_BACKEND_ERROR;
    resident = sms * per_sm;
    if (dev >= 0 && dev < 64) cache[dev].store(resident, std::memory_order_relaxed);
  }
  const int grid = a.n_items < resident ? a.n_items : resident;
  decode_warp_kernel<D, BITS, G><<<grid, 32, smem, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? TKV_OK : TKV_BACKEND_ERROR;
}

template <int D, int BITS>
static int launch_warp_g(const DecodeArgs& a, cudaStream_t stream) {
  switch (a.group) {
    case 16: return launch_warp_t<D, BITS, 16>(a, stream);
    case 32: return launch_warp_t<D, BITS, 32>(a, stream);
    case 64: return launch_warp_t<D, BITS, 64>(a, stream);
    case 128: return launch_warp_t<D, BITS, 128>(a, stream);
  }
  return TKV_NOT_IMPLEMENTED;
}

int launch_decode_splits(DecodeArgs a, int head_dim, int bits, int, cudaStream_t stream) {
  a.n_items = a.n_slots * a.num_seqs * a.n_kv_heads;
  if (a.n_items <= 0) return TKV_OK;
  if (head_dim == 128)
    return bits == 4 ? launch_warp_g<128, 4>(a, stream) : launch_warp_g<128, 2>(a, stream);
  if (head_dim == 64)
    return bits == 4 ? launch_warp_g<64, 4>(a, stream) : launch_warp_g<64, 2>(a, stream);
  return TKV_NOT_IMPLEMENTED;
}

int launch_reduce(const float* part_ml, const float* part_o, int n_slots, int num_seqs,
                  int num_q_heads, int head_dim, float* out_ml, float* out_o,
                  cudaStream_t stream) {
  if (head_dim > 128) return TKV_NOT_IMPLEMENTED;
  dim3 grid(num_q_heads, num_seqs);
  wide_merge_kernel<<<grid, 32 * kReduceWarps, 0, stream>>>(
      part_ml, part_o, n_slots, num_seqs, num_q_heads, head_dim, out_o, TKV_F32, out_ml);
  return cudaGetLastError() == cudaSuccess ? TKV_OK : TKV_BACKEND_ERROR;
}

int launch_merge(const float* part_ml, const float* part_o, int n_slots, int num_seqs,
                 int num_q_heads, int head_dim, void* out, int out_dtype, cudaStream_t stream) {
  if (n_slots > kWideMergeSlots && head_dim <= 128) {  // many slots: 8 warps per q head
    dim3 grid(num_q_heads, num_seqs);
    wide_merge_kernel<<<grid, 32 * kReduceWarps, 0, stream>>>(
        part_ml, part_o, n_slots, num_seqs, num_q_heads, head_dim, out, out_dtype, nullptr);
    return cudaGetLastError() == cudaSuccess ? TKV_OK : TKV_BACKEND_ERROR;
  }
  dim3 grid(num_q_heads, num_seqs);
  merge_kernel<<<grid, 32, 0, stream>>>(part_ml, part_o, n_slots, num_seqs, num_q_heads,
                                         head_dim, out, out_dtype);
  return cudaGetLastError() == cudaSuccess ? TKV_OK : TKV_BACKEND_ERROR;
}

}  // namespace tkv
