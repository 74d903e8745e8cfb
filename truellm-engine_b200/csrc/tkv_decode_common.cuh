// tkv_decode_common.cuh -- warp-level pieces shared by the paged KIVI decode
// kernels (the persistent split kernel in tkv_decode.cu and the balanced
// stream kernel in tkv_stream.cu): the per-warp online-softmax state, the
// softmax update over 16-token tiles, the move of P^T into the mma B-operand
// layout, q loads and the log-sum-exp merge of split partials.
#pragma once

#include "tkv_frag.cuh"

namespace tkv {

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
  // Adds the value-zero correction into the accumulator (o += w / oscale,
  // w = 0; the result oscale * o + w is unchanged).  The encoded value codes
  // carry an offset beta (1024 or 64 for INT4) that the correction removes:
  // until it is added, o holds beta * sum(p') and rounds at that magnitude,
  // so a state that runs over thousands of tokens folds it in every few pages.
  // Each thread's w covers only its token rows (lanes of equal lane & 3 hold
  // the rest), so it is summed over those lanes first; o covers all tokens.
  __device__ __forceinline__ void fold(float inv_oscale) {
    constexpr int MB_PER_VG = (D / 16) / NVG;
    float c[NVG][2];
#pragma unroll
    for (int v = 0; v < NVG; ++v)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        float x = w[v][hh];
        x += __shfl_xor_sync(0xffffffffu, x, 4);
        x += __shfl_xor_sync(0xffffffffu, x, 8);
        x += __shfl_xor_sync(0xffffffffu, x, 16);
        c[v][hh] = x * inv_oscale;
        w[v][hh] = 0.f;
      }
#pragma unroll
    for (int i = 0; i < D / 16; ++i)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        o[i][hh] += c[i / MB_PER_VG][hh];
        o[i][2 + hh] += c[i / MB_PER_VG][hh];
      }
  }
};

// Online-softmax update for NP 16-token tiles.  s[p][4]: raw S^T accumulators
// (rows g, g+8; cols = heads 2tig, 2tig+1), masked entries -inf; alpha =
// softmax scale * log2(e).  Replaces s by the unnormalised weights
// p = 2^(alpha * s - m) (m in log2 units).
template <int D, int NVG, int NP>
__device__ __forceinline__ void softmax_update(WarpState<D, NVG>& st, float (&s)[NP][4],
                                               float alpha) {
  float t[2];
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    float x = fmaxf(s[0][hh], s[0][2 + hh]);
#pragma unroll
    for (int p = 1; p < NP; ++p) x = fmaxf(x, fmaxf(s[p][hh], s[p][2 + hh]));
    x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, 4));
    x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, 8));
    x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, 16));
    t[hh] = x * alpha;  // raw scores: alpha > 0 keeps the order
  }
  const bool need = t[0] > st.m[0] + kLazyLog2 || t[1] > st.m[1] + kLazyLog2;
  if (__any_sync(0xffffffffu, need)) {
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const float mnew = fmaxf(st.m[hh], t[hh]);
      const float r = st.m[hh] == -INFINITY ? 0.f : fast_exp2(st.m[hh] - mnew);
      st.l[hh] *= r;
#pragma unroll
      for (int v = 0; v < NVG; ++v) st.w[v][hh] *= r;
#pragma unroll
      for (int i = 0; i < D / 16; ++i) {
        st.o[i][hh] *= r;
        st.o[i][2 + hh] *= r;
      }
      st.m[hh] = mnew;
    }
  }
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    const float nbase = st.m[hh] == -INFINITY ? 0.f : -st.m[hh];
    float sum = 0.f;
#pragma unroll
    for (int p = 0; p < NP; ++p) {
      s[p][hh] = fast_exp2(fmaf(s[p][hh], alpha, nbase));
      s[p][2 + hh] = fast_exp2(fmaf(s[p][2 + hh], alpha, nbase));
      sum += s[p][hh] + s[p][2 + hh];
    }
    st.l[hh] += sum;
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
// log-sum-exp merge of the split partials (paged_attention_v2.cu:132-170), one
// warp for nh consecutive q heads i0 .. i0+nh-1 of one sequence:
//   M = max_s m_s,  L = sum_s l_s 2^(m_s - M),
//   out[c] = (sum_s o_s[c] 2^(m_s - M)) / L,  slots with m_s = -inf skipped.
// The slots merged are t = 0 .. cnt-1 mapped to slot t for t < nv and to the
// last slot (n_slots - 1, the residual) otherwise; the standalone merge passes
// nv = cnt = n_slots.  M is a max (exact in any order); L and O are summed
// over t in order, so a merge over only the written slots equals one over all
// slots with -inf in the unwritten ones, bit for bit.  H heads and 128
// channels go per pass (lane l owns channels l + 32k), the loads of 16/H
// slots in flight at once: at the tail of the decode launch the merge's
// latency is exposed.  Partials are read with ld.global.cg: other CTAs of the
// same launch may have written them.
// ---------------------------------------------------------------------------
// Output rows are oi0 + j (j < nh).  RED: write the combined unnormalised
// partial, (M, L) to red_ml and O to out (f32), instead of O / L.
template <int H, bool RED = false>
__device__ __forceinline__ void merge_heads(const float* part_ml, const float* part_o,
                                            int n_slots, int nv, int cnt, int64_t stride,
                                            int64_t i0, int nh, int D, void* out, int out_dtype,
                                            int lane, int64_t oi0, float* red_ml = nullptr) {
  constexpr int CPL = 4, UB = 16 / H;
  static_assert(H == 1 || H == 2 || H == 4, "heads per merge pass");
  for (int j0 = 0; j0 < nh; j0 += H) {
    float M[H], m0[H], l0[H];
#pragma unroll
    for (int q = 0; q < H; ++q) M[q] = m0[q] = -INFINITY, l0[q] = 0.f;
    for (int t = lane; t < cnt; t += 32) {
      const int64_t s = t < nv ? t : n_slots - 1;
#pragma unroll
      for (int q = 0; q < H; ++q) {
        if (j0 + q >= nh) continue;
        const int64_t r = (s * stride + i0 + j0 + q) * 2;
        const float m = __ldcg(&part_ml[r]), l = __ldcg(&part_ml[r + 1]);
        if (t < 32) m0[q] = m, l0[q] = l;
        M[q] = fmaxf(M[q], m);
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1)
#pragma unroll
      for (int q = 0; q < H; ++q) M[q] = fmaxf(M[q], __shfl_xor_sync(0xffffffffu, M[q], off));
    for (int cb = 0; cb < D; cb += 32 * CPL) {
      float O[H][CPL], L[H];
#pragma unroll
      for (int q = 0; q < H; ++q) {
        L[q] = 0.f;
#pragma unroll
        for (int k = 0; k < CPL; ++k) O[q][k] = 0.f;
      }
      for (int c0 = 0; c0 < cnt; c0 += 32) {
        // lane u of this chunk holds weight and l of t = c0 + u
        float w[H], lw[H];
        const int t = c0 + lane;
        const int64_t s = t < nv ? t : n_slots - 1;
#pragma unroll
        for (int q = 0; q < H; ++q) {
          float m = m0[q], l = l0[q];
          if (c0 > 0) {
            const bool ok = t < cnt && j0 + q < nh;
            const int64_t r = (s * stride + i0 + j0 + q) * 2;
            m = ok ? __ldcg(&part_ml[r]) : -INFINITY;
            l = ok ? __ldcg(&part_ml[r + 1]) : 0.f;
          }
          w[q] = m != -INFINITY ? fast_exp2(m - M[q]) : 0.f;
          lw[q] = l;
        }
        const int n = min(32, cnt - c0);
        // UB slots per batch: all their loads are issued before the
        // shuffles and FMAs that use them
        for (int u0 = 0; u0 < n; u0 += UB) {
          float ov[UB][H][CPL];
#pragma unroll
          for (int uu = 0; uu < UB; ++uu) {
            const int tu = c0 + u0 + uu;
            const int64_t su = tu < nv ? tu : n_slots - 1;
            const int64_t row = (su * stride + i0 + j0) * D + cb + lane;
#pragma unroll
            for (int q = 0; q < H; ++q)
#pragma unroll
              for (int k = 0; k < CPL; ++k) {
                const bool ok = u0 + uu < n && j0 + q < nh && cb + lane + 32 * k < D;
                ov[uu][q][k] = ok ? __ldcg(&part_o[row + q * D + 32 * k]) : 0.f;
              }
          }
#pragma unroll
          for (int uu = 0; uu < UB; ++uu) {
            const int src = (u0 + uu) & 31;
#pragma unroll
            for (int q = 0; q < H; ++q) {
              const float wv = __shfl_sync(0xffffffffu, w[q], src);
              const float lq = __shfl_sync(0xffffffffu, lw[q], src);
              const float wq = u0 + uu < n ? wv : 0.f;
              L[q] = wq != 0.f ? fmaf(lq, wq, L[q]) : L[q];
#pragma unroll
              for (int k = 0; k < CPL; ++k)
                O[q][k] = wq != 0.f ? fmaf(ov[uu][q][k], wq, O[q][k]) : O[q][k];
            }
          }
        }
      }
#pragma unroll
      for (int q = 0; q < H; ++q) {
        if (j0 + q >= nh) continue;
        if (RED) {
          if (cb == 0 && lane == 0) {
            red_ml[(oi0 + j0 + q) * 2 + 0] = M[q];
            red_ml[(oi0 + j0 + q) * 2 + 1] = L[q];
          }
#pragma unroll
          for (int k = 0; k < CPL; ++k) {
            const int c = cb + lane + 32 * k;
            if (c < D) static_cast<float*>(out)[(oi0 + j0 + q) * D + c] = O[q][k];
          }
          continue;
        }
        const float inv = L[q] > 0.f ? 1.f / L[q] : 0.f;
#pragma unroll
        for (int k = 0; k < CPL; ++k) {
          const int c = cb + lane + 32 * k;
          if (c >= D) continue;
          const float v = O[q][k] * inv;
          const int64_t oi = (oi0 + j0 + q) * D + c;
          if (out_dtype == TKV_F32)
            static_cast<float*>(out)[oi] = v;
          else if (out_dtype == TKV_BF16)
            static_cast<__nv_bfloat16*>(out)[oi] = __float2bfloat16_rn(v);
          else
            static_cast<__half*>(out)[oi] = __float2half_rn(v);
        }
      }
    }
  }
}

}  // namespace tkv
