// tkv_append.cu -- quantize-on-append into the paged KIVI cache (sm_100a).
//
// Replaces reshape_and_cache (third_party/vllm_kernels/cache_kernels.cu:47-94,
// host wrapper :202-232) for a KIVI cache.  Two launches per call, in stream
// order:
//   1. flush:    one CTA per (key group, K or V, kv head, sequence).  It gathers the G
//                tokens of the group (old ones from the fp16 ring, new ones
//                from the input with cp.async), quantises keys per channel and
//                values per token with the reference quantizer
//                (kivi_cache.cu:92-124) and writes the group's pages with
//                coalesced 32- and 128-bit stores.
//   2. residual: copies the new tokens that stay in fp16 into the ring, whole
//                16-byte fragment vectors for fully written 16-token chunks.
// Running the flush before the residual write keeps ring slots that are read
// by (1) from being overwritten by (2) in the same call.
#include <atomic>

#include "tkv_common.cuh"

namespace tkv {

constexpr int kMaxAppendDevices = 64;


__device__ __forceinline__ int nq_of(int len, int R, int G) {
  int x = len - R;
  return x > 0 ? G * (x / G) : 0;
}

// Half offset of (token t in 0..15, channel c) in a ring chunk's K / V block.
__device__ __forceinline__ int ring_k_off(int c, int t) {
  int cc = c & 15, lane = 4 * (t & 7) + ((cc & 7) >> 1), r = 2 * (cc >> 3) + (t >> 3);
  return ((c >> 4) * 32 + lane) * 8 + 2 * r + (cc & 1);
}
__device__ __forceinline__ int ring_v_off(int c, int t) {
  int cc = c & 15, lane = 4 * (cc & 7) + ((t & 7) >> 1), r = 2 * (t >> 3) + (cc >> 3);
  return ((c >> 4) * 32 + lane) * 8 + 2 * r + (t & 1);
}

__device__ __forceinline__ uint16_t* ring_chunk(const AppendArgs& a, int slot_row, int h, int tok,
                                                int kv) {
  int s = tok % a.ring_cap;
  int64_t chunks = a.ring_cap / kPage;
  int64_t elems = static_cast<int64_t>(kPage) * a.head_dim;
  return a.ring + ((((int64_t)slot_row * a.n_kv_heads + h) * chunks + s / kPage) * 2 + kv) * elems;
}

// Every index a sequence's append touches stays inside the caller's buffers:
// input rows [c0, c1) within [0, total_new), the new length within the block
// table, the token count within the grid bound.
__device__ __forceinline__ bool append_lengths_ok(const AppendArgs& a, int L, int c0, int c1) {
  return L >= 0 && c0 >= 0 && c1 >= c0 && c1 <= a.total_new && c1 - c0 <= a.max_new &&
         (int64_t)L + (c1 - c0) <= (int64_t)a.max_blocks * kPage;
}

// threads of a flush CTA (one CTA per key group, K or V, kv head, sequence)
#ifndef TKV_FLUSH_THREADS
#define TKV_FLUSH_THREADS 128
#endif
constexpr int kFlushThreads = TKV_FLUSH_THREADS;


// Four 8x8 16-bit matrices transposed from shared memory: lane L gives the
// address of row L % 8 of matrix L / 8; register m of lane 4 g + t then holds
// the elements of rows 2t and 2t + 1 (low, high half) at column g of matrix m.
__device__ __forceinline__ void ldsm_x4_t(const void* p, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
// The same without the transpose: register m of lane 4 g + t holds row g,
// columns 2t and 2t + 1 (low, high half) of matrix m.
__device__ __forceinline__ void ldsm_x4(const void* p, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

__device__ __forceinline__ float h2f(uint16_t h) {
  return __half2float(*reinterpret_cast<const __half*>(&h));
}

// Sequential-scan extremes of the reference quantizer (kivi_cache.cu:92-124:
// gmin/gmax seeded with +/-FLT_MAX, strict compares, so NaN never enters and
// the first of equal values wins) from the packed-f16 min/max of the same
// values (min.f16x2 / max.f16x2 skip NaN).  The only equal values with
// different bits are +0 and -0: when an extreme is zero, its sign is that of
// the first zero in scan order, supplied by `first_zero_sign` (rare path).
template <typename FirstZero>
__device__ __forceinline__ void scan_extremes(__half hmn, __half hmx, float& gmin, float& gmax,
                                              FirstZero first_zero_sign) {
  gmin = __half2float(hmn);
  gmax = __half2float(hmx);
  if (gmin == INFINITY) gmin = FLT_MAX;      // no value below the seed
  if (gmax == -INFINITY) gmax = -FLT_MAX;
  if (gmin == 0.f || gmax == 0.f) {
    const float z = first_zero_sign();
    if (gmin == 0.f) gmin = z;
    if (gmax == 0.f) gmax = z;
  }
}

// Shared memory of the flush kernel: the group's fp16 K (or V) tile with rows
// padded by 8 halves (the fragment-order value reads then hit distinct
// banks), the quantisation parameters and meta words, partial key extremes.
template <int D, int G>
struct FlushSmem {
  static constexpr int TS = D + 8;               // row stride in halves
  static constexpr int NVG = D > G ? D / G : 1;  // value groups per token
  static constexpr int NPAR = D > G * NVG ? D : G * NVG;
  static constexpr int KSPLIT = kFlushThreads / (D / 2);  // token splits of the key scan
  uint16_t tile[G * TS];
  float2 par[NPAR];      // (gmin, scale) per key channel or per (token, value group)
  uint32_t meta[NPAR];   // step | zero << 16
  __half2 kmn[KSPLIT][D / 2], kmx[KSPLIT][D / 2];
  int phys[G / kPage];   // the group's pages
};

// One CTA per (key group, K or V, kv head, sequence): gathers the G tokens of
// the group (old ones from the fp16 ring, new ones from the input with
// 16-byte cp.async), rounds bf16 input to fp16, computes the quantisation
// parameters (keys per channel, values per token and value group), then packs
// and stores the group's K (or V) codes and meta into its pages.
template <int D, int BITS, int G>
__global__ void __launch_bounds__(kFlushThreads) flush_groups_kernel(AppendArgs a) {
  using S_t = FlushSmem<D, G>;
  constexpr int TS = S_t::TS, NVG = S_t::NVG, KSPLIT = S_t::KSPLIT, QMAX = (1 << BITS) - 1;
  constexpr int VG_CH = D > G ? G : D;  // channels per value group
  extern __shared__ __align__(16) uint8_t smem_raw[];
  S_t& S = *reinterpret_cast<S_t*>(smem_raw);
  const int tid = threadIdx.x;
  const int b = blockIdx.z, h = blockIdx.y, gi = blockIdx.x >> 1;
  const bool is_v = blockIdx.x & 1;
  const int L = a.lens_old[b];
  const int c0 = a.cu_new[b], c1 = a.cu_new[b + 1];
  const int T = c1 - c0;
  if (!append_lengths_ok(a, L, c0, c1)) {
    if (tid == 0 && blockIdx.x == 0 && h == 0) set_err(a.err, TKV_ERR_BAD_LENGTH);
    return;
  }
  const int L2 = L + T;
  const int nq0 = nq_of(L, a.residual, G), nq1 = nq_of(L2, a.residual, G);
  const int t0 = nq0 + gi * G;
  if (t0 >= nq1) return;
  const int row = a.seq_slots ? a.seq_slots[b] : b;
  if (t0 < L && (row < 0 || row >= a.max_seqs)) {
    if (tid == 0 && !is_v) set_err(a.err, TKV_ERR_BAD_SLOT);
    return;
  }
  const int32_t* bt = a.block_tables + (int64_t)b * a.max_blocks;
  const int n_old = min(max(L - t0, 0), G);  // tile rows [0, n_old) come from the ring
  uint16_t* tile = S.tile;

  // ---- gather ---------------------------------------------------------------
  // New tokens: input rows [cu_new[b] + (tok - L)][h][0:D], 16-byte vectors
  // (the entry point requires 16-byte aligned inputs).
  constexpr int VPR = D / 8;  // vectors per token row
  const uint16_t* src = static_cast<const uint16_t*>(is_v ? a.v_new : a.k_new);
  for (int i = n_old * VPR + tid; i < G * VPR; i += kFlushThreads) {
    const int t = i / VPR, v = i - t * VPR;
    const int64_t e0 = (((int64_t)c0 + (t0 + t - L)) * a.n_kv_heads + h) * D + v * 8;
    cp_async16(&tile[t * TS + v * 8], src + e0);
  }
  if (tid < G / kPage) {
    const int ph = bt[t0 / kPage + tid];
    S.phys[tid] = ph;
    if (ph < 0 || ph >= a.num_pages) set_err(a.err, TKV_ERR_BAD_PAGE);
  }
  // Old tokens: ring chunks (fragment order), each 16-byte vector read once.
  if (n_old > 0) {
    constexpr int VPC = kPage * D / 8;  // vectors per chunk block
    const int n_chunks = (n_old + kPage - 1) / kPage;
    for (int i = tid; i < n_chunks * VPC; i += kFlushThreads) {
      const int ch = i / VPC, v = i - ch * VPC;
      const int ctok = t0 + ch * kPage;  // t0 is a multiple of 16
      const uint4 w = reinterpret_cast<const uint4*>(ring_chunk(a, row, h, ctok, is_v))[v];
      const uint16_t* xs = reinterpret_cast<const uint16_t*>(&w);
      const int bi = v >> 5, l = v & 31, g = l >> 2, tig = l & 3;
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          // K block: r = 2*hi + th -> (t = g + 8 th, c = 16 bi + 2 tig + 8 hi + e)
          // V block: r = 2*th + rh -> (t = 8 th + 2 tig + e, c = 16 bi + g + 8 rh)
          const int t = ch * kPage + (is_v ? 8 * (r >> 1) + 2 * tig + e : g + 8 * (r & 1));
          const int c = 16 * bi + (is_v ? g + 8 * (r & 1) : 2 * tig + 8 * (r >> 1) + e);
          if (t < n_old) tile[t * TS + c] = xs[2 * r + e];
        }
    }
  }
  cp_async_wait_all();
  __syncthreads();
  // bf16 input -> fp16 (RN) in place, rows of new tokens
  if (a.in_bf16) {
    for (int i = n_old * VPR + tid; i < G * VPR; i += kFlushThreads) {
      const int t = i / VPR, v = i - t * VPR;
      uint4* p = reinterpret_cast<uint4*>(&tile[t * TS + v * 8]);
      uint4 x = *p;
      uint32_t* w = reinterpret_cast<uint32_t*>(&x);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float lo = __uint_as_float(w[j] << 16), hi = __uint_as_float(w[j] & 0xffff0000u);
        const __half2 hh = __floats2half2_rn(lo, hi);
        w[j] = *reinterpret_cast<const uint32_t*>(&hh);
      }
      *p = x;
    }
    __syncthreads();
  }

  // clamp(rint((x - gmin) * scale), 0, QMAX) of the reference with
  // p = (-gmin, scale), x - gmin as x + (-gmin).  The unsigned round-to-nearest
  // conversion saturates negatives and NaN to 0.  The top clamp never binds:
  // for finite values in [gmin, gmax], fl(x - gmin) <= fl(gmax - gmin) = range
  // (rounding is monotonic) and scale = fl(QMAX / range), so the product is at
  // most QMAX * (1 + 2^-24)^2 and rounds to QMAX; with an infinite extreme the
  // range is infinite, scale is 0 and every product is 0 or NaN.
  auto code = [&](float x, float2 p) {
    return __float2uint_rn(__fmul_rn(__fadd_rn(x, p.x), p.y));
  };
  // the group's page blocks for this kv head, once (nullptr for a page id
  // outside the pool, which is flagged above and skipped)
  uint8_t* pbase[G / kPage];
#pragma unroll
  for (int pi = 0; pi < G / kPage; ++pi) {
    const int ph = S.phys[pi];
    pbase[pi] = (ph < 0 || ph >= a.num_pages)
                    ? nullptr
                    : a.pool + ((int64_t)ph * a.n_kv_heads + h) * a.page_bytes;
  }
  auto page_base = [&](int pi) -> uint8_t* {
    uint8_t* r = pbase[0];
#pragma unroll
    for (int i = 1; i < G / kPage; ++i) r = i == pi ? pbase[i] : r;
    return r;
  };
  const __half2 pinf = __half2half2(__ushort_as_half(0x7c00u));
  const __half2 ninf = __half2half2(__ushort_as_half(0xfc00u));

  if (!is_v) {
    // ---- keys: extremes per channel over the G tokens, KSPLIT token ranges ----
    {
      const int cp = tid % (D / 2), ks = tid / (D / 2);
      __half2 mn = pinf, mx = ninf;
      const __half2* col = reinterpret_cast<const __half2*>(&tile[ks * (G / KSPLIT) * TS + 2 * cp]);
#pragma unroll 16
      for (int t = 0; t < G / KSPLIT; ++t) {
        const __half2 x = col[t * (TS / 2)];
        mn = __hmin2(mn, x);
        mx = __hmax2(mx, x);
      }
      S.kmn[ks][cp] = mn;
      S.kmx[ks][cp] = mx;
    }
    __syncthreads();
    if (tid < D / 2) {
      __half2 mn = S.kmn[0][tid], mx = S.kmx[0][tid];
#pragma unroll
      for (int ks = 1; ks < KSPLIT; ++ks) {
        mn = __hmin2(mn, S.kmn[ks][tid]);
        mx = __hmax2(mx, S.kmx[ks][tid]);
      }
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int c = 2 * tid + e;
        float gmin, gmax;
        scan_extremes(e ? __high2half(mn) : __low2half(mn), e ? __high2half(mx) : __low2half(mx),
                      gmin, gmax, [&]() {
                        for (int t = 0; t < G; ++t) {
                          const float x = h2f(tile[t * TS + c]);
                          if (x == 0.f) return x;
                        }
                        return 0.f;
                      });
        const QParams qp = quant_params(gmin, gmax, QMAX);
        S.par[c] = make_float2(-qp.gmin, qp.scale);
        S.meta[c] = (uint32_t)qp.hstep | ((uint32_t)qp.hzero << 16);
      }
    }
    __syncthreads();
    // ---- key codes, row-major [16 tokens][D * BITS / 8 bytes] ----------------
    constexpr int CPW = 32 / BITS;  // channels per 32-bit word
    constexpr int NWR = D / CPW;    // words per token row
    constexpr int TSTEP = kFlushThreads / NWR;
    const int w = tid % NWR;
    float2 p[CPW];
#pragma unroll
    for (int n = 0; n < CPW; ++n) p[n] = S.par[w * CPW + n];
    // fully unrolled: the page and row of each step are compile-time
    // functions of the thread's first row
    const int t_first = tid / NWR;
#pragma unroll
    for (int k = 0; k < (G + TSTEP - 1) / TSTEP; ++k) {
      const int t = t_first + k * TSTEP;
      if (TSTEP * (k + 1) > G && t >= G) break;
      uint32_t word = 0;
#pragma unroll
      for (int n8 = 0; n8 < CPW; n8 += 8) {
        const uint4 x = *reinterpret_cast<const uint4*>(&tile[t * TS + w * CPW + n8]);
        const uint16_t* hx = reinterpret_cast<const uint16_t*>(&x);
#pragma unroll
        for (int n = 0; n < 8; ++n)  // disjoint bit fields: + packs like |, as one LEA
          word += code(h2f(hx[n]), p[n8 + n]) << (BITS * (n8 + n));
      }
      // t / 16 is k * TSTEP / 16 (t_first < TSTEP) when TSTEP divides 16
      constexpr bool kStatic = TSTEP <= kPage && kPage % TSTEP == 0;
      uint8_t* blk = page_base(kStatic ? k * TSTEP / kPage : t / kPage);
      if (blk) reinterpret_cast<uint32_t*>(blk + a.k_codes_off)[(t % kPage) * NWR + w] = word;
    }
    // key meta slices: page pi holds channels [pi * KMW, (pi + 1) * KMW)
    constexpr int KMW = D * kPage / G;
    for (int i = tid; i < (G / kPage) * KMW; i += kFlushThreads) {
      const int pi = i / KMW, j = i - pi * KMW;
      uint8_t* blk = page_base(pi);
      if (blk) reinterpret_cast<uint32_t*>(blk + a.k_meta_off)[j] = S.meta[i];
    }
    return;
  }

  // ---- values: extremes per token and value group ---------------------------
  for (int j = tid; j < G * NVG; j += kFlushThreads) {
    const int t = j / NVG, vg = j - t * NVG;
    const uint16_t* rowp = &tile[t * TS + vg * VG_CH];
    __half2 mn = pinf, mx = ninf;
#pragma unroll
    for (int c = 0; c < VG_CH; c += 8) {
      const uint4 x = *reinterpret_cast<const uint4*>(rowp + c);
      const __half2* hx = reinterpret_cast<const __half2*>(&x);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        mn = __hmin2(mn, hx[k]);
        mx = __hmax2(mx, hx[k]);
      }
    }
    float gmin, gmax;
    scan_extremes(__hmin(__low2half(mn), __high2half(mn)), __hmax(__low2half(mx), __high2half(mx)),
                  gmin, gmax, [&]() {
                    for (int c = 0; c < VG_CH; ++c) {
                      const float x = h2f(rowp[c]);
                      if (x == 0.f) return x;
                    }
                    return 0.f;
                  });
    const QParams qp = quant_params(gmin, gmax, QMAX);
    S.par[j] = make_float2(-qp.gmin, qp.scale);
    S.meta[j] = (uint32_t)qp.hstep | ((uint32_t)qp.hzero << 16);
  }
  __syncthreads();
  // ---- value codes in mma A-fragment order ----------------------------------
  // Lane l = 4 g + tig of page pi packs, per word, tokens 2 tig + e + 8 th
  // and channels g + 8 rh (+ 16 per m-block): offsets from the lane's base
  // element are compile-time constants.
  {
    constexpr int W = D * BITS / 64;  // words per lane
    constexpr int VW = W < 4 ? W : 4;
#pragma unroll
    for (int k = 0; k < ((G / kPage) * 32 + kFlushThreads - 1) / kFlushThreads; ++k) {
      const int pl = tid + k * kFlushThreads;
      if (pl >= (G / kPage) * 32) break;
      const int pi = pl >> 5, l = pl & 31, tig = l & 3;
      const int tb = pi * kPage + 2 * tig;  // token of (th, e) = (0, 0)
      // ldmatrix.trans source row of this lane: matrix m = l / 8 covers
      // channels + 8 (m & 1) and tokens + 8 (m >> 1) of an m-block
      const uint16_t* lrow = &tile[(pi * kPage + 8 * (l >> 4) + (l & 7)) * TS + 8 * ((l >> 3) & 1)];
      // parameters of the lane's tokens (th, e), per value group
      float2 pv[2][2][NVG];
#pragma unroll
      for (int th = 0; th < 2; ++th)
#pragma unroll
        for (int e = 0; e < 2; ++e)
#pragma unroll
          for (int vg = 0; vg < NVG; ++vg) pv[th][e][vg] = S.par[(tb + 8 * th + e) * NVG + vg];
      uint8_t* blk = page_base(pi);
#pragma unroll
      for (int q = 0; q < W / VW; ++q) {
        uint32_t words[VW];
#pragma unroll
        for (int u = 0; u < VW; ++u) {
          const int wv = q * VW + u;
          uint32_t wd = 0;
          // register m of m-block mb: channel 16 mb + 8 rh + g, tokens
          // 2 tig + 8 th (+1 in the high half), rh = m & 1, th = m >> 1
#pragma unroll
          for (int mbi = 0; mbi < (BITS == 4 ? 1 : 2); ++mbi) {
            const int mb = BITS == 4 ? wv : 2 * wv + mbi;
            uint32_t r[4];
            ldsm_x4_t(lrow + 16 * mb, r);
#pragma unroll
            for (int m = 0; m < 4; ++m) {
              const int rh = m & 1, th = m >> 1, k = 2 * rh + th;
              const int vg = (16 * mb + 8 * rh) / VG_CH;
              const uint32_t c0 = code(h2f(static_cast<uint16_t>(r[m] & 0xffffu)), pv[th][0][vg]);
              const uint32_t c1 = code(h2f(static_cast<uint16_t>(r[m] >> 16)), pv[th][1][vg]);
              if (BITS == 4) {  // nibbles k (token e = 0) and k + 4 (e = 1)
                wd += c0 << (4 * k);
                wd += c1 << (4 * (k + 4));
              } else {          // 2-bit fields 4 mbi + k and 4 mbi + k + 8
                wd += c0 << (2 * (4 * mbi + k));
                wd += c1 << (2 * (4 * mbi + k + 8));
              }
            }
          }
          words[u] = wd;
        }
        if (blk) {
          uint8_t* dst = blk + a.v_codes_off + (q * 32 + l) * (4 * VW);
          if (VW == 4)
            *reinterpret_cast<uint4*>(dst) = make_uint4(words[0], words[VW > 1 ? 1 : 0],
                                                        words[VW > 2 ? 2 : 0], words[VW > 3 ? 3 : 0]);
          else
            *reinterpret_cast<uint2*>(dst) = make_uint2(words[0], words[VW > 1 ? 1 : 0]);
        }
      }
    }
  }
  // value meta [16 tokens][NVG] per page
  constexpr int VMW = kPage * NVG;
  for (int i = tid; i < (G / kPage) * VMW; i += kFlushThreads) {
    const int pi = i / VMW, j = i - pi * VMW;
    uint8_t* blk = page_base(pi);
    if (blk) reinterpret_cast<uint32_t*>(blk + a.v_meta_off)[j] = S.meta[i];
  }
}

// New tokens that stay in fp16: t in [max(nq1, L), L + T) -> ring slot t % C.
// One CTA per (16-token ring chunk, kv head, sequence); chunk q of the
// sequence covers tokens [16 q, 16 q + 16).  A chunk whose 16 tokens are all
// written here is staged through shared memory and stored as whole 16-byte
// fragment vectors; a partly written chunk (e.g. one decode token) is written
// element by element so the slots of older tokens stay untouched.
constexpr int kResThreads = 128;

template <int D>
__global__ void __launch_bounds__(kResThreads) residual_write_kernel(AppendArgs a) {
  constexpr int TS = D + 8, VPR = D / 8;
  __shared__ __align__(16) uint16_t st[2][kPage * TS];
  const int b = blockIdx.z, h = blockIdx.y, tid = threadIdx.x;
  const int L = a.lens_old[b];
  const int c0 = a.cu_new[b], c1 = a.cu_new[b + 1];
  if (!append_lengths_ok(a, L, c0, c1)) return;
  const int L2 = L + (c1 - c0);
  const int nq1 = nq_of(L2, a.residual, a.group);
  const int start = nq1 > L ? nq1 : L;
  const int q = start / kPage + blockIdx.x;
  const int lo = max(q * kPage, start), hi = min(q * kPage + kPage, L2);
  if (lo >= hi) return;
  const int row = a.seq_slots ? a.seq_slots[b] : b;
  if (row < 0 || row >= a.max_seqs) {
    if (tid == 0) set_err(a.err, TKV_ERR_BAD_SLOT);
    return;
  }
  auto in_elem = [&](const void* base, int tok, int c) -> const uint16_t* {
    return static_cast<const uint16_t*>(base) + (((int64_t)c0 + (tok - L)) * a.n_kv_heads + h) * D + c;
  };
  auto to_f16 = [&](uint16_t x) -> uint16_t {
    if (!a.in_bf16) return x;
    const __half y = __float2half_rn(__uint_as_float((uint32_t)x << 16));
    return __half_as_ushort(y);
  };
  uint16_t* kc = ring_chunk(a, row, h, q * kPage, 0);
  uint16_t* vc = ring_chunk(a, row, h, q * kPage, 1);
  if (hi - lo < kPage) {
    for (int i = tid; i < (hi - lo) * D; i += kResThreads) {
      const int tok = lo + i / D, c = i % D, t = tok % kPage;
      kc[ring_k_off(c, t)] = to_f16(*in_elem(a.k_new, tok, c));
      vc[ring_v_off(c, t)] = to_f16(*in_elem(a.v_new, tok, c));
    }
    return;
  }
  // full chunk: stage the 16 input rows (16-byte aligned by the entry point);
  // unrolled, so every thread's loads are in flight together
  static_assert((2 * kPage * VPR) % kResThreads == 0, "whole staging rounds");
#pragma unroll
  for (int i = tid; i < 2 * kPage * VPR; i += kResThreads) {
    const int kv = i / (kPage * VPR), r = i % (kPage * VPR), t = r / VPR, v = r % VPR;
    uint4 x = *reinterpret_cast<const uint4*>(in_elem(kv ? a.v_new : a.k_new, lo + t, v * 8));
    if (a.in_bf16) {
      uint32_t* w = reinterpret_cast<uint32_t*>(&x);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const __half2 hh = __floats2half2_rn(__uint_as_float(w[j] << 16),
                                             __uint_as_float(w[j] & 0xffff0000u));
        w[j] = *reinterpret_cast<const uint32_t*>(&hh);
      }
    }
    *reinterpret_cast<uint4*>(&st[kv][t * TS + v * 8]) = x;
  }
  __syncthreads();
  // vector v of a block = (bi = v / 32, lane l = 4 g + tig), halves 2 r + e:
  //   K: (t = g + 8 (r & 1), c = 16 bi + 2 tig + 8 (r >> 1) + e)
  //   V: (t = 8 (r >> 1) + 2 tig + e, c = 16 bi + g + 8 (r & 1))
  // i.e. the mma A fragment of the 16 x 16 block bi of K [token][channel]
  // (ldmatrix, matrix m: tokens + 8 (m & 1), channels + 8 (m >> 1)) and of
  // V^T (ldmatrix.trans, matrix m: channels + 8 (m & 1), tokens + 8 (m >> 1)).
  // A warp's 32 consecutive vectors share kv and bi.
#pragma unroll
  for (int i = tid; i < 2 * kPage * VPR; i += kResThreads) {
    const int kv = i / (kPage * VPR), v = i % (kPage * VPR);
    const int bi = v >> 5, l = v & 31, m = l >> 3;
    uint32_t x[4];
    if (kv == 0) {
      ldsm_x4(&st[0][(8 * (m & 1) + (l & 7)) * TS + 16 * bi + 8 * (m >> 1)], x);
    } else {
      ldsm_x4_t(&st[1][(8 * (m >> 1) + (l & 7)) * TS + 16 * bi + 8 * (m & 1)], x);
    }
    reinterpret_cast<uint4*>(kv ? vc : kc)[v] = make_uint4(x[0], x[1], x[2], x[3]);
  }
}

template <int D, int BITS, int G>
static int launch_flush_t(const AppendArgs& a, int num_seqs, cudaStream_t stream) {
  constexpr int smem = sizeof(FlushSmem<D, G>);
  // the attribute belongs to each device's context: set once per device
  // (atomic flags, so concurrent host threads may call this)
  static std::atomic<int> attr_set[kMaxAppendDevices];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return TKV_BACKEND_ERROR;
  if (dev < 0 || dev >= kMaxAppendDevices || !attr_set[dev].load(std::memory_order_relaxed)) {
    if (cudaFuncSetAttribute(flush_groups_kernel<D, BITS, G>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
      return TKV_BACKEND_ERROR;
    if (dev >= 0 && dev < kMaxAppendDevices) attr_set[dev].store(1, std::memory_order_relaxed);
  }
  dim3 grid(2 * (a.max_new / G + 1), a.n_kv_heads, num_seqs);  // x: (group, K or V)
  flush_groups_kernel<D, BITS, G><<<grid, kFlushThreads, smem, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? TKV_OK : TKV_BACKEND_ERROR;
}

template <int D, int BITS>
static int launch_flush_g(const AppendArgs& a, int num_seqs, cudaStream_t stream) {
  switch (a.group) {
    case 16: return launch_flush_t<D, BITS, 16>(a, num_seqs, stream);
    case 32: return launch_flush_t<D, BITS, 32>(a, num_seqs, stream);
    case 64: return launch_flush_t<D, BITS, 64>(a, num_seqs, stream);
    case 128: return launch_flush_t<D, BITS, 128>(a, num_seqs, stream);
  }
  return TKV_NOT_IMPLEMENTED;
}

int launch_append(const AppendArgs& a, int num_seqs, cudaStream_t stream) {
  int st = TKV_NOT_IMPLEMENTED;
  if (a.head_dim == 128)
    st = a.bits == 4 ? launch_flush_g<128, 4>(a, num_seqs, stream)
                     : launch_flush_g<128, 2>(a, num_seqs, stream);
  else if (a.head_dim == 64)
    st = a.bits == 4 ? launch_flush_g<64, 4>(a, num_seqs, stream)
                     : launch_flush_g<64, 2>(a, num_seqs, stream);
  if (st != TKV_OK) return st;
  // written tokens [start, L2): at most min(max_new, R + G - 1) of them (the
  // rest is quantised), from any offset, so they span at most that many
  // + 14, / 16, + 1 ring chunks
  const int span = min(a.max_new, a.residual + a.group - 1);
  dim3 g2((span + 2 * kPage - 2) / kPage, a.n_kv_heads, num_seqs);
  if (a.max_new > 0) {
    if (a.head_dim == 128)
      residual_write_kernel<128><<<g2, kResThreads, 0, stream>>>(a);
    else
      residual_write_kernel<64><<<g2, kResThreads, 0, stream>>>(a);
    if (cudaGetLastError() != cudaSuccess) return TKV_BACKEND_ERROR;
  }
  return TKV_OK;
}

}  // namespace tkv
