// tkv_append.cu -- quantize-on-append into the paged KIVI cache (sm_100a).
//
// Replaces reshape_and_cache (third_party/vllm_kernels/cache_kernels.cu:47-94,
// host wrapper :202-232) for a KIVI cache.  Two launches per call, in stream
// order:
//   1. flush:    one CTA per (key group, kv head, sequence).  It gathers the G
//                tokens of the group (old ones from the fp16 ring, new ones
//                from the input with cp.async), quantises keys per channel and
//                values per token with the reference quantizer
//                (kivi_cache.cu:92-124) and writes the group's pages with
//                coalesced 32- and 128-bit stores.
//   2. residual: copies the new tokens that stay in fp16 into the ring.
// Running the flush before the residual write keeps ring slots that are read
// by (1) from being overwritten by (2) in the same call.
#include "tkv_common.cuh"

namespace tkv {


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

constexpr int kFlushThreads = 128;

__device__ __forceinline__ void cp_async16(void* dst_smem, const void* src_gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_u32(dst_smem)),
               "l"(src_gmem)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;\n" ::: "memory");
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

// Shared memory of the flush kernel: the group's fp16 K and V tiles with
// rows padded by 8 halves (the fragment-order value reads then hit distinct
// banks), per-channel / per-token quantisation parameters and meta words.
template <int D, int G>
struct FlushSmem {
  static constexpr int TS = D + 8;               // row stride in halves
  static constexpr int NVG = D > G ? D / G : 1;  // value groups per token
  uint16_t kt[G * TS];
  uint16_t vt[G * TS];
  float2 kp[D];          // (gmin, scale) per channel
  float2 vp[G * NVG];    // (gmin, scale) per token and value group
  uint32_t kmeta[D];     // step | zero << 16
  uint32_t vmeta[G * NVG];
  int phys[G / kPage];   // the group's pages
};

// One CTA per (key group, kv head, sequence): gathers the G tokens of the
// group (old ones from the fp16 ring, new ones from the input with 16-byte
// cp.async), rounds bf16 input to fp16, computes the key parameters per
// channel and the value parameters per token (and value group), then packs
// and stores the group's pages.
template <int D, int BITS, int G>
__global__ void __launch_bounds__(kFlushThreads) flush_groups_kernel(AppendArgs a) {
  using S_t = FlushSmem<D, G>;
  constexpr int TS = S_t::TS, NVG = S_t::NVG, QMAX = (1 << BITS) - 1;
  constexpr int VG_CH = D > G ? G : D;  // channels per value group
  extern __shared__ __align__(16) uint8_t smem_raw[];
  S_t& S = *reinterpret_cast<S_t*>(smem_raw);
  const int tid = threadIdx.x;
  const int b = blockIdx.z, h = blockIdx.y, gi = blockIdx.x;
  const int L = a.lens_old[b];
  const int c0 = a.cu_new[b], c1 = a.cu_new[b + 1];
  const int T = c1 - c0;
  if (!append_lengths_ok(a, L, c0, c1)) {
    if (tid == 0 && gi == 0 && h == 0) set_err(a.err, TKV_ERR_BAD_LENGTH);
    return;
  }
  const int L2 = L + T;
  const int nq0 = nq_of(L, a.residual, G), nq1 = nq_of(L2, a.residual, G);
  const int t0 = nq0 + gi * G;
  if (t0 >= nq1) return;
  const int row = a.seq_slots ? a.seq_slots[b] : b;
  if (t0 < L && (row < 0 || row >= a.max_seqs)) {
    if (tid == 0) set_err(a.err, TKV_ERR_BAD_SLOT);
    return;
  }
  const int32_t* bt = a.block_tables + (int64_t)b * a.max_blocks;
  const int n_old = min(max(L - t0, 0), G);  // tile rows [0, n_old) come from the ring

  // ---- gather ---------------------------------------------------------------
  // New tokens: input rows [cu_new[b] + (tok - L)][h][0:D], 16-byte vectors
  // (the entry point requires 16-byte aligned inputs).
  constexpr int VPR = D / 8;  // vectors per token row
  for (int i = n_old * VPR + tid; i < G * VPR; i += kFlushThreads) {
    const int t = i / VPR, v = i - t * VPR;
    const int64_t e0 = (((int64_t)c0 + (t0 + t - L)) * a.n_kv_heads + h) * D + v * 8;
    cp_async16(&S.kt[t * TS + v * 8], static_cast<const uint16_t*>(a.k_new) + e0);
    cp_async16(&S.vt[t * TS + v * 8], static_cast<const uint16_t*>(a.v_new) + e0);
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
      const uint4 kw = reinterpret_cast<const uint4*>(ring_chunk(a, row, h, ctok, 0))[v];
      const uint4 vw = reinterpret_cast<const uint4*>(ring_chunk(a, row, h, ctok, 1))[v];
      const uint16_t* ks = reinterpret_cast<const uint16_t*>(&kw);
      const uint16_t* vs = reinterpret_cast<const uint16_t*>(&vw);
      const int bi = v >> 5, l = v & 31, g = l >> 2, tig = l & 3;
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          {  // K block: r = 2*hi + th -> (t = g + 8 th, c = 16 bi + 2 tig + 8 hi + e)
            const int t = ch * kPage + g + 8 * (r & 1), c = 16 * bi + 2 * tig + 8 * (r >> 1) + e;
            if (t < n_old) S.kt[t * TS + c] = ks[2 * r + e];
          }
          {  // V block: r = 2*th + rh -> (t = 8 th + 2 tig + e, c = 16 bi + g + 8 rh)
            const int t = ch * kPage + 8 * (r >> 1) + 2 * tig + e, c = 16 * bi + g + 8 * (r & 1);
            if (t < n_old) S.vt[t * TS + c] = vs[2 * r + e];
          }
        }
    }
  }
  cp_async_wait_all();
  __syncthreads();
  // bf16 input -> fp16 (RN) in place, rows of new tokens
  if (a.in_bf16) {
    for (int i = n_old * VPR + tid; i < G * VPR; i += kFlushThreads) {
      const int t = i / VPR, v = i - t * VPR;
#pragma unroll
      for (int kv = 0; kv < 2; ++kv) {
        uint4* p = reinterpret_cast<uint4*>(&(kv ? S.vt : S.kt)[t * TS + v * 8]);
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
    }
    __syncthreads();
  }

  // ---- pass 1: quantisation parameters -------------------------------------
  if (tid < 64) {
    // keys: channels 2 tid, 2 tid + 1 over the G tokens
    if (2 * tid < D) {
      __half2 mn = __half2half2(__ushort_as_half(0x7c00u)), mx = __half2half2(__ushort_as_half(0xfc00u));
#pragma unroll 8
      for (int t = 0; t < G; ++t) {
        const __half2 x = *reinterpret_cast<const __half2*>(&S.kt[t * TS + 2 * tid]);
        mn = __hmin2(mn, x);
        mx = __hmax2(mx, x);
      }
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int c = 2 * tid + e;
        float gmin, gmax;
        scan_extremes(e ? __high2half(mn) : __low2half(mn), e ? __high2half(mx) : __low2half(mx),
                      gmin, gmax, [&]() {
                        for (int t = 0; t < G; ++t) {
                          const float x = h2f(S.kt[t * TS + c]);
                          if (x == 0.f) return x;
                        }
                        return 0.f;
                      });
        const QParams qp = quant_params(gmin, gmax, QMAX);
        S.kp[c] = make_float2(qp.gmin, qp.scale);
        S.kmeta[c] = (uint32_t)qp.hstep | ((uint32_t)qp.hzero << 16);
      }
    }
  } else {
    // values: per token, per group of VG_CH channels
    for (int j = tid - 64; j < G * NVG; j += kFlushThreads - 64) {
      const int t = j / NVG, vg = j - t * NVG;
      const uint16_t* rowp = &S.vt[t * TS + vg * VG_CH];
      __half2 mn = __half2half2(__ushort_as_half(0x7c00u)), mx = __half2half2(__ushort_as_half(0xfc00u));
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
      S.vp[j] = make_float2(qp.gmin, qp.scale);
      S.vmeta[j] = (uint32_t)qp.hstep | ((uint32_t)qp.hzero << 16);
    }
  }
  __syncthreads();

  auto code = [&](float x, float2 p) {
    int q = __float2int_rn(__fmul_rn(__fsub_rn(x, p.x), p.y));
    q = q < 0 ? 0 : q;
    return static_cast<uint32_t>(q > QMAX ? QMAX : q);
  };
  auto page_base = [&](int pi) -> uint8_t* {
    const int ph = S.phys[pi];
    return (ph < 0 || ph >= a.num_pages)
               ? nullptr
               : a.pool + ((int64_t)ph * a.n_kv_heads + h) * a.page_bytes;
  };

  // ---- pass 2a: key codes, row-major [16 tokens][D * BITS / 8 bytes] --------
  {
    constexpr int CPW = 32 / BITS;     // channels per 32-bit word
    constexpr int NWR = D / CPW;       // words per token row
    constexpr int TSTEP = kFlushThreads / NWR;
    const int w = tid % NWR;
    float2 p[CPW];
#pragma unroll
    for (int n = 0; n < CPW; ++n) p[n] = S.kp[w * CPW + n];
    for (int t = tid / NWR; t < G; t += TSTEP) {
      uint32_t word = 0;
#pragma unroll
      for (int n8 = 0; n8 < CPW; n8 += 8) {
        const uint4 x = *reinterpret_cast<const uint4*>(&S.kt[t * TS + w * CPW + n8]);
        const uint16_t* hx = reinterpret_cast<const uint16_t*>(&x);
#pragma unroll
        for (int n = 0; n < 8; ++n) word |= code(h2f(hx[n]), p[n8 + n]) << (BITS * (n8 + n));
      }
      uint8_t* blk = page_base(t / kPage);
      if (blk)
        reinterpret_cast<uint32_t*>(blk + a.k_codes_off)[(t % kPage) * NWR + w] = word;
    }
  }

  // ---- pass 2b: value codes in mma A-fragment order --------------------------
  {
    constexpr int W = D * BITS / 64;  // words per lane
    constexpr int VW = W < 4 ? W : 4;
    for (int pl = tid; pl < (G / kPage) * 32; pl += kFlushThreads) {
      const int pi = pl >> 5, l = pl & 31, g = l >> 2, tig = l & 3;
      const int tb = pi * kPage;
      uint8_t* blk = page_base(pi);
#pragma unroll
      for (int q = 0; q < W / VW; ++q) {
        uint32_t words[VW];
#pragma unroll
        for (int u = 0; u < VW; ++u) {
          const int wv = q * VW + u;
          uint32_t wd = 0;
#pragma unroll
          for (int k = 0; k < 4; ++k)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int rh = k >> 1, th = k & 1;
              const int t = tb + 8 * th + 2 * tig + e;
              if (BITS == 4) {
                const int c = 16 * wv + g + 8 * rh;
                wd |= code(h2f(S.vt[t * TS + c]), S.vp[t * NVG + c / VG_CH]) << (4 * (k + 4 * e));
              } else {
#pragma unroll
                for (int mbi = 0; mbi < 2; ++mbi) {
                  const int c = 16 * (2 * wv + mbi) + g + 8 * rh;
                  wd |= code(h2f(S.vt[t * TS + c]), S.vp[t * NVG + c / VG_CH])
                        << (2 * (4 * mbi + k + 8 * e));
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

  // ---- pass 2c: value meta [16 tokens][NVG] and key meta slices per page -----
  {
    constexpr int VMW = kPage * NVG;   // value meta words per page
    constexpr int KMW = D * kPage / G; // key meta words per page (= k_meta_slice / 4)
    for (int i = tid; i < (G / kPage) * (VMW + KMW); i += kFlushThreads) {
      const int pi = i / (VMW + KMW), j = i - pi * (VMW + KMW);
      uint8_t* blk = page_base(pi);
      if (!blk) continue;
      if (j < VMW)
        reinterpret_cast<uint32_t*>(blk + a.v_meta_off)[j] = S.vmeta[pi * VMW + j];
      else
        reinterpret_cast<uint32_t*>(blk + a.k_meta_off)[j - VMW] = S.kmeta[pi * KMW + (j - VMW)];
    }
  }
}

// New tokens that stay in fp16: t in [max(nq1, L), L + T) -> ring slot t % C.
__global__ void __launch_bounds__(256) residual_write_kernel(AppendArgs a) {
  const int b = blockIdx.z, h = blockIdx.y;
  const int D = a.head_dim;
  const int L = a.lens_old[b];
  const int T = a.cu_new[b + 1] - a.cu_new[b];
  if (!append_lengths_ok(a, L, a.cu_new[b], a.cu_new[b + 1])) return;
  const int L2 = L + T;
  const int nq1 = nq_of(L2, a.residual, a.group);
  const int start = nq1 > L ? nq1 : L;
  const int i0 = blockIdx.x * kPage;  // new-token index range [i0, i0 + 16)
  if (L + i0 + kPage <= start || i0 >= T) return;
  const int row = a.seq_slots ? a.seq_slots[b] : b;
  if (row < 0 || row >= a.max_seqs) {
    if (threadIdx.x == 0) set_err(a.err, TKV_ERR_BAD_SLOT);
    return;
  }
  for (int i = threadIdx.x; i < kPage * D; i += blockDim.x) {
    const int ti = i / D, c = i % D;
    const int n = i0 + ti;
    const int tok = L + n;
    if (n >= T || tok < start) continue;
    const int64_t e0 = (((int64_t)a.cu_new[b] + n) * a.n_kv_heads + h) * D + c;
    uint16_t kh = static_cast<const uint16_t*>(a.k_new)[e0];
    uint16_t vh = static_cast<const uint16_t*>(a.v_new)[e0];
    if (a.in_bf16) {
      __half k16 = __float2half_rn(__bfloat162float(*reinterpret_cast<__nv_bfloat16*>(&kh)));
      __half v16 = __float2half_rn(__bfloat162float(*reinterpret_cast<__nv_bfloat16*>(&vh)));
      kh = *reinterpret_cast<uint16_t*>(&k16);
      vh = *reinterpret_cast<uint16_t*>(&v16);
    }
    const int t = (tok % a.ring_cap) % kPage;
    ring_chunk(a, row, h, tok, 0)[ring_k_off(c, t)] = kh;
    ring_chunk(a, row, h, tok, 1)[ring_v_off(c, t)] = vh;
  }
}

template <int D, int BITS, int G>
static int launch_flush_t(const AppendArgs& a, int num_seqs, cudaStream_t stream) {
  constexpr int smem = sizeof(FlushSmem<D, G>);
  static bool attr_set = false;
  if (!attr_set) {
    if (cudaFuncSetAttribute(flush_groups_kernel<D, BITS, G>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
      return TKV_BACKEND_ERROR;
    attr_set = true;
  }
  dim3 grid(a.max_new / G + 1, a.n_kv_heads, num_seqs);
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
  dim3 g2((a.max_new + kPage - 1) / kPage, a.n_kv_heads, num_seqs);
  if (g2.x > 0) {
    residual_write_kernel<<<g2, 256, 0, stream>>>(a);
    if (cudaGetLastError() != cudaSuccess) return TKV_BACKEND_ERROR;
  }
  return TKV_OK;
}

}  // namespace tkv
