// tkv_append.cu -- quantize-on-append into the paged KIVI cache (sm_100a).
//
// Replaces reshape_and_cache (third_party/vllm_kernels/cache_kernels.cu:47-94,
// host wrapper :202-232) for a KIVI cache.  Two launches per call, in stream
// order:
//   1. flush:    one CTA per (key group, kv head, sequence).  It gathers the G
//                tokens of the group (old ones from the fp16 ring, new ones
//                from the input), quantises keys per channel and values per
//                token with the reference quantizer (kivi_cache.cu:92-124) and
//                writes the group's pages with coalesced 32-bit stores.
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

constexpr int kFlushThreads = 256;
constexpr int kMaxG = 128, kMaxD = 128;

// Shared memory of the flush kernel: fp16 tiles with a padded row stride
// (D + 2 halves) so the per-token value scans hit distinct banks, plus 1-byte
// code matrices and the fp16 meta.
struct FlushSmem {
  uint16_t kt[kMaxG * (kMaxD + 2)];
  uint16_t vt[kMaxG * (kMaxD + 2)];
  uint8_t kq[kMaxG * kMaxD];
  uint8_t vq[kMaxG * kMaxD];
  uint32_t kmeta[kMaxD];          // (step | zero << 16) per channel
  uint32_t vmeta[kMaxG * 8];      // (step | zero << 16) per token and value group
};

__global__ void __launch_bounds__(kFlushThreads) flush_groups_kernel(AppendArgs a) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  FlushSmem& S = *reinterpret_cast<FlushSmem*>(smem_raw);
  const int b = blockIdx.z, h = blockIdx.y, gi = blockIdx.x;
  const int D = a.head_dim, G = a.group, TS = D + 2;
  const int L = a.lens_old[b];
  const int c0 = a.cu_new[b], c1 = a.cu_new[b + 1];
  const int T = c1 - c0;
  if (!append_lengths_ok(a, L, c0, c1)) {
    if (threadIdx.x == 0 && gi == 0 && h == 0) set_err(a.err, TKV_ERR_BAD_LENGTH);
    return;
  }
  const int L2 = L + T;
  const int nq0 = nq_of(L, a.residual, G), nq1 = nq_of(L2, a.residual, G);
  const int t0 = nq0 + gi * G;
  if (t0 >= nq1) return;
  const int row = a.seq_slots ? a.seq_slots[b] : b;
  if (t0 < L && (row < 0 || row >= a.max_seqs)) {
    if (threadIdx.x == 0) set_err(a.err, TKV_ERR_BAD_SLOT);
    return;
  }
  const int32_t* bt = a.block_tables + (int64_t)b * a.max_blocks;
  const int qmax = (1 << a.bits) - 1;

  // ---- gather the G x D tiles (fp16 values) --------------------------------
  // Old tokens come from ring chunks (fragment order, 16-byte vectors); new
  // tokens from input rows [cu_new[b] + (t - L)][h][0:D].
  const int vec_per_row = D / 8;  // 16-byte vectors per token row
  for (int i = threadIdx.x; i < G * vec_per_row; i += kFlushThreads) {
    const int t = i / vec_per_row, v = i % vec_per_row;
    const int tok = t0 + t;
    if (tok < L) continue;  // old token: gathered from its ring chunk below
    const int64_t in_row = ((int64_t)a.cu_new[b] + (tok - L)) * a.n_kv_heads + h;
    const int64_t e0 = in_row * D + v * 8;
    uint4 kw = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(a.k_new) + e0);
    uint4 vw = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(a.v_new) + e0);
    const uint16_t* ks = reinterpret_cast<const uint16_t*>(&kw);
    const uint16_t* vs = reinterpret_cast<const uint16_t*>(&vw);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      uint16_t kh = ks[j], vh = vs[j];
      if (a.in_bf16) {
        __half k16 = __float2half_rn(__bfloat162float(*reinterpret_cast<__nv_bfloat16*>(&kh)));
        __half v16 = __float2half_rn(__bfloat162float(*reinterpret_cast<__nv_bfloat16*>(&vh)));
        kh = *reinterpret_cast<uint16_t*>(&k16);
        vh = *reinterpret_cast<uint16_t*>(&v16);
      }
      S.kt[t * TS + v * 8 + j] = kh;
      S.vt[t * TS + v * 8 + j] = vh;
    }
  }
  // Ring chunks: handled chunk-wise so each 16-byte vector is read once.
  {
    const int first_chunk_tok = t0, last_tok = min(t0 + G, L);
    const int vecs_per_chunk = kPage * D / 8;
    const int n_chunks = last_tok > first_chunk_tok ? (last_tok - first_chunk_tok + kPage - 1) / kPage : 0;
    for (int i = threadIdx.x; i < n_chunks * vecs_per_chunk; i += kFlushThreads) {
      const int ch = i / vecs_per_chunk, v = i % vecs_per_chunk;
      const int ctok = t0 + ch * kPage;  // chunk's first token (t0 is a multiple of 16)
      const uint16_t* kc = ring_chunk(a, row, h, ctok, 0);
      const uint16_t* vc = ring_chunk(a, row, h, ctok, 1);
      uint4 kw = reinterpret_cast<const uint4*>(kc)[v];
      uint4 vw = reinterpret_cast<const uint4*>(vc)[v];
      const uint16_t* ks = reinterpret_cast<const uint16_t*>(&kw);
      const uint16_t* vs = reinterpret_cast<const uint16_t*>(&vw);
      // vector v = (block index bi, lane l): bi = v / 32, l = v % 32
      const int bi = v >> 5, l = v & 31;
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          // K block: lane l = 4*g + tig; r = 2*hi + th; element (t = g + 8 th, c = 16 bi + 2 tig + 8 hi + e)
          {
            const int g = l >> 2, tig = l & 3, hi = r >> 1, th = r & 1;
            const int t = g + 8 * th, c = 16 * bi + 2 * tig + 8 * hi + e;
            const int tt = ch * kPage + t;
            if (ctok + t < L) S.kt[tt * TS + c] = ks[2 * r + e];
          }
          // V block: lane l = 4*g + tig; r = 2*th + rh; element (t = 8 th + 2 tig + e, c = 16 bi + g + 8 rh)
          {
            const int g = l >> 2, tig = l & 3, th = r >> 1, rh = r & 1;
            const int t = 8 * th + 2 * tig + e, c = 16 * bi + g + 8 * rh;
            const int tt = ch * kPage + t;
            if (ctok + t < L) S.vt[tt * TS + c] = vs[2 * r + e];
          }
        }
    }
  }
  __syncthreads();

  // ---- quantise: keys per channel over G tokens, values per token over G channels
  const int nv = G * a.n_vgroups;
  for (int i = threadIdx.x; i < D + nv; i += kFlushThreads) {
    if (i < D) {
      const int c = i;
      float gmin = FLT_MAX, gmax = -FLT_MAX;
      for (int t = 0; t < G; ++t) {
        float x = __half2float(*reinterpret_cast<const __half*>(&S.kt[t * TS + c]));
        if (x < gmin) gmin = x;
        if (x > gmax) gmax = x;
      }
      QParams qp = quant_params(gmin, gmax, qmax);
      for (int t = 0; t < G; ++t) {
        float x = __half2float(*reinterpret_cast<const __half*>(&S.kt[t * TS + c]));
        S.kq[t * D + c] = static_cast<uint8_t>(quant_code(x, qp, qmax));
      }
      S.kmeta[c] = (uint32_t)qp.hstep | ((uint32_t)qp.hzero << 16);
    } else {
      const int j = i - D, t = j / a.n_vgroups, vg = j % a.n_vgroups;
      const int c0 = vg * G, c1 = min(D, c0 + G);
      float gmin = FLT_MAX, gmax = -FLT_MAX;
      for (int c = c0; c < c1; ++c) {
        float x = __half2float(*reinterpret_cast<const __half*>(&S.vt[t * TS + c]));
        if (x < gmin) gmin = x;
        if (x > gmax) gmax = x;
      }
      QParams qp = quant_params(gmin, gmax, qmax);
      for (int c = c0; c < c1; ++c) {
        float x = __half2float(*reinterpret_cast<const __half*>(&S.vt[t * TS + c]));
        S.vq[t * D + c] = static_cast<uint8_t>(quant_code(x, qp, qmax));
      }
      S.vmeta[t * a.n_vgroups + vg] = (uint32_t)qp.hstep | ((uint32_t)qp.hzero << 16);
    }
  }
  __syncthreads();

  // ---- pack and store the group's pages, one 32-bit word per thread step ---
  const int pages = G / kPage;
  const int rb = D * a.bits / 8;            // K code bytes per token row
  const int kwords = kPage * rb / 4;        // K code words per page
  const int W = D * a.bits / 64;            // V code words per lane
  const int VW = W < 4 ? W : 4;
  const int vwords = 32 * W;                // V code words per page
  const int vmwords = kPage * a.n_vgroups;  // V meta words per page
  const int kmwords = a.k_meta_slice / 4;   // K meta words per page
  const int per_page = kwords + vwords + vmwords + kmwords;
  for (int i = threadIdx.x; i < pages * per_page; i += kFlushThreads) {
    const int pi = i / per_page;
    int j = i % per_page;
    const int phys = bt[(t0 / kPage) + pi];
    if (phys < 0 || phys >= a.num_pages) {
      set_err(a.err, TKV_ERR_BAD_PAGE);
      continue;
    }
    uint8_t* blk = a.pool + ((int64_t)phys * a.n_kv_heads + h) * a.page_bytes;
    const int tb = pi * kPage;  // first token row of this page inside the tile
    if (j < kwords) {
      const int t = j / (rb / 4), wj = j % (rb / 4);
      const uint8_t* q = &S.kq[(tb + t) * D];
      uint32_t w = 0;
      if (a.bits == 4) {
#pragma unroll
        for (int n = 0; n < 8; ++n) w |= (uint32_t)q[8 * wj + n] << (4 * n);
      } else {
#pragma unroll
        for (int n = 0; n < 16; ++n) w |= (uint32_t)q[16 * wj + n] << (2 * n);
      }
      reinterpret_cast<uint32_t*>(blk + a.k_codes_off)[t * (rb / 4) + wj] = w;
      continue;
    }
    j -= kwords;
    if (j < vwords) {
      const int l = j / W, wv = j % W;
      const int g = l >> 2, tig = l & 3;
      uint32_t w = 0;
#pragma unroll
      for (int k = 0; k < 4; ++k)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int rh = k >> 1, th = k & 1;
          const int t = 8 * th + 2 * tig + e;
          if (a.bits == 4) {
            const int c = 16 * wv + g + 8 * rh;
            w |= (uint32_t)S.vq[(tb + t) * D + c] << (4 * (k + 4 * e));
          } else {
#pragma unroll
            for (int mbi = 0; mbi < 2; ++mbi) {
              const int c = 16 * (2 * wv + mbi) + g + 8 * rh;
              w |= (uint32_t)S.vq[(tb + t) * D + c] << (2 * (4 * mbi + k + 8 * e));
            }
          }
        }
      const int off = ((wv / VW) * 32 + l) * (4 * VW) + (wv % VW) * 4;
      *reinterpret_cast<uint32_t*>(blk + a.v_codes_off + off) = w;
      continue;
    }
    j -= vwords;
    if (j < vmwords) {
      const int t = j / a.n_vgroups, vg = j % a.n_vgroups;
      reinterpret_cast<uint32_t*>(blk + a.v_meta_off)[j] = S.vmeta[(tb + t) * a.n_vgroups + vg];
      continue;
    }
    j -= vmwords;
    // K meta slice pi: words [pi * kmwords, (pi+1) * kmwords) of kmeta
    reinterpret_cast<uint32_t*>(blk + a.k_meta_off)[j] = S.kmeta[pi * kmwords + j];
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

size_t flush_smem_bytes() { return sizeof(FlushSmem); }

int launch_append(const AppendArgs& a, int num_seqs, cudaStream_t stream) {
  static bool attr_set = false;
  const size_t smem = sizeof(FlushSmem);
  if (!attr_set) {
    if (cudaFuncSetAttribute(flush_groups_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
      return TKV_BACKEND_ERROR;
    attr_set = true;
  }
  const int max_groups = a.max_new / a.group + 1;
  dim3 g1(max_groups, a.n_kv_heads, num_seqs);
  flush_groups_kernel<<<g1, kFlushThreads, smem, stream>>>(a);
  if (cudaGetLastError() != cudaSuccess) return TKV_BACKEND_ERROR;
  dim3 g2((a.max_new + kPage - 1) / kPage, a.n_kv_heads, num_seqs);
  if (g2.x > 0) {
    residual_write_kernel<<<g2, 256, 0, stream>>>(a);
    if (cudaGetLastError() != cudaSuccess) return TKV_BACKEND_ERROR;
  }
  return TKV_OK;
}

}  // namespace tkv
