// tkv_refformat.cu -- the reference's per-vector KIVI format on sm_100a.
//
// Byte-compatible with kivi_compress_kernel / kivi_decompress_kernel
// (src/inference/backends/cuda/compression/kivi_cache.cu:23-198): per KV
// vector, the top-n_outliers channels by |x| as (u8 channel, fp16 value) in
// the reference's slot order, then the remaining channels min-max quantised to
// 4 bits in groups of `group_size`.
//
// B200 layout of the work: one warp per vector instead of one thread; the
// vector is read with coalesced loads into shared memory, the order-dependent
// outlier slot algorithm runs on one lane (it is inherently sequential and
// its slot order is part of the byte format), and the channel compaction,
// group statistics, codes and stores run across the warp.
#include "tkv_common.cuh"

namespace tkv {

constexpr int kRefMaxDim = 128;      // KIVI_MAX_HEAD_DIM (kivi_cache.cuh:27)
constexpr int kRefMaxOutliers = 64;  // KIVI_MAX_OUTLIERS (kivi_cache.cuh:28)
constexpr int kRefWarps = 8;         // vectors per CTA

enum RefMode { kCompress = 0, kDecompress = 1, kRoundtrip = 2 };

struct RefWarpSmem {
  float val[kRefMaxDim];        // input values (compress) / results (decompress)
  uint16_t raw[kRefMaxDim];     // raw fp16 bits of the input vector
  float omag[kRefMaxOutliers];  // outlier slot magnitudes
  uint8_t oidx[kRefMaxOutliers];
  uint8_t flag[kRefMaxDim];     // is_outlier (compress) / written (decompress)
  uint8_t rch[kRefMaxDim];      // residual index -> channel
  float res[kRefMaxDim];        // residual values in residual order
};

__host__ __device__ inline size_t ref_bytes(int head_dim, int n_outliers, int group_size) {
  int n_res = head_dim - n_outliers;
  int n_groups = (n_res + group_size - 1) / group_size;
  return static_cast<size_t>(n_outliers) * 3 +
         static_cast<size_t>(n_groups) * static_cast<size_t>(group_size / 2 + 4);
}

// Sequential outlier slot algorithm (kivi_cache.cu:33-63) on lane 0.
__device__ void select_outliers(RefWarpSmem& s, int head_dim, int n_out) {
  for (int i = 0; i < n_out; ++i) {
    s.oidx[i] = 0;
    s.omag[i] = -1.f;
  }
  float min_mag = -1.f;
  int min_pos = 0;
  for (int d = 0; d < head_dim; ++d) {
    float v = fabsf(s.val[d]);
    if (v > min_mag) {
      if (n_out > 0) {
        s.oidx[min_pos] = static_cast<uint8_t>(d);
        s.omag[min_pos] = v;
        min_mag = s.omag[0];
        min_pos = 0;
        for (int i = 1; i < n_out; ++i)
          if (s.omag[i] < min_mag) {
            min_mag = s.omag[i];
            min_pos = i;
          }
      } else {
        // n_out == 0: the reference still records v in slot 0 of its scratch
        // array, which makes the running minimum the running maximum; nothing
        // is ever written out, so only min_mag matters here.
        min_mag = v;
      }
    }
  }
}

template <int MODE>
__global__ void __launch_bounds__(kRefWarps * 32)
    ref_kivi_kernel(const void* in, void* out, int n_vecs, int head_dim,
                    int n_outliers, int group_size) {
  __shared__ RefWarpSmem smem[kRefWarps];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int vec = blockIdx.x * kRefWarps + warp;
  if (vec >= n_vecs) return;
  RefWarpSmem& s = smem[warp];

  const int n_out = n_outliers;  // validated on the host: 0 <= n_out <= min(64, head_dim)
  const int n_res = head_dim - n_out;
  const int n_groups = (n_res + group_size - 1) / group_size;
  const size_t stride = ref_bytes(head_dim, n_outliers, group_size);
  const int rec = group_size / 2 + 4;  // bytes of one full group record (group_size even)

  if (MODE == kCompress || MODE == kRoundtrip) {
    const uint16_t* src = static_cast<const uint16_t*>(in) + static_cast<size_t>(vec) * head_dim;
    for (int c = lane; c < head_dim; c += 32) {
      uint16_t h = src[c];
      s.raw[c] = h;
      s.val[c] = __half2float(*reinterpret_cast<__half*>(&h));
      s.flag[c] = 0;
    }
    __syncwarp();
    if (lane == 0) {
      select_outliers(s, head_dim, n_out);
      for (int i = 0; i < n_out; ++i) s.flag[s.oidx[i]] = 1;
    }
    __syncwarp();
    // residual compaction in channel order, first n_res non-outlier channels
    int running = 0;
    for (int c0 = 0; c0 < head_dim; c0 += 32) {
      int c = c0 + lane;
      bool f = (c < head_dim) && !s.flag[c];
      uint32_t m = __ballot_sync(0xffffffffu, f);
      int r = running + __popc(m & ((1u << lane) - 1u));
      if (f && r < n_res) {
        s.res[r] = s.val[c];
        s.rch[r] = static_cast<uint8_t>(c);
      }
      running += __popc(m);
    }
    __syncwarp();
    if (MODE == kCompress) {
      uint8_t* dst = static_cast<uint8_t*>(out) + static_cast<size_t>(vec) * stride;
      for (int i = lane; i < n_out; i += 32) {
        uint8_t ch = s.oidx[i];
        uint16_t h = s.raw[ch];
        dst[3 * i] = ch;
        dst[3 * i + 1] = static_cast<uint8_t>(h & 0xff);
        dst[3 * i + 2] = static_cast<uint8_t>(h >> 8);
      }
      for (int g = lane; g < n_groups; g += 32) {
        int gs = g * group_size, ge = min(gs + group_size, n_res);
        float gmin = FLT_MAX, gmax = -FLT_MAX;
        for (int i = gs; i < ge; ++i) {
          float v = s.res[i];
          if (v < gmin) gmin = v;
          if (v > gmax) gmax = v;
        }
        QParams qp = quant_params(gmin, gmax, 15);
        uint8_t* p = dst + 3 * n_out + static_cast<size_t>(g) * rec;
        for (int i = gs; i < ge; i += 2) {
          int q0 = quant_code(s.res[i], qp, 15);
          int q1 = (i + 1 < ge) ? quant_code(s.res[i + 1], qp, 15) : 0;
          *p++ = static_cast<uint8_t>((q1 << 4) | q0);
        }
        p[0] = static_cast<uint8_t>(qp.hstep & 0xff);
        p[1] = static_cast<uint8_t>(qp.hstep >> 8);
        p[2] = static_cast<uint8_t>(qp.hzero & 0xff);
        p[3] = static_cast<uint8_t>(qp.hzero >> 8);
      }
      return;
    }
    if constexpr (MODE == kRoundtrip) {
    // kRoundtrip: the vector the reference's compress + decompress pair
    // writes back (kv_compression_pass.cpp:207-212), without the byte record.
    // 1) each lane quantises and dequantises its groups in place in s.res,
    //    using the fp16 step/zero exactly as the decompress side reads them;
    for (int g = lane; g < n_groups; g += 32) {
      int gs = g * group_size, ge = min(gs + group_size, n_res);
      float gmin = FLT_MAX, gmax = -FLT_MAX;
      for (int i = gs; i < ge; ++i) {
        float v = s.res[i];
        if (v < gmin) gmin = v;
        if (v > gmax) gmax = v;
      }
      QParams qp = quant_params(gmin, gmax, 15);
      float sc = __half2float(*reinterpret_cast<__half*>(&qp.hstep));
      float zr = __half2float(*reinterpret_cast<__half*>(&qp.hzero));
      for (int i = gs; i < ge; ++i) {
        int q = quant_code(s.res[i], qp, 15);
        s.res[i] = __fmaf_rn(static_cast<float>(q), sc, zr);
      }
    }
    __syncwarp();
    // 2) assemble the decompressed vector: zeros, outliers in slot order
    //    (kivi_cache.cu:144-151), then residual channels, which are the
    //    channels no outlier record names -- the same list as s.rch.
    float* result = s.val;
    for (int c = lane; c < head_dim; c += 32) result[c] = 0.f;
    __syncwarp();
    if (lane == 0)
      for (int i = 0; i < n_out; ++i) {
        uint16_t h = s.raw[s.oidx[i]];
        result[s.oidx[i]] = __half2float(*reinterpret_cast<__half*>(&h));
      }
    __syncwarp();
    for (int r = lane; r < n_res; r += 32) result[s.rch[r]] = s.res[r];
    __syncwarp();
    uint16_t* dstv = static_cast<uint16_t*>(out) + static_cast<size_t>(vec) * head_dim;
    for (int c = lane; c < head_dim; c += 32) {
      __half h = __float2half_rn(result[c]);
      dstv[c] = *reinterpret_cast<uint16_t*>(&h);
    }
    }
    return;
  }

  // ---------------- kDecompress ----------------
  const uint8_t* src = static_cast<const uint8_t*>(in) + static_cast<size_t>(vec) * stride;
  uint16_t* dst = static_cast<uint16_t*>(out) + static_cast<size_t>(vec) * head_dim;
  for (int c = lane; c < head_dim; c += 32) {
    s.val[c] = 0.f;
    s.flag[c] = 0;
  }
  __syncwarp();
  if (lane == 0) {
    for (int i = 0; i < n_out; ++i) {
      uint8_t ch = src[3 * i];
      uint16_t h = static_cast<uint16_t>(src[3 * i + 1]) | (static_cast<uint16_t>(src[3 * i + 2]) << 8);
      if (ch < head_dim) {
        s.val[ch] = __half2float(*reinterpret_cast<__half*>(&h));
        s.flag[ch] = 1;
      }
    }
  }
  __syncwarp();
  int running = 0;
  for (int c0 = 0; c0 < head_dim; c0 += 32) {
    int c = c0 + lane;
    bool f = (c < head_dim) && !s.flag[c];
    uint32_t m = __ballot_sync(0xffffffffu, f);
    int r = running + __popc(m & ((1u << lane) - 1u));
    if (f && r < n_res) s.rch[r] = static_cast<uint8_t>(c);
    running += __popc(m);
  }
  const int n_rch = min(running, n_res);
  __syncwarp();
  for (int g = lane; g < n_groups; g += 32) {
    int gs = g * group_size, ge = min(gs + group_size, n_res);
    const uint8_t* pack = src + 3 * n_out + static_cast<size_t>(g) * rec;
    int pb = (ge - gs + 1) / 2;
    uint16_t hs = static_cast<uint16_t>(pack[pb]) | (static_cast<uint16_t>(pack[pb + 1]) << 8);
    uint16_t hz = static_cast<uint16_t>(pack[pb + 2]) | (static_cast<uint16_t>(pack[pb + 3]) << 8);
    float sc = __half2float(*reinterpret_cast<__half*>(&hs));
    float zr = __half2float(*reinterpret_cast<__half*>(&hz));
    for (int i = gs; i < ge; ++i) {
      int b = pack[(i - gs) / 2];
      int nib = ((i - gs) % 2 == 0) ? (b & 0x0f) : (b >> 4);
      if (i < n_rch) s.val[s.rch[i]] = __fmaf_rn(static_cast<float>(nib), sc, zr);
    }
  }
  __syncwarp();
  for (int c = lane; c < head_dim; c += 32) {
    __half h = __float2half_rn(s.val[c]);
    dst[c] = *reinterpret_cast<uint16_t*>(&h);
  }
}

int launch_ref_kivi(int mode, const void* in, void* out, int n_vecs, int head_dim, int n_outliers,
                    int group_size, cudaStream_t stream) {
  int blocks = (n_vecs + kRefWarps - 1) / kRefWarps;
  switch (mode) {
    case kCompress:
      ref_kivi_kernel<kCompress><<<blocks, kRefWarps * 32, 0, stream>>>(in, out, n_vecs, head_dim,
                                                                       n_outliers, group_size);
      break;
    case kDecompress:
      ref_kivi_kernel<kDecompress><<<blocks, kRefWarps * 32, 0, stream>>>(
          in, out, n_vecs, head_dim, n_outliers, group_size);
      break;
    default:
      ref_kivi_kernel<kRoundtrip><<<blocks, kRefWarps * 32, 0, stream>>>(
          in, out, n_vecs, head_dim, n_outliers, group_size);
      break;
  }
  return cudaGetLastError() == cudaSuccess ? TKV_OK : TKV_BACKEND_ERROR;
}

}  // namespace tkv
