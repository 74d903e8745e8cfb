// tkv_exchange.cu -- the peer-memory side of a token-split decode: the GPUs
// of one node each hold one range of a long sequence's quantised splits; each
// reduces its range to one unnormalised partial per (sequence, q head) and
// stores it into every GPU's exchange buffer over NVLink (the slot-parallel
// merge kernel of tkv_stream.cu does that in its publish mode), then raises
// its flag there.  This file holds the kernel that publishes empty partials
// for a GPU without splits and the kernel that waits for every GPU's flag and
// merges the world slots into the output.  Plain peer stores and loads: no
// NCCL call, no multicast.
//
// Ordering: a publishing CTA fences its peer stores at system scope before it
// counts itself; the last CTA of the launch fences again and releases the
// flags (st.release.sys).  The merge acquires every flag (ld.acquire.sys) and
// then reads the slots with ld.global.cv.  Consecutive steps use alternate
// sets, so a GPU one step ahead of a peer writes the other set.  The waits
// are bounded by the global timer (about 2 s, then TKV_ERR_TIMEOUT).
#include "tkv_common.cuh"

namespace tkv {
namespace {

constexpr uint64_t kExWaitNs = 2000000000ull;
constexpr int kExThreads = 128;

__device__ __forceinline__ uint32_t ex_step(const ExPub& x) {
  return *reinterpret_cast<volatile const uint32_t*>(x.state);
}

// A GPU whose range holds no token: m = -inf, l = 0, o = 0 for every row.
__global__ void __launch_bounds__(kExThreads) ex_publish_empty_kernel(ExPub pub, int D) {
  const uint32_t step = ex_step(pub);
  const int64_t i0 = blockIdx.x;
  for (int c = threadIdx.x; c < D; c += blockDim.x) ex_store_row(pub, step, i0, c, 0.f);
  if (threadIdx.x == 0) ex_store_ml(pub, step, i0, -INFINITY, 0.f);
  ex_signal(pub, step);
}

// One CTA per (sequence, q head) row: wait for every GPU's flag of this step,
// merge the world slots by log-sum-exp (paged_attention_v2.cu:132-170) into
// out; the last CTA advances this GPU's step.
__global__ void __launch_bounds__(kExThreads)
    ex_merge_kernel(ExPub pub, int D, void* __restrict__ out, int out_dtype, int* err) {
  __shared__ int s_ok;
  const uint32_t step = ex_step(pub);
  const uint32_t s = step & 1u;
  if (threadIdx.x == 0) {
    const uint32_t* fl = pub.flags[pub.rank] + s * kMaxPeers;
    const uint64_t t0 = global_ns();
    bool ok = false;
    for (;;) {
      ok = true;
      for (int r = 0; r < pub.world; ++r) ok = ok && ld_acquire_sys(fl + r) == step + 1u;
      if (ok || global_ns() - t0 > kExWaitNs) break;
      __nanosleep(128);
    }
    if (!ok) set_err(err, TKV_ERR_TIMEOUT);
    s_ok = ok;
  }
  __syncthreads();
  const bool ok = s_ok != 0;
  const int64_t i0 = blockIdx.x;
  const float* base = pub.set0[pub.rank] + s * pub.set_floats + i0 * pub.rs;
  const long long slot = static_cast<long long>(pub.rows) * pub.rs;
  float M = -INFINITY, L = 0.f;
  if (ok) {
    for (int r = 0; r < pub.world; ++r) M = fmaxf(M, __ldcv(base + r * slot));
    for (int r = 0; r < pub.world; ++r) {
      const float m = __ldcv(base + r * slot);
      if (m != -INFINITY) L = fmaf(__ldcv(base + r * slot + 1), fast_exp2(m - M), L);
    }
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    float acc = 0.f;
    if (ok)
      for (int r = 0; r < pub.world; ++r) {
        const float m = __ldcv(base + r * slot);
        if (m != -INFINITY) acc = fmaf(__ldcv(base + r * slot + kExRowPad + c), fast_exp2(m - M), acc);
      }
    const float v = acc * inv;
    const int64_t oi = i0 * D + c;
    if (out_dtype == TKV_F32)
      static_cast<float*>(out)[oi] = v;
    else if (out_dtype == TKV_BF16)
      static_cast<__nv_bfloat16*>(out)[oi] = __float2bfloat16_rn(v);
    else
      static_cast<__half*>(out)[oi] = __float2half_rn(v);
  }
  __syncthreads();
  if (threadIdx.x == 0 && atomicAdd(&pub.state[2], 1u) == gridDim.x - 1) {
    pub.state[2] = 0u;
    __threadfence();
    *reinterpret_cast<volatile uint32_t*>(pub.state) = step + 1u;
  }
}

}  // namespace

int launch_ex_publish_empty(const ExPub& pub, int head_dim, cudaStream_t stream) {
  ex_publish_empty_kernel<<<pub.rows, kExThreads, 0, stream>>>(pub, head_dim);
  return cudaGetLastError() == cudaSuccess ? TKV_OK : TKV_BACKEND_ERROR;
}

int launch_ex_merge(const ExPub& pub, int head_dim, void* out, int out_dtype, int* err,
                    cudaStream_t stream) {
  ex_merge_kernel<<<pub.rows, kExThreads, 0, stream>>>(pub, head_dim, out, out_dtype, err);
  return cudaGetLastError() == cudaSuccess ? TKV_OK : TKV_BACKEND_ERROR;
}

}  // namespace tkv
