// Test-only check of the tcgen05 pieces in tkv_umma.cuh (compiled by
// tests/test_gpu_umma.py): one CTA of 128 threads computes
//   D[128][N] (f32) = A0 B0^T + A1 B1^T
// from row-major 16-bit A [128][128] and B [N][128] staged into the K-major,
// no-swizzle shared-memory layout (or, with a_tmem, A written row by row into
// tensor memory with tcgen05.st), eight K = 16 MMAs per term accumulating in
// tensor memory, read back by the four warps with tcgen05.ld.
#include "tkv_umma.cuh"

using namespace tkv;

namespace {

constexpr int kM = 128, kK = 128, kMaxN = 256;

// a_tmem: A goes to tensor memory (columns kATmem.., each thread its row)
// instead of shared memory, and the MMAs read it from there.
constexpr uint32_t kATmem = 256;
__global__ void __launch_bounds__(128) umma_gemm_kernel(const uint16_t* A0, const uint16_t* B0,
                                                        const uint16_t* A1, const uint16_t* B1,
                                                        float* D, int N, int bf16, int a_tmem,
                                                        int* err) {
  extern __shared__ __align__(128) uint8_t sm[];
  uint8_t* sa = sm;
  uint8_t* sb = sm + kM * kK * 2;
  uint64_t* bar = reinterpret_cast<uint64_t*>(sb + kMaxN * kK * 2);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (warp == 0) umma::alloc(tslot, 2 * kMaxN);
  if (tid == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tmem = *tslot;
  bool ok = true;
  for (int round = 0; round < 2 && ok; ++round) {
    const uint16_t* A = round ? A1 : A0;
    const uint16_t* B = round ? B1 : B0;
    if (a_tmem) {
      // row tid of A: 64 columns of packed 16-bit pairs (lane = row)
      const uint32_t lane_base = static_cast<uint32_t>(32 * warp) << 16;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float v[32];
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const uint32_t lo = A[tid * kK + 2 * (32 * h + c)], hi = A[tid * kK + 2 * (32 * h + c) + 1];
          v[c] = __uint_as_float(lo | (hi << 16));
        }
        umma::st32(tmem + lane_base + kATmem + 32 * h, v);
      }
      umma::wait_st();
    } else {
      for (int i = tid; i < kM * kK; i += blockDim.x)
        *reinterpret_cast<uint16_t*>(sa + umma::umma_off(i / kK, i % kK, kK)) = A[i];
    }
    for (int i = tid; i < N * kK; i += blockDim.x)
      *reinterpret_cast<uint16_t*>(sb + umma::umma_off(i / kK, i % kK, kK)) = B[i];
    umma::fence_smem_to_async();
    umma::fence_before_sync();
    __syncthreads();
    if (tid == 0) {
      umma::fence_after_sync();
      const uint32_t idesc = umma::idesc_f16(kM, N, bf16 != 0);
      for (int kk = 0; kk < kK / 16; ++kk) {
        const uint64_t ad = umma::smem_desc(smem_u32(sa) + kk * 256, 128, 16 * kK);
        const uint64_t bd = umma::smem_desc(smem_u32(sb) + kk * 256, 128, 16 * kK);
        if (a_tmem)
          umma::mma_f16_ta(tmem, tmem + kATmem + 8 * kk, bd, idesc, round > 0 || kk > 0);
        else
          umma::mma_f16(tmem, ad, bd, idesc, round > 0 || kk > 0);
      }
      umma::commit(bar);
    }
    ok = mbar_wait(bar, round & 1, err);
    umma::fence_after_sync();
    __syncthreads();
  }
  if (ok) {
    for (int c0 = 0; c0 < N; c0 += 32) {
      float v[32];
      umma::ld32(tmem + (static_cast<uint32_t>(32 * warp) << 16) + c0, v);
      umma::wait_ld();
#pragma unroll
      for (int j = 0; j < 32; ++j) D[(32 * warp + lane) * N + c0 + j] = v[j];
    }
  }
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  if (warp == 0) umma::dealloc(tmem, 2 * kMaxN);
}

}  // namespace

extern "C" int umma_selftest(const void* A0, const void* B0, const void* A1, const void* B1,
                             float* D, int N, int bf16, int a_tmem, int* err, void* stream) {
  if (N < 16 || N > kMaxN || N % 32 != 0) return 1;
  const int smem = kM * kK * 2 + kMaxN * kK * 2 + 16;
  if (cudaFuncSetAttribute(umma_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
      cudaSuccess)
    return 2;
  umma_gemm_kernel<<<1, 128, smem, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t*>(A0), static_cast<const uint16_t*>(B0),
      static_cast<const uint16_t*>(A1), static_cast<const uint16_t*>(B1), D, N, bf16, a_tmem, err);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}
