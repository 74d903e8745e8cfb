// TEST INFRASTRUCTURE ONLY.  extern "C" entry points over the reference's own
// host wrappers truellm::kivi_compress / kivi_decompress
// (src/inference/backends/cuda/compression/kivi_cache.cu:213-239), so a test can
// call the unmodified reference kernels through ctypes on a GPU box.
#include "kivi_cache.cuh"

extern "C" {
int ref_kivi_compress(const void* d_in, void* d_out, int n_vecs, int head_dim, int n_outliers,
                      int group_size, void* stream) {
  truellm::kivi_compress(static_cast<const __half*>(d_in), static_cast<uint8_t*>(d_out), n_vecs,
                         head_dim, n_outliers, group_size, static_cast<cudaStream_t>(stream));
  return static_cast<int>(cudaGetLastError());
}
int ref_kivi_decompress(const void* d_in, void* d_out, int n_vecs, int head_dim, int n_outliers,
                        int group_size, void* stream) {
  truellm::kivi_decompress(static_cast<const uint8_t*>(d_in), static_cast<__half*>(d_out), n_vecs,
                           head_dim, n_outliers, group_size, static_cast<cudaStream_t>(stream));
  return static_cast<int>(cudaGetLastError());
}
unsigned long ref_kivi_compressed_bytes(int head_dim, int n_outliers, int group_size) {
  return truellm::kivi_compressed_bytes(head_dim, n_outliers, group_size);
}
int ref_kivi_params_supported(int head_dim, int n_outliers, int group_size) {
  return truellm::kivi_params_supported(head_dim, n_outliers, group_size) ? 1 : 0;
}
}
