// engine_loop.cpp -- drives libtruellm_kivi.so through the C++ adapter
// (include/truellm_kivi.hpp) in the order truellm-engine's CUDA backend calls
// its KV-cache kernels, for the GPU test tests/test_gpu_cpp_engine.py:
//
//   * KiviPageAllocator holds the sequences (allocate_sequence /
//     extend_sequence, the CudaAllocator slots of cuda_allocator.cpp:129-171)
//     and fills the block tables on the host; each step uploads them once
//     with cudaMemcpyAsync from pinned memory (cuda_engine.cpp:978-986), so
//     the kernels read device-resident tables;
//   * prompt: per layer, PagedKiviCache::append (the reshape_and_cache slot,
//     cuda_engine.cpp:1130-1136) then PagedKiviCache::prefill (the prompt's
//     attention, which the reference runs token by token at :842-860);
//   * decode steps: per layer, append of the new token then
//     PagedKiviCache::decode (the paged_attention_v1/v2 slot, :1137-1159);
//   * KvCompressionPass::run on a separate K/V buffer (run_kv_compression_pass,
//     :732-746).
// Everything is queued on one stream; the host waits once, at the end, and
// writes the results next to the inputs.
//
// usage: engine_loop <dir>   (reads <dir>/job.i32 and the *.f16 inputs)
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <initializer_list>
#include <stdexcept>
#include <string>
#include <vector>

#include <cuda_runtime.h>  // typed cudaMalloc overloads

#include "truellm_kivi.hpp"

namespace kb = truellm::kivi_b200;

namespace {

std::string g_dir;

void cuda_ok(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

template <class T>
std::vector<T> read_file(const char* name, size_t count) {
  std::vector<T> v(count);
  const std::string path = g_dir + "/" + name;
  FILE* f = std::fopen(path.c_str(), "rb");
  if (!f || std::fread(v.data(), sizeof(T), count, f) != count)
    throw std::runtime_error("cannot read " + path);
  std::fclose(f);
  return v;
}

void write_file(const char* name, const void* data, size_t bytes) {
  const std::string path = g_dir + "/" + name;
  FILE* f = std::fopen(path.c_str(), "wb");
  if (!f || std::fwrite(data, 1, bytes, f) != bytes) throw std::runtime_error("cannot write " + path);
  std::fclose(f);
}

template <class T>
T* device_copy(const std::vector<T>& h) {
  T* d = nullptr;
  cuda_ok(cudaMalloc(&d, h.size() * sizeof(T)), "cudaMalloc");
  cuda_ok(cudaMemcpy(d, h.data(), h.size() * sizeof(T), cudaMemcpyHostToDevice), "upload");
  return d;
}

// a view with the fields of truellm::TrueBuffer (include/truellm/types.h:69-77)
// and truellm::DataType's values, for the adapter's tensor-view overloads
enum class DataType : uint8_t { F32 = 0, F16 = 1, BF16 = 2, I32 = 3 };
struct TrueBuffer {
  void* data;
  std::size_t size_bytes;
  DataType dtype;
  int32_t device_id;
  int32_t ndim;
  int64_t shape[4];
  int64_t stride[4];
};
TrueBuffer view(const void* p, DataType t, std::size_t elem, std::initializer_list<int64_t> shape) {
  TrueBuffer b{const_cast<void*>(p), 0, t, 0, static_cast<int32_t>(shape.size()), {1, 1, 1, 1},
               {0, 0, 0, 0}};
  std::size_t n = 1;
  int i = 0;
  for (int64_t d : shape) {
    b.shape[i++] = d;
    n *= static_cast<std::size_t>(d);
  }
  int64_t st = 1;
  for (int k = b.ndim - 1; k >= 0; --k) {
    b.stride[k] = st;
    st *= b.shape[k];
  }
  b.size_bytes = n * elem;
  return b;
}

// stand-ins with the field names of truellm::CompressionConfig (config_schema.h:121-159)
struct KiviConfig { bool enabled = true; int bits = 4; int residual_length = 32; };
struct CompressionConfig { bool enabled = true; KiviConfig kv_kivi; };

}  // namespace

int main(int argc, char** argv) {
  if (argc != 2) {
    std::fprintf(stderr, "usage: %s <dir>\n", argv[0]);
    return 2;
  }
  g_dir = argv[1];
  try {
    // job: D G R bits Hkv Hq B T chunk num_pages max_blocks n_layers rt_vecs rt_outliers, lens[B]
    const std::vector<int32_t> hdr = read_file<int32_t>("job.i32", 14);
    const int D = hdr[0], G = hdr[1], R = hdr[2], bits = hdr[3], Hkv = hdr[4], Hq = hdr[5];
    const int B = hdr[6], T = hdr[7], chunk = hdr[8], num_pages = hdr[9], max_blocks = hdr[10];
    const int n_layers = hdr[11], rt_vecs = hdr[12], rt_outliers = hdr[13];
    const std::vector<int32_t> job = read_file<int32_t>("job.i32", 14 + B);
    std::vector<int32_t> lens(job.begin() + 14, job.end());
    int total = 0, max_len = 0;
    for (int b = 0; b < B; ++b) total += lens[b], max_len = lens[b] > max_len ? lens[b] : max_len;
    const size_t tok = static_cast<size_t>(Hkv) * D;  // halves per token
    const size_t row = static_cast<size_t>(Hq) * D;   // halves per query row
    const float scale = 1.0f / std::sqrt(static_cast<float>(D));

    // inputs (fp16 bits)
    const auto kp = read_file<uint16_t>("kp.f16", n_layers * total * tok);
    const auto vp = read_file<uint16_t>("vp.f16", n_layers * total * tok);
    const auto qp = read_file<uint16_t>("qp.f16", n_layers * B * chunk * row);
    const auto kd = read_file<uint16_t>("kd.f16", n_layers * T * B * tok);
    const auto vd = read_file<uint16_t>("vd.f16", n_layers * T * B * tok);
    const auto qd = read_file<uint16_t>("qd.f16", n_layers * T * B * row);
    const auto rt = read_file<uint16_t>("rt.f16", 2 * rt_vecs * D);

    cudaStream_t s;
    cuda_ok(cudaStreamCreate(&s), "stream");

    // ---- the page allocator: sequences 1..B with their prompts ----
    const tkv_format_t fmt = kb::PagedKiviCache::format(D, G, R, bits, Hkv);
    kb::KiviPageAllocator alloc(fmt, num_pages, B, max_blocks);
    std::vector<uint64_t> ids(B);
    for (int b = 0; b < B; ++b) {
      ids[b] = 1 + b;
      if (!alloc.allocate_sequence(ids[b], 0)) throw std::runtime_error("allocate_sequence");
      if (alloc.extend_sequence(ids[b], lens[b]) < 0) throw std::runtime_error("extend_sequence");
    }

    // ---- per-layer caches (caller-owned buffers) ----
    std::vector<void*> pools(n_layers), rings(n_layers);
    std::vector<kb::PagedKiviCache> caches;
    const size_t pool_bytes = static_cast<size_t>(fmt.page_bytes) * Hkv * num_pages;
    const size_t ring_bytes = static_cast<size_t>(tkv_ring_bytes(&fmt, B));
    for (int l = 0; l < n_layers; ++l) {
      cuda_ok(cudaMalloc(&pools[l], pool_bytes), "pool");
      cuda_ok(cudaMalloc(&rings[l], ring_bytes), "ring");
      cuda_ok(cudaMemset(pools[l], 0, pool_bytes), "pool zero");
      cuda_ok(cudaMemset(rings[l], 0, ring_bytes), "ring zero");
      caches.emplace_back(pools[l], rings[l], num_pages, B, D, G, R, bits, Hkv);
    }

    // ---- device buffers ----
    uint16_t* d_kp = device_copy(kp);
    uint16_t* d_vp = device_copy(vp);
    uint16_t* d_qp = device_copy(qp);
    uint16_t* d_kd = device_copy(kd);
    uint16_t* d_vd = device_copy(vd);
    uint16_t* d_qd = device_copy(qd);
    std::vector<int32_t> cu_prompt(B + 1, 0), cu_q(B + 1, 0), cu_one(B + 1, 0), zeros(B, 0);
    for (int b = 0; b < B; ++b) {
      cu_prompt[b + 1] = cu_prompt[b] + lens[b];
      cu_q[b + 1] = cu_q[b] + chunk;
      cu_one[b + 1] = b + 1;
    }
    int32_t* d_cu_prompt = device_copy(cu_prompt);
    int32_t* d_cu_q = device_copy(cu_q);
    int32_t* d_cu_one = device_copy(cu_one);
    int32_t* d_zeros = device_copy(zeros);
    int* d_err = device_copy(std::vector<int>(1, 0));
    float* d_out_prefill = nullptr;
    float* d_out_decode = nullptr;
    cuda_ok(cudaMalloc(&d_out_prefill, n_layers * B * chunk * row * sizeof(float)), "out");
    cuda_ok(cudaMalloc(&d_out_decode, n_layers * B * row * sizeof(float)), "out");
    const size_t ws_bytes = kb::PagedKiviCache::decode_workspace_bytes(B, Hq, D, max_len + T);
    void* d_ws = nullptr;
    cuda_ok(cudaMalloc(&d_ws, ws_bytes), "workspace");
    cuda_ok(cudaMemset(d_ws, 0, ws_bytes), "workspace zero");

    // block tables, lengths and ring rows: one pinned host set per upload
    // (the host never overwrites a set a pending copy still reads)
    const size_t tsz = static_cast<size_t>(B) * (max_blocks + 2);
    int32_t* h_tables = nullptr;
    cuda_ok(cudaMallocHost(&h_tables, (T + 1) * tsz * sizeof(int32_t)), "pinned tables");
    int32_t* d_tables = nullptr;  // [max_blocks * B][lens B][rows B]
    cuda_ok(cudaMalloc(&d_tables, tsz * sizeof(int32_t)), "tables");
    int32_t* d_lens_old = nullptr;
    cuda_ok(cudaMalloc(&d_lens_old, B * sizeof(int32_t)), "lens");
    auto upload_tables = [&](int set) {
      int32_t* h = h_tables + set * tsz;
      alloc.block_tables(ids.data(), B, h, h + static_cast<size_t>(B) * max_blocks,
                         h + static_cast<size_t>(B) * (max_blocks + 1));
      cuda_ok(cudaMemcpyAsync(d_tables, h, tsz * sizeof(int32_t), cudaMemcpyHostToDevice, s),
              "table upload");
    };
    int32_t* d_bt = d_tables;
    int32_t* d_lens = d_tables + static_cast<size_t>(B) * max_blocks;
    int32_t* d_rows = d_tables + static_cast<size_t>(B) * (max_blocks + 1);

    // ---- prompt ----
    upload_tables(0);
    for (int l = 0; l < n_layers; ++l) {
      caches[l].append(d_kp + l * total * tok, d_vp + l * total * tok, TKV_F16, d_cu_prompt,
                       d_zeros, d_bt, max_blocks, d_rows, B, total, max_len, d_err, s);
      caches[l].prefill(d_qp + l * B * chunk * row, TKV_F16, d_out_prefill + l * B * chunk * row,
                        TKV_F32, d_cu_q, d_bt, max_blocks, d_lens, d_rows, B, Hq, B * chunk,
                        chunk, scale, d_err, s);
    }
    // ---- decode steps ----
    for (int t = 0; t < T; ++t) {
      cuda_ok(cudaMemcpyAsync(d_lens_old, d_lens, B * sizeof(int32_t), cudaMemcpyDeviceToDevice,
                              s),
              "lens_old");
      for (int b = 0; b < B; ++b)
        if (alloc.extend_sequence(ids[b], lens[b] + t + 1) < 0)
          throw std::runtime_error("extend_sequence");
      upload_tables(t + 1);
      for (int l = 0; l < n_layers; ++l) {
        if (l == 0) {  // pointer forms
          caches[l].append(d_kd + (l * T + t) * B * tok, d_vd + (l * T + t) * B * tok, TKV_F16,
                           d_cu_one, d_lens_old, d_bt, max_blocks, d_rows, B, B, 1, d_err, s);
          caches[l].decode(d_qd + (l * T + t) * B * row, TKV_F16, d_out_decode + l * B * row,
                           TKV_F32, d_bt, max_blocks, d_lens, d_rows, B, Hq, scale, max_len + T,
                           d_ws, ws_bytes, d_err, s);
        } else {  // tensor views shaped like the reference's call sites
          const TrueBuffer k = view(d_kd + (l * T + t) * B * tok, DataType::F16, 2, {B, Hkv, D});
          const TrueBuffer v = view(d_vd + (l * T + t) * B * tok, DataType::F16, 2, {B, Hkv, D});
          const TrueBuffer cu = view(d_cu_one, DataType::I32, 4, {B + 1});
          const TrueBuffer lo = view(d_lens_old, DataType::I32, 4, {B});
          const TrueBuffer bt = view(d_bt, DataType::I32, 4, {B, max_blocks});
          const TrueBuffer ln = view(d_lens, DataType::I32, 4, {B});
          const TrueBuffer qv = view(d_qd + (l * T + t) * B * row, DataType::F16, 2, {B, Hq, D});
          TrueBuffer ov = view(d_out_decode + l * B * row, DataType::F32, 4, {B, Hq, D});
          caches[l].append(k, v, cu, lo, bt, 1, d_err, s, d_rows);
          caches[l].decode(ov, qv, bt, ln, scale, max_len + T, d_ws, ws_bytes, d_err, s, d_rows);
        }
      }
    }
    // ---- KvCompressionPass on a separate K/V buffer ----
    CompressionConfig cfg;
    cfg.kv_kivi.residual_length = rt_outliers;
    kb::KvCompressionPass pass(cfg, n_layers, 1, D, 16);
    if (!pass.enabled()) throw std::runtime_error("KvCompressionPass disabled");
    uint16_t* d_rt = device_copy(rt);
    pass.init(&alloc, s);
    pass.run(0, rt_vecs, d_rt, d_rt + static_cast<size_t>(rt_vecs) * D, s);

    cuda_ok(cudaStreamSynchronize(s), "synchronize");

    // ---- results ----
    int err = 0;
    cuda_ok(cudaMemcpy(&err, d_err, sizeof(int), cudaMemcpyDeviceToHost), "err");
    write_file("err.i32", &err, sizeof(err));
    std::vector<int32_t> tables(tsz);
    cuda_ok(cudaMemcpy(tables.data(), d_tables, tsz * sizeof(int32_t), cudaMemcpyDeviceToHost),
            "tables");
    write_file("tables.i32", tables.data(), tsz * sizeof(int32_t));
    for (int l = 0; l < n_layers; ++l) {
      std::vector<uint8_t> pool(caches[l].pool_bytes());
      cuda_ok(cudaMemcpy(pool.data(), pools[l], pool.size(), cudaMemcpyDeviceToHost), "pool");
      write_file(("pool" + std::to_string(l) + ".u8").c_str(), pool.data(), pool.size());
    }
    std::vector<float> op(n_layers * B * chunk * row), od(n_layers * B * row);
    cuda_ok(cudaMemcpy(op.data(), d_out_prefill, op.size() * 4, cudaMemcpyDeviceToHost), "out");
    cuda_ok(cudaMemcpy(od.data(), d_out_decode, od.size() * 4, cudaMemcpyDeviceToHost), "out");
    write_file("out_prefill.f32", op.data(), op.size() * 4);
    write_file("out_decode.f32", od.data(), od.size() * 4);
    std::vector<uint16_t> rt_out(rt.size());
    cuda_ok(cudaMemcpy(rt_out.data(), d_rt, rt_out.size() * 2, cudaMemcpyDeviceToHost), "rt");
    write_file("rt_out.f16", rt_out.data(), rt_out.size() * 2);
    std::printf("ok\n");
  } catch (const std::exception& e) {
    std::fprintf(stderr, "engine_loop: %s\n", e.what());
    return 1;
  }
  return 0;
}
