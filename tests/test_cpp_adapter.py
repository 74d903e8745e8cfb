"""The C++ drop-in adapter (include/truellm_kivi.hpp) compiles with g++ against
the C ABI and keeps the reference's host-side behaviour, checked without a
GPU: KvCompressionPass maps the config like kv_compression_pass.cpp:29-67 and
disables itself on unsupported parameters, the reference-format calls are
silent no-ops on unsupported parameters (kivi_cache.cu:219-220), a bad paged
call throws instead of returning an unchecked status, and the tensor-view
(TrueBuffer-shaped) overloads reject views of the wrong rank or type.
"""
import os
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "truellm-engine_b200"
CUDA_INC = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda")) / "include"

PROGRAM = r"""
#include <cstdio>
#include <stdexcept>
#include "truellm_kivi.hpp"

namespace kb = truellm::kivi_b200;

// stand-ins with the field names of truellm::CompressionConfig (config_schema.h:121-159)
struct KiviConfig { bool enabled = false; int bits = 8; int residual_length = 128; };
struct CompressionConfig { bool enabled = false; KiviConfig kv_kivi; };
struct CudaAllocator {};
// a view with the fields of truellm::TrueBuffer (include/truellm/types.h:69-77)
enum class DataType : uint8_t { F32 = 0, F16 = 1, BF16 = 2, I32 = 3 };
struct TrueBuffer {
  void* data; std::size_t size_bytes; DataType dtype; int32_t device_id; int32_t ndim;
  int64_t shape[4]; int64_t stride[4];
};

#define CHECK(x) do { if (!(x)) { std::printf("FAIL %s:%d %s\n", __FILE__, __LINE__, #x); return 1; } } while (0)

int main() {
  CompressionConfig cfg;
  cfg.kv_kivi.enabled = true;
  cfg.kv_kivi.bits = 4;
  cfg.kv_kivi.residual_length = 32;
  kb::KvCompressionPass pass(cfg, 32, 8, 128, 16);
  CHECK(pass.enabled());
  CHECK(pass.n_outliers() == 32 && pass.group_size() == 16);   // bits 4 -> group 16
  CudaAllocator alloc;
  pass.init(&alloc, nullptr);
  pass.run(0, 0, nullptr, nullptr, nullptr);                     // seq_len 0: no-op

  cfg.kv_kivi.bits = 8;
  kb::KvCompressionPass pass8(cfg, 32, 8, 128, 16);
  CHECK(pass8.group_size() == 8);
  kb::KvCompressionPass wide(cfg, 32, 8, 256, 16);                // head_dim > 128: disabled
  CHECK(!wide.enabled());
  wide.run(0, 4, nullptr, nullptr, nullptr);                      // disabled: no-op
  cfg.kv_kivi.enabled = false;
  CHECK(!kb::KvCompressionPass(cfg, 32, 8, 128, 16).enabled());

  CHECK(kb::kivi_params_supported(64, 32, 16));
  CHECK(!kb::kivi_params_supported(64, 0, 0));
  CHECK(kb::kivi_compressed_bytes(128, 0, 128) == 68);
  kb::kivi_compress(nullptr, nullptr, 0, 64, 0, 32, nullptr);     // n_vecs 0: no-op
  kb::kivi_compress(nullptr, nullptr, 10, 64, 0, 0, nullptr);     // unsupported: no-op
  kb::kivi_decompress(nullptr, nullptr, 10, 300, 0, 32, nullptr); // unsupported: no-op

  tkv_format_t f = kb::PagedKiviCache::format(128, 128, 128, 4, 8);
  CHECK(f.page_bytes == 2176);
  kb::PagedKiviCache cache(nullptr, nullptr, 16, 4, 128, 128, 128, 4, 8);
  CHECK(cache.pool_bytes() == 2176LL * 8 * 16);
  bool threw = false;
  try {  // null pool: rejected before any launch
    cache.decode(nullptr, TKV_BF16, nullptr, TKV_BF16, nullptr, 1, nullptr, nullptr, 1, 32,
                 0.1f, 16, nullptr, 0, nullptr, nullptr);
  } catch (const std::invalid_argument&) {
    threw = true;
  }
  CHECK(threw);
  threw = false;
  try {  // prefill with a null pool: rejected before any launch
    cache.prefill(nullptr, TKV_BF16, nullptr, TKV_BF16, nullptr, nullptr, 1, nullptr, nullptr, 1,
                  32, 4, 4, 0.1f, nullptr, nullptr);
  } catch (const std::invalid_argument&) {
    threw = true;
  }
  CHECK(threw);
  // tensor-view overloads (the reference's TrueBuffer call sites): a view of
  // the wrong rank or element type is rejected before any launch
  {
    int32_t idx[8] = {0};
    uint16_t qh[8] = {0};
    TrueBuffer q{qh, 16, DataType::F16, 0, 3, {1, 32, 128, 1}, {0, 0, 0, 0}};
    TrueBuffer out = q;
    TrueBuffer bt2{idx, 32, DataType::I32, 0, 2, {1, 8, 1, 1}, {0, 0, 0, 0}};
    TrueBuffer lens1{idx, 4, DataType::I32, 0, 1, {1, 1, 1, 1}, {0, 0, 0, 0}};
    TrueBuffer bad_bt = bt2;
    bad_bt.dtype = DataType::F16;
    threw = false;
    try {
      cache.decode(out, q, bad_bt, lens1, 0.1f, 16, nullptr, 0, nullptr, nullptr);
    } catch (const std::invalid_argument&) {
      threw = true;
    }
    CHECK(threw);
    TrueBuffer flat_q = q;
    flat_q.ndim = 2;
    threw = false;
    try {
      cache.decode(out, flat_q, bt2, lens1, 0.1f, 16, nullptr, 0, nullptr, nullptr);
    } catch (const std::invalid_argument&) {
      threw = true;
    }
    CHECK(threw);
    threw = false;
    try {  // well-formed views, null pool: rejected by the C ABI before any launch
      cache.decode(out, q, bt2, lens1, 0.1f, 16, nullptr, 0, nullptr, nullptr);
    } catch (const std::invalid_argument&) {
      threw = true;
    }
    CHECK(threw);
    TrueBuffer kv{qh, 16, DataType::F16, 0, 3, {1, 8, 128, 1}, {0, 0, 0, 0}};
    TrueBuffer vv = kv;
    vv.dtype = DataType::BF16;  // value of another type than key
    TrueBuffer cu{idx, 8, DataType::I32, 0, 1, {2, 1, 1, 1}, {0, 0, 0, 0}};
    threw = false;
    try {
      cache.append(kv, vv, cu, lens1, bt2, 1, nullptr, nullptr);
    } catch (const std::invalid_argument&) {
      threw = true;
    }
    CHECK(threw);
  }
  threw = false;
  try {
    kb::PagedKiviCache::format(96, 128, 128, 4, 8);
  } catch (const std::exception&) {
    threw = true;
  }
  CHECK(threw);
  // page allocator: reference bool / -1 returns, shared pages, -1 padded tables
  kb::KiviPageAllocator pa(f, 32, 2, 16);
  int32_t row = -1;
  CHECK(pa.allocate_sequence(1, 256, &row) && row == 0);        // 8 pages
  CHECK(!pa.allocate_sequence(1, 0));                           // duplicate
  CHECK(pa.extend_sequence(1, 384) == 8 && pa.extend_sequence(7, 384) == -1);
  int32_t sr = -1, dr = -1;
  CHECK(pa.copy_sequence(1, 2, &sr, &dr) && sr == 0 && dr == 1);
  CHECK(!pa.copy_sequence(1, 3));                               // out of ring rows
  CHECK(pa.stats().pages_shared == 16 && pa.num_free_blocks() == 16);
  uint64_t ids[2] = {1, 2};
  int32_t bt[32], lens[2], rows[2];
  pa.block_tables(ids, 2, bt, lens, rows);
  CHECK(bt[0] == 0 && bt[15] == 15 && bt[16] == 0 && lens[1] == 384 && rows[1] == 1);
  int32_t pages[16];
  int np = 0;
  CHECK(pa.evict_sequence(1, pages, &np, &row) && np == 16 && row == 0);
  CHECK(pa.stats().pages_used == 16 && pa.stats().evicted == 1);
  pa.free_sequence(2);
  CHECK(pa.num_free_blocks() == 32);
  CHECK(pa.reload_sequence(1, pages, &np, &row) && np == 16);
  threw = false;
  try {
    pa.block_tables(ids, 2, bt, lens, rows);                    // 2 is gone
  } catch (const std::invalid_argument&) {
    threw = true;
  }
  CHECK(threw);
  std::printf("ok\n");
  return 0;
}
"""


@pytest.mark.skipif(shutil.which("g++") is None, reason="g++ not installed")
def test_cpp_adapter_compiles_and_keeps_reference_behaviour(tmp_path):
    lib = PKG / "libtruellm_kivi.so"
    assert lib.exists(), "build the library first (truellm-engine_b200/build.py)"
    src = tmp_path / "adapter_test.cpp"
    src.write_text(PROGRAM)
    exe = tmp_path / "adapter_test"
    cmd = ["g++", "-std=c++17", "-O1", "-Wall", "-Werror", f"-I{ROOT / 'include'}",
           f"-I{CUDA_INC}", str(src), f"-L{PKG}", "-ltruellm_kivi", f"-Wl,-rpath,{PKG}",
           "-o", str(exe)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    assert res.returncode == 0, res.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert run.returncode == 0 and run.stdout.strip() == "ok", run.stdout + run.stderr
