"""truellm-engine_b200 -- B200 (sm_100a) KIVI quantized-KV attention path.

Host-side mirror of truellm-engine's quantized-KV interfaces over the C ABI in
include/truellm_kivi.h (library: libtruellm_kivi.so, built by build.py):

  ops          kivi_compress / kivi_decompress / kivi_params_supported /
               kivi_compressed_bytes (kivi_cache.cuh), paged_append (the KIVI
               reshape_and_cache), paged_decode (the paged_attention_v1/v2 slot),
               split partials + merge, chunked prefill, page / ring-row moves
  allocator    PageAllocator / KiviCacheAllocator: the CudaAllocator page pool,
               block tables, fork, evict / reload
  config       KvCompressionPass mapping + config switches (kv_kivi, kv_cache
               type_k/v) read from the reference's TOML files
  sharding     sequence / kv-head / token sharding over one process per GPU
  workloads    seeded synthetic inputs for the benchmark configurations
  build        compiles the sm_100a library in-tree

Import with importlib.import_module("truellm-engine_b200").
"""
from . import _lib  # noqa: F401
from .build import build  # noqa: F401

__all__ = ["build"]
