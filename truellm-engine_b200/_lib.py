"""ctypes binding of libtruellm_kivi.so (the C ABI in include/truellm_kivi.h).

The library is built in-tree by build.py.  There is no fallback: if the
library is missing or fails to load, every entry point raises.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libtruellm_kivi.so"

TKV_OK = 0
TKV_INVALID_ARGUMENT = 1
TKV_NOT_IMPLEMENTED = 3
TKV_OUT_OF_MEMORY = 4
TKV_BACKEND_ERROR = 5

TKV_F32, TKV_F16, TKV_BF16 = 0, 1, 2
TKV_PAGE_SIZE = 16
TKV_SPLIT_TOKENS = 512

TKV_ERR_BAD_PAGE = 0x1
TKV_ERR_BAD_SLOT = 0x2
TKV_ERR_BAD_LENGTH = 0x4
TKV_ERR_TIMEOUT = 0x8

TKV_NOALLOC_SCRATCH_BYTES = 16 << 20
TKV_MAX_PEERS = 8
TKV_IPC_HANDLE_BYTES = 64


class TkvFormat(C.Structure):
    _fields_ = [
        ("head_dim", C.c_int32), ("group_size", C.c_int32), ("residual", C.c_int32),
        ("bits", C.c_int32), ("n_kv_heads", C.c_int32), ("ring_cap", C.c_int32),
        ("n_vgroups", C.c_int32), ("k_codes_off", C.c_int32), ("v_codes_off", C.c_int32),
        ("v_meta_off", C.c_int32), ("k_meta_off", C.c_int32), ("k_meta_slice", C.c_int32),
        ("page_bytes", C.c_int64),
    ]


class TkvCache(C.Structure):
    _fields_ = [
        ("pool", C.c_void_p), ("ring", C.c_void_p), ("num_pages", C.c_int32),
        ("max_seqs", C.c_int32), ("fmt", TkvFormat),
    ]


class TkvExchange(C.Structure):
    _fields_ = [("world", C.c_int32), ("rank", C.c_int32),
                ("buffers", C.c_void_p * TKV_MAX_PEERS)]


class TruellmKernelManifest(C.Structure):
    _fields_ = [
        ("abi_version", C.c_uint32), ("name", C.c_char_p), ("version", C.c_char_p),
        ("category", C.c_int), ("min_sm_major", C.c_uint32), ("min_sm_minor", C.c_uint32),
        ("initialize", C.c_void_p), ("shutdown", C.c_void_p), ("kernel_state", C.c_void_p),
    ]


class TkvAllocatorStats(C.Structure):
    _fields_ = [
        ("pages_total", C.c_int32), ("pages_used", C.c_int32), ("pages_free", C.c_int32),
        ("pages_shared", C.c_int32), ("rows_total", C.c_int32), ("rows_free", C.c_int32),
        ("sequences", C.c_int32), ("evicted", C.c_int32), ("utilization_pct", C.c_float),
    ]


_vp, _i32, _i64, _sz, _f32 = C.c_void_p, C.c_int, C.c_int64, C.c_size_t, C.c_float
_ip = C.POINTER(C.c_int)
_u64 = C.c_uint64

# name -> (restype, argtypes); every symbol the header declares.
SIGNATURES = {
    "tkv_abi_version": (_i32, []),
    "tkv_status_string": (C.c_char_p, [_i32]),
    "tkv_format_init": (_i32, [C.POINTER(TkvFormat), _i32, _i32, _i32, _i32, _i32]),
    "tkv_ring_bytes": (_i64, [C.POINTER(TkvFormat), _i32]),
    "tkv_quantized_len": (_i32, [C.POINTER(TkvFormat), _i32]),
    "tkv_kivi_compressed_bytes": (_sz, [_i32, _i32, _i32]),
    "tkv_kivi_params_supported": (_i32, [_i32, _i32, _i32]),
    "tkv_kivi_compress": (_i32, [_vp, _vp, _i32, _i32, _i32, _i32, _vp]),
    "tkv_kivi_decompress": (_i32, [_vp, _vp, _i32, _i32, _i32, _i32, _vp]),
    "tkv_kivi_roundtrip_inplace": (_i32, [_vp, _i32, _i32, _i32, _i32, _vp]),
    "tkv_paged_append": (_i32, [C.POINTER(TkvCache), _vp, _vp, _i32, _vp, _vp, _vp, _i32, _vp,
                                _i32, _i32, _i32, _vp, _vp]),
    "tkv_decode_num_splits": (_i32, [_i32]),
    "tkv_decode_workspace_bytes": (_sz, [_i32, _i32, _i32, _i32]),
    "tkv_paged_decode": (_i32, [C.POINTER(TkvCache), _vp, _i32, _vp, _i32, _vp, _i32, _vp, _vp,
                                _i32, _i32, _f32, _i32, _vp, _sz, _vp, _vp]),
    "tkv_paged_decode_noalloc": (_i32, [C.POINTER(TkvCache), _vp, _i32, _vp, _i32, _vp, _i32,
                                        _vp, _vp, _i32, _i32, _f32, _i32, _vp, _vp]),
    "tkv_paged_decode_partials": (_i32, [C.POINTER(TkvCache), _vp, _i32, _vp, _i32, _vp, _vp,
                                         _i32, _i32, _f32, _i32, _i32, _i32, _vp, _vp, _vp,
                                         _vp, _vp]),
    "tkv_decode_launches": (_i32, [_i32, _i32, _i32, _i32]),
    "tkv_decode_range_workspace_bytes": (_sz, [_i32, _i32, _i32, _i32, _i32]),
    "tkv_paged_decode_range": (_i32, [C.POINTER(TkvCache), _vp, _i32, _vp, _i32, _vp, _vp,
                                      _i32, _i32, _f32, _i32, _i32, _i32, _vp, _vp, _vp, _sz,
                                      _vp, _vp]),
    "tkv_merge_partials": (_i32, [_vp, _vp, _i32, _i32, _i32, _i32, _vp, _i32, _vp]),
    "tkv_exchange_buffer_bytes": (_sz, [_i32, _i32, _i32, _i32]),
    "tkv_device_alloc": (_i32, [_sz, C.POINTER(_vp)]),
    "tkv_device_free": (_i32, [_vp]),
    "tkv_ipc_get_handle": (_i32, [_vp, _vp]),
    "tkv_ipc_open_handle": (_i32, [_vp, C.POINTER(_vp)]),
    "tkv_ipc_close_handle": (_i32, [_vp]),
    "tkv_exchange_decode_range": (_i32, [C.POINTER(TkvCache), _vp, _i32, _vp, _i32, _vp, _vp,
                                         _i32, _i32, _f32, _i32, _i32, _i32,
                                         C.POINTER(TkvExchange), _vp, _sz, _vp, _vp]),
    "tkv_exchange_merge": (_i32, [C.POINTER(TkvExchange), _i32, _i32, _i32, _vp, _i32, _vp,
                                  _vp]),
    "tkv_paged_prefill": (_i32, [C.POINTER(TkvCache), _vp, _i32, _vp, _i32, _vp, _vp, _i32, _vp,
                                 _vp, _i32, _i32, _i32, _i32, _f32, _vp, _vp]),
    "tkv_allocator_create": (_i32, [C.POINTER(TkvFormat), _i32, _i32, _i32, C.POINTER(_vp)]),
    "tkv_allocator_destroy": (None, [_vp]),
    "tkv_allocator_pages_for": (_i32, [_vp, _i32]),
    "tkv_allocator_add_sequence": (_i32, [_vp, _u64, _i32, _ip]),
    "tkv_allocator_extend": (_i32, [_vp, _u64, _i32, _ip]),
    "tkv_allocator_free_sequence": (_i32, [_vp, _u64]),
    "tkv_allocator_fork": (_i32, [_vp, _u64, _u64, _ip, _ip]),
    "tkv_allocator_tables": (_i32, [_vp, _vp, _i32, _vp, _vp, _vp]),
    "tkv_allocator_sequence": (_i32, [_vp, _u64, _ip, _ip, _ip, _ip]),
    "tkv_allocator_stats": (_i32, [_vp, C.POINTER(TkvAllocatorStats)]),
    "tkv_allocator_evict": (_i32, [_vp, _u64, _vp, _ip, _ip]),
    "tkv_allocator_reload": (_i32, [_vp, _u64, _vp, _ip, _ip]),
    "tkv_copy_pages": (_i32, [C.POINTER(TkvCache), _vp, _i32, _vp, _vp]),
    "tkv_swap_pages": (_i32, [C.POINTER(TkvCache), _vp, _i64, _vp, _i32, _i32, _vp, _vp]),
    "tkv_copy_ring_rows": (_i32, [C.POINTER(TkvCache), _vp, _i32, _vp, _vp]),
    "tkv_swap_ring_rows": (_i32, [C.POINTER(TkvCache), _vp, _i64, _vp, _i32, _i32, _vp, _vp]),
    "truellm_kernel_init": (C.POINTER(TruellmKernelManifest), []),
    "tkv_cache_kernel_manifest": (C.POINTER(TruellmKernelManifest), []),
}

_LIB = None


class TkvError(RuntimeError):
    def __init__(self, fn: str, status: int):
        super().__init__(f"{fn} failed: status {status} ({status_string(status)})")
        self.status = status


def lib() -> C.CDLL:
    """Load libtruellm_kivi.so (raises if it was not built)."""
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python {LIB_PATH.parent / 'build.py'}` "
                "(the KIVI path has no CPU fallback)")
        h = C.CDLL(os.fspath(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(h, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = h
    return _LIB


def status_string(status: int) -> str:
    return lib().tkv_status_string(int(status)).decode()


def check(fn: str, status: int) -> None:
    if status != TKV_OK:
        raise TkvError(fn, status)
