"""The C ABI without a GPU: libtruellm_kivi.so loads, exports every function
include/truellm_kivi.h declares (and the ctypes stub binds exactly those), and
the host-only entry points and argument checks answer before any CUDA call.
"""
import ctypes as C
import importlib
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
L = importlib.import_module("truellm-engine_b200._lib")


def declared():
    text = (ROOT / "include" / "truellm_kivi.h").read_text()
    text = re.sub(r"/\*.*?\*/", " ", text, flags=re.S)
    return set(re.findall(r"TKV_API\s+[\w\s\*]+?\b(\w+)\s*\(", text))


def test_every_declared_symbol_is_exported():
    names = declared()
    assert len(names) >= 20 and "tkv_paged_decode" in names and "truellm_kernel_init" in names
    lib = C.CDLL(str(L.LIB_PATH))
    missing = [n for n in sorted(names) if not hasattr(lib, n)]
    assert not missing, missing


def test_ctypes_stub_binds_exactly_the_header():
    assert set(L.SIGNATURES) == declared()


def test_host_entry_points():
    lib = L.lib()
    assert lib.tkv_abi_version() >= 1
    assert L.status_string(L.TKV_INVALID_ARGUMENT)
    f = L.TkvFormat()
    assert lib.tkv_format_init(C.byref(f), 128, 128, 128, 4, 8) == L.TKV_OK
    assert (f.page_bytes, f.ring_cap, f.n_vgroups) == (2176, 256, 1)
    assert lib.tkv_format_init(C.byref(f), 96, 128, 128, 4, 8) != L.TKV_OK  # D not 64/128
    assert lib.tkv_quantized_len(C.byref(f), 4587) == 128 * ((4587 - 128) // 128)
    assert lib.tkv_decode_num_splits(8192) == 17
    # partial slots for every (sequence, kv head) pair plus one per resident
    # warp (148 SMs x 12 at GQA 4), and small enough for the no-alloc scratch
    ws = lib.tkv_decode_workspace_bytes(64, 32, 128, 8192)
    assert (64 * 32 + 148 * 12 * 4) * 130 * 4 < ws <= L.TKV_NOALLOC_SCRATCH_BYTES
    assert lib.tkv_kivi_compressed_bytes(128, 0, 128) == 68       # reference mapping
    assert lib.tkv_kivi_params_supported(64, 32, 16) == 1
    assert lib.tkv_kivi_params_supported(64, 0, 0) == 0           # group_size must be > 0
    assert lib.tkv_kivi_params_supported(64, 65, 16) == 0         # more outliers than channels


def test_decode_launch_count_rule():
    """tkv_decode_launches: 0 for invalid sizes (the q heads must split evenly
    over the kv heads); a second, slot-parallel merge launch for pairs that
    each span many warps (one sequence, one kv head), one launch when every
    pair spans few (8192 pairs)."""
    lib = L.lib()
    assert lib.tkv_decode_launches(4, 32, 5, 100) == 0       # 32 q heads over 5 kv heads
    assert lib.tkv_decode_launches(0, 32, 8, 100) == 0
    assert lib.tkv_decode_launches(4, 32, 0, 100) == 0
    assert lib.tkv_decode_launches(4, 32, 8, -1) == 0
    assert lib.tkv_decode_launches(1, 4, 1, 131072) == 2
    assert lib.tkv_decode_launches(1024, 32, 8, 8192) == 1


def test_manifests():
    m = L.lib().truellm_kernel_init().contents
    assert m.abi_version == 1 and m.category == 0 and (m.min_sm_major, m.min_sm_minor) == (10, 0)
    assert m.name
    c = L.lib().tkv_cache_kernel_manifest().contents
    assert c.abi_version == 1 and c.category == 4


def test_bad_arguments_are_rejected_before_any_launch():
    lib = L.lib()
    # null cache / sizes: TKV_INVALID_ARGUMENT, nothing touches the GPU
    assert lib.tkv_paged_decode(None, None, L.TKV_BF16, None, L.TKV_BF16, None, 1, None, None,
                                1, 8, 0.1, 16, None, 0, None, None) == L.TKV_INVALID_ARGUMENT
    assert lib.tkv_merge_partials(None, None, 1, 1, 1, 128, None, L.TKV_F32,
                                  None) == L.TKV_INVALID_ARGUMENT
    c = L.TkvCache()
    assert lib.tkv_format_init(C.byref(c.fmt), 128, 128, 128, 4, 8) == L.TKV_OK
    c.num_pages, c.max_seqs = 16, 4
    # beyond the static scratch of the no-allocation entry point
    assert lib.tkv_paged_decode_noalloc(C.byref(c), None, L.TKV_BF16, None, L.TKV_BF16, None, 1,
                                        None, None, 4096, 32, 0.1, 131072, None,
                                        None) == L.TKV_OUT_OF_MEMORY
