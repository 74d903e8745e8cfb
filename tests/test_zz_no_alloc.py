"""tkv_paged_decode_noalloc: the decode entry point for callers that cannot
allocate device memory (a kernel plugin that only receives the engine's
tensors, a host whose allocator owns all device memory, a decode loop that
must not call cudaMalloc).  It takes its workspace from a static device array
instead of a caller buffer; its results must match tkv_paged_decode, on two
calls in a row (the second reuses the array the first one left behind).

This file is collected last on purpose, so a run that stops at the first
failure has already run every other test; it also passes on its own in a
fresh process.
"""
import ctypes as C
import importlib
import math

import numpy as np
import pytest
import torch

from kivi_helpers import Twin, bits_to_torch, i32

pytestmark = pytest.mark.gpu


def _cache(ops, O, wl, cuda, lengths, seed):
    rng = np.random.default_rng(seed)
    lengths = np.asarray(lengths, np.int32)
    num_pages = int(sum((int(L) + 15) // 16 for L in lengths)) + 5
    bt = wl.random_block_tables(lengths, num_pages, rng)
    k, v = wl.kv_tokens(rng, int(lengths.sum()), 8, 128, np.array([2, 9]), 8.0)
    tw = Twin(ops, O, 128, 128, 128, 4, 8, num_pages, len(lengths), cuda)
    cu = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)
    tw.append(wl.to_bits(k, "bf16"), wl.to_bits(v, "bf16"), "bf16", cu,
              np.zeros(len(lengths), np.int32), bt)
    q = bits_to_torch(wl.f32_to_bf16_bits(rng.standard_normal((len(lengths), 32, 128))),
                      "bf16", cuda)
    return tw, bt, lengths, q


def test_noalloc_decode_matches_workspace_decode(ops, O, wl, cuda):
    L = importlib.import_module("truellm-engine_b200._lib")
    lib = L.lib()
    tw, bt, lengths, q = _cache(ops, O, wl, cuda, [3000, 1, 700, 129, 2048], seed=31)
    B, Hq, D = q.shape
    max_ctx = int(lengths.max())
    scale = 1.0 / math.sqrt(D)
    bt_d, lens_d = i32(bt, cuda), i32(lengths, cuda)
    want = ops.paged_decode(tw.gpu, q, bt_d, lens_d, max_ctx, scale=scale,
                            out_dtype=torch.float32)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    c = tw.gpu.c_struct()
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    for _ in range(2):
        out = torch.full((B, Hq, D), float("nan"), dtype=torch.float32, device=cuda)
        st = lib.tkv_paged_decode_noalloc(
            C.byref(c), C.c_void_p(q.data_ptr()), L.TKV_BF16, C.c_void_p(out.data_ptr()),
            L.TKV_F32, C.c_void_p(bt_d.data_ptr()), int(bt.shape[1]),
            C.c_void_p(lens_d.data_ptr()), None, B, Hq, scale, max_ctx,
            C.c_void_p(err.data_ptr()), stream)
        assert st == L.TKV_OK, L.status_string(st)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        assert torch.allclose(out, want, atol=2e-3, rtol=2e-3)


def test_noalloc_rejects_work_beyond_its_scratch(ops, O, wl, cuda):
    L = importlib.import_module("truellm-engine_b200._lib")
    lib = L.lib()
    tw, bt, lengths, q = _cache(ops, O, wl, cuda, [600], seed=32)
    # a batch whose split-KV partials would not fit the static scratch
    B, Hq, D, max_ctx = 4096, 32, 128, 131072
    assert ops.decode_workspace_bytes(B, Hq, D, max_ctx) > L.TKV_NOALLOC_SCRATCH_BYTES
    c = tw.gpu.c_struct()
    st = lib.tkv_paged_decode_noalloc(C.byref(c), C.c_void_p(q.data_ptr()), L.TKV_BF16,
                                      C.c_void_p(q.data_ptr()), L.TKV_BF16, None, 1, None, None,
                                      B, Hq, 0.1, max_ctx, None, None)
    assert st == L.TKV_OUT_OF_MEMORY
