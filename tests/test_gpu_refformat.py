"""GPU parity of the reference-format KIVI kernels (tkv_kivi_compress /
tkv_kivi_decompress / tkv_kivi_roundtrip_inplace) against the CPU oracle and,
when `make -C oracle ref` built them, against the unmodified reference kernels
(src/inference/backends/cuda/compression/kivi_cache.cu) on the same inputs:
byte for byte against the -G build (the source semantics), and against the
default-optimised build up to the low byte of each fp16 step / zero, which
that build stores as sat_u8(value)."""
import ctypes as C
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

REF = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "libkivi_ref.so"
REF_O3 = REF.with_name("libkivi_ref_O3.so")

CASES = [(64, 32, 16), (128, 8, 16), (128, 8, 8), (128, 0, 128), (64, 0, 32), (96, 5, 16),
         (128, 64, 16), (64, 64, 16), (16, 3, 4), (128, 0, 2)]


def _inputs(D, n, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((n, D)).astype(np.float32)
    x[:, rng.choice(D, min(4, D), replace=False)] *= 12
    x[0] = 0.0
    if n > 3:
        x[1, ::3] = -0.0
        x[2] = 1.5
        x[3] = np.round(x[3])  # many ties
    return x.astype(np.float16).view(np.uint16)


def _t(bits, dev):
    return torch.from_numpy(bits.view(np.int16).copy()).to(dev)


@pytest.mark.parametrize("D,n_out,G", CASES)
def test_compress_decompress_match_oracle(O, ops, cuda, D, n_out, G):
    n = 203
    x = _inputs(D, n, D * 1000 + n_out * 10 + G)
    stride = ops.kivi_compressed_bytes(D, n_out, G)
    packed = torch.full((n * stride,), 0xCD, dtype=torch.uint8, device=cuda)
    ops.kivi_compress(_t(x, cuda), packed, n, D, n_out, G)
    got = packed.cpu().numpy().reshape(n, stride)
    want = O.kivi_compress(x, n_out, G, fill=0xCD)
    assert np.array_equal(got, want)  # slack bytes untouched on both sides
    out = torch.zeros(n * D, dtype=torch.int16, device=cuda)
    ops.kivi_decompress(packed, out, n, D, n_out, G)
    got_u = out.cpu().numpy().view(np.uint16).reshape(n, D)
    assert np.array_equal(got_u, O.kivi_decompress(want, D, n_out, G))
    # fused in-place round trip == decompress(compress(x))
    inplace = _t(x, cuda)
    ops.kivi_roundtrip_inplace(inplace, n, D, n_out, G)
    assert np.array_equal(inplace.cpu().numpy().view(np.uint16).reshape(n, D), got_u)


@pytest.mark.skipif(not REF.exists(), reason="reference kernels not built (make -C oracle ref)")
@pytest.mark.parametrize("D,n_out,G", CASES)
def test_compress_decompress_match_reference_kernels(ops, cuda, D, n_out, G):
    lib = C.CDLL(str(REF))
    n = 157
    x = _inputs(D, n, 7 + D + n_out + G)
    stride = ops.kivi_compressed_bytes(D, n_out, G)
    s = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    xin = _t(x, cuda)
    ref_packed = torch.full((n * stride,), 0x5A, dtype=torch.uint8, device=cuda)
    our_packed = torch.full((n * stride,), 0x5A, dtype=torch.uint8, device=cuda)
    assert lib.ref_kivi_compress(C.c_void_p(xin.data_ptr()), C.c_void_p(ref_packed.data_ptr()),
                                 n, D, n_out, G, s) == 0
    ops.kivi_compress(xin, our_packed, n, D, n_out, G)
    torch.cuda.synchronize()
    assert torch.equal(ref_packed, our_packed)
    ref_out = torch.zeros(n * D, dtype=torch.int16, device=cuda)
    our_out = torch.zeros(n * D, dtype=torch.int16, device=cuda)
    assert lib.ref_kivi_decompress(C.c_void_p(ref_packed.data_ptr()),
                                   C.c_void_p(ref_out.data_ptr()), n, D, n_out, G, s) == 0
    ops.kivi_decompress(ref_packed, our_out, n, D, n_out, G)
    torch.cuda.synchronize()
    assert torch.equal(ref_out, our_out)


@pytest.mark.skipif(not REF_O3.exists(), reason="reference kernels not built (make -C oracle ref)")
@pytest.mark.parametrize("D,n_out,G", CASES)
def test_optimised_reference_differs_only_in_meta_low_bytes(ops, cuda, D, n_out, G):
    from test_oracle_reference import meta_offsets, sat_u8_lowbyte
    lib = C.CDLL(str(REF_O3))
    n = 97
    x = _inputs(D, n, 3 + D + n_out + G)
    stride = ops.kivi_compressed_bytes(D, n_out, G)
    s = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    xin = _t(x, cuda)
    ref_packed = torch.full((n * stride,), 0x5A, dtype=torch.uint8, device=cuda)
    our_packed = torch.full((n * stride,), 0x5A, dtype=torch.uint8, device=cuda)
    assert lib.ref_kivi_compress(C.c_void_p(xin.data_ptr()), C.c_void_p(ref_packed.data_ptr()),
                                 n, D, n_out, G, s) == 0
    ops.kivi_compress(xin, our_packed, n, D, n_out, G)
    torch.cuda.synchronize()
    ours = our_packed.cpu().numpy().reshape(n, stride)
    theirs = ref_packed.cpu().numpy().reshape(n, stride)
    mo = meta_offsets(D, n_out, G)
    expect = ours.copy()
    expect[:, mo] = sat_u8_lowbyte(ours[:, mo].astype(np.uint16) |
                                   (ours[:, mo + 1].astype(np.uint16) << 8))
    assert np.array_equal(expect, theirs)


def test_unsupported_params_noop(ops, cuda):
    # test_kivi_roundtrip.cpp:207-229: head_dim 256 -> the wrapper does nothing
    x = torch.ones(256, dtype=torch.float16, device=cuda)
    stride = ops.kivi_compressed_bytes(256, 0, 16)
    packed = torch.full((stride,), 0xAB, dtype=torch.uint8, device=cuda)
    ops.kivi_compress(x, packed, 1, 256, 0, 16)
    torch.cuda.synchronize()
    assert bool((packed == 0xAB).all())


def test_odd_group_rejected(ops, cuda):
    from importlib import import_module
    L = import_module("truellm-engine_b200._lib")
    x = torch.ones(64, dtype=torch.float16, device=cuda)
    packed = torch.zeros(4096, dtype=torch.uint8, device=cuda)
    with pytest.raises(L.TkvError):
        ops.kivi_compress(x, packed, 1, 64, 0, 5)


def test_reference_roundtrip_tolerances_on_gpu(ops, cuda):
    """The reference's GPU round-trip tests (test_kivi_roundtrip.cpp:83-200)."""
    def rt(x, n_out, G):
        n, D = x.shape
        stride = ops.kivi_compressed_bytes(D, n_out, G)
        packed = torch.zeros(n * stride, dtype=torch.uint8, device=cuda)
        out = torch.zeros(n * D, dtype=torch.float16, device=cuda)
        xin = torch.from_numpy(x).to(torch.float16).to(cuda)
        ops.kivi_compress(xin, packed, n, D, n_out, G)
        ops.kivi_decompress(packed, out, n, D, n_out, G)
        return out.float().cpu().numpy().reshape(n, D)

    x = np.array([[0.1 * d + 0.5 * v for d in range(64)] for v in range(3)], np.float32)
    assert np.abs(rt(x, 0, 16) - x).max() <= 0.15
    x = np.array([[0.01 * (i % 64) for i in range(64)] for _ in range(2)], np.float32)
    for v in range(2):
        for k, ch in enumerate([3, 17, 33, 55]):
            x[v, ch] = 50.0 + k + v
    assert np.abs(rt(x, 4, 16) - x).max() <= 0.1
    x = np.full((1, 32), 2.5, np.float32)
    assert np.abs(rt(x, 0, 16) - 2.5).max() <= 1e-2


def test_compression_pass_mirror_matches_oracle(O, cuda):
    """KvCompressionPass (the reference class's call sequence) rounds the K and
    V of a 37-token prefill through the reference format in place: every
    vector equals the oracle's decompress(compress(x)); the reference skipped
    prefills longer than its 16-token scratch (kv_compression_pass.cpp:184-200)."""
    import importlib
    CF = importlib.import_module("truellm-engine_b200.config")
    cfg = CF.parse("[inference.compression.kv_kivi]\nenabled = true\nbits = 4\n"
                   "residual_length = 8\n")
    p = CF.KvCompressionPass(cfg, 32, 8, 128, 16)
    assert p.enabled()
    seq_len = 37
    xk = _inputs(128, seq_len * 8, 71)
    xv = _inputs(128, seq_len * 8, 72)
    k, v = _t(xk, cuda), _t(xv, cuda)
    p.init()
    p.run(0, seq_len, k, v)
    torch.cuda.synchronize()
    for got, x in ((k, xk), (v, xv)):
        want = O.kivi_decompress(O.kivi_compress(x, 8, 16), 128, 8, 16)
        assert np.array_equal(got.cpu().numpy().view(np.uint16).reshape(-1, 128), want)
