"""The C++ drop-in run on the GPU: tests/cpp/engine_loop.cpp, compiled with
g++ against include/truellm_kivi.hpp and libtruellm_kivi.so, drives the
library in the order truellm-engine's CUDA backend calls its KV-cache kernels
(allocator, per-layer prompt append and prefill attention, per-step table
upload, append and decode on one stream without host waits, then
KvCompressionPass::run).  Its results are checked against the CPU oracle fed
the same tokens in the same order: cache pages byte for byte, prefill and
decode attention within 2e-3, the KvCompressionPass round trip bit-exact
against the reference-format quantizer.  Cases: BASELINE config 1 and an
8-sequence subset of config 2, two layers, three decode steps.
"""
import math
import os
import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest

from kivi_helpers import check_close

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "truellm-engine_b200"
CUDA = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))


@pytest.fixture(scope="module")
def engine_exe(tmp_path_factory):
    if shutil.which("g++") is None:
        pytest.fail("g++ is needed to build the C++ harness")
    exe = tmp_path_factory.mktemp("cpp") / "engine_loop"
    cmd = ["g++", "-std=c++17", "-O1", "-Wall", "-Werror", f"-I{ROOT / 'include'}",
           f"-I{CUDA / 'include'}", str(ROOT / "tests" / "cpp" / "engine_loop.cpp"),
           f"-L{PKG}", "-ltruellm_kivi", f"-L{CUDA / 'lib64'}", "-lcudart",
           f"-Wl,-rpath,{PKG}", f"-Wl,-rpath,{CUDA / 'lib64'}", "-o", str(exe)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    assert res.returncode == 0, res.stderr
    return exe


def _f16(rng, shape, outliers=None, scale=8.0):
    x = rng.standard_normal(shape).astype(np.float32)
    if outliers is not None:
        x[..., outliers] *= scale
    return x.astype(np.float16).view(np.uint16)


@pytest.mark.parametrize("case", ["config1", "config2x8"])
def test_engine_call_order_matches_oracle(engine_exe, O, wl, tmp_path, case):
    if case == "config1":
        w = wl.config1()
        D, G, R, bits, Hkv, Hq = w.D, w.group, w.residual, w.bits, w.Hkv, w.Hq
        lens = np.array(w.lengths, np.int32)
        oc, rt_out = np.asarray(w.outlier_channels), 32
    else:
        w = wl.config2(seed=1000)
        D, G, R, bits, Hkv, Hq = w.D, w.group, w.residual, w.bits, w.Hkv, w.Hq
        lens = np.array(w.lengths[:8], np.int32)
        oc, rt_out = np.asarray(w.outlier_channels), 8
    B, T, chunk, L = len(lens), 3, 16, 2
    max_blocks = (int(lens.max()) + T + 15) // 16 + 1
    num_pages = B * max_blocks + 8
    rng = np.random.default_rng(77)
    total = int(lens.sum())
    kp = _f16(rng, (L, total, Hkv, D), oc)
    vp = _f16(rng, (L, total, Hkv, D))
    qp = _f16(rng, (L, B * chunk, Hq, D))
    kd = _f16(rng, (L, T, B, Hkv, D), oc)
    vd = _f16(rng, (L, T, B, Hkv, D))
    qd = _f16(rng, (L, T, B, Hq, D))
    rt_vecs = 64
    rt = _f16(rng, (2, rt_vecs, D), oc)
    hdr = np.array([D, G, R, bits, Hkv, Hq, B, T, chunk, num_pages, max_blocks, L, rt_vecs,
                    rt_out], np.int32)
    np.concatenate([hdr, lens]).astype(np.int32).tofile(tmp_path / "job.i32")
    for name, a in (("kp", kp), ("vp", vp), ("qp", qp), ("kd", kd), ("vd", vd), ("qd", qd),
                    ("rt", rt)):
        a.tofile(tmp_path / f"{name}.f16")
    run = subprocess.run([str(engine_exe), str(tmp_path)], capture_output=True, text=True,
                         timeout=300)
    assert run.returncode == 0 and run.stdout.strip() == "ok", run.stdout + run.stderr
    assert int(np.fromfile(tmp_path / "err.i32", np.int32)[0]) == 0

    tables = np.fromfile(tmp_path / "tables.i32", np.int32)
    bt = tables[:B * max_blocks].reshape(B, max_blocks)
    final_lens = tables[B * max_blocks:B * (max_blocks + 1)]
    rows = tables[B * (max_blocks + 1):]
    assert np.array_equal(final_lens, lens + T)
    assert np.array_equal(rows, np.arange(B))  # the oracle's ring is indexed by batch row
    out_prefill = np.fromfile(tmp_path / "out_prefill.f32", np.float32).reshape(L, B * chunk, Hq, D)
    out_decode = np.fromfile(tmp_path / "out_decode.f32", np.float32).reshape(L, B, Hq, D)
    scale = 1.0 / math.sqrt(D)
    cu_prompt = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    cu_q = (np.arange(B + 1) * chunk).astype(np.int32)
    cu_one = np.arange(B + 1, dtype=np.int32)
    f32 = lambda bits_: bits_.view(np.float16).astype(np.float32)
    for layer in range(L):
        st = O.PagedState(D, G, R, bits, Hkv, num_pages, B)
        st.append(kp[layer], vp[layer], False, cu_prompt, np.zeros(B, np.int32), bt)
        ref_p = st.prefill(f32(qp[layer]), cu_q, bt, lens, scale, n_threads=8)
        check_close(out_prefill[layer], ref_p)
        for t in range(T):
            st.append(kd[layer, t], vd[layer, t], False, cu_one, lens + t, bt)
        ref_d = st.decode(f32(qd[layer, T - 1]), bt, lens + T, scale, n_threads=8)
        check_close(out_decode[layer], ref_d)
        pool = np.fromfile(tmp_path / f"pool{layer}.u8", np.uint8).reshape(st.pool.shape)
        assert np.array_equal(pool, st.pool), f"layer {layer}: cache pages differ"

    # KvCompressionPass: n_outliers = residual_length, group = 16 (bits 4)
    rt_dev = np.fromfile(tmp_path / "rt_out.f16", np.uint16).reshape(2, rt_vecs, D)
    for half in range(2):
        packed = O.kivi_compress(rt[half], rt_out, 16)
        want = O.kivi_decompress(packed, D, rt_out, 16)
        assert np.array_equal(rt_dev[half], want.reshape(rt_vecs, D))
