"""The tcgen05 pieces of csrc/tkv_umma.cuh on the GPU: a one-CTA GEMM
(tests/cuda/umma_selftest.cu, compiled here with nvcc for sm_100a) stages
16-bit operands into the K-major no-swizzle layout, runs two accumulating
rounds of eight K = 16 `tcgen05.mma` into tensor memory and reads D back with
`tcgen05.ld`; D must equal A0 B0^T + A1 B1^T computed by torch in fp32, with A
read from shared memory or (a_tmem) from tensor memory.
"""
import ctypes as C
import os
import subprocess
import tempfile
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def selftest():
    nvcc = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
    out = Path(tempfile.mkdtemp()) / "umma_selftest.so"
    subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17",
                    "--expt-relaxed-constexpr", "-shared", "-Xcompiler", "-fPIC",
                    f"-I{ROOT / 'include'}", f"-I{ROOT / 'truellm-engine_b200' / 'csrc'}",
                    str(ROOT / "tests" / "cuda" / "umma_selftest.cu"), "-o", str(out)],
                   check=True)
    lib = C.CDLL(str(out))
    lib.umma_selftest.restype = C.c_int
    lib.umma_selftest.argtypes = [C.c_void_p] * 5 + [C.c_int, C.c_int, C.c_int, C.c_void_p,
                                                      C.c_void_p]
    return lib


@pytest.mark.parametrize("a_tmem", [0, 1])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("N", [64, 128, 256])
def test_tcgen05_gemm_matches_torch(selftest, cuda, dtype, N, a_tmem):
    g = torch.Generator(device=cuda).manual_seed(N)
    a0, a1 = (torch.randn((128, 128), generator=g, device=cuda).to(dtype) for _ in range(2))
    b0, b1 = (torch.randn((N, 128), generator=g, device=cuda).to(dtype) for _ in range(2))
    d = torch.full((128, N), float("nan"), device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    st = selftest.umma_selftest(a0.data_ptr(), b0.data_ptr(), a1.data_ptr(), b1.data_ptr(),
                                d.data_ptr(), N, int(dtype == torch.bfloat16), a_tmem,
                                err.data_ptr(),
                                torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert st == 0 and int(err.item()) == 0
    want = a0.float() @ b0.float().T + a1.float() @ b1.float().T
    assert torch.allclose(d, want, atol=1e-3, rtol=1e-4), (d - want).abs().max()
