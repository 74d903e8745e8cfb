"""Generate golden vectors for the reference-format KIVI quantizer by running
the reference's own kernels (src/inference/backends/cuda/compression/kivi_cache.cu,
compiled unmodified into oracle/_ref/libkivi_ref.so by `make -C oracle ref`)
on a GPU.

    python tests/golden/make_golden.py <out_dir>
    TKV_REF_LIB=oracle/_ref/libkivi_ref_O3.so python tests/golden/make_golden.py <out_dir>

Writes refkivi_<case>.npz with x (fp16 bits), packed (bytes after compress
into a buffer pre-filled with 0x00), unpacked (fp16 bits after decompress),
n_outliers, group_size.  The committed fixtures were made by this script on a
B200: tests/golden/ from the -G build (libkivi_ref.so, the source semantics)
and tests/golden/o3/ from the default-optimised build (libkivi_ref_O3.so).
"""
import ctypes as C
import os
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
REF = Path(os.environ.get("TKV_REF_LIB", ROOT / "oracle" / "_ref" / "libkivi_ref.so"))


def cases():
    rng = np.random.default_rng(20261201)
    out = {}
    # config-1 reference mapping (residual_length=32 -> 32 outliers, bits=4 -> G=16)
    x = rng.standard_normal((64, 64)).astype(np.float32)
    x[:, [5, 17, 40, 63]] *= 10
    out["cfg1_d64_o32_g16"] = (x, 32, 16)
    # cuda-kivi-compression.toml mapping (residual_length=8, bits=4), D=128
    x = rng.standard_normal((64, 128)).astype(np.float32)
    x[:, [3, 77, 100]] *= 8
    out["d128_o8_g16"] = (x, 8, 16)
    # bits=8 mapping -> G=8
    out["d128_o8_g8"] = (rng.standard_normal((32, 128)).astype(np.float32), 8, 8)
    # paged KIVI groups through the reference: n_out=0, one group of 128 / 32
    out["d128_o0_g128"] = (rng.standard_normal((64, 128)).astype(np.float32), 0, 128)
    out["d64_o0_g32"] = (rng.standard_normal((64, 64)).astype(np.float32), 0, 32)
    # partial last group and odd-sized residual count
    out["d96_o5_g16"] = (rng.standard_normal((16, 96)).astype(np.float32), 5, 16)
    # ties, signed zeros, constant groups, huge/small magnitudes
    x = np.zeros((8, 64), np.float32)
    x[0] = 1.0
    x[1, ::2] = -0.0
    x[2] = np.repeat(np.arange(8, dtype=np.float32), 8)
    x[3] = np.linspace(-1e-3, 1e-3, 64)
    x[4] = np.where(np.arange(64) % 3 == 0, 60000.0, -60000.0)
    x[5] = rng.standard_normal(64) * 1e-6
    x[6, :] = 2.0
    x[6, 10] = 2.0009765625
    x[7] = np.abs(rng.standard_normal(64))
    out["specials_d64_o4_g16"] = (x, 4, 16)
    out["specials_d64_o0_g32"] = (x, 0, 32)
    return out


def main(out_dir: Path):
    out_dir.mkdir(parents=True, exist_ok=True)
    lib = C.CDLL(str(REF))
    lib.ref_kivi_compressed_bytes.restype = C.c_ulong
    dev = torch.device("cuda:0")
    for name, (x, n_out, G) in cases().items():
        bits = x.astype(np.float16).view(np.uint16)
        n, D = bits.shape
        stride = lib.ref_kivi_compressed_bytes(D, n_out, G)
        xin = torch.from_numpy(bits.view(np.int16).copy()).to(dev)
        packed = torch.zeros(n * stride, dtype=torch.uint8, device=dev)
        unpacked = torch.zeros(n * D, dtype=torch.int16, device=dev)
        s = torch.cuda.current_stream().cuda_stream
        assert lib.ref_kivi_compress(C.c_void_p(xin.data_ptr()), C.c_void_p(packed.data_ptr()), n,
                                     D, n_out, G, C.c_void_p(s)) == 0
        assert lib.ref_kivi_decompress(C.c_void_p(packed.data_ptr()),
                                       C.c_void_p(unpacked.data_ptr()), n, D, n_out, G,
                                       C.c_void_p(s)) == 0
        torch.cuda.synchronize()
        np.savez_compressed(out_dir / f"refkivi_{name}.npz", x=bits,
                            packed=packed.cpu().numpy().reshape(n, stride),
                            unpacked=unpacked.cpu().numpy().view(np.uint16).reshape(n, D),
                            n_outliers=n_out, group_size=G)
        print("wrote", name, n, D, n_out, G, stride)


if __name__ == "__main__":
    main(Path(sys.argv[1]) if len(sys.argv) > 1 else Path(__file__).resolve().parent)
