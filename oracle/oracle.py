"""TEST INFRASTRUCTURE ONLY -- numpy/ctypes front end of the CPU oracle.

Loads oracle/liboracle.so (built from kivi_oracle.c by `make -C oracle`) and
exposes the reference quantizer, the paged KIVI format packer and an fp64
decode attention for tests/, __graft_entry__.smoke() and bench.py's CPU
baseline.  The product path never imports this module.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"
REF_LIB = HERE / "_ref" / "libkivi_ref.so"

_o = None


def build(ref_root: str | None = None) -> None:
    """Compile the oracle and, when ref_root names the truellm-engine source
    tree, the reference's own kivi_cache.cu into _ref/ (the checker)."""
    subprocess.run(["make", "-s", "-C", os.fspath(HERE), "liboracle.so"], check=True)
    if ref_root:
        subprocess.run(["make", "-s", "-C", os.fspath(HERE), "ref", f"REF_ROOT={ref_root}"],
                       check=True)


class Fmt(C.Structure):
    _fields_ = [(n, C.c_int) for n in (
        "head_dim", "group", "residual", "bits", "n_kv_heads", "ring_cap", "n_vgroups",
        "k_codes_off", "v_codes_off", "v_meta_off", "k_meta_off", "k_meta_slice")] + [
        ("page_bytes", C.c_long)]


def lib() -> C.CDLL:
    global _o
    if _o is None:
        if not LIB.exists():
            build()
        h = C.CDLL(os.fspath(LIB))
        P = np.ctypeslib.ndpointer
        h.or_kivi_compressed_bytes.restype = C.c_size_t
        h.or_kivi_compressed_bytes.argtypes = [C.c_int] * 3
        h.or_kivi_params_supported.argtypes = [C.c_int] * 3
        h.or_kivi_compress.argtypes = [P(np.uint16), P(np.uint8)] + [C.c_int] * 4
        h.or_kivi_decompress.argtypes = [P(np.uint8), P(np.uint16)] + [C.c_int] * 4
        h.or_quant_group.argtypes = [P(np.float32), C.c_int, C.c_int, C.c_int, P(np.uint8),
                                     P(np.uint16), P(np.uint16)]
        h.or_f2h.restype = C.c_uint16
        h.or_f2h.argtypes = [C.c_float]
        h.or_fmt_init.argtypes = [C.POINTER(Fmt)] + [C.c_int] * 5
        h.or_fmt_page_bytes.restype = C.c_long
        h.or_fmt_page_bytes.argtypes = [C.c_int] * 5
        h.or_append.argtypes = [C.POINTER(Fmt), P(np.uint8), P(np.uint16), P(np.uint16),
                                P(np.uint16), C.c_int, P(np.int32), P(np.int32), P(np.int32),
                                C.c_int, C.c_int]
        h.or_unpack_token.argtypes = [C.POINTER(Fmt), P(np.uint8), P(np.int32), C.c_int, C.c_int,
                                      P(np.uint8), P(np.uint16), P(np.uint16), P(np.uint8),
                                      P(np.uint16), P(np.uint16)]
        h.or_ring_get.restype = C.c_uint16
        h.or_ring_get.argtypes = [C.POINTER(Fmt), P(np.uint16), C.c_int, C.c_int, C.c_int,
                                  C.c_int, C.c_int]
        h.or_decode_partial.argtypes = [C.POINTER(Fmt), P(np.uint8), P(np.uint16), P(np.float32),
                                        P(np.int32), C.c_int, P(np.int32), C.c_int, C.c_int,
                                        C.c_double, C.c_int, C.c_int, P(np.float64),
                                        P(np.float64), P(np.float64), C.c_int]
        h.or_merge.argtypes = [C.c_int, C.c_int, C.c_int, P(np.float64), P(np.float64),
                               P(np.float64), P(np.float64)]
        h.or_decode.argtypes = [C.POINTER(Fmt), P(np.uint8), P(np.uint16), P(np.float32),
                                P(np.int32), C.c_int, P(np.int32), C.c_int, C.c_int, C.c_double,
                                P(np.float64), C.c_int]
        h.or_prefill.argtypes = [C.POINTER(Fmt), P(np.uint8), P(np.uint16), P(np.float32),
                                 P(np.int32), P(np.int32), C.c_int, P(np.int32), C.c_int,
                                 C.c_int, C.c_double, P(np.float64), C.c_int]
        _o = h
    return _o


def _c(a, dt):
    return np.ascontiguousarray(a, dtype=dt)


# ---------------------------------------------------------------- reference format
def kivi_compressed_bytes(head_dim, n_outliers, group_size) -> int:
    return int(lib().or_kivi_compressed_bytes(head_dim, n_outliers, group_size))


def kivi_params_supported(head_dim, n_outliers, group_size) -> bool:
    return bool(lib().or_kivi_params_supported(head_dim, n_outliers, group_size))


def kivi_compress(x_f16_bits: np.ndarray, n_outliers: int, group_size: int,
                  fill: int = 0) -> np.ndarray:
    """x: [n_vecs, head_dim] uint16 fp16 bits -> [n_vecs, stride] uint8.
    Bytes the reference leaves unwritten keep the value `fill`."""
    x = _c(x_f16_bits, np.uint16)
    n, d = x.shape
    stride = kivi_compressed_bytes(d, n_outliers, group_size)
    out = np.full((n, stride), fill, dtype=np.uint8)
    lib().or_kivi_compress(x, out, n, d, n_outliers, group_size)
    return out


def kivi_decompress(packed: np.ndarray, head_dim: int, n_outliers: int,
                    group_size: int) -> np.ndarray:
    p = _c(packed, np.uint8)
    n = p.shape[0]
    out = np.zeros((n, head_dim), dtype=np.uint16)
    lib().or_kivi_decompress(p, out, n, head_dim, n_outliers, group_size)
    return out


def written_mask(head_dim, n_outliers, group_size) -> np.ndarray:
    """Bytes of one record the reference writes (slack of a partial last group
    excluded)."""
    stride = kivi_compressed_bytes(head_dim, n_outliers, group_size)
    m = np.zeros(stride, dtype=bool)
    m[: 3 * n_outliers] = True
    n_res = head_dim - n_outliers
    pos = 3 * n_outliers
    for gs in range(0, n_res, group_size):
        ge = min(gs + group_size, n_res)
        nb = (ge - gs + 1) // 2 + 4
        m[pos: pos + nb] = True
        pos += group_size // 2 + 4
    return m


def quant_group(x: np.ndarray, qmax: int):
    x = _c(x, np.float32)
    q = np.zeros(x.size, dtype=np.uint8)
    hs = np.zeros(1, dtype=np.uint16)
    hz = np.zeros(1, dtype=np.uint16)
    lib().or_quant_group(x, x.size, 1, qmax, q, hs, hz)
    return q, int(hs[0]), int(hz[0])


def f2h_bits(x: np.ndarray) -> np.ndarray:
    f = np.vectorize(lambda v: lib().or_f2h(float(v)), otypes=[np.uint16])
    return f(np.asarray(x, dtype=np.float32))


# ---------------------------------------------------------------- paged format
class PagedState:
    """CPU copy of one paged KIVI cache (pool + ring) in the exact device layout."""

    def __init__(self, head_dim, group, residual, bits, n_kv_heads, num_pages, max_seqs):
        self.fmt = Fmt()
        if lib().or_fmt_init(C.byref(self.fmt), head_dim, group, residual, bits, n_kv_heads):
            raise ValueError("unsupported paged format")
        f = self.fmt
        self.num_pages = num_pages
        self.max_seqs = max_seqs
        self.pool = np.zeros((num_pages, n_kv_heads, f.page_bytes), dtype=np.uint8)
        self.ring = np.zeros((max_seqs, n_kv_heads, f.ring_cap // 16, 2, 16 * head_dim),
                             dtype=np.uint16)

    def nq(self, length: int) -> int:
        x = length - self.fmt.residual
        return self.fmt.group * (x // self.fmt.group) if x > 0 else 0

    def append(self, k_new_bits, v_new_bits, in_bf16, cu_new, lens_old, block_tables):
        k = _c(k_new_bits, np.uint16)
        v = _c(v_new_bits, np.uint16)
        bt = _c(block_tables, np.int32)
        lib().or_append(C.byref(self.fmt), self.pool, self.ring, k, v, int(bool(in_bf16)),
                        _c(cu_new, np.int32), _c(lens_old, np.int32), bt, bt.shape[1],
                        len(lens_old))

    def unpack_token(self, bt_row, h, tok):
        D = self.fmt.head_dim
        kc = np.zeros(D, np.uint8); vc = np.zeros(D, np.uint8)
        ks = np.zeros(D, np.uint16); kz = np.zeros(D, np.uint16)
        vs = np.zeros(8, np.uint16); vz = np.zeros(8, np.uint16)
        lib().or_unpack_token(C.byref(self.fmt), self.pool, _c(bt_row, np.int32), h, tok, kc, ks,
                              kz, vc, vs, vz)
        nvg = self.fmt.n_vgroups
        return kc, ks, kz, vc, vs[:nvg], vz[:nvg]

    def decode(self, q_f32, block_tables, seq_lens, scale, n_threads=1) -> np.ndarray:
        q = _c(q_f32, np.float32)
        B, Hq, D = q.shape
        bt = _c(block_tables, np.int32)
        out = np.zeros((B, Hq, D), dtype=np.float64)
        lib().or_decode(C.byref(self.fmt), self.pool, self.ring, q, bt, bt.shape[1],
                        _c(seq_lens, np.int32), B, Hq, float(scale), out, int(n_threads))
        return out

    def prefill(self, q_f32, cu_q, block_tables, seq_lens, scale, n_threads=1) -> np.ndarray:
        """Causal chunked-prefill attention: q [T, Hq, D] rows of each
        sequence's last cu_q[b+1]-cu_q[b] tokens; returns out [T, Hq, D] fp64."""
        q = _c(q_f32, np.float32)
        T, Hq, D = q.shape
        bt = _c(block_tables, np.int32)
        out = np.zeros((T, Hq, D), dtype=np.float64)
        lib().or_prefill(C.byref(self.fmt), self.pool, self.ring, q, _c(cu_q, np.int32), bt,
                         bt.shape[1], _c(seq_lens, np.int32), len(seq_lens), Hq, float(scale),
                         out, int(n_threads))
        return out

    def decode_partial(self, q_f32, block_tables, seq_lens, scale, tok_lo, tok_hi, n_threads=1):
        q = _c(q_f32, np.float32)
        B, Hq, D = q.shape
        bt = _c(block_tables, np.int32)
        m = np.zeros(B * Hq); l = np.zeros(B * Hq); o = np.zeros(B * Hq * D)
        lib().or_decode_partial(C.byref(self.fmt), self.pool, self.ring, q, bt, bt.shape[1],
                                _c(seq_lens, np.int32), B, Hq, float(scale), int(tok_lo),
                                int(tok_hi), m, l, o, int(n_threads))
        return m.reshape(B, Hq), l.reshape(B, Hq), o.reshape(B, Hq, D)


def merge(ms, ls, os_):
    """LSE merge of P partial states; ms/ls: [P, BH], os_: [P, BH, D]."""
    ms = _c(ms, np.float64); ls = _c(ls, np.float64); os_ = _c(os_, np.float64)
    P, BH, D = os_.shape
    out = np.zeros((BH, D))
    lib().or_merge(P, BH, D, ms, ls, os_, out)
    return out
