"""Seeded synthetic inputs with the shapes and distributions of the five
BASELINE configurations (there is no dataset for this path).

All generation happens on the host with numpy's PCG64 so CPU and GPU see
identical tensors.  fp16 / bf16 tensors are returned as uint16 bit patterns.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

PAGE = 16


@dataclass
class DecodeWorkload:
    name: str
    B: int
    Hq: int
    Hkv: int
    D: int
    group: int
    residual: int
    bits: int
    lengths: np.ndarray          # [B] int32
    block_tables: np.ndarray     # [B, max_blocks] int32, -1 padded
    num_pages: int
    q_dtype: str                 # "f16" | "bf16"
    kv_dtype: str                # "f16" | "bf16"
    seed: int
    outlier_channels: np.ndarray = field(default_factory=lambda: np.zeros(0, np.int64))
    outlier_scale: float = 1.0

    @property
    def max_context(self) -> int:
        return int(self.lengths.max()) if self.B else 0


def f32_to_f16_bits(x: np.ndarray) -> np.ndarray:
    return np.asarray(x, dtype=np.float32).astype(np.float16).view(np.uint16)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bit patterns."""
    u = np.asarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return rounded.astype(np.uint16)


def bits_to_f32(bits: np.ndarray, dtype: str) -> np.ndarray:
    bits = np.asarray(bits, dtype=np.uint16)
    if dtype == "f16":
        return bits.view(np.float16).astype(np.float32)
    return (bits.astype(np.uint32) << 16).view(np.float32)


def to_bits(x: np.ndarray, dtype: str) -> np.ndarray:
    return f32_to_f16_bits(x) if dtype == "f16" else f32_to_bf16_bits(x)


def random_block_tables(lengths: np.ndarray, num_pages: int, rng: np.random.Generator,
                        max_blocks: int | None = None) -> np.ndarray:
    """Pages drawn without replacement from a shared pool in random order."""
    need = [(int(L) + PAGE - 1) // PAGE for L in lengths]
    total = sum(need)
    if total > num_pages:
        raise ValueError(f"pool of {num_pages} pages cannot hold {total}")
    perm = rng.permutation(num_pages).astype(np.int32)
    mb = max(need) if max_blocks is None else max_blocks
    mb = max(mb, 1)
    bt = np.full((len(lengths), mb), -1, dtype=np.int32)
    pos = 0
    for i, n in enumerate(need):
        bt[i, :n] = perm[pos:pos + n]
        pos += n
    return bt


def kv_tokens(rng: np.random.Generator, n_tokens: int, Hkv: int, D: int,
              outlier_channels: np.ndarray, outlier_scale: float):
    """Keys N(0,1) with the given channels scaled; values N(0,1).  fp32 [T, Hkv, D]."""
    k = rng.standard_normal((n_tokens, Hkv, D), dtype=np.float32)
    v = rng.standard_normal((n_tokens, Hkv, D), dtype=np.float32)
    if len(outlier_channels):
        k[:, :, outlier_channels] *= np.float32(outlier_scale)
    return k, v


def config1(seed: int = 1) -> DecodeWorkload:
    """CPU-runnable reference case: B=1, Hq=Hkv=8, D=64, L=512, G=32, R=32,
    block table = random permutation of a 64-page pool, 4 of 64 key channels x10."""
    rng = np.random.default_rng(seed)
    lengths = np.array([512], dtype=np.int32)
    bt = rng.permutation(64).astype(np.int32).reshape(1, 64)[:, :32]
    oc = np.sort(rng.choice(64, 4, replace=False))
    return DecodeWorkload("config1", 1, 8, 8, 64, 32, 32, 4, lengths, bt, 64, "f16", "f16", seed,
                          oc, 10.0)


def config2(seed: int = 2, B: int = 64) -> DecodeWorkload:
    """Llama-3-8B-shape decode: B=64, Hq=32, Hkv=8, D=128, L ~ U[1024, 8192],
    pages from a shared pool (sum pages + 10% slack), G=R=128, 2% key outlier
    channels x8, bf16."""
    rng = np.random.default_rng(seed)
    lengths = rng.integers(1024, 8192, size=B, endpoint=True).astype(np.int32)
    pages = int(sum((int(L) + PAGE - 1) // PAGE for L in lengths))
    num_pages = int(pages * 1.1) + 1
    bt = random_block_tables(lengths, num_pages, rng)
    oc = np.sort(rng.choice(128, 3, replace=False))
    return DecodeWorkload("config2", B, 32, 8, 128, 128, 128, 4, lengths, bt, num_pages, "bf16",
                          "bf16", seed, oc, 8.0)


def config4(seed: int = 4, B: int = 8, L: int = 131072) -> DecodeWorkload:
    """Llama-3-70B long context: B=8, Hq=64, Hkv=8, D=128, L=131072, G=R=128."""
    rng = np.random.default_rng(seed)
    lengths = np.full(B, L, dtype=np.int32)
    pages = B * (L // PAGE)
    num_pages = pages
    bt = random_block_tables(lengths, num_pages, rng)
    oc = np.sort(rng.choice(128, 3, replace=False))
    return DecodeWorkload("config4", B, 64, 8, 128, 128, 128, 4, lengths, bt, num_pages, "bf16",
                          "bf16", seed, oc, 8.0)


def config5(seed: int = 5, B: int = 256, bits: int = 4) -> DecodeWorkload:
    """Continuous batching: log-uniform lengths in [128, 32768], pages scattered
    over a 2M-token pool (131072 pages), Hq=32, Hkv=8, D=128, G=R=128."""
    rng = np.random.default_rng(seed)
    lengths = np.exp(rng.uniform(np.log(128), np.log(32768), size=B)).astype(np.int32)
    num_pages = 2 * 1024 * 1024 // PAGE
    bt = random_block_tables(lengths, num_pages, rng)
    oc = np.sort(rng.choice(128, 3, replace=False))
    return DecodeWorkload("config5", B, 32, 8, 128, 128, 128, bits, lengths, bt, num_pages,
                          "bf16", "bf16", seed, oc, 8.0)


def subset(w: DecodeWorkload, seqs=None, Hkv: int = None, Hq: int = None,
           bits: int = None) -> DecodeWorkload:
    """The same workload restricted to sequences `seqs` (their block-table
    rows; the page pool keeps its size), `Hkv` kv heads / `Hq` q heads, or
    another bit width."""
    idx = np.arange(w.B) if seqs is None else np.asarray(seqs, np.int64)
    return DecodeWorkload(w.name, len(idx), Hq or w.Hq, Hkv or w.Hkv, w.D, w.group, w.residual,
                          bits or w.bits, np.ascontiguousarray(w.lengths[idx]),
                          np.ascontiguousarray(w.block_tables[idx]), w.num_pages, w.q_dtype,
                          w.kv_dtype, w.seed + 7919 * (1 + (int(idx[0]) if len(idx) else 0)),
                          w.outlier_channels, w.outlier_scale)


def token_split_bytes(w: DecodeWorkload, split_lo: int, split_hi: int, residual: bool) -> int:
    """HBM bytes of a decode restricted to quantised splits [split_lo,
    split_hi) (512 tokens each) and, if `residual`, the fp16 window, plus q,
    out and the block tables: the per-rank share of a token-split decode."""
    D, G, R, b, H = w.D, w.group, w.residual, w.bits, w.Hkv
    nvg = -(-D // G)
    per_tok = 2 * D * b // 8 + 4 * nvg + 4 * D // G
    total = 0
    for L in w.lengths:
        L = int(L)
        nq = G * ((L - R) // G) if L > R else 0
        lo, hi = min(nq, split_lo * 512), min(nq, split_hi * 512)
        total += H * (hi - lo) * per_tok + (H * (L - nq) * 4 * D if residual else 0)
        total += 4 * ((L + PAGE - 1) // PAGE)
    return total + w.B * w.Hq * w.D * 2 * 2


@dataclass
class AppendWorkload:
    """A batch of prompt chunks appended to empty sequences."""
    name: str
    B: int
    T: int            # tokens appended per sequence
    Hkv: int
    D: int
    group: int
    residual: int
    bits: int
    block_tables: np.ndarray  # [B, T / 16] int32
    num_pages: int
    outlier_channels: np.ndarray
    outlier_scale: float
    seed: int


def config3(seed: int = 3, B: int = 64, T: int = 2048) -> AppendWorkload:
    """64 sequences x 2048-token bf16 chunk, Hkv=8, D=128, G=R=128 INT4: per
    sequence-head 1920 quantised + 128 residual tokens; pages drawn from a
    shared pool (+10% slack) in random order."""
    rng = np.random.default_rng(seed)
    lengths = np.full(B, T, np.int32)
    num_pages = int(B * (T // PAGE) * 1.1) + 1
    bt = random_block_tables(lengths, num_pages, rng)
    outl = np.sort(rng.choice(128, size=3, replace=False))
    return AppendWorkload("config3", B, T, 8, 128, 128, 128, 4, bt, num_pages, outl, 8.0, seed)


def append_algorithmic_bytes(w: AppendWorkload) -> int:
    """HBM bytes one append call must move: the K/V input (2 B per element),
    the packed pages of the quantised tokens (codes, value meta, key meta) and
    the fp16 residual tokens written to the ring."""
    D, G, R, b, H, T = w.D, w.group, w.residual, w.bits, w.Hkv, w.T
    nvg = -(-D // G)
    nq = G * ((T - R) // G) if T > R else 0
    nr = T - nq
    per_head = 2 * T * D * 2 + nq * (2 * D * b // 8 + 4 * nvg) + (nq // G) * 4 * D + nr * 4 * D
    return w.B * H * per_head


@dataclass
class PrefillWorkload:
    """Chunked prefill: each sequence has `hist` cached tokens and appends a
    `chunk`-token prompt chunk whose query rows then attend causally to the
    whole cache (one attention layer)."""
    name: str
    B: int
    hist: int
    chunk: int
    Hq: int
    Hkv: int
    D: int
    group: int
    residual: int
    bits: int
    block_tables: np.ndarray  # [B, ceil((hist + chunk) / 16)] int32
    num_pages: int
    outlier_channels: np.ndarray
    outlier_scale: float
    seed: int


def prefill(seed: int = 6, B: int = 8, hist: int = 4096, chunk: int = 512) -> PrefillWorkload:
    """Llama-3-8B heads (Hq=32, Hkv=8, D=128), KIVI INT4 G=R=128: B sequences
    of `hist` cached tokens plus a `chunk`-token chunk; pages from a shared
    pool (+10% slack) in random order, 3 key outlier channels x8."""
    rng = np.random.default_rng(seed)
    lengths = np.full(B, hist + chunk, np.int32)
    num_pages = int(B * (-(-(hist + chunk) // PAGE)) * 1.1) + 1
    bt = random_block_tables(lengths, num_pages, rng)
    outl = np.sort(rng.choice(128, size=3, replace=False))
    return PrefillWorkload("prefill", B, hist, chunk, 32, 8, 128, 128, 128, 4, bt, num_pages,
                           outl, 8.0, seed)


def prefill_flops(w: PrefillWorkload) -> float:
    """QK^T and PV multiply-adds of the causal chunk: 4 * D * Hq per (query
    row, attended token), summed over the chunk's positions."""
    ctx = sum(w.hist + i + 1 for i in range(w.chunk))
    return 4.0 * w.D * w.Hq * w.B * ctx


def decode_algorithmic_bytes(w: DecodeWorkload) -> int:
    """HBM bytes one decode step must move: per quantised token-head
    2*D*b/8 codes + 4*ceil(D/G) value meta + 4*D/G key meta (136 B at D=128,
    G=128, INT4), per residual token-head 4*D (fp16 K and V), plus q, out
    (2 B each) and the block tables (4 B per 16-token page)."""
    D, G, R, b, H = w.D, w.group, w.residual, w.bits, w.Hkv
    nvg = -(-D // G)
    total = 0
    for L in w.lengths:
        L = int(L)
        nq = G * ((L - R) // G) if L > R else 0
        nr = L - nq
        total += H * (nq * (2 * D * b // 8 + 4 * nvg) + (nq // G) * 4 * D + nr * 4 * D)
        total += 4 * ((L + PAGE - 1) // PAGE)
    total += w.B * w.Hq * w.D * 2 * 2
    return total
