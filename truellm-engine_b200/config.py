"""The config switches that select this path, read the way the reference reads
them (src/host/config/config.cpp: backend :143, parse_kv_cache :78-86,
parse_cuda_engine :110-134, the kv_kivi block :215-224, validation :558-568;
defaults from include/truellm/config_schema.h:46-50, 66-84, 121-129, 204).

    [inference]                       backend: "cpu" | "ggml" | "cuda"
    [inference.compression.kv_kivi]   enabled, bits, residual_length, (group_size)
    [inference.kv_cache]              type_k / type_v: "f16" | "q8_0" | "q4_0" and,
                                      for this path, "kivi4" | "kivi2"
    [inference.cuda_engine]           paged_kv_block_size, max_num_blocks,
                                      max_num_seqs, use_megakernel

use_megakernel is read here although the reference's parse_cuda_engine omits
it (config.cpp:110-134; the field keeps its default, false,
config_schema.h:80).  The KIVI pass only runs on the megakernel path (after
the megakernel prefill, cuda_engine.cpp:834, and in inject_tokens, :1482), so
in the reference a config that enables both (configs/cuda-kivi-compression.toml
sets use_megakernel = true at :55) builds the pass and never runs it;
`PathConfig.pass_runs` reports what the config asks for.

Two consumers:
* the per-vector fake-quant pass (KvCompressionPass, kv_compression_pass.cpp
  :29-67): outliers = residual_length, group = 16 when bits == 4 else 8;
* the paged KIVI cache: selected by type_k/type_v = "kivi4"/"kivi2" (the same
  bit width on both), with G = group_size (default 128) and R =
  residual_length.

`KvCompressionPass` mirrors the reference class over the C ABI: the same
constructor arguments, `init`, `run`, `enabled`; unsupported parameters
disable it (as the reference logs and disables), and one fused launch per
tensor replaces compress + decompress through a scratch buffer, so prefills of
any length are handled.
"""
from __future__ import annotations

import tomllib
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Mapping, Optional, Union

KV_CACHE_TYPES = ("f16", "q8_0", "q4_0", "kivi4", "kivi2")


@dataclass
class KiviConfig:
    """[inference.compression.kv_kivi] (config_schema.h:121-129)."""
    enabled: bool = False
    bits: int = 8
    residual_length: int = 128
    key_granularity: str = "per_channel"
    value_granularity: str = "per_token"
    pre_rope_keys: bool = True
    group_size: int = 128        # this path's paged-cache key/value group G


@dataclass
class KvCacheConfig:
    """[inference.kv_cache] (config_schema.h:46-50)."""
    type_k: str = "f16"
    type_v: str = "f16"
    size_mb: int = 0


@dataclass
class CudaEngineConfig:
    """[inference.cuda_engine] (config_schema.h:66-84): the keys this path
    depends on."""
    paged_kv_block_size: int = 16  # tokens per block: the KIVI pages hold 16
    max_num_blocks: int = 0        # 0 = sized from free device memory
    max_num_seqs: int = 256        # live sequences (ring rows of the paged cache)
    use_megakernel: bool = False   # megakernel forward instead of the per-layer path


@dataclass
class PathConfig:
    kv_kivi: KiviConfig = field(default_factory=KiviConfig)
    kv_cache: KvCacheConfig = field(default_factory=KvCacheConfig)
    cuda_engine: CudaEngineConfig = field(default_factory=CudaEngineConfig)
    backend: str = "cpu"         # inference.backend (config_schema.h:204)

    @property
    def kivi_path(self) -> Optional[str]:
        """Which KIVI path the config selects: "paged" (the paged KIVI cache),
        "pass" (the per-vector pass over the fp16 cache, built whenever
        kv_kivi is enabled, cuda_engine.cpp:193-200 -- the CUDA engine does
        not read kv_cache.type_k/type_v) or None (the CPU/ggml backends,
        whose quantised caches are q8_0/q4_0)."""
        if self.backend != "cuda":
            return None
        if self.paged_kivi:
            return "paged"
        return "pass" if self.compression_pass else None

    @property
    def paged_kivi(self) -> bool:
        """True when the KV cache itself is the paged KIVI cache."""
        return self.kv_cache.type_k.startswith("kivi")

    @property
    def paged_bits(self) -> int:
        return 4 if self.kv_cache.type_k == "kivi4" else 2

    @property
    def compression_pass(self) -> bool:
        """True when the per-vector KIVI pass is built over an fp16 cache."""
        return self.kv_kivi.enabled and not self.paged_kivi

    @property
    def pass_runs(self) -> bool:
        """True when the built pass is also called: only the megakernel path
        calls it (cuda_engine.cpp:834, 1482)."""
        return self.backend == "cuda" and self.compression_pass and self.cuda_engine.use_megakernel


def _get(t: Mapping[str, Any], key: str, default, kind):
    v = t.get(key, default)
    if kind is int and isinstance(v, bool):
        raise ValueError(f"{key}: expected an integer")
    if not isinstance(v, kind):
        raise ValueError(f"{key}: expected {kind.__name__}, got {type(v).__name__}")
    return v


def parse(doc: Union[str, Path, Mapping[str, Any]]) -> PathConfig:
    """Reads the two tables from a TOML file, TOML text or a parsed mapping;
    absent keys keep the defaults, as toml::find_or does in the reference."""
    if isinstance(doc, Path) or (isinstance(doc, str) and doc.endswith(".toml")):
        data = tomllib.loads(Path(doc).read_text())
    elif isinstance(doc, str):
        data = tomllib.loads(doc)
    else:
        data = dict(doc)
    cfg = PathConfig()
    inf = data.get("inference", {})
    cfg.backend = _get(inf, "backend", cfg.backend, str)
    kc = inf.get("kv_cache")
    if kc is not None:
        cfg.kv_cache.type_k = _get(kc, "type_k", cfg.kv_cache.type_k, str)
        cfg.kv_cache.type_v = _get(kc, "type_v", cfg.kv_cache.type_v, str)
        cfg.kv_cache.size_mb = _get(kc, "size_mb", cfg.kv_cache.size_mb, int)
    ce = inf.get("cuda_engine")
    if ce is not None:
        e = cfg.cuda_engine
        e.paged_kv_block_size = _get(ce, "paged_kv_block_size", e.paged_kv_block_size, int)
        e.max_num_blocks = _get(ce, "max_num_blocks", e.max_num_blocks, int)
        e.max_num_seqs = _get(ce, "max_num_seqs", e.max_num_seqs, int)
        e.use_megakernel = _get(ce, "use_megakernel", e.use_megakernel, bool)
    ki = inf.get("compression", {}).get("kv_kivi")
    if ki is not None:
        k = cfg.kv_kivi
        k.enabled = _get(ki, "enabled", k.enabled, bool)
        k.bits = _get(ki, "bits", k.bits, int)
        k.residual_length = _get(ki, "residual_length", k.residual_length, int)
        k.key_granularity = _get(ki, "key_granularity", k.key_granularity, str)
        k.value_granularity = _get(ki, "value_granularity", k.value_granularity, str)
        k.pre_rope_keys = _get(ki, "pre_rope_keys", k.pre_rope_keys, bool)
        k.group_size = _get(ki, "group_size", k.group_size, int)
    return cfg


def validate(cfg: PathConfig) -> Optional[str]:
    """The reference's checks on these keys (config.cpp:562-568), extended with
    the paged KIVI types; returns the error message or None."""
    if cfg.backend not in ("cpu", "ggml", "cuda"):
        return f"inference.backend '{cfg.backend}' is not recognised (cpu|ggml|cuda)"
    for name, val in (("type_k", cfg.kv_cache.type_k), ("type_v", cfg.kv_cache.type_v)):
        if val not in KV_CACHE_TYPES:
            return (f"inference.kv_cache.{name} '{val}' is not recognised "
                    f"({'|'.join(KV_CACHE_TYPES)})")
    if cfg.paged_kivi != cfg.kv_cache.type_v.startswith("kivi") or (
            cfg.paged_kivi and cfg.kv_cache.type_k != cfg.kv_cache.type_v):
        return "inference.kv_cache: kivi4/kivi2 must be set on both type_k and type_v"
    if cfg.paged_kivi:
        if cfg.kv_kivi.group_size not in (16, 32, 64, 128):
            return "inference.compression.kv_kivi.group_size must be 16, 32, 64 or 128"
        if cfg.kv_kivi.residual_length < 0:
            return "inference.compression.kv_kivi.residual_length must be >= 0"
        if cfg.backend != "cuda":
            return 'inference.kv_cache: kivi4/kivi2 need inference.backend = "cuda"'
        if cfg.cuda_engine.paged_kv_block_size != 16:
            return ("inference.cuda_engine.paged_kv_block_size must be 16 with "
                    "kivi4/kivi2 (16-token pages)")
        if cfg.cuda_engine.use_megakernel:
            return ("inference.kv_cache: kivi4/kivi2 replace the per-layer cache and "
                    "attention calls; inference.cuda_engine.use_megakernel must be false")
    return None


class KvCompressionPass:
    """kv_compression_pass.h:38-58 over the C ABI (the KIVI half; the
    reference's VQ half is not part of this path and never enables it here)."""

    def __init__(self, cfg: PathConfig, n_layers: int, n_kv_heads: int, head_dim: int,
                 block_size: int):
        import importlib
        self.ops = importlib.import_module("truellm-engine_b200.ops")
        self.n_layers, self.n_kv_heads, self.head_dim = n_layers, n_kv_heads, head_dim
        self.block_size = block_size
        self.n_outliers = cfg.kv_kivi.residual_length
        self.group_size = 16 if cfg.kv_kivi.bits == 4 else 8
        self._enabled = cfg.compression_pass and self.ops.kivi_params_supported(
            head_dim, self.n_outliers, self.group_size)

    def init(self, allocator=None, stream=None) -> None:
        """No scratch to allocate (kept for the reference call sequence)."""

    def enabled(self) -> bool:
        return self._enabled

    def run(self, layer_idx: int, seq_len: int, k, v, stream=None) -> None:
        """Rounds K and V of `seq_len` new tokens ([seq_len, n_kv_heads, D]
        fp16 device tensors) through the reference KIVI format in place."""
        if not self._enabled or seq_len <= 0:
            return
        n = seq_len * self.n_kv_heads
        for t in (k, v):
            self.ops.kivi_roundtrip_inplace(t, n, self.head_dim, self.n_outliers,
                                            self.group_size, stream=stream)
