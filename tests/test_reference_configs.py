"""The reference's own switch files select the path they name (CPU).

* configs/cuda-kivi-compression.toml -- backend "cuda" (:25) and
  [inference.compression.kv_kivi] enabled, bits = 4, residual_length = 8
  (:73-79): the per-vector KIVI pass (kv_compression_pass.cpp:29-67) with 8
  outlier channels and 16-channel groups, built whenever kv_kivi is enabled
  (cuda_engine.cpp:193-200; the file's q8_0 kv_cache types at :34-36 are not
  read by the CUDA engine) and run because [inference.cuda_engine] sets
  use_megakernel = true (:55); not the paged cache.
* configs/scenario-quantized-kv.toml -- backend "cpu" (:27) with a q8_0
  [inference.kv_cache] (:36-39): the ggml CPU backend's q8_0 cache, so neither
  the pass nor the paged KIVI cache is selected.

The files are read from the reference tree named by TKV_REFERENCE_ROOT when
it is set and holds them; otherwise from tests/golden/reference_configs/,
which hold the same blocks with their line citations.
"""
import importlib
import os
from pathlib import Path

import pytest

CF = importlib.import_module("truellm-engine_b200.config")
FIXTURES = Path(__file__).resolve().parent / "golden" / "reference_configs"


def source(name: str) -> Path:
    root = os.environ.get("TKV_REFERENCE_ROOT")
    if root and (Path(root) / "configs" / name).is_file():
        return Path(root) / "configs" / name
    return FIXTURES / name


def test_cuda_kivi_compression_selects_the_pass_with_8_outliers_g16():
    cfg = CF.parse(source("cuda-kivi-compression.toml"))
    assert CF.validate(cfg) is None
    k = cfg.kv_kivi
    assert (k.enabled, k.bits, k.residual_length) == (True, 4, 8)
    assert (k.key_granularity, k.value_granularity, k.pre_rope_keys) == (
        "per_channel", "per_token", True)
    assert cfg.backend == "cuda" and cfg.kivi_path == "pass"
    assert cfg.compression_pass and not cfg.paged_kivi
    # [inference.cuda_engine] (:49-55) asks for the megakernel, the only path
    # that calls the pass (cuda_engine.cpp:834, 1482); the reference's parser
    # drops the key, so there the pass is built but never run
    e = cfg.cuda_engine
    assert (e.use_megakernel, e.paged_kv_block_size, e.max_num_seqs) == (True, 16, 4)
    assert cfg.pass_runs
    # the KvCompressionPass mirror: outliers = residual_length, G = 16 for 4 bits
    p = CF.KvCompressionPass(cfg, n_layers=32, n_kv_heads=8, head_dim=128, block_size=16)
    assert p.enabled() and (p.n_outliers, p.group_size) == (8, 16)
    # bytes per compressed vector: 8 x (idx u8 + fp16 value), 120 channels in
    # 8 groups of 16 at 4 bits plus an fp16 (scale, zero) per group
    assert p.ops.kivi_compressed_bytes(128, 8, 16) == 8 * 3 + 8 * (16 // 2 + 4)


def test_scenario_quantized_kv_selects_q8_0_not_this_path():
    cfg = CF.parse(source("scenario-quantized-kv.toml"))
    assert CF.validate(cfg) is None
    assert (cfg.kv_cache.type_k, cfg.kv_cache.type_v, cfg.kv_cache.size_mb) == ("q8_0", "q8_0", 0)
    assert cfg.backend == "cpu" and cfg.kivi_path is None
    assert not cfg.paged_kivi and not cfg.compression_pass and not cfg.pass_runs
    assert not CF.KvCompressionPass(cfg, 32, 8, 128, 16).enabled()


@pytest.mark.skipif(not os.environ.get("TKV_REFERENCE_ROOT"), reason="reference tree not named")
def test_fixtures_hold_the_reference_blocks():
    """With the reference tree present, the fixtures parse to the same config
    as the reference's whole files."""
    root = Path(os.environ["TKV_REFERENCE_ROOT"]) / "configs"
    for name in ("cuda-kivi-compression.toml", "scenario-quantized-kv.toml"):
        if not (root / name).is_file():
            pytest.skip(f"{name} not in the reference tree")
        assert CF.parse(root / name) == CF.parse(FIXTURES / name)
