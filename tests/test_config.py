"""Config switches of the path (CPU): the reference's keys and defaults, the
kv-cache type validation extended with kivi4/kivi2, the [inference.cuda_engine]
keys (use_megakernel included), and the KvCompressionPass mirror's enable rule
(config_schema.h:46-50,66-84,121-129; config.cpp:78-86,110-134,215-224,
562-568; kv_compression_pass.cpp:29-67)."""
import importlib

import pytest

CF = importlib.import_module("truellm-engine_b200.config")

FP16_PASS = """
[inference]
backend = "cuda"

[inference.compression.kv_kivi]
enabled = true
bits = 4
residual_length = 32
"""

PAGED = """
[inference]
backend = "cuda"

[inference.kv_cache]
type_k = "kivi4"
type_v = "kivi4"

[inference.compression.kv_kivi]
enabled = true
residual_length = 128
group_size = 128
"""


def test_defaults_match_the_reference_schema():
    cfg = CF.parse("")
    assert (cfg.kv_kivi.enabled, cfg.kv_kivi.bits, cfg.kv_kivi.residual_length) == (False, 8, 128)
    assert (cfg.kv_cache.type_k, cfg.kv_cache.type_v, cfg.kv_cache.size_mb) == ("f16", "f16", 0)
    assert cfg.backend == "cpu"
    e = cfg.cuda_engine
    assert (e.paged_kv_block_size, e.max_num_blocks, e.max_num_seqs, e.use_megakernel) == (
        16, 0, 256, False)
    assert CF.validate(cfg) is None
    assert not cfg.paged_kivi and not cfg.compression_pass and cfg.kivi_path is None


def test_fp16_cache_with_the_compression_pass():
    cfg = CF.parse(FP16_PASS)
    assert cfg.kv_kivi.enabled and cfg.kv_kivi.bits == 4 and cfg.kv_kivi.residual_length == 32
    assert cfg.compression_pass and not cfg.paged_kivi
    assert CF.validate(cfg) is None
    assert cfg.kivi_path == "pass"
    assert CF.parse(FP16_PASS.replace('"cuda"', '"cpu"')).kivi_path is None
    # built, but only the megakernel path calls it (cuda_engine.cpp:834, 1482)
    assert not cfg.pass_runs
    mk = CF.parse(FP16_PASS + "\n[inference.cuda_engine]\nuse_megakernel = true\n")
    assert mk.pass_runs and CF.validate(mk) is None


def test_paged_kivi_cache():
    cfg = CF.parse(PAGED)
    assert cfg.paged_kivi and cfg.paged_bits == 4 and not cfg.compression_pass
    assert CF.validate(cfg) is None and cfg.kivi_path == "paged"
    cfg2 = CF.parse(PAGED.replace("kivi4", "kivi2"))
    assert cfg2.paged_bits == 2 and CF.validate(cfg2) is None


@pytest.mark.parametrize("text,msg", [
    ('[inference.kv_cache]\ntype_k = "q5_1"', "type_k 'q5_1' is not recognised"),
    ('[inference.kv_cache]\ntype_v = "int3"', "type_v 'int3' is not recognised"),
    ('[inference.kv_cache]\ntype_k = "kivi4"\ntype_v = "f16"', "both type_k and type_v"),
    ('[inference.kv_cache]\ntype_k = "kivi4"\ntype_v = "kivi2"', "both type_k and type_v"),
    (PAGED.replace("group_size = 128", "group_size = 96"), "group_size must be"),
    (PAGED.replace('backend = "cuda"', 'backend = "cpu"'), 'need inference.backend = "cuda"'),
    ('[inference]\nbackend = "vulkan"', "backend 'vulkan' is not recognised"),
    (PAGED + "\n[inference.cuda_engine]\npaged_kv_block_size = 32\n",
     "paged_kv_block_size must be 16"),
    (PAGED + "\n[inference.cuda_engine]\nuse_megakernel = true\n",
     "use_megakernel must be false"),
])
def test_validation_messages(text, msg):
    assert msg in CF.validate(CF.parse(text))


def test_type_errors_are_reported():
    with pytest.raises(ValueError):
        CF.parse('[inference.compression.kv_kivi]\nbits = "four"')
    with pytest.raises(ValueError):
        CF.parse('[inference.cuda_engine]\nuse_megakernel = 1')


def test_compression_pass_enable_rule():
    cfg = CF.parse(FP16_PASS)
    p = CF.KvCompressionPass(cfg, 32, 8, 128, 16)
    assert p.enabled() and (p.n_outliers, p.group_size) == (32, 16)
    p.init()
    p.run(0, 0, None, None)          # no new tokens: nothing to do
    assert CF.KvCompressionPass(CF.parse(FP16_PASS.replace("bits = 4", "bits = 8")),
                                32, 8, 128, 16).group_size == 8
    assert not CF.KvCompressionPass(cfg, 32, 8, 256, 16).enabled()   # head_dim > 128
    assert not CF.KvCompressionPass(CF.parse(PAGED), 32, 8, 128, 16).enabled()  # paged cache
