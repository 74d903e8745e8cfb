"""bench.py's host-side rules (CPU).

* An ncu DRAM figure is reported only for the build it was captured from:
  `ncu_traffic` returns the committed per-launch traffic while the kernel's
  sources hash to the profile's `source_sha256`, and None once any of those
  sources changes (a stale profile never reaches the bench line).
* The CPU sample of a long-context workload is bounded by its token budget and
  never empty.
"""
import importlib.util
import json
import shutil
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    sys.modules["bench_under_test"] = mod
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture
def tree(bench, tmp_path, monkeypatch):
    """A copy of the append kernel's sources and an empty profiles folder,
    with bench.py pointed at them."""
    csrc = tmp_path / "csrc"
    csrc.mkdir()
    for name in bench.KERNEL_SOURCES["append"]:
        shutil.copy(bench.CSRC / name, csrc / name)
    (tmp_path / "profiles").mkdir()
    monkeypatch.setattr(bench, "CSRC", csrc)
    monkeypatch.setattr(bench, "ROOT", tmp_path)
    return tmp_path


def test_traffic_only_for_the_profiled_sources(bench, tree):
    profile = tree / "profiles" / "append_x.json"
    profile.write_text(json.dumps({"dram_bytes_per_call": 123,
                                   "source_sha256": bench.source_sha("append")}))
    assert bench.ncu_traffic("append_x", "append", "dram_bytes_per_call") == 123
    # any edit to a source of the kernel makes the committed figure stale
    src = tree / "csrc" / bench.KERNEL_SOURCES["append"][0]
    src.write_text(src.read_text() + "\n// edited\n")
    assert bench.ncu_traffic("append_x", "append", "dram_bytes_per_call") is None


def test_missing_profile_reports_no_traffic(bench, tree):
    assert bench.ncu_traffic("absent", "append", "dram_bytes_per_call") is None


def test_source_hash_covers_every_listed_file(bench):
    for kernel, names in bench.KERNEL_SOURCES.items():
        for name in names:
            assert (bench.CSRC / name).is_file(), (kernel, name)
        assert len(bench.source_sha(kernel)) == 64


def test_cpu_sample_is_bounded_and_never_empty(bench):
    assert bench.cpu_sample_size([1000] * 64, cap=64) == 64
    assert bench.cpu_sample_size([131072] * 8, cap=8) == 3          # 400K-token budget
    assert bench.cpu_sample_size([10 ** 6] * 4, cap=4) == 1         # one long sequence
    assert bench.cpu_sample_size([100] * 10, cap=3) == 3
