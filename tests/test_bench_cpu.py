"""The CPU legs of bench.py (the reference arm and every cpu_baseline) on small samples: they run
the oracle's vector kernels and return the fields the bench line carries."""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


def _check(d, unit):
    assert set(d) >= {"value", "unit", "cores", "kind", "sample"}
    assert d["unit"] == unit and d["kind"] == "port" and d["value"] > 0
    assert d["cores"] == bench.host_threads() >= 1


def test_cpu_chain_baseline_small():
    d = bench.cpu_chain_baseline([(12, 256, 512), (12, 64, 896), (14, 128, 896), (8, 96, 256)],
                                 seed0=11, seconds=0.2)
    _check(d, "GB/s")
    assert "4 projections" in d["sample"]


def test_cpu_prefill_baseline_small():
    d = bench.cpu_prefill_baseline(seconds=0.2, tokens=8)
    _check(d, "TOPS")
    assert "8 tokens" in d["sample"]


def test_cpu_isa_names_the_vector_form():
    assert bench.cpu_isa().split(" on ")[0] in ("AVX-VNNI", "AVX2", "scalar")


def test_cpu_prefill70_baseline_small():
    d = bench.cpu_prefill70_baseline(seconds=0.2, tokens=8)
    _check(d, "TOPS")
    assert "8 tokens" in d["sample"]
