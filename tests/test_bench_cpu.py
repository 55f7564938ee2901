"""bench.py's workload definitions: its model dicts (what the reference arm hands the oracle
without loading the library) are the library's presets."""
import importlib.util
import os

import pytest

import infb200 as I

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench():
    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(ROOT, "bench.py"))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


@pytest.mark.parametrize("preset", [1, 2, 3, 6])
def test_bench_models_are_the_library_presets(preset):
    b = _bench()
    want = I.oracle_dict(I.preset(preset))
    got = dict(b.DECODE[preset]["model"])
    assert set(got) == set(want)
    for k, v in want.items():
        assert got[k] == pytest.approx(v, rel=1e-7) if isinstance(v, float) else got[k] == v, k


def test_bench_does_not_import_the_library_at_module_level():
    src = open(os.path.join(ROOT, "bench.py")).read()
    top = [l for l in src.splitlines() if l.startswith("import ") or l.startswith("from ")]
    assert not any("infb200" in l for l in top)
    ref = src[src.index("def run_reference("):src.index("def run_ours(")]
    assert "infb200" not in ref and "I." not in ref
