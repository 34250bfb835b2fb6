"""The microbenchmark configuration's reference arm degrades to one
``unavailable`` line when the reference is not installed, and its option
parsing routes ``--config micro`` to the microbenchmark runners."""

import argparse
import importlib.util
import json
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _bench_module():
    spec = importlib.util.spec_from_file_location("bench_under_test", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_reference_micro_without_install(tmp_path, monkeypatch, capsys):
    bench = _bench_module()
    monkeypatch.setattr(bench, "ROOT", tmp_path)  # no baseline/_ref below it
    monkeypatch.setenv("RANK", "0")
    monkeypatch.setenv("WORLD_SIZE", "1")
    args = argparse.Namespace(steps=2, warmup=1, steps_given=True)
    assert bench.run_reference_micro(args) == 0
    line = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["config"] == "micro" and "unavailable" in line


def test_micro_config_is_listed():
    bench = _bench_module()
    assert "micro" in bench.CONFIGS
    assert callable(bench.run_micro) and callable(bench.run_reference_micro)
