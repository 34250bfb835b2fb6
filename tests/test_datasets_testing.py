"""Text dataset inspection, the sample corpus writer and the dependency-free
test runner (CPU)."""

import sys
import types

from underhfs_b200.datasets import SAMPLE_TEXT, inspect_text_dataset, write_sample_text_dataset
from underhfs_b200.testing import run_test_functions


def test_sample_dataset_report(tmp_path):
    rep = write_sample_text_dataset(tmp_path / "corpus" / "sample.txt")
    raw = SAMPLE_TEXT.encode("utf-8")
    assert rep.bytes == len(raw) and rep.characters == len(SAMPLE_TEXT)
    assert rep.lines == 1 and rep.unique_bytes == len(set(raw))
    assert rep.to_dict()["path"].endswith("sample.txt")


def test_inspect_counts_unterminated_last_line_and_multibyte(tmp_path):
    p = tmp_path / "t.txt"
    p.write_bytes("a\nbé".encode("utf-8"))  # é is two bytes
    rep = inspect_text_dataset(p)
    assert rep.bytes == 5 and rep.characters == 4 and rep.lines == 2


def test_runner_calls_every_test_function():
    mod = types.ModuleType("uhfs_runner_probe")
    calls = []
    mod.test_b = lambda: calls.append("b")
    mod.test_a = lambda: calls.append("a")
    mod.helper = lambda: calls.append("helper")
    mod.test_value = 3  # not callable: skipped
    sys.modules[mod.__name__] = mod
    try:
        passed = run_test_functions([mod.__name__])
    finally:
        del sys.modules[mod.__name__]
    assert calls == ["a", "b"]
    assert passed == ["uhfs_runner_probe.test_a", "uhfs_runner_probe.test_b"]
