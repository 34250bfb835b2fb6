"""Dependency-free test runner (reference testing.py:7-18): calls every
``test_*`` callable of the given modules; tests take ``tmp_path=None``."""

from __future__ import annotations

import importlib
from collections.abc import Iterable


def run_test_functions(modules: Iterable[str]) -> list[str]:
    passed: list[str] = []
    for module_name in modules:
        module = importlib.import_module(module_name)
        for name in sorted(n for n in dir(module) if n.startswith("test_")):
            fn = getattr(module, name)
            if callable(fn):
                fn()
                passed.append(f"{module_name}.{name}")
    return passed
