"""Text dataset inspection and a sample corpus (reference datasets.py:7-42)."""

from __future__ import annotations

from dataclasses import asdict, dataclass
from pathlib import Path

SAMPLE_TEXT = "underHFS trains beyond the box.\n"


@dataclass(frozen=True)
class TextDatasetReport:
    path: str
    bytes: int
    characters: int
    lines: int
    unique_bytes: int

    def to_dict(self) -> dict[str, int | str]:
        return asdict(self)


def inspect_text_dataset(path: str | Path) -> TextDatasetReport:
    p = Path(path)
    raw = p.read_bytes()
    text = raw.decode("utf-8", errors="ignore")
    n_lines = text.count("\n") + (1 if text and not text.endswith("\n") else 0)
    return TextDatasetReport(str(p), len(raw), len(text), n_lines, len(set(raw)))


def write_sample_text_dataset(path: str | Path) -> TextDatasetReport:
    p = Path(path)
    p.parent.mkdir(parents=True, exist_ok=True)
    p.write_text(SAMPLE_TEXT, encoding="utf-8")
    return inspect_text_dataset(p)
