"""Shared helpers of the example projects: import path and artifact writing."""

from __future__ import annotations

import json
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def write_metrics(project_dir: Path, report: dict) -> Path:
    out = project_dir / "artifacts"
    out.mkdir(parents=True, exist_ok=True)
    path = out / "metrics.json"
    path.write_text(json.dumps(report, indent=2), encoding="utf-8")
    return path


def fit(model, opt, loss_fn, steps: int) -> list[float]:
    """Plain training loop: returns the loss of every step."""
    losses = []
    for _ in range(steps):
        opt.zero_grad()
        loss = loss_fn(model)
        losses.append(loss.item())
        loss.backward()
        opt.step()
    return losses
