"""text -> 4x4 pixel regression: prompt bytes -> MLP(8-16-16) trained with MSE + SGD."""

from __future__ import annotations

import json
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
from _common import fit, write_metrics  # noqa: E402

from underhfs.functional import mse_loss  # noqa: E402
from underhfs.nn import Linear, ReLU, Sequential  # noqa: E402
from underhfs.optim import SGD  # noqa: E402
from underhfs.tensor import tensor  # noqa: E402

PROMPT = "a small red sun"


def encode_prompt(prompt: str, features: int = 8):
    codes = list(prompt.encode("utf-8")[:features])
    codes += [127.5] * (features - len(codes))  # pads map to 0.0
    return tensor([[c / 127.5 - 1.0 for c in codes]])


def target_pixels(prompt: str):
    seed = sum(prompt.encode("utf-8")) or 1
    return tensor([[((seed * (i + 3)) % 257) / 128.0 - 1.0 for i in range(16)]])


def build_model() -> Sequential:
    return Sequential(Linear(8, 16), ReLU(), Linear(16, 16))


def run_smoke(*, steps: int = 8, write_artifacts: bool = False) -> dict:
    x, y = encode_prompt(PROMPT), target_pixels(PROMPT)
    model = build_model()
    losses = fit(model, SGD(model.parameters(), lr=0.03), lambda m: mse_loss(m(x), y), steps)
    flat = model(x).tolist()[0]
    report = {"project": "text2image_text2pixel", "prompt": PROMPT, "steps": steps, "initial_loss": losses[0],
              "final_loss": losses[-1], "pixel_shape": [1, 4, 4],
              "generated_pixels": [flat[r * 4 : r * 4 + 4] for r in range(4)]}
    if write_artifacts:
        write_metrics(Path(__file__).resolve().parent, report)
    return report


if __name__ == "__main__":
    print(json.dumps(run_smoke(write_artifacts=True), indent=2))
