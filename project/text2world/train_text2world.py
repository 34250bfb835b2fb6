"""text command -> 6-d world vector: byte features -> MLP(10-12-6), MSE + SGD."""

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

COMMAND = "move north east toward forest"
SCHEMA = ["agent_x", "agent_y", "goal_x", "goal_y", "resource", "hazard"]


def encode_command(command: str, features: int = 10):
    vals = [(b % 32) / 16.0 - 1.0 for b in command.lower().encode("utf-8")[:features]]
    return tensor([vals + [0.0] * (features - len(vals))])


def target_world(command: str):
    words = command.lower()

    def axis(pos: str, neg: str) -> float:
        return 1.0 if pos in words else (-1.0 if neg in words else 0.0)

    resource = 1.0 if any(w in words for w in ("forest", "water")) else 0.25
    hazard = 1.0 if any(w in words for w in ("storm", "lava")) else 0.0
    return tensor([[0.0, 0.0, axis("east", "west"), axis("north", "south"), resource, hazard]])


def build_model() -> Sequential:
    return Sequential(Linear(10, 12), ReLU(), Linear(12, 6))


def run_smoke(*, steps: int = 10, write_artifacts: bool = False) -> dict:
    x, y = encode_command(COMMAND), target_world(COMMAND)
    model = build_model()
    losses = fit(model, SGD(model.parameters(), lr=0.04), lambda m: mse_loss(m(x), y), steps)
    report = {"project": "text2world", "command": COMMAND, "steps": steps, "initial_loss": losses[0],
              "final_loss": losses[-1], "world_vector": model(x).tolist()[0], "schema": SCHEMA}
    if write_artifacts:
        write_metrics(Path(__file__).resolve().parent, report)
    return report


if __name__ == "__main__":
    print(json.dumps(run_smoke(write_artifacts=True), indent=2))
